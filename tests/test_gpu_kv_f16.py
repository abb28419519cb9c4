"""The opt-in f16 K/V cache mode (qtts.h QTTS_SESSION_KV_F16) against the
CPU oracle, whose caches are f32 like the reference's (gemv.rs:77-86).

The mode rounds every cached K and V element to f16 (nearest even) and keeps
all arithmetic in f32, so it is not bit-faithful to the reference: its bar is
the logit tolerance.  Teacher-forced runs (the oracle's codes drive every
step) must keep each frame's codec-head logits within KV16_LOGIT_TOL of the
largest logit, and the GPU's own code choices may differ from the oracle's
only rarely: code 0 only at a near-tie of the oracle's logits (gap within the
tolerance), the predictor's groups 1-15 (greedy argmax over logits the
goldens do not hold) on at most KV16_GROUP_FLIPS of the entries.
"""
import numpy as np
import pytest

from conftest import golden
from test_gpu_model import LOGIT_TOL, _forced_batch, rel_err, tiny_case

pytestmark = pytest.mark.gpu

KV16_LOGIT_TOL = LOGIT_TOL  # 1e-2 of the frame's largest |logit|, as the f32 path
KV16_GROUP_FLIPS = 0.01     # share of predictor code entries allowed to differ


def _check_kv16(codes_gpu, g, logits_gpu):
    F = int(g["frames"])
    ref, got = g["codes"][:F], codes_gpu[:F]
    worst = 0.0
    for i, f in enumerate(g["logit_frames"]):
        worst = max(worst, rel_err(logits_gpu[f], g["logits"][i]))
    for f in range(F):
        idx = g["top_idx"][f]
        worst = max(worst, float(np.max(np.abs(logits_gpu[f][idx] - g["top_val"][f])) / g["absmax"][f]))
    assert worst <= KV16_LOGIT_TOL, worst
    for f in np.nonzero(got[:, 0] != ref[:, 0])[0]:
        gap = float(g["top_val"][f, 0] - g["top_val"][f, 1])
        assert gap <= KV16_LOGIT_TOL * float(g["absmax"][f]), ("code 0", f, gap)
    flips = int(np.count_nonzero(got[:, 1:] != ref[:, 1:]))
    assert flips <= KV16_GROUP_FLIPS * got[:, 1:].size, flips
    return worst, flips


@pytest.mark.parametrize("case", ["tiny_greedy", "tiny_sampled", "tiny_speaker", "tiny_notext"])
def test_kv_f16_teacher_forced_tiny(qtts, gpu_tiny, case):
    g = golden(case)
    F = g["codes"].shape[0]
    s = qtts.Session(gpu_tiny, 1, 10 + F, kv_f16=True)
    codes, frames, lg, _ = qtts.generate(s, [tiny_case(case, gpu_tiny.dims.t_hidden)], F,
                                         forced=g["codes"][None], dump_logits=True)
    s.close()
    assert frames[0] == F
    worst, flips = _check_kv16(codes[0], g, lg[0])
    print(f"{case}: worst logit deviation {worst:.2e}, predictor flips {flips}")


def test_kv_f16_differs_from_f32_and_is_deterministic(qtts, gpu_tiny):
    # the flag must reach the kernels (the logits move by the cache rounding)
    # and the mode stays run-to-run deterministic
    g = golden("tiny_sampled")
    F = g["codes"].shape[0]
    u = tiny_case("tiny_sampled", gpu_tiny.dims.t_hidden)
    out = {}
    for key, f16 in (("f32", False), ("f16a", True), ("f16b", True)):
        s = qtts.Session(gpu_tiny, 1, 10 + F, kv_f16=f16)
        out[key] = qtts.generate(s, [u], F, forced=g["codes"][None], dump_logits=True)[2][0]
        s.close()
    assert not np.array_equal(out["f32"], out["f16a"])
    assert np.array_equal(out["f16a"], out["f16b"])


@pytest.mark.parametrize("n", [12, 128])
def test_kv_f16_batched_tiny(qtts, gpu_tiny, n):
    # 12 utterances: the batch kernel's epilogue writes the caches; 128: the
    # tensor-core q/k/v epilogue (two row blocks in the predictor's first
    # step) and the attention kernel over the f16 pages
    H = gpu_tiny.dims.t_hidden
    cases = (["tiny_greedy", "tiny_sampled", "tiny_speaker", "tiny_notext"] * 32)[:n]
    F = 24
    s = qtts.Session(gpu_tiny, len(cases), 10 + F, kv_f16=True)
    codes, frames, lg, _ = qtts.generate(s, [tiny_case(c, H) for c in cases], F,
                                         forced=_forced_batch(cases, F), dump_logits=True)
    s.close()
    worst = 0.0
    for i, c in enumerate(cases):
        worst = max(worst, _check_kv16(codes[i], golden(c), lg[i])[0])
    print(f"{n} utterances: worst logit deviation {worst:.2e}")


def test_kv_f16_long_kv_tiny_2000_frames(qtts, gpu_tiny):
    # the rounding of ~2000 cached positions per head must stay inside the
    # tolerance over the whole run
    g = golden("tiny_long_kv")
    F = g["codes"].shape[0]
    s = qtts.Session(gpu_tiny, 1, 10 + F + 1, kv_f16=True)
    codes, frames, lg, _ = qtts.generate(s, [tiny_case("tiny_sampled", gpu_tiny.dims.t_hidden)], F,
                                         forced=g["codes"][None], dump_logits=True)
    s.close()
    assert frames[0] == F
    worst, flips = _check_kv16(codes[0], g, lg[0])
    print(f"2000 frames: worst logit deviation {worst:.2e}, predictor flips {flips}")


@pytest.mark.slow
def test_kv_f16_1p7b_config1_teacher_forced(qtts, gpu_1p7b):
    from qtts_b200 import workload as W
    g = golden("p1p7b_config1")
    u, F = W.config1(2048)
    s = qtts.Session(gpu_1p7b, 1, 10 + F, kv_f16=True)
    codes, frames, lg, _ = qtts.generate(s, [u], F, forced=g["codes"][None], dump_logits=True)
    s.close()
    assert frames[0] == F
    worst, flips = _check_kv16(codes[0], g, lg[0])
    print(f"1.7B config 1: worst logit deviation {worst:.2e}, predictor flips {flips}")


def test_session_rejects_unknown_flags(qtts, gpu_tiny):
    import ctypes as C
    h = C.c_void_p()
    assert qtts.lib.qtts_session_create_ex(gpu_tiny.h, 1, 16, 0x80, C.byref(h)) == qtts.ERR_BADARG
    assert not h.value
