"""CPU checks of the oracle (oracle/qtts_oracle.c): known-answer tests for
the pieces the Rust reference specifies exactly, an independent Python
restatement of the sampler, and the committed golden fixtures.

Parity with the Rust crate itself is unpinned (it cannot be built here and
ships no golden vectors for this path); these tests pin the transcription.
"""
import ctypes
import os

import numpy as np
import pytest

from conftest import GOLDEN, golden, quantize_edge_data, quantize_np

LIBM = ctypes.CDLL("libm.so.6")
LIBM.expf.restype = ctypes.c_float
LIBM.expf.argtypes = [ctypes.c_float]
F32 = np.float32


def test_f16_roundtrip_all(oracle_mod):
    O = oracle_mod
    hs = np.arange(65536, dtype=np.uint16)
    ref = hs.view(np.float16).astype(np.float32)
    got = np.array([O.lib().oq_h2f(int(h)) for h in hs], np.float32)
    finite = np.isfinite(ref)
    assert np.array_equal(got[finite].view(np.uint32), ref[finite].view(np.uint32))
    assert np.all(np.isnan(got[np.isnan(ref)]))
    back = np.array([O.lib().oq_f2h(float(v)) for v in got[finite]], np.uint16)
    assert np.array_equal(back, hs[finite])


def test_f2h_round_to_nearest_even(oracle_mod):
    rng = np.random.default_rng(1)
    vals = np.concatenate([rng.standard_normal(20000) * 0.02, rng.standard_normal(2000) * 1e-5,
                           rng.standard_normal(2000) * 1e4]).astype(np.float32)
    got = np.array([oracle_mod.lib().oq_f2h(float(v)) for v in vals], np.uint16)
    assert np.array_equal(got, vals.astype(np.float16).view(np.uint16))


def test_quantize_layout_and_nibble_order(oracle_mod):
    # gemv.rs:92-130: scale = absmax/7, q = round(v/scale)+8, low nibble = even column
    k, n = 2, 64
    data = np.zeros((k, n), np.float32)
    data[0, :32] = np.linspace(-7, 7, 32, dtype=np.float32) * 0.5
    data[0, 32:] = 0.0
    data[1, 1] = 3.0
    packed, scales = oracle_mod.quantize_q4(data, k, n)
    assert oracle_mod.lib().oq_h2f(int(scales[0])) == np.float32(0.5)
    assert scales[1] == 0  # all-zero group
    q0 = packed[0] & 0xF
    q1 = packed[0] >> 4
    assert (q0, q1) == (1, 1)  # round(-7)+8, round(-6.548)+8
    q = np.array([(packed[j // 2] >> (4 * (j % 2))) & 0xF for j in range(32)])
    assert np.array_equal(q, np.clip(np.round(data[0, :32] / 0.5), -8, 7) + 8)
    # row 1, group 0: column 1 is the high nibble of byte 0, value +7 -> 15
    assert packed[32] == (8 | (15 << 4))
    deq = np.stack([oracle_mod.embed_q4(packed, scales, n, r) for r in range(k)])
    assert np.max(np.abs(deq - data)) <= 0.5 * 0.5 / 7 * 7 + 1e-6


@pytest.mark.parametrize("k,n", [(8, 96), (64, 2048)])
def test_quantize_matches_numpy_restatement(oracle_mod, k, n):
    # pins the oracle's quantize_f32_to_q4 on the special cases (NaN, inf,
    # ties, subnormals, f16 overflow) against an independent restatement
    data = quantize_edge_data(np.random.default_rng(k), k, n)
    packed, scales = oracle_mod.quantize_q4(data, k, n)
    ref_p, ref_s = quantize_np(data)
    assert np.array_equal(scales, ref_s)
    assert np.array_equal(packed, ref_p)
    g = packed[:16 * 4].reshape(4, 16)
    # group 1 (absmax 7, scale 1): 0.5 -> 1+8, -0.5 -> -1+8, 2.5 -> 3+8 (half away from zero)
    assert (g[1, 0] & 0xF, g[1, 0] >> 4) == (9, 7)
    assert (g[1, 2] & 0xF, g[1, 2] >> 4) == (11, 5)
    assert np.all(g[0] == 0x88) and scales[0] == 0          # all-zero group
    assert np.all(g[3] == 0) and scales[3] == 0              # all-NaN group: NaN as u8 = 0


def dequant_np(packed, scales, k, n):
    p = packed.reshape(k, n // 2)
    q = np.empty((k, n), np.int32)
    q[:, 0::2] = p & 0xF
    q[:, 1::2] = p >> 4
    s = scales.view(np.float16).astype(np.float32).reshape(k, n // 32)
    return (np.repeat(s, 32, axis=1) * (q - 8).astype(np.float32)).astype(np.float32)


@pytest.mark.parametrize("k,n", [(64, 96), (2048, 1024), (1024, 2048)])
def test_gemv_q4_matches_float64(oracle_mod, k, n):
    rng = np.random.default_rng(k + n)
    packed = rng.integers(0, 256, k * n // 2, dtype=np.uint8)
    scales = np.abs(rng.standard_normal(k * n // 32) * 0.02).astype(np.float16).view(np.uint16)
    x = rng.standard_normal(k).astype(np.float32)
    W = dequant_np(packed, scales, k, n)
    ref = x.astype(np.float64) @ W.astype(np.float64)
    y = oracle_mod.gemv_q4(x, packed, scales, k, n)
    assert np.max(np.abs(y - ref)) <= 1e-5 * np.max(np.abs(ref))
    # dequant row helper is exact
    assert np.array_equal(oracle_mod.embed_q4(packed, scales, n, 3), W[3])


def test_gemm_rows_are_sequential_gemv(oracle_mod):
    # gemv.rs:311-375: every gemm row is a full-K gemv_q4_inner
    rng = np.random.default_rng(3)
    k, n = 2048, 2048  # k*n >= 4e6: gemv threads, gemm does not split K
    packed = rng.integers(0, 256, k * n // 2, dtype=np.uint8)
    scales = np.abs(rng.standard_normal(k * n // 32) * 0.02).astype(np.float16).view(np.uint16)
    x = rng.standard_normal((3, k)).astype(np.float32)
    y = oracle_mod.gemm_q4(x, packed, scales, k, n)
    oracle_mod.set_threads(1)
    try:
        y1 = np.stack([oracle_mod.gemv_q4(x[i], packed, scales, k, n) for i in range(3)])
    finally:
        oracle_mod.set_threads(8)
    assert np.array_equal(y, y1)


def xorshift_py(state):
    state ^= (state << 13) & 0xFFFFFFFFFFFFFFFF
    state ^= state >> 7
    state ^= (state << 17) & 0xFFFFFFFFFFFFFFFF
    return state


def test_xorshift_kat(oracle_mod):
    st = 42
    for _ in range(1000):
        r, new = oracle_mod.simple_rand(st)
        exp = xorshift_py(st)
        assert new == exp
        assert np.float32(r) == F32(np.float32(exp) / np.float32(2.0 ** 64))
        st = new
    assert oracle_mod.simple_rand(0) == (0.0, 0)  # seed 0 is a fixed point


def test_argmax_last_index_wins(oracle_mod):
    lg = np.zeros(2048, np.float32)
    lg[[5, 700, 1999]] = 3.0
    assert oracle_mod.sample_argmax(lg) == 1999
    lg[2047] = 3.0
    assert oracle_mod.sample_argmax(lg) == 2047


def sample_token_py(logits, T, top_k, rep, prev, state):
    """Independent restatement of generate_new.rs:329-391 with numpy f32
    scalars (sequential sums) and glibc expf via ctypes."""
    s = [F32(v) for v in logits]
    V = len(s)
    if F32(rep) != F32(1.0):
        for t in prev:
            t = int(t)
            if t < V:
                s[t] = F32(s[t] / F32(rep)) if s[t] > 0 else F32(s[t] * F32(rep))
    if F32(T) != F32(1.0):
        s = [F32(v / F32(T)) for v in s]
    mx = max(s)
    s = [F32(LIBM.expf(float(F32(v - mx)))) for v in s]
    tot = F32(0.0)
    for v in s:
        tot = F32(tot + v)
    s = [F32(v / tot) for v in s]
    if 0 < top_k < V:
        order = sorted(range(V), key=lambda i: -float(s[i]))  # Python sort is stable
        for i in order[top_k:]:
            s[i] = F32(0.0)
        tot = F32(0.0)
        for v in s:
            tot = F32(tot + v)
        if tot > 0:
            s = [F32(v / tot) for v in s]
    state = xorshift_py(state)
    r = F32(F32(np.float32(state)) / F32(2.0 ** 64))
    cum = F32(0.0)
    for i, p in enumerate(s):
        cum = F32(cum + p)
        if r < cum:
            return i, state
    return 0, state


def test_sampler_matches_independent_restatement(oracle_mod):
    k = golden("sampler_kats")
    for i in range(0, len(k["token"]), 3):
        tok, st = sample_token_py(k["logits"][i], k["temperature"][i], int(k["top_k"][i]), 1.05,
                                  k["prev"][i], int(k["state"][i]))
        assert (tok, st) == (int(k["token"][i]), int(k["state_out"][i])), i


def test_sampler_kats_reproduce(oracle_mod):
    k = golden("sampler_kats")
    for i in range(len(k["token"])):
        p = oracle_mod.make_params(1, float(k["temperature"][i]), int(k["top_k"][i]), 1.05)
        tok, st = oracle_mod.sample_token(k["logits"][i], p, k["prev"][i], int(k["state"][i]))
        assert (tok, st) == (int(k["token"][i]), int(k["state_out"][i]))


def test_top1_picks_lowest_index_among_maxima(oracle_mod):
    lg = np.full(3072, -5.0, np.float32)
    lg[[17, 900, 3000]] = 9.0
    p = oracle_mod.make_params(1, 1.0, 1, 1.0)
    tok, _ = oracle_mod.sample_token(lg, p, np.zeros(16, np.uint32), 12345)
    assert tok == 17


def test_rope_tables_follow_reference_formula(oracle_mod):
    import math
    half, P = 64, 40
    cs = np.zeros(P * half, np.float32)
    sn = np.zeros(P * half, np.float32)
    sec = (ctypes.c_int * 3)(24, 20, 20)
    oracle_mod.lib().oq_build_mrope_tables(128, P, 1e6, sec, 3, oracle_mod.fptr(cs), oracle_mod.fptr(sn))
    for p in (0, 1, 7, 39):
        for i in (0, 1, 23, 24, 47, 63):
            f = 1.0 / math.pow(1e6, (2 * i) / 128.0)
            assert cs[p * half + i] == np.float32(math.cos(p * f))
            assert sn[p * half + i] == np.float32(math.sin(p * f))


@pytest.mark.parametrize("case", ["tiny_greedy", "tiny_sampled", "tiny_speaker", "tiny_notext"])
def test_tiny_golden_reproduces(oracle_mod, tiny_oracle, case):
    from qtts_b200 import make_params
    from qtts_b200 import workload as W
    g = golden(case)
    H = tiny_oracle.dims.t_hidden
    if case == "tiny_greedy":
        u, _ = W.config1(H)
    elif case == "tiny_sampled":
        u, _ = W.config3(H)
    elif case == "tiny_speaker":
        u = dict(text=W.tokens(11, 7), voice=None, speaker_id=3001, language_id=2055, seed=9,
                 params=make_params(0.9, 20, 1.05))
    else:
        u = dict(text=np.zeros(0, np.uint32), voice=W.voice_embedding(5, H), seed=3,
                 params=make_params(1.0, 1, 1.05))
    F = g["codes"].shape[0]
    p = oracle_mod.make_params(F, u["params"].temperature, u["params"].top_k, u["params"].repetition_penalty)
    n, codes, lg, _ = tiny_oracle.generate(u["text"], p, u["seed"], speaker_id=u.get("speaker_id", 0),
                                           language_id=u.get("language_id", 2050), voice=u.get("voice"),
                                           dump_logits=True)
    assert n == int(g["frames"])
    assert np.array_equal(codes, g["codes"])
    assert np.array_equal(lg[g["logit_frames"]], g["logits"])


def test_golden_meta_present():
    meta = np.load(os.path.join(GOLDEN, "meta.npz"))
    assert int(meta["threads"]) == 8
    assert len(str(meta["tiny_sha256"])) == 64


def test_oracle_full_prompt_mode(oracle_mod, tiny_path):
    # the benchmark mode that prefills the whole text: runs, and its first
    # logits differ from the generate_new mode's (the text lands in the cache)
    m = oracle_mod.Model(tiny_path)
    text = np.arange(7, dtype=np.uint32) * 1013 + 55
    p = oracle_mod.make_params(3, 1.0, 1, 1.05)
    n0, c0, l0, _ = m.generate(text, p, 1, dump_logits=True)
    n1, c1, l1, _ = m.generate(text, p, 1, dump_logits=True, full_prompt=True)
    m.close()
    assert n0 == n1 == 3
    assert np.abs(l0[0] - l1[0]).max() > 0
