"""The speech decoder's first stage on the GPU (qtts_decode_latent:
codebook_lookup decoder.rs:142-187, the causal pre-conv conv.rs:114-191,
decoder_transformer decoder.rs:195-335) against the CPU oracle's
restatement, on the synthetic full-size decoder.

Bar: the transformer output [1024][T] within DEC_TOL of its largest
magnitude (f32 arithmetic throughout; the GPU's GEMMs sum in tiles with
FMAs and its RMSNorm reduces in a tree, so the last bits differ from the
reference's sequential sums; above 15 frames the layer projections run on
the tensor cores from an fp16 hi/lo split of the f32 weights, ~22 bits).
Frame counts cover one frame, fewer frames than the 72-frame attention
window, the window edge, several windows, and each path boundary.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

DEC_TOL = 1e-4


@pytest.fixture(scope="module")
def dec_path(qtts):
    from qtts_b200 import workload as W
    return W.model_path("decoder")


@pytest.fixture(scope="module")
def gpu_dec(qtts, dec_path):
    from conftest import has_gpu
    if not has_gpu():
        pytest.skip("no GPU")
    d = qtts.Decoder(dec_path, 0)
    yield d
    d.close()


@pytest.fixture(scope="module")
def orc_dec(oracle_mod, dec_path):
    d = oracle_mod.Decoder(dec_path)
    yield d
    d.close()


def _rel(a, b):
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


@pytest.mark.parametrize("T", [1, 5, 15, 16, 40, 72, 73, 150, 257])
def test_decode_latent_matches_oracle(qtts, gpu_dec, orc_dec, T):
    # 1-15 frames: CUDA-core GEMMs; from 16 the layer projections on the
    # tensor cores (16-64: one-pass instance with in-kernel row split; above
    # 64: rows split by their producers; 257: a ragged third row block)
    from qtts_b200 import workload as W
    codes = W.decoder_codes(T, seed=700 + T)
    got = gpu_dec.decode_latent(codes)
    ref = orc_dec.decode_latent(codes)
    assert got.shape == (1024, T)
    e = _rel(got, ref)
    print(f"T={T}: max rel deviation {e:.2e}")
    assert e <= DEC_TOL, e


def test_decode_latent_deterministic_and_frames_independent_of_batch(qtts, gpu_dec):
    # run-to-run identical; and a frame's output depends only on the frames
    # before it (causal conv + causal attention): the first 40 frames of a
    # 120-frame run equal a 40-frame run
    from qtts_b200 import workload as W
    codes = W.decoder_codes(120, seed=9)
    a = gpu_dec.decode_latent(codes)
    b = gpu_dec.decode_latent(codes)
    assert np.array_equal(a, b)
    c = gpu_dec.decode_latent(np.ascontiguousarray(codes[:, :40]))
    assert _rel(a[:, :40], c) <= 1e-6


def test_device_entry_matches_host_entry(qtts, gpu_dec):
    import torch
    from qtts_b200 import workload as W
    T = 64
    codes = W.decoder_codes(T, seed=21)
    ref = gpu_dec.decode_latent(codes)
    cd = torch.from_numpy(codes.astype(np.int32)).cuda()
    out = torch.empty((1024, T), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    gpu_dec.decode_latent_dev(cd.data_ptr(), T, out.data_ptr())
    gpu_dec.sync()
    assert np.array_equal(out.cpu().numpy(), ref)


def test_bad_code_rejected_then_decoder_usable(qtts, gpu_dec):
    import torch
    from qtts_b200 import workload as W
    codes = W.decoder_codes(8, seed=3)
    codes[5, 4] = 4096
    with pytest.raises(qtts.QttsError) as e:
        gpu_dec.decode_latent(codes)
    assert e.value.code == qtts.ERR_RANGE
    # the device entry records it in the error flag, reported by sync
    cd = torch.from_numpy(codes.astype(np.int32)).cuda()
    out = torch.empty((1024, 8), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    gpu_dec.decode_latent_dev(cd.data_ptr(), 8, out.data_ptr())
    with pytest.raises(qtts.QttsError) as e:
        gpu_dec.sync()
    assert e.value.code == qtts.ERR_RANGE
    good = W.decoder_codes(8, seed=4)
    assert np.isfinite(gpu_dec.decode_latent(good)).all()


def test_decoder_load_needs_a_decoder_section(qtts, tiny_path):
    from conftest import has_gpu
    if not has_gpu():
        pytest.skip("no GPU")
    with pytest.raises(qtts.QttsError) as e:
        qtts.Decoder(tiny_path, 0)
    assert e.value.code == qtts.ERR_FORMAT
