"""GPU kernel parity through the C ABI: Q4 dequant (bit-exact), Q4 GEMV /
skinny GEMM (f32 tolerance), F16 GEMV (bit-exact with gemv.rs:183-196), the
sampler's exp (bit-exact with glibc expf) and the code-0 sampler (bit-exact
with the oracle on identical logits and rng state)."""
import ctypes

import numpy as np
import pytest

from conftest import golden, has_gpu, quantize_edge_data

pytestmark = pytest.mark.gpu
if has_gpu():
    import torch

LIBM = ctypes.CDLL("libm.so.6")
LIBM.expf.restype = ctypes.c_float
LIBM.expf.argtypes = [ctypes.c_float]

# GEMV tolerance: max|y - y64| <= RTOL * max|y64| (f32 accumulation in a
# different order than the reference's sequential loop).
RTOL = 2e-6 * 8


def rand_q4(rng, k, n):
    packed = rng.integers(0, 256, k * n // 2, dtype=np.uint8)
    scales = np.abs(rng.standard_normal(k * n // 32) * 0.02).astype(np.float16).view(np.uint16)
    return packed, scales


def dequant_np(packed, scales, k, n):
    p = packed.reshape(k, n // 2)
    q = np.empty((k, n), np.int32)
    q[:, 0::2] = p & 0xF
    q[:, 1::2] = p >> 4
    s = scales.view(np.float16).astype(np.float32).reshape(k, n // 32)
    return (np.repeat(s, 32, axis=1) * (q - 8).astype(np.float32)).astype(np.float32)


def test_dequant_bit_exact(qtts):
    rng = np.random.default_rng(0)
    for k, n in [(64, 96), (2048, 1024), (3, 4096)]:
        packed, scales = rand_q4(rng, k, n)
        dp = torch.from_numpy(packed).cuda()
        ds = torch.from_numpy(scales.view(np.int16)).cuda()
        out = torch.empty(k * n, dtype=torch.float32, device="cuda")
        qtts.q4_dequant_dev(dp.data_ptr(), ds.data_ptr(), k, n, out.data_ptr())
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy().reshape(k, n), dequant_np(packed, scales, k, n))


@pytest.mark.parametrize("k,n", [(8, 96), (3, 96), (1, 32), (64, 2048), (2048, 6144)])
def test_quantize_bit_exact(qtts, oracle_mod, k, n):
    # gemv.rs:92-130 on the GPU against the oracle: packed nibbles and f16
    # scales bit-identical, special cases included (NaN, inf, ties, subnormals)
    rng = np.random.default_rng(k * n)
    if k * n >= 8 * 96:
        data = quantize_edge_data(rng, k, n)
    else:
        data = (rng.standard_normal((k, n)) * 0.02).astype(np.float32)
        data.reshape(-1)[20] = np.nan
        data.reshape(-1)[:16] = np.array([0.5, -2.5, 7.0, 3.5] * 4, np.float32) * (1.0 if k > 1 else 1e-3)
    ref_p, ref_s = oracle_mod.quantize_q4(data, k, n)
    dd = torch.from_numpy(data).cuda()
    dp = torch.full((k * n // 2,), 0xAB, dtype=torch.uint8, device="cuda")
    ds = torch.full((k * n // 32,), 0x5A5A, dtype=torch.int16, device="cuda")
    qtts.q4_quantize_dev(dd.data_ptr(), k, n, dp.data_ptr(), ds.data_ptr())
    torch.cuda.synchronize()
    assert np.array_equal(ds.cpu().numpy().view(np.uint16), ref_s)
    assert np.array_equal(dp.cpu().numpy(), ref_p)
    hp, hs = qtts.quantize_f32_to_q4(data, k, n)  # host-buffer entry point
    assert np.array_equal(hp, ref_p) and np.array_equal(hs, ref_s)


def test_quantize_round_trip_and_errors(qtts):
    # dequantised weights quantise back to themselves when every group's
    # absmax is 7 * scale (q = 1 or 15 present) and the scale is a power of two
    rng = np.random.default_rng(7)
    k, n = 128, 256
    q = rng.integers(1, 16, (k, n)).astype(np.int32)  # q = 0 (value -8s) would raise the absmax
    q[:, ::32] = 15  # absmax = 7 * scale in every group
    s = np.exp2(rng.integers(-12, -4, (k, n // 32))).astype(np.float32)
    w = (np.repeat(s, 32, axis=1) * (q - 8)).astype(np.float32)
    packed, scales = qtts.quantize_f32_to_q4(w, k, n)
    assert np.array_equal(scales.view(np.float16).astype(np.float32).reshape(k, n // 32), s)
    back = np.empty((k, n), np.int32)
    back[:, 0::2] = packed.reshape(k, n // 2) & 0xF
    back[:, 1::2] = packed.reshape(k, n // 2) >> 4
    assert np.array_equal(back, q)
    with pytest.raises(qtts.QttsError):
        qtts.quantize_f32_to_q4(np.zeros((2, 48), np.float32), 2, 48)  # n % 32 != 0
    dd = torch.zeros(2 * 64 + 4, dtype=torch.float32, device="cuda")
    dp = torch.zeros(64, dtype=torch.uint8, device="cuda")
    ds = torch.zeros(4, dtype=torch.int16, device="cuda")
    with pytest.raises(qtts.QttsError):  # misaligned source: rejected on the host
        qtts.q4_quantize_dev(dd.data_ptr() + 4, 2, 64, dp.data_ptr(), ds.data_ptr())


SHAPES = [  # (k=in, n=out): benchmark config 2 and the real model shapes
    (2048, 4096), (2048, 2048), (2048, 1024), (2048, 6144), (6144, 2048), (2048, 3072),
    (1024, 2048), (1024, 1024), (1024, 3072), (3072, 1024), (64, 96), (100, 160), (33, 32)]


@pytest.mark.parametrize("k,n", SHAPES)
@pytest.mark.parametrize("m", [1, 2, 3, 5, 8, 9, 15, 16, 64, 130])
def test_q4_gemv_matches_float64(qtts, k, n, m):
    # m = 3..15 runs the batch kernel (8 rows per CTA: 9 and 15 leave a
    # partial second row block); m >= 16 the tcgen05 path (fp16 hi/lo
    # operands, f32 accumulate)
    rng = np.random.default_rng(k * 7 + n + m)
    packed, scales = rand_q4(rng, k, n)
    x = rng.standard_normal((m, k)).astype(np.float32)
    y = qtts.q4_gemv(packed, scales, k, n, x)
    ref = x.astype(np.float64) @ dequant_np(packed, scales, k, n).astype(np.float64)
    err = np.max(np.abs(y - ref), axis=1)
    scale = np.max(np.abs(ref), axis=1)
    assert np.all(err <= RTOL * scale), (err / scale).max()


@pytest.mark.parametrize("k,n", [(2048, 2048), (1024, 2048)])
def test_q4_gemv_matches_oracle(qtts, oracle_mod, k, n):
    rng = np.random.default_rng(11)
    packed, scales = rand_q4(rng, k, n)
    x = rng.standard_normal(k).astype(np.float32)
    y = qtts.q4_gemv(packed, scales, k, n, x[None])[0]
    yo = oracle_mod.gemv_q4(x, packed, scales, k, n)
    assert np.max(np.abs(y - yo)) <= RTOL * np.max(np.abs(yo))


@pytest.mark.parametrize("m", [1, 8, 15])
def test_q4_gemv_dev_deterministic(qtts, m):
    rng = np.random.default_rng(5)
    k, n = 2048, 6144
    packed, scales = rand_q4(rng, k, n)
    dp = torch.from_numpy(packed).cuda()
    ds = torch.from_numpy(scales.view(np.int16)).cuda()
    x = torch.randn(m, k, device="cuda")
    sb = qtts.q4_gemv_scratch_bytes(k, n, m)
    scr = torch.zeros(sb, dtype=torch.uint8, device="cuda")
    outs = []
    for _ in range(3):
        y = torch.empty(m, n, device="cuda")
        qtts.q4_gemv_dev(dp.data_ptr(), ds.data_ptr(), k, n, x.data_ptr(), m, y.data_ptr(), scr.data_ptr(), sb)
        outs.append(y)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])
    if m > 1:  # row i of a batch equals the same row computed alone, to f32 rounding
        y1 = torch.empty(1, n, device="cuda")
        sb1 = qtts.q4_gemv_scratch_bytes(k, n, 1)
        scr1 = torch.zeros(sb1, dtype=torch.uint8, device="cuda")
        qtts.q4_gemv_dev(dp.data_ptr(), ds.data_ptr(), k, n, x[m - 1:].data_ptr(), 1, y1.data_ptr(),
                         scr1.data_ptr(), sb1)
        torch.cuda.synchronize()
        d = (outs[0][m - 1] - y1[0]).abs().max().item()
        assert d <= RTOL * y1.abs().max().item(), d
    if m != 1:
        return
    with pytest.raises(qtts.QttsError):
        qtts.q4_gemv_dev(dp.data_ptr(), ds.data_ptr(), k, n, x.data_ptr(), m, outs[0].data_ptr(),
                         scr.data_ptr(), 16)


def test_f16_gemv_bit_exact(qtts, oracle_mod):
    rng = np.random.default_rng(2)
    k, n = 512, 1024
    w = (rng.standard_normal((k, n)) * 0.02).astype(np.float16).view(np.uint16)
    x = rng.standard_normal(k).astype(np.float32)
    dw = torch.from_numpy(w.view(np.int16)).cuda()
    dx = torch.from_numpy(x).cuda()
    y = torch.empty(n, device="cuda")
    qtts.f16_gemv_dev(dw.data_ptr(), k, n, dx.data_ptr(), 1, y.data_ptr())
    torch.cuda.synchronize()
    assert np.array_equal(y.cpu().numpy(), oracle_mod.gemv_f16(x, w, k, n))


def test_expf_matches_glibc():
    import qtts_b200 as qtts
    bits = np.arange(0, 2**32, 97, dtype=np.uint64).astype(np.uint32)
    x = bits.view(np.float32)
    x = x[np.isfinite(x) & (x > -110) & (x < 90)]
    x = np.concatenate([x, np.array([-np.inf, 0.0, -0.0, 88.7, -103.9, -104.0, 89.0], np.float32)])
    dx = torch.from_numpy(x).cuda()
    dy = torch.empty_like(dx)
    qtts.expf_dev(dx.data_ptr(), dy.data_ptr(), x.size)
    torch.cuda.synchronize()
    y = dy.cpu().numpy()
    idx = np.random.default_rng(0).choice(x.size, 200000, replace=False)
    ref = np.array([LIBM.expf(float(v)) for v in x[idx]], np.float32)
    assert np.array_equal(y[idx].view(np.uint32), ref.view(np.uint32))


def test_sampler_bit_exact_kats(qtts, gpu_tiny):
    sess = qtts.Session(gpu_tiny, 1, 64)
    k = golden("sampler_kats")
    for i in range(len(k["token"])):
        p = qtts.make_params(float(k["temperature"][i]), int(k["top_k"][i]), 1.05)
        tok, st = qtts.sample_token(sess, k["logits"][i], p, k["prev"][i], int(k["state"][i]))
        assert (tok, st) == (int(k["token"][i]), int(k["state_out"][i])), i
    sess.close()


def test_sampler_bit_exact_random(qtts, oracle_mod, gpu_tiny):
    sess = qtts.Session(gpu_tiny, 1, 64)
    rng = np.random.default_rng(99)
    for i in range(60):
        V = int(rng.choice([3072, 2048, 100, 4096]))
        lg = (rng.standard_normal(V) * rng.choice([1.0, 4.0, 20.0])).astype(np.float32)
        T = float(rng.choice([1.0, 0.8, 0.95, 1.5]))
        kk = int(rng.choice([0, 1, 2, 50, V - 1, V]))
        prev = rng.integers(0, V, 16).astype(np.uint32)
        st = int(rng.integers(1, 2**63))
        p = qtts.make_params(T, kk, 1.05)
        po = oracle_mod.make_params(1, T, kk, 1.05)
        assert qtts.sample_token(sess, lg, p, prev, st) == oracle_mod.sample_token(lg, po, prev, st), i
    sess.close()
