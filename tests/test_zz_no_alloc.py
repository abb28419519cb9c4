"""The Q4 GEMV entry point that allocates nothing (qtts_q4_gemv_dev_noalloc).

It exists for callers that cannot allocate device memory -- a real-time
audio thread that may not block in a driver allocation, or a process whose
GPU memory belongs to another framework's caching allocator -- and takes its
split-K scratch from a static device array instead of a caller buffer.  This
file is collected last so that a failure here leaves every other test run.
It calls the entry point through the C ABI and checks it against a float64
product and against qtts_q4_gemv_dev (caller-provided scratch) on two calls
in a row, that a call after the first leaves the device's free memory
unchanged, and that shapes beyond the static array are refused on the host.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import has_gpu

pytestmark = pytest.mark.gpu

RTOL = 2e-6 * 8  # the GEMV tolerance of test_gpu_kernels.py


def _fn(qtts):
    f = qtts.lib.qtts_q4_gemv_dev_noalloc
    f.restype = C.c_int
    f.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]
    return f


def _host_case(rng, k, n, m):
    packed = rng.integers(0, 256, k * n // 2, dtype=np.uint8)
    scales = np.abs(rng.standard_normal(k * n // 32) * 0.02).astype(np.float16)
    x = rng.standard_normal((m, k)).astype(np.float32)
    return packed, scales, x


def _float64_product(packed, scales, x, k, n):
    """y = x @ W in float64 with W[r][c] = f32(scale[r][c/32]) * (q - 8),
    low nibble = even column (gemv.rs:26-51, :124)."""
    q = np.empty((k, n), np.int8)
    p = packed.reshape(k, n // 2)
    q[:, 0::2] = (p & 15).astype(np.int8) - 8
    q[:, 1::2] = (p >> 4).astype(np.int8) - 8
    w = q.astype(np.float64) * np.repeat(scales.astype(np.float64).reshape(k, n // 32), 32, axis=1)
    return x.astype(np.float64) @ w


def test_noalloc_matches_float64_and_scratch_entry_two_calls(qtts):
    if not has_gpu():
        pytest.skip("no GPU")
    import torch
    fn = _fn(qtts)
    rng = np.random.default_rng(2024)
    for k, n, m in [(2048, 6144, 1), (2048, 6144, 1), (1024, 2048, 3)]:
        hp, hs, hx = _host_case(rng, k, n, m)
        packed, scales, x = torch.from_numpy(hp).cuda(), torch.from_numpy(hs).cuda(), torch.from_numpy(hx).cuda()
        y_ref = torch.empty(m, n, device="cuda")
        sb = qtts.q4_gemv_scratch_bytes(k, n, m)
        scr = torch.zeros(sb, dtype=torch.uint8, device="cuda")
        qtts.q4_gemv_dev(packed.data_ptr(), scales.data_ptr(), k, n, x.data_ptr(), m, y_ref.data_ptr(),
                         scr.data_ptr(), sb)
        outs = []
        for _ in range(2):  # two calls in a row share the static scratch
            y = torch.full((m, n), float("nan"), device="cuda")
            rc = fn(packed.data_ptr(), scales.data_ptr(), k, n, x.data_ptr(), m, y.data_ptr(), None)
            assert rc == 0, qtts.lib.qtts_last_error()
            outs.append(y)
        torch.cuda.synchronize()
        ref = y_ref.cpu().numpy()
        y64 = _float64_product(hp, hs, hx, k, n)
        scale = np.max(np.abs(y64))
        for y in outs:
            got = y.cpu().numpy()
            assert np.all(np.isfinite(got))
            assert np.max(np.abs(got - y64)) <= RTOL * scale
            assert np.max(np.abs(got - ref)) <= RTOL * np.max(np.abs(ref))


def test_noalloc_second_call_takes_no_device_memory(qtts):
    if not has_gpu():
        pytest.skip("no GPU")
    import torch
    fn = _fn(qtts)
    rng = np.random.default_rng(7)
    k, n, m = 2048, 6144, 1
    hp, hs, hx = _host_case(rng, k, n, m)
    packed, scales, x = torch.from_numpy(hp).cuda(), torch.from_numpy(hs).cuda(), torch.from_numpy(hx).cuda()
    y = torch.empty(m, n, device="cuda")
    assert fn(packed.data_ptr(), scales.data_ptr(), k, n, x.data_ptr(), m, y.data_ptr(), None) == 0  # warm-up
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        assert fn(packed.data_ptr(), scales.data_ptr(), k, n, x.data_ptr(), m, y.data_ptr(), None) == 0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, (free0, free1)


def test_noalloc_rejects_oversized(qtts):
    if not has_gpu():
        pytest.skip("no GPU")
    import torch
    fn = _fn(qtts)
    # (a) 32 tiles x 256 row blocks = 8192 tile counters > the 4096 it holds;
    # (b) 16 tiles x 4 row blocks of counters fit, but 32 K slices x 15 rows x
    #     4096 columns of f32 partial sums (7.9 MB) exceed the 4 MiB array
    import re
    for k, n, m, what in [(32, 8192, 1024, "counters"), (65536, 4096, 15, "partials")]:
        packed = torch.zeros(k * n // 2, dtype=torch.uint8, device="cuda")
        scales = torch.zeros(k * n // 32, dtype=torch.float16, device="cuda")
        x = torch.zeros(m, k, device="cuda")
        y = torch.zeros(m, n, device="cuda")
        rc = fn(packed.data_ptr(), scales.data_ptr(), k, n, x.data_ptr(), m, y.data_ptr(), None)
        assert rc == qtts.ERR_RANGE
        err = qtts.lib.qtts_last_error().decode()
        assert "static scratch" in err, err
        cb, pb, ccap, pcap = (int(v) for v in re.findall(r"\d+", err)[:4])
        if what == "counters":
            assert cb > ccap, err
        else:
            assert cb <= ccap and pb > pcap, err
        del packed, scales, x, y
