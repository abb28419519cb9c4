"""The Q4 GEMV entry point that allocates nothing (qtts_q4_gemv_dev_noalloc).

It exists for callers that cannot allocate device memory -- a real-time
audio thread that may not block in a driver allocation, or a process whose
GPU memory belongs to another framework's caching allocator -- and takes its
split-K scratch from a static device array instead of a caller buffer.  This
file is collected last so that a failure here leaves every other test run.
It calls the entry point through the C ABI and checks it against
qtts_q4_gemv_dev (caller-provided scratch) on two calls in a row.
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


def _case(torch, rng, k, n, m):
    packed = torch.from_numpy(rng.integers(0, 256, k * n // 2, dtype=np.uint8)).cuda()
    scales = torch.from_numpy(np.abs(rng.standard_normal(k * n // 32) * 0.02).astype(np.float16)).cuda()
    x = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).cuda()
    return packed, scales, x


def test_noalloc_matches_scratch_entry_two_calls(qtts):
    if not has_gpu():
        pytest.skip("no GPU")
    import torch
    fn = _fn(qtts)
    rng = np.random.default_rng(2024)
    for k, n, m in [(2048, 6144, 1), (2048, 6144, 1), (1024, 2048, 3)]:
        packed, scales, x = _case(torch, rng, k, n, m)
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
        for y in outs:
            got = y.cpu().numpy()
            assert np.all(np.isfinite(got))
            assert np.max(np.abs(got - ref)) <= RTOL * np.max(np.abs(ref))


def test_noalloc_rejects_oversized(qtts):
    if not has_gpu():
        pytest.skip("no GPU")
    import torch
    fn = _fn(qtts)
    k, n, m = 32, 8192, 1024  # 32 tiles x 256 row blocks = 8192 counters > 4096
    packed = torch.zeros(k * n // 2, dtype=torch.uint8, device="cuda")
    scales = torch.zeros(k * n // 32, dtype=torch.float16, device="cuda")
    x = torch.zeros(m, k, device="cuda")
    y = torch.zeros(m, n, device="cuda")
    rc = fn(packed.data_ptr(), scales.data_ptr(), k, n, x.data_ptr(), m, y.data_ptr(), None)
    assert rc == qtts.ERR_RANGE
    assert b"static scratch" in qtts.lib.qtts_last_error()
