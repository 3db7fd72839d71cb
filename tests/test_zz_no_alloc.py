"""The allocation-free RMSNorm-backward entry point, called through its exported C symbol.

It serves callers that cannot allocate device memory at call time (their memory belongs
to their own pool, or allocation is not allowed where they run): they pass inputs and
outputs only, and the kernel's scratch is a fixed device array inside the library.  This
file is collected last so that a failing run has already run every other test.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("no CUDA device", allow_module_level=True)

from neural_scaling_weather_b200.ops import _ext  # noqa: E402

MAX_N = 2048
ERR_TOO_LARGE = 1001
ERR_BAD_ARG = 1002


def _lib():
    ext = _ext.require()
    lib = ctypes.CDLL(ext.__file__)
    fn = lib.nsw_rmsnorm_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    lib.nsw_noalloc_error_string.restype = ctypes.c_char_p
    lib.nsw_noalloc_error_string.argtypes = [ctypes.c_int]
    return ext, lib


def _call(lib, dy, x, w, rstd, dx, dw, dtype_code):
    stream = torch.cuda.current_stream().cuda_stream
    return lib.nsw_rmsnorm_bwd_noalloc(dy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr(), dx.data_ptr(),
                                       dw.data_ptr(), x.shape[0], x.shape[1], dtype_code, stream)


def rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("n,dtype", [(1024, torch.bfloat16), (64, torch.float16), (2048, torch.bfloat16)])
def test_noalloc_matches_allocating_entry_point_twice(n, dtype):
    ext, lib = _lib()
    code = 0 if dtype == torch.bfloat16 else 1
    for call in range(2):  # two calls in a row reuse (and must fully rewrite) the scratch
        torch.manual_seed(100 + call)
        rows = 777 + 300 * call
        x = torch.randn(rows, n, device="cuda").to(dtype)
        w = 1 + 0.1 * torch.randn(n, device="cuda")
        y, rstd = ext.rmsnorm_fwd(x, w, float(torch.finfo(torch.float32).eps))
        dy = torch.randn(rows, n, device="cuda").to(dtype)
        dx_ref, dw_ref = ext.rmsnorm_bwd(dy, x, w, rstd)
        dx = torch.empty_like(x)
        dw = torch.full((n,), float("nan"), device="cuda")
        rc = _call(lib, dy, x, w, rstd, dx, dw, code)
        assert rc == 0, lib.nsw_noalloc_error_string(rc)
        torch.cuda.synchronize()
        assert rel(dx, dx_ref) < 1e-2
        assert rel(dw, dw_ref) < 1e-4


def test_noalloc_rejects_sizes_beyond_maximum():
    _, lib = _lib()
    n = MAX_N + 8
    x = torch.zeros(4, n, device="cuda", dtype=torch.bfloat16)
    w = torch.ones(n, device="cuda")
    rstd = torch.ones(4, device="cuda")
    dx = torch.empty_like(x)
    dw = torch.empty(n, device="cuda")
    rc = _call(lib, x, x, w, rstd, dx, dw, 0)
    assert rc == ERR_TOO_LARGE
    assert b"exceeds" in lib.nsw_noalloc_error_string(rc)


def test_noalloc_zero_rows_writes_zero_weight_gradient():
    _, lib = _lib()
    n = 256
    x = torch.zeros(0, n, device="cuda", dtype=torch.bfloat16)
    w = torch.ones(n, device="cuda")
    rstd = torch.ones(1, device="cuda")  # not read; any valid pointer
    dx = torch.empty(1, n, device="cuda", dtype=torch.bfloat16)
    dw = torch.full((n,), float("nan"), device="cuda")
    dy = torch.empty(1, n, device="cuda", dtype=torch.bfloat16)
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.nsw_rmsnorm_bwd_noalloc(dy.data_ptr(), dy.data_ptr(), w.data_ptr(), rstd.data_ptr(), dx.data_ptr(),
                                     dw.data_ptr(), 0, n, 0, stream)
    assert rc == 0, lib.nsw_noalloc_error_string(rc)
    torch.cuda.synchronize()
    assert torch.equal(dw, torch.zeros_like(dw))


def test_noalloc_rejects_pointers_not_16_byte_aligned():
    _, lib = _lib()
    n, rows = 64, 8
    buf = torch.randn(rows * n + 8, device="cuda").to(torch.bfloat16)
    w = torch.ones(n, device="cuda")
    rstd = torch.ones(rows, device="cuda")
    dw = torch.empty(n, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    ok = buf.data_ptr()
    odd = ok + 2  # one bf16 element in: 2-byte aligned only
    for dy_p, x_p, dx_p in ((odd, ok, ok), (ok, odd, ok), (ok, ok, odd)):
        dx = torch.empty(rows * n + 8, device="cuda", dtype=torch.bfloat16)
        rc = lib.nsw_rmsnorm_bwd_noalloc(dy_p, x_p, w.data_ptr(), rstd.data_ptr(),
                                         dx.data_ptr() + (dx_p - ok), dw.data_ptr(), rows, n, 0, stream)
        assert rc == ERR_BAD_ARG
        assert b"aligned" in lib.nsw_noalloc_error_string(rc)
    torch.cuda.synchronize()
