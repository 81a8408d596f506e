"""The allocation-free RMSNorm backward C entry point, called through its
exported C symbol the way a caller that cannot allocate device memory would
(ctypes, raw device pointers, a raw stream handle): checked against the
framework's regular RMSNorm backward on two calls in a row, checked to leave
the device's free memory and torch's allocator counters unchanged, and
checked to refuse rows wider than its kernel or larger than its scratch array.

This file is named so that pytest collects it last."""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

import nano_megatron_b200._C as _C  # noqa: E402  (loads the library and its torch dependencies)
from nano_megatron_b200.ops import cuda as KC  # noqa: E402

DEV = torch.device("cuda", 0)


def _lib():
    lib = ctypes.CDLL(_C.__file__)
    fn = lib.nmb_rmsnorm_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    lib.nmb_noalloc_error_string.restype = ctypes.c_char_p
    lib.nmb_noalloc_error_string.argtypes = [ctypes.c_int]
    lib.nmb_rmsnorm_bwd_noalloc_scratch_floats.restype = ctypes.c_long
    lib.nmb_rmsnorm_bwd_noalloc_max_cols.restype = ctypes.c_int
    lib.nmb_noalloc_prepare.restype = ctypes.c_int
    return lib


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("dtype,rows,cols", [(torch.bfloat16, 4096, 4096), (torch.float32, 1000, 2560)])
def test_noalloc_matches_regular_entry_point_twice(dtype, rows, cols):
    lib = _lib()
    torch.cuda.set_device(DEV)
    assert lib.nmb_noalloc_prepare() == 0
    stream = torch.cuda.current_stream(DEV).cuda_stream
    tol = 1e-2 if dtype == torch.bfloat16 else 1e-5
    w = torch.rand(cols, device=DEV) + 0.5
    dw_new = torch.zeros(cols, device=DEV)
    dw_old = torch.zeros(cols, device=DEV)
    for call in range(2):  # the second call reuses the shared scratch array
        torch.manual_seed(100 + call)
        x = torch.randn(rows, cols, device=DEV).to(dtype)
        dy = torch.randn(rows, cols, device=DEV).to(dtype)
        _, rstd = KC.rmsnorm(x, w, 1e-6)
        dx_new = torch.empty_like(x)
        code = lib.nmb_rmsnorm_bwd_noalloc(dy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr(),
                                           dx_new.data_ptr(), dw_new.data_ptr(), rows, cols,
                                           1 if dtype == torch.bfloat16 else 0, stream)
        assert code == 0, lib.nmb_noalloc_error_string(code)
        dx_old, _ = KC.rmsnorm_bwd(dy, x, w, rstd, dw_old)
        torch.cuda.synchronize(DEV)
        assert _rel(dx_new, dx_old) < tol, (call, _rel(dx_new, dx_old))
        assert _rel(dw_new, dw_old) < tol, (call, _rel(dw_new, dw_old))


def test_noalloc_rejects_sizes_beyond_the_scratch_array():
    lib = _lib()
    # 20000 rows use the maximum of 296 partial rows; 296 x 8192 floats do not fit.
    cols, rows = 8192, 20000
    assert _C.rmsnorm_bwd_blocks(rows, 296) * cols > lib.nmb_rmsnorm_bwd_noalloc_scratch_floats()
    x = torch.zeros(rows, cols, device=DEV, dtype=torch.bfloat16)
    w = torch.ones(cols, device=DEV)
    rstd = torch.ones(rows, device=DEV)
    dw = torch.zeros(cols, device=DEV)
    code = lib.nmb_rmsnorm_bwd_noalloc(x.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr(),
                                       x.data_ptr(), dw.data_ptr(), rows, cols, 1,
                                       torch.cuda.current_stream(DEV).cuda_stream)
    assert code == 1
    assert b"scratch" in lib.nmb_noalloc_error_string(code)


def test_noalloc_call_allocates_nothing():
    lib = _lib()
    torch.cuda.set_device(DEV)
    assert lib.nmb_noalloc_prepare() == 0
    rows, cols = 2048, 4096
    x = torch.randn(rows, cols, device=DEV).to(torch.bfloat16)
    dy = torch.randn(rows, cols, device=DEV).to(torch.bfloat16)
    w = torch.rand(cols, device=DEV) + 0.5
    _, rstd = KC.rmsnorm(x, w, 1e-6)
    dx = torch.empty_like(x)
    dw = torch.zeros(cols, device=DEV)
    stream = torch.cuda.current_stream(DEV).cuda_stream

    def call():
        return lib.nmb_rmsnorm_bwd_noalloc(dy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr(),
                                           dx.data_ptr(), dw.data_ptr(), rows, cols, 1, stream)

    assert call() == 0  # warm-up: module and symbol already resolved by prepare
    torch.cuda.synchronize(DEV)
    free_before, _ = torch.cuda.mem_get_info(DEV)
    stats_before = torch.cuda.memory_stats(DEV)
    for _ in range(3):
        assert call() == 0
    torch.cuda.synchronize(DEV)
    free_after, _ = torch.cuda.mem_get_info(DEV)
    stats_after = torch.cuda.memory_stats(DEV)
    assert free_after == free_before
    for key in ("allocation.all.allocated", "segment.all.allocated", "reserved_bytes.all.current"):
        assert stats_after.get(key, 0) == stats_before.get(key, 0), key


def test_noalloc_rejects_rows_wider_than_its_kernel():
    lib = _lib()
    cols = lib.nmb_rmsnorm_bwd_noalloc_max_cols() + 8
    rows = 16  # few rows: the scratch array alone would have room
    assert _C.rmsnorm_bwd_blocks(rows, 296) * cols <= lib.nmb_rmsnorm_bwd_noalloc_scratch_floats()
    x = torch.zeros(rows, cols, device=DEV, dtype=torch.bfloat16)
    w = torch.ones(cols, device=DEV)
    rstd = torch.ones(rows, device=DEV)
    dw = torch.zeros(cols, device=DEV)
    code = lib.nmb_rmsnorm_bwd_noalloc(x.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr(),
                                       x.data_ptr(), dw.data_ptr(), rows, cols, 1,
                                       torch.cuda.current_stream(DEV).cuda_stream)
    assert code == 2
    assert b"8192" in lib.nmb_noalloc_error_string(code)
