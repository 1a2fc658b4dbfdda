"""The allocation-free GEMM entry point, called through its exported C symbol.

``lb_gemm_bf16_noalloc`` serves callers that cannot allocate device memory (allocator
callbacks, runtimes that own every allocation, real-time paths): its split-K scratch lives in
a static device array inside the library.  This test allocates the inputs and outputs itself
(the caller's job), calls the symbol twice in a row through ctypes and compares each result
with the regular entry point (``ops.gemm`` with the same split count) and an fp32 reference.
After each call it reads the kernel's error word through ``lb_gemm_bf16_noalloc_status``,
the non-allocating way such a caller learns that a bounded wait inside the kernel expired.
It runs last so that a failure here never hides the other tests' results.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from lightbulb_b200 import _C
    lib = ctypes.CDLL(_C.__file__)
    fn = lib.lb_gemm_bf16_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                   ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                   ctypes.c_int, ctypes.c_void_p]
    return fn


def _status(stream):
    from lightbulb_b200 import _C
    fn = ctypes.CDLL(_C.__file__).lb_gemm_bf16_noalloc_status
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.POINTER(ctypes.c_int), ctypes.c_void_p]
    code = ctypes.c_int(-1)
    rc = fn(ctypes.byref(code), stream)
    return rc, code.value


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


@pytest.mark.parametrize("m,n,k,splits", [(77, 512, 2048, 3), (256, 1024, 4096, 4),
                                          (5, 384, 1024, 1)])
def test_noalloc_matches_regular_entry_point(m, n, k, splits):
    from lightbulb_b200 import ops
    fn = _lib()
    torch.manual_seed(m + n + k)
    a = torch.randn(m, k, device="cuda").to(torch.bfloat16)
    w = (torch.randn(n, k, device="cuda") * 0.05).to(torch.bfloat16)
    ref = a.float() @ w.float().T
    regular = ops.gemm(a, w, splits=splits)
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):  # the shared scratch must be reusable call after call
        out = torch.full((m, n), float("nan"), device="cuda", dtype=torch.bfloat16)
        rc = fn(a.data_ptr(), k, w.data_ptr(), k, out.data_ptr(), n, m, n, k, splits, stream)
        assert rc == 0
        assert _status(stream) == (0, 0)      # no bounded wait expired inside the kernel
        torch.cuda.synchronize()
        assert _rel(out, regular) < 1e-2
        assert _rel(out, ref) < 1e-2


def test_noalloc_rejects_oversized_plan():
    fn = _lib()
    m, n, k = 256, 8192, 4096  # 64 tiles x 16 splits x 256 x 128 floats > 16 MiB of scratch
    a = torch.zeros(m, k, device="cuda", dtype=torch.bfloat16)
    w = torch.zeros(n, k, device="cuda", dtype=torch.bfloat16)
    out = torch.zeros(m, n, device="cuda", dtype=torch.bfloat16)
    rc = fn(a.data_ptr(), k, w.data_ptr(), k, out.data_ptr(), n, m, n, k, 16,
            torch.cuda.current_stream().cuda_stream)
    assert rc == 2
