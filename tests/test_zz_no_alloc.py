"""The allocation-free grad-norm entry point, called through its exported C symbol.

It serves callers that cannot allocate device memory (runtimes that own all device memory and
forbid cudaMalloc on the hot path, non-PyTorch C/C++ hosts without an allocator to hand it).  Its results must equal the regular
entry point's on two calls in a row (the second call reuses the library's fixed scratch array).
This file is named so pytest collects it last."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _fn():
    import trida_stack_b200._C as C   # loads the library (and the torch libraries it links)
    lib = ctypes.CDLL(C.__file__)
    fn = lib.trida_grad_norm_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_longlong), ctypes.c_int,
                   ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    err = lib.trida_noalloc_error_string
    err.restype = ctypes.c_char_p
    err.argtypes = [ctypes.c_int]
    return fn, err


def _call(fn, grads, max_norm, norm, coef):
    ptrs = (ctypes.c_void_p * len(grads))(*[g.data_ptr() for g in grads])
    sizes = (ctypes.c_longlong * len(grads))(*[g.numel() for g in grads])
    stream = torch.cuda.current_stream().cuda_stream
    return fn(ptrs, sizes, len(grads), max_norm, norm.data_ptr(), coef.data_ptr(), stream)


def test_grad_norm_noalloc_matches_regular_entry_point():
    from trida_stack_b200.ops._ext import ext
    fn, err = _fn()
    torch.manual_seed(0)
    grads = [torch.randn(n, device="cuda") for n in (1000, 123457, 777, 4096)]
    for call, (scale, max_norm) in enumerate([(1.0, 1.0), (0.01, 50.0)]):
        gs = [g * scale for g in grads]
        norm_ref = torch.zeros(1, device="cuda")
        coef_ref = torch.zeros(1, device="cuda")
        ext().grad_norm(gs, max_norm, norm_ref, coef_ref)
        norm = torch.full((1,), -1.0, device="cuda")
        coef = torch.full((1,), -1.0, device="cuda")
        rc = _call(fn, gs, max_norm, norm, coef)
        assert rc == 0, err(rc)
        torch.cuda.synchronize()
        torch.testing.assert_close(norm, norm_ref, rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(coef, coef_ref, rtol=1e-5, atol=1e-6)
        exact = torch.sqrt(sum((g.double() ** 2).sum() for g in gs)).float()
        assert abs(norm.item() - exact.item()) <= 1e-3 * exact.item(), f"call {call}"


def test_grad_norm_noalloc_rejects_too_many_buffers():
    fn, err = _fn()
    grads = [torch.ones(8, device="cuda")] * 65
    norm = torch.zeros(1, device="cuda")
    coef = torch.zeros(1, device="cuda")
    rc = _call(fn, grads, 1.0, norm, coef)
    assert rc != 0
    assert b"at most" in err(rc)

