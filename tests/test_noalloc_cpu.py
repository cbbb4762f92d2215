"""Host-side argument checks of the allocation-free grad-norm entry point.

These run without a GPU: every rejected call returns before it touches the CUDA runtime, so the
pointer values below are never dereferenced (they are plain integers, not device memory)."""
import ctypes

import pytest


def _lib():
    C = pytest.importorskip("trida_stack_b200._C")
    lib = ctypes.CDLL(C.__file__)
    fn = lib.trida_grad_norm_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_longlong), ctypes.c_int,
                   ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    err = lib.trida_noalloc_error_string
    err.restype = ctypes.c_char_p
    err.argtypes = [ctypes.c_int]
    return fn, err


def _call(fn, ptrs, sizes, out=0x10000):
    p = (ctypes.c_void_p * len(ptrs))(*ptrs)
    s = (ctypes.c_longlong * len(sizes))(*sizes)
    return fn(p, s, len(ptrs), 1.0, out, out + 16, None)


def test_misaligned_gradient_pointer_is_rejected():
    fn, err = _lib()
    rc = _call(fn, [0x20000, 0x30004], [64, 64])        # the second buffer starts 4 bytes off
    assert rc == 1
    assert b"aligned" in err(rc)


def test_null_negative_and_too_many_are_rejected():
    fn, err = _lib()
    assert _call(fn, [0], [8]) == 1
    assert _call(fn, [0x20000], [-1]) == 1
    rc = _call(fn, [0x20000] * 65, [8] * 65)
    assert rc == 2 and b"at most" in err(rc)
