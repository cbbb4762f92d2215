"""Loads the in-tree sm_100a extension (``trida_stack_b200/_C*.so``).

On a machine with a CUDA device the extension is mandatory: every CUDA op raises if it failed to
load, so nothing silently runs on a PyTorch fallback.  On a CPU-only machine the ops run their
plain-PyTorch statements (``ops.reference``) and the extension is never touched.
"""
import importlib

_C = None
_ERR = None


def load():
    global _C, _ERR
    if _C is not None or _ERR is not None:
        return _C
    try:
        _C = importlib.import_module("trida_stack_b200._C")
    except ImportError as e:  # not built yet / built for another torch
        _ERR = e
    return _C


def ext():
    """The compiled module; raises with the import error if it is unavailable."""
    m = load()
    if m is None:
        raise RuntimeError(
            "trida_stack_b200 CUDA extension is not built or failed to load "
            f"({_ERR}); run `python setup.py build_ext --inplace`")
    return m


def available():
    return load() is not None
