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


# Kernels each entry point launches (for the launch count the benchmark reports).
KERNELS_PER_CALL = {
    "gemm": 1, "rmsnorm_fwd": 1, "rmsnorm_bwd": 1, "qk_norm_rope_fwd": 1, "qk_norm_rope_bwd": 1,
    "swiglu_fwd": 1, "swiglu_bwd": 1, "embed_fwd": 1, "embed_bwd": 1, "bd_attn_plan": 2, "bd_attn_fwd": 1,
    "bd_attn_bwd": 3, "ce_rows": 1, "adamw": 1, "bd_attn_lists128": 1, "bd_attn_fwd_sm100": 1, "bd_attn_bwd_sm100": 5, "bd_attn_tile_masks": 1,
    "gemm_error": 0, "gdn_state_numel": 0, "gdn_fwd": 2, "gdn_bwd": 3, "gdn_conv_fwd": 1, "gdn_conv_bwd": 2,
    "gdn_gnorm_fwd": 1, "gdn_gnorm_bwd": 1, "attn_gate_fwd": 1, "attn_gate_bwd": 1,
    "canvas_attention": 2, "kv_append": 1, "canvas_conv": 1, "conv_commit": 1, "gdn_canvas": 2, "gdn_prep_numel": 0, "gdn_commit": 1, "gdn_canvas_tc": 1, "gdn_commit_tc": 1, "spec_sample": 1, "gemm_argmax": 2,
    "argmax_rows": 1, "conf_argmax_rows": 1, "gemm_swiglu": 1, "gemm_allreduce": 1, "symm_malloc": 0, "symm_free": 0, "symm_handle": 0, "symm_open": 0, "symm_close": 0,
    "symm_tensor": 0, "symm_allreduce": 1, "symm_rs_sumsq": 1, "symm_norm_coef": 1, "symm_adamw_ag": 1,
}


class _Counting:
    """Proxy over the extension that counts kernel launches while ``counting`` is on."""

    def __init__(self, mod):
        self._mod = mod
        self.counting = False
        self.launches = 0

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        if not callable(fn):
            return fn

        def wrapped(*a, **k):
            if self.counting:
                if name == "grad_norm":
                    self.launches += len(a[0]) + 1
                else:
                    self.launches += KERNELS_PER_CALL.get(name, 1)
            return fn(*a, **k)
        return wrapped


_PROXY = None


def ext():
    """The compiled module; raises with the import error if it is unavailable."""
    global _PROXY
    m = load()
    if m is None:
        raise RuntimeError(
            "trida_stack_b200 CUDA extension is not built or failed to load "
            f"({_ERR}); run `python setup.py build_ext --inplace`")
    if _PROXY is None:
        _PROXY = _Counting(m)
    return _PROXY


def count_launches(on=True):
    """Start (reset) or stop counting launches of this package's kernels; returns the count."""
    p = ext()
    n = p.launches
    if on:
        p.launches = 0
    p.counting = on
    return n


def available():
    return load() is not None
