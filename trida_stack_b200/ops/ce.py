"""Fused linear cross-entropy: ``sum_i weight_i * CE(h_i . W^T, target_i)`` without an [N, V] logit tensor.

CUDA path, per chunk of rows: tensor-core GEMM for fp32 logits -> one row kernel computes the
per-row CE and, in the same pass, the bf16 logit gradient ``(softmax - onehot) * weight`` ->
two GEMMs turn it into dH (stored) and dW (accumulated in fp32).  The loss is final when the
forward returns, so the backward only scales the stored dH / dW by the incoming gradient: the
logits are computed exactly once (the reference's checkpointed chunked CE computes them twice).

Weights carry every coefficient of the objective (1/gamma ELBO weights normalised to sum 1,
the AR mean, and the ``(diff + w * ar) / (1 + w)`` mix), so the diffusion and AR losses share
one call.  Per-row CE values are returned (detached) for logging.
"""
import torch

from . import reference as R
from ._ext import ext
from .blocks import main_grad, NT, TN, TT, gemm


class _FusedLinearCE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, w, target, weight, chunk):
        N, D = h.shape
        V = w.shape[0]
        C = ext()
        dev = h.device
        ce = torch.empty(N, dtype=torch.float32, device=dev)
        dh = torch.empty(N, D, dtype=h.dtype, device=dev)
        need_w = w.requires_grad
        dw = torch.empty(V, D, dtype=torch.float32, device=dev) if need_w else None
        c0 = max(1, min(chunk, N))
        logits = torch.empty(c0, V, dtype=torch.float32, device=dev)
        dlog = torch.empty(c0, V, dtype=torch.bfloat16, device=dev)
        for i in range(0, N, c0):
            c = min(c0, N - i)
            hs = h[i:i + c]
            gemm(TN, hs, w, logits[:c])
            C.ce_rows(logits[:c], target[i:i + c], weight[i:i + c], 1.0, ce[i:i + c], dlog[:c])
            gemm(TT, dlog[:c], w, dh[i:i + c])
            if need_w:
                if i == 0:
                    gemm(NT, dlog[:c], hs, dw)
                else:
                    gemm(NT, dlog[:c], hs, dw, dw, 1.0, 1.0)
        del logits, dlog
        loss = torch.dot(ce, weight)
        ctx.save_for_backward(dh, dw if need_w else torch.empty(0, device=dev))
        ctx.need_w = need_w
        ctx.w = w
        ctx.mark_non_differentiable(ce)
        return loss, ce

    @staticmethod
    def backward(ctx, gloss, gce):
        dh, dw = ctx.saved_tensors
        g = gloss.float()
        gh = (dh.float() * g).to(dh.dtype)
        gw = None
        if ctx.need_w:
            w = ctx.w
            mg = main_grad(w)
            if mg is not None:
                mg.addcmul_(dw, g)
            else:
                gw = (dw * g).to(w.dtype)
        return gh, gw, None, None, None


def fused_linear_ce(h, w, target, weight, chunk=4096):
    """Returns (loss, per-row CE).  ``weight`` [N] fp32 multiplies each row's CE."""
    if h.shape[0] == 0:
        z = h.sum() * 0.0
        return z, torch.zeros(0, dtype=torch.float32, device=h.device)
    if h.is_cuda:
        return _FusedLinearCE.apply(h.contiguous(), w, target.contiguous(), weight.float().contiguous(), chunk)
    logits = h.float() @ w.float().t()
    ce = torch.nn.functional.cross_entropy(logits, target, reduction="none")
    return (ce * weight.float()).sum(), ce.detach()


__all__ = ["fused_linear_ce", "R"]
