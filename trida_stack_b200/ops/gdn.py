"""Gated-delta sub-block dispatch: CUDA kernels on GPU tensors, the PyTorch statement on CPU."""
from dataclasses import dataclass
from typing import Optional

import torch

from . import gdn_reference as G
from . import reference as R


@dataclass
class LinearLayout:
    """How the gated-delta layers see a row: ``causal`` (one stream of length T, documents start
    where ``doc_start`` is True) or ``two_stream`` (``[x0 ; xt_1..xt_V]`` streams of length L,
    blocks of ``bd``; ``doc_start`` [B, L] marks clean-stream document starts)."""
    mode: str = "causal"
    L: int = 0
    V: int = 0
    bd: int = 32
    causal_clean: bool = True
    causal_noisy: bool = False
    doc_start: Optional[torch.Tensor] = None


def _proj_split(proj, kd, vd, hv):
    qkv = proj[:, : 2 * kd + vd]
    z = proj[:, 2 * kd + vd: 2 * kd + 2 * vd]
    b = proj[:, 2 * kd + 2 * vd: 2 * kd + 2 * vd + hv]
    a = proj[:, 2 * kd + 2 * vd + hv:]
    return qkv, z, b, a


def gdn_block_reference(x, layer, actx, cfg):
    """x + out_proj(gated_norm(GDN(conv(qkv)), z)) on CPU, fp32 math (autograd-differentiable)."""
    lay = actx.linear
    B, T = actx.B, actx.T
    kd, vd, hv = layer.dims
    hk, dk, dv = cfg.lin_k_heads, cfg.lin_k_dim, cfg.lin_v_dim
    h = R.rmsnorm(x, layer.input_norm, cfg.eps)
    proj = h @ layer.w_in.t()
    qkv, z, b, a = _proj_split(proj, kd, vd, hv)
    qkv = qkv.reshape(B, T, -1)
    if lay.mode == "two_stream":
        mixed = G.two_stream_conv(qkv, layer.conv_w, lay.L, lay.V, lay.bd, lay.doc_start)
    else:
        mixed = G.causal_conv(qkv, layer.conv_w, lay.doc_start)
    q = mixed[..., :kd].reshape(B, T, hk, dk)
    k = mixed[..., kd:2 * kd].reshape(B, T, hk, dk)
    v = mixed[..., 2 * kd:].reshape(B, T, hv, dv)
    q, k = G.l2norm(q.float()), G.l2norm(k.float())
    rep = hv // hk
    if rep > 1:
        q, k = q.repeat_interleave(rep, 2), k.repeat_interleave(rep, 2)
    g, beta = G.gates(a.reshape(B, T, hv), b.reshape(B, T, hv), layer.A_log, layer.dt_bias)
    if lay.mode == "two_stream":
        o = G.gdn_two_stream(q, k, v.float(), g, beta, lay.L, lay.V, lay.bd, lay.causal_clean, lay.causal_noisy,
                             lay.doc_start)
    else:
        o, _ = G.gdn_causal(q, k, v.float(), g, beta, lay.doc_start)
    o = G.gated_rmsnorm(o.to(x.dtype), z.reshape(B, T, hv, dv), layer.gnorm, cfg.eps)
    return x + o.reshape(B * T, vd) @ layer.w_out.t()


def gdn_block(x, layer, actx, cfg):
    if x.is_cuda:
        from .gdn_cuda import gdn_block_cuda
        return gdn_block_cuda(x, layer, actx, cfg)
    return gdn_block_reference(x, layer, actx, cfg)
