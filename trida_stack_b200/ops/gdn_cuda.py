"""Gated-delta sub-block on the sm_100a kernels (``csrc/gdn.cu``).

``out = x + out_proj(gated_rmsnorm(GDN(conv(qkv)), z))`` with ``[qkv | z | b | a] =
rmsnorm(x) W_in^T``; the same math as ``ops.gdn.gdn_block_reference`` (reference:
``train/models/hybrid.py:215-451``).  Forward keeps the projection, the conv output, the recurrence
output and the per-chunk state checkpoints; backward recomputes the normalised input and the
gated-norm output instead of storing them.
"""
import torch

from ._ext import ext
from .blocks import TN, TT, _vec_buf, _vec_ret, _vgrad, _wgrad, gemm


def _geometry(lay, B, T):
    if lay.mode == "two_stream":
        return 1, lay.L, lay.V, lay.bd
    return 0, T, 0, 32


def _doc_u8(lay):
    if lay.doc_start is None:
        return None
    d = getattr(lay, "_doc_u8", None)
    if d is None:
        d = lay.doc_start.to(torch.uint8).contiguous()
        lay._doc_u8 = d
    return d


class _GdnBlock(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, norm_w, w_in, conv_w, dt_bias, A_log, gnorm, w_out, actx, cfg):
        lay = actx.linear
        B, T = actx.B, actx.T
        M, D = x.shape
        Hk, Hv, dk = cfg.lin_k_heads, cfg.lin_v_heads, cfg.lin_k_dim
        kd, vd = Hk * dk, Hv * cfg.lin_v_dim
        Cc = 2 * kd + vd
        mode, L, V, bd = _geometry(lay, B, T)
        doc = _doc_u8(lay)
        C = ext()
        h = torch.empty_like(x)
        _, rstd = C.rmsnorm_fwd(x, norm_w, cfg.eps, h)
        proj = torch.empty(M, w_in.shape[0], dtype=x.dtype, device=x.device)
        gemm(TN, h, w_in, proj)
        del h
        mixed = torch.empty(M, Cc, dtype=x.dtype, device=x.device)
        C.gdn_conv_fwd(proj[:, :Cc], conv_w, mixed, doc, B, T, mode, L, V, bd)
        z = proj[:, Cc:Cc + vd]
        gb = proj[:, Cc + vd:Cc + vd + Hv]
        ga = proj[:, Cc + vd + Hv:Cc + vd + 2 * Hv]
        a_log, dtb = A_log.float().contiguous(), dt_bias.float().contiguous()
        scale = dk ** -0.5
        flags = (lay.causal_clean, lay.causal_noisy)
        chunked = use_chunk_kernels(lay)
        if chunked:
            o, saved = chunk_forward(mixed, ga, gb, a_log, dtb, doc, B, T, Hk, Hv, lay, scale)
            ckpt = saved["bufs"]
            ctx.chunk_geo = saved["geo"]
        else:
            ckpt = [torch.empty(C.gdn_state_numel(B, T, Hv, mode, L, bd), dtype=torch.float32, device=x.device)]
            o = torch.empty(M, vd, dtype=x.dtype, device=x.device)
            C.gdn_fwd(mixed, ga, gb, a_log, dtb, doc, o, ckpt[0], B, T, Hk, Hv, mode, L, V, bd, flags[0], flags[1],
                      scale)
        ctx.chunked = chunked
        y = torch.empty(M, vd, dtype=x.dtype, device=x.device)
        C.gdn_gnorm_fwd(o, z, gnorm, y, Hv, cfg.eps)
        out = torch.empty_like(x)
        gemm(TN, y, w_out, out, x, 1.0, 1.0)
        ctx.save_for_backward(x, rstd, proj, mixed, o, *ckpt)
        ctx.params = (norm_w, w_in, conv_w, dt_bias, A_log, gnorm, w_out)   # see ops.blocks._AttnBlock
        ctx.geo = (B, T, Hk, Hv, dk, kd, vd, Cc, mode, L, V, bd, flags, scale)
        ctx.doc, ctx.eps = doc, cfg.eps
        return out

    @staticmethod
    def backward(ctx, dout):
        x, rstd, proj, mixed, o, *ckpt = ctx.saved_tensors
        norm_w, w_in, conv_w, dt_bias, A_log, gnorm, w_out = ctx.params
        B, T, Hk, Hv, dk, kd, vd, Cc, mode, L, V, bd, flags, scale = ctx.geo
        doc, eps = ctx.doc, ctx.eps
        M, D = x.shape
        C = ext()
        dout = dout.contiguous()
        z = proj[:, Cc:Cc + vd]
        gb = proj[:, Cc + vd:Cc + vd + Hv]
        ga = proj[:, Cc + vd + Hv:Cc + vd + 2 * Hv]
        # out_proj
        y = torch.empty(M, vd, dtype=x.dtype, device=x.device)
        C.gdn_gnorm_fwd(o, z, gnorm, y, Hv, eps)
        g_wout = _wgrad(dout, y, w_out)
        dy = y
        gemm(TT, dout, w_out, dy)
        # gated norm
        dproj = torch.empty_like(proj)
        do = torch.empty(M, vd, dtype=x.dtype, device=x.device)
        g_gn = _vec_buf(gnorm)
        C.gdn_gnorm_bwd(dy, o, z, gnorm, do, dproj[:, Cc:Cc + vd], g_gn, Hv, eps)
        del dy, y
        # recurrence (+ q/k L2-norm and gate backward)
        dmixed = torch.empty(M, Cc, dtype=x.dtype, device=x.device)
        dA = torch.zeros(Hv, dtype=torch.float32, device=x.device)
        ddt = torch.zeros(Hv, dtype=torch.float32, device=x.device)
        dga, dgb = dproj[:, Cc + vd + Hv:Cc + vd + 2 * Hv], dproj[:, Cc + vd:Cc + vd + Hv]
        if ctx.chunked:
            from .blocks import device_error_word
            C.gdn_chunk_bwd(mixed, ga, gb, A_log.float().contiguous(), dt_bias.float().contiguous(), doc, o, ckpt,
                            device_error_word(x.device), ctx.chunk_geo, scale, do, dmixed, dga, dgb, dA, ddt)
        else:
            C.gdn_bwd(mixed, ga, gb, A_log.float().contiguous(), dt_bias.float().contiguous(), doc, ckpt[0], do,
                      dmixed, dga, dgb, dA, ddt, B, T, Hk, Hv, mode, L, V, bd, flags[0], flags[1], scale)
        del do
        # conv
        g_conv = torch.zeros(conv_w.shape, dtype=torch.float32, device=x.device)
        C.gdn_conv_bwd(dmixed, proj[:, :Cc], conv_w, dproj[:, :Cc], g_conv, doc, B, T, mode, L, V, bd)
        del dmixed
        # in_proj (recompute the normalised input)
        h = torch.empty_like(x)
        C.rmsnorm_fwd(x, norm_w, eps, h)
        g_win = _wgrad(dproj, h, w_in)
        dh = h
        gemm(TT, dproj, w_in, dh)
        dx = torch.empty_like(x)
        gnw = _vec_buf(norm_w)
        C.rmsnorm_bwd(dh, x, norm_w, rstd, dout, dx, gnw)
        return (dx, _vec_ret(norm_w, gnw), g_win, _vgrad(conv_w, g_conv), _vgrad(dt_bias, ddt), _vgrad(A_log, dA),
                _vec_ret(gnorm, g_gn), g_wout, None, None)


def gdn_block_cuda(x, layer, actx, cfg):
    if cfg.lin_k_dim != 128 or cfg.lin_v_dim != 128 or cfg.conv_kernel > 4:
        raise NotImplementedError("the GDN kernels are built for 128-dim key/value heads and conv width <= 4")
    return _GdnBlock.apply(x, layer.input_norm, layer.w_in, layer.conv_w, layer.dt_bias, layer.A_log, layer.gnorm,
                           layer.w_out, actx, cfg)


def use_chunk_kernels(lay):
    """The chunked tcgen05 kernels serve every layout whose chunk length they support (override with
    TRIDA_GDN=scan to run the per-token recurrent scan instead)."""
    import os
    return os.environ.get("TRIDA_GDN", "chunk") == "chunk" and chunk_len(lay) is not None


def chunk_len(lay):
    """Chunk length of the tcgen05 chunk kernels for a layout (None: not supported, use the scan)."""
    if lay.mode == "two_stream":
        return lay.bd if lay.bd in (16, 32, 64) and lay.L % lay.bd == 0 else None
    return 64


def chunk_forward(mixed, ga, gb, A_log, dt_bias, doc, B, T, Hk, Hv, lay, scale, final_state=None):
    """Chunked gated-delta forward on the tcgen05 kernels (``csrc/gdn_chunk.cu``).  ``mixed`` is the
    conv output [B*T, >= 2*Hk*128 + Hv*128] (q | k | v columns), ``ga`` / ``gb`` the gate
    pre-activation views [B*T, Hv].  Returns (o [B*T, Hv*128] bf16, saved buffers)."""
    from .blocks import device_error_word
    C = chunk_len(lay)
    two = lay.mode == "two_stream"
    L, V = (lay.L, lay.V) if two else (0, 0)
    Lc = L if two else T
    nch = (Lc + C - 1) // C
    dev = mixed.device
    rows = B * T
    bf, f32 = torch.bfloat16, torch.float32
    bufs = [torch.empty(rows * Hk * 2 * 128, dtype=bf, device=dev), torch.empty(rows * Hv * 2, dtype=f32, device=dev)]
    bufs += [torch.empty(rows * Hv * 128, dtype=bf, device=dev) for _ in range(4)]
    bufs += [torch.empty(B * Hv * nch, dtype=f32, device=dev), torch.empty(B * Hv * nch * 128 * 128, dtype=bf, device=dev)]
    o = torch.empty(rows, Hv * 128, dtype=bf, device=dev)
    geo = [B, T, Hk, Hv, 1 if two else 0, L, V, C, int(lay.causal_clean), int(lay.causal_noisy)]
    ext().gdn_chunk_fwd(mixed, ga, gb, A_log.float().contiguous(), dt_bias.float().contiguous(), doc, o, bufs,
                        device_error_word(dev), geo, scale, final_state)
    return o, dict(bufs=bufs, geo=geo, C=C, nch=nch)
