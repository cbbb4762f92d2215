"""Fused decoder sub-blocks with hand-written backward passes.

A pre-norm residual sub-block ``out = x + f(rmsnorm(x))`` is one autograd node.  Its forward runs
the sm_100a kernels (tensor-core GEMMs with the residual add in the GEMM epilogue, RMSNorm,
q/k-norm + RoPE, block-diffusion attention, SwiGLU) and saves only what the backward cannot
cheaply recompute; its backward receives ``d out`` and returns ``d x = d out + d(norm path)``
with the residual gradient added inside the RMSNorm-backward kernel, so no separate gradient-add
kernels run.

Weight gradients go straight into each parameter's fp32 ``main_grad`` buffer (accumulating GEMM
epilogue, beta = 1) when the trainer attached one, so gradient accumulation over micro-batches
costs nothing extra; without ``main_grad`` they are returned to autograd as ordinary gradients.

On CPU every block runs the plain-PyTorch statement of the same math under autograd
(``ops.reference``), which is also the numerics oracle for the GPU path.
"""
import math
import os

import torch

from . import reference as R
from ._ext import ext

_MLP_RECOMPUTE = os.environ.get("TRIDA_MLP_RECOMPUTE", "0") == "1"

TN, TT, NT = 0, 1, 2


_ERR_WORDS = {}


def device_error_word(device):
    """int32 word that bounded device-side waits set (non-zero) instead of hanging."""
    key = str(device)
    if key not in _ERR_WORDS:
        _ERR_WORDS[key] = torch.zeros(1, dtype=torch.int32, device=device)
    return _ERR_WORDS[key]


def check_device_errors():
    """Raise if any kernel recorded a timed-out wait (host sync; call between steps)."""
    for key, w in _ERR_WORDS.items():
        code = int(w.item())
        if code:
            w.zero_()
            raise RuntimeError(f"device-side wait timed out on {key} (code {code})")
    if _ERR_WORDS:
        code = int(ext().gemm_error())
        if code:
            raise RuntimeError(f"GEMM mbarrier wait timed out (code {code})")


def use_tcgen05_attention(head_dim, which="FWD"):
    import os
    return head_dim in (64, 128, 256) and os.environ.get(f"TRIDA_ATTN_{which}", "tcgen05") == "tcgen05"


def gemm(layout, a, b, d, c=None, alpha=1.0, beta=0.0, tile=0):
    ext().gemm(layout, a, b, d, c, alpha, beta, tile)
    return d


def main_grad(w):
    """The fp32 gradient buffer of parameter ``w``: bound at construction (resident buffers) or on
    first use inside a backward (streamed per-layer gradients: ``w._grad_acquire`` binds a ring
    slot to the parameter's group); None for parameters outside the sharded optimizer."""
    mg = getattr(w, "main_grad", None)
    if mg is None:
        acq = getattr(w, "_grad_acquire", None)
        if acq is not None:
            acq()
            mg = w.main_grad
    return mg


def _wgrad(dy, x, w):
    """dW = dy^T x, accumulated into ``w.main_grad`` when present; else returned (fp32 -> w dtype)."""
    mg = main_grad(w)
    if mg is not None:
        gemm(NT, dy, x, mg, mg, 1.0, 1.0)
        return None
    out = torch.empty(w.shape, dtype=torch.float32, device=dy.device)
    gemm(NT, dy, x, out)
    return out.to(w.dtype)


def _vgrad(w, g):
    """Accumulate a vector-parameter gradient (fp32 ``g``) into main_grad, or return it."""
    mg = main_grad(w)
    if mg is not None:
        mg.add_(g)
        return None
    return g.to(w.dtype)


def _vec_buf(w):
    mg = main_grad(w)
    return mg if mg is not None else torch.zeros(w.shape, dtype=torch.float32, device=w.device)


def _vec_ret(w, buf):
    return None if getattr(w, "main_grad", None) is not None else buf.to(w.dtype)


# ---------------------------------------------------------------------------------------------
# attention context: per-forward metadata shared by every attention layer
# ---------------------------------------------------------------------------------------------
class AttnContext:
    """Mask metadata, tile plan and RoPE tables for one forward of a [B, T] layout.

    ``meta`` is int32 [B, T, 4] = (opos, rblk, segid, seg | view << 8); ``pos`` are the RoPE
    positions [B, T]; ``flags`` bit 0 = x0 token-causal, bit 1 = within-block causal.
    """

    def __init__(self, seg, opos, rblk, segid, view, pos, x0_token_causal, within_block_causal,
                 cos_t=None, sin_t=None):
        self.seg, self.opos, self.rblk, self.segid, self.view = seg, opos, rblk, segid, view
        self.pos = pos
        self.x0_token_causal = bool(x0_token_causal)
        self.within_block_causal = bool(within_block_causal)
        self.flags = (1 if x0_token_causal else 0) | (2 if within_block_causal else 0)
        self.B, self.T = seg.shape
        self.cos_t, self.sin_t = cos_t, sin_t
        self._plan = None
        if seg.is_cuda:
            self.meta = torch.stack([opos.int(), rblk.int(), segid.int(),
                                     (seg.int() | (view.int() << 8))], -1).contiguous()
            self.pos32 = pos.reshape(-1).int().contiguous()

    @property
    def plan(self):
        if self._plan is None:
            self._plan = ext().bd_attn_plan(self.meta, self.flags)
        return self._plan

    @property
    def plan128(self):
        """Non-empty 128x128 tile lists for the tcgen05 kernels."""
        if getattr(self, "_plan128", None) is None:
            self._plan128 = ext().bd_attn_lists128(self.plan[0], self.T, 0)
        return self._plan128

    @property
    def masks(self):
        """(row, column) bit masks of the PARTIAL 128x128 tiles, shared by all layers and heads."""
        if getattr(self, "_masks", None) is None:
            self._masks = ext().bd_attn_tile_masks(self.meta, self.plan[0], self.flags)
        return self._masks

    @property
    def plan128t(self):
        """Per 128-key tile, the non-empty 128-query tiles (tcgen05 backward)."""
        if getattr(self, "_plan128t", None) is None:
            self._plan128t = ext().bd_attn_lists128(self.plan[0], self.T, 1)
        return self._plan128t

    def meta_dict(self):
        return {"seg": self.seg, "opos": self.opos, "rblk": self.rblk, "segid": self.segid,
                "view": self.view}

    def set_rope_angles(self, ang):
        """Per-token rotary angles [B, T, rotary_dim / 2] (3-D RoPE of vision-language rows) instead
        of the shared position table: the CUDA path indexes per-token cos / sin rows by token."""
        self.rope_angles = ang
        if self.seg.is_cuda:
            flat = ang.reshape(-1, ang.shape[-1]).float()
            self.cos_t, self.sin_t = flat.cos().contiguous(), flat.sin().contiguous()
            self.pos32 = torch.arange(flat.shape[0], dtype=torch.int32, device=ang.device)


def rope_tables(max_pos, rotary_dim, theta, device):
    """fp32 cos/sin tables [max_pos, rotary_dim/2] (HF default RoPE, half-split pairs)."""
    inv = 1.0 / (theta ** (torch.arange(0, rotary_dim, 2, dtype=torch.float32, device=device) / rotary_dim))
    f = torch.arange(max_pos, dtype=torch.float32, device=device)[:, None] * inv[None]
    return f.cos().contiguous(), f.sin().contiguous()


def attn_fwd(q, k, v, o, lse, actx):
    """Block-diffusion attention forward: tcgen05 kernel for head_dim 64/128, else the warp-MMA one."""
    d = q.shape[-1]
    if use_tcgen05_attention(d):
        l128, c128 = actx.plan128
        ext().bd_attn_fwd_sm100(q, k, v, o, lse, actx.meta, l128, c128, actx.masks[0], actx.flags,
                                1.0 / math.sqrt(d), device_error_word(q.device))
    else:
        _, fl, fc, _, _ = actx.plan
        ext().bd_attn_fwd(q, k, v, o, lse, actx.meta, fl, fc, actx.flags, 1.0 / math.sqrt(d))


def attn_bwd(q, k, v, o, lse, do, dq, dk, dv, actx):
    d = q.shape[-1]
    if use_tcgen05_attention(d, "BWD"):
        lt, ct = actx.plan128t
        extra = {}
        if d == 256:   # the dQ kernel walks the forward lists with the row masks
            l128, c128 = actx.plan128
            extra = {"list128": l128, "cnt128": c128, "rowmask": actx.masks[0]}
        ext().bd_attn_bwd_sm100(q, k, v, o, lse, do, dq, dk, dv, actx.meta, lt, ct, actx.masks[1], actx.flags,
                                1.0 / math.sqrt(d), device_error_word(q.device), **extra)
    else:
        _, _, _, bl, bc = actx.plan
        ext().bd_attn_bwd(q, k, v, o, lse, do, dq, dk, dv, actx.meta, bl, bc, actx.flags, 1.0 / math.sqrt(d))


# ---------------------------------------------------------------------------------------------
# attention sub-block:  out = x + o_proj(attn(rope(qk_norm(qkv_proj(rmsnorm(x))))))
# ---------------------------------------------------------------------------------------------
class _AttnBlock(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, norm_w, wqkv, qn, kn, wo, actx, cfg):
        B, T, Hq, Hkv, d, rd, eps = actx.B, actx.T, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.rotary_dim, cfg.eps
        M, D = x.shape
        C = ext()
        h = torch.empty_like(x)
        _, rstd = C.rmsnorm_fwd(x, norm_w, eps, h)
        qkv = torch.empty(M, wqkv.shape[0], dtype=x.dtype, device=x.device)
        gemm(TN, h, wqkv, qkv)
        del h
        qs = 2 * d if cfg.attn_output_gate else d      # gated: per head [query (d) | gate (d)]
        q = torch.empty(B, T, Hq, d, dtype=x.dtype, device=x.device)
        k = torch.empty(B, T, Hkv, d, dtype=x.dtype, device=x.device)
        rstd_qk = C.qk_norm_rope_fwd(qkv, qn, kn, actx.cos_t, actx.sin_t, actx.pos32, q, k, Hq, Hkv, d, rd, eps, qs)
        v = qkv.view(B, T, -1)[:, :, Hq * qs + Hkv * d:].view(B, T, Hkv, d)
        o = torch.empty(B, T, Hq, d, dtype=x.dtype, device=x.device)
        lse = torch.empty(B, Hq, T, dtype=torch.float32, device=x.device)
        attn_fwd(q, k, v, o, lse, actx)
        out = torch.empty_like(x)
        if cfg.attn_output_gate:
            og = torch.empty(M, Hq * d, dtype=x.dtype, device=x.device)
            C.attn_gate_fwd(o.view(M, Hq * d), qkv, og, Hq, d)
            gemm(TN, og, wo, out, x, 1.0, 1.0)
            del og
        else:
            gemm(TN, o.view(M, Hq * d), wo, out, x, 1.0, 1.0)
        # parameters ride on ctx (not saved tensors): recomputation under activation checkpointing
        # unpacks saved tensors as fresh aliases without the parameters' gradient-buffer attributes
        ctx.save_for_backward(x, rstd, qkv, rstd_qk, q, k, o, lse)
        ctx.params = (norm_w, wqkv, qn, kn, wo)
        ctx.actx, ctx.cfg = actx, cfg
        return out

    @staticmethod
    def backward(ctx, dout):
        x, rstd, qkv, rstd_qk, q, k, o, lse = ctx.saved_tensors
        norm_w, wqkv, qn, kn, wo = ctx.params
        actx, cfg = ctx.actx, ctx.cfg
        B, T, Hq, Hkv, d, rd, eps = actx.B, actx.T, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.rotary_dim, cfg.eps
        M, D = x.shape
        C = ext()
        dout = dout.contiguous()
        qs = 2 * d if cfg.attn_output_gate else d
        # o_proj (and the sigmoid output gate)
        dqkv = torch.empty_like(qkv)
        do = torch.empty(M, Hq * d, dtype=x.dtype, device=x.device)
        gemm(TT, dout, wo, do)
        if cfg.attn_output_gate:
            og = torch.empty(M, Hq * d, dtype=x.dtype, device=x.device)
            C.attn_gate_fwd(o.view(M, Hq * d), qkv, og, Hq, d)
            g_wo = _wgrad(dout, og, wo)
            d_o = og
            C.attn_gate_bwd(do, o.view(M, Hq * d), qkv, d_o, dqkv, Hq, d)
            do = d_o
        else:
            g_wo = _wgrad(dout, o.view(M, Hq * d), wo)
        # attention
        dq = torch.empty_like(q)
        dk = torch.empty_like(k)
        dv = dqkv.view(B, T, -1)[:, :, Hq * qs + Hkv * d:].view(B, T, Hkv, d)
        v = qkv.view(B, T, -1)[:, :, Hq * qs + Hkv * d:].view(B, T, Hkv, d)
        attn_bwd(q, k, v, o, lse, do.view(B, T, Hq, d), dq, dk, dv, actx)
        del do
        gqn, gkn = _vec_buf(qn), _vec_buf(kn)
        C.qk_norm_rope_bwd(dq, dk, qkv, qn, kn, actx.cos_t, actx.sin_t, actx.pos32, rstd_qk, dqkv, gqn, gkn,
                           Hq, Hkv, d, rd, qs)
        del dq, dk
        # qkv_proj (recompute the normalised input)
        h = torch.empty_like(x)
        C.rmsnorm_fwd(x, norm_w, eps, h)
        g_wqkv = _wgrad(dqkv, h, wqkv)
        dh = h
        gemm(TT, dqkv, wqkv, dh)
        dx = torch.empty_like(x)
        gnw = _vec_buf(norm_w)
        C.rmsnorm_bwd(dh, x, norm_w, rstd, dout, dx, gnw)
        return dx, _vec_ret(norm_w, gnw), g_wqkv, _vec_ret(qn, gqn), _vec_ret(kn, gkn), g_wo, None, None


def _attn_block_ref(x, norm_w, wqkv, qn, kn, wo, actx, cfg):
    B, T, Hq, Hkv, d, eps = actx.B, actx.T, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.eps
    h = R.rmsnorm(x, norm_w, eps)
    qkv = h @ wqkv.t()
    gate = None
    if cfg.attn_output_gate:
        qg = qkv[:, : 2 * Hq * d].view(B, T, Hq, 2 * d)
        q, gate = qg[..., :d], qg[..., d:].reshape(B * T, Hq * d)
        k = qkv[:, 2 * Hq * d:(2 * Hq + Hkv) * d].view(B, T, Hkv, d)
        v = qkv[:, (2 * Hq + Hkv) * d:].view(B, T, Hkv, d)
    else:
        q = qkv[:, : Hq * d].view(B, T, Hq, d)
        k = qkv[:, Hq * d:(Hq + Hkv) * d].view(B, T, Hkv, d)
        v = qkv[:, (Hq + Hkv) * d:].view(B, T, Hkv, d)
    q = R.rmsnorm(q, qn, eps)
    k = R.rmsnorm(k, kn, eps)
    ang = getattr(actx, "rope_angles", None)
    if ang is not None:
        cos, sin = torch.cat([ang, ang], -1).cos(), torch.cat([ang, ang], -1).sin()
    else:
        cos, sin = R.rope_cos_sin(actx.pos, d, cfg.rope_theta, cfg.rotary_dim, dtype=torch.float32)
    q = R.apply_rope(q.float(), cos, sin).to(x.dtype)
    k = R.apply_rope(k.float(), cos, sin).to(x.dtype)
    o = R.bd_attention(q, k, v, actx.meta_dict(), actx.x0_token_causal, actx.within_block_causal)
    o = o.reshape(B * T, Hq * d)
    if gate is not None:
        o = o * torch.sigmoid(gate.float()).to(o.dtype)
    return x + o @ wo.t()


def attn_block(x, norm_w, wqkv, qn, kn, wo, actx, cfg):
    if x.is_cuda:
        return _AttnBlock.apply(x, norm_w, wqkv, qn, kn, wo, actx, cfg)
    return _attn_block_ref(x, norm_w, wqkv, qn, kn, wo, actx, cfg)


# ---------------------------------------------------------------------------------------------
# MLP sub-block:  out = x + down(silu(gate(h)) * up(h)),  h = rmsnorm(x);  wgu = [gate; up]
# ---------------------------------------------------------------------------------------------
class _MlpBlock(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, norm_w, wgu, wd, eps):
        M, D = x.shape
        F2 = wgu.shape[0]
        C = ext()
        h = torch.empty_like(x)
        _, rstd = C.rmsnorm_fwd(x, norm_w, eps, h)
        gu = torch.empty(M, F2, dtype=x.dtype, device=x.device)
        a = torch.empty(M, F2 // 2, dtype=x.dtype, device=x.device)
        if F2 % 128 == 0:
            C.gemm_swiglu(h, wgu, gu, a)        # SwiGLU in the GEMM epilogue
        else:
            gemm(TN, h, wgu, gu)
            C.swiglu_fwd(gu, a)
        del h
        out = torch.empty_like(x)
        gemm(TN, a, wd, out, x, 1.0, 1.0)
        # keeping a (M x F bf16) saves one SwiGLU pass in the backward; TRIDA_MLP_RECOMPUTE=1
        # trades it back for memory
        keep = not _MLP_RECOMPUTE
        ctx.save_for_backward(x, rstd, gu, a if keep else None)
        ctx.params = (norm_w, wgu, wd)
        ctx.eps = eps
        return out

    @staticmethod
    def backward(ctx, dout):
        x, rstd, gu, a = ctx.saved_tensors
        norm_w, wgu, wd = ctx.params
        M, D = x.shape
        F = gu.shape[1] // 2
        C = ext()
        dout = dout.contiguous()
        if a is None:
            a = torch.empty(M, F, dtype=x.dtype, device=x.device)
            C.swiglu_fwd(gu, a)
        g_wd = _wgrad(dout, a, wd)
        da = a
        gemm(TT, dout, wd, da)
        dgu = torch.empty_like(gu)
        C.swiglu_bwd(da, gu, dgu)
        del a, da
        h = torch.empty_like(x)
        C.rmsnorm_fwd(x, norm_w, ctx.eps, h)
        g_wgu = _wgrad(dgu, h, wgu)
        dh = h
        gemm(TT, dgu, wgu, dh)
        dx = torch.empty_like(x)
        gnw = _vec_buf(norm_w)
        C.rmsnorm_bwd(dh, x, norm_w, rstd, dout, dx, gnw)
        return dx, _vec_ret(norm_w, gnw), g_wgu, g_wd, None


def mlp_block(x, norm_w, wgu, wd, eps):
    if x.is_cuda:
        return _MlpBlock.apply(x, norm_w, wgu, wd, eps)
    h = R.rmsnorm(x, norm_w, eps)
    return x + R.swiglu(h @ wgu.t()) @ wd.t()


# ---------------------------------------------------------------------------------------------
# final RMSNorm and the embedding
# ---------------------------------------------------------------------------------------------
class _Norm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        h = torch.empty_like(x)
        _, rstd = ext().rmsnorm_fwd(x, w, eps, h)
        ctx.save_for_backward(x, rstd)
        ctx.w = w
        return h

    @staticmethod
    def backward(ctx, dh):
        x, rstd = ctx.saved_tensors
        w = ctx.w
        dx = torch.empty_like(x)
        gw = _vec_buf(w)
        ext().rmsnorm_bwd(dh.contiguous(), x, w, rstd, None, dx, gw)
        return dx, _vec_ret(w, gw), None


def rmsnorm(x, w, eps):
    if x.is_cuda:
        return _Norm.apply(x, w, eps)
    return R.rmsnorm(x, w, eps)


class _Embed(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, table):
        ids = ids.reshape(-1).contiguous()
        out = torch.empty(ids.numel(), table.shape[1], dtype=table.dtype, device=table.device)
        ext().embed_fwd(ids, table, out)
        ctx.save_for_backward(ids)
        ctx.table = table
        return out

    @staticmethod
    def backward(ctx, dout):
        ids, = ctx.saved_tensors
        table = ctx.table
        mg = main_grad(table)
        buf = mg if mg is not None else torch.zeros(table.shape, dtype=torch.float32, device=table.device)
        ext().embed_bwd(ids, dout.contiguous(), buf)
        return None, (None if mg is not None else buf.to(table.dtype))


def embedding(ids, table):
    """ids [...] -> [ids.numel(), D] rows of ``table``."""
    if table.is_cuda:
        return _Embed.apply(ids, table)
    return table[ids.reshape(-1)]
