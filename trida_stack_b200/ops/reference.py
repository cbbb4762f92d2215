"""Plain PyTorch statements of every hot op (fp32 math).

These are the CPU execution path of the framework and the numerics oracles the CUDA kernels are
tested against.  Each function states the math once, in the simplest form; nothing here is tuned.
"""
import math

import torch
import torch.nn.functional as F

# Segment classes of the block-diffusion layout (same numbering as the reference's mask_mod,
# ``train/models/block_diffusion.py:32``): padding, shared prompt, noised response, clean response.
PAD, SHARED, XT, X0 = 0, 1, 2, 3


def rmsnorm(x, w, eps):
    xf = x.float()
    r = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (xf * r * w.float()).to(x.dtype)


def rope_cos_sin(pos, head_dim, theta, rotary_dim=None, dtype=torch.float32):
    """cos/sin tables [*, rotary_dim] for integer positions ``pos`` (half-split layout)."""
    rd = head_dim if rotary_dim is None else rotary_dim
    inv = 1.0 / (theta ** (torch.arange(0, rd, 2, dtype=torch.float32, device=pos.device) / rd))
    f = pos.float()[..., None] * inv
    emb = torch.cat([f, f], -1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def apply_rope(x, cos, sin):
    """x [..., T, H, d] with cos/sin [..., T, rd]; rotates the first rd channels (half-split)."""
    rd = cos.shape[-1]
    xr, xp = x[..., :rd], x[..., rd:]
    x1, x2 = xr[..., : rd // 2], xr[..., rd // 2:]
    c, s = cos[..., None, :], sin[..., None, :]
    rot = torch.cat([-x2, x1], -1)
    return torch.cat([xr * c + rot * s, xp], -1)


def swiglu(gu):
    g, u = gu.chunk(2, dim=-1)
    return (F.silu(g.float()) * u.float()).to(gu.dtype)


def bd_allowed(meta_q, meta_k, x0_token_causal, within_block_causal, same_index):
    """Dense boolean mask [B, Tq, Tk] of the block-diffusion attention rule.

    ``meta_*`` are dicts of int tensors [B, T]: ``seg`` (PAD/SHARED/XT/X0), ``opos`` (original
    position), ``rblk`` (response block), ``segid`` (packed document id, -1 = none) and ``view``
    (complementary view, 0 for shared regions).  ``same_index`` [Tq, Tk] marks q == kv (every row
    keeps itself so no softmax row is empty).  Rules: ``train/models/block_diffusion.py:245-264``
    (single row), ``:312-328`` (packed: ``same_seg``), ``:344-361`` (merged views: ``same view``).
    """
    sq, sk = meta_q["seg"][:, :, None], meta_k["seg"][:, None, :]
    oq, ok = meta_q["opos"][:, :, None], meta_k["opos"][:, None, :]
    bq, bk = meta_q["rblk"][:, :, None], meta_k["rblk"][:, None, :]
    gq, gk = meta_q["segid"][:, :, None], meta_k["segid"][:, None, :]
    vq, vk = meta_q["view"][:, :, None], meta_k["view"][:, None, :]
    kv_ok = sk != PAD
    same_seg = gq == gk
    to_shared = (sk == SHARED) & (ok <= oq)
    xt_diag = (sq == XT) & (sk == XT) & (bq == bk) & (vq == vk)
    if within_block_causal:
        xt_diag = xt_diag & (ok <= oq)
    xt_offset = (sq == XT) & (sk == X0) & (bk < bq)
    if x0_token_causal:
        x0c = (sq == X0) & (sk == X0) & (ok <= oq)
    else:
        x0c = (sq == X0) & (sk == X0) & (bk <= bq)
    rule = to_shared | xt_diag | xt_offset | x0c
    return (kv_ok & same_seg & rule) | same_index[None]


def bd_attention(q, k, v, meta, x0_token_causal, within_block_causal, scale=None):
    """q [B, T, Hq, d], k/v [B, T, Hkv, d] -> [B, T, Hq, d] under the block-diffusion mask."""
    B, T, Hq, d = q.shape
    Hkv = k.shape[2]
    scale = 1.0 / math.sqrt(d) if scale is None else scale
    eye = torch.eye(T, dtype=torch.bool, device=q.device)
    allowed = bd_allowed(meta, meta, x0_token_causal, within_block_causal, eye)  # [B, T, T]
    qf = q.float().transpose(1, 2)
    kf = k.float().transpose(1, 2).repeat_interleave(Hq // Hkv, 1)
    vf = v.float().transpose(1, 2).repeat_interleave(Hq // Hkv, 1)
    s = (qf @ kf.transpose(-1, -2)) * scale
    s = s.masked_fill(~allowed[:, None], float("-inf"))
    p = torch.softmax(s, -1)
    return (p @ vf).transpose(1, 2).to(q.dtype)


def doc_causal_attention(q, k, v, segid, scale=None):
    """Causal attention restricted to equal ``segid`` (packed AR rows)."""
    B, T, Hq, d = q.shape
    Hkv = k.shape[2]
    scale = 1.0 / math.sqrt(d) if scale is None else scale
    ar = torch.arange(T, device=q.device)
    allowed = (ar[:, None] >= ar[None, :])[None] & (segid[:, :, None] == segid[:, None, :])
    allowed = allowed | torch.eye(T, dtype=torch.bool, device=q.device)[None]
    qf = q.float().transpose(1, 2)
    kf = k.float().transpose(1, 2).repeat_interleave(Hq // Hkv, 1)
    vf = v.float().transpose(1, 2).repeat_interleave(Hq // Hkv, 1)
    s = (qf @ kf.transpose(-1, -2)) * scale
    s = s.masked_fill(~allowed[:, None], float("-inf"))
    return (torch.softmax(s, -1) @ vf).transpose(1, 2).to(q.dtype)


def linear_ce(h, w, target, weight=None):
    """Per-token CE of ``h @ w^T`` against ``target``; returns the weighted sum (or the mean)."""
    logits = h.float() @ w.float().t()
    ce = F.cross_entropy(logits, target, reduction="none")
    return ce.mean() if weight is None else (ce * weight).sum()


def l2norm(x, eps=1e-6):
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).sum(-1, keepdim=True) + eps)).to(x.dtype)
