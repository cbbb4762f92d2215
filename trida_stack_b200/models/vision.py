"""Qwen3.5 vision tower (image encoder + 2x2 patch merger) and the text side's 3-D RoPE.

The vision-language Qwen3.5 checkpoints (``Qwen3_5ForConditionalGeneration``) carry a ViT under
``model.visual.*``.  The reference trains them with the encoder frozen and the merger ("projector")
trainable at ``--projector_lr_scale`` (``train/models/block_diffusion.py:180-201``,
``train/models/build.py:52-57``); image features replace the ``<|image_pad|>`` embeddings of the
clean stream and of every noisy view (``train/models/hybrid.py:990-1004``), and the full-attention
layers rotate q / k with interleaved 3-D (t, h, w) positions (``train/data/text_sft_data.py:155-182``).

Architecture (the checkpoint's contract, stated here from the published model):

* patch embedding: a linear map of each flattened ``[C, T_patch, p, p]`` patch (the Conv3d with
  stride = kernel of the checkpoint, stored as ``patch_embed.proj.weight [D, C, T, p, p]``) plus bias,
  plus a learned ``[G*G, D]`` position table bilinearly resampled to the image's patch grid;
* ``depth`` pre-LayerNorm blocks: bidirectional attention inside each image frame with 2-D RoPE
  (row angles on the first quarter of the head, column angles on the second, half-split rotation)
  and a GELU(tanh) MLP, all linear layers with bias;
* merger: LayerNorm, then every 2x2 group of neighbouring patches concatenated (patches arrive in
  merge-block order) and mapped by Linear -> GELU -> Linear to the language model's width.

Patches are ordered ``(t, block_row, block_col, row_in_block, col_in_block)`` -- the image
processor's layout (``data.images``) -- so the merge is a reshape.

The tower runs on PyTorch ops (cuBLAS GEMMs, SDPA); it is outside every benchmarked configuration,
its 72-wide heads fit none of the attention kernels, and only the merger needs gradients.
"""
import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass
class VisionConfig:
    depth: int = 27
    hidden_size: int = 1152
    intermediate_size: int = 4304
    num_heads: int = 16
    in_channels: int = 3
    patch_size: int = 16
    temporal_patch_size: int = 2
    spatial_merge_size: int = 2
    out_hidden_size: int = 2560
    num_position_embeddings: int = 2304
    hidden_act: str = "gelu_pytorch_tanh"

    @classmethod
    def from_dict(cls, d):
        keys = cls.__dataclass_fields__
        return cls(**{k: d[k] for k in keys if k in d})

    @property
    def head_dim(self):
        return self.hidden_size // self.num_heads

    @property
    def patch_dim(self):
        return self.in_channels * self.temporal_patch_size * self.patch_size ** 2


def _gelu(x, act):
    return F.gelu(x, approximate="tanh") if act in ("gelu_pytorch_tanh", "gelu_new") else F.gelu(x)


class _Attn(nn.Module):
    def __init__(self, c: VisionConfig):
        super().__init__()
        self.qkv = nn.Linear(c.hidden_size, 3 * c.hidden_size)
        self.proj = nn.Linear(c.hidden_size, c.hidden_size)


class _Mlp(nn.Module):
    def __init__(self, c: VisionConfig):
        super().__init__()
        self.linear_fc1 = nn.Linear(c.hidden_size, c.intermediate_size)
        self.linear_fc2 = nn.Linear(c.intermediate_size, c.hidden_size)


class _Block(nn.Module):
    def __init__(self, c: VisionConfig):
        super().__init__()
        self.norm1 = nn.LayerNorm(c.hidden_size, eps=1e-6)
        self.norm2 = nn.LayerNorm(c.hidden_size, eps=1e-6)
        self.attn = _Attn(c)
        self.mlp = _Mlp(c)


class _PatchEmbed(nn.Module):
    def __init__(self, c: VisionConfig):
        super().__init__()
        # stored in the checkpoint's Conv3d shape; applied as one GEMM over flattened patches
        self.proj = nn.Module()
        self.proj.weight = nn.Parameter(torch.empty(c.hidden_size, c.in_channels, c.temporal_patch_size,
                                                    c.patch_size, c.patch_size))
        self.proj.bias = nn.Parameter(torch.zeros(c.hidden_size))


class _Merger(nn.Module):
    def __init__(self, c: VisionConfig):
        super().__init__()
        wide = c.hidden_size * c.spatial_merge_size ** 2
        self.norm = nn.LayerNorm(c.hidden_size, eps=1e-6)
        self.linear_fc1 = nn.Linear(wide, wide)
        self.linear_fc2 = nn.Linear(wide, c.out_hidden_size)


class VisionTower(nn.Module):
    """``forward(pixel_values [P, patch_dim], grid_thw [N, 3]) -> [P / merge^2, out_hidden]``.

    Parameter names equal the checkpoint's names under ``model.visual.`` (``hf_items``)."""

    def __init__(self, c: VisionConfig, dtype=torch.bfloat16, device=None):
        super().__init__()
        self.c = c
        with torch.device(device or "cpu"):
            self.patch_embed = _PatchEmbed(c)
            self.pos_embed = nn.Embedding(c.num_position_embeddings, c.hidden_size)
            self.blocks = nn.ModuleList([_Block(c) for _ in range(c.depth)])
            self.merger = _Merger(c)
        self.side = int(math.isqrt(c.num_position_embeddings))
        self.reset_parameters()
        self.to(dtype)

    @torch.no_grad()
    def reset_parameters(self, std=0.02):
        for name, p in self.named_parameters():
            if name.endswith("bias"):
                p.zero_()
            elif p.dim() >= 2:
                p.normal_(0.0, std)
            else:
                p.fill_(1.0)

    def freeze_encoder(self):
        """Encoder frozen, merger trainable (the reference's VL training recipe)."""
        for name, p in self.named_parameters():
            p.requires_grad_(name.startswith("merger."))

    # ------------------------------------------------------------------------------- geometry
    def _grid_list(self, grid_thw):
        return [tuple(int(v) for v in row) for row in grid_thw.tolist()]

    def _block_order(self, t, h, w):
        """(row, col) of every patch in merge-block order, [t*h*w, 2]."""
        m = self.c.spatial_merge_size
        r = torch.arange(h).view(h // m, 1, m, 1).expand(h // m, w // m, m, m)
        cidx = torch.arange(w).view(1, w // m, 1, m).expand(h // m, w // m, m, m)
        rc = torch.stack([r.reshape(-1), cidx.reshape(-1)], -1)
        return rc.repeat(t, 1)

    def rope_angles(self, grids, device):
        """Per patch, the 2-D rotary angles [P, head_dim / 2]: row angles then column angles, each
        over ``head_dim / 4`` inverse frequencies of base 10000 on a ``head_dim / 2`` rotary width."""
        dim = self.c.head_dim // 2
        inv = 1.0 / (10000.0 ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))
        rc = torch.cat([self._block_order(t, h, w) for t, h, w in grids]).float()
        ang = torch.cat([rc[:, :1] * inv[None], rc[:, 1:] * inv[None]], -1)
        return ang.to(device)

    def pos_embedding(self, grids):
        """Learned G x G position table bilinearly resampled to each image's grid (corner-aligned
        sample points ``linspace(0, G - 1, n)``), in merge-block order."""
        G = self.side
        W = self.pos_embed.weight
        outs = []
        for t, h, w in grids:
            ys = torch.linspace(0, G - 1, h)
            xs = torch.linspace(0, G - 1, w)
            y0, x0 = ys.floor().long(), xs.floor().long()
            y1, x1 = (y0 + 1).clamp(max=G - 1), (x0 + 1).clamp(max=G - 1)
            fy, fx = (ys - y0.float())[:, None], (xs - x0.float())[None, :]
            idx = torch.stack([(y0[:, None] * G + x0[None]), (y0[:, None] * G + x1[None]),
                               (y1[:, None] * G + x0[None]), (y1[:, None] * G + x1[None])]).reshape(4, -1)
            wts = torch.stack([(1 - fy) * (1 - fx), (1 - fy) * fx, fy * (1 - fx), fy * fx]).reshape(4, -1)
            wts = wts.to(W.device, W.dtype)
            e = (W[idx.to(W.device)] * wts[..., None]).sum(0)                   # [h*w, D], raster order
            rc = self._block_order(1, h, w)
            e = e[(rc[:, 0] * w + rc[:, 1]).to(W.device)]
            outs.append(e.repeat(t, 1))
        return torch.cat(outs)

    # -------------------------------------------------------------------------------- forward
    def encode(self, pixel_values, grid_thw):
        """Encoder output before the merger, [P, D]."""
        c = self.c
        grids = self._grid_list(grid_thw)
        dt = self.pos_embed.weight.dtype
        pw = self.patch_embed.proj
        x = F.linear(pixel_values.to(dt).reshape(-1, c.patch_dim), pw.weight.reshape(c.hidden_size, -1), pw.bias)
        x = x + self.pos_embedding(grids)
        ang = self.rope_angles(grids, x.device)
        cos = torch.cat([ang, ang], -1).cos()[:, None]                        # [P, 1, hd]
        sin = torch.cat([ang, ang], -1).sin()[:, None]
        lens = [h * w for t, h, w in grids for _ in range(t)]
        H, hd = c.num_heads, c.head_dim
        for blk in self.blocks:
            y = blk.norm1(x)
            q, k, v = blk.attn.qkv(y).view(-1, 3, H, hd).unbind(1)
            q = _rotate(q.float(), cos, sin).to(dt)
            k = _rotate(k.float(), cos, sin).to(dt)
            outs, o0 = [], 0
            for n in lens:                                                     # bidirectional per frame
                sl = slice(o0, o0 + n)
                outs.append(F.scaled_dot_product_attention(q[sl].transpose(0, 1), k[sl].transpose(0, 1),
                                                           v[sl].transpose(0, 1)).transpose(0, 1))
                o0 += n
            x = x + blk.attn.proj(torch.cat(outs).reshape(-1, H * hd))
            x = x + blk.mlp.linear_fc2(_gelu(blk.mlp.linear_fc1(blk.norm2(x)), c.hidden_act))
        return x

    def merge(self, x):
        m2 = self.c.spatial_merge_size ** 2
        mg = self.merger
        y = mg.norm(x).reshape(-1, self.c.hidden_size * m2)
        return mg.linear_fc2(F.gelu(mg.linear_fc1(y)))

    def forward(self, pixel_values, grid_thw):
        enc_trainable = any(p.requires_grad for n, p in self.named_parameters() if not n.startswith("merger."))
        with torch.set_grad_enabled(torch.is_grad_enabled() and enc_trainable):
            x = self.encode(pixel_values, grid_thw)
        return self.merge(x)

    def hf_items(self, prefix="model.visual."):
        return [(prefix + n, p, None) for n, p in self.named_parameters()]


def _rotate(x, cos, sin):
    h = x.shape[-1] // 2
    return x * cos + torch.cat([-x[..., h:], x[..., :h]], -1) * sin


# ------------------------------------------------------------------------------------------------
# text side: interleaved 3-D RoPE
# ------------------------------------------------------------------------------------------------
def mrope_axis(half, section):
    """For each of the ``half`` rotary frequencies, which position axis (0 = t, 1 = h, 2 = w) it
    reads: frequencies are interleaved t, h, w, t, h, w, ... while each axis has frequencies left
    (``section`` = per-axis counts), the remainder on t."""
    ax = torch.zeros(half, dtype=torch.long)
    for a in (1, 2):
        for j in range(a, min(3 * section[a], half), 3):
            ax[j] = a
    return ax


def mrope_axis_chunked(half, section):
    """Chunked layout (GLM): the first ``section[0]`` frequencies read t, the next ``section[1]`` h,
    the rest w."""
    ax = torch.full((half,), 2, dtype=torch.long)
    ax[:section[0]] = 0
    ax[section[0]:section[0] + section[1]] = 1
    return ax


def mrope_angles(pos3, rotary_dim, theta, section, layout="interleaved"):
    """Rotary angles [B, T, rotary_dim / 2] for 3-D positions ``pos3`` [B, 3, T]; a token whose three
    positions agree gets exactly the 1-D RoPE angles."""
    half = rotary_dim // 2
    inv = 1.0 / (theta ** (torch.arange(0, rotary_dim, 2, dtype=torch.float32, device=pos3.device) / rotary_dim))
    ax = (mrope_axis_chunked if layout == "chunked" else mrope_axis)(half, section).to(pos3.device)
    p = pos3.float().permute(0, 2, 1)                                          # [B, T, 3]
    return torch.gather(p, 2, ax[None, None].expand(p.shape[0], p.shape[1], -1)) * inv
