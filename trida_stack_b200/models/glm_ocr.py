"""GLM-OCR (``GlmOcrForConditionalGeneration``): the model behind GravityOCR, natively.

GravityOCR is GLM-OCR (a CogViT-style image encoder and a 0.5B GLM text decoder) fine-tuned as a
block-diffusion model; the architecture is unchanged (``inference/gravityocr/MODEL_CONTRACT.md``).
This module holds its text decoder and image encoder with the checkpoint's weight names, loading
and saving, 3-D RoPE positions, and a plain-PyTorch full-sequence forward (the CPU statement the
serving runtime is checked against).  Serving runs on ``serve.runtime.Runtime`` like the Qwen
models: the decoder exposes the same layer attributes, plus GLM's output norms.

Text decoder (stated from the published architecture): per layer ``x += N2(o_proj(attn(N1(x))))``
and ``x += N4(down(silu(gate) * up)(N3(x)))`` with RMSNorms N1..N4 (no per-head q / k norm), GQA
attention, RoPE on the first ``partial_rotary_factor * head_dim`` channels with pairwise-interleaved
rotation and chunked 3-D frequency sections (t, h, w).  The q / k projection rows of the rotary
channels are stored permuted (pair (2i, 2i+1) -> (i, i + rd/2)) so the half-split RoPE kernels apply
unchanged: q.k is invariant under the same permutation of q and k.

Image encoder: patch embedding (Conv3d of stride = kernel as one GEMM), ``depth`` blocks of RMSNorm
-> attention (qkv with bias, per-head q / k RMSNorm, 2-D RoPE, bidirectional per frame) and RMSNorm
-> SwiGLU MLP (with bias), a final RMSNorm, a 2x2 stride-2 convolution merging each 2x2 patch block
(applied as one GEMM: patches arrive in merge-block order), then the merger: Linear -> LayerNorm ->
GELU -> SwiGLU to the text width.  It runs on PyTorch ops (cuBLAS GEMMs, SDPA), once per request.
"""
import json
import os
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..ops import blocks
from ..ops import reference as R
from .config import ModelConfig
from .vision import mrope_angles


def glm_ocr_config(d):
    """ModelConfig of the text decoder (with the vision config attached) from a GLM-OCR config dict."""
    t = d.get("text_config") or d
    rp = t.get("rope_parameters") or t.get("rope_scaling") or {}
    theta = rp.get("rope_theta", t.get("rope_theta", 10000.0))
    n = t["num_hidden_layers"]
    return ModelConfig(
        model_type="glm_ocr", vocab_size=t["vocab_size"], hidden_size=t["hidden_size"],
        intermediate_size=t["intermediate_size"], num_layers=n, n_heads=t["num_attention_heads"],
        n_kv_heads=t.get("num_key_value_heads") or t["num_attention_heads"],
        head_dim=t.get("head_dim") or t["hidden_size"] // t["num_attention_heads"], eps=t.get("rms_norm_eps", 1e-5),
        rope_theta=float(theta), partial_rotary_factor=float(rp.get("partial_rotary_factor",
                                                                    t.get("partial_rotary_factor", 0.5))),
        tie_embeddings=bool(d.get("tie_word_embeddings", False)),
        max_position=t.get("max_position_embeddings", 131072), layer_types=["full_attention"] * n,
        vision=dict(d["vision_config"]) if isinstance(d.get("vision_config"), dict) else None,
        image_token_id=int(d.get("image_token_id", 59280)),
        mrope_section=tuple(rp.get("mrope_section") or (8, 12, 12)), mrope_layout="chunked",
        qk_norm=False, post_norms=True, hf=dict(d))


def rope_perm(d, rd):
    """Row order turning pairwise-interleaved rotary channels into half-split ones (per head)."""
    idx = list(range(0, rd, 2)) + list(range(1, rd, 2)) + list(range(rd, d))
    return torch.tensor(idx)


def _rms(x, w, eps):
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype) * w


# ------------------------------------------------------------------------------------ text
class GlmLayer(nn.Module):
    layer_type = "full_attention"
    q_norm = k_norm = None

    def __init__(self, cfg, dtype):
        super().__init__()
        D, d, I = cfg.hidden_size, cfg.head_dim, cfg.intermediate_size
        self.input_norm = nn.Parameter(torch.ones(D, dtype=dtype))
        self.wqkv = nn.Parameter(torch.empty((cfg.n_heads + 2 * cfg.n_kv_heads) * d, D, dtype=dtype))
        self.wo = nn.Parameter(torch.empty(D, cfg.n_heads * d, dtype=dtype))
        self.post_attn_norm = nn.Parameter(torch.ones(D, dtype=dtype))
        self.post_norm = nn.Parameter(torch.ones(D, dtype=dtype))
        self.wgu = nn.Parameter(torch.empty(2 * I, D, dtype=dtype))
        self.wdown = nn.Parameter(torch.empty(D, I, dtype=dtype))
        self.post_mlp_norm = nn.Parameter(torch.ones(D, dtype=dtype))

    def hf_items(self, prefix, cfg):
        """(name, parameter, rows, heads whose rotary rows are permuted, or None)."""
        d, Hq, Hkv = cfg.head_dim, cfg.n_heads, cfg.n_kv_heads
        qn, kn = Hq * d, Hkv * d
        return [(prefix + "input_layernorm.weight", self.input_norm, None, None),
                (prefix + "self_attn.q_proj.weight", self.wqkv, (0, qn), Hq),
                (prefix + "self_attn.k_proj.weight", self.wqkv, (qn, qn + kn), Hkv),
                (prefix + "self_attn.v_proj.weight", self.wqkv, (qn + kn, qn + 2 * kn), None),
                (prefix + "self_attn.o_proj.weight", self.wo, None, None),
                (prefix + "post_self_attn_layernorm.weight", self.post_attn_norm, None, None),
                (prefix + "post_attention_layernorm.weight", self.post_norm, None, None),
                (prefix + "mlp.gate_up_proj.weight", self.wgu, None, None),
                (prefix + "mlp.down_proj.weight", self.wdown, None, None),
                (prefix + "post_mlp_layernorm.weight", self.post_mlp_norm, None, None)]


# ------------------------------------------------------------------------------------ vision
@dataclass
class GlmVisionConfig:
    depth: int = 24
    hidden_size: int = 1024
    intermediate_size: int = 4096
    num_heads: int = 16
    in_channels: int = 3
    patch_size: int = 14
    temporal_patch_size: int = 2
    spatial_merge_size: int = 2
    out_hidden_size: int = 1536
    rms_norm_eps: float = 1e-5
    attention_bias: bool = True
    hidden_act: str = "silu"

    @classmethod
    def from_dict(cls, d):
        return cls(**{k: d[k] for k in cls.__dataclass_fields__ if k in d})


def _weight(n):
    m = nn.Module()
    m.weight = nn.Parameter(torch.ones(n))
    return m


class _VAttn(nn.Module):
    def __init__(self, c):
        super().__init__()
        hd = c.hidden_size // c.num_heads
        self.qkv = nn.Linear(c.hidden_size, 3 * c.hidden_size, bias=c.attention_bias)
        self.proj = nn.Linear(c.hidden_size, c.hidden_size, bias=c.attention_bias)
        self.q_norm, self.k_norm = _weight(hd), _weight(hd)


class _VMlp(nn.Module):
    def __init__(self, c):
        super().__init__()
        b = c.attention_bias
        self.gate_proj = nn.Linear(c.hidden_size, c.intermediate_size, bias=b)
        self.up_proj = nn.Linear(c.hidden_size, c.intermediate_size, bias=b)
        self.down_proj = nn.Linear(c.intermediate_size, c.hidden_size, bias=b)


class _VBlock(nn.Module):
    def __init__(self, c):
        super().__init__()
        self.norm1, self.norm2 = _weight(c.hidden_size), _weight(c.hidden_size)
        self.attn, self.mlp = _VAttn(c), _VMlp(c)


class GlmVision(nn.Module):
    """``forward(pixel_values [P, C*T*p*p], grid_thw [N, 3]) -> [P / merge^2, text hidden]``."""

    def __init__(self, c: GlmVisionConfig, dtype=torch.bfloat16, device=None):
        super().__init__()
        self.c = c
        D, O, m = c.hidden_size, c.out_hidden_size, c.spatial_merge_size
        with torch.device(device or "cpu"):
            self.patch_embed = nn.Module()
            self.patch_embed.proj = nn.Module()
            self.patch_embed.proj.weight = nn.Parameter(
                torch.empty(D, c.in_channels, c.temporal_patch_size, c.patch_size, c.patch_size))
            self.patch_embed.proj.bias = nn.Parameter(torch.zeros(D))
            self.blocks = nn.ModuleList([_VBlock(c) for _ in range(c.depth)])
            self.post_layernorm = _weight(D)
            self.downsample = nn.Module()
            self.downsample.weight = nn.Parameter(torch.empty(O, D, m, m))
            self.downsample.bias = nn.Parameter(torch.zeros(O))
            self.merger = nn.Module()
            self.merger.proj = nn.Linear(O, O, bias=False)
            self.merger.post_projection_norm = nn.LayerNorm(O)
            self.merger.gate_proj = nn.Linear(O, O * c.in_channels, bias=False)
            self.merger.up_proj = nn.Linear(O, O * c.in_channels, bias=False)
            self.merger.down_proj = nn.Linear(O * c.in_channels, O, bias=False)
        with torch.no_grad():
            for n, p in self.named_parameters():
                if n.endswith("bias"):
                    p.zero_()
                elif p.dim() >= 2:
                    p.normal_(0.0, 0.02)
        self.to(dtype)

    def _block_order(self, t, h, w):
        m = self.c.spatial_merge_size
        r = torch.arange(h).view(h // m, 1, m, 1).expand(h // m, w // m, m, m)
        c = torch.arange(w).view(1, w // m, 1, m).expand(h // m, w // m, m, m)
        return torch.stack([r.reshape(-1), c.reshape(-1)], -1).repeat(t, 1)

    def forward(self, pixel_values, grid_thw):
        c = self.c
        grids = [tuple(int(v) for v in g) for g in grid_thw.tolist()]
        dt = self.patch_embed.proj.weight.dtype
        D, H = c.hidden_size, c.num_heads
        hd = D // H
        x = F.linear(pixel_values.to(dt).reshape(len(pixel_values), -1),
                     self.patch_embed.proj.weight.reshape(D, -1), self.patch_embed.proj.bias)
        dim = hd // 2
        inv = 1.0 / (10000.0 ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))
        rc = torch.cat([self._block_order(*g) for g in grids]).float()
        ang = torch.cat([rc[:, :1] * inv, rc[:, 1:] * inv], -1).to(x.device)
        cos = torch.cat([ang, ang], -1).cos()[:, None]
        sin = torch.cat([ang, ang], -1).sin()[:, None]
        lens = [h * w for t, h, w in grids for _ in range(t)]
        eps = c.rms_norm_eps
        for b in self.blocks:
            y = _rms(x, b.norm1.weight, eps)
            q, k, v = b.attn.qkv(y).view(-1, 3, H, hd).unbind(1)
            q = _rms(q, b.attn.q_norm.weight, eps)
            k = _rms(k, b.attn.k_norm.weight, eps)
            q = _rotate(q.float(), cos, sin).to(dt)
            k = _rotate(k.float(), cos, sin).to(dt)
            outs, o0 = [], 0
            for n in lens:                                                     # bidirectional per frame
                sl = slice(o0, o0 + n)
                outs.append(F.scaled_dot_product_attention(q[sl].transpose(0, 1), k[sl].transpose(0, 1),
                                                           v[sl].transpose(0, 1)).transpose(0, 1))
                o0 += n
            x = x + b.attn.proj(torch.cat(outs).reshape(-1, D))
            h = _rms(x, b.norm2.weight, eps)
            x = x + b.mlp.down_proj(F.silu(b.mlp.gate_proj(h)) * b.mlp.up_proj(h))
        x = _rms(x, self.post_layernorm.weight, eps)
        m = c.spatial_merge_size
        x = x.view(-1, m, m, D).permute(0, 3, 1, 2).reshape(-1, D * m * m)
        x = F.linear(x, self.downsample.weight.reshape(c.out_hidden_size, -1), self.downsample.bias)
        mg = self.merger
        x = F.gelu(mg.post_projection_norm(mg.proj(x)))
        return mg.down_proj(F.silu(mg.gate_proj(x)) * mg.up_proj(x))


def _rotate(x, cos, sin):
    h = x.shape[-1] // 2
    return x * cos + torch.cat([-x[..., h:], x[..., :h]], -1) * sin


# ------------------------------------------------------------------------------------ model
class GlmOcrDecoder(nn.Module):
    """Text decoder + image encoder with the attribute interface of ``models.decoder.Decoder``."""

    def __init__(self, cfg: ModelConfig, dtype=torch.bfloat16, device=None):
        super().__init__()
        self.cfg = cfg
        D, V = cfg.hidden_size, cfg.vocab_size
        with torch.device(device or "cpu"):
            self.embed = nn.Parameter(torch.empty(V, D, dtype=dtype))
            self.layers = nn.ModuleList([GlmLayer(cfg, dtype) for _ in range(cfg.num_layers)])
            self.norm = nn.Parameter(torch.ones(D, dtype=dtype))
            self.lm_head = None if cfg.tie_embeddings else nn.Parameter(torch.empty(V, D, dtype=dtype))
        with torch.no_grad():
            for p in self.parameters():
                if p.dim() >= 2:
                    p.normal_(0.0, cfg.initializer_range)
        self.visual = None
        if cfg.vision is not None:
            self.visual = GlmVision(GlmVisionConfig.from_dict(cfg.vision), dtype=dtype, device=device)
            self.visual.requires_grad_(False)

    @property
    def lm_weight(self):
        return self.embed if self.lm_head is None else self.lm_head

    def embed_tokens(self, ids):
        return blocks.embedding(ids, self.embed)

    # ---------------------------------------------------------------- checkpoint names
    def hf_items(self):
        base = "model.language_model."
        items = [(base + "embed_tokens.weight", self.embed, None, None)]
        for i, layer in enumerate(self.layers):
            items += layer.hf_items(f"{base}layers.{i}.", self.cfg)
        items.append((base + "norm.weight", self.norm, None, None))
        if self.lm_head is not None:
            items.append(("lm_head.weight", self.lm_head, None, None))
        if self.visual is not None:
            items += [("model.visual." + n, p, None, None) for n, p in self.visual.named_parameters()]
        return items

    def _perm(self, heads):
        d = self.cfg.head_dim
        p = rope_perm(d, self.cfg.rotary_dim)
        return torch.cat([p + h * d for h in range(heads)])

    @torch.no_grad()
    def load_hf_state_dict(self, sd, strict=True):
        missing = []
        for name, p, rows, heads in self.hf_items():
            src = sd.get(name)
            if src is None:
                missing.append(name)
                continue
            dst = p if rows is None else p[rows[0]:rows[1]]
            if heads is not None:
                src = src[self._perm(heads)]
            if tuple(src.shape) != tuple(dst.shape):
                raise ValueError(f"{name}: checkpoint shape {tuple(src.shape)} != model {tuple(dst.shape)}")
            dst.copy_(src.to(dst.dtype))
        if strict and missing:
            raise KeyError(f"missing weights: {missing[:8]}{'...' if len(missing) > 8 else ''}")
        return missing

    @torch.no_grad()
    def hf_state_dict(self, dtype=None):
        out = {}
        for name, p, rows, heads in self.hf_items():
            t = p if rows is None else p[rows[0]:rows[1]]
            if heads is not None:
                t = t[torch.argsort(self._perm(heads))]
            out[name] = t.to(dtype or p.dtype).detach().contiguous()
        return out

    # ---------------------------------------------------------------- plain-PyTorch statement
    def rope_angles(self, pos3):
        c = self.cfg
        return mrope_angles(pos3, c.rotary_dim, c.rope_theta, c.mrope_section, layout="chunked")

    @torch.no_grad()
    def forward_ref(self, input_ids, pos3, image_feats=None):
        """Causal logits [T, V] of one sequence ``input_ids`` [T] with 3-D positions ``pos3`` [3, T]
        (image features, if any, replace the image tokens' embeddings in order)."""
        c = self.cfg
        T = input_ids.shape[0]
        x = self.embed[input_ids].float()
        if image_feats is not None:
            x[input_ids == c.image_token_id] = image_feats.float()
        ang = self.rope_angles(pos3[None])[0]                                   # [T, rd/2]
        cos, sin = torch.cat([ang, ang], -1).cos(), torch.cat([ang, ang], -1).sin()
        Hq, Hkv, d = c.n_heads, c.n_kv_heads, c.head_dim
        mask = torch.ones(T, T, dtype=torch.bool).tril()
        for L in self.layers:
            h = _rms(x, L.input_norm.float(), c.eps)
            qkv = h @ L.wqkv.float().t()
            q = R.apply_rope(qkv[:, :Hq * d].view(T, Hq, d), cos, sin)
            k = R.apply_rope(qkv[:, Hq * d:(Hq + Hkv) * d].view(T, Hkv, d), cos, sin)
            v = qkv[:, (Hq + Hkv) * d:].view(T, Hkv, d)
            G = Hq // Hkv
            sc = torch.einsum("thd,khd->htk", q, k.repeat_interleave(G, 1)) / d ** 0.5
            p = sc.masked_fill(~mask, float("-inf")).softmax(-1)
            o = torch.einsum("htk,khd->thd", p, v.repeat_interleave(G, 1)).reshape(T, Hq * d)
            x = x + _rms(o @ L.wo.float().t(), L.post_attn_norm.float(), c.eps)
            h = _rms(x, L.post_norm.float(), c.eps)
            g, u = (h @ L.wgu.float().t()).chunk(2, -1)
            x = x + _rms((F.silu(g) * u) @ L.wdown.float().t(), L.post_mlp_norm.float(), c.eps)
        return _rms(x, self.norm.float(), c.eps) @ self.lm_weight.float().t()


def load_glm_ocr(path, device, dtype=torch.bfloat16):
    """(decoder, ``block_diffusion.json`` dict) of a GLM-OCR / GravityOCR checkpoint directory."""
    from ..checkpoint import read_hf_weights
    with open(os.path.join(path, "config.json")) as f:
        cfg = glm_ocr_config(json.load(f))
    dec = GlmOcrDecoder(cfg, dtype=dtype, device=device)
    dec.load_hf_state_dict(read_hf_weights(path))
    side = os.path.join(path, "block_diffusion.json")
    bd = json.load(open(side)) if os.path.exists(side) else {}
    return dec, bd


def is_glm_ocr_dir(path):
    try:
        with open(os.path.join(path, "config.json")) as f:
            return json.load(f).get("model_type") == "glm_ocr"
    except OSError:
        return False
