"""Native Qwen3 / Qwen3.5 decoder (no HF modules).

Weights are stored fused for the tensor-core GEMMs -- ``wqkv = [q; k; v]`` and ``wgu = [gate; up]``
-- and mapped to the HF safetensors names on load/save (``hf_state_dict`` /
``load_hf_state_dict``), so checkpoints stay interchangeable with transformers.  The decoder math
is HF's Qwen3 math (pre-norm residual blocks, per-head q/k RMSNorm, half-split RoPE, SwiGLU).
"""
import torch
import torch.nn as nn

from ..ops import blocks
from .config import ModelConfig


class AttentionLayer(nn.Module):
    """Pre-norm attention sub-block + SwiGLU MLP sub-block (one HF decoder layer)."""

    def __init__(self, cfg: ModelConfig, dtype):
        super().__init__()
        D, d = cfg.hidden_size, cfg.head_dim
        q_out = cfg.n_heads * d * (2 if cfg.attn_output_gate else 1)
        self.input_norm = nn.Parameter(torch.ones(D, dtype=dtype))
        self.wqkv = nn.Parameter(torch.empty(q_out + 2 * cfg.n_kv_heads * d, D, dtype=dtype))
        self.q_norm = nn.Parameter(torch.ones(d, dtype=dtype))
        self.k_norm = nn.Parameter(torch.ones(d, dtype=dtype))
        self.wo = nn.Parameter(torch.empty(D, cfg.n_heads * d, dtype=dtype))
        self.post_norm = nn.Parameter(torch.ones(D, dtype=dtype))
        self.wgu = nn.Parameter(torch.empty(2 * cfg.intermediate_size, D, dtype=dtype))
        self.wdown = nn.Parameter(torch.empty(D, cfg.intermediate_size, dtype=dtype))
        self.layer_type = "full_attention"

    def forward(self, x, actx, cfg):
        x = blocks.attn_block(x, self.input_norm, self.wqkv, self.q_norm, self.k_norm, self.wo, actx, cfg)
        return blocks.mlp_block(x, self.post_norm, self.wgu, self.wdown, cfg.eps)

    # q_proj rows of the gated (Qwen3.5) attention are per head [query (d) ; gate (d)]

    # HF <-> fused names
    def hf_items(self, prefix, cfg):
        d, Hq, Hkv, F = cfg.head_dim, cfg.n_heads, cfg.n_kv_heads, cfg.intermediate_size
        qn = Hq * d * (2 if cfg.attn_output_gate else 1)
        kn = Hkv * d
        return [
            (prefix + "input_layernorm.weight", self.input_norm, None),
            (prefix + "self_attn.q_proj.weight", self.wqkv, (0, qn)),
            (prefix + "self_attn.k_proj.weight", self.wqkv, (qn, qn + kn)),
            (prefix + "self_attn.v_proj.weight", self.wqkv, (qn + kn, qn + 2 * kn)),
            (prefix + "self_attn.q_norm.weight", self.q_norm, None),
            (prefix + "self_attn.k_norm.weight", self.k_norm, None),
            (prefix + "self_attn.o_proj.weight", self.wo, None),
            (prefix + "post_attention_layernorm.weight", self.post_norm, None),
            (prefix + "mlp.gate_proj.weight", self.wgu, (0, F)),
            (prefix + "mlp.up_proj.weight", self.wgu, (F, 2 * F)),
            (prefix + "mlp.down_proj.weight", self.wdown, None),
        ]


class Decoder(nn.Module):
    """Token embedding -> decoder layers -> final RMSNorm; LM head tied or separate."""

    def __init__(self, cfg: ModelConfig, dtype=torch.bfloat16, device=None):
        super().__init__()
        self.cfg = cfg
        D = cfg.hidden_size
        with torch.device(device or "cpu"):
            self.embed = nn.Parameter(torch.empty(cfg.vocab_size, D, dtype=dtype))
            layers = []
            for t in cfg.layer_types:
                if t == "linear_attention":
                    from .gdn import GatedDeltaLayer
                    layers.append(GatedDeltaLayer(cfg, dtype))
                else:
                    layers.append(AttentionLayer(cfg, dtype))
            self.layers = nn.ModuleList(layers)
            self.norm = nn.Parameter(torch.ones(D, dtype=dtype))
            self.lm_head = None if cfg.tie_embeddings else nn.Parameter(torch.empty(cfg.vocab_size, D, dtype=dtype))
        self.reset_parameters()
        self.visual = None
        if cfg.is_vl:                          # vision-language checkpoint: ViT + merger, encoder frozen
            from .vision import VisionConfig, VisionTower
            self.visual = VisionTower(VisionConfig.from_dict(cfg.vision), dtype=dtype, device=device)
            self.visual.freeze_encoder()

    @property
    def lm_weight(self):
        return self.embed if self.lm_head is None else self.lm_head

    @torch.no_grad()
    def reset_parameters(self, generator=None):
        """HF ``_init_weights``: N(0, initializer_range) for matrices, ones for norms."""
        std = self.cfg.initializer_range
        for name, p in self.named_parameters():
            if name.startswith("visual."):
                continue
            if p.dim() >= 2:
                p.normal_(0.0, std, generator=generator)
            elif name.endswith("A_log"):
                p.copy_(torch.log(torch.empty_like(p, dtype=torch.float32).uniform_(0, 16, generator=generator)))
            elif name.endswith("dt_bias"):
                p.fill_(1.0)
            elif name.endswith("conv_w"):
                p.normal_(0.0, std, generator=generator)
            else:
                p.fill_(1.0)

    def resize_vocab(self, new_size):
        """Grow/shrink the vocabulary rows (HF ``resize_token_embeddings``): kept rows unchanged,
        new rows initialised N(0, initializer_range)."""
        old = self.cfg.vocab_size
        if new_size == old:
            return
        with torch.no_grad():
            for attr in ("embed", "lm_head"):
                p = getattr(self, attr)
                if p is None:
                    continue
                n = torch.empty(new_size, p.shape[1], dtype=p.dtype, device=p.device)
                k = min(old, new_size)
                n[:k] = p[:k]
                if new_size > old:
                    n[old:].normal_(0.0, self.cfg.initializer_range)
                setattr(self, attr, nn.Parameter(n))
        self.cfg.vocab_size = new_size

    def embed_tokens(self, ids):
        return blocks.embedding(ids, self.embed)

    def forward(self, x, actx, layer_hook=None):
        """x: embedded tokens [B*T, D] -> final-normed hidden states [B*T, D]."""
        for i, layer in enumerate(self.layers):
            x = layer_hook(i, layer, x) if layer_hook is not None else layer(x, actx, self.cfg)
        return blocks.rmsnorm(x, self.norm, self.cfg.eps)

    # ---------------------------------------------------------------- HF state dict mapping
    @property
    def text_prefix(self):
        """Language-model weight prefix: ``model.language_model.`` in vision-language checkpoints."""
        return "model.language_model." if self.cfg.is_vl else "model."

    def hf_items(self):
        base = self.text_prefix
        items = [(base + "embed_tokens.weight", self.embed, None)]
        for i, layer in enumerate(self.layers):
            items += layer.hf_items(f"{base}layers.{i}.", self.cfg)
        items.append((base + "norm.weight", self.norm, None))
        if self.lm_head is not None:
            items.append(("lm_head.weight", self.lm_head, None))
        if self.visual is not None:
            items += self.visual.hf_items("model.visual.")
        return items

    _CENTERED = ("input_layernorm.weight", "post_attention_layernorm.weight", "self_attn.q_norm.weight",
                 "self_attn.k_norm.weight")

    def _norm_offset(self, name):
        """Qwen3.5 stores RMSNorm weights zero-centred (applied as 1 + w); the native layers keep the
        effective weight, so 1 is added on load and removed on save."""
        if not self.cfg.model_type.startswith("qwen3_5"):
            return 0.0
        if name.startswith("model.visual."):
            return 0.0
        return 1.0 if (name.endswith(self._CENTERED) or name == self.text_prefix + "norm.weight") else 0.0

    @staticmethod
    def _view(p, sl):
        if sl is None:
            return p
        if sl == "conv":          # HF depthwise conv1d weight [C, 1, K] <-> native [C, K]
            return p.unsqueeze(1)
        return p[sl[0]:sl[1]]

    @torch.no_grad()
    def hf_state_dict(self, dtype=None):
        out = {}
        for name, p, sl in self.hf_items():
            t = self._view(p, sl).float() - self._norm_offset(name)
            out[name] = t.to(dtype or p.dtype).detach().contiguous()
        return out

    @torch.no_grad()
    def load_hf_state_dict(self, sd, strict=True):
        missing = []
        for name, p, sl in self.hf_items():
            src = sd.get(name)
            if src is None:                    # text-only <-> vision-language naming of the same weights
                for a, b in (("model.language_model.", "model."), ("model.", "model.language_model.")):
                    if name.startswith(a) and (b + name[len(a):]) in sd:
                        src = sd[b + name[len(a):]]
                        break
            if src is None:
                missing.append(name)
                continue
            dst = self._view(p, sl)
            if tuple(src.shape) != tuple(dst.shape):
                raise ValueError(f"{name}: checkpoint shape {tuple(src.shape)} != model {tuple(dst.shape)}")
            dst.copy_((src.float() + self._norm_offset(name)).to(dst.dtype))
        if strict and missing:
            raise KeyError(f"missing weights: {missing[:8]}{'...' if len(missing) > 8 else ''}")
        return missing
