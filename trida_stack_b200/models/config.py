"""Model configuration read from an HF ``config.json`` (Qwen3 dense / Qwen3.5 hybrid)."""
import json
import os
from dataclasses import dataclass, field


@dataclass
class ModelConfig:
    model_type: str = "qwen3"
    vocab_size: int = 151936
    hidden_size: int = 2560
    intermediate_size: int = 9728
    num_layers: int = 36
    n_heads: int = 32
    n_kv_heads: int = 8
    head_dim: int = 128
    eps: float = 1e-6
    rope_theta: float = 1e6
    partial_rotary_factor: float = 1.0
    tie_embeddings: bool = True
    max_position: int = 40960
    initializer_range: float = 0.02
    layer_types: list = field(default_factory=list)
    # gated-delta (linear attention) layers of the hybrid family
    lin_k_heads: int = 16
    lin_v_heads: int = 32
    lin_k_dim: int = 128
    lin_v_dim: int = 128
    conv_kernel: int = 4
    # full-attention layers of the hybrid family gate their output with sigmoid(q_proj gate half)
    attn_output_gate: bool = False
    # vision-language checkpoints: the ViT's config dict, the <|image_pad|> id and the interleaved
    # 3-D RoPE split (frequencies per t / h / w axis)
    vision: dict = None
    image_token_id: int = 248056
    mrope_section: tuple = (11, 11, 10)
    # 3-D RoPE frequency layout: "interleaved" t,h,w,t,h,w,... (Qwen3.5) or "chunked" t..t h..h w..w (GLM)
    mrope_layout: str = "interleaved"
    # GLM-style layers: no per-head q / k RMSNorm; RMSNorm on the attention and MLP outputs before
    # each residual add
    qk_norm: bool = True
    post_norms: bool = False
    # raw HF dict (written back on save so the checkpoint stays loadable by transformers)
    hf: dict = field(default_factory=dict, repr=False)

    def __post_init__(self):
        if not self.layer_types:
            self.layer_types = ["full_attention"] * self.num_layers

    @property
    def rotary_dim(self):
        return int(self.head_dim * self.partial_rotary_factor)

    @property
    def is_vl(self):
        return self.vision is not None

    @property
    def is_hybrid(self):
        return any(t == "linear_attention" for t in self.layer_types)

    @classmethod
    def from_hf_dict(cls, d):
        full = d
        if "text_config" in d and isinstance(d["text_config"], dict):
            d = d["text_config"]
        rp = d.get("rope_parameters") or {}
        theta = rp.get("rope_theta", d.get("rope_theta", 1e4))
        prf = rp.get("partial_rotary_factor", d.get("partial_rotary_factor", 1.0))
        mt = d.get("model_type", "qwen3")
        hybrid_family = mt.startswith("qwen3_5") or mt == "qwen3_next"
        n_layers = d["num_hidden_layers"]
        return cls(
            model_type=mt,
            vocab_size=d["vocab_size"],
            hidden_size=d["hidden_size"],
            intermediate_size=d["intermediate_size"],
            num_layers=n_layers,
            n_heads=d["num_attention_heads"],
            n_kv_heads=d.get("num_key_value_heads", d["num_attention_heads"]),
            head_dim=d.get("head_dim") or d["hidden_size"] // d["num_attention_heads"],
            eps=d.get("rms_norm_eps", 1e-6),
            rope_theta=float(theta),
            partial_rotary_factor=float(prf),
            tie_embeddings=bool(full.get("tie_word_embeddings", d.get("tie_word_embeddings", False))),
            max_position=d.get("max_position_embeddings", 32768),
            initializer_range=d.get("initializer_range", 0.02),
            layer_types=list(d.get("layer_types") or ["full_attention"] * n_layers),
            lin_k_heads=d.get("linear_num_key_heads", 16),
            lin_v_heads=d.get("linear_num_value_heads", 32),
            lin_k_dim=d.get("linear_key_head_dim", 128),
            lin_v_dim=d.get("linear_value_head_dim", 128),
            conv_kernel=d.get("linear_conv_kernel_dim", 4),
            attn_output_gate=hybrid_family,
            vision=dict(full["vision_config"]) if isinstance(full.get("vision_config"), dict) else None,
            image_token_id=int(full.get("image_token_id", 248056)),
            mrope_section=tuple(rp.get("mrope_section") or (11, 11, 10)),
            hf=dict(full),
        )

    @classmethod
    def from_pretrained(cls, path):
        with open(os.path.join(path, "config.json")) as f:
            return cls.from_hf_dict(json.load(f))

    def to_hf_dict(self):
        """HF config dict with the (possibly resized) vocab written back."""
        d = json.loads(json.dumps(self.hf)) if self.hf else {}
        if not d:
            d = {"model_type": self.model_type, "architectures": ["Qwen3ForCausalLM"],
                 "hidden_size": self.hidden_size, "intermediate_size": self.intermediate_size,
                 "num_hidden_layers": self.num_layers, "num_attention_heads": self.n_heads,
                 "num_key_value_heads": self.n_kv_heads, "head_dim": self.head_dim,
                 "rms_norm_eps": self.eps, "max_position_embeddings": self.max_position,
                 "rope_parameters": {"rope_theta": self.rope_theta, "rope_type": "default"},
                 "hidden_act": "silu", "initializer_range": self.initializer_range,
                 "attention_bias": False, "layer_types": self.layer_types}
        tgt = d["text_config"] if isinstance(d.get("text_config"), dict) else d
        tgt["vocab_size"] = self.vocab_size
        d["tie_word_embeddings"] = self.tie_embeddings
        return d


def qwen3_config(vocab_size=151936, hidden_size=2560, intermediate_size=9728, num_layers=36, n_heads=32,
                 n_kv_heads=8, head_dim=128, rope_theta=1e6, tie_embeddings=True, eps=1e-6):
    """A Qwen3 dense config (defaults = Qwen3-4B) with a matching HF dict."""
    c = ModelConfig(model_type="qwen3", vocab_size=vocab_size, hidden_size=hidden_size,
                    intermediate_size=intermediate_size, num_layers=num_layers, n_heads=n_heads,
                    n_kv_heads=n_kv_heads, head_dim=head_dim, rope_theta=rope_theta,
                    tie_embeddings=tie_embeddings, eps=eps)
    c.hf = c.to_hf_dict()
    return c
