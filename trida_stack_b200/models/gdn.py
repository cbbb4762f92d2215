"""Gated-delta (linear-attention) decoder layer of the Qwen3.5 hybrid family.

Math (HF ``Qwen3_5GatedDeltaNet``): ``[qkv | z | b | a] = rmsnorm(x) W_in^T`` (one fused GEMM),
depthwise width-K causal conv + SiLU over qkv, q/k L2-normalised per head (q scaled by dk^-0.5),
``beta = sigmoid(b)``, ``g = -exp(A_log) softplus(a + dt_bias)``, key heads shared by
``Hv / Hk`` value heads, gated-delta recurrence, gated RMSNorm ``norm(o) * w * silu(z)``, output
projection, residual add; then the SwiGLU MLP sub-block.

The layer runs in one of two layouts carried by ``actx.linear``: ``causal`` (one causal stream per
row, recurrence and conv restarting at document starts) or ``two_stream`` (a
``[x0 ; xt_1 .. xt_V]`` row, see ``ops.gdn_reference``).
"""
import torch
import torch.nn as nn

from ..ops import blocks
from ..ops import gdn as gdn_ops
from .config import ModelConfig


class GatedDeltaLayer(nn.Module):
    def __init__(self, cfg: ModelConfig, dtype):
        super().__init__()
        D = cfg.hidden_size
        kd, vd, hv = cfg.lin_k_heads * cfg.lin_k_dim, cfg.lin_v_heads * cfg.lin_v_dim, cfg.lin_v_heads
        self.dims = (kd, vd, hv)
        self.input_norm = nn.Parameter(torch.ones(D, dtype=dtype))
        self.w_in = nn.Parameter(torch.empty(2 * kd + vd + vd + 2 * hv, D, dtype=dtype))
        self.conv_w = nn.Parameter(torch.empty(2 * kd + vd, cfg.conv_kernel, dtype=dtype))
        self.dt_bias = nn.Parameter(torch.ones(hv, dtype=dtype))
        self.A_log = nn.Parameter(torch.zeros(hv, dtype=dtype))
        self.gnorm = nn.Parameter(torch.ones(cfg.lin_v_dim, dtype=dtype))
        self.w_out = nn.Parameter(torch.empty(D, vd, dtype=dtype))
        self.post_norm = nn.Parameter(torch.ones(D, dtype=dtype))
        self.wgu = nn.Parameter(torch.empty(2 * cfg.intermediate_size, D, dtype=dtype))
        self.wdown = nn.Parameter(torch.empty(D, cfg.intermediate_size, dtype=dtype))
        self.layer_type = "linear_attention"

    def forward(self, x, actx, cfg):
        x = gdn_ops.gdn_block(x, self, actx, cfg)
        return blocks.mlp_block(x, self.post_norm, self.wgu, self.wdown, cfg.eps)

    def hf_items(self, prefix, cfg):
        kd, vd, hv = self.dims
        la = prefix + "linear_attn."
        o = 0
        items = [(prefix + "input_layernorm.weight", self.input_norm, None)]
        for name, n in (("in_proj_qkv", 2 * kd + vd), ("in_proj_z", vd), ("in_proj_b", hv), ("in_proj_a", hv)):
            items.append((la + name + ".weight", self.w_in, (o, o + n)))
            o += n
        F = cfg.intermediate_size
        items += [
            (la + "conv1d.weight", self.conv_w, "conv"),
            (la + "dt_bias", self.dt_bias, None),
            (la + "A_log", self.A_log, None),
            (la + "norm.weight", self.gnorm, None),
            (la + "out_proj.weight", self.w_out, None),
            (prefix + "post_attention_layernorm.weight", self.post_norm, None),
            (prefix + "mlp.gate_proj.weight", self.wgu, (0, F)),
            (prefix + "mlp.up_proj.weight", self.wgu, (F, 2 * F)),
            (prefix + "mlp.down_proj.weight", self.wdown, None),
        ]
        return items
