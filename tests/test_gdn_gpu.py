"""Gated-delta sub-block on the sm_100a kernels vs the fp32 PyTorch statement (ops.gdn_reference)."""
import copy
from types import SimpleNamespace

import pytest
import torch

from trida_stack_b200.models.config import ModelConfig
from trida_stack_b200.models.gdn import GatedDeltaLayer
from trida_stack_b200.ops.gdn import LinearLayout, gdn_block_reference

pytestmark = pytest.mark.gpu


def _cfg():
    return ModelConfig.from_hf_dict({
        "model_type": "qwen3_5_text", "vocab_size": 256, "hidden_size": 256, "intermediate_size": 512,
        "num_hidden_layers": 1, "num_attention_heads": 2, "num_key_value_heads": 1, "head_dim": 128,
        "linear_num_key_heads": 2, "linear_num_value_heads": 4, "linear_key_head_dim": 128,
        "linear_value_head_dim": 128, "linear_conv_kernel_dim": 4, "layer_types": ["linear_attention"],
        "rms_norm_eps": 1e-6})


def _layer(cfg, seed=0):
    g = torch.Generator().manual_seed(seed)
    lay = GatedDeltaLayer(cfg, torch.float32)
    with torch.no_grad():
        for n, p in lay.named_parameters():
            if n == "A_log":
                p.copy_(torch.log(torch.empty(p.shape).uniform_(0.5, 8, generator=g)))
            elif n == "dt_bias":
                p.copy_(torch.randn(p.shape, generator=g) * 0.5)
            elif p.dim() == 1:
                p.copy_(1 + 0.1 * torch.randn(p.shape, generator=g))
            else:
                p.copy_(torch.randn(p.shape, generator=g) * 0.05)
    return lay.to(torch.bfloat16).float()        # bf16-representable values on both sides


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


def _run(cfg, lay_cpu, layout, B, T, seed=1):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(B * T, cfg.hidden_size, generator=g)).to(torch.bfloat16).float()
    dy = torch.randn(B * T, cfg.hidden_size, generator=g) * 0.1
    # CPU fp32 oracle
    xr = x.clone().requires_grad_(True)
    actx = SimpleNamespace(B=B, T=T, linear=layout)
    out_r = gdn_block_reference(xr, lay_cpu, actx, cfg)
    out_r.backward(dy)
    # CUDA kernels (bf16 storage, fp32 math)
    lay_g = copy.deepcopy(lay_cpu).to("cuda", torch.bfloat16)
    lg = copy.copy(layout)
    if layout.doc_start is not None:
        lg.doc_start = layout.doc_start.cuda()
    xg = x.cuda().to(torch.bfloat16).requires_grad_(True)
    actx_g = SimpleNamespace(B=B, T=T, linear=lg)
    from trida_stack_b200.ops.gdn_cuda import gdn_block_cuda
    out_g = gdn_block_cuda(xg, lay_g, actx_g, cfg)
    out_g.backward(dy.cuda().to(torch.bfloat16))
    torch.cuda.synchronize()
    assert _rel(out_g.cpu() - x, out_r.detach() - x) < 5e-2     # bf16 rounding of out (|x| ~ 1)
    assert _rel(xg.grad.cpu(), xr.grad) < 3e-2
    for (n, p), (_, q) in zip(lay_cpu.named_parameters(), lay_g.named_parameters()):
        if p.grad is None:
            continue
        assert q.grad is not None, n
        assert _rel(q.grad.cpu(), p.grad) < 4e-2, (n, _rel(q.grad.cpu(), p.grad))


@pytest.fixture(params=["chunk", "scan"])
def path(request, monkeypatch):
    """Both gated-delta implementations: the chunked tcgen05 kernels and the per-token scan."""
    monkeypatch.setenv("TRIDA_GDN", request.param)
    return request.param


@pytest.mark.parametrize("docs", [False, True])
def test_gdn_causal_matches_reference(docs, path):
    cfg = _cfg()
    lay = _layer(cfg)
    B, T = 2, 100
    doc = None
    if docs:
        doc = torch.zeros(B, T, dtype=torch.bool)
        doc[:, 0] = True
        doc[0, 37] = True
        doc[1, 64] = True
    _run(cfg, lay, LinearLayout("causal", doc_start=doc), B, T)


@pytest.mark.parametrize("causal_clean,causal_noisy,docs", [(True, False, False), (False, False, False),
                                                            (True, True, False), (True, False, True)])
def test_gdn_two_stream_matches_reference(causal_clean, causal_noisy, docs, path):
    cfg = _cfg()
    lay = _layer(cfg)
    B, L, V, bd = 2, 64, 2, 16
    doc = None
    if docs:
        doc = torch.zeros(B, L, dtype=torch.bool)
        doc[:, 0] = True
        doc[0, 32] = True
        doc[1, 16] = True
    layout = LinearLayout("two_stream", L=L, V=V, bd=bd, causal_clean=causal_clean, causal_noisy=causal_noisy,
                          doc_start=doc)
    _run(cfg, lay, layout, B, (1 + V) * L)


@pytest.mark.parametrize("T,docs", [(300, False), (300, True)])
def test_gdn_chunk_causal_multi_tile(T, docs):
    """Rows over several 128-row tiles (and a partial last chunk) on the chunk kernels."""
    cfg = _cfg()
    lay = _layer(cfg, seed=2)
    B = 2
    doc = None
    if docs:
        doc = torch.zeros(B, T, dtype=torch.bool)
        doc[:, 0] = True
        doc[0, 150] = doc[1, 64] = doc[1, 201] = True
    _run(cfg, lay, LinearLayout("causal", doc_start=doc), B, T, seed=3)


@pytest.mark.parametrize("bd,L,causal_noisy", [(32, 128, False), (32, 256, True), (64, 192, False)])
def test_gdn_chunk_two_stream_blocks(bd, L, causal_noisy):
    """Two-stream rows with diffusion blocks of 32 and 64 tokens on the chunk kernels."""
    cfg = _cfg()
    lay = _layer(cfg, seed=4)
    B, V = 1, 2
    doc = torch.zeros(B, L, dtype=torch.bool)
    doc[:, 0] = True
    doc[0, L // 2] = True
    layout = LinearLayout("two_stream", L=L, V=V, bd=bd, causal_clean=True, causal_noisy=causal_noisy,
                          doc_start=doc)
    _run(cfg, lay, layout, B, (1 + V) * L, seed=5)
