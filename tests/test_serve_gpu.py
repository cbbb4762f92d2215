"""Serving runtime on the CUDA kernels vs the CPU statement of the same step."""
import copy

import pytest
import torch

from trida_stack_b200.models import Decoder, ModelConfig, qwen3_config
from trida_stack_b200.serve import Engine, Runtime

pytestmark = pytest.mark.gpu


def _hybrid(head_dim):
    cfg = ModelConfig.from_hf_dict({
        "model_type": "qwen3_5_text", "vocab_size": 512, "hidden_size": 256, "intermediate_size": 512,
        "num_hidden_layers": 4, "num_attention_heads": 4, "num_key_value_heads": 2, "head_dim": head_dim,
        "linear_num_key_heads": 2, "linear_num_value_heads": 4, "linear_key_head_dim": 128,
        "linear_value_head_dim": 128, "linear_conv_kernel_dim": 4, "partial_rotary_factor": 0.25,
        "layer_types": ["linear_attention"] * 3 + ["full_attention"], "tie_word_embeddings": True})
    return cfg


def _dense():
    return qwen3_config(vocab_size=512, hidden_size=256, intermediate_size=512, num_layers=2, n_heads=4,
                        n_kv_heads=2, head_dim=128)


def _init(cfg, seed=0):
    torch.manual_seed(seed)
    dec = Decoder(cfg, dtype=torch.float32)
    with torch.no_grad():
        for n, p in dec.named_parameters():
            if p.dim() >= 2:
                p.normal_(0, 0.06)
            elif n.endswith("A_log"):
                p.copy_(torch.log(torch.empty_like(p).uniform_(0.5, 4)))
            else:
                p.copy_(1 + 0.1 * torch.randn_like(p))
    return dec.to(torch.bfloat16).float()


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


@pytest.mark.parametrize("cfg", [_hybrid(256), _hybrid(128), _dense()], ids=["hybrid-d256", "hybrid-d128", "dense"])
def test_cuda_runtime_matches_cpu(cfg):
    dec = _init(cfg)
    dec_g = copy.deepcopy(dec).to("cuda", torch.bfloat16)
    torch.manual_seed(1)
    ids = torch.randint(0, 500, (3, 90))
    out = {}
    for name, d in (("cpu", dec), ("gpu", dec_g)):
        rt = Runtime(d, max_slots=4, max_len=256)
        slots = [rt.alloc() for _ in range(3)]
        last = rt.prefill(slots, ids[:, :70].tolist())
        lg = rt.canvas(slots, ids[:, 70:77], 4)          # self-spec shaped canvas (N = 4)
        rt.commit(slots, [1, 3, 4])
        lg2 = rt.canvas(slots, ids[:, 77:84], 4)
        rt.commit(slots, [4, 4, 4])
        out[name] = [t.float().cpu() for t in (last, lg, lg2)]
    for a, b in zip(out["gpu"], out["cpu"]):
        assert _rel(a, b) < 3e-2, _rel(a, b)


@pytest.mark.parametrize("canvas", ["tc", "scan"])
@pytest.mark.parametrize("cfg", [_hybrid(256), _hybrid(128)], ids=["hybrid-d256", "hybrid-d128"])
def test_cuda_runtime_long_canvases_match_cpu(cfg, canvas, monkeypatch):
    """Canvases of 33 and 63 rows (token-causal row counts that are not multiples of 16) and commits
    of 1 .. 32 accepted rows, vs the CPU statement: the tensor-core chunk step with its commit from
    the stored U rows ("tc", the default) and the per-token scan kernels ("scan")."""
    monkeypatch.setenv("TRIDA_GDN_CANVAS", canvas)
    dec = _init(cfg)
    dec_g = copy.deepcopy(dec).to("cuda", torch.bfloat16)
    torch.manual_seed(3)
    ids = torch.randint(0, 500, (3, 200))
    out = {}
    for name, d in (("cpu", dec), ("gpu", dec_g)):
        rt = Runtime(d, max_slots=4, max_len=320)
        slots = [rt.alloc() for _ in range(3)]
        last = rt.prefill(slots, ids[:, :37].tolist())
        lg = rt.canvas(slots, ids[:, 37:100], 32)         # draft block 32: 63 rows, 32 token-causal
        rt.commit(slots, [20, 17, 32])
        lg2 = rt.canvas(slots, ids[:, 100:133], 17)       # 33 rows, 17 token-causal
        rt.commit(slots, [17, 5, 16])
        lg3 = rt.canvas(slots, ids[:, 133:140], 4)
        rt.commit(slots, [3, 4, 1])
        out[name] = [t.float().cpu() for t in (last, lg, lg2, lg3)]
    for a, b in zip(out["gpu"], out["cpu"]):
        assert _rel(a, b) < 3e-2, _rel(a, b)


def test_paged_kv_pool_is_shared_and_recycled():
    """Full-attention KV in a pool of 64-position pages: a pool smaller than slots x max_len serves
    requests while they fit, refuses growth past it, and takes pages back on release; outputs match
    the CPU runtime's dense cache."""
    cfg = _hybrid(128)
    dec = _init(cfg)
    dec_g = copy.deepcopy(dec).to("cuda", torch.bfloat16)
    torch.manual_seed(5)
    ids = torch.randint(0, 500, (2, 150))
    rt = Runtime(dec_g, max_slots=4, max_len=1024, kv_pages=8)     # 8 pages: 512 positions in all
    cpu = Runtime(dec, max_slots=4, max_len=1024)
    s_g = [rt.alloc() for _ in range(2)]
    s_c = [cpu.alloc() for _ in range(2)]
    lg = rt.prefill(s_g, ids[:, :130].tolist())
    lc = cpu.prefill(s_c, ids[:, :130].tolist())
    assert _rel(lg.cpu(), lc) < 3e-2
    used = sum(len(p) for p in rt.pages.owned[:4])
    assert used == 2 * 3                       # 130 positions (+ a canvas) -> 3 pages per request
    a = rt.canvas(s_g, ids[:, 130:137], 4)
    rt.commit(s_g, [4, 4])
    b = cpu.canvas(s_c, ids[:, 130:137], 4)
    cpu.commit(s_c, [4, 4])
    assert _rel(a.cpu(), b) < 3e-2
    s3 = rt.alloc()
    with pytest.raises(RuntimeError, match="page pool"):
        rt.prefill([s3], [ids[0, :200].tolist()])
    rt.pending = None
    rt.release(s_g[0])
    rt.release(s3)
    assert len(rt.pages.free) >= 4


@pytest.mark.parametrize("mode", ["self-spec", "causal", "diffusion"])
def test_cuda_engine_graphs_match_eager(mode):
    dec = _init(_hybrid(256)).to("cuda", torch.bfloat16)
    torch.manual_seed(2)
    prompts = [torch.randint(0, 500, (40,)).tolist() for _ in range(6)]
    outs = []
    for graphs in (False, True):
        eng = Engine(Runtime(dec, max_slots=8, max_len=512), mask_id=511, mode=mode, n=4, graphs=graphs)
        reqs = eng.generate(prompts, max_new_tokens=50)
        assert all(len(r.output) == 50 for r in reqs)
        if mode != "diffusion":           # pure diffusion pays a commit forward per block
            assert eng.summary(reqs)["tokens_per_forward"] >= 1.0
        outs.append([r.output for r in reqs])
    assert outs[0] == outs[1]


def test_conf_argmax_rows_matches_softmax():
    """Fused greedy token + softmax probability per row (strided rows of a canvas) vs fp32 torch."""
    from trida_stack_b200.ops._ext import ext
    torch.manual_seed(0)
    lg = torch.randn(5, 9, 248320, device="cuda") * 3
    lg[1, 2, 77] = 40.0                               # a confident row
    view = lg[:, :8]                                  # non-contiguous batch stride
    idx = torch.empty(5, 8, dtype=torch.long, device="cuda")
    mx = torch.empty(5, 8, device="cuda")
    z = torch.empty(5, 8, device="cuda")
    ext().conf_argmax_rows(view, idx, mx, z)
    p = torch.softmax(view.double(), -1)
    conf, ref = p.max(-1)
    assert torch.equal(idx, ref)
    torch.testing.assert_close((1.0 / z).double(), conf, rtol=1e-4, atol=1e-6)
    torch.testing.assert_close(mx, view.max(-1).values)


def test_glm_ocr_runtime_cuda_matches_cpu():
    """GLM-OCR text decoder on the serving kernels (RoPE-only q / k path, output norms, image prefill
    with per-token 3-D RoPE tables, draft / verify canvases) vs the CPU statement of the same steps."""
    from trida_stack_b200.data.images import mrope_position_ids
    from trida_stack_b200.models.glm_ocr import GlmOcrDecoder, glm_ocr_config
    torch.manual_seed(0)
    cfg = glm_ocr_config({
        "model_type": "glm_ocr", "image_token_id": 500,
        "text_config": {"vocab_size": 512, "hidden_size": 256, "intermediate_size": 512, "num_hidden_layers": 2,
                        "num_attention_heads": 4, "num_key_value_heads": 2, "head_dim": 128,
                        "rope_parameters": {"rope_theta": 10000.0, "partial_rotary_factor": 0.5,
                                            "mrope_section": [8, 12, 12]}}})
    dec = GlmOcrDecoder(cfg, dtype=torch.float32)
    with torch.no_grad():
        for p in dec.parameters():
            if p.dim() == 1:
                p.add_(0.1 * torch.randn_like(p))
    dec = dec.to(torch.bfloat16).float()
    dec_g = copy.deepcopy(dec).to("cuda", torch.bfloat16)
    grid = torch.tensor([[1, 8, 12]])
    ids = torch.tensor([5, 6, 7] + [500] * 24 + list(range(10, 40)))
    feats = torch.randn(24, 256) * 0.5
    pos3 = mrope_position_ids(ids, grid, 500)
    out = {}
    for name, d in (("cpu", dec), ("gpu", dec_g)):
        rt = Runtime(d, max_slots=2, max_len=256)
        s = rt.alloc()
        last = rt.prefill([s], [ids.tolist()], vis=[(feats, pos3)], pos_offset=1)
        draft = rt.canvas([s], [[7] + [511] * 8], 1)
        rt.discard()
        ver = rt.canvas([s], [[7, 8, 9, 10, 11, 12, 13, 14, 15]], 9)
        rt.commit([s], [4])
        nxt = rt.canvas([s], [[20, 21, 22]], 3)
        rt.commit([s], [3])
        out[name] = [t.float().cpu() for t in (last, draft, ver, nxt)]
    for a, b in zip(out["gpu"], out["cpu"]):
        assert _rel(a, b) < 3e-2, _rel(a, b)


@pytest.mark.parametrize("n,n_clean,adv", [(7, 4, [1, 4, 3]), (33, 17, [17, 5, 9]), (64, 64, [64, 20, 1])])
def test_canvas_tc_kernels_match_recurrence(n, n_clean, adv):
    """The tensor-core canvas step and its commit from the stored U rows against the fp32 per-token
    recurrence (clean rows read their own state, the others the state after the canvas)."""
    from trida_stack_b200.ops._ext import ext
    from trida_stack_b200.ops.blocks import check_device_errors, device_error_word
    C = ext()
    torch.manual_seed(n)
    B, Hk, Hv, D = 3, 2, 4, 128
    dev = "cuda"
    kd = Hk * D
    mixed = (torch.randn(B * n, 2 * kd + Hv * D, device=dev) * 0.5).to(torch.bfloat16)
    gates = torch.randn(B * n, 2 * Hv, device=dev).to(torch.bfloat16)
    ga, gb = gates[:, :Hv], gates[:, Hv:]
    A_log = torch.log(torch.empty(Hv, device=dev).uniform_(0.5, 4))
    dtb = torch.randn(Hv, device=dev) * 0.1
    ssm = torch.randn(5, Hv, D, D, device=dev) * 0.05
    slot = torch.tensor([3, 0, 2], dtype=torch.int32, device=dev)
    o = torch.empty(B * n, Hv * D, dtype=torch.bfloat16, device=dev)
    kbuf = torch.empty(B * n, Hv, D, dtype=torch.bfloat16, device=dev)
    ubuf = torch.empty_like(kbuf)
    gbuf = torch.empty(B * n, Hv, device=dev)
    S_before = ssm.clone()
    err = device_error_word(dev)
    C.gdn_canvas_tc(mixed, ga, gb, A_log, dtb, o, kbuf, ubuf, gbuf, ssm, slot, n, Hk, Hv, n_clean, D ** -0.5, err)
    # the same step with the gated RMSNorm fused into the epilogue
    z = (torch.randn(B * n, Hv * D, device=dev)).to(torch.bfloat16)
    gw = (1 + 0.1 * torch.randn(D, device=dev)).to(torch.bfloat16)
    y = torch.empty_like(o)
    C.gdn_canvas_tc(mixed, ga, gb, A_log, dtb, y, kbuf, ubuf, gbuf, ssm, slot, n, Hk, Hv, n_clean, D ** -0.5, err,
                    z=z, gnorm_w=gw, eps=1e-6)
    adv_t = torch.tensor(adv, dtype=torch.int32, device=dev)
    C.gdn_commit_tc(kbuf, ubuf, gbuf, ssm, slot, adv_t, n, Hv, err)
    torch.cuda.synchronize()
    check_device_errors()
    # fp32 statement
    m = mixed.float().view(B, n, -1)
    q = torch.nn.functional.normalize(m[..., :kd].view(B, n, Hk, D), dim=-1) * D ** -0.5
    k = torch.nn.functional.normalize(m[..., kd:2 * kd].view(B, n, Hk, D), dim=-1)
    v = m[..., 2 * kd:].view(B, n, Hv, D)
    rep = Hv // Hk
    q, k = q.repeat_interleave(rep, 2), k.repeat_interleave(rep, 2)
    g = -A_log.exp() * torch.nn.functional.softplus(ga.float().view(B, n, Hv) + dtb)
    beta = torch.sigmoid(gb.float().view(B, n, Hv))
    o_ref = torch.zeros(B, n, Hv, D, device=dev)
    for bi in range(B):
        S = S_before[int(slot[bi])].clone()
        states = []
        for t in range(n):
            a_t = g[bi, t].exp()[:, None, None]
            u = beta[bi, t][:, None] * (v[bi, t] - a_t[:, :, 0] * torch.einsum("hkv,hk->hv", S, k[bi, t]))
            S = a_t * S + torch.einsum("hk,hv->hkv", k[bi, t], u)
            states.append(S.clone())
        for t in range(n):
            St = states[t if t < n_clean else n - 1]
            o_ref[bi, t] = torch.einsum("hkv,hk->hv", St, q[bi, t])
        ref_S = states[adv[bi] - 1]
        got_S = ssm[int(slot[bi])]
        assert _rel(got_S, ref_S) < 2e-2, (bi, _rel(got_S, ref_S))
    assert _rel(o.view(B, n, Hv, D), o_ref) < 2e-2, _rel(o.view(B, n, Hv, D), o_ref)
    from trida_stack_b200.ops.gdn_reference import gated_rmsnorm
    y_ref = gated_rmsnorm(o_ref, z.float().view(B, n, Hv, D), gw.float(), 1e-6)
    assert _rel(y.view(B, n, Hv, D), y_ref) < 2e-2, _rel(y.view(B, n, Hv, D), y_ref)
