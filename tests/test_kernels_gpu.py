"""sm_100a kernels vs plain-PyTorch fp32 statements of the same ops (B200 only)."""
import math

import pytest
import torch

from trida_stack_b200.ops import reference as R

pytestmark = pytest.mark.gpu


def C():
    from trida_stack_b200.ops._ext import ext
    return ext()


def rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("M,N,K", [(512, 384, 256), (2048, 3072, 2560), (300, 136, 72), (64, 2560, 9216),
                                   (448, 2560, 4096), (100, 136, 1000)])
def test_gemm_layouts(M, N, K):
    torch.manual_seed(0)
    dev = "cuda"
    x = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=dev, dtype=torch.bfloat16)
    # TN: y = x w^T (+ residual)
    res = torch.randn(M, N, device=dev, dtype=torch.bfloat16)
    y = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    C().gemm(0, x, w, y, res, 1.0, 1.0, 0)
    ref = x.float() @ w.float().t() + res.float()
    assert rel_err(y, ref) < 1e-2
    # TT: dx = dy w
    dy = torch.randn(M, N, device=dev, dtype=torch.bfloat16)
    dx = torch.empty(M, K, device=dev, dtype=torch.bfloat16)
    C().gemm(1, dy, w, dx, None, 1.0, 0.0, 0)
    assert rel_err(dx, dy.float() @ w.float()) < 1e-2
    # NT: dw = dy^T x accumulated into fp32
    acc = torch.randn(N, K, device=dev, dtype=torch.float32)
    ref_w = acc + dy.float().t() @ x.float()
    C().gemm(2, dy, x, acc, acc, 1.0, 1.0, 0)
    assert rel_err(acc, ref_w) < 1e-3


@pytest.mark.parametrize("tile", [1, 2, 3])
def test_gemm_tiles(tile):
    torch.manual_seed(1)
    a = torch.randn(1024, 512, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(768, 512, device="cuda", dtype=torch.bfloat16)
    d = torch.empty(1024, 768, device="cuda", dtype=torch.bfloat16)
    C().gemm(0, a, b, d, None, 1.0, 0.0, tile)
    assert rel_err(d, a.float() @ b.float().t()) < 1e-2


@pytest.mark.parametrize("M,D,res", [(1000, 2560, True), (777, 2560, False), (300, 5120, True), (129, 1536, False),
                                     (64, 1000, True)])
def test_rmsnorm_fwd_bwd(M, D, res):
    """Row-resident kernels (D = 256 k, x / dy kept in registers up to D = 2560, re-read above) and
    the general loop kernel (D = 1000)."""
    torch.manual_seed(0)
    x = torch.randn(M, D, device="cuda", dtype=torch.bfloat16)
    w = (1 + 0.1 * torch.randn(D, device="cuda")).to(torch.bfloat16)
    y = torch.empty_like(x)
    _, rstd = C().rmsnorm_fwd(x, w, 1e-6, y)
    xr = x.float().requires_grad_()
    wr = w.float().requires_grad_()
    yr = xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + 1e-6) * wr
    assert rel_err(y, yr) < 1e-2
    torch.testing.assert_close(rstd, torch.rsqrt(x.float().pow(2).mean(-1) + 1e-6), rtol=1e-4, atol=1e-5)
    dy = torch.randn_like(x)
    dres = torch.randn_like(x) if res else None
    yr.backward(dy.float())
    dx = torch.empty_like(x)
    dw = torch.zeros(D, device="cuda")
    C().rmsnorm_bwd(dy, x, w, rstd, dres, dx, dw)
    assert rel_err(dx, xr.grad + (dres.float() if res else 0)) < 1e-2
    assert rel_err(dw, wr.grad) < 1e-3


@pytest.mark.parametrize("d,rd,shape", [(128, 128, (2, 96, 4, 2)), (256, 64, (2, 96, 4, 2)),
                                        (128, 64, (1, 95, 4, 1)), (64, 64, (1, 95, 4, 1)),
                                        (128, 96, (2, 33, 4, 2)), (128, 72, (2, 33, 4, 2))])
def test_qk_norm_rope(d, rd, shape):
    """Vector kernels (d in 64 / 128 / 256, rd a multiple of 16; an odd head count leaves the last
    warp's second head group empty) and the per-element kernels (rd = 72)."""
    torch.manual_seed(0)
    B, T, Hq, Hkv = shape
    M = B * T
    qkv = torch.randn(M, (Hq + 2 * Hkv) * d, device="cuda", dtype=torch.bfloat16)
    qw = (1 + 0.1 * torch.randn(d, device="cuda")).to(torch.bfloat16)
    kw = (1 + 0.1 * torch.randn(d, device="cuda")).to(torch.bfloat16)
    pos = torch.randint(0, 4000, (B, T), device="cuda")
    from trida_stack_b200.ops.blocks import rope_tables
    cos_t, sin_t = rope_tables(4096, rd, 1e6, "cuda")
    q = torch.empty(B, T, Hq, d, device="cuda", dtype=torch.bfloat16)
    k = torch.empty(B, T, Hkv, d, device="cuda", dtype=torch.bfloat16)
    rstd = C().qk_norm_rope_fwd(qkv, qw, kw, cos_t, sin_t, pos.int().reshape(-1).contiguous(), q, k, Hq, Hkv, d,
                                rd, 1e-6)
    src = qkv.float().requires_grad_()
    qwr, kwr = qw.float().requires_grad_(), kw.float().requires_grad_()
    qs = src[:, :Hq * d].view(B, T, Hq, d)
    ks = src[:, Hq * d:(Hq + Hkv) * d].view(B, T, Hkv, d)
    cos, sin = R.rope_cos_sin(pos, d, 1e6, rd)
    qr = R.apply_rope(R.rmsnorm(qs, qwr, 1e-6), cos, sin)
    kr = R.apply_rope(R.rmsnorm(ks, kwr, 1e-6), cos, sin)
    assert rel_err(q, qr) < 1e-2 and rel_err(k, kr) < 1e-2
    gq, gk = torch.randn_like(q), torch.randn_like(k)
    (qr * gq.float()).sum().add((kr * gk.float()).sum()).backward()
    dqkv = torch.zeros_like(qkv)
    dqw = torch.zeros(d, device="cuda")
    dkw = torch.zeros(d, device="cuda")
    C().qk_norm_rope_bwd(gq, gk, qkv, qw, kw, cos_t, sin_t, pos.int().reshape(-1).contiguous(), rstd, dqkv, dqw,
                         dkw, Hq, Hkv, d, rd)
    assert rel_err(dqkv[:, :(Hq + Hkv) * d], src.grad[:, :(Hq + Hkv) * d]) < 1e-2
    assert rel_err(dqw, qwr.grad) < 1e-2 and rel_err(dkw, kwr.grad) < 1e-2
    # RoPE only (no per-head norm weights): the rotation of the raw q / k
    C().qk_norm_rope_fwd(qkv, None, None, cos_t, sin_t, pos.int().reshape(-1).contiguous(), q, k, Hq, Hkv, d, rd,
                         1e-6)
    assert rel_err(q, R.apply_rope(qs.detach(), cos, sin)) < 1e-2
    assert rel_err(k, R.apply_rope(ks.detach(), cos, sin)) < 1e-2


@pytest.mark.parametrize("M,K,F", [(777, 512, 320), (2048, 640, 1280), (130, 2560, 9728)])
def test_gemm_swiglu_epilogue(M, K, F):
    """Gate / up GEMM with SwiGLU in the epilogue: gu matches the plain GEMM and act matches the
    SwiGLU kernel applied to that gu (both from the same bf16-rounded values), for both tile heights.  F = 320 leaves half
    of the last 128-feature tile past the end; (2048, 1280) takes the 256-row tiles."""
    torch.manual_seed(0)
    x = (torch.randn(M, K, device="cuda") * 0.5).to(torch.bfloat16)
    w = (torch.randn(2 * F, K, device="cuda") / K ** 0.5).to(torch.bfloat16)
    gu = torch.empty(M, 2 * F, device="cuda", dtype=torch.bfloat16)
    act = torch.empty(M, F, device="cuda", dtype=torch.bfloat16)
    C().gemm_swiglu(x, w, gu, act)
    ref = torch.empty_like(gu)
    C().gemm(0, x, w, ref, None, 1.0, 0.0, 0)
    torch.testing.assert_close(gu, ref, rtol=1e-2, atol=1e-2)     # the plain GEMM may split K
    act_ref = torch.empty_like(act)
    C().swiglu_fwd(gu, act_ref)
    torch.testing.assert_close(act, act_ref, rtol=1e-2, atol=1e-3)
    for tile in (1, 2):
        act2 = torch.empty_like(act)
        C().gemm_swiglu(x, w, gu, act2, tile)
        torch.testing.assert_close(act2, act, rtol=0, atol=0)
    assert rel_err(gu, x.float() @ w.float().t()) < 1e-2


def test_swiglu():
    torch.manual_seed(0)
    M, F = 777, 9728
    gu = torch.randn(M, 2 * F, device="cuda", dtype=torch.bfloat16)
    a = torch.empty(M, F, device="cuda", dtype=torch.bfloat16)
    C().swiglu_fwd(gu, a)
    gr = gu.float().requires_grad_()
    ar = R.swiglu(gr)
    assert rel_err(a, ar) < 1e-2
    da = torch.randn_like(a)
    ar.backward(da.float())
    dgu = torch.empty_like(gu)
    C().swiglu_bwd(da, gu, dgu)
    assert rel_err(dgu, gr.grad) < 1e-2


def bd_layout(B, P, Rr, bd, device, packed=False):
    """Metadata of [S | x_t] + [x_0] rows (the single-row block-diffusion layout)."""
    L = P + Rr
    T = L + Rr
    seg = torch.full((B, T), R.SHARED, dtype=torch.int32)
    seg[:, P:L] = R.XT
    seg[:, L:] = R.X0
    opos = torch.cat([torch.arange(L), torch.arange(P, L)])[None].expand(B, -1).clone().int()
    rblk = torch.cat([torch.clamp(torch.arange(L) - P, min=0) // bd, torch.arange(Rr) // bd])[None].expand(B, -1)
    rblk = rblk.clone().int()
    segid = torch.zeros(B, T, dtype=torch.int32)
    view = torch.zeros(B, T, dtype=torch.int32)
    # ragged padding on the second row: last 40 prompt-region slots and the tail of x_0 are PAD
    if B > 1:
        seg[1, L - 40:L] = R.PAD
        seg[1, T - 40:] = R.PAD
    if packed:
        segid[:, T // 2:] = 1
    return {k: v.to(device) for k, v in dict(seg=seg, opos=opos, rblk=rblk, segid=segid, view=view).items()}


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("x0tok,wbc,packed", [(True, False, False), (False, False, False), (True, True, True)])
def test_bd_attention_fwd_bwd(d, x0tok, wbc, packed):
    torch.manual_seed(0)
    B, P, Rr, bd, Hq, Hkv = 2, 96, 160, 32, 4, 2
    meta = bd_layout(B, P, Rr, bd, "cuda", packed)
    T = meta["seg"].shape[1]
    q = torch.randn(B, T, Hq, d, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(B, T, Hkv, d, device="cuda", dtype=torch.bfloat16)
    kv = torch.randn(B, T, 2 * Hkv, d, device="cuda", dtype=torch.bfloat16)
    v = kv[:, :, Hkv:]  # strided view, like the v slice of the fused qkv projection
    from trida_stack_b200.ops.blocks import AttnContext
    actx = AttnContext(meta["seg"], meta["opos"], meta["rblk"], meta["segid"], meta["view"], meta["opos"], x0tok, wbc)
    _, fl, fc, bl, bc = actx.plan
    o = torch.empty_like(q)
    lse = torch.empty(B, Hq, T, device="cuda")
    scale = 1 / math.sqrt(d)
    C().bd_attn_fwd(q, k, v, o, lse, actx.meta, fl, fc, actx.flags, scale)
    qr, kr, vr = (t.float().requires_grad_() for t in (q, k, v))
    orf = R.bd_attention(qr, kr, vr, actx.meta_dict(), x0tok, wbc)
    valid_q = (meta["seg"] != R.PAD)[:, :, None, None]
    assert rel_err(o * valid_q, orf * valid_q) < 1e-2
    do = torch.randn_like(q) * valid_q
    (orf * do.float()).sum().backward()
    dq, dk = torch.empty_like(q), torch.empty_like(k)
    dkv = torch.zeros_like(kv)
    dv = dkv[:, :, Hkv:]
    C().bd_attn_bwd(q, k, v, o, lse, do, dq, dk, dv, actx.meta, bl, bc, actx.flags, scale)
    assert rel_err(dq, qr.grad) < 2e-2
    assert rel_err(dk, kr.grad) < 2e-2
    assert rel_err(dv, vr.grad) < 2e-2


@pytest.mark.parametrize("d", [64, 128, 256])
@pytest.mark.parametrize("x0tok,wbc,packed", [(True, False, False), (False, True, False), (True, False, True)])
def test_bd_attention_fwd_tcgen05(d, x0tok, wbc, packed):
    torch.manual_seed(0)
    B, P, Rr, bd, Hq, Hkv = 2, 160, 192, 32, 4, 2   # T = 544: ragged last 128-tile
    meta = bd_layout(B, P, Rr, bd, "cuda", packed)
    T = meta["seg"].shape[1]
    q = torch.randn(B, T, Hq, d, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(B, T, Hkv, d, device="cuda", dtype=torch.bfloat16)
    kv = torch.randn(B, T, 2 * Hkv, d, device="cuda", dtype=torch.bfloat16)
    v = kv[:, :, Hkv:]
    from trida_stack_b200.ops.blocks import AttnContext, device_error_word, check_device_errors
    actx = AttnContext(meta["seg"], meta["opos"], meta["rblk"], meta["segid"], meta["view"], meta["opos"], x0tok, wbc)
    l128, c128 = actx.plan128
    o = torch.full_like(q, float("nan"))
    lse = torch.empty(B, Hq, T, device="cuda")
    C().bd_attn_fwd_sm100(q, k, v, o, lse, actx.meta, l128, c128, actx.masks[0], actx.flags, 1 / math.sqrt(d),
                          device_error_word("cuda"))
    torch.cuda.synchronize()
    check_device_errors()
    ref = R.bd_attention(q.float(), k.float(), v.float(), actx.meta_dict(), x0tok, wbc)
    valid_q = (meta["seg"] != R.PAD)[:, :, None, None]
    assert torch.isfinite(o).all()
    assert rel_err(o * valid_q, ref * valid_q) < 1e-2
    # LSE agrees with the warp-MMA kernel's
    o2, lse2 = torch.empty_like(q), torch.empty_like(lse)
    _, fl, fc, _, _ = actx.plan
    C().bd_attn_fwd(q, k, v, o2, lse2, actx.meta, fl, fc, actx.flags, 1 / math.sqrt(d))
    assert (lse - lse2).abs().max().item() < 1e-2


@pytest.mark.parametrize("d", [64, 128, 256])
@pytest.mark.parametrize("x0tok,wbc,packed", [(True, False, False), (False, True, False), (True, False, True)])
def test_bd_attention_bwd_tcgen05(d, x0tok, wbc, packed):
    """head_dim 64 / 128: one kernel per (key tile, query head) with TMA-reduced fp32 dQ; head_dim
    256: a dK / dV kernel per half of d plus a dQ kernel over the forward tile lists."""
    torch.manual_seed(0)
    B, P, Rr, bd, Hq, Hkv = 2, 160, 192, 32, 4, 2   # T = 544: ragged last 128-tile
    meta = bd_layout(B, P, Rr, bd, "cuda", packed)
    T = meta["seg"].shape[1]
    q = torch.randn(B, T, Hq, d, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(B, T, Hkv, d, device="cuda", dtype=torch.bfloat16)
    kv = torch.randn(B, T, 2 * Hkv, d, device="cuda", dtype=torch.bfloat16)
    v = kv[:, :, Hkv:]
    from trida_stack_b200.ops.blocks import AttnContext, device_error_word, check_device_errors
    actx = AttnContext(meta["seg"], meta["opos"], meta["rblk"], meta["segid"], meta["view"], meta["opos"], x0tok, wbc)
    _, fl, fc, _, _ = actx.plan
    o = torch.empty_like(q)
    lse = torch.empty(B, Hq, T, device="cuda")
    scale = 1 / math.sqrt(d)
    C().bd_attn_fwd(q, k, v, o, lse, actx.meta, fl, fc, actx.flags, scale)
    qr, kr, vr = (t.float().requires_grad_() for t in (q, k, v))
    orf = R.bd_attention(qr, kr, vr, actx.meta_dict(), x0tok, wbc)
    valid_q = (meta["seg"] != R.PAD)[:, :, None, None]
    do = torch.randn_like(q) * valid_q
    (orf * do.float()).sum().backward()
    lt, ct = actx.plan128t
    dq = torch.full_like(q, float("nan"))
    dk = torch.full_like(k, float("nan"))
    dkv = torch.zeros_like(kv)
    dv = dkv[:, :, Hkv:]
    extra = {}
    if d == 256:
        l128, c128 = actx.plan128
        extra = {"list128": l128, "cnt128": c128, "rowmask": actx.masks[0]}
    C().bd_attn_bwd_sm100(q, k, v, o, lse, do, dq, dk, dv, actx.meta, lt, ct, actx.masks[1], actx.flags, scale,
                          device_error_word("cuda"), **extra)
    torch.cuda.synchronize()
    check_device_errors()
    assert torch.isfinite(dq).all() and torch.isfinite(dk).all() and torch.isfinite(dv).all()
    assert rel_err(dq, qr.grad) < 2e-2
    assert rel_err(dk, kr.grad) < 2e-2
    assert rel_err(dv, vr.grad) < 2e-2


def test_attention_plan_skips_and_classifies():
    meta = bd_layout(1, 128, 256, 32, "cuda")
    from trida_stack_b200.ops.blocks import AttnContext
    actx = AttnContext(meta["seg"], meta["opos"], meta["rblk"], meta["segid"], meta["view"], meta["opos"], True, False)
    cls = actx.plan[0].cpu()
    eye = torch.eye(meta["seg"].shape[1], dtype=torch.bool, device="cuda")
    dense = R.bd_allowed(actx.meta_dict(), actx.meta_dict(), True, False, eye)[0].cpu()
    nt = cls.shape[1]
    for i in range(nt):
        for j in range(nt):
            blk = dense[i * 64:(i + 1) * 64, j * 64:(j + 1) * 64]
            want = 0 if not blk.any() else (1 if blk.all() else 2)
            assert int(cls[0, i, j]) == want


def test_fused_linear_ce():
    torch.manual_seed(0)
    from trida_stack_b200.ops.ce import fused_linear_ce
    N, D, V = 3000, 256, 50000
    h = (torch.randn(N, D, device="cuda") * 0.5).to(torch.bfloat16).requires_grad_()
    w = (torch.randn(V, D, device="cuda") * 0.05).to(torch.bfloat16).requires_grad_()
    tgt = torch.randint(0, V, (N,), device="cuda")
    wt = torch.rand(N, device="cuda")
    wt = wt / wt.sum()
    loss, ce = fused_linear_ce(h, w, tgt, wt, chunk=1024)
    (loss * 3.0).backward()
    hr, wr = h.detach().float().requires_grad_(), w.detach().float().requires_grad_()
    lr = R.linear_ce(hr, wr, tgt, wt)
    (lr * 3.0).backward()
    assert abs(loss.item() - lr.item()) < 1e-3 * max(1, abs(lr.item()))
    assert rel_err(h.grad, hr.grad) < 2e-2
    assert rel_err(w.grad, wr.grad) < 2e-2


def test_adamw_matches_torch():
    torch.manual_seed(0)
    n = 100003
    p = torch.randn(n, device="cuda")
    g = torch.randn(n, device="cuda")
    ref = p.clone().requires_grad_()
    opt = torch.optim.AdamW([ref], lr=1e-3, betas=(0.9, 0.95), weight_decay=0.1, eps=1e-8)
    m = torch.zeros(n, device="cuda")
    v = torch.zeros(n, device="cuda")
    for step in range(1, 4):
        ref.grad = g * 0.5
        opt.step()
        norm = torch.zeros(1, device="cuda")
        coef = torch.zeros(1, device="cuda")
        C().grad_norm([g], 1e9, norm, coef)
        assert abs(norm.item() - g.norm().item()) < 1e-3 * g.norm().item()
        C().adamw(p, None, g * 0.5, m, v, 1e-3, 0.9, 0.95, 1e-8, 0.1, step, coef)
    assert rel_err(p, ref.detach()) < 1e-5


@pytest.mark.parametrize("n,offset", [(100003, 0), (4096, 3)])
def test_adamw_bf16_params_match_torch(n, offset):
    """bf16 parameters updated in place (8-wide vector kernel plus scalar tail; an offset view
    takes the unaligned path) against torch AdamW in fp32 with the parameter rounded to bf16
    after every step."""
    torch.manual_seed(0)
    base = torch.randn(n + offset, device="cuda").to(torch.bfloat16)
    p = base[offset:]
    g = torch.randn(n, device="cuda")
    ref = p.float().clone().requires_grad_()
    opt = torch.optim.AdamW([ref], lr=1e-3, betas=(0.9, 0.95), weight_decay=0.1, eps=1e-8)
    m = torch.zeros(n, device="cuda")
    v = torch.zeros(n, device="cuda")
    for step in range(1, 4):
        ref.grad = g.clone()
        opt.step()
        with torch.no_grad():
            ref.copy_(ref.bfloat16().float())
        C().adamw(p, None, g, m, v, 1e-3, 0.9, 0.95, 1e-8, 0.1, step, None)
    assert rel_err(p, ref.detach()) < 2e-3
    torch.testing.assert_close(m, opt.state[ref]["exp_avg"], rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(v, opt.state[ref]["exp_avg_sq"], rtol=1e-5, atol=1e-7)


def test_blocks_match_cpu_reference():
    """Whole attention + MLP sub-blocks, forward and backward, GPU bf16 vs CPU fp32."""
    torch.manual_seed(0)
    from trida_stack_b200.models import qwen3_config
    from trida_stack_b200.ops import blocks
    cfg = qwen3_config(vocab_size=512, hidden_size=256, intermediate_size=512, num_layers=1, n_heads=4,
                       n_kv_heads=2, head_dim=64)
    B, P, Rr, bd = 2, 64, 128, 32
    meta = bd_layout(B, P, Rr, bd, "cpu")
    T = meta["seg"].shape[1]
    D = cfg.hidden_size
    params = [torch.randn(D) * 0.1 + 1, torch.randn(cfg.n_heads * 64 + 2 * cfg.n_kv_heads * 64, D) * 0.05,
              torch.randn(64) * 0.1 + 1, torch.randn(64) * 0.1 + 1, torch.randn(D, cfg.n_heads * 64) * 0.05,
              torch.randn(D) * 0.1 + 1, torch.randn(2 * 512, D) * 0.05, torch.randn(D, 512) * 0.05]
    x = torch.randn(B * T, D)
    dy = torch.randn(B * T, D)

    def run(dev, dtype):
        ps = [p.detach().to(dev, dtype).requires_grad_() for p in params]
        xx = x.detach().to(dev, dtype).requires_grad_()
        m = {k: v.to(dev) for k, v in meta.items()}
        cos_t = sin_t = None
        if dev == "cuda":
            cos_t, sin_t = blocks.rope_tables(4096, 64, cfg.rope_theta, dev)
        actx = blocks.AttnContext(m["seg"], m["opos"], m["rblk"], m["segid"], m["view"], m["opos"], True, False,
                                  cos_t, sin_t)
        h = blocks.attn_block(xx, *ps[:5], actx, cfg)
        y = blocks.mlp_block(h, ps[5], ps[6], ps[7], cfg.eps)
        y.backward(dy.to(dev, dtype))
        return y.float().cpu(), xx.grad.float().cpu(), [p.grad.float().cpu() for p in ps]

    y0, gx0, gp0 = run("cpu", torch.float32)
    y1, gx1, gp1 = run("cuda", torch.bfloat16)
    assert rel_err(y1, y0) < 2e-2
    assert rel_err(gx1, gx0) < 3e-2
    for a, b in zip(gp1, gp0):
        assert rel_err(a, b) < 5e-2


@pytest.mark.parametrize("mrope", [False, True])
def test_gated_attention_block_d256_matches_cpu_reference(mrope):
    """Qwen3.5 full-attention sub-block: head_dim 256, partial RoPE (64 of 256), q/gate interleaved
    per head and the sigmoid output gate; GPU bf16 vs CPU fp32.  ``mrope``: per-token 3-D (t, h, w)
    RoPE angles of vision-language rows instead of the shared position table."""
    torch.manual_seed(0)
    from trida_stack_b200.models.config import ModelConfig
    from trida_stack_b200.ops import blocks
    cfg = ModelConfig.from_hf_dict({
        "model_type": "qwen3_5_text", "vocab_size": 256, "hidden_size": 256, "intermediate_size": 512,
        "num_hidden_layers": 1, "num_attention_heads": 4, "num_key_value_heads": 2, "head_dim": 256,
        "partial_rotary_factor": 0.25, "layer_types": ["full_attention"], "rms_norm_eps": 1e-6})
    assert cfg.attn_output_gate and cfg.rotary_dim == 64
    d, Hq, Hkv, D = 256, cfg.n_heads, cfg.n_kv_heads, cfg.hidden_size
    B, P, Rr, bd = 2, 64, 128, 32
    meta = bd_layout(B, P, Rr, bd, "cpu")
    T = meta["seg"].shape[1]
    params = [torch.randn(D) * 0.1 + 1, torch.randn(2 * Hq * d + 2 * Hkv * d, D) * 0.05,
              torch.randn(d) * 0.1 + 1, torch.randn(d) * 0.1 + 1, torch.randn(D, Hq * d) * 0.05]
    x = torch.randn(B * T, D)
    dy = torch.randn(B * T, D)

    def run(dev, dtype):
        ps = [p.detach().to(dev, dtype).requires_grad_() for p in params]
        xx = x.detach().to(dev, dtype).requires_grad_()
        m = {k: v.to(dev) for k, v in meta.items()}
        cos_t = sin_t = None
        if dev == "cuda":
            cos_t, sin_t = blocks.rope_tables(4096, cfg.rotary_dim, cfg.rope_theta, dev)
        actx = blocks.AttnContext(m["seg"], m["opos"], m["rblk"], m["segid"], m["view"], m["opos"], True, False,
                                  cos_t, sin_t)
        if mrope:
            from trida_stack_b200.models.vision import mrope_angles
            op = m["opos"].long()
            t = torch.arange(T, device=dev)[None]
            pos3 = torch.stack([op, op + t % 5, op + t % 3], 1)
            actx.set_rope_angles(mrope_angles(pos3, cfg.rotary_dim, cfg.rope_theta, cfg.mrope_section))
        y = blocks.attn_block(xx, *ps, actx, cfg)
        y.backward(dy.to(dev, dtype))
        return y.float().cpu(), xx.grad.float().cpu(), [p.grad.float().cpu() for p in ps]

    y0, gx0, gp0 = run("cpu", torch.float32)
    y1, gx1, gp1 = run("cuda", torch.bfloat16)
    assert rel_err(y1 - x, y0 - x) < 2e-2
    assert rel_err(gx1, gx0) < 3e-2
    for a, b in zip(gp1, gp0):
        assert rel_err(a, b) < 5e-2


@pytest.mark.parametrize("tile", [1, 2])
def test_gemm_tile_shapes_ragged_all_layouts(tile):
    """128- and 256-row tiles on ragged shapes (partial row halves, partial N tiles) in all layouts."""
    torch.manual_seed(3)
    M, N, K = 600, 520, 200
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
    y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    C().gemm(0, x, w, y, None, 1.0, 0.0, tile)
    assert rel_err(y, x.float() @ w.float().t()) < 1e-2
    dy = torch.randn(M, N, device="cuda", dtype=torch.bfloat16)
    dx = torch.empty(M, K, device="cuda", dtype=torch.bfloat16)
    C().gemm(1, dy, w, dx, None, 1.0, 0.0, tile)
    assert rel_err(dx, dy.float() @ w.float()) < 1e-2
    acc = torch.randn(N, K, device="cuda", dtype=torch.float32)
    ref = acc + dy.float().t() @ x.float()
    C().gemm(2, dy, x, acc, acc, 1.0, 1.0, tile)
    assert rel_err(acc, ref) < 1e-3


def test_streamed_layer_gradients_cuda_match_resident():
    """On the CUDA blocks (weight gradients written into main_grad by the GEMM epilogue), streaming
    each layer's gradients through the two-slot ring equals the resident full buffers."""
    import copy

    from trida_stack_b200.engine import TrainEngine
    from trida_stack_b200.models import BlockDiffusionLM, Decoder, qwen3_config
    torch.manual_seed(0)
    cfg = qwen3_config(vocab_size=512, hidden_size=256, intermediate_size=512, num_layers=3, n_heads=4,
                       n_kv_heads=2, head_dim=64)
    dec = Decoder(cfg, dtype=torch.bfloat16, device="cuda")
    outs = []
    for stream, ckpt in ((False, "none"), (True, "none"), (True, "layer")):
        m = BlockDiffusionLM(copy.deepcopy(dec), mask_id=511, pad_id=510, bd_size=32, ar_loss_weight=1.0,
                             activation_checkpoint=ckpt)
        m.train()
        eng = TrainEngine(m, lr=1e-3, warmup=0, max_steps=10, device=torch.device("cuda"), grad_stream=stream)
        g = torch.Generator().manual_seed(1)
        torch.manual_seed(5)
        for step in range(2):
            ids = torch.randint(0, 509, (2, 128), generator=g)
            labels = ids.clone()
            labels[:, :64] = -100
            eng.train_step([{"input_ids": ids, "labels": labels, "attention_mask": torch.ones_like(ids)}], step)
        outs.append([p.detach().float().cpu() for p in m.parameters()])
        if stream:
            # every streamed weight gradient went through the ring, also under activation checkpointing
            eng.micro_step({"input_ids": ids, "labels": labels, "attention_mask": torch.ones_like(ids)})
            leaked = [n for n, p in m.named_parameters() if hasattr(p, "_grad_acquire") and p.grad is not None]
            assert not leaked, leaked
    for o in outs[1:]:
        for a, b in zip(o, outs[0]):
            assert rel_err(a, b) < 1e-3


@pytest.mark.parametrize("M,N,K", [(300, 5000, 512), (4032, 248320 // 8, 2560), (7, 1000, 256)])
def test_gemm_argmax_epilogue(M, N, K):
    """The LM head's argmax from the GEMM epilogue (per-tile partials + reduce) equals argmax of the
    materialised product; near ties the chosen column's value is within rounding of the max."""
    torch.manual_seed(M)
    A = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    B = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(M, dtype=torch.long, device="cuda")
    C().gemm_argmax(A, B, out)
    ref = A.float() @ B.float().t()
    best = ref.max(-1).values
    got = ref.gather(1, out[:, None])[:, 0]
    assert bool((out >= 0).all()) and bool((out < N).all())
    assert (best - got).abs().max().item() <= 1e-2 * best.abs().max().item()
    assert (out == ref.argmax(-1)).float().mean().item() > 0.98
