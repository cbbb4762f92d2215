"""Kernel microbenchmarks on the benchmark configs' shapes (device-timed with CUDA events).

    python -m trida_stack_b200.ops.kernel_bench --op gemm [--m 24576 --n 6144 --k 2560 --layout tn]
    python -m trida_stack_b200.ops.kernel_bench --op attn_fwd|attn_bwd [--rows 4] [--heads 32 --kv-heads 8 --head-dim 128]
    python -m trida_stack_b200.ops.kernel_bench --op gdn_fwd|gdn_bwd [--length 3072] [--gdn-path chunk|scan]
                                                     [--gdn-layout two_stream|causal]
    python -m trida_stack_b200.ops.kernel_bench --op gdn_core_fwd|gdn_core_bwd [--length 3072]
    python -m trida_stack_b200.ops.kernel_bench --op canvas_attn|canvas_attn_tc|canvas_gdn|canvas_gdn_tc|commit_gdn_tc
                                                     [--requests 64 --blk 7]
    python -m trida_stack_b200.ops.kernel_bench --op rmsnorm_fwd|rmsnorm_bwd|qk_rope_fwd|qk_rope_bwd|
                                                     swiglu_fwd|swiglu_bwd [--m 24576 --hidden 2560]

Each run does ``--warmup`` untimed launches, then times ``--iters`` launches and prints one JSON
line with the mean time, the achieved rate and its fraction of the measured B200 peaks in
``MEASURED_PEAKS.json`` (repository root) when present.  The same command line under
``ncu -k <kernel> -s <warm-up launches> -c 1`` gives the per-kernel profile.
"""
import argparse
import json
import math
import os

import torch


def _peaks():
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                     "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f)
    return {}


def _time(fn, warmup, iters):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def bench_gemm(a):
    from ._ext import ext
    C = ext()
    M, N, K = a.m, a.n, a.k
    layout = {"tn": 0, "tt": 1, "nt": 2}[a.layout]
    if layout == 0:
        A = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
        B = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
    elif layout == 1:
        A = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
        B = torch.randn(K, N, device="cuda", dtype=torch.bfloat16)
    else:
        A = torch.randn(K, M, device="cuda", dtype=torch.bfloat16)
        B = torch.randn(K, N, device="cuda", dtype=torch.bfloat16)
    D = torch.empty(M, N, device="cuda", dtype=torch.float32 if layout == 2 else torch.bfloat16)
    if a.op == "gemm_swiglu":   # gate / up projection with SwiGLU in the epilogue (N = 2F)
        act = torch.empty(M, N // 2, device="cuda", dtype=torch.bfloat16)
        ms = _time(lambda: C.gemm_swiglu(A, B, D, act, a.tile), a.warmup, a.iters)
        return ms, {"tflops": 2 * M * N * K / ms / 1e9}, 2 * M * N * K, None
    ms = _time(lambda: C.gemm(layout, A, B, D, None, 1.0, 0.0, a.tile), a.warmup, a.iters)
    return ms, {"tflops": 2 * M * N * K / ms / 1e9}, 2 * M * N * K, None


def _bd_actx(rows, P, R, bd, dev):
    from ..models.block_diffusion import BlockDiffusionLM  # noqa: F401  (layout helpers live with the model)
    from . import blocks
    from .reference import SHARED, X0, XT
    T = P + 2 * R
    seg = torch.tensor([SHARED] * P + [XT] * R + [X0] * R, device=dev)[None].repeat(rows, 1)
    opos = torch.cat([torch.arange(P), torch.arange(P, P + R), torch.arange(P, P + R)]).to(dev)[None].repeat(rows, 1)
    rblk = torch.where(seg == SHARED, torch.zeros_like(opos), (opos - P) // bd)
    segid = torch.zeros_like(opos)
    view = torch.where(seg == XT, torch.ones_like(opos), torch.zeros_like(opos))
    cos_t, sin_t = blocks.rope_tables(P + R + 1, 128, 1e6, dev)
    return blocks.AttnContext(seg, opos, rblk, segid, view, opos, True, False, cos_t, sin_t), T


def bench_attn(a, backward):
    from . import blocks
    dev = "cuda"
    actx, T = _bd_actx(a.rows, 1024, 1024, 32, dev)
    B, Hq, Hkv, d = a.rows, a.heads, a.kv_heads, a.head_dim
    q = torch.randn(B, T, Hq, d, device=dev, dtype=torch.bfloat16)
    k = torch.randn(B, T, Hkv, d, device=dev, dtype=torch.bfloat16)
    v = torch.randn(B, T, Hkv, d, device=dev, dtype=torch.bfloat16)
    o = torch.empty_like(q)
    lse = torch.empty(B, Hq, T, device=dev, dtype=torch.float32)
    blocks.attn_fwd(q, k, v, o, lse, actx)
    # FLOPs of the allowed (key, query) pairs: 4 d per pair forward (QK^T and PV), 2.5x backward
    allowed = _allowed_pairs(actx)
    flops = 4 * d * Hq * allowed * (2.5 if backward else 1.0)
    if not backward:
        ms = _time(lambda: blocks.attn_fwd(q, k, v, o, lse, actx), a.warmup, a.iters)
    else:
        do = torch.randn_like(o)
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        ms = _time(lambda: blocks.attn_bwd(q, k, v, o, lse, do, dq, dk, dv, actx), a.warmup, a.iters)
    return ms, {"tflops": flops / ms / 1e9, "allowed_pairs": allowed}, flops, None


def _allowed_pairs(actx):
    from .reference import bd_allowed
    m = {k: v[:1].cpu() for k, v in actx.meta_dict().items()}
    T = m["seg"].shape[1]
    same = torch.eye(T, dtype=torch.bool)
    return int(bd_allowed(m, m, actx.x0_token_causal, actx.within_block_causal, same).sum()) * actx.B


def bench_gdn(a, backward):
    from types import SimpleNamespace

    from ..models.config import ModelConfig
    from ..models.gdn import GatedDeltaLayer
    from .gdn import LinearLayout
    from .gdn_cuda import gdn_block_cuda
    cfg = ModelConfig.from_hf_dict({
        "model_type": "qwen3_5_text", "vocab_size": 256, "hidden_size": 2560, "intermediate_size": 9216,
        "num_hidden_layers": 1, "num_attention_heads": 16, "num_key_value_heads": 4, "head_dim": 256,
        "linear_num_key_heads": 16, "linear_num_value_heads": 32, "linear_key_head_dim": 128,
        "linear_value_head_dim": 128, "linear_conv_kernel_dim": 4, "layer_types": ["linear_attention"]})
    lay = GatedDeltaLayer(cfg, torch.bfloat16).cuda()
    with torch.no_grad():
        for n, p in lay.named_parameters():
            if p.dim() >= 2:
                p.normal_(0, 0.02)
            elif n == "A_log":
                p.copy_(torch.log(torch.empty_like(p, dtype=torch.float32).uniform_(1, 16)))
            else:
                p.fill_(1.0)
    os.environ["TRIDA_GDN"] = a.gdn_path
    if a.layout_gdn == "causal":
        T = a.length
        actx = SimpleNamespace(B=1, T=T, linear=LinearLayout("causal"))
    else:
        L, V = a.length, 2
        T = (1 + V) * L
        actx = SimpleNamespace(B=1, T=T, linear=LinearLayout("two_stream", L=L, V=V, bd=32))
    x = torch.randn(T, 2560, device="cuda", dtype=torch.bfloat16, requires_grad=backward)
    if not backward:
        with torch.no_grad():
            ms = _time(lambda: gdn_block_cuda(x, lay, actx, cfg), a.warmup, a.iters)
    else:
        dy = torch.randn(T, 2560, device="cuda", dtype=torch.bfloat16)
        ms = _time(lambda: gdn_block_cuda(x, lay, actx, cfg).backward(dy), a.warmup, a.iters)
    # recurrence FLOPs per token and value head: 3 (dk x dv) multiply-adds forward
    flops = T * 32 * 3 * 2 * 128 * 128 * (3 if backward else 1)
    return ms, {"recurrence_tflops": flops / ms / 1e9, "path": a.gdn_path, "layout": a.layout_gdn,
                "tokens": T}, None, None


def bench_gdn_core(a, backward):
    """The gated-delta core alone (chunk kernels: prep, local, scan, ...) on config-3 shapes: 16 key
    / 32 value heads of 128, a [x0 ; xt_1 ; xt_2] row of streams of ``--length`` (two-stream, block
    32) or one causal row."""
    from types import SimpleNamespace

    from ._ext import ext
    from .blocks import device_error_word
    from .gdn import LinearLayout
    from .gdn_cuda import chunk_forward
    Hk, Hv, D = 16, 32, 128
    if a.layout_gdn == "causal":
        T, lay = a.length, LinearLayout("causal")
    else:
        T, lay = 3 * a.length, LinearLayout("two_stream", L=a.length, V=2, bd=32)
    dev = "cuda"
    mixed = torch.randn(T, 2 * Hk * D + Hv * D, device=dev, dtype=torch.bfloat16)
    gates = torch.randn(T, 2 * Hv, device=dev, dtype=torch.bfloat16)
    ga, gb = gates[:, :Hv], gates[:, Hv:]
    A_log = torch.log(torch.empty(Hv, device=dev).uniform_(1, 16))
    dtb = torch.zeros(Hv, device=dev)
    scale = D ** -0.5
    o, saved = chunk_forward(mixed, ga, gb, A_log, dtb, None, 1, T, Hk, Hv, lay, scale)
    if not backward:
        ms = _time(lambda: chunk_forward(mixed, ga, gb, A_log, dtb, None, 1, T, Hk, Hv, lay, scale), a.warmup, a.iters)
    else:
        d_o = torch.randn_like(o)
        dmixed = torch.empty_like(mixed)
        dgates = torch.empty_like(gates)
        dA, ddt = torch.zeros(Hv, device=dev), torch.zeros(Hv, device=dev)
        err = device_error_word(mixed.device)
        ms = _time(lambda: ext().gdn_chunk_bwd(mixed, ga, gb, A_log, dtb, None, o, saved["bufs"], err, saved["geo"],
                                               scale, d_o, dmixed, dgates[:, :Hv], dgates[:, Hv:], dA, ddt),
                   a.warmup, a.iters)
    # chunk-form tensor-core FLOPs are layout dependent; report the recurrence-equivalent rate
    flops = T * Hv * 3 * 2 * D * D * (2 if backward else 1)
    return ms, {"recurrence_equiv_tflops": flops / ms / 1e9, "layout": a.layout_gdn, "tokens": T}, None, None


def bench_canvas(a, which):
    from ._ext import ext
    C = ext()
    B, blk = a.requests, a.blk
    dev = "cuda"
    if which in ("canvas_attn", "canvas_attn_tc"):
        Hq, Hkv, d, maxlen = 16, 4, 256, 1088
        kc = torch.randn(B, maxlen, Hkv, d, device=dev, dtype=torch.bfloat16)
        vc = torch.randn_like(kc)
        q = torch.randn(B * blk, Hq, d, device=dev, dtype=torch.bfloat16)
        out = torch.empty_like(q)
        slot = torch.arange(B, device=dev, dtype=torch.int32)
        pos = torch.full((B,), maxlen - blk, device=dev, dtype=torch.int32)
        err = None
        if which == "canvas_attn_tc":          # the tensor-core kernel runs when given the error word
            from .blocks import device_error_word
            err = device_error_word(torch.device(dev))
        ms = _time(lambda: C.canvas_attention(q, kc, vc, slot, pos, out, blk, (blk + 1) // 2, maxlen,
                                              1.0 / math.sqrt(d), None, err), a.warmup, a.iters)
        nbytes = 2 * B * maxlen * Hkv * d * 2
        return ms, {"gbs": nbytes / ms / 1e6}, None, nbytes
    Hk, Hv = 16, 32
    Cc = 2 * Hk * 128 + Hv * 128
    mixed = torch.randn(B * blk, Cc, device=dev, dtype=torch.bfloat16)
    proj = torch.randn(B * blk, 2 * Hv, device=dev, dtype=torch.bfloat16)
    ga, gb = proj[:, :Hv], proj[:, Hv:]
    al, dtb = torch.zeros(Hv, device=dev), torch.zeros(Hv, device=dev)
    ssm = torch.zeros(B, Hv, 128, 128, device=dev)
    o = torch.empty(B * blk, Hv * 128, device=dev, dtype=torch.bfloat16)
    slot = torch.arange(B, device=dev, dtype=torch.int32)
    nbytes = ssm.numel() * 4
    if which in ("canvas_gdn_tc", "commit_gdn_tc"):
        from .blocks import device_error_word
        err = device_error_word(dev)
        kbuf = torch.empty(B * blk, Hv, 128, device=dev, dtype=torch.bfloat16)
        ubuf, gbuf = torch.empty_like(kbuf), torch.empty(B * blk, Hv, device=dev)
        z = torch.randn(B * blk, Hv * 128, device=dev, dtype=torch.bfloat16)
        gw = torch.ones(128, device=dev, dtype=torch.bfloat16)

        def canvas():
            C.gdn_canvas_tc(mixed, ga, gb, al, dtb, o, kbuf, ubuf, gbuf, ssm, slot, blk, Hk, Hv, (blk + 1) // 2,
                            128 ** -0.5, err, z=z if a.fused_norm else None, gnorm_w=gw if a.fused_norm else None)
        canvas()
        if which == "canvas_gdn_tc":
            ms = _time(canvas, a.warmup, a.iters)
        else:
            adv = torch.full((B,), (blk + 1) // 2, device=dev, dtype=torch.int32)
            ms = _time(lambda: C.gdn_commit_tc(kbuf, ubuf, gbuf, ssm, slot, adv, blk, Hv, err), a.warmup, a.iters)
        return ms, {"state_gbs": nbytes / ms / 1e6, "fused_norm": bool(a.fused_norm)}, None, nbytes
    prep = torch.empty(C.gdn_prep_numel(B * blk, Hk, Hv), device=dev)
    ms = _time(lambda: C.gdn_canvas(mixed, ga, gb, al, dtb, o, prep, ssm, slot, blk, Hk, Hv, (blk + 1) // 2,
                                    128 ** -0.5), a.warmup, a.iters)
    return ms, {"state_gbs": nbytes / ms / 1e6}, None, nbytes


def bench_elementwise(a):
    """Bandwidth-bound kernels of a decoder layer on the config-2 shapes (Qwen3-4B: hidden 2560,
    32 / 8 heads x 128, ffn 9728); bytes are the algorithmic reads + writes of one launch."""
    from .blocks import rope_tables
    from ._ext import ext
    C = ext()
    M, D, F, Hq, Hkv, d = a.m, a.hidden, a.ffn, a.heads, a.kv_heads, 128
    bf = dict(device="cuda", dtype=torch.bfloat16)
    if a.op.startswith("rmsnorm"):
        x, w = torch.randn(M, D, **bf), torch.ones(D, **bf)
        y = torch.empty_like(x)
        _, rstd = C.rmsnorm_fwd(x, w, 1e-6, y)
        if a.op == "rmsnorm_fwd":
            return _time(lambda: C.rmsnorm_fwd(x, w, 1e-6, y), a.warmup, a.iters), {}, None, 2 * M * D * 2
        dy, dres, dx, dw = torch.randn_like(x), torch.randn_like(x), torch.empty_like(x), torch.zeros(D, device="cuda")
        return (_time(lambda: C.rmsnorm_bwd(dy, x, w, rstd, dres, dx, dw), a.warmup, a.iters), {}, None,
                4 * M * D * 2)
    if a.op.startswith("qk_rope"):
        qkv = torch.randn(M, (Hq + 2 * Hkv) * d, **bf)
        qw, kw = torch.ones(d, **bf), torch.ones(d, **bf)
        cos_t, sin_t = rope_tables(4096, d, 1e6, "cuda")
        pos = (torch.arange(M, device="cuda", dtype=torch.int32) % 4096).contiguous()
        q, k = torch.empty(M, Hq, d, **bf), torch.empty(M, Hkv, d, **bf)
        rstd = C.qk_norm_rope_fwd(qkv, qw, kw, cos_t, sin_t, pos, q, k, Hq, Hkv, d, d, 1e-6)
        qk_bytes = M * (Hq + Hkv) * d * 2
        if a.op == "qk_rope_fwd":
            return (_time(lambda: C.qk_norm_rope_fwd(qkv, qw, kw, cos_t, sin_t, pos, q, k, Hq, Hkv, d, d, 1e-6),
                          a.warmup, a.iters), {}, None, 2 * qk_bytes)
        dqkv = torch.empty_like(qkv)
        dqw, dkw = torch.zeros(d, device="cuda"), torch.zeros(d, device="cuda")
        return (_time(lambda: C.qk_norm_rope_bwd(q, k, qkv, qw, kw, cos_t, sin_t, pos, rstd, dqkv, dqw, dkw, Hq,
                                                 Hkv, d, d), a.warmup, a.iters), {}, None, 3 * qk_bytes)
    gu = torch.randn(M, 2 * F, **bf)
    act = torch.empty(M, F, **bf)
    if a.op == "swiglu_fwd":
        return _time(lambda: C.swiglu_fwd(gu, act), a.warmup, a.iters), {}, None, 3 * M * F * 2
    dgu = torch.empty_like(gu)
    return _time(lambda: C.swiglu_bwd(act, gu, dgu), a.warmup, a.iters), {}, None, 5 * M * F * 2


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--op", required=True,
                    choices=["gemm", "gemm_swiglu", "attn_fwd", "attn_bwd", "gdn_fwd", "gdn_bwd", "gdn_core_fwd", "gdn_core_bwd",
                             "canvas_attn", "canvas_attn_tc", "canvas_gdn", "canvas_gdn_tc", "commit_gdn_tc",
                             "rmsnorm_fwd", "rmsnorm_bwd", "qk_rope_fwd", "qk_rope_bwd", "swiglu_fwd", "swiglu_bwd"])
    ap.add_argument("--m", type=int, default=24576)
    ap.add_argument("--n", type=int, default=6144)
    ap.add_argument("--k", type=int, default=2560)
    ap.add_argument("--layout", default="tn", choices=["tn", "tt", "nt"])
    ap.add_argument("--tile", type=int, default=0)
    ap.add_argument("--hidden", type=int, default=2560)
    ap.add_argument("--ffn", type=int, default=9728)
    ap.add_argument("--heads", type=int, default=32)
    ap.add_argument("--kv-heads", type=int, default=8)
    ap.add_argument("--head-dim", dest="head_dim", type=int, default=128, help="attention head dim (64 / 128 / 256)")
    ap.add_argument("--rows", type=int, default=4, help="attention: forward rows (2 views x micro-batch)")
    ap.add_argument("--length", type=int, default=3072, help="gated delta: stream length L")
    ap.add_argument("--gdn-path", dest="gdn_path", default="chunk", choices=["chunk", "scan"],
                    help="gated delta sub-block: chunked tcgen05 kernels or the per-token scan")
    ap.add_argument("--gdn-layout", dest="layout_gdn", default="two_stream", choices=["two_stream", "causal"])
    ap.add_argument("--requests", type=int, default=64)
    ap.add_argument("--blk", type=int, default=7)
    ap.add_argument("--fused-norm", dest="fused_norm", type=int, default=1, help="canvas_gdn_tc: 1 fuses the gated norm")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=10)
    a = ap.parse_args()
    if a.op in ("gemm", "gemm_swiglu"):
        ms, extra, flops, nbytes = bench_gemm(a)
    elif a.op.startswith("attn"):
        ms, extra, flops, nbytes = bench_attn(a, a.op == "attn_bwd")
    elif a.op.startswith("gdn_core"):
        ms, extra, flops, nbytes = bench_gdn_core(a, a.op == "gdn_core_bwd")
    elif a.op.startswith("gdn"):
        ms, extra, flops, nbytes = bench_gdn(a, a.op == "gdn_bwd")
    elif a.op.split("_")[0] in ("rmsnorm", "qk", "swiglu"):
        ms, extra, flops, nbytes = bench_elementwise(a)
        extra = {"gbs": nbytes / ms / 1e6}
    else:
        ms, extra, flops, nbytes = bench_canvas(a, a.op)
    pk = _peaks()
    out = {"op": a.op, "ms": round(ms, 4), **{k: (round(v, 2) if isinstance(v, float) else v) for k, v in extra.items()}}
    if flops and pk.get("bf16_tflops"):
        out["frac_of_measured_bf16"] = round(flops / ms / 1e9 / pk["bf16_tflops"], 3)
    if nbytes and pk.get("hbm_gbs"):
        out["frac_of_measured_hbm"] = round(nbytes / ms / 1e6 / pk["hbm_gbs"], 3)
    print(json.dumps(out))


if __name__ == "__main__":
    main()
