"""Self-speculative serving benchmark (the serving config of the reference's headline metric).

Model: Qwen3.5-4B-style hybrid (32 layers, 3 gated-delta : 1 full attention, hidden 2560, FFN 9216,
vocab 248320, full layers 16 Q / 4 KV x 256 with the output gate and partial RoPE, gated-delta
16 key / 32 value heads x 128, conv 4), random init, bf16.  Load: ``--requests`` concurrent
requests of ``--prompt`` uniform random tokens each, ``--max-new`` output tokens each, greedy.
Decoding: self-speculative with ``--gen-block`` (N) causal rows per canvas (canvas of 2N-1 rows), or
``--mode causal``.

Reports (one JSON line): decode tokens/s (all generated tokens / device-timed decode phase),
tokens per forward, p50 TTFT, and the device-timed prefill.  Random weights make the drafts
nearly never match, so tokens per forward stays near its floor of 1 (the reference's ~2.3 is a
trained-checkpoint figure); the throughput per forward is what the kernels determine.

    python bench_serve.py [--requests 64 --prompt 512 --max-new 512 --gen-block 16 --layers 32 --tp 1]
"""
import argparse
import json
import os
import sys
import time

import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))


def hybrid_config(layers):
    from trida_stack_b200.models.config import ModelConfig
    return ModelConfig.from_hf_dict({
        "model_type": "qwen3_5_text", "vocab_size": 248320, "hidden_size": 2560, "intermediate_size": 9216,
        "num_hidden_layers": layers, "num_attention_heads": 16, "num_key_value_heads": 4, "head_dim": 256,
        "linear_num_key_heads": 16, "linear_num_value_heads": 32, "linear_key_head_dim": 128,
        "linear_value_head_dim": 128, "linear_conv_kernel_dim": 4, "partial_rotary_factor": 0.25,
        "rope_theta": 1e7, "layer_types": (["linear_attention"] * 3 + ["full_attention"]) * (layers // 4),
        "tie_word_embeddings": True, "rms_norm_eps": 1e-6})


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--requests", type=int, default=64)
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--max-new", type=int, default=512)
    ap.add_argument("--gen-block", type=int, default=16, help="N: causal rows per canvas (canvas = 2N-1 rows)")
    ap.add_argument("--mode", default="self-spec", choices=["self-spec", "causal", "diffusion"])
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-graphs", action="store_true", help="launch every kernel eagerly (no CUDA graphs)")
    ap.add_argument("--tp", type=int, default=1, help="tensor-parallel ranks (launch with torchrun)")
    ap.add_argument("--kernel-breakdown", type=int, default=0, metavar="STEPS",
                    help="after the timed run, print the per-kernel device-time table of STEPS eager decode "
                         "steps of a fresh batch (taken under the PyTorch profiler; not a benchmark number)")
    ap.add_argument("--tp-fused", action="store_true",
                    help="TP all-reduce in the GEMM epilogue instead of a separate kernel after the GEMM")
    ap.add_argument("--tp-allreduce", action="store_true",
                    help="replicated residual with a one-shot all-reduce kernel after each row-parallel GEMM "
                         "instead of the sequence-parallel reduce-scatter + norm + all-gather kernel")
    args = ap.parse_args()

    from trida_stack_b200.models import Decoder
    from trida_stack_b200.serve import Engine, Runtime, SamplingParams
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    tp = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", torch.cuda.current_device()))
    if world != args.tp:
        raise SystemExit(f"--tp {args.tp} but WORLD_SIZE={world}")
    torch.manual_seed(args.seed)
    cfg = hybrid_config(args.layers)
    dec = Decoder(cfg, dtype=torch.bfloat16, device="cuda")
    mask_id = cfg.vocab_size - 1
    max_len = args.prompt + args.max_new + 2 * args.gen_block + 8
    if world > 1:
        from trida_stack_b200.serve.tp import TPContext, shard_decoder
        dec = shard_decoder(dec, rank, world)
        torch.cuda.empty_cache()
        tp = TPContext(max_rows=args.requests * 64, hidden=cfg.hidden_size, fused=args.tp_fused,
                        seq_parallel=not args.tp_allreduce)
    rt = Runtime(dec, max_slots=args.requests, max_len=max_len, tp=tp)
    eng = Engine(rt, mask_id=mask_id, mode=args.mode, n=args.gen_block, max_running=args.requests, graphs=not args.no_graphs)
    g = torch.Generator().manual_seed(args.seed)

    def prompts(k):
        return [torch.randint(0, cfg.vocab_size - 2, (args.prompt,), generator=g).tolist() for _ in range(k)]

    # warm-up: a short run at the full batch (captures the decode graph of that batch size)
    eng.generate(prompts(args.requests), max_new_tokens=6)
    torch.cuda.synchronize()

    reqs = [eng.submit(__import__("trida_stack_b200.serve", fromlist=["Request"]).Request(
        p, args.max_new, SamplingParams(temperature=0.0))) for p in prompts(args.requests)]
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    from bench import ClockSampler, physical_gpu_index
    clocks = ClockSampler(physical_gpu_index(int(os.environ.get("LOCAL_RANK", "0"))))
    clocks.start()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ev[0].record()
    eng._admit()                       # batched prefill of all requests
    ev[1].record()
    f0 = eng.stats["forwards"]
    while eng.running:
        eng._decode()
    ev[2].record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    clk = clocks.stop()
    prefill_ms = ev[0].elapsed_time(ev[1])
    decode_ms = ev[1].elapsed_time(ev[2])
    if world > 1:      # device time, max over ranks
        t = torch.tensor([prefill_ms, decode_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        prefill_ms, decode_ms = t.tolist()
        tp.heap.check()
    toks = sum(len(r.output) for r in reqs)
    s = eng.summary(reqs)
    steps = eng.stats["forwards"] - f0
    if rank != 0:
        _finish(rt, world)
        return
    print(json.dumps({
        "metric": "self-spec decode tokens/s", "value": round(toks / (decode_ms / 1e3), 1), "unit": "tokens/s",
        "tokens_per_forward": round(s["tokens_per_forward"], 3), "p50_ttft_ms": round(s["p50_ttft_s"] * 1e3, 2),
        "prefill_ms": round(prefill_ms, 2), "decode_ms": round(decode_ms, 2), "decode_steps": steps,
        "ms_per_step": round(decode_ms / max(steps, 1), 3), "wall_s": round(wall, 2), "tp": world, "clocks": clk,
        "config": {"model": f"Qwen3.5-4B-style hybrid ({args.layers}L)", "requests": args.requests,
                   "prompt": args.prompt, "max_new": args.max_new, "mode": args.mode, "n": args.gen_block,
                   "canvas_rows": 2 * args.gen_block - 1 if args.mode == "self-spec" else 1, "greedy": True,
                   "cuda_graphs": not args.no_graphs,
                   "tp_collective": ("all-reduce fused into the GEMM epilogue" if args.tp_fused else
                                     "one-shot all-reduce kernel" if args.tp_allreduce else
                                     "sequence-parallel reduce-scatter + RMSNorm + all-gather kernel")
                   if world > 1 else None},
        "data": "synthetic uniform prompts, random-init weights", "dtype": "bf16"}), flush=True)
    if args.kernel_breakdown > 0 and world == 1:
        from trida_stack_b200.utils.trace import kernel_breakdown
        for p in prompts(args.requests):
            eng.submit(__import__("trida_stack_b200.serve", fromlist=["Request"]).Request(
                p, args.kernel_breakdown + 2, SamplingParams(temperature=0.0)))
        eng._admit()
        eng._decode()
        kernel_breakdown(eng._decode, args.kernel_breakdown)
    _finish(rt, world)


def _finish(rt, world):
    if world > 1:
        import torch.distributed as dist
        rt._graphs = None          # graphs holding NCCL calls go before the process group
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
