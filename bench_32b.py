"""Qwen3-32B block-diffusion SFT benchmark (config 5 of the reference's headline metric).

Model: Qwen3-32B architecture (64 layers, hidden 5120, 64 Q / 8 KV heads x 128, SwiGLU 25600,
vocab 151936, tied embeddings off), random init, bf16.  Rows [prompt 4096 | response 2048] as the
block-diffusion layout [S 4096 | x_t 2048 | x_0 2048] (8192 tokens, two complementary views),
block size 64, micro-batch 1 per GPU, per-layer activation checkpointing.  Memory: bf16 weights
stay resident on every GPU (64 GB); fp32 gradients are streamed layer by layer through a two-slot
ring and reduce-scattered into each rank's shard as soon as the layer's backward ends; AdamW
moments exist for the local shard only -- about 122 GB per GPU at 8 GPUs (fewer GPUs do not fit).
Launch with torchrun (one rank per GPU); prints one JSON line (tokens/s counted as input rows,
max over ranks of the device-timed steps).

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 bench_32b.py --gpus 8 --steps 2 --warmup 3
"""
import argparse
import datetime
import json
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
PROMPT, RESP, BD, MB, VOCAB = 4096, 2048, 64, 1, 151936


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=8)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--layers", type=int, default=64, help="debug only: fewer layers (reported as reduced)")
    ap.add_argument("--comm", choices=["fused", "nccl"], default="fused")
    ap.add_argument("--shard", choices=["full", "stream"], default="stream",
                    help="full: decoder-layer bf16 weights sharded and gathered per layer (FSDP full shard; fits 4 "
                         "GPUs); stream: bf16 weights resident, fp32 gradients streamed per layer (8 GPUs)")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    from trida_stack_b200.engine import TrainEngine
    from trida_stack_b200.models import BlockDiffusionLM, Decoder, qwen3_config
    from trida_stack_b200.ops._ext import ext
    ext()
    cfg = qwen3_config(vocab_size=VOCAB, hidden_size=5120, intermediate_size=25600, num_layers=args.layers,
                       n_heads=64, n_kv_heads=8, head_dim=128, tie_embeddings=False)
    torch.manual_seed(0)
    dec = Decoder(cfg, dtype=torch.bfloat16, device="cuda")
    model = BlockDiffusionLM(dec, mask_id=VOCAB - 1, pad_id=VOCAB - 2, bd_size=BD, ar_loss_weight=1.0,
                             activation_checkpoint="layer")
    model.train()
    full = args.shard == "full" and world > 1
    engine = TrainEngine(model, lr=1e-5, warmup=50, max_steps=2000, device=torch.device("cuda"), comm=args.comm,
                         grad_stream=True, full_shard=full)
    g = torch.Generator().manual_seed(1234 + rank)
    batches = []
    for _ in range(args.warmup + args.steps):
        ids = torch.randint(0, VOCAB - 2, (MB, PROMPT + RESP), generator=g)
        labels = ids.clone()
        labels[:, :PROMPT] = -100
        batches.append({"input_ids": ids.cuda(), "labels": labels.cuda(), "attention_mask": torch.ones_like(ids).cuda()})
    from trida_stack_b200.engine import host_rpad
    rpad = host_rpad(batches[0]["labels"].cpu(), BD, model.response_buckets)
    for i in range(args.warmup):
        engine.micro_step(batches[i], rpad=rpad)
        engine.optimizer_step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for i in range(args.warmup, args.warmup + args.steps):
        engine.micro_step(batches[i], rpad=rpad)
        engine.optimizer_step(i)
    t1.record()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1) / args.steps
    peak = torch.cuda.max_memory_allocated() / 1e9
    if world > 1:
        t = torch.tensor([ms, peak], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, peak = t.tolist()
        if engine.optim.heap is not None:
            engine.optim.heap.check()
        dist.barrier()
    if rank == 0:
        toks = world * MB * (PROMPT + RESP)
        print(json.dumps({
            "metric": "32B block-diffusion SFT tokens/s", "value": round(toks / (ms / 1e3), 1), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 1),
            "higher_is_better": True, "scaling": "weak", "dtype": "bf16",
            "data": "synthetic uniform token ids, random-init weights", "peak_mem_gb_max_rank": round(peak, 1),
            "config": {"model": "Qwen3-32B architecture (64L, d5120, 64/8 heads x128, ffn 25600, vocab 151936)"
                       + ("" if args.layers == 64 else f" REDUCED to {args.layers} layers (not a valid bench)"),
                       "row": "[S 4096 | x_t 2048 | x_0 2048] x 2 views", "micro_batch": MB, "bd_size": BD,
                       "activation_checkpoint": "layer",
                       "parallelism": f"dp{world}, " + ("bf16 weight shards gathered per layer over NVLink, "
                                                         if full else "bf16 weights resident, ")
                                      + f"fp32 gradients streamed per layer and reduce-scattered ({args.comm}), "
                                        f"sharded AdamW"}}), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
