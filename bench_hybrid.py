"""Hybrid two-stream block-diffusion SFT benchmark (config 3 of the reference's headline metric).

Model: Qwen3.5-4B-style hybrid (32 layers: 3 gated-delta then 1 full attention, hidden 2560, FFN
9216, vocab 248320, full layers 16 Q / 4 KV x 256 with output gate and partial RoPE, gated-delta
16 key / 32 value heads x 128, conv 4), random init, bf16.  Rows [prompt 2048 | response 1024]
run as the two-stream layout [x0 ; xt_1 ; xt_2] (9216 forward tokens per row), block size 32,
diffusion + AR loss; joint training with the typed-decision pointer head: every 4th step adds a
decision micro-step (a packed causal row of 2-4-option questions, loss weight 0.5).  Synthetic
uniform tokens.  Launch like ``bench.py`` (torchrun for N > 1); prints one JSON line.

    python bench_hybrid.py --steps 4 --warmup 3 [--mb 1] [--layers 32]
"""
import argparse
import json
import os
import sys
import time

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PROMPT, RESP, BD, VOCAB = 2048, 1024, 32, 248320


def hybrid_cfg(layers):
    from trida_stack_b200.models.config import ModelConfig
    return ModelConfig.from_hf_dict({
        "model_type": "qwen3_5_text", "vocab_size": VOCAB, "hidden_size": 2560, "intermediate_size": 9216,
        "num_hidden_layers": layers, "num_attention_heads": 16, "num_key_value_heads": 4, "head_dim": 256,
        "linear_num_key_heads": 16, "linear_num_value_heads": 32, "linear_key_head_dim": 128,
        "linear_value_head_dim": 128, "linear_conv_kernel_dim": 4, "partial_rotary_factor": 0.25,
        "rope_theta": 1e7, "layer_types": (["linear_attention"] * 3 + ["full_attention"]) * (layers // 4),
        "tie_word_embeddings": True, "rms_norm_eps": 1e-6})


def decision_batch(g, n_q=8, state=600):
    """A packed causal row of n_q questions (2-4 options) over one random state."""
    ids, seg, decide, opts, owner, questions = [], [], [], [], [], []
    for qi in range(n_q):
        k = int(torch.randint(2, 5, (1,), generator=g))
        base = len(ids)
        row = torch.randint(0, VOCAB - 8, (state,), generator=g).tolist()
        ends = []
        for _ in range(k):
            row += torch.randint(0, VOCAB - 8, (12,), generator=g).tolist()
            ends.append(len(row) - 1)
        row.append(VOCAB - 3)
        ids += row
        seg += [qi] * len(row)
        decide.append(base + len(row) - 1)
        questions.append({"start": len(opts), "k": k, "label": int(torch.randint(0, k, (1,), generator=g)),
                          "variant": qi})
        opts += [base + e for e in ends]
        owner += [qi] * k
    return {"input_ids": torch.tensor([ids]), "seg_id": torch.tensor([seg]), "decide": torch.tensor(decide),
            "opts": torch.tensor(opts), "owner": torch.tensor(owner), "questions": questions}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=4)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--mb", type=int, default=1)
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--comm", choices=["fused", "nccl"], default="fused")
    ap.add_argument("--kernel-breakdown", type=int, default=0, metavar="STEPS",
                    help="after the timed steps, print the per-kernel device-time table of STEPS more steps "
                         "(taken under the PyTorch profiler; not a benchmark number)")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    from trida_stack_b200.engine import TrainEngine
    from trida_stack_b200.models import Decoder
    from trida_stack_b200.models.hybrid import HybridBlockDiffusionLM
    from trida_stack_b200.ops._ext import ext
    ext()
    torch.manual_seed(0)
    dec = Decoder(hybrid_cfg(args.layers), dtype=torch.bfloat16, device="cuda")
    model = HybridBlockDiffusionLM(dec, mask_id=VOCAB - 1, pad_id=VOCAB - 2, bd_size=BD, ar_loss_weight=1.0,
                                   decision_head_dim=256)
    model.train()
    engine = TrainEngine(model, lr=1e-5, warmup=50, max_steps=2000, device=torch.device("cuda"), comm=args.comm)
    g = torch.Generator().manual_seed(1234 + rank)
    batches, dec_batches = [], []
    for _ in range(args.warmup + args.steps):
        ids = torch.randint(0, VOCAB - 8, (args.mb, PROMPT + RESP), generator=g)
        labels = ids.clone()
        labels[:, :PROMPT] = -100
        batches.append({"input_ids": ids.cuda(), "labels": labels.cuda(), "attention_mask": torch.ones_like(ids).cuda()})
        dec_batches.append({k: (v.cuda() if torch.is_tensor(v) else v) for k, v in decision_batch(g).items()})

    def step_fn(i, step):
        engine.micro_step(batches[i])
        if i % 4 == 3:           # 25% of steps add a decision micro-step (weight 0.5)
            loss, _ = model(None, None, None, decision=dec_batches[i])
            (0.5 * loss).backward()
        engine.optimizer_step(step)

    for i in range(args.warmup):
        step_fn(i, i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for i in range(args.warmup, args.warmup + args.steps):
        step_fn(i, i)
    t1.record()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
        dist.barrier()
    if rank == 0:
        toks = world * args.mb * (PROMPT + RESP)
        print(json.dumps({
            "metric": "4B hybrid two-stream block-diffusion SFT tokens/s", "value": round(toks / (ms / 1e3), 1),
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 2), "higher_is_better": True, "scaling": "weak", "dtype": "bf16",
            "data": "synthetic uniform token ids, random-init weights",
            "peak_mem_gb": round(torch.cuda.max_memory_allocated() / 1e9, 1),
            "config": {"model": f"Qwen3.5-4B-style hybrid ({args.layers}L)", "micro_batch": args.mb,
                       "row": "[prompt 2048 | response 1024] as [x0 ; xt_1 ; xt_2] (9216 forward tokens)",
                       "bd_size": BD, "decision": "pointer head, every 4th step, weight 0.5",
                       "parallelism": f"dp{world}"}}), flush=True)
    if args.kernel_breakdown > 0 and rank == 0 and world == 1:
        from trida_stack_b200.utils.trace import kernel_breakdown
        i0 = args.warmup + args.steps
        extra = iter(range(args.kernel_breakdown))

        def one():
            j = next(extra)
            engine.micro_step(batches[(i0 + j) % len(batches)])
            engine.optimizer_step(i0 + j)
        kernel_breakdown(one, args.kernel_breakdown)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
