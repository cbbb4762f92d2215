"""Fused peer-memory collectives against the NVLink roofline, next to their NCCL counterparts.

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \\
        -m trida_stack_b200.parallel.collective_bench [--rows 4032] [--hidden 2560] [--params 100663296]

One JSON line per operation (rank 0): device time per call (CUDA events around ``--iters`` calls
after warm-up, max over ranks), the bytes one rank must move over NVLink in one direction, and the
achieved fraction of the link: roofline time = those bytes / 770 GB/s (the measured per-direction
peer-copy bandwidth of this pool; 900 GB/s nominal).  Operations and their per-rank bytes (N ranks):

- ``sp_rs_norm_ag``: tensor-parallel sequence-parallel boundary (``csrc/symm.cu``: reduce-scatter of
  the row-parallel partials + residual + RMSNorm + all-gather in one kernel), [rows, hidden] bf16:
  (N-1)/N x rows x hidden x 2 B in and the same out.
- ``oneshot_allreduce``: the replicated-residual all-reduce kernel: every peer's whole buffer is read,
  (N-1) x rows x hidden x 2 B in.
- ``rs_sumsq``: gradient reduce-scatter fused with the squared-norm partials, fp32 [params]:
  (N-1)/N x params x 4 B in.
- ``adamw_ag``: sharded AdamW fused with the bf16 parameter all-gather: (N-1)/N x params x 2 B out.
- ``gather_copy`` / ``gather_kernel``: the full-shard layer gather (copy engines / P2P kernel):
  (N-1)/N x params x 2 B in.
- ``nccl_*``: ``all_reduce`` / ``reduce_scatter_tensor`` / ``all_gather_into_tensor`` on the same
  sizes, bytes counted as the algorithm's per-rank traffic (ring: 2 (N-1)/N x S for the all-reduce).
"""
import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist

LINK_GBS = 770.0


def _time(fn, warmup, iters):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    ms = torch.tensor([s.elapsed_time(e) / iters], device="cuda")
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    return ms.item()


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--rows", type=int, default=4032, help="tensor-parallel rows (64 requests x 63-row canvases)")
    ap.add_argument("--hidden", type=int, default=2560)
    ap.add_argument("--params", type=int, default=100663296, help="flat parameters of one layer group")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args()
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    rank, world = dist.get_rank(), dist.get_world_size()
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    from ..ops._ext import ext
    from ..serve.tp import TPContext
    from .symm import SymmetricHeap
    C = ext()
    out = []

    def report(op, ms, nbytes, note):
        gbs = nbytes / (ms / 1e3) / 1e9
        out.append({"op": op, "ranks": world, "ms": round(ms, 4), "bytes_per_rank": int(nbytes),
                    "gbs": round(gbs, 1), "frac_of_link": round(gbs / LINK_GBS, 3), "note": note})

    M, H, N = args.rows, args.hidden, world
    # ---- tensor-parallel boundary: sequence-parallel kernel and the one-shot all-reduce ----
    tp = TPContext(max_rows=M, hidden=H, seq_parallel=True)
    part = tp.part.local[:M * H].view(M, H)
    part.copy_(torch.randn(M, H, device="cuda").to(torch.bfloat16))
    r0, n = tp.own_rows(M)
    xs = torch.randn(n, H, device="cuda").to(torch.bfloat16)
    norm_w = torch.ones(H, device="cuda", dtype=torch.bfloat16)

    def sp():
        C.symm_rs_norm_ag(tp.part.ptrs, tp.gath.ptrs, tp.heap.flags.ptrs, tp.rank, tp.sp_ctr, r0, xs, norm_w, 1e-6,
                          tp.heap.err)
    report("sp_rs_norm_ag", _time(sp, args.warmup, args.iters), (N - 1) / N * M * H * 2,
           f"[{M}, {H}] bf16, reduce-scatter + residual + RMSNorm + all-gather")
    res = torch.zeros(M, H, device="cuda", dtype=torch.bfloat16)
    for _ in range(2):                           # fill both buffers the calls alternate between
        _, view = tp.next_buffer(M)
        view.copy_(part)

    def oneshot():
        b, _ = tp.next_buffer(M)
        tp.allreduce(b, M, res)
    report("oneshot_allreduce", _time(oneshot, args.warmup, args.iters), (N - 1) * M * H * 2,
           f"[{M}, {H}] bf16 + residual")
    x = part.clone()
    report("nccl_all_reduce", _time(lambda: dist.all_reduce(x), args.warmup, args.iters),
           2 * (N - 1) / N * M * H * 2, f"[{M}, {H}] bf16")
    tp.heap.check()
    tp.heap.close()

    # ---- data-parallel optimizer traffic: one layer group of --params parameters ----
    P = args.params - args.params % (64 * N)
    shard = P // N
    heap = SymmetricHeap()
    grad = heap.alloc(P, torch.float32)
    grad.local.normal_()
    partials = heap.alloc(296, torch.float32)
    gshard = torch.empty(shard, device="cuda")

    def rs():
        C.symm_rs_sumsq(grad.ptrs, heap.flags.ptrs, heap.rank, heap.next_epoch(1), rank * shard, shard, 1.0 / N,
                        gshard, partials.local, heap.err)
    report("rs_sumsq", _time(rs, args.warmup, args.iters), (N - 1) / N * P * 4,
           f"fp32 [{P}] gradient reduce-scatter + squared-norm partials")
    params = heap.alloc(P, torch.bfloat16)
    params.local.zero_()
    m, v = torch.zeros(shard, device="cuda"), torch.zeros(shard, device="cuda")
    step = [0]

    def adamw():
        step[0] += 1
        C.symm_adamw_ag(params.ptrs, heap.flags.ptrs, heap.rank, heap.next_epoch(2), rank * shard, shard, gshard, None,
                        m, v, 1e-5, 0.9, 0.95, 1e-8, 0.0, step[0], None, heap.done, heap.err)
    report("adamw_ag", _time(adamw, args.warmup, args.iters), (N - 1) / N * P * 2,
           f"AdamW on a [{shard}] shard + bf16 all-gather of [{P}]")
    sh = heap.alloc(shard, torch.bfloat16)
    sh.local.normal_()
    dst = torch.empty(P, device="cuda", dtype=torch.bfloat16)
    report("gather_copy", _time(lambda: C.symm_gather_copy(sh.ptrs, rank, shard, dst), args.warmup, args.iters),
           (N - 1) / N * P * 2, f"bf16 [{P}] layer gather, one peer copy per shard (copy engines)")
    ref = dst.clone()
    dst.zero_()
    report("gather_kernel", _time(lambda: C.symm_gather(sh.ptrs, rank, shard, dst, 32), args.warmup, args.iters),
           (N - 1) / N * P * 2, f"bf16 [{P}] layer gather, P2P-load kernel (32 CTAs)")
    if not torch.equal(dst, ref):
        raise RuntimeError("the P2P gather kernel and the copy-engine gather disagree")
    del ref
    g = grad.local.clone()
    report("nccl_reduce_scatter", _time(lambda: dist.reduce_scatter_tensor(gshard, g), args.warmup, args.iters),
           (N - 1) / N * P * 4, f"fp32 [{P}]")
    report("nccl_all_gather", _time(lambda: dist.all_gather_into_tensor(dst, sh.local), args.warmup, args.iters),
           (N - 1) / N * P * 2, f"bf16 [{P}]")
    heap.check()
    torch.cuda.synchronize()
    del g
    heap.close()
    if rank == 0:
        for line in out:
            print(json.dumps(line), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
