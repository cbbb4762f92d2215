"""All-reduce bandwidth probe (the reference's ``train/tools/draftalign/nccl_probe.py``).

    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 -m trida_stack_b200.parallel.probe

Times a 256 MB fp32 all-reduce with CUDA events (max over ranks) and prints the bus bandwidth
(2 (n - 1) / n x bytes / time).
"""
import datetime
import os

import torch
import torch.distributed as dist


def main(mb=256, iters=5):
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    r, n = dist.get_rank(), dist.get_world_size()
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", r)))
    x = torch.ones(mb * 1024 * 1024 // 4, device="cuda")
    dist.all_reduce(x)
    torch.cuda.synchronize()
    dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        dist.all_reduce(x)
    e.record()
    torch.cuda.synchronize()
    ms = torch.tensor([s.elapsed_time(e) / iters], device="cuda")
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    if r == 0:
        gbs = 2 * (n - 1) / n * x.numel() * 4 / (ms.item() / 1e3) / 1e9
        print(f"PROBE_OK allreduce {mb}MB x{n} ranks: {ms.item():.2f} ms/iter (~{gbs:.1f} GB/s bus)", flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
