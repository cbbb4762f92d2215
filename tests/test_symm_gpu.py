"""Symmetric peer-memory collectives (csrc/symm.cu) vs NCCL on 2 GPUs (skipped with fewer)."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from trida_stack_b200.parallel.symm import SymmetricHeap
        from trida_stack_b200.parallel.zero import ShardedAdamW
        heap = SymmetricHeap()
        # one-shot all-reduce (two halves, alternating) vs NCCL
        n = 4096
        buf = heap.alloc(2 * n, torch.bfloat16)
        errs = []
        for it in range(4):
            x = torch.randn(n, device="cuda", dtype=torch.bfloat16, generator=torch.Generator("cuda").manual_seed(
                100 * it + rank))
            res = torch.randn(n, device="cuda", dtype=torch.bfloat16)
            off = (it % 2) * n
            buf.local[off:off + n].copy_(x)
            out = torch.empty(n, device="cuda", dtype=torch.bfloat16)
            heap.allreduce_(buf, off, n, out, res)
            ref = x.float().clone()
            dist.all_reduce(ref)
            errs.append(((out.float() - (ref + res.float())).abs().max() / (ref.abs().max() + 1e-6)).item())
        heap.check()
        # fused reduce-scatter + norm + AdamW + all-gather vs the NCCL optimizer path
        torch.manual_seed(0)
        base = [torch.randn(1000, 64), torch.randn(333), torch.randn(77, 5)]
        outs = {}
        for comm in ("nccl", "fused"):
            params = [torch.nn.Parameter(b.clone().to("cuda", torch.bfloat16)) for b in base]
            opt = ShardedAdamW([{"params": params}], lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1, comm=comm)
            for step in range(3):
                opt.zero_grad()
                g = torch.Generator().manual_seed(1000 * step + 7 * rank)
                for p in params:
                    p.main_grad.copy_(torch.randn(p.shape, generator=g))
                opt.reduce_gradients()
                opt.clip_grad_norm_(1.0)
                opt.step()
            torch.cuda.synchronize()
            outs[comm] = [p.detach().float().cpu() for p in params]
            if comm == "fused":
                opt.heap.check()
        perr = max(((a - b).abs().max() / (b.abs().max() + 1e-6)).item() for a, b in zip(outs["fused"], outs["nccl"]))
        # streamed per-layer gradients through the ring (fused and NCCL reduce) vs resident buffers
        for comm in ("nccl", "fused"):
            params = [torch.nn.Parameter(b_.clone().to("cuda", torch.bfloat16)) for b_ in base]
            groups = [{"params": [params[0]], "stream": True, "layer": 0},
                      {"params": [params[1]], "stream": True, "layer": 1}, {"params": [params[2]]}]
            opt = ShardedAdamW(groups, lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1, comm=comm)
            for step in range(3):
                opt.zero_grad()
                g = torch.Generator().manual_seed(1000 * step + 7 * rank)
                grads = [torch.randn(p_.shape, generator=g) for p_ in params]
                for li in (1, 0):                     # backward order: last layer first
                    opt.layer_stream.acquire(li)
                    params[li].main_grad.copy_(grads[li])
                    opt.layer_stream.release(li)
                params[2].main_grad.copy_(grads[2])
                opt.reduce_gradients()
                opt.clip_grad_norm_(1.0)
                opt.step()
            torch.cuda.synchronize()
            serr = max(((p_.detach().float().cpu() - r).abs().max() / (r.abs().max() + 1e-6)).item()
                       for p_, r in zip(params, outs["nccl"]))
            perr = max(perr, serr)
        q.put((rank, max(errs), perr))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_symmetric_collectives_match_nccl():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    res = [q.get(timeout=5) for _ in range(2)]
    for rank, ar_err, opt_err in res:
        assert ar_err < 2e-2, (rank, ar_err)
        assert opt_err < 2e-2, (rank, opt_err)
    assert all(p.exitcode == 0 for p in procs)


def _fused_worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from trida_stack_b200.serve.tp import TPContext
        tp = TPContext(max_rows=1200, hidden=2560, fused=True)
        assert tp.fused
        errs = []
        g = torch.Generator("cuda").manual_seed(10 + rank)
        for M, K in ((70, 512), (448, 512), (1100, 512), (448, 4608), (448, 512)):   # split K and whole tiles
            x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16, generator=g)
            w = torch.randn(2560, K, device="cuda", dtype=torch.bfloat16, generator=g) * 0.05
            res = torch.randn(M, 2560, device="cuda", dtype=torch.bfloat16)
            dist.broadcast(res, 0)
            out = tp.row_parallel(x, w, res)
            ref = (x.float() @ w.float().t()).to(torch.bfloat16).float()
            dist.all_reduce(ref)
            ref += res.float()
            errs.append(((out.float() - ref).abs().max() / ref.abs().max()).item())
        # replayed from a CUDA graph: the call counter (and buffer parity) lives on the device
        x = torch.randn(448, 512, device="cuda", dtype=torch.bfloat16, generator=g)
        w = torch.randn(2560, 512, device="cuda", dtype=torch.bfloat16, generator=g) * 0.05
        res = torch.zeros(448, 2560, device="cuda", dtype=torch.bfloat16)
        ref = (x.float() @ w.float().t()).to(torch.bfloat16).float()
        dist.all_reduce(ref)
        torch.cuda.synchronize()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=s):
                o1 = tp.row_parallel(x, w, res)
                o2 = tp.row_parallel(x, w, o1)
        for _ in range(3):
            gr.replay()
            torch.cuda.synchronize()
            errs.append(((o2.float() - 2 * ref).abs().max() / (2 * ref).abs().max()).item())
        del gr
        from trida_stack_b200.ops._ext import ext
        assert int(ext().gemm_error()) == 0
        q.put((rank, max(errs)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_gemm_allreduce_matches_nccl():
    """Row-parallel GEMM with the all-reduce in its epilogue (pushes over NVLink, per-tile arrival
    counters) vs GEMM + NCCL all-reduce, eager and replayed from a CUDA graph, on 2 GPUs."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_fused_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    res = [q.get(timeout=5) for _ in range(2)]
    for rank, err in res:
        assert err < 2e-2, (rank, err)
    assert all(p.exitcode == 0 for p in procs)
