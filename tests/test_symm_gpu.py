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


def _seqpar_worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from trida_stack_b200.serve.tp import TPContext
        bf = torch.bfloat16
        H, eps = 2560, 1e-6
        tp = TPContext(max_rows=1200, hidden=H)
        assert tp.seq_parallel
        errs = []
        g = torch.Generator("cuda").manual_seed(10 + rank)

        def rel(a, b):
            return ((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-6)).item()

        def reference(a, w, res, nw):
            part = (a.float() @ w.float().t()).to(bf)               # each rank's GEMM output is bf16
            allp = [torch.zeros_like(part) for _ in range(world)]
            dist.all_gather(allp, part)
            x = (res.float() + sum(p.float() for p in allp)).to(bf).float()
            return x, x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * nw.float()

        for M, K in ((1, 512), (301, 512), (448, 1024), (1100, 512)):   # fewer rows than ranks, uneven split
            a = torch.randn(M, K, device="cuda", dtype=bf, generator=g)
            w = torch.randn(H, K, device="cuda", dtype=bf, generator=g) * 0.05
            res = torch.randn(M, H, device="cuda", dtype=bf)
            nw = (1 + 0.1 * torch.randn(H, device="cuda")).to(bf)
            dist.broadcast(res, 0)
            dist.broadcast(nw, 0)
            x_ref, h_ref = reference(a, w, res, nw)
            r0, n = tp.own_rows(M)
            xs, h = tp.reduce_norm(a, w, res[r0:r0 + n].clone(), nw, eps)
            if n:
                errs.append(rel(xs, x_ref[r0:r0 + n]))
            errs.append(rel(h, h_ref))
            hs = [torch.zeros_like(h) for _ in range(world)]
            dist.all_gather(hs, h.contiguous())
            assert all(torch.equal(hs[0], t) for t in hs), "ranks hold different normalised rows"
        # two boundaries in a row, replayed from a CUDA graph (the epoch counter lives on the device)
        M, K = 448, 512
        a = torch.randn(M, K, device="cuda", dtype=bf, generator=g)
        w = torch.randn(H, K, device="cuda", dtype=bf, generator=g) * 0.05
        res = torch.randn(M, H, device="cuda", dtype=bf)
        nw = (1 + 0.1 * torch.randn(H, device="cuda")).to(bf)
        dist.broadcast(res, 0)
        dist.broadcast(nw, 0)
        r0, n = tp.own_rows(M)
        xs = res[r0:r0 + n].clone()
        torch.cuda.synchronize()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=s):
                tp.reduce_norm(a, w, xs, nw, eps)
                _, h = tp.reduce_norm(a, w, xs, nw, eps)
        x_full = res.clone()
        for _ in range(3):
            gr.replay()
            torch.cuda.synchronize()
            for _ in range(2):
                x_next, h_ref = reference(a, w, x_full, nw)
                x_full = x_next.to(bf)
            errs.append(rel(xs, x_full[r0:r0 + n]))
            errs.append(rel(h, h_ref))
        del gr
        tp.heap.check()
        # a sharded hybrid decoder on the CUDA runtime reproduces the single-GPU logits
        from test_serve_gpu import _hybrid, _init

        from trida_stack_b200.serve import Runtime
        from trida_stack_b200.serve.tp import shard_decoder
        cfg = _hybrid(128)
        cfg.lin_v_heads = 8          # per-rank in_proj width (2 x value heads in the gates) stays 16-byte aligned
        dec = _init(cfg).to("cuda", bf)
        torch.manual_seed(4)
        prompts = [torch.randint(0, 500, (40,)).tolist() for _ in range(3)]
        canv = [torch.randint(0, 500, (9,)).tolist() for _ in range(3)]
        ref_rt = Runtime(dec, max_slots=4, max_len=256)
        sl = [ref_rt.alloc() for _ in prompts]
        ref_rt.prefill(sl, prompts)
        want = ref_rt.canvas(sl, canv, 5).float()
        ref_rt.discard()
        local = shard_decoder(dec, rank, world)
        rt = Runtime(local, max_slots=4, max_len=256, tp=TPContext(max_rows=512, hidden=dec.cfg.hidden_size))
        sl = [rt.alloc() for _ in prompts]
        rt.prefill(sl, prompts)
        got = rt.canvas(sl, canv, 5).float()
        vp = got.shape[-1]
        errs.append(rel(got[..., :min(vp, want.shape[-1] - rank * vp)], want[..., rank * vp:(rank + 1) * vp]))
        q.put((rank, max(errs)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sequence_parallel_boundary_matches_reference():
    """Reduce-scatter + residual + RMSNorm + all-gather in one kernel (tensor-parallel serving) vs an
    fp32 statement over NCCL-gathered partials: uneven row splits, fewer rows than ranks, CUDA-graph
    replay, and a sharded hybrid decoder's logits against the single-GPU runtime, on 2 GPUs."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_seqpar_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    res = [q.get(timeout=5) for _ in range(2)]
    for rank, err in res:
        assert err < 3e-2, (rank, err)
    assert all(p.exitcode == 0 for p in procs)


def _shard_worker(rank, world, port, q):
    """A tiny dense decoder (3 layers, CUDA blocks) trained for 3 steps with replicated weights
    (fused optimizer collectives) and with full-shard weights gathered per layer over NVLink (with
    and without keeping the gathered weights to backward): same losses, same final weights; the
    P2P gather kernel itself against NCCL's all-gather."""
    import datetime

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from trida_stack_b200.engine import TrainEngine
        from trida_stack_b200.models import BlockDiffusionLM, Decoder, qwen3_config
        from trida_stack_b200.ops._ext import ext
        from trida_stack_b200.parallel.symm import SymmetricHeap
        heap = SymmetricHeap()
        shard = torch.randn(4096, device="cuda").to(torch.bfloat16)
        buf = heap.alloc(4096, torch.bfloat16)
        buf.local.copy_(shard)
        torch.cuda.synchronize()
        dist.barrier()
        got = torch.empty(world * 4096, device="cuda", dtype=torch.bfloat16)
        ext().symm_gather(buf.ptrs, rank, 4096, got, 8)
        ref = torch.empty_like(got)
        dist.all_gather_into_tensor(ref, shard)
        torch.cuda.synchronize()
        gather_ok = torch.equal(got, ref)
        res = {}
        for mode in ("zero2", "full", "keep"):
            cfg = qwen3_config(vocab_size=4096, hidden_size=256, intermediate_size=512, num_layers=3, n_heads=4,
                               n_kv_heads=2, head_dim=128)
            torch.manual_seed(0)
            model = BlockDiffusionLM(Decoder(cfg, dtype=torch.bfloat16, device="cuda"), mask_id=4095, bd_size=32,
                                     ar_loss_weight=1.0)
            model.train()
            eng = TrainEngine(model, lr=1e-3, warmup=0, device=torch.device("cuda"), comm="fused",
                              full_shard=mode != "zero2", keep_params=mode == "keep")
            g = torch.Generator().manual_seed(11 + rank)
            losses = []
            for step in range(3):
                ids = torch.randint(0, 4094, (2, 256), generator=g)
                labels = ids.clone()
                labels[:, :128] = -100
                loss, _, _, _ = eng.train_step([{"input_ids": ids, "labels": labels,
                                                 "attention_mask": torch.ones_like(ids)}], step)
                losses.append(loss.item())
            if eng.optim.param_ring is not None:
                eng.optim.param_ring.materialize()
            torch.cuda.synchronize()
            eng.optim.heap.check()
            res[mode] = (losses, {n: p.detach().float().cpu() for n, p in model.named_parameters()})
        lerr = max(abs(a - b) / max(1.0, abs(b)) for m in ("full", "keep")
                   for a, b in zip(res[m][0], res["zero2"][0]))
        # full shard vs replicated: the same math but different AdamW kernels, whose last-bit
        # differences Adam turns into full-size updates where a gradient is near zero
        werr = max(((res["full"][1][n] - p).abs().max() / (p.abs().max() + 1e-6)).item()
                   for n, p in res["zero2"][1].items())
        # gathering again for backward or keeping the forward's gather: bit-identical training
        same = all(torch.equal(res["keep"][1][n], p) for n, p in res["full"][1].items())
        q.put((rank, gather_ok, lerr, werr, same))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_full_shard_training_matches_replicated():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_shard_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    res = [q.get(timeout=5) for _ in range(2)]
    for rank, gather_ok, lerr, werr, same in res:
        assert gather_ok, rank
        assert lerr < 1e-3, (rank, lerr)
        assert werr < 5e-2, (rank, werr)
        assert same, rank
    assert all(p.exitcode == 0 for p in procs)
