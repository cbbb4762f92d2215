"""Serving runtime and self-speculative engine on CPU: prefill logits match the model's causal
forward, and greedy self-speculative decoding equals greedy autoregressive decoding."""
import pytest
import torch

from trida_stack_b200.models import Decoder, ModelConfig, qwen3_config
from trida_stack_b200.models.hybrid import HybridBlockDiffusionLM
from trida_stack_b200.serve import Engine, Runtime, SamplingParams


def tiny_hybrid(seed=0):
    cfg = ModelConfig.from_hf_dict({
        "model_type": "qwen3_5_text", "vocab_size": 97, "hidden_size": 64, "intermediate_size": 128,
        "num_hidden_layers": 4, "num_attention_heads": 2, "num_key_value_heads": 1, "head_dim": 32,
        "linear_num_key_heads": 2, "linear_num_value_heads": 4, "linear_key_head_dim": 16,
        "linear_value_head_dim": 16, "linear_conv_kernel_dim": 4, "partial_rotary_factor": 0.5,
        "layer_types": ["linear_attention"] * 3 + ["full_attention"], "tie_word_embeddings": True})
    torch.manual_seed(seed)
    dec = Decoder(cfg, dtype=torch.float32)
    with torch.no_grad():
        for n, p in dec.named_parameters():
            if p.dim() >= 2:
                p.normal_(0, 0.2)
            elif n.endswith("A_log"):
                p.copy_(torch.log(torch.empty_like(p).uniform_(0.5, 4)))
            else:
                p.copy_(1 + 0.1 * torch.randn_like(p))
    return dec


def tiny_dense(seed=0):
    torch.manual_seed(seed)
    cfg = qwen3_config(vocab_size=97, hidden_size=64, intermediate_size=128, num_layers=2, n_heads=4,
                       n_kv_heads=2, head_dim=16)
    dec = Decoder(cfg, dtype=torch.float32)
    with torch.no_grad():
        for p in dec.parameters():
            if p.dim() >= 2:
                p.normal_(0, 0.3)
    return dec


def full_logits(dec, ids):
    m = HybridBlockDiffusionLM(dec, mask_id=96, ar_only=True)
    with torch.no_grad():
        actx = m._causal_rows(ids, None)
        h = dec(dec.embed_tokens(ids), actx)
        return (h @ dec.lm_weight.t()).view(ids.shape[0], ids.shape[1], -1)


@pytest.mark.parametrize("make", [tiny_hybrid, tiny_dense])
def test_prefill_and_canvas_match_causal_forward(make):
    dec = make()
    torch.manual_seed(1)
    ids = torch.randint(0, 96, (2, 150))
    ref = full_logits(dec, ids)
    rt = Runtime(dec, max_slots=4, max_len=256)
    slots = [rt.alloc(), rt.alloc()]
    # prefill 130 tokens (3 chunks), then a fully causal canvas of the next 20
    last = rt.prefill(slots, ids[:, :130].tolist())
    torch.testing.assert_close(last, ref[:, 129], rtol=1e-4, atol=1e-4)
    lg = rt.canvas(slots, ids[:, 130:150], 20)
    torch.testing.assert_close(lg, ref[:, 130:150], rtol=1e-4, atol=1e-4)
    # commit only 7 rows, then re-run the rest: the cache must continue from row 137
    rt.commit(slots, [7, 7])
    lg2 = rt.canvas(slots, ids[:, 137:150], 13)
    torch.testing.assert_close(lg2, ref[:, 137:150], rtol=1e-4, atol=1e-4)
    rt.commit(slots, [13, 13])


@pytest.mark.parametrize("make", [tiny_hybrid, tiny_dense])
@pytest.mark.parametrize("n", [2, 4])
def test_greedy_self_spec_equals_autoregressive(make, n):
    dec = make()
    torch.manual_seed(2)
    prompts = [torch.randint(0, 96, (L,)).tolist() for L in (9, 9, 14)]
    ar = Engine(Runtime(dec, max_slots=4, max_len=256), mask_id=96, mode="causal")
    ref = [r.output for r in ar.generate(prompts, max_new_tokens=40)]
    ss = Engine(Runtime(dec, max_slots=4, max_len=256), mask_id=96, mode="self-spec", n=n)
    reqs = ss.generate(prompts, max_new_tokens=40)
    for r, want in zip(reqs, ref):
        assert r.output == want
        assert r.finish_reason == "length"
    s = ss.summary(reqs)
    assert s["tokens_per_forward"] >= 1.0


def test_sampled_self_spec_runs_and_respects_eos():
    dec = tiny_hybrid()
    eng = Engine(Runtime(dec, max_slots=2, max_len=256), mask_id=96, mode="self-spec", n=3)
    sp = SamplingParams(temperature=0.8, top_k=20, top_p=0.9, seed=3)
    reqs = eng.generate([[1, 2, 3, 4, 5]], max_new_tokens=30, sampling=sp, eos=(7,))
    r = reqs[0]
    assert r.done and 7 not in r.output and len(r.output) <= 30


class _ThreadTP:
    """CPU stand-in for TPContext: W runtimes in W threads sum their row-parallel partials and
    gather their argmax pairs through shared slots and a barrier."""

    def __init__(self, shared, rank, world, seq_parallel=False):
        self.s, self.rank, self.world, self.seq_parallel = shared, rank, world, seq_parallel

    def _exchange_list(self, t):
        self.s["slots"][self.rank] = t
        self.s["bar"].wait()
        out = list(self.s["slots"])
        self.s["bar"].wait()
        return out

    def _exchange(self, t):
        return torch.stack(self._exchange_list(t))

    def row_parallel(self, x, w, residual):
        return residual + self._exchange(x @ w.t()).sum(0)

    # sequence-parallel boundary, as TPContext.own_rows / shard / reduce_norm state it
    def own_rows(self, rows):
        per = -(-rows // self.world)
        r0 = min(rows, self.rank * per)
        return r0, min(rows, r0 + per) - r0

    def shard(self, x):
        r0, n = self.own_rows(x.shape[0])
        return x[r0:r0 + n].clone()

    def reduce_norm(self, a, w, xs, norm_w, eps):
        from trida_stack_b200.ops import reference as R
        tot = self._exchange(a @ w.t()).sum(0)
        r0, n = self.own_rows(a.shape[0])
        assert xs.shape[0] == n
        xs = xs + tot[r0:r0 + n]
        return xs, torch.cat(self._exchange_list(R.rmsnorm(xs, norm_w, eps)))

    def gather(self, t):
        return self._exchange(t)


@pytest.mark.parametrize("seq_parallel", [False, True])
@pytest.mark.parametrize("world", [2, 4])
def test_tensor_parallel_shards_reproduce_full_model(world, seq_parallel):
    import threading

    from trida_stack_b200.serve.tp import shard_decoder
    dec = tiny_hybrid()
    dec.cfg.lin_k_heads, dec.cfg.lin_v_heads = 2, 4          # tiny_hybrid's GDN heads
    torch.manual_seed(3)
    prompts = [torch.randint(0, 96, (12,)).tolist() for _ in range(2)]
    ref = Engine(Runtime(dec, max_slots=4, max_len=128), mask_id=96, mode="self-spec", n=3)
    want = [r.output for r in ref.generate(prompts, max_new_tokens=16)]
    if 2 % world and dec.cfg.n_kv_heads < world:
        pytest.skip("shape does not split")
    shared = {"slots": [None] * world, "bar": threading.Barrier(world)}
    outs = [None] * world
    errs = []

    def run(r):
        try:
            local = shard_decoder(dec, r, world)
            eng = Engine(Runtime(local, max_slots=4, max_len=128, tp=_ThreadTP(shared, r, world, seq_parallel)), mask_id=96,
                         mode="self-spec", n=3)
            outs[r] = [q.output for q in eng.generate(prompts, max_new_tokens=16)]
        except Exception as e:   # surface in the main thread
            errs.append(e)
            shared["bar"].abort()

    ths = [threading.Thread(target=run, args=(r,)) for r in range(world)]
    for t in ths:
        t.start()
    for t in ths:
        t.join(timeout=300)
    assert not errs, errs
    for o in outs:
        assert o == want


def _manual_block(dec, prompt, Bk, threshold, max_steps, mask_id=96):
    """First denoised block of greedy LowConfidenceShift decoding, stepped by hand."""
    rt = Runtime(dec, max_slots=2, max_len=256)
    s = rt.alloc()
    t0 = int(rt.prefill([s], [prompt])[0].argmax())
    canvas = [t0] + [mask_id] * (Bk - 1)
    rounds = 0
    while mask_id in canvas[1:]:
        lg = rt.canvas([s], [canvas], 1)[0]
        rt.discard()
        p = torch.softmax(lg[:Bk - 1].double(), -1)
        conf, pred = p.max(-1)
        rounds += 1
        masked = [i for i in range(1, Bk) if canvas[i] == mask_id]
        if rounds >= max_steps:
            take = masked
        else:
            take = [i for i in masked if conf[i - 1] > threshold] or [max(masked, key=lambda i: conf[i - 1])]
        for i in take:
            canvas[i] = int(pred[i - 1])
    return [t0] + canvas[1:], rounds


@pytest.mark.parametrize("make", [tiny_hybrid, tiny_dense])
@pytest.mark.parametrize("threshold", [0.0, 0.05, 2.0])
def test_diffusion_decode_low_confidence_shift(make, threshold):
    dec = make()
    torch.manual_seed(4)
    Bk = 4
    prompts = [torch.randint(0, 96, (L,)).tolist() for L in (9, 13)]
    eng = Engine(Runtime(dec, max_slots=4, max_len=256), mask_id=96, mode="diffusion", block_size=Bk,
                 threshold=threshold)
    reqs = eng.generate(prompts, max_new_tokens=3 * Bk + 1)
    for p, r in zip(prompts, reqs):
        assert len(r.output) == 3 * Bk + 1
        # the first block follows the gate rule
        blk, rounds = _manual_block(dec, p, Bk, threshold, Bk - 1)
        assert r.output[:Bk] == blk
        if threshold == 0.0:
            assert rounds == 1            # everything passes in the first round
        if threshold == 2.0:
            assert rounds == Bk - 1       # one forced token per round
        # every block seed is the causal (greedy AR) continuation of what precedes it
        ref = full_logits(dec, torch.tensor([p + r.output[:-1]]))[0]
        for j in range(0, len(r.output), Bk):
            assert int(ref[len(p) + j - 1].argmax()) == r.output[j]


def test_sampled_diffusion_decode_respects_eos():
    dec = tiny_dense()
    torch.manual_seed(7)
    eng = Engine(Runtime(dec, max_slots=4, max_len=256), mask_id=96, mode="diffusion", block_size=4,
                 threshold=0.3)
    sp = SamplingParams(temperature=1.0, top_k=10, top_p=0.9, seed=3)
    reqs = eng.generate([[1, 2, 3, 4, 5]] * 2, max_new_tokens=30, sampling=sp, eos=(7,))
    for r in reqs:
        assert r.finish_reason in ("stop", "length") and 7 not in r.output


def _lockstep_rank(rank, world, port, out):
    import os

    import torch.distributed as dist

    from trida_stack_b200.serve.lockstep import LockstepDriver
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        eng = Engine(Runtime(tiny_dense(), max_slots=4, max_len=256), mask_id=96, mode="self-spec", n=3,
                     max_running=2)
        drv = LockstepDriver(eng)
        if rank == 0:
            reqs = [eng.submit(__import__("trida_stack_b200.serve", fromlist=["Request"]).Request(
                [1 + i, 2, 3, 4 + i], 12, SamplingParams(temperature=0.0 if i % 2 == 0 else 1.0)))
                for i in range(5)]
            while not all(r.done for r in reqs):
                drv.step_leader()
            drv._stop = True
            drv.step_leader()
        else:
            drv.run_follower()
            reqs = drv.submitted
        out.put((rank, [r.output for r in reqs]))
    finally:
        dist.destroy_process_group()


def test_lockstep_driver_keeps_ranks_identical():
    """Tensor-parallel serving front end: requests (incl. sampled ones without a seed) reach every
    rank in the same order and every rank decodes the same tokens (gloo, 2 CPU ranks)."""
    import socket

    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    procs = [ctx.Process(target=_lockstep_rank, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(out.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res[0] == res[1] and len(res[0]) == 5 and all(len(o) > 0 for o in res[0])


@pytest.mark.parametrize("make", [tiny_hybrid, tiny_dense])
def test_greedy_draft_verify_equals_autoregressive(make):
    """GravityOCR-style fresh-window self-speculation (draft [seed, MASK x B], causal verify) commits
    exactly the greedy autoregressive tokens."""
    dec = make()
    torch.manual_seed(3)
    prompts = [torch.randint(0, 96, (L,)).tolist() for L in (9, 9, 14)]
    ar = Engine(Runtime(dec, max_slots=4, max_len=256), mask_id=96, mode="causal")
    ref = [r.output for r in ar.generate(prompts, max_new_tokens=30)]
    dv = Engine(Runtime(dec, max_slots=4, max_len=256), mask_id=96, mode="draft-verify", block_size=4)
    reqs = dv.generate(prompts, max_new_tokens=30)
    assert [r.output for r in reqs] == ref
    assert all(r.forwards > 0 for r in reqs)


def test_sampled_draft_verify_runs_and_respects_eos():
    dec = tiny_dense()
    eng = Engine(Runtime(dec, max_slots=4, max_len=256), mask_id=96, mode="draft-verify", block_size=4)
    sp = SamplingParams(temperature=1.0, top_k=10, top_p=0.9, seed=5)
    reqs = eng.generate([[1, 2, 3, 4, 5]] * 2, max_new_tokens=25, sampling=sp, eos=(7,))
    for r in reqs:
        assert r.finish_reason in ("stop", "length") and 7 not in r.output


def test_kv_page_allocator():
    """Pages are taken from one pool as slots grow, never past the pool or the page table, and
    come back on release in an order that reuses them."""
    from trida_stack_b200.serve.runtime import PAGE, KVPages
    p = KVPages(n_pages=5, n_slots=3, max_pages=4)
    assert p.ensure(0, 1) and p.owned[0] == [0]
    assert not p.ensure(0, PAGE)                   # still one page
    assert p.ensure(0, PAGE + 1) and p.owned[0] == [0, 1]
    assert p.ensure(1, 3 * PAGE) and p.owned[1] == [2, 3, 4]
    assert p.table[1, :3].tolist() == [2, 3, 4] and p.used() == 5
    with pytest.raises(RuntimeError, match="exhausted"):
        p.ensure(2, 1)
    with pytest.raises(RuntimeError, match="page table"):
        p.ensure(0, 5 * PAGE)
    p.release(1)
    assert p.used() == 2 and p.ensure(2, 2 * PAGE) and p.owned[2] == [2, 3]


def test_guards_name_bad_steps():
    """TRIDA_GUARDS=1 turns a bad slot, token, canvas shape, commit advance or page-table state into
    a named error at the call (checked on the CPU runtime; the same checks run before CUDA steps)."""
    from trida_stack_b200.serve.runtime import PAGE, KVPages
    rt = Runtime(tiny_hybrid(), max_slots=3, max_len=64)
    rt.guards = True
    a, b = rt.alloc(), rt.alloc()
    rt.prefill([a, b], [[1, 2, 3, 4], [5, 6, 7, 8]])
    with pytest.raises(RuntimeError, match="twice"):
        rt.canvas([a, a], [[1, 2], [3, 4]], 1)
    free = rt.free[-1]
    with pytest.raises(RuntimeError, match="not allocated"):
        rt.canvas([a, free], [[1, 2], [3, 4]], 1)
    with pytest.raises(RuntimeError, match="vocabulary"):
        rt.canvas([a, b], [[1, 2], [3, 97]], 1)
    with pytest.raises(RuntimeError, match="n_clean"):
        rt.canvas([a, b], [[1, 2], [3, 4]], 3)
    lg = rt.canvas([a, b], [[1, 2], [3, 4]], 1)
    assert torch.isfinite(lg).all()
    with pytest.raises(RuntimeError, match="outside"):
        rt.commit([a, b], [1, 2])                  # advance past n_clean
    with pytest.raises(RuntimeError, match="pending canvas has"):
        rt.commit([b, a], [1, 1])
    rt.commit([a, b], [1, 1])
    with pytest.raises(RuntimeError, match="without a pending canvas"):
        rt.commit([a, b], [1, 1])
    # page-table ownership
    p = KVPages(n_pages=6, n_slots=3, max_pages=4)
    p.ensure(0, 2 * PAGE)
    p.ensure(1, PAGE)
    p.check([0, 1])
    p.owned[1].append(p.owned[0][0])               # one page handed to two slots
    with pytest.raises(RuntimeError, match="held by slots"):
        p.check([0, 1])
    p.owned[1].pop()
    p.table[0, 1] = 5                              # table row disagrees with the owner list
    with pytest.raises(RuntimeError, match="page table"):
        p.check([0, 1])


def test_engine_picks_gdn_canvas_path_by_canvas_size(monkeypatch):
    """Small canvases take the per-token scan kernels, large ones the tensor-core chunk kernels; the
    choice is made only before any slot holds state and yields to TRIDA_GDN_CANVAS."""
    from types import SimpleNamespace

    from trida_stack_b200.serve.engine import GDN_SCAN_MAX_ROWS, choose_gdn_canvas_path
    monkeypatch.delenv("TRIDA_GDN_CANVAS", raising=False)

    def fresh():
        return SimpleNamespace(cuda=True, gdn_tc=True, free=[3, 2, 1, 0], max_slots=4, pending=None)
    rt = fresh()
    choose_gdn_canvas_path(rt, 7)
    assert rt.gdn_tc is False
    choose_gdn_canvas_path(rt, 63)
    assert rt.gdn_tc is True
    choose_gdn_canvas_path(rt, GDN_SCAN_MAX_ROWS)
    assert rt.gdn_tc is False
    rt = fresh()
    rt.free.pop()                                   # a slot in use: its state layout is fixed
    choose_gdn_canvas_path(rt, 7)
    assert rt.gdn_tc is True
    rt = fresh()
    monkeypatch.setenv("TRIDA_GDN_CANVAS", "tc")
    choose_gdn_canvas_path(rt, 7)
    assert rt.gdn_tc is True
    cpu = SimpleNamespace(cuda=False, free=[0], max_slots=1, pending=None)
    choose_gdn_canvas_path(cpu, 7)
    assert not hasattr(cpu, "gdn_tc")
