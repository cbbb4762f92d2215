"""Batched self-speculative (and autoregressive) decoding over the slot runtime.

Self-speculation (the reference's ``HybridDiffusionSelfSpec``, variant ``bd_bidir_shift``;
algorithm as stated in ``inference/zoro-1/mlx/trida_mlx/decode.py:1-17,293-386``), with
``blk = 2N - 1`` canvas rows of which the first N are token-causal:

    cold start : [t0, MASK x (2N-2)]              -> clean = row 0, specs = rows 1..N-1; commit 1
    verify     : [pending, spec_1..spec_{N-1}, MASK x (N-1)]
                 spec_j is accepted while it equals the causal prediction of row j-1;
                 all accepted -> emit specs + row N-1, new specs = rows N..2N-2; commit N
                 rejected at j -> emit accepted specs + correction; commit 1 + j; cold start next

Row i of a canvas predicts canvas position i + 1 (shift read-out).  Cold starts and verifies have
the same canvas shape, so every running request advances in ONE batched forward per step.  Greedy
decoding is lossless (the output equals autoregressive greedy decoding token for token).  With
temperature > 0 the ``strict_truncated`` policy applies: drafts come from the same top-k / top-p
truncated distribution the verifier uses, accepted with probability ``min(1, p / q)`` and
corrected from ``norm(max(0, p - q))``.

``mode="causal"`` decodes one token per forward (a one-row canvas).

``mode="draft-verify"`` is GravityOCR's self-speculation (``inference/gravityocr/sglang/python/sglang/
srt/speculative/selfspec_diffusion_worker.py``: the "fresh-window" draft): every round runs a draft
forward over ``[seed, MASK x B]`` (row 0 token-causal, the masks see the whole window; draft i+1 =
read-out of row i) and a causal verify forward over ``[seed, draft_1..draft_B]``; the longest
prefix of drafts equal to the verifier's choices is kept, plus the verifier's token after it as the
next seed (greedy; with sampling a draft is kept with the probability the verifier gives it and the
first rejection is redrawn from the verifier's distribution without the rejected token).  The
prompt may carry images (``Request.images``), encoded by the model's vision tower at admission.

``mode="diffusion"`` is pure block-diffusion decoding with the LowConfidenceShift gate (the
reference's SGLang ``LowConfidenceShiftHybridDiffusion`` and vLLM ``_denoise_shift_step``,
``inference/zoro-1/vllm/vllm_native_diffusion/qwen3_5_diffusion.py:449-632``): a block canvas
``[seed, MASK x (B-1)]`` whose row 0 is token-causal and whose other rows see the whole canvas is
denoised in rounds; position i reads the prediction of row i-1 (softmax in fp32); masked
positions whose confidence exceeds ``threshold`` are committed, and when none does the single most
confident one is forced; the last allowed round commits every remaining mask.  A finished block is
then run once more as clean token-causal rows, which advances the caches and yields the next seed
from its last row.
"""
import itertools
import queue
import threading
import time
from dataclasses import dataclass, field
from typing import List, Optional

import torch

from .runtime import Runtime


@dataclass
class SamplingParams:
    temperature: float = 0.0
    top_k: int = 20
    top_p: float = 0.95
    seed: Optional[int] = None

    @property
    def greedy(self):
        return self.temperature <= 0


@dataclass
class Request:
    prompt: List[int]
    max_new_tokens: int = 256
    sampling: SamplingParams = field(default_factory=SamplingParams)
    eos: tuple = ()
    rid: int = 0
    # results
    output: List[int] = field(default_factory=list)
    finish_reason: Optional[str] = None
    forwards: int = 0
    accept_hist: List[int] = field(default_factory=list)
    t_submit: float = 0.0
    t_first: Optional[float] = None
    t_done: Optional[float] = None
    # decode state
    slot: int = -1
    t0: Optional[int] = None
    t0_emitted: bool = False
    pending: Optional[int] = None
    canvas: Optional[List[int]] = None        # diffusion mode: the block being denoised
    images: Optional[tuple] = None            # (pixel_values, image_grid_thw) of the prompt's images
    rounds: int = 0
    specs: Optional[List[int]] = None
    spec_q: Optional[torch.Tensor] = None
    sampler_seed: Optional[int] = None        # device sampler: the request's random stream
    gen: Optional[torch.Generator] = None
    on_tokens: Optional[object] = None      # callable(list[int]) for streaming
    done_event: threading.Event = field(default_factory=threading.Event)

    @property
    def done(self):
        return self.finish_reason is not None


def truncated_probs(logits, sp):
    """Softmax of logits / T restricted to the top-k and top-p nucleus (rows renormalised)."""
    x = logits.float() / max(sp.temperature, 1e-6)
    if sp.top_k and sp.top_k > 0 and sp.top_k < x.shape[-1]:
        kth = torch.topk(x, sp.top_k, dim=-1).values[..., -1:]
        x = x.masked_fill(x < kth, float("-inf"))
    p = torch.softmax(x, -1)
    if sp.top_p and sp.top_p < 1.0:
        sp_, idx = torch.sort(p, dim=-1, descending=True)
        cum = sp_.cumsum(-1)
        drop = (cum - sp_) > sp.top_p
        sp_ = sp_.masked_fill(drop, 0.0)
        p = torch.zeros_like(p).scatter(-1, idx, sp_)
        p = p / p.sum(-1, keepdim=True)
    return p


# Canvases of at most this many rows run the gated-delta layers on the per-token scan kernels, larger
# ones on the tensor-core chunk kernels: one 64-row chunk costs the same whatever the canvas size
# (measured at 64 requests: 9.7 ms per decode step with 7-row canvases on the scan kernels against
# 14.0 ms on the chunk kernels; with 63-row canvases the chunk kernels are the faster).
GDN_SCAN_MAX_ROWS = 16


def choose_gdn_canvas_path(runtime, canvas_rows):
    """Pick the CUDA runtime's gated-delta canvas path for this engine's canvas size, unless
    ``TRIDA_GDN_CANVAS`` names one.  The two paths keep the cached state in different layouts, so
    the choice is made only while no slot holds state (every cache is still zero in both)."""
    import os
    if not getattr(runtime, "cuda", False) or not hasattr(runtime, "gdn_tc") or "TRIDA_GDN_CANVAS" in os.environ:
        return
    if len(runtime.free) != runtime.max_slots or runtime.pending is not None:
        return
    runtime.gdn_tc = canvas_rows > GDN_SCAN_MAX_ROWS


class Engine:
    """Continuous-batching decode engine over one ``Runtime``."""

    def __init__(self, runtime: Runtime, mask_id: int, mode: str = "self-spec", n: int = 4,
                 max_running: Optional[int] = None, graphs: bool = False, block_size: int = 8,
                 threshold: float = 0.9, max_steps: Optional[int] = None, pos_offset: int = 0):
        assert mode in ("self-spec", "causal", "diffusion", "draft-verify")
        self.rt = runtime
        if graphs and runtime.cuda:
            runtime.use_graphs()
        self.mask_id = mask_id
        self.mode = mode
        self.n = n if mode == "self-spec" else 1
        self.blk = {"diffusion": block_size, "draft-verify": block_size + 1}.get(mode, 2 * self.n - 1)
        self.pos_offset = pos_offset     # RoPE shift of every generated token (GravityOCR's layout: 1)
        self.threshold = threshold
        self.max_steps = max_steps or max(block_size - 1, 1)
        self.max_running = min(max_running or runtime.max_slots, runtime.max_slots)
        choose_gdn_canvas_path(runtime, self.blk)
        self.waiting: "queue.Queue[Request]" = queue.Queue()
        self.inbox: "Optional[queue.Queue[Request]]" = None   # set by a lock-step (TP) driver
        self.running: List[Request] = []
        self._ids = itertools.count()
        self._lock = threading.Lock()
        self._thread = None
        self._stop = False
        self.stats = {"forwards": 0, "tokens": 0, "steps": 0, "prefill_tokens": 0}
        self.stats_interval = 0.0            # seconds between stats lines on stdout (0 = off)
        from ..utils.trace import RequestTrace
        self.trace = RequestTrace.from_env()  # $TRIDA_TRACE_JSONL: one line per finished request
        self._stats_t = time.perf_counter()
        # sampled self-spec steps on the device sampler (top-k <= 64) unless TRIDA_SAMPLER=host
        import os
        self._dev_sampler = (runtime.cuda and self.mode == "self-spec" and
                             os.environ.get("TRIDA_SAMPLER", "device") == "device")
        self._sampler_state = None

    # ------------------------------------------------------------------ API
    def submit(self, req: Request) -> Request:
        req.rid = next(self._ids)
        req.t_submit = time.perf_counter()
        req.accept_hist = [0] * (self.blk if self.mode == "draft-verify" else self.n)
        self._seed_request(req)
        (self.inbox if self.inbox is not None else self.waiting).put(req)
        return req

    def _seed_request(self, req):
        if req.sampling.seed is not None:
            req.gen = torch.Generator(device=self.rt.device).manual_seed(req.sampling.seed)

    def generate(self, prompts, max_new_tokens=256, sampling=None, eos=()):
        """Synchronous batch generation (runs the loop in the caller's thread)."""
        reqs = [self.submit(Request(list(p), max_new_tokens, sampling or SamplingParams(), tuple(eos)))
                for p in prompts]
        while not all(r.done for r in reqs):
            self.step()
        return reqs

    def start(self):
        if self._thread is None:
            self._thread = threading.Thread(target=self._loop, daemon=True)
            self._thread.start()

    def stop(self):
        self._stop = True
        if self._thread is not None:
            self._thread.join(timeout=30)

    def _loop(self):
        while not self._stop:
            if not self.running and self.waiting.empty():
                time.sleep(0.001)
                continue
            self.step()

    # ------------------------------------------------------------------ scheduling
    def step(self):
        self._admit()
        if self.running:
            self._decode()
        self.stats["steps"] += 1
        if self.stats_interval and time.perf_counter() - self._stats_t >= self.stats_interval:
            self._stats_t = time.perf_counter()
            st = self.stats
            print(f"[trida-engine] mode={self.mode} running={len(self.running)} fwd={st['forwards']} "
                  f"tok={st['tokens']} tok/fwd={st['tokens'] / max(st['forwards'], 1):.3f} "
                  f"prefill_tok={st['prefill_tokens']}", flush=True)

    def _admit(self):
        new = []
        while len(self.running) + len(new) < self.max_running and self.rt.free:
            try:
                req = self.waiting.get_nowait()
            except queue.Empty:
                break
            req.slot = self.rt.alloc()
            new.append(req)
        if not new:
            return
        # batch prefills of equal prompt length
        new.sort(key=lambda r: len(r.prompt))
        for _, grp in itertools.groupby(new, key=lambda r: len(r.prompt)):
            grp = list(grp)
            vis = [self._vision(r) for r in grp]
            logits = self.rt.prefill([r.slot for r in grp], [r.prompt for r in grp],
                                     vis=vis if any(v is not None for v in vis) else None,
                                     pos_offset=self.pos_offset)
            self.stats["prefill_tokens"] += sum(len(r.prompt) for r in grp)
            for b, r in enumerate(grp):
                r.t0 = self._pick(logits[b:b + 1], r)[0]
                r.t0_emitted = False
                if self.mode in ("causal", "diffusion", "draft-verify"):
                    self._emit(r, [r.t0])
                    r.t0_emitted = True
                if self.mode == "diffusion":
                    r.canvas, r.rounds = [r.t0] + [self.mask_id] * (self.blk - 1), 0
            self.running.extend(grp)
        self._reap()

    def _vision(self, r):
        """(image features, 3-D positions) of a request with images, else None."""
        if r.images is None:
            return None
        from ..data.images import mrope_position_ids
        vis_model = self.rt.dec.visual
        if vis_model is None:
            raise ValueError("the model has no vision tower")
        pv, grid = r.images
        p = next(vis_model.parameters())
        with torch.no_grad():
            feats = vis_model(pv.to(p.device), grid)
        merge = getattr(vis_model, "c").spatial_merge_size
        return feats, mrope_position_ids(torch.tensor(r.prompt), grid, self.rt.cfg.image_token_id, merge)

    def _pick(self, logits, req):
        if req.sampling.greedy:
            return self.rt.argmax(logits).tolist()
        p = truncated_probs(logits, req.sampling)
        return torch.multinomial(p, 1, generator=req.gen).squeeze(-1).tolist()

    def _emit(self, req, toks):
        out = []
        for t in toks:
            if t in req.eos:
                req.finish_reason = "stop"
                break
            out.append(t)
            if len(req.output) + len(out) >= req.max_new_tokens:
                req.finish_reason = "length"
                break
        if out:
            if req.t_first is None:
                req.t_first = time.perf_counter()
            req.output.extend(out)
            self.stats["tokens"] += len(out)
            if req.on_tokens is not None:
                req.on_tokens(out)

    def _reap(self):
        keep = []
        for r in self.running:
            if r.done:
                r.t_done = time.perf_counter()
                self.rt.release(r.slot)
                if self.trace is not None:
                    self.trace.write(r, self.mode)
                r.done_event.set()
                if r.on_tokens is not None:
                    r.on_tokens(None)
            else:
                keep.append(r)
        self.running = keep

    # ------------------------------------------------------------------ one decode forward
    def _decode(self):
        if self.mode == "diffusion":
            return self._decode_diffusion()
        if self.mode == "draft-verify":
            return self._decode_draft_verify()
        reqs = self.running
        slots = [r.slot for r in reqs]
        n, blk, K = self.n, self.blk, self.n - 1
        greedy = all(r.sampling.greedy for r in reqs)
        if self.mode == "causal":
            toks = [[r.output[-1] if r.output else r.t0] for r in reqs]
            logits = self.rt.canvas(slots, toks, 1, greedy=greedy)
            am = self.rt.argmax(logits)[:, 0].tolist() if greedy else None
            picks = [[am[b]] if greedy else self._pick(logits[b], r) for b, r in enumerate(reqs)]
            self.rt.commit(slots, [1] * len(reqs))
            self.stats["forwards"] += 1
            for b, r in enumerate(reqs):
                r.forwards += 1
                self._emit(r, picks[b])
            self._reap()
            return
        canv = []
        for r in reqs:
            if r.specs is not None:
                canv.append([r.pending] + r.specs + [self.mask_id] * (n - 1))
            else:
                canv.append([r.t0] + [self.mask_id] * (blk - 1))
        logits = self.rt.canvas(slots, canv, n, greedy=greedy)
        self.stats["forwards"] += 1
        if not greedy and self._device_sampling_ok(reqs):
            return self._decode_spec_device(reqs, slots, logits)
        am = self.rt.argmax(logits).tolist() if greedy else None
        adv = []
        for b, r in enumerate(reqs):
            r.forwards += 1
            if r.specs is not None:
                acc, corr, clean, new_specs, new_q = self._verify(r, logits[b], am[b] if greedy else None)
                if corr is not None:
                    adv.append(1 + acc)
                    r.accept_hist[acc] += 1
                    self._emit(r, r.specs[:acc] + [corr])
                    r.t0, r.t0_emitted = corr, True
                    r.pending, r.specs, r.spec_q = None, None, None
                else:
                    adv.append(n)
                    r.accept_hist[K] += 1
                    self._emit(r, r.specs + [clean])
                    r.pending, r.specs, r.spec_q = clean, new_specs, new_q
            else:
                if r.sampling.greedy:
                    vals = am[b][:n] if greedy else logits[b, :n].argmax(-1).tolist()
                    new_q = None
                else:
                    P = truncated_probs(logits[b, :n], r.sampling)
                    vals = torch.multinomial(P, 1, generator=r.gen).squeeze(-1).tolist()
                    new_q = P[1:n]
                clean, new_specs = vals[0], vals[1:n]
                adv.append(1)
                self._emit(r, ([] if r.t0_emitted else [r.t0]) + [clean])
                r.t0_emitted = True
                r.pending, r.specs, r.spec_q = clean, new_specs, new_q
        self.rt.commit(slots, adv)
        self._reap()

    # ------------------------------------------------------------------ device sampler
    def _device_sampling_ok(self, reqs):
        """Every sampled request truncates to at most 64 candidates (top-k 1 .. 64), and none carries
        draft distributions from the host path."""
        if not self._dev_sampler:
            return False
        for r in reqs:
            if not r.sampling.greedy and not (0 < r.sampling.top_k <= 64):
                return False
            if r.specs is not None and r.spec_q is not None:
                return False
        return True

    def _state(self):
        """Per-slot draw counters and draft q lists of the device sampler (allocated once)."""
        if self._sampler_state is None:
            dev, S, K = self.rt.device, self.rt.max_slots + 1, self.n - 1
            self._sampler_state = {
                "ctr": torch.zeros(S, dtype=torch.long, device=dev),
                "q_idx": torch.full((S, max(K, 1), 64), -1, dtype=torch.int32, device=dev),
                "q_prob": torch.zeros(S, max(K, 1), 64, dtype=torch.float32, device=dev)}
        return self._sampler_state

    def _decode_spec_device(self, reqs, slots, logits):
        """One sampled self-spec step for the whole batch: one top-k pass over the canvas logits and
        one sampler launch (proposals, verification, corrections, new drafts and their q lists on the
        device), then one host read of [B, 3 + K] integers."""
        n, K = self.n, self.n - 1
        st = self._state()
        B = len(reqs)
        kc = max((r.sampling.top_k if not r.sampling.greedy else 1) for r in reqs)
        vals, idx = torch.topk(logits[:B].float(), kc, dim=-1, sorted=True)
        host = torch.empty(B, 6, dtype=torch.float64)
        specs = torch.zeros(B, max(K, 1), dtype=torch.int32)
        for b, r in enumerate(reqs):
            sp = r.sampling
            if r.sampler_seed is None:
                r.sampler_seed = sp.seed if sp.seed is not None else int(torch.randint(0, 2 ** 62, (1,)))
                st["ctr"][r.slot] = 0
            g = sp.greedy
            host[b] = torch.tensor([1.0 if g else sp.temperature, 1 if g else sp.top_k, 1.0 if g else sp.top_p,
                                    r.sampler_seed, r.slot, 1 if r.specs is not None else 0], dtype=torch.float64)
            if r.specs is not None:
                specs[b, :K] = torch.tensor(r.specs, dtype=torch.int32)
        dev = logits.device
        temp = host[:, 0].float().to(dev, non_blocking=True)
        topk = host[:, 1].int().to(dev, non_blocking=True)
        topp = host[:, 2].float().to(dev, non_blocking=True)
        seed = torch.tensor([r.sampler_seed for r in reqs], dtype=torch.long).to(dev, non_blocking=True)
        slot_t = host[:, 4].int().to(dev, non_blocking=True)
        has = host[:, 5].int().to(dev, non_blocking=True)
        out = torch.empty(B, 3 + K, dtype=torch.int32, device=dev)
        self.rt.C.spec_sample(vals.contiguous(), idx.contiguous(), temp, topk, topp, seed, st["ctr"], slot_t,
                              specs.to(dev, non_blocking=True), has, st["q_idx"], st["q_prob"], out, n)
        res = out.tolist()
        adv = []
        for b, r in enumerate(reqs):
            r.forwards += 1
            acc, corr, clean, new_specs = res[b][0], res[b][1], res[b][2], res[b][3:3 + K]
            if r.specs is not None:
                if corr >= 0:
                    adv.append(1 + acc)
                    r.accept_hist[acc] += 1
                    self._emit(r, r.specs[:acc] + [corr])
                    r.t0, r.t0_emitted = corr, True
                    r.pending, r.specs = None, None
                else:
                    adv.append(n)
                    r.accept_hist[K] += 1
                    self._emit(r, r.specs + [clean])
                    r.pending, r.specs = clean, new_specs
            else:
                adv.append(1)
                self._emit(r, ([] if r.t0_emitted else [r.t0]) + [clean])
                r.t0_emitted = True
                r.pending, r.specs = clean, new_specs
            r.spec_q = None
        self.rt.commit(slots, adv)
        self._reap()

    def _decode_diffusion(self):
        Bk, M = self.blk, self.mask_id
        den = [r for r in self.running if M in r.canvas[1:]]
        fin = [r for r in self.running if M not in r.canvas[1:]]
        if den:                                          # one denoise round
            logits = self.rt.canvas([r.slot for r in den], [r.canvas for r in den], 1)
            greedy = all(r.sampling.greedy for r in den)
            if greedy:
                idx, conf = self.rt.conf_argmax(logits[:, :Bk - 1])
                idx, conf = idx.tolist(), conf.tolist()
            self.rt.discard()
            self.stats["forwards"] += 1
            for b, r in enumerate(den):
                if greedy:
                    pred, cf = idx[b], conf[b]
                else:
                    pred, cf = self._sample_rows(logits[b, :Bk - 1], r)
                r.forwards += 1
                r.rounds += 1
                masked = [i for i in range(1, Bk) if r.canvas[i] == M]
                if r.rounds >= self.max_steps:
                    take = masked
                else:
                    take = [i for i in masked if cf[i - 1] > self.threshold]
                    if not take:
                        take = [max(masked, key=lambda i: cf[i - 1])]
                for i in take:
                    r.canvas[i] = pred[i - 1]
        if fin:                                          # commit finished blocks causally
            slots = [r.slot for r in fin]
            logits = self.rt.canvas(slots, [r.canvas for r in fin], Bk)
            greedy = all(r.sampling.greedy for r in fin)
            am = self.rt.argmax(logits)[:, Bk - 1].tolist() if greedy else None
            seeds = [am[b] if greedy else self._pick(logits[b, Bk - 1:Bk], r)[0] for b, r in enumerate(fin)]
            self.rt.commit(slots, [Bk] * len(fin))
            self.stats["forwards"] += 1
            for b, r in enumerate(fin):
                r.forwards += 1
                self._emit(r, r.canvas[1:] + [seeds[b]])
                r.canvas, r.rounds = [seeds[b]] + [M] * (Bk - 1), 0
        self._reap()

    def _decode_draft_verify(self):
        reqs = self.running
        slots = [r.slot for r in reqs]
        K, M = self.blk, self.mask_id
        # draft: a fresh window [seed, MASK x (K-1)], read out shifted (row i proposes token i+1)
        lg = self.rt.canvas(slots, [[r.t0] + [M] * (K - 1) for r in reqs], 1)
        drafts = self.rt.argmax(lg)[:, :K - 1].tolist()
        self.rt.discard()
        # verify: the causal path over [seed, drafts]
        lg = self.rt.canvas(slots, [[r.t0] + drafts[b] for b, r in enumerate(reqs)], K)
        greedy = all(r.sampling.greedy for r in reqs)
        am = self.rt.argmax(lg).tolist() if greedy else None
        self.stats["forwards"] += 2
        adv, outs = [], []
        for b, r in enumerate(reqs):
            r.forwards += 2
            d = drafts[b]
            if r.sampling.greedy:
                p = am[b] if greedy else lg[b].argmax(-1).tolist()
                acc = 0
                while acc < K - 1 and d[acc] == p[acc]:
                    acc += 1
                bonus = p[acc]
            else:
                acc, bonus = self._verify_sampled(r, lg[b], d)
            r.accept_hist[min(acc, len(r.accept_hist) - 1)] += 1
            adv.append(1 + acc)
            outs.append(d[:acc] + [bonus])
        self.rt.commit(slots, adv)
        for b, r in enumerate(reqs):
            self._emit(r, outs[b])
            r.t0 = outs[b][-1]
        self._reap()

    def _verify_sampled(self, r, L, d):
        """Speculative sampling against a deterministic draft: keep draft j with probability p_j(d_j);
        at the first rejection draw from p_j with d_j removed; after a full block draw the bonus."""
        P = truncated_probs(L, r.sampling)                     # [K, V]
        K1 = len(d)
        for j in range(K1):
            pj = float(P[j, d[j]])
            u = float(torch.rand((), device=L.device, generator=r.gen))
            if u < pj:
                continue
            resid = P[j].clone()
            resid[d[j]] = 0.0
            z = resid.sum()
            resid = resid / z if z > 0 else P[j]
            return j, int(torch.multinomial(resid, 1, generator=r.gen))
        return K1, int(torch.multinomial(P[K1], 1, generator=r.gen))

    def _sample_rows(self, L, r):
        """Sampled denoise read-out: a token per row from the truncated distribution and its probability."""
        P = truncated_probs(L, r.sampling)
        tok = torch.multinomial(P, 1, generator=r.gen)
        return tok.squeeze(-1).tolist(), P.gather(1, tok).squeeze(-1).tolist()

    def _verify(self, r, L, am):
        n, blk, K = self.n, self.blk, self.n - 1
        if r.sampling.greedy:
            vals = am if am is not None else L.argmax(-1).tolist()
            acc = 0
            while acc < K and vals[acc] == r.specs[acc]:
                acc += 1
            corr = vals[acc] if acc < K else None
            return acc, corr, vals[n - 1], vals[n:blk], None
        P = truncated_probs(L, r.sampling)
        sv = torch.tensor(r.specs, device=L.device)
        p = P[:K].gather(1, sv[:, None])[:, 0]
        q = r.spec_q.gather(1, sv[:, None])[:, 0]
        ratio = torch.where(q > 0, p / q.clamp_min(1e-30), torch.zeros_like(p))
        u = torch.rand(K, device=L.device, generator=r.gen)
        accepted = ((ratio >= 1.0) | (u < ratio)).tolist()
        acc = 0
        while acc < K and accepted[acc]:
            acc += 1
        if acc < K:
            resid = (P[acc] - r.spec_q[acc]).clamp_min(0.0)
            rs = resid.sum()
            resid = resid / rs if rs > 0 else P[acc]
            corr = int(torch.multinomial(resid, 1, generator=r.gen))
            return acc, corr, None, None, None
        samp = torch.multinomial(P[n - 1:blk], 1, generator=r.gen).squeeze(-1).tolist()
        return acc, None, samp[0], samp[1:], P[n:blk]

    # ------------------------------------------------------------------ stats
    def summary(self, reqs):
        toks = sum(len(r.output) for r in reqs)
        fwd = sum(r.forwards for r in reqs)
        ttft = sorted((r.t_first - r.t_submit) for r in reqs if r.t_first is not None)
        return {"tokens": toks, "forwards": fwd, "tokens_per_forward": toks / max(fwd, 1),
                "p50_ttft_s": ttft[len(ttft) // 2] if ttft else None}
