"""Lock-step driving of one engine per tensor-parallel rank behind a single HTTP front end.

Every TP rank runs the same ``Engine`` over its shard of the model; the ranks' kernels meet in the
row-parallel all-reduces, so every rank must take exactly the same decode steps with the same
requests in the same order.  Rank 0 owns the request inbox (the HTTP handlers submit there); at
every step it broadcasts the requests that arrived since the last step over a CPU (gloo) group,
and every rank -- rank 0 included -- admits exactly those requests before stepping.  Sampled
requests without a seed get one from rank 0, so every rank draws the same tokens from its
identical (all-gathered) logits.  A stop flag in the same broadcast ends every rank's loop.

(The reference runs TP inside SGLang's scheduler, ``inference/zoro-1/serve.py:174,204``.)
"""
import queue
import random
import threading
import time
from dataclasses import asdict

import torch.distributed as dist

from .engine import Request, SamplingParams


class LockstepDriver:
    def __init__(self, engine, group=None, idle_sleep=0.002):
        self.engine = engine
        self.group = group
        self.rank = dist.get_rank(group)
        self.idle_sleep = idle_sleep
        self._stop = False
        self._thread = None
        self.submitted = []                 # followers: the requests received from rank 0
        if self.rank == 0:
            engine.inbox = queue.Queue()

    # ------------------------------------------------------------------ rank 0
    def start(self):
        assert self.rank == 0, "only rank 0 runs the front-end loop"
        self._thread = threading.Thread(target=self._leader_loop, daemon=True)
        self._thread.start()

    def stop(self):
        self._stop = True
        if self._thread is not None:
            self._thread.join(timeout=60)

    def _drain(self):
        new = []
        while True:
            try:
                new.append(self.engine.inbox.get_nowait())
            except queue.Empty:
                return new

    def step_leader(self):
        """One lock-step iteration on rank 0; returns False once the stop flag went out."""
        eng = self.engine
        new = self._drain()
        specs = []
        for r in new:
            if r.sampling.seed is None and not r.sampling.greedy:
                r.sampling.seed = random.getrandbits(31)
                eng._seed_request(r)
            specs.append({"prompt": r.prompt, "max_new_tokens": r.max_new_tokens, "eos": list(r.eos),
                          "sampling": asdict(r.sampling)})
        obj = [specs, self._stop]
        dist.broadcast_object_list(obj, src=0, group=self.group)
        for r in new:
            eng.waiting.put(r)
        if self._stop:
            return False
        self._maybe_step(bool(new))
        return True

    def _leader_loop(self):
        while self.step_leader():
            pass

    # ------------------------------------------------------------------ ranks > 0
    def step_follower(self):
        eng = self.engine
        obj = [None, None]
        dist.broadcast_object_list(obj, src=0, group=self.group)
        specs, stop = obj
        for sp in specs:
            self.submitted.append(eng.submit(Request(list(sp["prompt"]), sp["max_new_tokens"],
                                                     SamplingParams(**sp["sampling"]), tuple(sp["eos"]))))
        if stop:
            return False
        self._maybe_step(bool(specs), sleep=False)
        return True

    def run_follower(self):
        while self.step_follower():
            pass

    # ------------------------------------------------------------------ shared
    def _maybe_step(self, had_new, sleep=True):
        eng = self.engine
        if eng.running or had_new or not eng.waiting.empty():
            eng.step()
        elif sleep:
            time.sleep(self.idle_sleep)
