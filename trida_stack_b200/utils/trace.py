"""Step tracing for training (``--profile_steps``) and per-request decode traces for serving.

Training: inside the window ``[--profile_start, --profile_start + --profile_steps)`` every phase of
a step (data transfer, forward, backward, optimizer) is wrapped in an NVTX range (visible to
Nsight / ncu) and bracketed by CUDA events on the current stream; at the end of each traced step
the device-timed phase durations are appended as one JSON line to
``<--profile_dir>/rank<R>.jsonl``.  Outside the window the tracer does nothing.

Serving: with ``$TRIDA_TRACE_JSONL`` set, the engine appends one JSON line per finished request
(prompt / output lengths, forwards, acceptance histogram, time to first token, latency).
"""
import json
import os
import time

import torch


class StepTracer:
    def __init__(self, start=0, steps=0, out_dir="profile", rank=0, device=None):
        self.start, self.steps, self.rank = start, steps, rank
        self.out_dir = out_dir
        self.cuda = device is not None and torch.device(device).type == "cuda"
        self.step = None
        self._marks = []
        self._fh = None

    def active(self, step):
        return self.steps > 0 and self.start <= step < self.start + self.steps

    def begin(self, step):
        self.step = step if self.active(step) else None
        self._marks = []
        if self.step is not None:
            self._mark("begin")

    def _mark(self, name):
        if self.cuda:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self._marks.append((name, ev))
        else:
            self._marks.append((name, time.perf_counter()))

    def phase(self, name):
        """Context manager: NVTX range + event marks around one phase of a traced step."""
        tracer = self

        class _P:
            def __enter__(self_):
                if tracer.step is not None:
                    if tracer.cuda:
                        torch.cuda.nvtx.range_push(f"step{tracer.step}:{name}")
                    tracer._mark(name + ":start")

            def __exit__(self_, *exc):
                if tracer.step is not None:
                    tracer._mark(name + ":end")
                    if tracer.cuda:
                        torch.cuda.nvtx.range_pop()
                return False
        return _P()

    def end(self, **extra):
        """Close a traced step: write its phase durations (ms, device-timed on CUDA)."""
        if self.step is None:
            return None
        self._mark("end")
        if self.cuda:
            torch.cuda.synchronize()

        def dt(a, b):
            return a.elapsed_time(b) if self.cuda else (b - a) * 1e3
        rec = {"step": self.step, "rank": self.rank,
               "total_ms": round(dt(self._marks[0][1], self._marks[-1][1]), 3)}
        pending = {}
        for name, t in self._marks:             # phases may repeat (gradient accumulation): sum them
            if name.endswith(":start"):
                pending[name[:-6]] = t
            elif name.endswith(":end") and name[:-4] in pending:
                ph = name[:-4]
                rec[ph + "_ms"] = round(rec.get(ph + "_ms", 0.0) + dt(pending.pop(ph), t), 3)
        rec.update(extra)
        if self._fh is None:
            os.makedirs(self.out_dir, exist_ok=True)
            self._fh = open(os.path.join(self.out_dir, f"rank{self.rank}.jsonl"), "a")
        self._fh.write(json.dumps(rec) + "\n")
        self._fh.flush()
        self.step = None
        return rec


class RequestTrace:
    """Appends one JSON line per finished request to ``path`` (``$TRIDA_TRACE_JSONL``)."""

    def __init__(self, path):
        self.path = path
        self._fh = open(path, "a")

    @classmethod
    def from_env(cls):
        p = os.environ.get("TRIDA_TRACE_JSONL")
        return cls(p) if p else None

    def write(self, req, mode):
        rec = {"rid": req.rid, "mode": mode, "prompt_tokens": len(req.prompt), "output_tokens": len(req.output),
               "forwards": req.forwards, "tokens_per_forward": round(len(req.output) / max(req.forwards, 1), 3),
               "accept_hist": list(req.accept_hist), "finish_reason": req.finish_reason,
               "ttft_s": None if req.t_first is None else round(req.t_first - req.t_submit, 4),
               "latency_s": None if req.t_done is None else round(req.t_done - req.t_submit, 4)}
        self._fh.write(json.dumps(rec) + "\n")
        self._fh.flush()


def kernel_breakdown(fn, steps=1, top=16, out=None):
    """Per-kernel device-time shares of ``steps`` calls of ``fn`` (CUDA activity of the PyTorch
    profiler), printed as a table to ``out`` (stderr by default) and returned as rows of
    (share, total ms, launches, kernel).  For finding where a step's time goes; the numbers are
    taken under a profiler and are not benchmark values."""
    import sys

    from torch.profiler import ProfilerActivity, profile
    cuda = torch.cuda.is_available()
    if cuda:
        torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA] if cuda else [ProfilerActivity.CPU]) as prof:
        for _ in range(steps):
            fn()
        if cuda:
            torch.cuda.synchronize()
    ev = [(e.device_time_total, e.count, e.key) for e in prof.key_averages() if e.device_time_total > 0]
    ev.sort(reverse=True)
    tot = sum(t for t, _, _ in ev) or 1.0
    rows = [(t / tot, t / 1e3, c, k) for t, c, k in ev[:top]]
    out = out or sys.stderr
    print(f"kernel breakdown: {tot / 1e3:.1f} ms device time over {steps} step(s)", file=out)
    for share, ms, c, k in rows:
        print(f"{100 * share:5.1f}% {ms:9.2f} ms x{c:5d}  {k[:100]}", file=out)
    return rows
