"""Failure detection for multi-rank training and serving, all on the host.

The reference relies on NCCL's watchdog (a collective times out after the process-group timeout)
and on every rank taking the same early returns (``train/checkpoint.py:64-67``).  This module adds
what a long job needs to fail fast and cleanly instead of hanging:

* ``Heartbeat``: every rank publishes ``(time, step)`` in the process group's key-value store from
  a background thread; the same thread reads the other ranks' entries.  A rank whose entry stops
  advancing for ``timeout`` seconds, or that published a failure, is reported.  ``check()`` (call
  it between steps, before the next collective is launched) raises ``RankFailure`` naming the
  ranks, so the survivors exit before they block in a collective that can never complete.
* ``fail(reason)``: a rank that hits an error it cannot recover from publishes it, so the others
  stop at their next ``check()`` rather than at the process-group timeout.
* ``check_device()``: the CUDA kernels' bounded waits record a non-zero error word instead of
  hanging (GEMM mbarriers, symmetric-memory barriers); this turns a recorded code into
  ``DeviceWaitTimeout`` on the host.

Recovery is restart-based: the launcher (``torchrun --max-restarts``) starts the job again and the
trainer resumes from the last checkpoint, whose files ``checkpoint.py`` verifies against a manifest
of sizes and SHA-256 digests (``verify_manifest``) before loading.
"""
import threading
import time

import torch.distributed as dist


class RankFailure(RuntimeError):
    def __init__(self, failed):
        self.failed = dict(failed)
        super().__init__("rank failure detected: " + "; ".join(f"rank {r}: {why}" for r, why in sorted(failed.items())))


class DeviceWaitTimeout(RuntimeError):
    pass


def default_store():
    """A store client of its own for the heartbeat thread (store clients are not shared between
    threads): a new connection to the rendezvous TCPStore, else the process group's store."""
    import datetime
    import os
    host, port = os.environ.get("MASTER_ADDR"), os.environ.get("MASTER_PORT")
    if host and port:
        try:
            return dist.TCPStore(host, int(port), is_master=False, timeout=datetime.timedelta(seconds=30))
        except Exception:
            pass
    from torch.distributed import distributed_c10d as c10d
    return c10d._get_default_store()


class Heartbeat:
    """Background liveness exchange through the process group's store (``dist`` must be initialised,
    or pass ``store``, ``rank`` and ``world``)."""

    def __init__(self, interval=0.5, timeout=10.0, store=None, rank=None, world=None, prefix="trida/hb"):
        self.store = store if store is not None else default_store()
        self.rank = dist.get_rank() if rank is None else rank
        self.world = dist.get_world_size() if world is None else world
        self.interval, self.timeout, self.prefix = interval, timeout, prefix
        self.step = 0
        self.status = "ok"
        self.failed = {}
        self._seen = {}                 # rank -> (last value, local time it last changed)
        self._stop = threading.Event()
        self._wake = threading.Event()
        self._published = threading.Event()
        self._lock = threading.Lock()
        self._thread = None

    def _key(self, r):
        return f"{self.prefix}/{r}"

    def _publish(self):
        self.store.set(self._key(self.rank), f"{self.status}|{time.time():.3f}|{self.step}")

    def start(self):
        self._publish()
        now = time.monotonic()
        for r in range(self.world):
            self._seen[r] = (None, now)
        self._thread = threading.Thread(target=self._run, name="trida-heartbeat", daemon=True)
        self._thread.start()
        return self

    def beat(self, step):
        """Record training progress (called by the loop; the thread publishes it)."""
        self.step = step

    def fail(self, reason):
        """Tell the other ranks this one is going down (published by the heartbeat thread, which
        owns the store connection; waits up to a few intervals for it to go out)."""
        self.status = "failed:" + str(reason).replace("|", "/")
        self._published.clear()
        if self._thread is not None and self._thread.is_alive():
            self._wake.set()
            self._published.wait(timeout=4 * self.interval + 1)

    def _poll(self):
        now = time.monotonic()
        for r in range(self.world):
            if r == self.rank:
                continue
            try:
                # a missing key would block in store.get: ask the store whether it exists first
                if not self.store.check([self._key(r)]):
                    val = None
                else:
                    val = self.store.get(self._key(r)).decode()
            except Exception as e:      # the store itself is gone (its host rank died)
                with self._lock:
                    self.failed.setdefault(r, f"store unreachable ({type(e).__name__})")
                continue
            if val is not None and val.startswith("failed:"):
                with self._lock:
                    self.failed.setdefault(r, val.split("|", 1)[0][len("failed:"):] or "failed")
                continue
            last, since = self._seen.get(r, (None, now))
            if val != last:
                self._seen[r] = (val, now)
            elif now - since > self.timeout:
                with self._lock:
                    self.failed.setdefault(r, f"no heartbeat for {now - since:.1f} s")

    def _run(self):
        while not self._stop.is_set():
            self._wake.wait(self.interval)
            self._wake.clear()
            if self._stop.is_set():
                break
            try:
                self._publish()
                self._published.set()
            except Exception:
                pass
            self._poll()

    def check(self):
        """Raise ``RankFailure`` if any other rank failed or went silent."""
        with self._lock:
            failed = dict(self.failed)
        if failed:
            raise RankFailure(failed)

    def stop(self):
        self._stop.set()
        self._wake.set()
        if self._thread is not None:
            self._thread.join(timeout=5 * self.interval + 1)


def check_device():
    """Raise ``DeviceWaitTimeout`` if a CUDA kernel's bounded wait gave up (host sync)."""
    from ..ops import blocks
    try:
        blocks.check_device_errors()
    except RuntimeError as e:
        raise DeviceWaitTimeout(str(e)) from None
