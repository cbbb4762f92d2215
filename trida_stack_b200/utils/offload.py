"""Activation offload: tensors saved for backward go to pinned host memory and come back on demand.

The reference wraps its checkpointed decoder layers in ``torch.autograd.graph.save_on_cpu``
(``train/models/block_diffusion.py:773-781``, ``--activation_offload``) so that the per-layer
checkpoint inputs -- the only activations kept between forward and backward when every layer is
recomputed -- live in host RAM at long context.  Here the same tensors move on a dedicated copy
stream, so the device-to-host copies overlap the next layers' forward instead of blocking it:

* pack (forward): the producing stream records an event, the copy stream waits on it and copies
  the tensor into a pinned host buffer taken from a size-keyed pool; the device tensor is marked as
  used by the copy stream (``record_stream``) so the caching allocator cannot hand its memory out
  before the copy has read it.
* unpack (backward): the copy stream copies the host buffer into a fresh device tensor after the
  offload copy has finished; the consuming stream waits on that copy's event.  The host buffer
  goes back to the pool once the upload has been issued and the event has completed.

Tensors smaller than ``min_bytes`` (norm statistics, indices) and CPU tensors stay where they are.
"""
import torch


class _Offloaded:
    __slots__ = ("host", "done", "device", "shape", "dtype", "key")

    def __init__(self, host, done, device, shape, dtype, key):
        self.host, self.done, self.device, self.shape, self.dtype, self.key = host, done, device, shape, dtype, key


class PinnedPool:
    """Pinned host buffers reused by size (bytes), so a training run allocates them once."""

    def __init__(self):
        self.free = {}
        self.pending = []     # (event, key, buffer): uploads in flight; recycled once they complete

    def take(self, nbytes):
        self.reclaim()
        lst = self.free.get(nbytes)
        if lst:
            return lst.pop()
        return torch.empty(nbytes, dtype=torch.uint8, pin_memory=torch.cuda.is_available())

    def give_back(self, nbytes, buf, event=None):
        if event is None:
            self.free.setdefault(nbytes, []).append(buf)
        else:
            self.pending.append((event, nbytes, buf))

    def reclaim(self):
        keep = []
        for ev, n, buf in self.pending:
            if ev.query():
                self.free.setdefault(n, []).append(buf)
            else:
                keep.append((ev, n, buf))
        self.pending = keep

    def nbytes(self):
        return sum(b.numel() for lst in self.free.values() for b in lst)


class ActivationOffload(torch.autograd.graph.saved_tensors_hooks):
    """Context manager: saved-for-backward CUDA tensors of at least ``min_bytes`` go to pinned host
    memory during forward and are copied back when backward unpacks them."""

    def __init__(self, pool=None, min_bytes=1 << 20, stream=None):
        self.pool = pool if pool is not None else PinnedPool()
        self.min_bytes = min_bytes
        self._stream = stream
        self.offloaded_bytes = 0
        super().__init__(self._pack, self._unpack)

    def _copy_stream(self, device):
        if self._stream is None:
            self._stream = torch.cuda.Stream(device=device)
        return self._stream

    def _pack(self, t):
        if not t.is_cuda or t.numel() * t.element_size() < self.min_bytes:
            return t
        nbytes = t.numel() * t.element_size()
        src = t.contiguous()
        host = self.pool.take(nbytes)
        cs = self._copy_stream(t.device)
        cs.wait_stream(torch.cuda.current_stream(t.device))
        with torch.cuda.stream(cs):
            host.copy_(src.view(-1).view(torch.uint8), non_blocking=True)
            done = torch.cuda.Event()
            done.record(cs)
        src.record_stream(cs)
        self.offloaded_bytes += nbytes
        return _Offloaded(host, done, t.device, t.shape, t.dtype, nbytes)

    def _unpack(self, h):
        if not isinstance(h, _Offloaded):
            return h
        cs = self._copy_stream(h.device)
        cur = torch.cuda.current_stream(h.device)
        out = torch.empty(h.key, dtype=torch.uint8, device=h.device)
        cs.wait_event(h.done)
        cs.wait_stream(cur)          # `out` was allocated on the consuming stream
        with torch.cuda.stream(cs):
            out.copy_(h.host, non_blocking=True)
            up = torch.cuda.Event()
            up.record(cs)
        cur.wait_event(up)
        self.pool.give_back(h.key, h.host, up)
        return out.view(h.dtype).view(h.shape)
