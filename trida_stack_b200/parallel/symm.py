"""Symmetric peer memory: per-rank CUDA buffers mapped into every other rank of one node.

``SymmetricHeap(group)`` allocates buffers with ``cudaMalloc`` on every rank (same size), exchanges
their CUDA IPC handles over the process group and opens the peers' handles, so the collective
kernels of ``csrc/symm.cu`` can load from and store to any rank's buffer over NVLink.  Each heap
owns one flag array per rank (epochs for the kernels' bounded barriers) and host-side epoch
counters that every rank advances identically.
"""
import torch
import torch.distributed as dist

from ..ops._ext import ext

NSLOTS = 8          # barrier slots: all-reduce, reduce-scatter, AdamW close, norm, streamed reduce-scatter close,
                    # full-shard update close, tensor-parallel sequence-parallel open and close
RING_CLOSE_SLOT = 4
SHARD_CLOSE_SLOT = 5
MAXR = 8


class SymBuffer:
    """One symmetric allocation: ``local`` (tensor view of this rank's buffer) and ``ptrs``
    (device addresses of every rank's buffer, index = rank)."""

    def __init__(self, heap, numel, dtype):
        C = ext()
        self.numel, self.dtype = numel, dtype
        nbytes = numel * torch.empty((), dtype=dtype).element_size()
        self._own = C.symm_malloc(max(nbytes, 256))
        dev = torch.cuda.current_device()
        self.local = C.symm_tensor(self._own, numel, dtype, dev)
        handles = heap._exchange(C.symm_handle(self._own))
        self.ptrs, self._opened = [], []
        for r, h in enumerate(handles):
            if r == heap.rank:
                self.ptrs.append(self._own)
            else:
                p = C.symm_open(h)
                self.ptrs.append(p)
                self._opened.append(p)

    def close(self):
        C = ext()
        for p in self._opened:
            C.symm_close(p)
        self._opened = []
        if self._own:
            C.symm_free(self._own)
            self._own = 0


class SymmetricHeap:
    def __init__(self, group=None):
        if not (dist.is_available() and dist.is_initialized()):
            raise RuntimeError("SymmetricHeap needs an initialised process group")
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > MAXR:
            raise ValueError(f"symmetric memory spans at most {MAXR} ranks of one node")
        self.buffers = []
        self.flags = SymBuffer(self, NSLOTS * MAXR, torch.int32)
        self.err = torch.zeros(1, dtype=torch.int32, device="cuda")
        self.done = torch.zeros(1, dtype=torch.int32, device="cuda")
        self.ar_ctr = torch.zeros(2, dtype=torch.int32, device="cuda")   # all-reduce epoch, finished CTAs
        self.epochs = [0] * NSLOTS
        dist.barrier(group)

    def _exchange(self, handle):
        out = [None] * self.world
        dist.all_gather_object(out, handle, group=self.group)
        return out

    def alloc(self, numel, dtype):
        b = SymBuffer(self, numel, dtype)
        self.buffers.append(b)
        return b

    def next_epoch(self, slot):
        self.epochs[slot] += 1
        return self.epochs[slot]

    def check(self):
        """Raise if a bounded device wait gave up (host sync)."""
        code = int(self.err.item())
        if code:
            self.err.zero_()
            raise RuntimeError(f"symmetric-memory barrier timed out (code {code})")

    def allreduce_(self, buf, off, n, out, residual=None):
        """out = sum over ranks of buf[off:off+n] (+ residual); ``buf`` already holds this rank's
        contribution.  Callers alternate between two buffers (or halves) from call to call.  The
        epoch lives on the device, so the call can be captured in a CUDA graph."""
        ext().symm_allreduce(buf.ptrs, self.flags.ptrs, self.rank, self.ar_ctr, off, n, residual, out, self.err)

    def close(self):
        torch.cuda.synchronize()
        dist.barrier(self.group)
        for b in self.buffers:
            b.close()
        self.flags.close()
        self.buffers = []
