"""Sharded data parallelism over flat parameter / gradient buffers.

Every optimizer group's parameters live in ONE contiguous bf16 buffer (the parameters are views
into it) with a matching fp32 gradient buffer (each parameter's ``main_grad``), both padded to a
multiple of ``world * 64`` elements.  The optimizer state -- fp32 first/second moments and, with
``fp32_master``, fp32 master weights -- exists only for this rank's 1/world shard, as in the
reference's FSDP2 full-shard setup (``train/distributed.py:32-59``: bf16 compute weights, fp32
gradient reduction).

Step: reduce-scatter (average) the fp32 gradients -> global grad norm of the shards (one scalar
all-reduce, no host sync) -> fused AdamW on the shard with the clip coefficient read on the device
-> all-gather the updated bf16 shard into every rank's full buffer.  On one GPU the collectives
vanish and the same kernels run over the whole buffer.  The gradient reduce-scatter is bucketed
per layer and can be issued from backward hooks, overlapping communication with the backward of
earlier layers (``overlap=True``).

Full shard (``full_shard=True``, the reference's FSDP ``fully_shard`` of every decoder layer,
``train/distributed.py:32-59``): a decoder layer's bf16 weights persist only as this rank's 1/world
shard; ``ParamRing`` gathers a layer into a local buffer right before it runs (prefetching the
next layer on a side stream while the current one computes) and drops it afterwards -- again in
backward -- unless ``keep_params`` keeps the gathered weights from forward to backward (the
reference's ``--fsdp_keep_params``).  The update then touches only the local shard.
"""
import os

import torch
import torch.distributed as dist

from ..ops._ext import ext
from .symm import RING_CLOSE_SLOT, SHARD_CLOSE_SLOT

ALIGN = 64
GATHER_ENGINE = os.environ.get("TRIDA_GATHER", "copy")    # full-shard gathers: copy engines or a P2P kernel


def _world():
    return dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1


def _rank():
    return dist.get_rank() if dist.is_available() and dist.is_initialized() else 0


class FlatGroup:
    """One optimizer group flattened into contiguous buffers (symmetric peer buffers when a heap
    is given, so the fused collectives can read and write them from every rank)."""

    def __init__(self, params, lr_scale, world, rank, fp32_master, device, heap=None, stream=False,
                 full_shard=False):
        self.params = list(params)
        self.full_shard = full_shard
        self.lr_scale = lr_scale
        self.world, self.rank = world, rank
        n = sum(p.numel() for p in self.params)
        unit = world * ALIGN
        self.numel = n
        self.padded = (n + unit - 1) // unit * unit
        self.shard = self.padded // world
        dtype = self.params[0].dtype if self.params else torch.bfloat16
        self.flat_sym = self.grad_sym = self.shard_sym = None
        self.stream = stream        # gradients live in a shared ring slot only while this group's backward runs
        if full_shard:
            self.flat = torch.zeros(self.padded, dtype=dtype, device=device)   # staging only, freed below
        elif heap is not None:
            self.flat_sym = heap.alloc(self.padded, dtype)
            self.flat = self.flat_sym.local
        else:
            self.flat = torch.zeros(self.padded, dtype=dtype, device=device)
        self.grad = None
        if not stream:
            if heap is not None:
                self.grad_sym = heap.alloc(self.padded, torch.float32)
                self.grad = self.grad_sym.local
            else:
                self.grad = torch.zeros(self.padded, dtype=torch.float32, device=device)
        off = 0
        self.offsets = []
        with torch.no_grad():
            for p in self.params:
                k = p.numel()
                view = self.flat[off:off + k].view_as(p)
                view.copy_(p.data)
                p.data = view
                p.main_grad = self.grad[off:off + k].view(p.shape) if not stream else None
                self.offsets.append((off, k))
                off += k
        lo = rank * self.shard
        self.lo, self.hi = lo, lo + self.shard
        self.grad_shard = (torch.zeros(self.shard, dtype=torch.float32, device=device) if world > 1 or stream
                           else None)
        if full_shard:
            # keep only this rank's shard (in peer memory when the gathers run over NVLink)
            if heap is not None:
                self.shard_sym = heap.alloc(self.shard, dtype)
                self.pshard = self.shard_sym.local
            else:
                self.pshard = torch.empty(self.shard, dtype=dtype, device=device)
            self.pshard.copy_(self.flat[lo:lo + self.shard])
            if world > 1:
                self.flat = None
                self.unbind_params()
            else:
                self.pshard = self.flat       # one rank: the shard is the whole buffer, params stay bound
        self.master = None
        if fp32_master:
            self.master = self.shard_param().float().clone()
        self.m = torch.zeros(self.shard, dtype=torch.float32, device=device)
        self.v = torch.zeros(self.shard, dtype=torch.float32, device=device)

    def shard_grad(self):
        return self.grad if (self.world == 1 and not self.stream) else self.grad_shard

    def shard_param(self):
        if self.full_shard:
            return self.pshard if self.world > 1 else self.flat[self.lo:self.hi]
        return self.flat[self.lo:self.hi]

    def bind_params(self, buf):
        """Point every parameter's data into ``buf`` (this group's gathered flat weights)."""
        for p, (off, k) in zip(self.params, self.offsets):
            p.data = buf[off:off + k].view(p.shape)

    def unbind_params(self):
        """Leave every parameter without storage of its own (a zero-stride view of one element),
        so nothing reads stale gathered weights."""
        for p in self.params:
            p.data = torch.zeros(1, dtype=p.dtype, device=p.device).expand(p.shape)

    def bind_grads(self, buf):
        """Point every parameter's ``main_grad`` into ``buf`` (a zeroed ring slot)."""
        for p, (off, k) in zip(self.params, self.offsets):
            p.main_grad = buf[off:off + k].view(p.shape)

    def unbind_grads(self):
        for p in self.params:
            p.main_grad = None


class GradRing:
    """Two fp32 gradient slots shared by the streamed groups (one decoder layer each).  A group's
    slot is bound to its parameters' ``main_grad`` by the first weight gradient its backward
    writes.  Backward runs the layers one after another, so when the next group binds a slot the
    previous group's gradients are complete: its reduce-scatter into the fp32 shard is issued then,
    on a side stream with a quarter of the SMs' worth of CTAs, and runs under the next layer's
    backward.  A slot is zeroed for reuse only after the event of the reduction that last read it
    (whose closing barrier guarantees every rank has finished reading it).  Full-size fp32
    gradients exist for at most two layers."""

    RS_BLOCKS = 64

    def __init__(self, opt, size, device):
        self.opt = opt
        self.slots = []
        for _ in range(2):
            if opt.fused:
                b = opt.heap.alloc(size, torch.float32)
                self.slots.append((b.local, b))
            else:
                self.slots.append((torch.zeros(size, dtype=torch.float32, device=device), None))
        self.free = [0, 1]
        self.held = {}
        self.ready = [None, None]
        cuda = torch.device(device).type == "cuda"
        self.comm = torch.cuda.Stream(device=device) if (cuda and opt.world > 1) else None
        self.partial = torch.zeros(self.RS_BLOCKS, dtype=torch.float32, device=device)
        self.done = torch.zeros(1, dtype=torch.int32, device=device) if cuda else None

    def acquire(self, gi):
        if gi in self.held:
            return
        for other in list(self.held):          # the previous layer's backward has finished
            self.release(other)
        si = self.free.pop(0)
        if self.ready[si] is not None:
            torch.cuda.current_stream().wait_event(self.ready[si])
            self.ready[si] = None
        g = self.opt.groups[gi]
        buf = self.slots[si][0][:g.padded]
        buf.zero_()
        g.bind_grads(buf)
        self.held[gi] = si

    def release(self, gi):
        si = self.held.pop(gi, None)
        if si is None:
            return
        o = self.opt
        g = o.groups[gi]
        local, sym = self.slots[si]
        if self.comm is not None:
            self.comm.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(self.comm):
                self._reduce(g, local, sym)
                ev = torch.cuda.Event()
                ev.record(self.comm)
            self.ready[si] = ev
        else:
            self._reduce(g, local, sym)
        g.unbind_grads()
        self.free.append(si)

    def _reduce(self, g, local, sym):
        o = self.opt
        if o.world == 1:
            g.grad_shard.add_(local[:g.padded])
        elif o.fused:
            h = o.heap
            ext().symm_rs_sumsq(sym.ptrs, h.flags.ptrs, h.rank, h.next_epoch(1), g.lo, g.shard, 1.0 / o.world,
                                g.grad_shard, self.partial, h.err, accumulate=True, done=self.done,
                                close_slot=RING_CLOSE_SLOT)
        else:
            tmp = torch.empty(g.shard, dtype=torch.float32, device=local.device)
            avg = dist.get_backend(o.pg) == "nccl"
            dist.reduce_scatter_tensor(tmp, local[:g.padded], op=dist.ReduceOp.AVG if avg else dist.ReduceOp.SUM,
                                       group=o.pg)
            if not avg:
                tmp.div_(o.world)
            g.grad_shard.add_(tmp)

    def flush(self):
        for gi in list(self.held):
            self.release(gi)
        if self.comm is not None:
            torch.cuda.current_stream().wait_stream(self.comm)


class LayerGradStream:
    """Explicit per-layer control of the ring (layer index -> group): ``acquire(i)`` binds layer
    i's slot, ``release(i)`` reduces it.  The training blocks bind slots lazily instead."""

    def __init__(self, ring, layer_groups):
        self.ring, self.map = ring, layer_groups    # layer index -> optimizer group index

    def acquire(self, i):
        if i in self.map:
            self.ring.acquire(self.map[i])

    def release(self, i):
        if i in self.map:
            self.ring.release(self.map[i])



class ParamRing:
    """Gathered weights of full-shard layer groups.  Two local buffers serve as a ring: ``fetch(i,
    nxt)`` waits for layer i's gather (issuing it now if it was not prefetched), binds its
    parameters, and starts gathering layer ``nxt`` into the other buffer on a side stream;
    ``done(i)`` marks the compute stream's last use of layer i's buffer, which the next gather into
    that buffer waits for.  With ``keep`` (and always on CPU, where plain autograd saves the weight
    tensors themselves) every layer gets its own buffer and a gather stays valid until the next
    optimizer step (weights kept from forward to backward).

    With the fused collectives a gather is one peer-to-peer copy per rank's shard on the copy
    engines (``symm_gather_copy``: no SM is taken from the compute it overlaps), or with
    ``TRIDA_GATHER=kernel`` one ``symm_gather`` kernel of P2P loads; ``all_gather_into_tensor``
    otherwise; on one rank nothing is gathered."""

    GATHER_BLOCKS = 32     # CTAs of a gather kernel: enough for NVLink, few SMs taken from compute

    def __init__(self, opt, layer_groups, keep=False):
        self.opt, self.map = opt, dict(layer_groups)
        self.groups = opt.groups
        first = self.groups[self.map[next(iter(self.map))]]
        dev = first.pshard.device
        self.keep = keep or dev.type != "cuda"
        size = max(self.groups[gi].padded for gi in self.map.values())
        nbuf = len(self.map) if self.keep else 2
        self.bufs = [torch.empty(size, dtype=first.pshard.dtype, device=dev) for _ in range(nbuf)]
        self.owner = [None] * nbuf        # group whose weights the buffer holds (valid until the next step)
        self.ready = [None] * nbuf        # gather-complete events
        self.free = [None] * nbuf         # last-use events on the compute stream
        self.cuda = dev.type == "cuda"
        self.stream = torch.cuda.Stream(device=dev) if self.cuda else None
        self.active = opt.world > 1
        self.cur = None                   # buffer of the layer bound last
        self.order = list(self.map.values())

    def _held(self, gi):
        for bi, o in enumerate(self.owner):
            if o == gi:
                return bi
        return None

    def _gather_into(self, g, dst):
        o = self.opt
        if o.fused and GATHER_ENGINE == "copy":
            ext().symm_gather_copy(g.shard_sym.ptrs, o.rank, g.shard, dst)
        elif o.fused:
            ext().symm_gather(g.shard_sym.ptrs, o.rank, g.shard, dst, self.GATHER_BLOCKS)
        else:
            dist.all_gather_into_tensor(dst, g.pshard, group=o.pg)

    def _gather(self, gi, bi):
        """Gather layer group gi into buffer bi (side stream) after the buffer's last use."""
        g = self.groups[gi]
        dst = self.bufs[bi][:g.padded]
        if self.cuda:
            self.stream.wait_stream(torch.cuda.current_stream())   # shard updates of the last step
            if self.free[bi] is not None:
                self.stream.wait_event(self.free[bi])
            with torch.cuda.stream(self.stream):
                self._gather_into(g, dst)
                ev = torch.cuda.Event()
                ev.record(self.stream)
            self.ready[bi] = ev
        else:
            self._gather_into(g, dst)
        self.owner[bi] = gi

    def fetch(self, layer, nxt=None):
        if not self.active or layer not in self.map:
            return
        gi = self.map[layer]
        bi = self._held(gi)
        if bi is None:
            bi = self.order.index(gi) if self.keep else (0 if self.cur is None else 1 - self.cur)
            self._gather(gi, bi)
        self.cur = bi
        if self.cuda and self.ready[bi] is not None:
            torch.cuda.current_stream().wait_event(self.ready[bi])
        self.groups[gi].bind_params(self.bufs[bi][:self.groups[gi].padded])
        if nxt is not None and nxt in self.map:
            gn = self.map[nxt]
            if self._held(gn) is None:
                self._gather(gn, self.order.index(gn) if self.keep else 1 - bi)

    def done(self, layer):
        if not self.active or layer not in self.map or self.keep or not self.cuda:
            return
        bi = self._held(self.map[layer])
        if bi is not None:
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream())
            self.free[bi] = ev

    def invalidate(self):
        """Every gathered copy is stale after an optimizer step."""
        self.owner = [None] * len(self.owner)

    def materialize(self):
        """Bind every full-shard group to freshly gathered weights of its own (checkpointing)."""
        if not self.active:
            return
        for gi in self.map.values():
            g = self.groups[gi]
            full = torch.empty(g.padded, dtype=g.pshard.dtype, device=g.pshard.device)
            self._gather_into(g, full)
            g.bind_params(full)

    def release_all(self):
        if not self.active:
            return
        for gi in self.map.values():
            self.groups[gi].unbind_params()


def _adamw_torch(param, master, grad, m, v, lr, b1, b2, eps, wd, step, coef):
    """CPU statement of the fused AdamW kernel (torch.optim.AdamW math, fp32 moments)."""
    p = master if master is not None else param.float()
    g = grad * coef
    p.mul_(1 - lr * wd)
    m.mul_(b1).add_(g, alpha=1 - b1)
    v.mul_(b2).addcmul_(g, g, value=1 - b2)
    bc1, bc2 = 1 - b1 ** step, 1 - b2 ** step
    p.addcdiv_(m, v.sqrt().div_(bc2 ** 0.5).add_(eps), value=-lr / bc1)
    param.copy_(p)


class ShardedAdamW:
    """AdamW over flat sharded buffers; torch.optim-like surface (``param_groups``, ``step``,
    ``zero_grad``, ``state_dict``)."""

    NB = 296          # partial-sum blocks of the fused reduce-scatter (2 per SM)

    def __init__(self, groups, lr, betas=(0.9, 0.95), weight_decay=0.0, eps=1e-8, fp32_master=False,
                 device=None, process_group=None, comm="nccl", full_shard=False, keep_params=False):
        self.world, self.rank = _world(), _rank()
        self.pg = process_group
        device = device or groups[0]["params"][0].device
        # comm="fused": gradient reduce-scatter + norm + AdamW + parameter all-gather run as
        # symmetric-memory kernels over NVLink (csrc/symm.cu); "nccl": NCCL collectives.
        self.fused = comm == "fused" and self.world > 1 and torch.device(device).type == "cuda"
        self.heap = None
        if self.fused:
            from .symm import SymmetricHeap
            self.heap = SymmetricHeap(process_group)
        groups = [g for g in groups if g["params"]]
        self.groups = [FlatGroup(g["params"], g.get("lr_scale", 1.0), self.world, self.rank, fp32_master, device,
                                 self.heap, stream=bool(g.get("stream")),
                                 full_shard=full_shard and "layer" in g)
                       for g in groups]
        self.param_ring = None
        if full_shard:
            layer_groups = {gg["layer"]: i for i, gg in enumerate(groups) if "layer" in gg}
            if not layer_groups:
                raise ValueError("full_shard needs per-layer parameter groups (param_groups(per_layer=True))")
            self.param_ring = ParamRing(self, layer_groups, keep=keep_params)
        if self.fused:
            self.partials = self.heap.alloc(len(self.groups) * self.NB, torch.float32)
        self._clipped = False
        self.ring = None
        streamed = [g for g in self.groups if g.stream]
        if streamed:
            self.ring = GradRing(self, max(g.padded for g in streamed), device)
            for gi, g in enumerate(self.groups):
                if g.stream:
                    for p in g.params:   # bound lazily by the first gradient written in a backward
                        p._grad_acquire = (lambda gi=gi: self.ring.acquire(gi))
            self.layer_stream = LayerGradStream(
                self.ring, {gg["layer"]: i for i, gg in enumerate(groups) if gg.get("stream")})
        self.param_groups = [{"params": g.params, "lr": lr * g.lr_scale, "lr_scale": g.lr_scale}
                             for g in self.groups]
        self.defaults = {"lr": lr, "betas": betas, "weight_decay": weight_decay, "eps": eps}
        self.betas, self.wd, self.eps = betas, weight_decay, eps
        self.step_count = 0
        self.norm = torch.zeros(1, dtype=torch.float32, device=device)
        self.coef = torch.zeros(1, dtype=torch.float32, device=device)
        self._partial = None

    # ---- gradients -----------------------------------------------------------------------
    def zero_grad(self, set_to_none=True):
        for g in self.groups:
            if g.stream:
                g.grad_shard.zero_()
            else:
                g.grad.zero_()
            for p in g.params:
                p.grad = None

    def collect_autograd_grads(self):
        """Fold ordinary ``.grad`` tensors (CPU path, plain torch modules) into the flat fp32
        buffers; the CUDA blocks write ``main_grad`` directly and leave ``.grad`` unset."""
        for g in self.groups:
            if g.stream:
                continue
            for p in g.params:
                if p.grad is not None:
                    p.main_grad.add_(p.grad.float())
                    p.grad = None

    def reduce_gradients(self):
        """Average gradients across ranks into each rank's shard (reduce-scatter)."""
        self.collect_autograd_grads()
        self._clipped = False
        if self.ring is not None:
            self.ring.flush()       # a layer whose input needed no gradient never released its slot
            for g in self.groups:   # plain-autograd (CPU) gradients of streamed groups
                if not g.stream:
                    continue
                if not any(p.grad is not None for p in g.params):
                    continue
                flat = torch.zeros(g.padded, dtype=torch.float32, device=g.grad_shard.device)
                for p, (off, k) in zip(g.params, g.offsets):
                    if p.grad is not None:
                        flat[off:off + k].add_(p.grad.float().reshape(-1))
                        p.grad = None
                if self.world == 1:
                    g.grad_shard.add_(flat)
                else:
                    tmp = torch.empty(g.shard, dtype=torch.float32, device=flat.device)
                    dist.reduce_scatter_tensor(tmp, flat, group=self.pg)
                    g.grad_shard.add_(tmp.div_(self.world))
        if self.world == 1:
            return
        if self.fused:
            h = self.heap
            for i, g in enumerate(self.groups):
                if g.stream:
                    continue
                ext().symm_rs_sumsq(g.grad_sym.ptrs, h.flags.ptrs, h.rank, h.next_epoch(1), g.lo, g.shard,
                                    1.0 / self.world, g.grad_shard,
                                    self.partials.local[i * self.NB:(i + 1) * self.NB], h.err)
            return
        avg = dist.get_backend(self.pg) == "nccl"   # gloo has no AVG reduction
        for g in self.groups:
            if g.stream:
                continue
            dist.reduce_scatter_tensor(g.grad_shard, g.grad, op=dist.ReduceOp.AVG if avg else dist.ReduceOp.SUM,
                                       group=self.pg)
            if not avg:
                g.grad_shard.div_(self.world)

    def _local_norm(self, shards, max_norm):
        if self.norm.is_cuda:
            ext().grad_norm(shards, max_norm, self.norm, self.coef)
        else:
            self.norm.copy_(torch.sqrt(sum((s.double() ** 2).sum() for s in shards)).float().view(1))
            torch.clamp(max_norm / (self.norm + 1e-6), max=1.0, out=self.coef)

    def clip_grad_norm_(self, max_norm):
        """Global L2 norm of the (reduced) gradients; writes the clip coefficient on the device and
        returns the norm as a device tensor (no host sync)."""
        shards = [g.shard_grad() for g in self.groups]
        self._clipped = True
        if self.world == 1:
            self._local_norm(shards, max_norm)
            return self.norm[0]
        if self.fused and self.ring is None:
            h = self.heap
            ext().symm_norm_coef(self.partials.ptrs, h.flags.ptrs, h.rank, h.next_epoch(3),
                                 len(self.groups) * self.NB, max_norm, self.norm, self.coef, h.err)
            return self.norm[0]
        # partial sums of squares on each rank, summed across ranks, then the coefficient
        sq = torch.zeros(1, dtype=torch.float32, device=self.norm.device)
        self._local_norm(shards, 1e30)  # norm of this rank's shards
        sq.copy_(self.norm * self.norm)
        dist.all_reduce(sq, group=self.pg)
        torch.sqrt(sq, out=self.norm)
        torch.clamp(max_norm / (self.norm + 1e-6), max=1.0, out=self.coef)
        return self.norm[0]

    # ---- update ----------------------------------------------------------------------------
    def _step_full_shard(self, g, lr, b1, b2):
        """AdamW on a full-shard group: only this rank's shard changes (no all-gather)."""
        if self.coef.is_cuda:
            ext().adamw(g.shard_param(), g.master, g.shard_grad(), g.m, g.v, lr, b1, b2, self.eps, self.wd,
                        self.step_count, self.coef)
        else:
            _adamw_torch(g.shard_param(), g.master, g.shard_grad(), g.m, g.v, lr, b1, b2, self.eps, self.wd,
                         self.step_count, self.coef)

    def step(self):
        self.step_count += 1
        b1, b2 = self.betas
        if not self._clipped and self.param_ring is not None:
            self.coef.fill_(1.0)
        if self.fused:
            h = self.heap
            coef = self.coef if self._clipped else None
            for g, pg in zip(self.groups, self.param_groups):
                if g.full_shard:
                    self._step_full_shard(g, pg["lr"], b1, b2)
                    continue
                ext().symm_adamw_ag(g.flat_sym.ptrs, h.flags.ptrs, h.rank, h.next_epoch(2), g.lo, g.shard,
                                    g.grad_shard, g.master, g.m, g.v, pg["lr"], b1, b2, self.eps, self.wd,
                                    self.step_count, coef, h.done, h.err)
            if self.param_ring is not None:
                # no rank gathers a shard that a peer is still updating
                ext().symm_barrier(h.flags.ptrs, h.rank, h.next_epoch(SHARD_CLOSE_SLOT), SHARD_CLOSE_SLOT, h.err)
                self.param_ring.invalidate()
            return
        if self.param_ring is not None:
            self.param_ring.invalidate()
        for g, pg in zip(self.groups, self.param_groups):
            if g.full_shard:
                self._step_full_shard(g, pg["lr"], b1, b2)
                continue
            lr = pg["lr"]
            if self.coef.is_cuda:
                ext().adamw(g.shard_param(), g.master, g.shard_grad(), g.m, g.v, lr, b1, b2, self.eps, self.wd,
                            self.step_count, self.coef)
            else:
                _adamw_torch(g.shard_param(), g.master, g.shard_grad(), g.m, g.v, lr, b1, b2, self.eps, self.wd,
                             self.step_count, self.coef)
        if self.world > 1:
            for g in self.groups:
                if g.full_shard:
                    continue
                # in place: this rank's input is its own slice of the output buffer
                dist.all_gather_into_tensor(g.flat, g.flat[g.lo:g.hi], group=self.pg)

    # ---- checkpoint ------------------------------------------------------------------------
    def state_dict(self):
        return {"step": self.step_count, "world": self.world, "rank": self.rank,
                "groups": [{"m": g.m, "v": g.v, "master": g.master, "lo": g.lo, "hi": g.hi,
                            "numel": g.numel} for g in self.groups]}

    def load_state_dict(self, sd):
        if sd["world"] != self.world:
            raise ValueError(f"optimizer state was saved with world {sd['world']}, running with {self.world}")
        self.step_count = sd["step"]
        for g, s in zip(self.groups, sd["groups"]):
            g.m.copy_(s["m"])
            g.v.copy_(s["v"])
            if g.master is not None and s["master"] is not None:
                g.master.copy_(s["master"])
