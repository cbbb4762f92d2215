"""Tensor-parallel serving: shard a decoder over the ranks of one node (one process per GPU).

Megatron-style split (survey P4; the reference leaves TP to SGLang's engine flag):
  full attention  query heads split (column-parallel ``[q|gate]``/k/v rows), key/value heads split
                  or, with more ranks than KV heads, replicated so every rank holds the KV head of
                  its query heads; ``o_proj`` row-parallel
  gated delta     key / value heads split (``in_proj`` rows, conv channels, ``A_log``, ``dt_bias``);
                  ``out_proj`` row-parallel
  MLP             gate / up rows split, ``down_proj`` row-parallel
  LM head         vocabulary split; greedy tokens come from each rank's (max, argmax) pair
Between sublayers the residual stream is sequence-parallel (``seq_parallel=True``, the default):
rank r keeps only its block of rows of the residual, and after every row-parallel GEMM (partial sum
in this rank's symmetric buffer) one kernel (``csrc/symm.cu``, ``rs_norm_ag``) reduce-scatters the
partials to the owning ranks, adds the residual, applies the next sublayer's RMSNorm and
all-gathers the normalised rows into every rank's input buffer of the next column-parallel GEMM --
(W-1)/W of the activation crosses NVLink each way.  ``seq_parallel=False`` keeps replicated
residuals with a one-shot all-reduce kernel (every rank reads all partials), and ``fused=True`` the
all-reduce inside the GEMM epilogue.  No NCCL on the decode path.
"""
import copy

import torch
import torch.distributed as dist

from ..parallel.symm import SymmetricHeap


def _split(n, world, rank, what):
    if n % world:
        raise ValueError(f"{what} ({n}) must divide evenly over {world} ranks")
    k = n // world
    return rank * k, (rank + 1) * k


def shard_decoder(dec, rank, world):
    """A copy of ``dec`` holding this rank's shard (config head counts divided accordingly)."""
    cfg = dec.cfg
    local = copy.copy(dec)
    local._modules = dict(dec._modules)          # own registries: the original stays untouched
    local._parameters = dict(dec._parameters)
    lcfg = copy.deepcopy(cfg)
    Hq, Hkv, d = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
    q0, q1 = _split(Hq, world, rank, "query heads")
    lcfg.n_heads = q1 - q0
    if Hkv >= world:
        k0, k1 = _split(Hkv, world, rank, "key/value heads")
    else:                                     # replicate: the KV head of this rank's query heads
        if world % Hkv or (Hq // Hkv) % (Hq // world):
            raise ValueError(f"{world} ranks cannot share {Hkv} key/value heads of {Hq} query heads")
        k0 = q0 // (Hq // Hkv)
        k1 = k0 + 1
    lcfg.n_kv_heads = k1 - k0
    F = cfg.intermediate_size
    f0, f1 = _split(F, world, rank, "FFN width")
    lcfg.intermediate_size = f1 - f0
    if cfg.layer_types and "linear_attention" in cfg.layer_types:
        hk0, hk1 = _split(cfg.lin_k_heads, world, rank, "gated-delta key heads")
        hv0, hv1 = _split(cfg.lin_v_heads, world, rank, "gated-delta value heads")
        lcfg.lin_k_heads, lcfg.lin_v_heads = hk1 - hk0, hv1 - hv0
    local.cfg = lcfg
    layers = torch.nn.ModuleList()
    with torch.no_grad():
        for layer in dec.layers:
            L = copy.copy(layer)
            L._parameters = dict(layer._parameters)
            P = lambda t: torch.nn.Parameter(t.contiguous(), requires_grad=False)   # noqa: E731
            L.wgu = P(torch.cat([layer.wgu[f0:f1], layer.wgu[F + f0:F + f1]]))
            L.wdown = P(layer.wdown[:, f0:f1])
            if layer.layer_type == "full_attention":
                qs = 2 * d if cfg.attn_output_gate else d
                wq = layer.wqkv[:Hq * qs].view(Hq, qs, -1)[q0:q1].reshape(-1, layer.wqkv.shape[1])
                wk = layer.wqkv[Hq * qs:Hq * qs + Hkv * d].view(Hkv, d, -1)[k0:k1].reshape(-1, layer.wqkv.shape[1])
                wv = layer.wqkv[Hq * qs + Hkv * d:].view(Hkv, d, -1)[k0:k1].reshape(-1, layer.wqkv.shape[1])
                L.wqkv = P(torch.cat([wq, wk, wv]))
                L.wo = P(layer.wo.view(layer.wo.shape[0], Hq, d)[:, q0:q1].reshape(layer.wo.shape[0], -1))
            else:
                dk, dv = cfg.lin_k_dim, cfg.lin_v_dim
                Hk, Hv = cfg.lin_k_heads, cfg.lin_v_heads
                kd, vd = Hk * dk, Hv * dv
                w = layer.w_in
                rows = [w[hk0 * dk:hk1 * dk], w[kd + hk0 * dk:kd + hk1 * dk], w[2 * kd + hv0 * dv:2 * kd + hv1 * dv],
                        w[2 * kd + vd + hv0 * dv:2 * kd + vd + hv1 * dv],
                        w[2 * kd + 2 * vd + hv0:2 * kd + 2 * vd + hv1],
                        w[2 * kd + 2 * vd + Hv + hv0:2 * kd + 2 * vd + Hv + hv1]]
                L.w_in = P(torch.cat(rows))
                c = layer.conv_w
                L.conv_w = P(torch.cat([c[hk0 * dk:hk1 * dk], c[kd + hk0 * dk:kd + hk1 * dk],
                                        c[2 * kd + hv0 * dv:2 * kd + hv1 * dv]]))
                L.A_log = P(layer.A_log[hv0:hv1])
                L.dt_bias = P(layer.dt_bias[hv0:hv1])
                L.w_out = P(layer.w_out[:, hv0 * dv:hv1 * dv])
            layers.append(L)
    local.layers = layers
    V = cfg.vocab_size
    vp = (V + world - 1) // world
    lm = dec.lm_weight
    sl = lm[rank * vp:min(V, (rank + 1) * vp)]
    if sl.shape[0] < vp:     # pad the last shard; padded rows never win the argmax
        sl = torch.cat([sl, torch.zeros(vp - sl.shape[0], sl.shape[1], dtype=sl.dtype, device=sl.device)])
    local.lm_shard = sl.contiguous()
    local.vocab_offset = rank * vp
    local.vocab_size_full = V
    return local


class TPContext:
    """Per-process TP state: the process group, the symmetric buffers of the row-parallel
    all-reduces and the vocabulary-parallel greedy pick.

    ``seq_parallel=True`` (default): the runtime keeps this rank's block of residual rows and calls
    ``reduce_norm`` after every row-parallel GEMM (reduce-scatter + residual + RMSNorm + all-gather
    in one kernel, two barriers).
    ``seq_parallel=False``: the GEMM writes this rank's partial into its symmetric buffer and a
    one-shot all-reduce kernel pulls every rank's partial over NVLink and adds the residual.
    ``fused=True``: every row-parallel GEMM runs the all-reduce in its own epilogue
    (``csrc/gemm_sm100.cu``, ``gemm_bf16_allreduce``): partial tiles are pushed over NVLink into
    every rank's receive buffer as they come out of the tensor cores and each rank sums its rows
    as soon as all ranks' tiles have arrived -- one kernel per layer output.  Measured on 2 B200s it
    is still about twice as slow as the two-kernel path on decode and prefill shapes, so it is
    opt-in until its exchange is faster."""

    def __init__(self, max_rows, hidden, group=None, fused=False, seq_parallel=True):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.heap = SymmetricHeap(group)
        self.max_rows, self.hidden = max_rows, hidden
        self.fused = fused and hidden % 64 == 0
        self.seq_parallel = seq_parallel and not self.fused and hidden % 8 == 0 and hidden <= 8192
        self.turn = 0
        if self.seq_parallel:
            self.part = self.heap.alloc(max_rows * hidden, torch.bfloat16)
            self.gath = self.heap.alloc(max_rows * hidden, torch.bfloat16)
            self.sp_ctr = torch.zeros(2, dtype=torch.int32, device="cuda")
        if self.fused:
            self.tiles_cap = -(-max_rows // 128) * -(-hidden // 256)
            self.recv = self.heap.alloc(2 * self.world * max_rows * hidden, torch.bfloat16)
            self.flags = self.heap.alloc(2 * self.tiles_cap * 4, torch.int32)
            self.ctr_done = torch.zeros(2, dtype=torch.int32, device="cuda")
            # split-K scratch for skinny (decode) products: one 128 x 256 fp32 tile per SM
            sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
            self.ws = torch.empty(sms * 128 * 256, dtype=torch.float32, device="cuda")
            self.tile_ctr = torch.zeros(self.tiles_cap * 4, dtype=torch.int32, device="cuda")
        elif not self.seq_parallel:
            self.bufs = [self.heap.alloc(max_rows * hidden, torch.bfloat16) for _ in range(2)]

    def own_rows(self, rows):
        """(first row, count) of the residual rows this rank owns out of ``rows``."""
        per = -(-rows // self.world)
        r0 = min(rows, self.rank * per)
        return r0, min(rows, r0 + per) - r0

    def shard(self, x):
        """This rank's rows of a replicated residual stream."""
        r0, n = self.own_rows(x.shape[0])
        return x[r0:r0 + n].contiguous()

    def reduce_norm(self, a, w, xs, norm_w, eps):
        """Row-parallel output at a sequence-parallel boundary: ``xs += rows of sum_r a_r w_r^T``
        (this rank's rows, in place) and the all-gathered ``RMSNorm(x) * norm_w`` of every row,
        returned as a view of this rank's gather buffer (valid until the next call)."""
        from ..ops import blocks
        M = a.shape[0]
        if M > self.max_rows:
            raise RuntimeError(f"{M} rows exceed the TP buffers ({self.max_rows})")
        part = self.part.local[:M * self.hidden].view(M, self.hidden)
        blocks.gemm(blocks.TN, a, w, part)
        r0, n = self.own_rows(M)
        assert xs.shape[0] == n
        blocks.ext().symm_rs_norm_ag(self.part.ptrs, self.gath.ptrs, self.heap.flags.ptrs, self.rank, self.sp_ctr,
                                     r0, xs, norm_w, eps, self.heap.err)
        return xs, self.gath.local[:M * self.hidden].view(M, self.hidden)

    def next_buffer(self, rows):
        if rows > self.max_rows:
            raise RuntimeError(f"{rows} rows exceed the TP buffers ({self.max_rows})")
        if not hasattr(self, "bufs"):      # replicated-residual calls in sequence-parallel mode (collective)
            self.bufs = [self.heap.alloc(self.max_rows * self.hidden, torch.bfloat16) for _ in range(2)]
        b = self.bufs[self.turn]
        self.turn ^= 1
        return b, b.local[:rows * self.hidden].view(rows, self.hidden)

    def row_parallel(self, x, w, residual):
        """residual + sum over ranks of x_r w_r^T."""
        from ..ops import blocks
        rows = x.shape[0]
        if self.fused:
            if rows > self.max_rows:
                raise RuntimeError(f"{rows} rows exceed the TP buffers ({self.max_rows})")
            out = torch.empty(rows, self.hidden, dtype=torch.bfloat16, device=x.device)
            blocks.ext().gemm_allreduce(x.contiguous(), w, out, residual.contiguous(), self.recv.ptrs,
                                        self.flags.ptrs, self.rank, self.ctr_done, self.max_rows, self.tiles_cap,
                                        self.ws, self.tile_ctr)
            return out
        buf, part = self.next_buffer(rows)
        blocks.gemm(blocks.TN, x, w, part)
        return self.allreduce(buf, x.shape[0], residual)

    def allreduce(self, buf, rows, residual):
        out = torch.empty(rows, self.hidden, dtype=torch.bfloat16, device=residual.device)
        self.heap.allreduce_(buf, 0, rows * self.hidden, out.view(-1), residual.contiguous().view(-1))
        return out

    def gather(self, t):
        out = torch.empty((self.world,) + tuple(t.shape), dtype=t.dtype, device=t.device)
        dist.all_gather_into_tensor(out, t.contiguous(), group=self.group)
        return out
