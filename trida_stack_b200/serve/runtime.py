"""Slot-based inference runtime: KV / gated-delta caches and the batched canvas step.

The decode step of the self-speculative engine is one forward over a *canvas* of ``blk`` rows per
active request: rows ``< n_clean`` are token-causal, the remaining rows see the whole canvas, and
every row sees the request's cached prefix.  Full-attention layers append the canvas K/V to the
slot's cache rows ``pos .. pos+blk`` (a later commit keeps the first ``adv``); gated-delta layers
run the recurrence from the slot's cached state (clean rows read their own state, the rest read
the state after the last row) and the commit advances that state and the conv window by ``adv``
rows.  Reference semantics: ``inference/zoro-1/mlx/trida_mlx/model.py:282-330`` (canvas GDN),
``:461-470`` (canvas mask), ``:486-507`` (commit); the reference serves through vLLM / SGLang
(``inference/zoro-1/vllm/vllm_native_diffusion/qwen3_5_diffusion.py:1337-2094``).

A prompt is prefilled as a sequence of fully causal canvas steps (``n_clean = blk``) of at most
``PREFILL_CHUNK`` rows each, so prefill and decode share one code path.  On CUDA every op runs on
the extension's kernels; on CPU the same step is stated in PyTorch (the oracle of the GPU path and
the runtime of the CPU tests).
"""
import math
import os

import torch
import torch.nn.functional as F

from ..ops import gdn_reference as G
from ..ops import reference as R

PREFILL_CHUNK = 64
PAGE = 64                 # positions per KV page
# TRIDA_GUARDS=1: bounds guards on every step -- slot ids, token ids, positions, commit advances and
# page-table ownership on the host, then the device error word and the logits after the step (a
# device sync, which is why they are off unless asked).  A race or a bad index then surfaces as a
# named error at the call that caused it instead of a corrupted cache or a fault in a later kernel.
# The reference keeps the same kind of opt-in guards in its vLLM self-spec backend
# (inference/zoro-1/vllm/vllm_native_diffusion/qwen3_5_diffusion.py:92-95, 1146, 1882-1888).
GUARDS = os.environ.get("TRIDA_GUARDS") == "1"


class Runtime:
    def __init__(self, decoder, max_slots=8, max_len=4096, device=None, tp=None, kv_pages=None):
        """``tp``: a ``serve.tp.TPContext`` when ``decoder`` is this rank's tensor-parallel shard
        (``serve.tp.shard_decoder``); greedy decoding only.  ``max_len`` caps one request's
        positions; on CUDA the full-attention KV lives in a pool of ``kv_pages`` pages of 64
        positions shared by all slots (default: enough for every slot at ``max_len``), so a few long
        requests and many short ones share the same memory."""
        self.dec = decoder
        self.tp = tp
        self.guards = GUARDS
        self.cfg = cfg = decoder.cfg
        p = next(decoder.parameters())
        self.device = torch.device(device) if device is not None else p.device
        self.dtype = p.dtype
        self.cuda = self.device.type == "cuda"
        self.max_slots, self.max_len = max_slots, max_len
        self.kinds = [l.layer_type for l in decoder.layers]
        d, Hkv = cfg.head_dim, cfg.n_kv_heads
        self.kc, self.vc, self.ssm, self.win = {}, {}, {}, {}
        nslot = max_slots + 1              # + one scratch slot that pads graph-captured batches
        self.dummy = max_slots
        # paged KV (CUDA): page tables [slot, max_len / 64] into per-layer pools [pages, 64, Hkv, d];
        # the CPU statement keeps a dense [slot, max_len] cache
        self.paged = self.cuda
        self.max_pages = (max_len + PAGE - 1) // PAGE
        if self.paged:
            self.n_pages = kv_pages or nslot * self.max_pages
            self.pages = KVPages(self.n_pages, nslot, self.max_pages, pin=True)
            self.ptab = torch.zeros(nslot, self.max_pages, dtype=torch.int32, device=self.device)
        for i, kind in enumerate(self.kinds):
            if kind == "full_attention":
                shape = (self.n_pages, PAGE, Hkv, d) if self.paged else (nslot, max_len, Hkv, d)
                self.kc[i] = torch.zeros(*shape, dtype=self.dtype, device=self.device)
                self.vc[i] = torch.zeros(*shape, dtype=self.dtype, device=self.device)
            else:
                Cc = 2 * cfg.lin_k_heads * cfg.lin_k_dim + cfg.lin_v_heads * cfg.lin_v_dim
                # fp32 state per value head [k, v]; the per-token scan kernels (TRIDA_GDN_CANVAS=scan)
                # keep it in their thread-native order instead
                self.ssm[i] = torch.zeros(nslot, cfg.lin_v_heads, cfg.lin_k_dim, cfg.lin_v_dim,
                                          dtype=torch.float32, device=self.device)
                self.win[i] = torch.zeros(nslot, cfg.conv_kernel - 1, Cc, dtype=self.dtype, device=self.device)
        self.pos = [0] * max_slots
        # RoPE position = cache index + delta (3-D RoPE prompts advance positions more slowly than
        # cache rows; an optional offset shifts every generated token)
        self.rope_delta = [0] * max_slots
        self.free = list(range(max_slots))[::-1]
        self.pending = None
        self._graphs = None
        if self.cuda:
            from ..ops import blocks
            from ..ops._ext import ext
            self.C = ext()
            self.cos_t, self.sin_t = blocks.rope_tables(max_len + 64, cfg.rotary_dim, cfg.rope_theta, self.device)
            self.blocks = blocks
            self._gdn_f32 = {i: (decoder.layers[i].A_log.float().contiguous(),
                                 decoder.layers[i].dt_bias.float().contiguous()) for i in self.ssm}
            import os
            # canvas gated-delta step: the chunked form on tensor cores (commit from the stored U
            # rows), or the per-token scan kernels (commit re-runs the accepted rows)
            self.gdn_tc = os.environ.get("TRIDA_GDN_CANVAS", "tc") == "tc"
            # gated RMSNorm in the canvas kernel's epilogue (TRIDA_GDN_FUSED_NORM=1) or as its own
            # kernel after it (default: measured 0.26 + 0.03 ms against 0.37 ms fused at 64 x 63 rows)
            self.gdn_fused_norm = os.environ.get("TRIDA_GDN_FUSED_NORM", "0") == "1"
            # canvas attention on tensor cores (TMA-gathered query tiles, tcgen05 S / PV with TMEM
            # accumulators), or the split-K warp-MMA kernel (TRIDA_CANVAS_ATTN=mma)
            self.attn_tc = os.environ.get("TRIDA_CANVAS_ATTN", "tc") == "tc"
            self.err = blocks.device_error_word(self.device)

    # ------------------------------------------------------------------ slots
    def alloc(self):
        if not self.free:
            raise RuntimeError("no free cache slot")
        s = self.free.pop()
        self.pos[s] = 0
        self.rope_delta[s] = 0
        for i in self.ssm:
            self.ssm[i][s].zero_()
            self.win[i][s].zero_()
        return s

    def release(self, s):
        self.pos[s] = 0
        self.free.append(s)
        if self.paged and s != self.dummy:
            self.pages.release(s)

    def _ensure_pages(self, slots, blk):
        """Pages for positions [0, pos + blk) of every slot (the scratch slot of padded graph
        batches writes positions [0, blk)); the device page table is refreshed when it changed."""
        if not self.paged or not self.kc:
            return
        changed = False
        for s in list(slots) + [self.dummy]:
            changed |= self.pages.ensure(s, (self.pos[s] if s < self.max_slots else 0) + blk)
        if changed:
            self.ptab.copy_(self.pages.table, non_blocking=True)

    # ------------------------------------------------------------------ public steps
    @torch.no_grad()
    def prefill(self, slots, prompts, vis=None, pos_offset=0):
        """Feed equal-length prompts into fresh slots; returns fp32 logits of each last token [B, V].

        ``vis`` (vision-language prompts): per slot ``None`` or ``(features [n_img, D], pos3 [3, L])``
        -- the image features replace the embeddings of the prompt's image tokens in order and the
        prompt rows use 3-D RoPE; later tokens continue from the prompt's largest position + 1
        (+ ``pos_offset``)."""
        L = len(prompts[0])
        assert all(len(p) == L for p in prompts) and L >= 1
        ids = torch.tensor(prompts, dtype=torch.long, device=self.device)
        ang = inject = None
        if vis is not None and any(v is not None for v in vis):
            pos3 = torch.stack([v[1] if v is not None else torch.arange(L).expand(3, -1) for v in vis]).to(self.device)
            ang = self.dec.rope_angles(pos3) if hasattr(self.dec, "rope_angles") else None
            img = ids == self.cfg.image_token_id
            feats = torch.cat([v[0] for v in vis if v is not None]).to(self.device, self.dtype)
            if int(img.sum()) != feats.shape[0]:
                raise ValueError(f"{int(img.sum())} image tokens but {feats.shape[0]} image features")
            fidx = torch.full(ids.shape, -1, dtype=torch.long, device=self.device)
            fidx[img] = torch.arange(feats.shape[0], device=self.device)
            inject = (fidx, feats)
            for b, s in enumerate(slots):
                self.rope_delta[s] = int(pos3[b].max()) + 1 - L
        out = None
        for c0 in range(0, L, PREFILL_CHUNK):
            n = min(PREFILL_CHUNK, L - c0)
            last = c0 + n == L
            extra = {}
            if inject is not None:
                extra = {"inject": (inject[0][:, c0:c0 + n], inject[1]),
                         "rope_ang": ang[:, c0:c0 + n] if ang is not None else None}
            logits = self.canvas(slots, ids[:, c0:c0 + n], n, rows=(n - 1, n) if last else (0, 0), **extra)
            self.commit(slots, [n] * len(slots))
            if last:
                out = logits[:, 0]
        for s in slots:
            self.rope_delta[s] += pos_offset
        return out

    def use_graphs(self, buckets=(1, 2, 4, 8, 16, 32, 64, 128)):
        """Replay decode-shaped canvases (all rows read out) and their commits from CUDA graphs,
        one per (padded batch, canvas) shape; batches are padded with the scratch slot."""
        assert self.cuda, "CUDA graphs need the CUDA runtime"
        self.graph_buckets = sorted(b for b in buckets if b <= self.max_slots) or [self.max_slots]
        if self.graph_buckets[-1] < self.max_slots:
            self.graph_buckets.append(self.max_slots)
        self._graphs = {}

    @torch.no_grad()
    def canvas(self, slots, tokens, n_clean, rows=None, inject=None, rope_ang=None, greedy=False):
        """One forward over a [B, blk] canvas per slot.  Returns fp32 logits [B, r1 - r0, V] for the
        canvas rows ``rows = (r0, r1)`` (all rows by default).  Call ``commit`` afterwards.  With
        graphs on, the returned tensor is a static buffer valid until the next canvas.  ``greedy``
        (CUDA, no tensor parallelism, all rows): the LM head's argmax is fused into its GEMM and the
        result only carries the greedy tokens (``argmax`` reads them); no logits are written."""
        greedy = greedy and self.cuda and self.tp is None and rows is None
        assert self.pending is None, "commit the previous canvas first"
        B = len(slots)
        blk = len(tokens[0])
        if self.guards:
            self._guard_canvas(slots, tokens, n_clean, blk)
        for s in slots:
            if self.pos[s] + blk > self.max_len:
                raise RuntimeError(f"slot {s}: sequence exceeds the cache length {self.max_len}")
        self._ensure_pages(slots, blk)
        if self.guards and self.paged:
            self.pages.check([s for s in range(self.max_slots) if s not in self.free] + [self.dummy])
        r0, r1 = rows if rows is not None else (0, blk)
        if self._graphs is not None and (r0, r1) == (0, blk) and inject is None and rope_ang is None:
            out = self._canvas_graph(slots, tokens, n_clean, greedy)
        else:
            out = self._canvas_eager(slots, tokens, n_clean, B, blk, r0, r1, inject, rope_ang, greedy)
        if self.guards:
            self._guard_after(out)
        return out

    def _canvas_eager(self, slots, tokens, n_clean, B, blk, r0, r1, inject, rope_ang, greedy):
        tokens = torch.as_tensor(tokens, dtype=torch.long, device=self.device)
        st = _Step(self, slots, B, blk, n_clean)
        st.inject, st.rope_ang = inject, rope_ang
        x = self._forward(st, tokens)
        self.pending = st
        if r1 <= r0:
            return torch.empty(B, 0, self.cfg.vocab_size, device=self.device)
        if greedy:
            return GreedyTokens(self._greedy_tokens(x).view(B, blk))
        normed = isinstance(x, _SeqPar)
        x = self._rms(x, self.dec.norm) if normed else x
        h = x.view(B, blk, -1)[:, r0:r1].reshape(B * (r1 - r0), -1)
        return self._logits(h, normed).view(B, r1 - r0, -1)

    def _greedy_tokens(self, x):
        """Greedy tokens of hidden rows: final norm, then the LM-head GEMM with its argmax epilogue."""
        h = self._rms(x, self.dec.norm)
        out = torch.empty(h.shape[0], dtype=torch.long, device=h.device)
        self.C.gemm_argmax(h, self.dec.lm_weight, out)
        return out

    def argmax(self, logits):
        """Greedy tokens [B, rows] of fp32 logits [B, rows, V] (the argmax kernel on CUDA; taken
        from the captured graph when ``logits`` is the graph's output)."""
        if isinstance(logits, GreedyTokens):
            return logits.tokens
        g = self.pending
        if isinstance(g, _Graph) and g.logits is not None and logits.data_ptr() == g.logits.data_ptr():
            return g.am[:logits.shape[0]]
        if not self.cuda:
            out = logits.argmax(-1)
        else:
            out = torch.empty(logits.shape[:-1], dtype=torch.long, device=logits.device)
            self.C.argmax_rows(logits.reshape(-1, logits.shape[-1]), out.view(-1))
        if self.tp is not None:
            # vocabulary-parallel: every rank's (max, global index); the first maximum wins
            val = logits.gather(-1, out.unsqueeze(-1)).squeeze(-1)
            pair = torch.stack([val, (out + self.dec.vocab_offset).float()], -1)
            allp = self.tp.gather(pair)                                      # [W, ..., 2]
            best = allp[..., 0].argmax(0, keepdim=True)
            out = allp[..., 1].gather(0, best).squeeze(0).long()
        return out

    def conf_argmax(self, logits):
        """Greedy token and its softmax probability per row of fp32 logits [B, R, V] (``R`` may be a
        row slice of a canvas's logits): one fused pass on CUDA; vocabulary-parallel shards combine
        their (max, normaliser, index) triples across ranks."""
        if not self.cuda:
            p = torch.softmax(logits.float(), -1)
            conf, idx = p.max(-1)
            return idx, conf
        B, R, _ = logits.shape
        idx = torch.empty(B, R, dtype=torch.long, device=logits.device)
        mx = torch.empty(B, R, dtype=torch.float32, device=logits.device)
        z = torch.empty(B, R, dtype=torch.float32, device=logits.device)
        self.C.conf_argmax_rows(logits, idx, mx, z)
        if self.tp is None:
            return idx, 1.0 / z
        trip = torch.stack([mx, z, (idx + self.dec.vocab_offset).float()], -1)
        allt = self.tp.gather(trip)                                          # [W, B, R, 3]
        M = allt[..., 0].max(0).values
        Z = (allt[..., 1] * torch.exp(allt[..., 0] - M[None])).sum(0)
        best = allt[..., 0].argmax(0, keepdim=True)
        return allt[..., 2].gather(0, best).squeeze(0).long(), 1.0 / Z

    def discard(self):
        """Drop the last canvas without committing any row (a denoise round)."""
        self.pending = None

    def _forward(self, st, tokens):
        x = self.dec.embed_tokens(tokens.reshape(-1)) if self.cuda else self.dec.embed[tokens.reshape(-1)]
        if getattr(st, "inject", None) is not None:
            fidx, feats = st.inject
            sel = fidx.reshape(-1) >= 0
            if bool(sel.any()):
                x = x.clone()
                x[sel] = feats[fidx.reshape(-1)[sel]].to(x.dtype)
        layers = self.dec.layers
        seqpar = self.tp is not None and getattr(self.tp, "seq_parallel", False)
        if seqpar:     # this rank's residual rows; the first input norm runs on the replicated embedding
            x = _SeqPar(self.tp.shard(x), self._rms(x, layers[0].input_norm), layers[0].input_norm)
        for i, layer in enumerate(layers):
            if seqpar:
                x.next = layer.post_norm
            if self.kinds[i] == "full_attention":
                x = self._attn(st, i, layer, x)
            else:
                x = self._gdn(st, i, layer, x)
            if seqpar:
                x.next = layers[i + 1].input_norm if i + 1 < len(layers) else self.dec.norm
            x = self._mlp(layer, x)
        return x

    def _canvas_graph(self, slots, tokens, n_clean, greedy=False):
        B, blk = len(slots), len(tokens[0])
        Bp = next(b for b in self.graph_buckets if b >= B)
        key = (Bp, blk, n_clean, greedy)
        g = self._graphs.get(key)
        if g is None:
            g = self._graphs[key] = _Graph(self, Bp, blk, n_clean, greedy)
        pad = Bp - B
        g.host_tok[:B] = torch.as_tensor(tokens, dtype=torch.long)
        g.host_tok[B:] = 0
        g.host_slot[:] = torch.tensor(list(slots) + [self.dummy] * pad, dtype=torch.int32)
        pos = [self.pos[s] for s in slots] + [0] * pad
        g.host_pos[:] = torch.tensor(pos, dtype=torch.int32)
        rp = torch.tensor([self.pos[s] + self.rope_delta[s] for s in slots] + [0] * pad, dtype=torch.int32)
        g.host_rowpos[:] = (rp[:, None] + torch.arange(blk, dtype=torch.int32)[None]).reshape(-1)
        g.st.tokens.copy_(g.host_tok, non_blocking=True)
        g.st.slot_t.copy_(g.host_slot, non_blocking=True)
        g.st.pos_t.copy_(g.host_pos, non_blocking=True)
        g.st.rowpos32.copy_(g.host_rowpos, non_blocking=True)
        g.fwd.replay()
        g.st.slots = list(slots)
        self.pending = g
        return GreedyTokens(g.am[:B]) if greedy else g.logits[:B]

    # ------------------------------------------------------------------ guards (TRIDA_GUARDS=1)
    def _guard_canvas(self, slots, tokens, n_clean, blk):
        if len(set(slots)) != len(slots):
            raise RuntimeError(f"[guards] a slot appears twice in one canvas step: {list(slots)}")
        for s in slots:
            if not 0 <= s < self.max_slots:
                raise RuntimeError(f"[guards] slot {s} outside [0, {self.max_slots})")
            if s in self.free:
                raise RuntimeError(f"[guards] slot {s} is not allocated (released or never taken)")
        if not 1 <= n_clean <= blk:
            raise RuntimeError(f"[guards] n_clean={n_clean} outside [1, canvas rows {blk}]")
        t = torch.as_tensor(tokens)
        if t.dim() != 2 or t.shape[0] != len(slots) or t.shape[1] != blk:
            raise RuntimeError(f"[guards] tokens of shape {tuple(t.shape)} for {len(slots)} slots x {blk} rows")
        lo, hi = int(t.min()), int(t.max())          # a device sync when the tokens live on the GPU
        if lo < 0 or hi >= self.cfg.vocab_size:
            raise RuntimeError(f"[guards] token ids span [{lo}, {hi}] outside the vocabulary [0, {self.cfg.vocab_size})")

    def _guard_attention(self, i, st, q, o, blk):
        """Canvas attention output of layer ``i``: every row written and finite (device sync)."""
        code = int(self.err.item())
        bad = ~torch.isfinite(o.float()).all(-1)          # [rows, heads]
        if code or bool(bad.any()):
            rows = bad.any(-1).nonzero().flatten()[:8].tolist()
            pos = st.pos_t.tolist() if hasattr(st, "pos_t") else None
            raise RuntimeError(
                f"[guards] canvas attention, layer {i}: error word {code}, {int(bad.sum())} non-finite "
                f"(row, head) outputs, first rows {rows}; q finite {bool(torch.isfinite(q).all())}, "
                f"B={st.B} blk={blk} n_clean={st.n_clean} max_keys={st.max_keys} "
                f"pos=[{min(pos) if pos else None}, {max(pos) if pos else None}] kernel="
                f"{'tc' if self.attn_tc else 'mma'}")

    def _guard_after(self, logits):
        """Device error word and finite logits after a step (device sync)."""
        if self.cuda:
            code = int(self.err.item())
            if code:
                raise RuntimeError(f"[guards] a kernel of this step gave up a bounded wait (code {code})")
        if torch.is_tensor(logits) and logits.numel() and not bool(torch.isfinite(logits).all()):
            raise RuntimeError("[guards] non-finite logits after the canvas step")
        if isinstance(logits, GreedyTokens) and logits.tokens.numel():
            t = logits.tokens
            lo, hi = int(t.min()), int(t.max())
            if lo < 0 or hi >= self.cfg.vocab_size:
                raise RuntimeError(f"[guards] greedy tokens span [{lo}, {hi}] outside the vocabulary "
                                   f"(an all-NaN logits row has no argmax)")

    @torch.no_grad()
    def commit(self, slots, adv):
        """Keep the first ``adv[b]`` canvas rows of every slot (1 <= adv <= n_clean)."""
        st = self.pending
        if self.guards:
            if st is None:
                raise RuntimeError("[guards] commit without a pending canvas")
            nc = st.st.n_clean if isinstance(st, _Graph) else st.n_clean
            pend = st.st.slots if isinstance(st, _Graph) else st.slots
            if list(slots) != list(pend):
                raise RuntimeError(f"[guards] commit for slots {list(slots)} but the pending canvas has {list(pend)}")
            if len(adv) != len(slots) or not all(1 <= a <= nc for a in adv):
                raise RuntimeError(f"[guards] commit advances {list(adv)} outside [1, n_clean={nc}]")
        if isinstance(st, _Graph):
            g = st
            assert list(slots) == g.st.slots and all(1 <= a <= g.st.n_clean for a in adv)
            g.host_adv[:len(adv)] = torch.tensor(adv, dtype=torch.int32)
            g.host_adv[len(adv):] = 1
            g.adv.copy_(g.host_adv, non_blocking=True)
            g.com.replay()
            for b, s in enumerate(slots):
                self.pos[s] += adv[b]
            self.pending = None
            return
        assert st is not None and list(slots) == list(st.slots)
        assert all(1 <= a <= st.n_clean for a in adv)
        if self.cuda:
            adv_t = torch.tensor(adv, dtype=torch.int32, device=self.device)
        self._commit_kernels(st, adv_t if self.cuda else None, adv)
        for b, s in enumerate(st.slots):
            self.pos[s] += adv[b]
        self.pending = None

    def _commit_kernels(self, st, adv_t, adv=None):
        cfg = self.cfg
        for i, rec in st.gdn.items():
            layer = self.dec.layers[i]
            if self.cuda and self.gdn_tc:
                mixed, kbuf, ubuf, gbuf, proj = rec
                self.C.gdn_commit_tc(kbuf, ubuf, gbuf, self.ssm[i], st.slot_t, adv_t, st.blk, cfg.lin_v_heads,
                                     self.err)
                Cc = mixed.shape[1]
                self.C.conv_commit(proj[:, :Cc], st.blk, self.win[i], st.slot_t, adv_t)
            elif self.cuda:
                mixed, ga, gb, proj, prep = rec
                a_log, dtb = self._gdn_f32[i]
                self.C.gdn_commit(mixed, ga, gb, a_log, dtb, prep, self.ssm[i], st.slot_t, adv_t, st.blk,
                                  cfg.lin_k_heads, cfg.lin_v_heads, cfg.lin_k_dim ** -0.5)
                Cc = mixed.shape[1]
                self.C.conv_commit(proj[:, :Cc], st.blk, self.win[i], st.slot_t, adv_t)
            else:
                q, k, v, g, beta, conv_in = rec
                for b, s in enumerate(st.slots):
                    S = self.ssm[i][s].clone()
                    for t in range(adv[b]):
                        S, _ = G._step(S, q[b, t], k[b, t], v[b, t], g[b, t], beta[b, t])
                    self.ssm[i][s] = S
                    K1 = cfg.conv_kernel - 1
                    self.win[i][s] = conv_in[b, adv[b]:adv[b] + K1]

    # ------------------------------------------------------------------ layers
    def _rms(self, x, w):
        if isinstance(x, _SeqPar):          # normalised and gathered by the previous sublayer's output
            if x.norm is not w:
                raise RuntimeError("sequence-parallel stream normalised with another weight")
            return x.h
        if self.cuda:
            h = torch.empty_like(x)
            self.C.rmsnorm_fwd(x, w, self.cfg.eps, h)
            return h
        return R.rmsnorm(x, w, self.cfg.eps)

    def _lin(self, x, w, residual=None):
        if isinstance(residual, _SeqPar):
            xs, h = self.tp.reduce_norm(x, w, residual.xs, residual.next, self.cfg.eps)
            return _SeqPar(xs, h, residual.next)
        if self.tp is not None and residual is not None:
            return self.tp.row_parallel(x, w, residual)
        if self.cuda:
            out = torch.empty(x.shape[0], w.shape[0], dtype=x.dtype, device=x.device)
            if residual is None:
                self.blocks.gemm(self.blocks.TN, x, w, out)
            else:
                self.blocks.gemm(self.blocks.TN, x, w, out, residual, 1.0, 1.0)
            return out
        y = x @ w.t()
        return y if residual is None else residual + y

    def _mlp(self, layer, x):
        h = self._rms(x, layer.post_norm)
        if self.cuda:
            M, F2 = h.shape[0], layer.wgu.shape[0]
            a = torch.empty(M, F2 // 2, dtype=h.dtype, device=h.device)
            if F2 % 128 == 0 and 2 * (-(-M // 128)) * (F2 // 256) >= self._sm_count():
                # enough 128 x 256 tiles to fill the GPU without splitting K: SwiGLU in the epilogue
                gu = torch.empty(M, F2, dtype=h.dtype, device=h.device)
                self.C.gemm_swiglu(h, layer.wgu, gu, a)
            else:
                gu = self._lin(h, layer.wgu)
                self.C.swiglu_fwd(gu, a)
        else:
            a = R.swiglu(self._lin(h, layer.wgu))
        return self._out(a, layer.wdown, x, getattr(layer, "post_mlp_norm", None))

    def _sm_count(self):
        if getattr(self, "_sms", None) is None:
            self._sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        return self._sms

    def _out(self, a, w, x, post_norm):
        """Sub-block output: ``x + a w^T`` (residual fused into the GEMM epilogue), or GLM's
        ``x + RMSNorm(a w^T)`` when the layer normalises its outputs."""
        if post_norm is None:
            return self._lin(a, w, x)
        if self.tp is not None:
            raise NotImplementedError("tensor parallelism for layers with output norms")
        return x + self._rms(self._lin(a, w), post_norm)

    def _logits(self, h, normed=False):
        if not normed:
            h = self._rms(h, self.dec.norm)
        W = self.dec.lm_shard if self.tp is not None else self.dec.lm_weight
        if self.cuda:
            out = torch.empty(h.shape[0], W.shape[0], dtype=torch.float32, device=h.device)
            self.blocks.gemm(self.blocks.TN, h, W, out)
            return out
        return (h @ W.t()).float()

    def _attn(self, st, i, layer, x):
        cfg = self.cfg
        B, blk = st.B, st.blk
        Hq, Hkv, d = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
        qs = 2 * d if cfg.attn_output_gate else d
        h = self._rms(x, layer.input_norm)
        qkv = self._lin(h, layer.wqkv)
        M = B * blk
        ang = getattr(st, "rope_ang", None)
        if self.cuda:
            q = torch.empty(M, Hq, d, dtype=x.dtype, device=x.device)
            k = torch.empty(M, Hkv, d, dtype=x.dtype, device=x.device)
            cos_t, sin_t, rp = self.cos_t, self.sin_t, st.rowpos32
            if ang is not None:                      # per-row tables (3-D RoPE prompt rows)
                fa = ang.reshape(M, -1).float()
                cos_t, sin_t = fa.cos().contiguous(), fa.sin().contiguous()
                rp = torch.arange(M, dtype=torch.int32, device=x.device)
            self.C.qk_norm_rope_fwd(qkv, layer.q_norm, layer.k_norm, cos_t, sin_t, rp, q, k,
                                    Hq, Hkv, d, cfg.rotary_dim, cfg.eps, qs)
            v = qkv[:, Hq * qs + Hkv * d:]
            ptab = self.ptab if self.paged else None
            self.C.kv_append(k, v, self.kc[i], self.vc[i], st.slot_t, st.pos_t, blk, ptab)
            o = torch.empty(M, Hq, d, dtype=x.dtype, device=x.device)
            if self.guards:
                o.fill_(float("nan"))                # rows the kernel leaves unwritten stay NaN
            self.C.canvas_attention(q, self.kc[i], self.vc[i], st.slot_t, st.pos_t, o, blk, st.n_clean, st.max_keys,
                                    1.0 / math.sqrt(d), ptab, self.err if self.attn_tc else None)
            if self.guards and not torch.cuda.is_current_stream_capturing():
                self._guard_attention(i, st, q, o, blk)
            o = o.view(M, Hq * d)
            if cfg.attn_output_gate:
                og = torch.empty_like(o)
                self.C.attn_gate_fwd(o, qkv, og, Hq, d)
                o = og
            return self._out(o, layer.wo, x, getattr(layer, "post_attn_norm", None))
        # CPU statement
        if cfg.attn_output_gate:
            qg = qkv[:, :2 * Hq * d].view(M, Hq, 2 * d)
            q, gate = qg[..., :d], qg[..., d:].reshape(M, Hq * d)
        else:
            q, gate = qkv[:, :Hq * d].view(M, Hq, d), None
        k = qkv[:, Hq * qs:Hq * qs + Hkv * d].view(M, Hkv, d)
        v = qkv[:, Hq * qs + Hkv * d:].view(M, Hkv, d)
        if layer.q_norm is not None:
            q = R.rmsnorm(q, layer.q_norm, cfg.eps)
            k = R.rmsnorm(k, layer.k_norm, cfg.eps)
        if ang is not None:
            a2 = torch.cat([ang, ang], -1).reshape(M, -1)
            cos, sin = a2.cos(), a2.sin()
        else:
            cos, sin = R.rope_cos_sin(st.rowpos, d, cfg.rope_theta, cfg.rotary_dim)
        q = R.apply_rope(q.float()[None], cos[None], sin[None])[0].to(x.dtype)
        k = R.apply_rope(k.float()[None], cos[None], sin[None])[0].to(x.dtype)
        q, k, v = q.view(B, blk, Hq, d), k.view(B, blk, Hkv, d), v.view(B, blk, Hkv, d)
        outs = []
        G_ = Hq // Hkv
        r = torch.arange(blk)[:, None]
        c = torch.arange(blk)[None, :]
        inner = (c <= r) | (r >= st.n_clean)
        for b, s in enumerate(st.slots):
            p0 = self.pos[s]
            self.kc[i][s, p0:p0 + blk] = k[b]
            self.vc[i][s, p0:p0 + blk] = v[b]
            K = self.kc[i][s, :p0 + blk].float().repeat_interleave(G_, 1)       # [Lk, Hq, d]
            V = self.vc[i][s, :p0 + blk].float().repeat_interleave(G_, 1)
            sc = torch.einsum("thd,khd->htk", q[b].float(), K) / math.sqrt(d)
            mask = torch.cat([torch.ones(blk, p0, dtype=torch.bool), inner], 1)
            sc = sc.masked_fill(~mask[None], float("-inf"))
            outs.append(torch.einsum("htk,khd->thd", sc.softmax(-1), V))
        o = torch.stack(outs).reshape(M, Hq * d).to(x.dtype)
        if gate is not None:
            o = o * torch.sigmoid(gate.float()).to(o.dtype)
        return self._out(o, layer.wo, x, getattr(layer, "post_attn_norm", None))

    def _gdn(self, st, i, layer, x):
        cfg = self.cfg
        B, blk = st.B, st.blk
        Hk, Hv, dk, dv = cfg.lin_k_heads, cfg.lin_v_heads, cfg.lin_k_dim, cfg.lin_v_dim
        kd, vd = Hk * dk, Hv * dv
        Cc = 2 * kd + vd
        M = B * blk
        h = self._rms(x, layer.input_norm)
        proj = self._lin(h, layer.w_in)
        z = proj[:, Cc:Cc + vd]
        gb = proj[:, Cc + vd:Cc + vd + Hv]
        ga = proj[:, Cc + vd + Hv:Cc + vd + 2 * Hv]
        if self.cuda:
            mixed = torch.empty(M, Cc, dtype=x.dtype, device=x.device)
            self.C.canvas_conv(proj[:, :Cc], self.win[i], layer.conv_w, mixed, st.slot_t, blk)
            a_log, dtb = self._gdn_f32[i]
            o = torch.empty(M, vd, dtype=x.dtype, device=x.device)
            if self.gdn_tc:
                kbuf = torch.empty(M, Hv, dk, dtype=x.dtype, device=x.device)
                ubuf = torch.empty(M, Hv, dv, dtype=x.dtype, device=x.device)
                gbuf = torch.empty(M, Hv, dtype=torch.float32, device=x.device)
                st.gdn[i] = (mixed, kbuf, ubuf, gbuf, proj)
                if self.gdn_fused_norm:    # o receives the normalised, gated rows directly
                    self.C.gdn_canvas_tc(mixed, ga, gb, a_log, dtb, o, kbuf, ubuf, gbuf, self.ssm[i], st.slot_t,
                                         blk, Hk, Hv, st.n_clean, dk ** -0.5, self.err, z=z, gnorm_w=layer.gnorm,
                                         eps=cfg.eps)
                    return self._lin(o, layer.w_out, x)
                self.C.gdn_canvas_tc(mixed, ga, gb, a_log, dtb, o, kbuf, ubuf, gbuf, self.ssm[i], st.slot_t, blk,
                                     Hk, Hv, st.n_clean, dk ** -0.5, self.err)
                y = torch.empty(M, vd, dtype=x.dtype, device=x.device)
                self.C.gdn_gnorm_fwd(o, z, layer.gnorm, y, Hv, cfg.eps)
                return self._lin(y, layer.w_out, x)
            else:
                prep = torch.empty(self.C.gdn_prep_numel(M, Hk, Hv), dtype=torch.float32, device=x.device)
                self.C.gdn_canvas(mixed, ga, gb, a_log, dtb, o, prep, self.ssm[i], st.slot_t, blk, Hk, Hv,
                                  st.n_clean, dk ** -0.5)
                rec = (mixed, ga, gb, proj, prep)
            y = torch.empty(M, vd, dtype=x.dtype, device=x.device)
            self.C.gdn_gnorm_fwd(o, z, layer.gnorm, y, Hv, cfg.eps)
            st.gdn[i] = rec
            return self._lin(y, layer.w_out, x)
        # CPU statement
        K1 = cfg.conv_kernel - 1
        qkv = proj[:, :Cc].view(B, blk, Cc)
        win = torch.stack([self.win[i][s] for s in st.slots])                  # [B, K-1, Cc]
        conv_in = torch.cat([win.to(qkv.dtype), qkv], 1)                       # [B, K-1+blk, Cc]
        w = layer.conv_w.float()
        acc = sum(conv_in[:, j:j + blk].float() * w[:, j] for j in range(cfg.conv_kernel))
        mixed = F.silu(acc).to(x.dtype)
        q = G.l2norm(mixed[..., :kd].reshape(B, blk, Hk, dk).float()) * dk ** -0.5
        k = G.l2norm(mixed[..., kd:2 * kd].reshape(B, blk, Hk, dk).float())
        v = mixed[..., 2 * kd:].reshape(B, blk, Hv, dv).float()
        rep = Hv // Hk
        if rep > 1:
            q, k = q.repeat_interleave(rep, 2), k.repeat_interleave(rep, 2)
        g, beta = G.gates(ga.reshape(B, blk, Hv), gb.reshape(B, blk, Hv), layer.A_log, layer.dt_bias)
        outs = []
        for b, s in enumerate(st.slots):
            S = self.ssm[i][s].clone()
            ob = []
            for t in range(blk):
                S, o_t = G._step(S, q[b, t], k[b, t], v[b, t], g[b, t], beta[b, t])
                ob.append(o_t)
            for t in range(st.n_clean, blk):
                ob[t] = torch.einsum("hkv,hk->hv", S, q[b, t])
            outs.append(torch.stack(ob))
        o = torch.stack(outs).to(x.dtype)                                      # [B, blk, Hv, dv]
        y = G.gated_rmsnorm(o, z.reshape(B, blk, Hv, dv), layer.gnorm, cfg.eps)
        st.gdn[i] = (q, k, v, g, beta, conv_in)
        return self._lin(y.reshape(M, vd), layer.w_out, x)


class _SeqPar:
    """The residual stream in tensor-parallel sequence-parallel form: this rank's rows ``xs`` of the
    residual and ``h`` = RMSNorm(x) * ``norm`` over all rows (the gathered input of the next
    sublayer).  ``next`` names the norm weight that the next row-parallel output applies."""

    def __init__(self, xs, h, norm):
        self.xs, self.h, self.norm, self.next = xs, h, norm, None

    @property
    def dtype(self):
        return self.h.dtype

    @property
    def device(self):
        return self.h.device


class GreedyTokens:
    """The result of a greedy canvas: the tokens [B, rows] in place of the logits."""

    def __init__(self, tokens):
        self.tokens = tokens
        self.shape = tuple(tokens.shape)

    def __getitem__(self, i):
        return GreedyTokens(self.tokens[i])


class KVPages:
    """Host allocator of a paged KV cache: pages of ``PAGE`` positions taken from one pool as a slot
    grows and returned when it is released; ``table[slot, i]`` is the page of positions
    ``[PAGE i, PAGE (i + 1))`` (the page table the KV kernels read)."""

    def __init__(self, n_pages, n_slots, max_pages, pin=False):
        self.n_pages = n_pages
        self.free = list(range(n_pages))[::-1]
        self.owned = [[] for _ in range(n_slots)]
        t = torch.zeros(n_slots, max_pages, dtype=torch.int32)
        self.table = t.pin_memory() if pin and torch.cuda.is_available() else t

    def ensure(self, slot, upto):
        """Pages covering positions [0, upto) of ``slot``; True when the table changed."""
        need = (upto + PAGE - 1) // PAGE
        pages = self.owned[slot]
        if need > self.table.shape[1]:
            raise RuntimeError(f"slot {slot}: {upto} positions exceed the page table ({self.table.shape[1]} pages)")
        changed = False
        while len(pages) < need:
            if not self.free:
                raise RuntimeError(f"KV page pool exhausted ({self.n_pages} pages of {PAGE} positions)")
            pg = self.free.pop()
            self.table[slot, len(pages)] = pg
            pages.append(pg)
            changed = True
        return changed

    def release(self, slot):
        self.free.extend(reversed(self.owned[slot]))
        self.owned[slot] = []

    def check(self, live):
        """Guard: the pages of the ``live`` slots are in range, owned by exactly one slot, not on
        the free list, and the table rows say so (raises naming the first violation)."""
        seen = {}
        free = set(self.free)
        for s in live:
            for i, pg in enumerate(self.owned[s]):
                if not 0 <= pg < self.n_pages:
                    raise RuntimeError(f"[guards] slot {s} page {i}: page {pg} outside the pool of {self.n_pages}")
                if pg in seen:
                    raise RuntimeError(f"[guards] page {pg} held by slots {seen[pg]} and {s}")
                if pg in free:
                    raise RuntimeError(f"[guards] page {pg} of slot {s} is also on the free list")
                if int(self.table[s, i]) != pg:
                    raise RuntimeError(f"[guards] page table [{s}, {i}] = {int(self.table[s, i])}, slot owns page {pg}")
                seen[pg] = s

    def used(self):
        return self.n_pages - len(self.free)


class _Step:
    """Per-canvas bookkeeping shared by the layers and kept until the commit."""

    def __init__(self, rt, slots, B, blk, n_clean, static=False):
        self.slots, self.B, self.blk, self.n_clean = list(slots), B, blk, n_clean
        self.gdn = {}
        if static:      # device buffers refilled before every graph replay
            dev = rt.device
            self.max_keys = rt.max_len
            self.tokens = torch.zeros(B, blk, dtype=torch.long, device=dev)
            self.slot_t = torch.full((B,), rt.dummy, dtype=torch.int32, device=dev)
            self.pos_t = torch.zeros(B, dtype=torch.int32, device=dev)
            self.rowpos32 = torch.arange(blk, dtype=torch.int32, device=dev).repeat(B)
            return
        pos = [rt.pos[s] for s in self.slots]
        self.max_keys = max(pos) + blk
        self.rowpos = torch.tensor([p + rt.rope_delta[s] + j for p, s in zip(pos, self.slots) for j in range(blk)],
                                   dtype=torch.long)
        if rt.cuda:
            dev = rt.device
            self.slot_t = torch.tensor(self.slots, dtype=torch.int32, device=dev)
            self.pos_t = torch.tensor(pos, dtype=torch.int32, device=dev)
            self.rowpos32 = self.rowpos.to(dev, torch.int32)


class _Graph:
    """A captured decode canvas (embedding -> logits of every row) and its commit for one
    (padded batch, canvas rows, clean rows) shape.  Captured after one eager warm-up run on the
    scratch slot, which also initialises every kernel's launch attributes."""

    def __init__(self, rt, B, blk, n_clean, greedy=False):
        self.st = _Step(rt, [rt.dummy] * B, B, blk, n_clean, static=True)
        self.adv = torch.ones(B, dtype=torch.int32, device=rt.device)
        self.host_tok = torch.zeros(B, blk, dtype=torch.long).pin_memory()
        self.host_slot = torch.zeros(B, dtype=torch.int32).pin_memory()
        self.host_pos = torch.zeros(B, dtype=torch.int32).pin_memory()
        self.host_rowpos = torch.zeros(B * blk, dtype=torch.int32).pin_memory()
        self.host_adv = torch.ones(B, dtype=torch.int32).pin_memory()

        def fwd():
            x = rt._forward(self.st, self.st.tokens)
            if greedy:                   # tokens only: the LM head's argmax runs in its GEMM epilogue
                return None, rt._greedy_tokens(x).view(B, blk)
            lg = rt._logits(x).view(B, blk, -1)
            return lg, rt.argmax(lg)

        def com():
            rt._commit_kernels(self.st, self.adv)

        s = torch.cuda.Stream(device=rt.device)
        s.wait_stream(torch.cuda.current_stream(rt.device))
        with torch.cuda.stream(s):
            fwd()
            com()
        torch.cuda.current_stream(rt.device).wait_stream(s)
        self.fwd = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.fwd):
            self.logits, self.am = fwd()
        self.com = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.com):
            com()
