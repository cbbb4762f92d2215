"""Block-diffusion SFT objective on the native decoder.

Row layout per complementary view (batch doubled to 2B), identical to the reference
(``train/models/block_diffusion.py:1-18``, ``forward`` ``:911-1018``)::

    [ S (prompt) | x_t (response, noised) | pad ]  [ x_0 (clean response, right-padded to rpad) ]
      region A, length L                              region B, length rpad

Attention rules (``ops.reference.bd_allowed``): the prompt is causal and visible to everything
after it; an x_t block sees itself bidirectionally (or token-causally with
``within_block_causal``) and the earlier clean blocks of x_0; x_0 is block-causal, or
token-causal when the AR auxiliary loss is on.  Loss: token-shifted diffusion CE over the masked
x_t tokens (1/gamma ELBO weights normalised to 1, or uniform) mixed with the token-shifted AR CE
over x_0 as ``(diff + w * ar) / (1 + w)``.

Noising draws the same random numbers in the same order as the reference -- one
``rand(B, n_blocks)`` for the per-block rate, then one ``rand(B, L)`` for the token draws -- so a
fixed seed gives the same views.  The B200 path differs only in how the work is done: one fused
attention kernel reads the mask from per-token metadata, the two CE terms share one fused
linear-CE call, and host synchronisation happens once, before any layer runs.
"""
import json
import math
import os

import torch
import torch.nn as nn

from ..ops import blocks
from ..ops.ce import fused_linear_ce
from ..ops.reference import PAD, SHARED, X0, XT


def bucketed_clean_len(needed, block_size, buckets):
    """Smallest bucket (rounded up to ``block_size``) that holds ``needed``; ``needed`` rounded
    up to ``block_size`` when no bucket does.  Same rule as ``block_diffusion.py:35-47``."""
    needed = math.ceil(max(needed, 1) / block_size) * block_size
    if not buckets:
        return needed
    for b in sorted(buckets):
        b = math.ceil(b / block_size) * block_size
        if b >= needed:
            return b
    return needed


class BlockDiffusionLM(nn.Module):
    def __init__(self, decoder, mask_id, pad_id=0, bd_size=32, ar_loss_weight=0.0, loss_weighting="weighted",
                 pos_decay_gamma=0.0, full_mask=False, within_block_causal=False, mask_pattern="random",
                 response_buckets=(512, 1024, 2048, 4096), max_length=16384, max_response_length=4096,
                 merged_views=False, ar_only=False, activation_checkpoint="auto", ce_chunk=4096,
                 tokenizer=None, activation_offload=False):
        super().__init__()
        assert loss_weighting in ("weighted", "uniform"), loss_weighting
        assert mask_pattern in ("random", "canvas"), mask_pattern
        self.decoder = decoder
        self.mask_id = mask_id
        self.pad_id = pad_id
        self.bd_size = bd_size
        self.ar_loss_weight = ar_loss_weight
        self.loss_weighting = loss_weighting
        self.pos_decay_gamma = pos_decay_gamma
        self.full_mask = full_mask
        self.within_block_causal = within_block_causal
        self.mask_pattern = mask_pattern
        self.response_buckets = tuple(response_buckets) if response_buckets else None
        self.max_length = max_length
        self.max_response_length = max_response_length
        self.merged_views = merged_views
        self.ar_only = ar_only
        self.activation_checkpoint = activation_checkpoint
        self.activation_offload = activation_offload
        self._offload_pool = None
        self.ce_chunk = ce_chunk
        self.tokenizer = tokenizer
        self.is_vl = decoder.cfg.is_vl
        self.image_processor = None
        self._rope = {}

    # ------------------------------------------------------------------ helpers
    @property
    def cfg(self):
        return self.decoder.cfg

    def param_groups(self, projector_lr_scale=1.0, decision_head_lr_scale=1.0, per_layer=False, stream=True):
        """Optimizer groups tagged with ``lr_scale`` (order: backbone, projector, decision head --
        the reference's frozen group order, ``block_diffusion.py:180-201``).  ``per_layer`` splits
        the backbone into the non-layer parameters plus one group per decoder layer (tagged with
        its ``layer`` index, the unit of full sharding), and with ``stream`` marks them for
        gradients streamed through a two-slot ring (for models whose full fp32 gradients do not
        fit next to the optimizer state)."""
        backbone, projector, head = [], [], []
        for name, p in self.named_parameters():
            if not p.requires_grad:
                continue
            if ".visual." in name and ".visual.merger." not in name:
                raise RuntimeError(f"vision encoder parameter {name} is trainable; expected it frozen")
            if name.startswith("jev_head."):
                head.append(p)
            else:
                (projector if ".visual.merger." in name else backbone).append(p)
        if per_layer:
            layer_ids = {}
            for i, layer in enumerate(self.decoder.layers):
                for p in layer.parameters():
                    layer_ids[id(p)] = i
            rest = [p for p in backbone if id(p) not in layer_ids]
            groups = [{"params": rest, "lr_scale": 1.0}]
            for i, layer in enumerate(self.decoder.layers):
                groups.append({"params": [p for p in layer.parameters() if p.requires_grad], "lr_scale": 1.0,
                               "stream": stream, "layer": i})
        else:
            groups = [{"params": backbone, "lr_scale": 1.0}]
        if projector:
            groups.append({"params": projector, "lr_scale": projector_lr_scale})
        if head:
            groups.append({"params": head, "lr_scale": decision_head_lr_scale})
        return groups

    def rope(self, device):
        key = str(device)
        if key not in self._rope:
            c = self.cfg
            self._rope[key] = blocks.rope_tables(c.max_position, c.rotary_dim, c.rope_theta, device)
        return self._rope[key]

    def make_actx(self, seg, opos, rblk, segid, view, pos, x0_token_causal, pos3=None):
        """``pos3`` [B, 3, T]: 3-D (t, h, w) RoPE positions of vision-language rows."""
        cos_t = sin_t = None
        if seg.is_cuda and pos3 is None:
            cos_t, sin_t = self.rope(seg.device)
        actx = blocks.AttnContext(seg, opos, rblk, segid, view, pos, x0_token_causal, self.within_block_causal,
                                  cos_t, sin_t)
        if pos3 is not None:
            from .vision import mrope_angles
            c = self.cfg
            actx.set_rope_angles(mrope_angles(pos3, c.rotary_dim, c.rope_theta, c.mrope_section))
        return actx

    def _activations_fit(self, x):
        """``activation_checkpoint="auto"``: do every layer's saved activations fit in the device
        memory that is free now?  Per layer and token the block kernels keep about
        4 D + 2 F + 2 (Hq + 2 Hkv) d bf16 values (the normed inputs, the q / k / v projections, the
        attention output and the SwiGLU inputs), counted against 90 % of the free plus cached-unused
        memory."""
        if not x.is_cuda:
            return True
        c = self.cfg
        per_tok = 4 * c.hidden_size + 2 * c.intermediate_size + 2 * (c.n_heads + 2 * c.n_kv_heads) * c.head_dim
        need = x.shape[0] * per_tok * 2 * len(self.decoder.layers)
        free = torch.cuda.mem_get_info(x.device)[0] + torch.cuda.memory_reserved(x.device) \
            - torch.cuda.memory_allocated(x.device)
        return need < 0.9 * free

    def run_stack(self, x, actx):
        mode = self.activation_checkpoint
        train = self.training and torch.is_grad_enabled()
        ckpt = train and (mode == "layer" or (mode == "auto" and not self._activations_fit(x)))
        if ckpt and self.activation_offload:
            # the checkpoint inputs (one [tokens, D] tensor per layer) wait in pinned host memory
            from ..utils.offload import ActivationOffload, PinnedPool
            if self._offload_pool is None:
                self._offload_pool = PinnedPool()
            with ActivationOffload(self._offload_pool):
                return self._run_stack(x, actx, ckpt)
        return self._run_stack(x, actx, ckpt)

    def _run_stack(self, x, actx, ckpt):
        ring = getattr(self, "param_ring", None)
        if ring is None or not ring.active:
            if ckpt:
                from torch.utils.checkpoint import checkpoint

                def hook(i, layer, h):
                    return checkpoint(layer, h, actx, self.cfg, use_reentrant=False)
                return self.decoder(x, actx, layer_hook=hook)
            return self.decoder(x, actx)
        # full-shard weights: gather layer i (prefetching i + 1) before it runs, drop it after; in
        # backward the gradient of layer i's output arrives once layer i + 1's backward is done,
        # which is when layer i is gathered again (prefetching i - 1)
        n = len(self.decoder.layers)

        def sharded(i, layer, h):
            ring.fetch(i, i + 1 if i + 1 < n else None)
            if ckpt:
                from torch.utils.checkpoint import checkpoint
                out = checkpoint(layer, h, actx, self.cfg, use_reentrant=False)
            else:
                out = layer(h, actx, self.cfg)
            ring.done(i)
            if out.requires_grad:
                def before_backward(g, i=i):
                    ring.done(i + 1)
                    ring.fetch(i, i - 1 if i > 0 else None)
                    return g
                out.register_hook(before_backward)
            return out
        return self.decoder(x, actx, layer_hook=sharded)

    def _weights(self, rate_sel, pos_sel=None):
        n = rate_sel.numel()
        w = None
        if self.loss_weighting == "weighted" and n:
            w = 1.0 / (rate_sel.float() + 1e-8)
        if self.pos_decay_gamma > 0 and pos_sel is not None and n:
            pw = torch.exp(-pos_sel.float() / self.pos_decay_gamma)
            w = pw if w is None else w * pw
        if w is None:
            return torch.full((n,), 1.0 / max(n, 1), dtype=torch.float32, device=rate_sel.device)
        return w / w.sum()

    # ------------------------------------------------------------------ noising
    def _make_views(self, input_ids, labels, s0, eps=1e-3):
        """Two complementary views stacked to [2B, L] (``block_diffusion.py:213-236``); with
        ``full_mask`` every response token is masked in a single view (rate 1)."""
        B, L = input_ids.shape
        dev = input_ids.device
        answer = labels != -100
        if self.full_mask:
            noisy = torch.where(answer, torch.full_like(input_ids, self.mask_id), input_ids)
            return noisy, labels.clone(), torch.ones(B, L, dtype=torch.float32, device=dev)
        rel = (torch.arange(L, device=dev)[None, :] - s0[:, None]).clamp(min=0)
        rblk = rel // self.bd_size
        nblk = (L + self.bd_size - 1) // self.bd_size
        p_block = (1 - eps) * torch.rand(B, nblk, device=dev) + eps
        p_tok = torch.gather(p_block, 1, rblk)
        picked = (torch.rand(B, L, device=dev) < p_tok) & answer

        def view(sel):
            apply = sel & answer
            noisy = torch.where(apply, torch.full_like(input_ids, self.mask_id), input_ids)
            vl = torch.where(apply, labels, torch.full_like(labels, -100))
            return noisy, vl

        na, la = view(picked)
        nb, lb = view(~picked)
        return torch.cat([na, nb], 0), torch.cat([la, lb], 0), p_tok.repeat(2, 1)

    # ------------------------------------------------------------------ forward
    def forward(self, input_ids, labels, attention_mask, seg_id=None, resp_pos=None, resp_block=None,
                turn_id=None, rpad=None, **_images):
        if self.ar_only:
            return self.forward_ar(input_ids, labels, attention_mask, seg_id=seg_id)
        if resp_block is not None:
            from .layouts import forward_multiturn
            return forward_multiturn(self, input_ids, labels, attention_mask, resp_block, turn_id)
        if seg_id is not None:
            from .layouts import forward_packed
            return forward_packed(self, input_ids, labels, attention_mask, seg_id, resp_pos)
        return self.forward_single(input_ids, labels, attention_mask, rpad=rpad)

    def forward_single(self, input_ids, labels, attention_mask, rpad=None):
        dev = input_ids.device
        B, L = input_ids.shape
        valid = attention_mask.bool()
        ans = labels != -100
        s0 = torch.argmax(ans.int(), dim=1)
        last = L - 1 - torch.argmax(torch.flip(ans, [1]).int(), dim=1)
        if not input_ids.is_cuda:  # the GPU path validates in the collator (no host sync here)
            assert ans.any(dim=1).all(), "every sample must have at least one response token"
            ar = torch.arange(L)[None]
            assert (ans == ((ar >= s0[:, None]) & (ar <= last[:, None]))).all(), \
                "response (loss) tokens must form one contiguous span"
        resp_len = last - s0 + 1

        noisy, view_labels, rate = self._make_views(input_ids, labels, s0)
        V = 1 if self.full_mask else 2
        clean = input_ids.repeat(V, 1)
        s0 = s0.repeat(V)
        resp_len = resp_len.repeat(V)
        valid = valid.repeat(V, 1)
        BB = V * B

        if rpad is None:
            rpad = bucketed_clean_len(int(resp_len.max().item()), self.bd_size, self.response_buckets)
        r_idx = torch.arange(rpad, device=dev)[None, :]
        src_c = (s0[:, None] + r_idx).clamp(max=L - 1)
        b_valid = r_idx < resp_len[:, None]
        ids_b = torch.gather(clean, 1, src_c)
        tokens = torch.cat([noisy, ids_b], 1)                       # [BB, T]
        T = L + rpad

        posA = torch.arange(L, device=dev)[None, :].expand(BB, -1)
        pos = torch.cat([posA, src_c], 1)
        is_resp = (posA >= s0[:, None]) & valid
        segA = torch.where(valid, torch.where(is_resp, XT, SHARED), PAD)
        rblkA = (posA - s0[:, None]).clamp(min=0) // self.bd_size
        segB = torch.where(b_valid, X0, PAD)
        rblkB = (r_idx // self.bd_size).expand(BB, -1)
        seg = torch.cat([segA, segB], 1)
        rblk = torch.cat([rblkA, rblkB], 1)
        zeros = torch.zeros(BB, T, dtype=torch.int32, device=dev)
        actx = self.make_actx(seg, pos, rblk, zeros, zeros, pos, self.ar_loss_weight > 0)

        # loss-row selection (one host sync, before any layer is launched)
        sel = view_labels[:, 1:] != -100                             # [BB, L-1]
        d_idx = torch.nonzero(sel.reshape(-1)).squeeze(1)
        bi, ti = d_idx // (L - 1), d_idx % (L - 1)
        d_rows = bi * T + ti                                         # hidden[b, t] predicts label[b, t+1]
        d_tgt = view_labels[bi, ti + 1]
        w_diff = self._weights(rate[bi, ti + 1])
        ar_w = self.ar_loss_weight
        if ar_w > 0:
            ar_sel = (r_idx + 1 < resp_len[:, None])[:, :-1]         # slot j valid and j+1 in response
            a_idx = torch.nonzero(ar_sel.reshape(-1)).squeeze(1)
            ab, aj = a_idx // (rpad - 1), a_idx % (rpad - 1)
            a_rows = ab * T + L + aj
            a_tgt = ids_b[ab, aj + 1]
            n_ar = a_idx.numel()
            rows = torch.cat([d_rows, a_rows])
            tgt = torch.cat([d_tgt, a_tgt])
            wts = torch.cat([w_diff / (1 + ar_w),
                             torch.full((n_ar,), ar_w / ((1 + ar_w) * max(n_ar, 1)), device=dev)])
        else:
            n_ar = 0
            rows, tgt, wts = d_rows, d_tgt, w_diff
        n_diff = d_idx.numel()

        x = self.decoder.embed_tokens(tokens)                       # [BB*T, D]
        hidden = self.run_stack(x, actx)
        h_sel = hidden.index_select(0, rows)
        loss, ce = fused_linear_ce(h_sel, self.decoder.lm_weight, tgt, wts, chunk=self.ce_chunk)
        with torch.no_grad():
            diff_loss = torch.dot(ce[:n_diff], w_diff) if n_diff else torch.zeros((), device=dev)
            ar_loss = ce[n_diff:].mean() if n_ar else torch.zeros((), device=dev)
        return loss, {"diff_loss": diff_loss, "ar_loss": ar_loss, "ntok": n_diff}

    # ------------------------------------------------------------------ pure AR SFT
    def forward_ar(self, input_ids, labels, attention_mask, seg_id=None):
        """Causal-LM SFT (``block_diffusion.py:792-908``): shift CE on supervised tokens; with
        ``seg_id`` (packing) attention is causal within each document only."""
        dev = input_ids.device
        B, L = input_ids.shape
        valid = attention_mask.bool()
        pos = torch.arange(L, device=dev)[None].expand(B, -1)
        seg = torch.where(valid, SHARED, PAD)
        if seg_id is not None:
            segid = torch.where(valid, seg_id, torch.full_like(seg_id, -1)).int()
            pos_rope = pos
        else:
            segid = torch.zeros(B, L, dtype=torch.int32, device=dev)
            pos_rope = pos
        zeros = torch.zeros(B, L, dtype=torch.int32, device=dev)
        actx = self.make_actx(seg, pos, zeros, segid, zeros, pos_rope, True)
        sel = labels[:, 1:] != -100
        idx = torch.nonzero(sel.reshape(-1)).squeeze(1)
        bi, ti = idx // (L - 1), idx % (L - 1)
        rows = bi * L + ti
        tgt = labels[bi, ti + 1]
        n = idx.numel()
        wts = torch.full((n,), 1.0 / max(n, 1), device=dev)
        x = self.decoder.embed_tokens(input_ids)
        hidden = self.run_stack(x, actx)
        loss, ce = fused_linear_ce(hidden.index_select(0, rows), self.decoder.lm_weight, tgt, wts,
                                   chunk=self.ce_chunk)
        return loss, {"diff_loss": torch.zeros((), device=dev), "ar_loss": loss.detach(), "ntok": n}

    # ------------------------------------------------------------------ checkpoint sidecar
    def bd_json(self):
        return {"bd_size": self.bd_size, "mask_id": self.mask_id, "ar_loss_weight": self.ar_loss_weight,
                "max_length": self.max_length, "max_response_length": self.max_response_length,
                "response_buckets": list(self.response_buckets) if self.response_buckets else None}

    def save_sidecar(self, path):
        os.makedirs(path, exist_ok=True)
        with open(os.path.join(path, "block_diffusion.json"), "w") as f:
            json.dump(self.bd_json(), f, indent=2)
