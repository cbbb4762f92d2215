"""Two-stream block-diffusion objective for the hybrid (gated-delta + full-attention) decoder.

Reference: ``train/models/hybrid.py`` (``forward_flare`` ``:1020-1135``, ``_make_flare_views``
``:916-949``, ``forward_decision`` ``:886-913``).  Each row's layer input is
``[x0 ; xt_1 ; xt_2]`` (the clean row shared by two complementary noisy views; one fully masked
view with ``full_mask``), every stream reusing the row's positions (reset per packed document).
Full-attention layers use the two-stream rule (x0 token- or block-causal; a noisy token sees its
own block of its own view and the strictly earlier clean blocks); gated-delta layers run the
two-stream recurrence (``ops.gdn_reference``).  Loss: diffusion CE on the noisy streams over masked
response tokens (1/gamma weights, optional intra-block position decay) mixed with the AR CE on the
clean stream, bounded by turn and document.

Typed decisions: every question row is a document of one causal row; the pointer head scores the
``</opt>`` states against the ``<decide>`` state.
"""
import torch

from ..ops.ce import fused_linear_ce
from ..ops.gdn import LinearLayout
from ..ops.reference import SHARED, X0, XT
from .block_diffusion import BlockDiffusionLM
from .decision import PointerHead, decision_loss


def doc_starts(seg):
    """True at the first token of every contiguous same-id run of ``seg`` [B, L]."""
    s = torch.ones_like(seg, dtype=torch.bool)
    s[:, 1:] = seg[:, 1:] != seg[:, :-1]
    return s


def doc_positions(seg):
    """Positions restarting at 0 at every document start."""
    B, L = seg.shape
    ar = torch.arange(L, device=seg.device)[None].expand(B, -1)
    start = torch.cummax(torch.where(doc_starts(seg), ar, torch.zeros_like(ar)), 1).values
    return ar - start


class HybridBlockDiffusionLM(BlockDiffusionLM):
    def __init__(self, decoder, linear_block_mode="bidirectional", decision_head_dim=0, **kw):
        super().__init__(decoder, **kw)
        assert linear_block_mode in ("causal", "bidirectional"), linear_block_mode
        self.linear_block_mode = linear_block_mode
        self.share_x0 = True
        self.jev_head = None
        if decision_head_dim:
            p = next(decoder.parameters())
            self.jev_head = PointerHead(decoder.cfg.hidden_size, dp=decision_head_dim).to(p.device, p.dtype)

    @property
    def decision_head(self):
        return self.jev_head

    # ----------------------------------------------------------------------------------------
    def forward(self, input_ids, labels, attention_mask, seg_id=None, resp_pos=None, resp_block=None,
                turn_id=None, decision=None, rpad=None, pixel_values=None, image_grid_thw=None, mrope_pos=None,
                pointer=None):
        if decision is not None:
            return self.forward_decision(decision)
        images = pixel_values is not None
        if images and (self.ar_only or self.linear_block_mode != "bidirectional"):
            raise NotImplementedError("image inputs are supported only by the two-stream objective "
                                      "(--linear_block_mode bidirectional)")
        if self.ar_only:
            return self.forward_ar(input_ids, labels, attention_mask, seg_id=seg_id)
        if self.linear_block_mode == "bidirectional":
            return self.forward_flare(input_ids, labels, attention_mask, seg_id=seg_id, turn_id=turn_id,
                                      pixel_values=pixel_values, image_grid_thw=image_grid_thw, mrope_pos=mrope_pos,
                                      pointer=pointer)
        if seg_id is not None or resp_pos is not None or resp_block is not None:
            raise NotImplementedError("hybrid causal mode covers single-turn unpacked rows (as the reference's)")
        if pointer is not None:
            raise NotImplementedError("pointer-head rows are trained with --linear_block_mode bidirectional")
        # causal mode (``train/models/hybrid.py`` ``linear_block_mode="causal"``): the dense
        # [S | x_t | x_0] row with the block-diffusion mask on the full-attention layers, while the
        # linear layers scan region A = [S | x_t] and region B = [x_0] as two causal documents
        self._region_split = input_ids.shape[1]
        try:
            return self.forward_single(input_ids, labels, attention_mask, rpad=rpad)
        finally:
            self._region_split = None

    def make_actx(self, seg, opos, rblk, segid, view, pos, x0_token_causal, pos3=None):
        actx = super().make_actx(seg, opos, rblk, segid, view, pos, x0_token_causal, pos3=pos3)
        split = getattr(self, "_region_split", None)
        if split is not None:
            doc = torch.zeros(seg.shape, dtype=torch.bool, device=seg.device)
            doc[:, 0] = True
            doc[:, split] = True
            actx.linear = LinearLayout("causal", doc_start=doc)
        return actx

    def _flare_views(self, input_ids, labels, answer, eps=1e-3):
        B, L = input_ids.shape
        dev = input_ids.device
        if self.full_mask:
            noisy = torch.where(answer, torch.full_like(input_ids, self.mask_id), input_ids)
            vl = torch.where(answer, labels, torch.full_like(labels, -100))
            return noisy, vl, torch.ones(B, L, device=dev)
        bd = self.bd_size
        nblk = (L + bd - 1) // bd
        blk = (torch.arange(L, device=dev) // bd)[None].expand(B, -1)
        p_block = (1 - eps) * torch.rand(B, nblk, device=dev) + eps
        p_tok = torch.gather(p_block, 1, blk)
        picked = (torch.rand(B, L, device=dev) < p_tok) & answer

        def view(sel):
            apply = sel & answer
            return (torch.where(apply, torch.full_like(input_ids, self.mask_id), input_ids),
                    torch.where(apply, labels, torch.full_like(labels, -100)))
        na, la = view(picked)
        nb, lb = view(~picked)
        return torch.cat([na, nb], 0), torch.cat([la, lb], 0), p_tok.repeat(2, 1)

    def _scatter_images(self, x, input_ids, tokens, pixel_values, image_grid_thw):
        """Vision features at every ``<|image_pad|>`` of the clean stream and of each noisy view
        (image tokens are prompt tokens, never masked, so every stream holds the row's image tokens
        at the same positions); features are consumed in row-major order of ``input_ids``."""
        vis = self.decoder.visual
        if vis is None:
            raise ValueError("image inputs given but the checkpoint has no vision tower")
        img = self.cfg.image_token_id
        feats = vis(pixel_values, image_grid_thw).to(x.dtype)
        row_img = input_ids == img
        n = int(row_img.sum())
        if n != feats.shape[0]:
            raise ValueError(f"{n} image tokens but {feats.shape[0]} image features")
        B, L = input_ids.shape
        S = tokens.shape[1] // L
        fidx = (torch.cumsum(row_img.reshape(-1).long(), 0) - 1).view(B, L).repeat(1, S).reshape(-1)
        tok_img = (tokens == img).reshape(-1)
        if not torch.equal(tok_img, row_img.repeat(1, S).reshape(-1)):
            raise ValueError("an image token was masked in a noisy view (image tokens must be prompt tokens)")
        where = torch.nonzero(tok_img).squeeze(1)
        return x.index_put((where,), feats.index_select(0, fidx[where]))

    def forward_flare(self, input_ids, labels, attention_mask, seg_id=None, turn_id=None, pixel_values=None,
                      image_grid_thw=None, mrope_pos=None, pointer=None):
        """Two-stream objective.  ``pointer`` (optional) trains the decision head on some of the same
        rows: ``decide`` / ``opts`` are clean-stream positions ``row * L + p``, ``owner`` the question
        of each option, ``questions`` the per-question records of ``decision_loss`` and ``weight``
        the loss weight; the pointer loss is added to the row's block-diffusion loss."""
        dev = input_ids.device
        B, L = input_ids.shape
        assert L % self.bd_size == 0, "two-stream rows must be a multiple of bd_size (collator bucket)"
        answer = (labels != -100) & attention_mask.bool()
        noisy, vlab, rate = self._flare_views(input_ids, labels, answer)
        if self.full_mask:
            V = 1
            xt_tok, vl, rt = noisy, vlab[:, None], rate[:, None]
        else:
            V = 2
            xt_tok = noisy.view(2, B, L).transpose(0, 1).reshape(B, 2 * L)
            vl = vlab.view(2, B, L).transpose(0, 1)
            rt = rate.view(2, B, L).transpose(0, 1)
        S = 1 + V
        T = S * L
        tokens = torch.cat([input_ids, xt_tok], 1)                         # [B, S*L]
        pos1 = doc_positions(seg_id) if seg_id is not None else torch.arange(L, device=dev)[None].expand(B, -1)
        pos = pos1.repeat(1, S)
        spos = torch.arange(L, device=dev)[None].expand(B, -1).repeat(1, S)  # position inside the stream
        stream = torch.arange(S, device=dev).repeat_interleave(L)[None].expand(B, -1)
        seg = torch.where(stream == 0, X0, XT)
        rblk = spos // self.bd_size
        segid = seg_id.repeat(1, S) if seg_id is not None else torch.zeros(B, T, dtype=torch.long, device=dev)
        pos3 = mrope_pos.repeat(1, 1, S) if mrope_pos is not None else None   # every stream shares positions
        actx = self.make_actx(seg, spos, rblk, segid, stream, pos, self.ar_loss_weight > 0, pos3=pos3)
        actx.linear = LinearLayout("two_stream", L=L, V=V, bd=self.bd_size, causal_clean=self.ar_loss_weight > 0,
                                   causal_noisy=self.within_block_causal,
                                   doc_start=doc_starts(seg_id) if seg_id is not None else None)
        # loss rows (host sync once, before the stack)
        shift_vl = vl[:, :, 1:]                                            # [B, V, L-1]
        sel = shift_vl != -100
        idx = torch.nonzero(sel.reshape(-1)).squeeze(1)
        r, rem = idx // (V * (L - 1)), idx % (V * (L - 1))
        v, t = rem // (L - 1), rem % (L - 1)
        d_rows = r * T + (1 + v) * L + t
        d_tgt = vl[r, v, t + 1]
        pos_sel = (pos1[r, t + 1] % self.bd_size) if self.pos_decay_gamma > 0 else None
        w_diff = self._weights(rt[r, v, t + 1], pos_sel)
        ar_w = self.ar_loss_weight
        n_diff = idx.numel()
        if ar_w > 0:
            clean_lab = torch.where(answer, input_ids, torch.full_like(input_ids, -100))
            ok = torch.ones(B, L - 1, dtype=torch.bool, device=dev)
            if turn_id is not None:
                ok &= (turn_id[:, :-1] == turn_id[:, 1:]) & (turn_id[:, 1:] >= 0)
            if seg_id is not None:
                ok &= seg_id[:, :-1] == seg_id[:, 1:]
            selc = (clean_lab[:, 1:] != -100) & ok
            aidx = torch.nonzero(selc.reshape(-1)).squeeze(1)
            ab, at = aidx // (L - 1), aidx % (L - 1)
            n_ar = aidx.numel()
            rows = torch.cat([d_rows, ab * T + at])
            tgt = torch.cat([d_tgt, clean_lab[ab, at + 1]])
            wts = torch.cat([w_diff / (1 + ar_w),
                             torch.full((n_ar,), ar_w / ((1 + ar_w) * max(n_ar, 1)), device=dev)])
        else:
            n_ar = 0
            rows, tgt, wts = d_rows, d_tgt, w_diff
        x = self.decoder.embed_tokens(tokens)
        if pixel_values is not None:
            x = self._scatter_images(x, input_ids, tokens, pixel_values, image_grid_thw)
        hidden = self.run_stack(x, actx)
        loss, ce = fused_linear_ce(hidden.index_select(0, rows), self.decoder.lm_weight, tgt, wts, chunk=self.ce_chunk)
        with torch.no_grad():
            diff = torch.dot(ce[:n_diff], w_diff) if n_diff else torch.zeros((), device=dev)
            ar = ce[n_diff:].mean() if n_ar else torch.zeros((), device=dev)
        logs = {"diff_loss": diff, "ar_loss": ar, "ntok": n_diff}
        if pointer is not None and pointer["questions"]:
            if self.decision_head is None:
                raise RuntimeError("pointer rows given but the model has no decision head (decision_head_dim=0)")

            def clean(flat):          # clean-stream position row * L + p -> hidden row row * T + p
                return (flat // L) * T + flat % L
            z = self.decision_head(hidden.index_select(0, clean(pointer["decide"])),
                                   hidden.index_select(0, clean(pointer["opts"])), pointer["owner"])
            dloss, acc = decision_loss(z, pointer)
            loss = loss + pointer.get("weight", 1.0) * dloss
            logs.update(decision_loss=dloss.detach(), decision_acc=acc)
        return loss, logs

    # ----------------------------------------------------------------------------------------
    def _causal_rows(self, input_ids, seg_id, valid=None):
        """Attention + linear layout of document-isolated causal rows."""
        dev = input_ids.device
        B, L = input_ids.shape
        valid = torch.ones_like(input_ids, dtype=torch.bool) if valid is None else valid
        segid = torch.where(valid, seg_id, torch.full_like(seg_id, -1)) if seg_id is not None else \
            torch.where(valid, 0, -1)
        pos = doc_positions(seg_id) if seg_id is not None else torch.arange(L, device=dev)[None].expand(B, -1)
        seg = torch.where(valid, SHARED, 0)
        opos = torch.arange(L, device=dev)[None].expand(B, -1)
        zeros = torch.zeros(B, L, dtype=torch.int32, device=dev)
        actx = self.make_actx(seg, opos, zeros, segid, zeros, pos, True)
        actx.linear = LinearLayout("causal", doc_start=doc_starts(segid) if seg_id is not None else None)
        return actx

    def forward_ar(self, input_ids, labels, attention_mask, seg_id=None):
        dev = input_ids.device
        B, L = input_ids.shape
        actx = self._causal_rows(input_ids, seg_id, attention_mask.bool())
        sel = labels[:, 1:] != -100
        idx = torch.nonzero(sel.reshape(-1)).squeeze(1)
        bi, ti = idx // (L - 1), idx % (L - 1)
        n = idx.numel()
        x = self.decoder.embed_tokens(input_ids)
        hidden = self.run_stack(x, actx)
        loss, _ = fused_linear_ce(hidden.index_select(0, bi * L + ti), self.decoder.lm_weight, labels[bi, ti + 1],
                                  torch.full((n,), 1.0 / max(n, 1), device=dev), chunk=self.ce_chunk)
        return loss, {"diff_loss": torch.zeros((), device=dev), "ar_loss": loss.detach(), "ntok": n}

    def forward_decision(self, decision):
        if self.decision_head is None:
            raise RuntimeError("decision batch given but the model has no decision head (decision_head_dim=0)")
        ids, seg = decision["input_ids"], decision["seg_id"]
        T = ids.shape[1]
        actx = self._causal_rows(ids, seg)
        hidden = self.run_stack(self.decoder.embed_tokens(ids), actx)
        z = self.decision_head(hidden[decision["decide"]], hidden[decision["opts"]], decision["owner"])
        loss, acc = decision_loss(z, decision)
        return loss, {"decision_loss": loss.detach(), "decision_acc": acc,
                      "decision_questions": len(decision["questions"]), "decision_tokens": T}
