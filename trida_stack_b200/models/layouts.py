"""Packed, merged-view and multi-turn block-diffusion layouts (the non-default forward paths).

* ``forward_packed`` -- several ``[prompt | response]`` documents per row, isolated from each
  other (``segid``); region B is the clean copy of every response token, gathered in position order
  (``train/models/block_diffusion.py:431-524``).
* ``forward_packed_merged`` -- the same objective with the prompt stored once: the row is
  ``[region A (view 1) | view-2 response tokens | clean response]`` and the mask isolates views
  (``view``); losses equal ``forward_packed``'s (``:526-661``).
* ``forward_multiturn`` -- every assistant turn of one conversation; a global, conversation-ordered
  block id makes later turns see earlier clean turns, and the AR loss never crosses a turn
  (``:666-759``).

Noise is drawn per key (one Bernoulli rate per (document, response block) or per global block)
with the reference's draw order, so a fixed seed gives the same views.
"""
import torch
import torch.nn.functional as F

from ..ops.ce import fused_linear_ce
from ..ops.reference import PAD, SHARED, X0, XT
from .block_diffusion import bucketed_clean_len


def _keyed_noise(m, answer, block_key, eps=1e-3):
    B, L = answer.shape
    nkey = int(block_key.max().item()) + 1 if block_key.numel() else 1
    p_key = (1 - eps) * torch.rand(B, nkey, device=answer.device) + eps
    p_tok = torch.gather(p_key, 1, block_key.clamp(min=0))
    return (torch.rand(B, L, device=answer.device) < p_tok) & answer, p_tok


def _views(m, input_ids, labels, answer, picked):
    def one(sel):
        apply = sel & answer
        return (torch.where(apply, torch.full_like(input_ids, m.mask_id), input_ids),
                torch.where(apply, labels, torch.full_like(labels, -100)))
    na, la = one(picked)
    nb, lb = one(~picked)
    return torch.cat([na, nb], 0), torch.cat([la, lb], 0)


def _gather_order(answer, rpad):
    """Indices of the response tokens of each row, in position order, padded to ``rpad``."""
    B, L = answer.shape
    ar = torch.arange(L, device=answer.device)
    order = torch.argsort((~answer).int() * (L + 1) + ar[None, :], dim=1)
    src = order[:, :rpad].clamp(max=L - 1)
    valid = torch.arange(rpad, device=answer.device)[None, :] < answer.sum(1, keepdim=True)
    return src, valid


def _rows(sel, row_len, offset):
    """Flat hidden-row indices (b * T + offset + t) of the True entries of ``sel`` [B, n]."""
    idx = torch.nonzero(sel.reshape(-1)).squeeze(1)
    n = sel.shape[1]
    return idx // n, idx % n, (idx // n) * row_len + offset + idx % n


def _finish(m, tokens, pos, seg, rblk, segid, view, d_rows, d_tgt, d_rate, a_rows, a_tgt):
    """Run the decoder over the layout and the combined diffusion + AR fused CE."""
    dev = tokens.device
    actx = m.make_actx(seg, pos, rblk, segid, view, pos, m.ar_loss_weight > 0)
    w_diff = m._weights(d_rate)
    ar_w = m.ar_loss_weight
    n_diff, n_ar = d_rows.numel(), (a_rows.numel() if ar_w > 0 else 0)
    if ar_w > 0:
        rows = torch.cat([d_rows, a_rows])
        tgt = torch.cat([d_tgt, a_tgt])
        wts = torch.cat([w_diff / (1 + ar_w), torch.full((n_ar,), ar_w / ((1 + ar_w) * max(n_ar, 1)), device=dev)])
    else:
        rows, tgt, wts = d_rows, d_tgt, w_diff
    x = m.decoder.embed_tokens(tokens)
    hidden = m.run_stack(x, actx)
    loss, ce = fused_linear_ce(hidden.index_select(0, rows), m.decoder.lm_weight, tgt, wts, chunk=m.ce_chunk)
    with torch.no_grad():
        diff = torch.dot(ce[:n_diff], w_diff) if n_diff else torch.zeros((), device=dev)
        ar = ce[n_diff:].mean() if n_ar else torch.zeros((), device=dev)
    return loss, {"diff_loss": diff, "ar_loss": ar, "ntok": n_diff}


def _two_view_region_b(m, input_ids, labels, attention_mask, block_key, rblk_tok, segid_tok, bound_tok):
    """Shared body of the packed and multi-turn layouts (2B rows of [A | B])."""
    dev = input_ids.device
    B, L = input_ids.shape
    valid = attention_mask.bool()
    answer = (labels != -100) & valid
    picked, p_tok = _keyed_noise(m, answer, block_key)
    noisy, vlab = _views(m, input_ids, labels, answer, picked)
    rate = p_tok.repeat(2, 1)
    clean = input_ids.repeat(2, 1)
    valid2, ans2 = valid.repeat(2, 1), answer.repeat(2, 1)
    rblkA = rblk_tok.repeat(2, 1)
    segidA = segid_tok.repeat(2, 1)
    boundA = bound_tok.repeat(2, 1)
    BB = 2 * B
    rpad = bucketed_clean_len(int(ans2.sum(1).max().item()), m.bd_size, m.response_buckets)
    src, bval = _gather_order(ans2, rpad)
    T = L + rpad
    posA = torch.arange(L, device=dev)[None].expand(BB, -1)
    tokens = torch.cat([noisy, torch.gather(clean, 1, src)], 1)
    pos = torch.cat([posA, src], 1)
    segA = torch.where(valid2, torch.where(ans2, XT, SHARED), PAD)
    segB = torch.where(bval, X0, PAD)
    seg = torch.cat([segA, segB], 1)
    rblk = torch.cat([rblkA, torch.gather(rblkA, 1, src)], 1)
    segidB = torch.where(bval, torch.gather(segidA, 1, src), torch.full_like(src, -1))
    segid = torch.cat([segidA, segidB], 1)
    view = torch.zeros(BB, T, dtype=torch.int32, device=dev)
    # diffusion rows: region A, hidden[t] predicts label[t + 1]
    sel = vlab[:, 1:] != -100
    bi, ti, d_rows = _rows(sel, T, 0)
    d_tgt, d_rate = vlab[bi, ti + 1], rate[bi, ti + 1]
    # AR rows: region B, next token within the same bound (document / turn)
    boundB = torch.gather(boundA, 1, src)
    ar_sel = bval[:, 1:] & (boundB[:, :-1] == boundB[:, 1:]) & (boundB[:, 1:] >= 0)
    ab, aj, a_rows = _rows(ar_sel, T, L)
    a_tgt = torch.gather(clean, 1, src)[ab, aj + 1]
    return _finish(m, tokens, pos, seg, rblk, segid, view, d_rows, d_tgt, d_rate, a_rows, a_tgt)


def forward_packed(m, input_ids, labels, attention_mask, seg_id, resp_pos):
    if m.merged_views:
        return forward_packed_merged(m, input_ids, labels, attention_mask, seg_id, resp_pos)
    B, L = input_ids.shape
    valid = attention_mask.bool()
    answer = (labels != -100) & valid
    bd = m.bd_size
    nb = L // bd + 2
    zero = torch.zeros_like(resp_pos)
    rblk_tok = torch.where(answer, resp_pos.clamp(min=0) // bd, zero)
    block_key = torch.where(answer, seg_id.clamp(min=0) * nb + rblk_tok, zero)
    segid_tok = torch.where(valid, seg_id, torch.full_like(seg_id, -1))
    return _two_view_region_b(m, input_ids, labels, attention_mask, block_key, rblk_tok, segid_tok, segid_tok)


def forward_multiturn(m, input_ids, labels, attention_mask, resp_block, turn_id):
    valid = attention_mask.bool()
    answer = (labels != -100) & valid
    zero = torch.zeros_like(resp_block)
    block_key = torch.where(answer, resp_block.clamp(min=0), zero)
    rblk_tok = torch.where(answer, resp_block.clamp(min=0), zero)
    # no document isolation: one conversation per row; the global block order carries causality
    segid_tok = torch.where(valid, torch.zeros_like(resp_block), torch.full_like(resp_block, -1))
    return _two_view_region_b(m, input_ids, labels, attention_mask, block_key, rblk_tok, segid_tok, turn_id)


def forward_packed_merged(m, input_ids, labels, attention_mask, seg_id, resp_pos):
    """``[A (view 1, prompt once) | view-2 response tokens | clean response]``, batch B."""
    dev = input_ids.device
    B, L = input_ids.shape
    valid = attention_mask.bool()
    answer = (labels != -100) & valid
    bd = m.bd_size
    nb = L // bd + 2
    zero = torch.zeros_like(resp_pos)
    rblk_tok = torch.where(answer, resp_pos.clamp(min=0) // bd, zero)
    block_key = torch.where(answer, seg_id.clamp(min=0) * nb + rblk_tok, zero)
    picked, p_tok = _keyed_noise(m, answer, block_key)
    m1, m2 = picked & answer, (~picked) & answer
    noisy1 = torch.where(m1, torch.full_like(input_ids, m.mask_id), input_ids)
    noisy2 = torch.where(m2, torch.full_like(input_ids, m.mask_id), input_ids)
    lab1 = torch.where(m1, labels, torch.full_like(labels, -100))
    lab2 = torch.where(m2, labels, torch.full_like(labels, -100))
    rpad = bucketed_clean_len(int(answer.sum(1).max().item()), bd, m.response_buckets)
    src, bval = _gather_order(answer, rpad)
    T = L + 2 * rpad
    posA = torch.arange(L, device=dev)[None].expand(B, -1)
    x0_ids = torch.gather(input_ids, 1, src)
    tokens = torch.cat([noisy1, torch.gather(noisy2, 1, src), x0_ids], 1)
    pos = torch.cat([posA, src, src], 1)
    segA = torch.where(valid, torch.where(answer, XT, SHARED), PAD)
    segX = torch.where(bval, XT, PAD)
    segB = torch.where(bval, X0, PAD)
    seg = torch.cat([segA, segX, segB], 1)
    rb = torch.gather(rblk_tok, 1, src)
    rblk = torch.cat([rblk_tok, rb, rb], 1)
    segidA = torch.where(valid, seg_id, torch.full_like(seg_id, -1))
    sg = torch.where(bval, torch.gather(seg_id, 1, src), torch.full_like(src, -1))
    segid = torch.cat([segidA, sg, sg], 1)
    view = torch.cat([answer.long(), torch.where(bval, 2, 0), torch.zeros_like(src)], 1)
    # view-1 rows in A, plus view-2's first response token of each document (its predecessor is the
    # document's last prompt token, whose hidden state does not depend on the view)
    first = answer & ~F.pad(answer[:, :-1], (1, 0))
    a_lab = torch.where(first & m2, labels, lab1)
    selA = a_lab[:, 1:] != -100
    biA, tiA, rowsA = _rows(selA, T, 0)
    xlab = torch.where(bval, torch.gather(lab2, 1, src), torch.full_like(src, -100))
    selX = (xlab[:, 1:] != -100) & (sg[:, :-1] == sg[:, 1:])
    biX, tiX, rowsX = _rows(selX, T, L)
    d_rows = torch.cat([rowsA, rowsX])
    d_tgt = torch.cat([a_lab[biA, tiA + 1], xlab[biX, tiX + 1]])
    rate_x = torch.gather(p_tok, 1, src)
    d_rate = torch.cat([p_tok[biA, tiA + 1], rate_x[biX, tiX + 1]])
    ar_sel = bval[:, 1:] & (sg[:, :-1] == sg[:, 1:])
    ab, aj, a_rows = _rows(ar_sel, T, L + rpad)
    a_tgt = x0_ids[ab, aj + 1]
    return _finish(m, tokens, pos, seg, rblk, segid, view, d_rows, d_tgt, d_rate, a_rows, a_tgt)
