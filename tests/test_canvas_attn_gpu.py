"""Serving canvas attention kernels against an fp32 PyTorch statement of the canvas rule.

The rule: canvas row i of a request attends every cached prefix key; among the canvas keys it sees
key c iff c <= i (the first n_clean rows are token-causal) or i >= n_clean (MASK rows see the whole
canvas).  Both kernels are checked: the tensor-core one (called with the device error word) and the
split-K warp-MMA one, on dense and paged caches, head_dim 128 and 256, one and several key splits.
"""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _reference(q, K, V, pos, blk, n_clean, scale):
    """q [B*blk, Hq, D]; K / V: per request [keys, Hkv, D] (fp32).  Returns fp32 [B*blk, Hq, D]."""
    B = q.shape[0] // blk
    Hq = q.shape[1]
    out = torch.empty(q.shape, dtype=torch.float32)
    for b in range(B):
        p = int(pos[b])
        kend = p + blk
        G = Hq // K[b].shape[1]
        kb = K[b][:kend].repeat_interleave(G, dim=1)
        vb = V[b][:kend].repeat_interleave(G, dim=1)
        qb = q[b * blk:(b + 1) * blk].float()
        s = torch.einsum("ihd,khd->hik", qb, kb) * scale
        i = torch.arange(blk)[:, None]
        c = torch.arange(kend)[None, :] - p
        vis = (c < 0) | (c <= i) | (i >= n_clean)
        s = s.masked_fill(~vis, float("-inf"))
        out[b * blk:(b + 1) * blk] = torch.einsum("hik,khd->ihd", torch.softmax(s, -1), vb)
    return out


def _case(D, Hq, Hkv, blk, maxlen, paged, seed=0):
    g = torch.Generator().manual_seed(seed)
    B, n_slots = 3, 5
    slot = torch.tensor([3, 0, 4], dtype=torch.int32)
    pos = torch.tensor([maxlen - blk, 5, (maxlen - blk) // 2 + 3], dtype=torch.int32)
    q = torch.randn(B * blk, Hq, D, generator=g)
    if paged:
        maxpages = maxlen // 64
        n_pages = n_slots * maxpages + 3
        kc = torch.randn(n_pages, 64, Hkv, D, generator=g)
        vc = torch.randn(n_pages, 64, Hkv, D, generator=g)
        ptab = torch.zeros(n_slots, maxpages, dtype=torch.int32)
        perm = torch.randperm(n_pages, generator=g)
        used = 0
        K, V = [], []
        for b in range(B):
            s = int(slot[b])
            need = (int(pos[b]) + blk + 63) // 64
            ptab[s, :need] = perm[used:used + need].int()
            used += need
            pages = ptab[s, :need].long()
            K.append(kc[pages].reshape(-1, Hkv, D))
            V.append(vc[pages].reshape(-1, Hkv, D))
    else:
        ptab = None
        kc = torch.randn(n_slots, maxlen, Hkv, D, generator=g)
        vc = torch.randn(n_slots, maxlen, Hkv, D, generator=g)
        K = [kc[int(s)] for s in slot]
        V = [vc[int(s)] for s in slot]
    bf = lambda t: t.to(torch.bfloat16)
    K = [bf(k).float() for k in K]
    V = [bf(v).float() for v in V]
    return slot, pos, bf(q), bf(kc), bf(vc), ptab, K, V


@pytest.mark.parametrize("paged", [False, True], ids=["dense", "paged"])
@pytest.mark.parametrize("D,Hq,Hkv", [(256, 16, 4), (128, 4, 2), (128, 8, 8)], ids=["d256-g4", "d128-g2", "d128-g1"])
@pytest.mark.parametrize("blk", [7, 33, 63])
@pytest.mark.parametrize("maxlen", [256, 1024], ids=["one-split", "splits"])
@pytest.mark.parametrize("impl", ["tc", "mma"])
def test_canvas_attention_matches_fp32(impl, maxlen, blk, D, Hq, Hkv, paged):
    from trida_stack_b200.ops._ext import ext
    from trida_stack_b200.ops.blocks import device_error_word
    C = ext()
    slot, pos, q, kc, vc, ptab, K, V = _case(D, Hq, Hkv, blk, maxlen, paged)
    n_clean = blk // 2 + 1
    scale = 1.0 / math.sqrt(D)
    ref = _reference(q, K, V, pos, blk, n_clean, scale)
    dev = torch.device("cuda")
    # the output is a view of a larger buffer whose tail must stay untouched
    buf = torch.full((q.shape[0] + 5, Hq, D), float("nan"), dtype=torch.bfloat16, device=dev)
    out = buf[:q.shape[0]]
    err = device_error_word(dev) if impl == "tc" else None
    if err is not None:
        err.zero_()
    C.canvas_attention(q.to(dev), kc.to(dev), vc.to(dev), slot.to(dev), pos.to(dev), out, blk, n_clean, maxlen,
                       scale, ptab.to(dev) if ptab is not None else None, err)
    torch.cuda.synchronize()
    if err is not None:
        assert int(err.item()) == 0, f"device wait timed out (code {int(err.item())})"
    got = out.float().cpu()
    assert torch.isfinite(got).all()
    assert torch.isnan(buf[q.shape[0]:].float()).all()
    rel = ((got - ref).norm() / ref.norm()).item()
    assert rel < 1e-2, rel
    torch.testing.assert_close(got, ref, atol=3e-2, rtol=3e-2)


@pytest.mark.parametrize("qscale", [1.0, 8.0], ids=["scores-small", "scores-large"])
@pytest.mark.parametrize("impl", ["tc", "mma"])
def test_canvas_attention_many_requests(impl, qscale):
    """Serving-sized grid (64 requests x 64 causal rows after a 256-position prefix, several waves of
    CTAs per SM) with pages handed out chunk by chunk as the runtime's allocator does; large query
    scales make row maxima grow by more than 2^16 between key tiles (the lazy O rescale)."""
    from trida_stack_b200.ops._ext import ext
    from trida_stack_b200.ops.blocks import device_error_word
    C = ext()
    g = torch.Generator().manual_seed(3)
    B, blk, Hq, Hkv, D, pos0 = 64, 64, 16, 4, 256, 256
    maxpages = 18
    n_slots = B + 1
    kend = pos0 + blk
    need = kend // 64
    n_pages = n_slots * maxpages
    ptab = torch.zeros(n_slots, maxpages, dtype=torch.int32)
    nxt = 0
    for c in range(need):                          # chunk by chunk, slot by slot
        for s in range(B):
            ptab[s, c] = nxt
            nxt += 1
    kc = torch.randn(n_pages, 64, Hkv, D, generator=g).to(torch.bfloat16)
    vc = torch.randn(n_pages, 64, Hkv, D, generator=g).to(torch.bfloat16)
    q = (torch.randn(B * blk, Hq, D, generator=g) * qscale).to(torch.bfloat16)
    slot = torch.arange(B, dtype=torch.int32)
    pos = torch.full((B,), pos0, dtype=torch.int32)
    K = [kc[ptab[s, :need].long()].reshape(-1, Hkv, D).float() for s in range(B)]
    V = [vc[ptab[s, :need].long()].reshape(-1, Hkv, D).float() for s in range(B)]
    scale = 1.0 / math.sqrt(D)
    ref = _reference(q, K, V, pos, blk, blk, scale)
    dev = torch.device("cuda")
    out = torch.full((B * blk, Hq, D), float("nan"), dtype=torch.bfloat16, device=dev)
    err = device_error_word(dev) if impl == "tc" else None
    if err is not None:
        err.zero_()
    C.canvas_attention(q.to(dev), kc.to(dev), vc.to(dev), slot.to(dev), pos.to(dev), out, blk, blk, 1152, scale,
                       ptab.to(dev), err)
    torch.cuda.synchronize()
    if err is not None:
        assert int(err.item()) == 0
    got = out.float().cpu()
    bad = (~torch.isfinite(got)).any(-1)
    assert not bad.any(), f"non-finite (row, head) outputs: {bad.nonzero()[:8].tolist()}"
    rel = ((got - ref).norm() / ref.norm()).item()
    assert rel < 1e-2, rel
