"""Chunked (WY) form of the gated-delta rule, stated in PyTorch: the exact decomposition that the
sm_100a chunk kernels in ``csrc/gdn_chunk.cu`` compute, with an explicit backward.

The per-token recurrence (``ops.gdn_reference``; reference semantics ``train/models/hybrid.py:137-212``
for the causal rule with document resets and ``:215-324`` for the two-stream block-diffusion form)::

    S_t = a_t S_{t-1} + k_t u_t^T,   u_t = beta_t (v_t - a_t S_{t-1}^T k_t),   o_t = S_{r(t)}^T q_t

is regrouped over chunks of C tokens (Yang, Kautz, Hatamizadeh, "Gated Delta Networks", 2024, and
Yang et al., "Parallelizing Linear Transformers with the Delta Rule over Sequence Length", 2024).
Inside a chunk, with S0 the state entering it:

* segments: a document start inside the chunk begins a new segment whose recurrence starts from
  zero (a reset is a decay of 0), ``carry_t`` = 1 for tokens of the first segment when the chunk
  does not itself start a document;
* ``G_t`` = cumulative log-decay from the start of t's segment, ``r(t)`` = t (token-causal
  read-out) or the last token of the segment (block-end read-out), ``Gr_t = G_{r(t)}``;
* ``A_ts = beta_t (k_t . k_s) exp(G_t - G_s)`` for s < t in one segment, ``T = (I + A)^-1``;
* ``W = T diag(beta carry e^G) K``, ``U~ = T diag(beta) V``, and the pseudo-values
  ``U = U~ - W S0``;
* ``P_ts = (q_t . k_s) exp(Gr_t - G_s)`` for s <= r(t) in one segment,
  ``O = diag(carry e^Gr) Q S0 + P U``;
* state after the chunk ``S1 = carry_last e^{G_last} S0 + K~^T U`` with
  ``K~_s = [s in the last segment] exp(G_last - G_s) k_s``.

Every exponent is <= 0, so no factor can overflow whatever the chunk length.  All products are
chunk-local except ``W S0`` and ``K~^T U``: the state recurrence over chunks is the only
sequential part.  ``chunk_fwd`` / ``chunk_bwd`` below work on a batch of chunks ``[..., C, d]``;
``causal_fwd`` / ``two_stream_fwd`` chain them like the kernels do (the clean stream's chunk is the
diffusion block, so every block start is a chunk start and the noisy blocks restart from the
stored chunk-start states).
"""
import torch


def chunk_meta(g, rs, readout_block):
    """Per-chunk metadata from log-decays ``g`` [..., C] and segment-start flags ``rs`` [..., C]
    (``rs[..., 0]``: the chunk itself starts a document).  Returns (G, Gr, rd, seg, carry)."""
    C = g.shape[-1]
    rs = rs.bool()
    seg = torch.cumsum(rs.long(), -1) - rs[..., :1].long()
    carry = (seg == 0) & ~rs[..., :1]
    G = torch.zeros_like(g)
    run = torch.zeros_like(g[..., 0])
    for t in range(C):
        run = g[..., t] if t == 0 else torch.where(rs[..., t], g[..., t], run + g[..., t])
        G[..., t] = run
    idx = torch.arange(C, device=g.device).expand_as(seg)
    if readout_block:
        # last index of each token's segment: the next segment start minus one (C - 1 for the last)
        nxt = torch.full_like(idx, C)
        last = torch.full_like(idx[..., 0], C)
        for t in range(C - 1, -1, -1):
            nxt[..., t] = last
            last = torch.where(rs[..., t], torch.full_like(last, t), last)
        rd = nxt - 1
    else:
        rd = idx
    Gr = torch.gather(G, -1, rd)
    return G, Gr, rd, seg, carry.to(g.dtype)


def _masks(seg, rd):
    C = seg.shape[-1]
    t = torch.arange(C, device=seg.device)
    same = seg[..., :, None] == seg[..., None, :]
    mA = same & (t[None, :] < t[:, None])                         # s < t
    mP = same & (t[None, :] <= rd[..., :, None])                  # s <= r(t)
    return mA, mP


def _expdiff(a, b, mask):
    """exp(a_t - b_s) where mask, else 0 (never evaluates exp of a positive masked-out exponent)."""
    d = a[..., :, None] - b[..., None, :]
    return torch.where(mask, torch.exp(torch.where(mask, d, torch.zeros_like(d))), torch.zeros_like(d))


def chunk_fwd(q, k, v, g, beta, rs, S0, readout_block=False):
    """One chunk (batched): q (scaled) / k [..., C, dk], v [..., C, dv], g / beta / rs [..., C],
    S0 [..., dk, dv].  Returns (O, U, S1, cache)."""
    G, Gr, rd, seg, carry = chunk_meta(g, rs, readout_block)
    mA, mP = _masks(seg, rd)
    EA = _expdiff(G, G, mA)
    EP = _expdiff(Gr, G, mP)
    KK = k @ k.transpose(-1, -2)
    QK = q @ k.transpose(-1, -2)
    A = beta[..., :, None] * KK * EA
    eye = torch.eye(A.shape[-1], dtype=A.dtype, device=A.device)
    T = torch.linalg.solve_triangular(eye + A, eye.expand_as(A), upper=False, unitriangular=True)
    kb_s = beta * carry * torch.exp(G)
    Kb = kb_s[..., None] * k
    Vb = beta[..., None] * v
    W = T @ Kb
    Ut = T @ Vb
    U = Ut - W @ S0
    P = QK * EP
    og = carry * torch.exp(Gr)
    O = og[..., None] * (q @ S0) + P @ U
    Gl = G[..., -1:]
    ml = (seg == seg[..., -1:]).to(g.dtype)
    kt_s = ml * torch.exp(torch.where(ml.bool(), Gl - G, torch.zeros_like(G)))
    Kt = kt_s[..., None] * k
    cl = carry[..., -1] * torch.exp(G[..., -1])
    S1 = cl[..., None, None] * S0 + Kt.transpose(-1, -2) @ U
    cache = dict(G=G, Gr=Gr, rd=rd, seg=seg, carry=carry, mA=mA, mP=mP, EA=EA, EP=EP, KK=KK, QK=QK, A=A, T=T,
                 Kb=Kb, Vb=Vb, W=W, U=U, P=P, og=og, Kt=Kt, kt_s=kt_s, cl=cl, ml=ml, O=O)
    return O, U, S1, cache


def _rev_segcumsum(x, rs):
    """y_t = sum of x_t' over t' >= t in t's segment (segments start where rs is set)."""
    C = x.shape[-1]
    y = torch.zeros_like(x)
    run = torch.zeros_like(x[..., 0])
    for t in range(C - 1, -1, -1):
        run = run + x[..., t]
        y[..., t] = run
        run = torch.where(rs[..., t].bool(), torch.zeros_like(run), run)
    return y


def chunk_bwd(q, k, v, g, beta, rs, S0, dO, dS1, cache):
    """Explicit backward of ``chunk_fwd``: returns (dq, dk, dv, dg, dbeta, dS0)."""
    c = cache
    T, U, P, W = c["T"], c["U"], c["P"], c["W"]
    tr = lambda x: x.transpose(-1, -2)  # noqa: E731
    dU = tr(P) @ dO + c["Kt"] @ dS1
    dP = (dO @ tr(U)) * c["mP"]
    dPE = dP * c["EP"]                                             # gradient w.r.t. (q . k) entries
    dq = dPE @ k + c["og"][..., None] * (dO @ tr(S0))
    dk = tr(dPE) @ q
    dG = torch.zeros_like(g)
    # every term of o_t scales with e^{Gr_t}: dGr_t = dO_t . O_t
    dGr = (dO * c["O"]).sum(-1)
    dG = dG.scatter_add(-1, c["rd"], dGr)
    dG = dG - (dP * P).sum(-2)
    # end state
    dKt = U @ tr(dS1)                                              # [C, dk]: dS1 u_s
    dk = dk + c["kt_s"][..., None] * dKt
    ktk = (c["Kt"] * dKt).sum(-1)
    dG = dG - ktk
    dG[..., -1] += ktk.sum(-1) + c["cl"] * (S0 * dS1).sum((-1, -2))
    dS0 = tr(c["og"][..., None] * q) @ dO + c["cl"][..., None, None] * dS1 - tr(W) @ dU
    # WY factors
    dW = -dU @ tr(S0)
    dT = dU @ tr(c["Vb"]) + dW @ tr(c["Kb"])
    dVb = tr(T) @ dU
    dKb = tr(T) @ dW
    dA = -(tr(T) @ dT @ tr(T)) * c["mA"]
    dv = beta[..., None] * dVb
    kb_s = beta * c["carry"] * torch.exp(c["G"])
    dk = dk + kb_s[..., None] * dKb
    dAE = dA * beta[..., :, None] * c["EA"]
    dk = dk + dAE @ k + tr(dAE) @ k
    dAA = dA * c["A"]
    dbeta = (dA * c["KK"] * c["EA"]).sum(-1) + c["carry"] * torch.exp(c["G"]) * (dKb * k).sum(-1) + (dVb * v).sum(-1)
    dG = dG + dAA.sum(-1) - dAA.sum(-2) + (dKb * c["Kb"]).sum(-1)
    dg = _rev_segcumsum(dG, rs)
    return dq, dk, dv, dg, dbeta, dS0


def _pad_chunks(x, C, n):
    pad = (-n) % C
    if pad:
        shape = list(x.shape)
        shape[1] = pad
        x = torch.cat([x, x.new_zeros(shape)], 1)
    return x


def _to_chunks(x, C):
    """[B, n, H, ...] -> [B, H, nch, C, ...]"""
    B, n, H = x.shape[:3]
    x = _pad_chunks(x, C, n)
    x = x.reshape(B, -1, C, H, *x.shape[3:])
    return x.permute(0, 3, 1, 2, *range(4, x.dim())).contiguous()


def _from_chunks(x, n):
    B, H, nch, C = x.shape[:4]
    x = x.permute(0, 2, 3, 1, *range(4, x.dim())).reshape(B, nch * C, H, *x.shape[4:])
    return x[:, :n]


def stream_scan(q, k, v, g, beta, rs, readout_block=False):
    """Chunks of one stream [B, H, nch, C, ...] chained through the state.  Returns (O, states
    entering each chunk [B, H, nch, dk, dv], caches)."""
    B, H, nch = q.shape[:3]
    S = q.new_zeros(B, H, k.shape[-1], v.shape[-1])
    outs, states, caches = [], [], []
    for ci in range(nch):
        states.append(S)
        O, U, S, cache = chunk_fwd(q[:, :, ci], k[:, :, ci], v[:, :, ci], g[:, :, ci], beta[:, :, ci], rs[:, :, ci],
                                   S, readout_block)
        outs.append(O)
        caches.append(cache)
    return torch.stack(outs, 2), torch.stack(states, 2), caches


def causal_fwd(q, k, v, g, beta, doc_start=None, C=64):
    """Causal rule over [B, T, H, d] (q already scaled and both L2-normalised) -> o [B, T, H, dv]."""
    B, T = q.shape[:2]
    rs = torch.zeros(B, T, dtype=torch.bool, device=q.device) if doc_start is None else doc_start.bool()
    ch = lambda x: _to_chunks(x, C)  # noqa: E731
    rsc = _to_chunks(rs[:, :, None].expand(-1, -1, q.shape[2]), C)
    O, _, _ = stream_scan(ch(q), ch(k), ch(v), ch(g), ch(beta), rsc)
    return _from_chunks(O, T)


def two_stream_fwd(q, k, v, g, beta, L, V, bd, causal_clean=True, causal_noisy=False, doc_start=None):
    """Two-stream rule over a [x0 ; xt_1..xt_V] row [B, (1+V)L, H, d]: the clean stream in chunks
    of one block, then every noisy block from the stored state at its block start."""
    B, _, H = q.shape[:3]
    rs = torch.zeros(B, L, dtype=torch.bool, device=q.device) if doc_start is None else doc_start.bool()
    rsc = _to_chunks(rs[:, :, None].expand(-1, -1, H), bd)
    sl = lambda x, i: _to_chunks(x[:, i * L:(i + 1) * L], bd)  # noqa: E731
    O0, states, _ = stream_scan(sl(q, 0), sl(k, 0), sl(v, 0), sl(g, 0), sl(beta, 0), rsc, not causal_clean)
    outs = [_from_chunks(O0, L)]
    # noisy chunk n starts from the clean state entering block n; only a document start at the
    # block start matters (documents start on block boundaries)
    rs_n = torch.zeros_like(rsc)
    rs_n[..., 0] = rsc[..., 0]
    for vi in range(V):
        On, _, _, _ = chunk_fwd(sl(q, 1 + vi), sl(k, 1 + vi), sl(v, 1 + vi), sl(g, 1 + vi), sl(beta, 1 + vi), rs_n,
                                states, not causal_noisy)
        outs.append(_from_chunks(On, L))
    return torch.cat(outs, 1)
