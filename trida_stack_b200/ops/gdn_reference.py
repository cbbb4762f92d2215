"""Plain-PyTorch statements of the gated-delta-rule (GDN) ops: the CPU path and the oracle of the
CUDA kernels.

Recurrence (per value head, fp32 state ``S`` of shape [dk, dv], q pre-scaled by dk^-0.5, q/k
L2-normalised)::

    S <- exp(g_t) * S
    u_t = beta_t * (v_t - S^T k_t)
    S <- S + k_t u_t^T
    o_t = S^T q_t

Two-stream block-diffusion form on a ``[x0 ; xt_1 ; ... ; xt_V]`` row of streams of length L with
blocks of ``bd`` tokens (the reference's FLARE kernels, ``train/models/hybrid.py:215-324``): the
clean stream x0 runs the plain causal recurrence (token-causal read-out, or block-end read-out when
``causal_clean`` is False) and records its state at every block end; each noisy block k of every
view restarts from the clean state at the end of block k-1 (zero for block 0 / at a document
start), runs its own tokens and -- bidirectional mode -- every token of the block reads the state
at the END of that noisy block (token-causal read-out when ``causal_noisy``).  Documents (packed
rows) restart the recurrence at their first token.
"""
import torch
import torch.nn.functional as F


def l2norm(x, eps=1e-6):
    return x * torch.rsqrt((x * x).sum(-1, keepdim=True) + eps)


def gates(a, b, A_log, dt_bias):
    """beta = sigmoid(b); g = -exp(A_log) * softplus(a + dt_bias)  (log decay, <= 0)."""
    beta = torch.sigmoid(b.float())
    g = -A_log.float().exp() * F.softplus(a.float() + dt_bias.float())
    return g, beta


def causal_conv(x, w, doc_start=None):
    """Depthwise causal conv + SiLU.  x [B, T, C], w [C, K]; the window restarts where
    ``doc_start`` [B, T] is True (zero left padding per document)."""
    B, T, C = x.shape
    K = w.shape[1]
    xf = x.float()
    out = torch.zeros_like(xf)
    if doc_start is None:
        doc_start = torch.zeros(B, T, dtype=torch.bool, device=x.device)
        doc_start[:, 0] = True
    # distance (in tokens) back to the start of each token's document
    ar = torch.arange(T, device=x.device)[None].expand(B, -1)
    start_pos = torch.cummax(torch.where(doc_start, ar, torch.zeros_like(ar)), 1).values
    back = ar - start_pos
    for j in range(K):
        shift = K - 1 - j           # tap j reads x[t - shift]
        if shift == 0:
            src = xf
        else:
            src = F.pad(xf, (0, 0, shift, 0))[:, :T]
        ok = (back >= shift)[..., None]
        out = out + torch.where(ok, src, torch.zeros_like(src)) * w[:, j].float()
    return F.silu(out).to(x.dtype)


def two_stream_conv(x, w, L, V, bd, doc_start=None):
    """Conv over a ``[x0 ; xt_1..xt_V]`` row: x0 is a plain causal conv; inside a noisy block the
    taps that fall in the same block read the noisy stream, earlier taps read the clean stream."""
    B, T, C = x.shape
    K = w.shape[1]
    x0 = x[:, :L]
    out = [causal_conv(x0, w, doc_start)]
    if doc_start is None:
        doc_start = torch.zeros(B, L, dtype=torch.bool, device=x.device)
        doc_start[:, 0] = True
    ar = torch.arange(L, device=x.device)[None].expand(B, -1)
    start_pos = torch.cummax(torch.where(doc_start, ar, torch.zeros_like(ar)), 1).values
    back = ar - start_pos
    inblk = ar % bd
    for v in range(V):
        xn = x[:, (1 + v) * L:(2 + v) * L].float()
        acc = torch.zeros_like(xn)
        for j in range(K):
            shift = K - 1 - j
            srcn = F.pad(xn, (0, 0, shift, 0))[:, :L] if shift else xn
            srcc = F.pad(x0.float(), (0, 0, shift, 0))[:, :L] if shift else x0.float()
            src = torch.where((inblk >= shift)[..., None], srcn, srcc)
            ok = (back >= shift)[..., None]
            acc = acc + torch.where(ok, src, torch.zeros_like(src)) * w[:, j].float()
        out.append(F.silu(acc).to(x.dtype))
    return torch.cat(out, 1)


def _step(S, q, k, v, g, beta):
    """One recurrence step on batched states S [..., dk, dv]."""
    S = S * g.exp()[..., None, None]
    u = beta[..., None] * (v - torch.einsum("...kv,...k->...v", S, k))
    S = S + k[..., :, None] * u[..., None, :]
    return S, torch.einsum("...kv,...k->...v", S, q)


def gdn_causal(q, k, v, g, beta, doc_start=None, readout_block=0):
    """Causal recurrence over [B, T, H, d] (q, k L2-normalised, q NOT yet scaled).  Returns
    (o [B, T, H, dv], block_end_states or None).  ``readout_block`` > 0 makes every token read the
    state at the end of its block of that size (block-causal read-out) and also returns the state
    at every block end [B, T // bd, H, dk, dv]."""
    B, T, H, dk = q.shape
    dv = v.shape[-1]
    qs = q.float() * dk ** -0.5
    S = torch.zeros(B, H, dk, dv, dtype=torch.float32, device=q.device)
    outs = []
    ends = []
    for t in range(T):
        if doc_start is not None:
            S = torch.where(doc_start[:, t][:, None, None, None], torch.zeros_like(S), S)
        S, o = _step(S, qs[:, t], k[:, t].float(), v[:, t].float(), g[:, t].float(), beta[:, t].float())
        outs.append(o)
        if readout_block and (t + 1) % readout_block == 0:
            ends.append(S)
    o = torch.stack(outs, 1)
    if readout_block:
        E = torch.stack(ends, 1)                                      # [B, nblk, H, dk, dv]
        return o, E
    return o, None


def gdn_block_bidirectional(q, k, v, g, beta, block_ids, initial_state=None):
    """Block-local bidirectional recurrence (the reference's research-level single-stream variant,
    ``train/models/hybrid.py:461-536``, superseded there by the two-stream form).

    ``block_ids`` [B, T] tags each token with its diffusion block (contiguous equal ids).  A block's
    entry state E is the causal state after everything before it; the forward sub-scan from E over
    the block gives the causal outputs, a backward sub-scan from E over the block's tokens in
    reverse gives a second read-out, and every token outputs their mean.  The next block enters
    with the forward (causal) exit state.  Inputs [B, T, H, d] (q, k L2-normalised, q not scaled);
    returns (o [B, T, H, dv] fp32, final state [B, H, dk, dv])."""
    B, T, H, dk = q.shape
    dv = v.shape[-1]
    qs, kf, vf, gf, bf = q.float() * dk ** -0.5, k.float(), v.float(), g.float(), beta.float()
    start = torch.ones(B, T, dtype=torch.bool, device=q.device)
    start[:, 1:] = block_ids[:, 1:] != block_ids[:, :-1]
    last = torch.ones(B, T, dtype=torch.bool, device=q.device)
    last[:, :-1] = block_ids[:, 1:] != block_ids[:, :-1]
    S = (torch.zeros(B, H, dk, dv, dtype=torch.float32, device=q.device) if initial_state is None
         else initial_state.float())
    entry, entries, fwd = S, [], []
    for t in range(T):
        entry = torch.where(start[:, t][:, None, None, None], S, entry)
        entries.append(entry)
        S, o = _step(S, qs[:, t], kf[:, t], vf[:, t], gf[:, t], bf[:, t])
        fwd.append(o)
    bwd = [None] * T
    R = torch.zeros_like(S)
    for t in range(T - 1, -1, -1):
        R = torch.where(last[:, t][:, None, None, None], entries[t], R)
        R, bwd[t] = _step(R, qs[:, t], kf[:, t], vf[:, t], gf[:, t], bf[:, t])
    return 0.5 * (torch.stack(fwd, 1) + torch.stack(bwd, 1)), S


def gdn_two_stream(q, k, v, g, beta, L, V, bd, causal_clean=True, causal_noisy=False, doc_start=None):
    """Two-stream recurrence over a ``[x0 ; xt_1..xt_V]`` row ([B, (1+V)L, H, d] inputs)."""
    B, T, H, dk = q.shape
    assert T == (1 + V) * L and L % bd == 0
    sl = slice(0, L)
    o0, E = gdn_causal(q[:, sl], k[:, sl], v[:, sl], g[:, sl], beta[:, sl], doc_start, readout_block=bd)
    nb = L // bd
    qs = q.float() * dk ** -0.5
    if not causal_clean:   # block-end read-out for the clean stream as well
        o0 = torch.einsum("bnhkv,bnthk->bnthv", E, qs[:, :L].reshape(B, nb, bd, H, dk)).reshape(B, L, H, -1)
    zero = torch.zeros_like(E[:, :1])
    Eprev = torch.cat([zero, E[:, :-1]], 1)                           # state entering each block
    if doc_start is not None:
        blk_start = doc_start[:, ::bd]                                # docs start on block boundaries
        Eprev = torch.where(blk_start[:, :, None, None, None], torch.zeros_like(Eprev), Eprev)
    outs = [o0]
    for vi in range(V):
        base = (1 + vi) * L
        S = Eprev.clone()                                             # [B, nb, H, dk, dv]
        per_tok = []
        for j in range(bd):
            idx = torch.arange(nb, device=q.device) * bd + j + base
            S, o = _step(S, qs[:, idx], k[:, idx].float(), v[:, idx].float(), g[:, idx].float(),
                         beta[:, idx].float())
            per_tok.append(o)
        if causal_noisy:
            on = torch.stack(per_tok, 2)                              # [B, nb, bd, H, dv]
        else:
            qb = qs[:, base:base + L].reshape(B, nb, bd, H, dk)
            on = torch.einsum("bnhkv,bnthk->bnthv", S, qb)
        outs.append(on.reshape(B, L, H, -1))
    return torch.cat(outs, 1)


def gated_rmsnorm(o, z, w, eps):
    """RMSNorm over the head dim, times w, times silu(z) (Qwen3.5 gated norm)."""
    of = o.float()
    y = of * torch.rsqrt(of.pow(2).mean(-1, keepdim=True) + eps) * w.float()
    return (y * F.silu(z.float())).to(o.dtype)
