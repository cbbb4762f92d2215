"""The chunked (WY) statement of the gated-delta rule that the sm_100a chunk kernels compute
(``ops.gdn_chunked``) against the per-token recurrence (``ops.gdn_reference``), in fp64 on CPU:
forward outputs, and the explicit chunk backward against autograd."""
import pytest
import torch

from trida_stack_b200.ops import gdn_chunked as K
from trida_stack_b200.ops import gdn_reference as R


def _inputs(B, T, H, d=16, seed=0):
    g = torch.Generator().manual_seed(seed)
    q = R.l2norm(torch.randn(B, T, H, d, generator=g, dtype=torch.float64))
    k = R.l2norm(torch.randn(B, T, H, d, generator=g, dtype=torch.float64))
    v = torch.randn(B, T, H, d, generator=g, dtype=torch.float64)
    gl = -torch.rand(B, T, H, generator=g, dtype=torch.float64) * 0.7
    beta = torch.rand(B, T, H, generator=g, dtype=torch.float64)
    return q, k, v, gl, beta


@pytest.mark.parametrize("docs", [False, True])
def test_causal_chunked_matches_recurrence(docs):
    B, T, H, d = 2, 45, 2, 16
    q, k, v, gl, beta = _inputs(B, T, H, d)
    doc = None
    if docs:
        doc = torch.zeros(B, T, dtype=torch.bool)
        doc[:, 0] = True
        doc[0, 7] = doc[0, 16] = doc[1, 30] = True
    ref, _ = R.gdn_causal(q, k, v, gl, beta, doc)
    out = K.causal_fwd(q * d ** -0.5, k, v, gl, beta, doc, C=16)
    torch.testing.assert_close(out.float(), ref, rtol=1e-4, atol=2e-5)   # the recurrence runs in fp32


@pytest.mark.parametrize("cc,cn,docs", [(True, False, False), (False, False, False), (True, True, False),
                                         (True, False, True), (False, True, True)])
def test_two_stream_chunked_matches_recurrence(cc, cn, docs):
    B, L, V, bd, H, d = 2, 32, 2, 8, 2, 16
    q, k, v, gl, beta = _inputs(B, (1 + V) * L, H, d, seed=1)
    doc = None
    if docs:
        doc = torch.zeros(B, L, dtype=torch.bool)
        doc[:, 0] = True
        doc[0, 16] = doc[1, 8] = True
    ref = R.gdn_two_stream(q, k, v, gl, beta, L, V, bd, cc, cn, doc)
    out = K.two_stream_fwd(q * d ** -0.5, k, v, gl, beta, L, V, bd, cc, cn, doc)
    torch.testing.assert_close(out.float(), ref, rtol=1e-4, atol=2e-5)   # the recurrence runs in fp32


@pytest.mark.parametrize("readout_block,resets", [(False, False), (False, True), (True, False), (True, True)])
def test_chunk_backward_matches_autograd(readout_block, resets):
    torch.manual_seed(0)
    N, C, d = 3, 12, 8
    q = R.l2norm(torch.randn(N, C, d, dtype=torch.float64)).requires_grad_()
    k = R.l2norm(torch.randn(N, C, d, dtype=torch.float64)).requires_grad_()
    v = torch.randn(N, C, d, dtype=torch.float64, requires_grad=True)
    gl = (-torch.rand(N, C, dtype=torch.float64) * 0.5).requires_grad_()
    beta = torch.rand(N, C, dtype=torch.float64, requires_grad=True)
    S0 = torch.randn(N, d, d, dtype=torch.float64, requires_grad=True)
    rs = torch.zeros(N, C, dtype=torch.bool)
    if resets:
        rs[0, 0] = True
        rs[1, 5] = True
        rs[2, 3] = rs[2, 9] = True
    O, U, S1, cache = K.chunk_fwd(q, k, v, gl, beta, rs, S0, readout_block)
    dO = torch.randn_like(O)
    dS1 = torch.randn_like(S1)
    torch.autograd.backward([O, S1], [dO, dS1])
    with torch.no_grad():
        _, _, _, c2 = K.chunk_fwd(q, k, v, gl, beta, rs, S0, readout_block)
        grads = K.chunk_bwd(q, k, v, gl, beta, rs, S0, dO, dS1, c2)
    for name, got, x in zip(["q", "k", "v", "g", "beta", "S0"], grads, [q, k, v, gl, beta, S0]):
        torch.testing.assert_close(got, x.grad, rtol=1e-8, atol=1e-9, msg=name)
