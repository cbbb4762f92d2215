"""Chunked gated-delta kernels (tcgen05, ``csrc/gdn_chunk.cu``) vs the fp32 per-token recurrence
(``ops.gdn_reference``) on the same bf16 inputs."""
import pytest
import torch

from trida_stack_b200.ops import gdn_reference as R
from trida_stack_b200.ops.gdn import LinearLayout

pytestmark = pytest.mark.gpu

HK, HV, D = 2, 4, 128


def _inputs(B, T, seed=0):
    g = torch.Generator().manual_seed(seed)
    mixed = (torch.randn(B * T, 2 * HK * D + HV * D, generator=g) * 0.5).to(torch.bfloat16)
    ga = (torch.randn(B * T, HV, generator=g)).to(torch.bfloat16)
    gb = (torch.randn(B * T, HV, generator=g)).to(torch.bfloat16)
    A_log = torch.log(torch.empty(HV).uniform_(0.5, 8, generator=g))
    dt_bias = torch.randn(HV, generator=g) * 0.5
    return mixed, ga, gb, A_log, dt_bias


def _reference(mixed, ga, gb, A_log, dt_bias, B, T, lay):
    m = mixed.float().reshape(B, T, -1)
    q = R.l2norm(m[..., :HK * D].reshape(B, T, HK, D))
    k = R.l2norm(m[..., HK * D:2 * HK * D].reshape(B, T, HK, D))
    v = m[..., 2 * HK * D:].reshape(B, T, HV, D)
    rep = HV // HK
    q, k = q.repeat_interleave(rep, 2), k.repeat_interleave(rep, 2)
    g, beta = R.gates(ga.float().reshape(B, T, HV), gb.float().reshape(B, T, HV), A_log, dt_bias)
    if lay.mode == "two_stream":
        return R.gdn_two_stream(q, k, v, g, beta, lay.L, lay.V, lay.bd, lay.causal_clean, lay.causal_noisy,
                                lay.doc_start)
    o, _ = R.gdn_causal(q, k, v, g, beta, lay.doc_start)
    return o


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


def _run(B, T, lay, seed=0):
    from trida_stack_b200.ops.gdn_cuda import chunk_forward
    from trida_stack_b200.ops.blocks import check_device_errors
    mixed, ga, gb, A_log, dt_bias = _inputs(B, T, seed)
    ref = _reference(mixed, ga, gb, A_log, dt_bias, B, T, lay).reshape(B * T, HV * D)
    doc = None if lay.doc_start is None else lay.doc_start.to(torch.uint8).cuda().contiguous()
    o, _ = chunk_forward(mixed.cuda(), ga.cuda(), gb.cuda(), A_log.cuda(), dt_bias.cuda(), doc, B, T, HK, HV, lay,
                         D ** -0.5)
    torch.cuda.synchronize()
    check_device_errors()
    return o.cpu(), ref


@pytest.mark.parametrize("docs", [False, True])
def test_chunk_causal_forward(docs):
    B, T = 2, 200
    doc = None
    if docs:
        doc = torch.zeros(B, T, dtype=torch.bool)
        doc[:, 0] = True
        doc[0, 37] = doc[0, 64] = doc[1, 130] = True
    o, ref = _run(B, T, LinearLayout("causal", doc_start=doc))
    assert _rel(o, ref) < 2e-2, _rel(o, ref)


@pytest.mark.parametrize("bd,L,cc,cn,docs", [(32, 128, True, False, False), (32, 128, False, False, False),
                                             (16, 64, True, True, False), (64, 192, True, False, True),
                                             (16, 64, True, False, True)])
def test_chunk_two_stream_forward(bd, L, cc, cn, docs):
    B, V = 2, 2
    doc = None
    if docs:
        doc = torch.zeros(B, L, dtype=torch.bool)
        doc[:, 0] = True
        doc[0, L // 2] = True
        doc[1, bd] = True
    lay = LinearLayout("two_stream", L=L, V=V, bd=bd, causal_clean=cc, causal_noisy=cn, doc_start=doc)
    o, ref = _run(B, (1 + V) * L, lay)
    Lr = L
    for s in range(1 + V):
        part = o.reshape(B, (1 + V) * L, -1)[:, s * Lr:(s + 1) * Lr]
        rpart = ref.reshape(B, (1 + V) * L, -1)[:, s * Lr:(s + 1) * Lr]
        assert _rel(part, rpart) < 2e-2, (s, _rel(part, rpart))


def _ref_grads(mixed, ga, gb, A_log, dt_bias, B, T, lay, dO):
    m = mixed.float().clone().requires_grad_(True)
    a = ga.float().clone().requires_grad_(True)
    b = gb.float().clone().requires_grad_(True)
    o = _reference(m, a, b, A_log, dt_bias, B, T, lay).reshape(B * T, HV * D)
    o.backward(dO.float())
    return m.grad, a.grad, b.grad


@pytest.mark.parametrize("case", ["causal64", "causal200docs", "ts32", "ts16blk"])
def test_chunk_backward_op(case):
    """Op-level backward of the chunk kernels: q / k / v columns of d(conv output), d(decay
    pre-activation) and d(beta pre-activation) against CPU autograd through the recurrence."""
    from trida_stack_b200.ops._ext import ext
    from trida_stack_b200.ops.blocks import check_device_errors, device_error_word
    from trida_stack_b200.ops.gdn_cuda import chunk_forward
    B = 2
    if case == "causal64":
        T, lay = 64, LinearLayout("causal")
    elif case == "causal200docs":
        T = 200
        doc = torch.zeros(B, T, dtype=torch.bool)
        doc[:, 0] = True
        doc[0, 37] = doc[1, 130] = True
        lay = LinearLayout("causal", doc_start=doc)
    elif case == "ts32":
        T, lay = 3 * 128, LinearLayout("two_stream", L=128, V=2, bd=32, causal_clean=True, causal_noisy=False)
    else:
        T, lay = 3 * 64, LinearLayout("two_stream", L=64, V=2, bd=16, causal_clean=False, causal_noisy=False)
    mixed, ga, gb, A_log, dt_bias = _inputs(B, T, seed=7)
    g = torch.Generator().manual_seed(8)
    dO = (torch.randn(B * T, HV * D, generator=g) * 0.1).to(torch.bfloat16)
    dm_r, da_r, db_r = _ref_grads(mixed, ga, gb, A_log, dt_bias, B, T, lay, dO)
    dev = "cuda"
    doc = None if lay.doc_start is None else lay.doc_start.to(torch.uint8).cuda().contiguous()
    mg, gag, gbg = mixed.to(dev), ga.to(dev), gb.to(dev)
    Al, dtb = A_log.to(dev).float(), dt_bias.to(dev).float()
    o, saved = chunk_forward(mg, gag, gbg, Al, dtb, doc, B, T, HK, HV, lay, D ** -0.5)
    dmixed = torch.zeros_like(mg)
    dga = torch.zeros(B * T, HV, dtype=torch.bfloat16, device=dev)
    dgb = torch.zeros_like(dga)
    dA = torch.zeros(HV, device=dev)
    ddt = torch.zeros(HV, device=dev)
    ext().gdn_chunk_bwd(mg, gag, gbg, Al, dtb, doc, o, saved["bufs"], device_error_word(mg.device), saved["geo"],
                        D ** -0.5, dO.to(dev), dmixed, dga, dgb, dA, ddt)
    torch.cuda.synchronize()
    check_device_errors()
    parts = {"dq": slice(0, HK * D), "dk": slice(HK * D, 2 * HK * D), "dv": slice(2 * HK * D, None)}
    errs = {k: _rel(dmixed[:, s].cpu(), dm_r[:, s]) for k, s in parts.items()}
    errs["dbeta_pre"] = _rel(dgb.cpu(), db_r)
    errs["ddecay_pre"] = _rel(dga.cpu(), da_r)
    if errs["ddecay_pre"] >= 3e-2:
        a, r_ = dga.float().cpu(), da_r
        print("ddecay rows (gpu / ref), head 0:", [(round(a[i, 0].item(), 4), round(r_[i, 0].item(), 4))
                                                  for i in range(0, min(B * T, 24))])
        print("ratio mean/std:", (a / r_).mean().item(), (a / r_).std().item())
    assert all(v < 3e-2 for v in errs.values()), sorted(errs.items())
