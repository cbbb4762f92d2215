"""CPU parity with the reference trainer's objective (config 1 of the benchmark spec: tiny
Qwen3, fp32).  The reference forward runs eagerly on CPU (flex-attention has no CPU backward, so
gradients are checked against our own autograd oracle elsewhere)."""
import pytest
import torch

from helpers import import_reference, make_tiny_qwen3, patch_flex_for_cpu, reference_available
from trida_stack_b200.models import BlockDiffusionLM, Decoder, ModelConfig

pytestmark = pytest.mark.skipif(not reference_available(), reason="reference not installed in baseline/_ref")


def _batch(B=2, P=64, Rr=64, seed=1):
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, 1022, (B, P + Rr), generator=g)
    labels = ids.clone()
    labels[:, :P] = -100
    return ids, labels, torch.ones_like(ids)


@pytest.mark.parametrize("ar_w", [0.0, 1.0])
@pytest.mark.parametrize("wbc", [False, True])
def test_dense_bd_loss_matches_reference(tmp_path, ar_w, wbc):
    patch_flex_for_cpu()
    bd = import_reference()
    make_tiny_qwen3(str(tmp_path))
    ref = bd.HFBlockDiffusion(model_id=str(tmp_path), bd_size=16, ar_loss_weight=ar_w, dtype=torch.float32,
                              response_buckets=None, within_block_causal=wbc)
    ref.eval()
    cfg = ModelConfig.from_pretrained(str(tmp_path))
    cfg.vocab_size = ref.model.get_input_embeddings().weight.shape[0]
    dec = Decoder(cfg, dtype=torch.float32)
    dec.load_hf_state_dict(ref.model.state_dict())
    ours = BlockDiffusionLM(dec, mask_id=ref.mask_id, bd_size=16, ar_loss_weight=ar_w, response_buckets=None,
                            within_block_causal=wbc)
    ids, labels, am = _batch()
    torch.manual_seed(123)
    with torch.no_grad():
        l_ref, logs_ref = ref(ids, labels, am)
    torch.manual_seed(123)
    with torch.no_grad():
        l_ours, logs_ours = ours(ids, labels, am)
    assert logs_ours["ntok"] == logs_ref["ntok"]
    torch.testing.assert_close(l_ours, l_ref, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(logs_ours["diff_loss"], logs_ref["diff_loss"], rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(logs_ours["ar_loss"], logs_ref["ar_loss"], rtol=1e-5, atol=1e-5)


def _packed_batch(seed=3):
    """Two rows; row 0 has 2 documents, row 1 has 3, with right padding (seg_id -1)."""
    g = torch.Generator().manual_seed(seed)
    L = 160
    ids = torch.randint(0, 1022, (2, L), generator=g)
    labels = torch.full((2, L), -100)
    seg = torch.full((2, L), -1)
    rpos = torch.full((2, L), -1)
    am = torch.zeros(2, L, dtype=torch.long)
    docs = {0: [(0, 30, 70), (70, 100, 150)], 1: [(0, 10, 40), (40, 60, 90), (90, 100, 130)]}
    for b, spans in docs.items():
        for k, (s, r, e) in enumerate(spans):
            seg[b, s:e] = k
            am[b, s:e] = 1
            labels[b, r:e] = ids[b, r:e]
            rpos[b, r:e] = torch.arange(e - r)
    return ids, labels, am, seg, rpos


def _ours_and_ref(tmp_path, ar_w, **kw):
    patch_flex_for_cpu()
    bd = import_reference()
    make_tiny_qwen3(str(tmp_path))
    ref = bd.HFBlockDiffusion(model_id=str(tmp_path), bd_size=16, ar_loss_weight=ar_w, dtype=torch.float32,
                              response_buckets=None, **kw)
    ref.eval()
    cfg = ModelConfig.from_pretrained(str(tmp_path))
    cfg.vocab_size = ref.model.get_input_embeddings().weight.shape[0]
    dec = Decoder(cfg, dtype=torch.float32)
    dec.load_hf_state_dict(ref.model.state_dict())
    ours = BlockDiffusionLM(dec, mask_id=ref.mask_id, bd_size=16, ar_loss_weight=ar_w, response_buckets=None, **kw)
    return ref, ours


def _check(out_ours, out_ref):
    (l_o, g_o), (l_r, g_r) = out_ours, out_ref
    assert g_o["ntok"] == g_r["ntok"]
    torch.testing.assert_close(l_o, l_r, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(g_o["diff_loss"], g_r["diff_loss"], rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(g_o["ar_loss"], g_r["ar_loss"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("merged", [False, True])
def test_packed_layout_matches_reference(tmp_path, merged):
    ref, ours = _ours_and_ref(tmp_path, 1.0, merged_views=merged)
    ids, labels, am, seg, rpos = _packed_batch()
    torch.manual_seed(7)
    with torch.no_grad():
        r = ref(ids, labels, am, seg_id=seg, resp_pos=rpos)
    torch.manual_seed(7)
    with torch.no_grad():
        o = ours(ids, labels, am, seg_id=seg, resp_pos=rpos)
    _check(o, r)


def test_multiturn_layout_matches_reference(tmp_path):
    ref, ours = _ours_and_ref(tmp_path, 0.5)
    g = torch.Generator().manual_seed(5)
    L = 150
    ids = torch.randint(0, 1022, (2, L), generator=g)
    labels = torch.full((2, L), -100)
    rb = torch.full((2, L), -1)
    tid = torch.full((2, L), -1)
    am = torch.ones(2, L, dtype=torch.long)
    am[1, 130:] = 0
    for b in range(2):
        blk = 0
        for t, (s, e) in enumerate([(20, 55), (70, 100), (110, 128)]):
            labels[b, s:e] = ids[b, s:e]
            tid[b, s:e] = t
            w = torch.arange(e - s) // 16
            rb[b, s:e] = blk + w
            blk += int(w.max()) + 1
    torch.manual_seed(9)
    with torch.no_grad():
        r = ref(ids, labels, am, resp_block=rb, turn_id=tid)
    torch.manual_seed(9)
    with torch.no_grad():
        o = ours(ids, labels, am, resp_block=rb, turn_id=tid)
    _check(o, r)


def test_ar_only_matches_reference(tmp_path):
    patch_flex_for_cpu()
    bd = import_reference()
    make_tiny_qwen3(str(tmp_path))
    ref = bd.HFBlockDiffusion(model_id=str(tmp_path), ar_only=True, dtype=torch.float32, attn_impl="eager")
    ref.eval()
    cfg = ModelConfig.from_pretrained(str(tmp_path))
    cfg.vocab_size = ref.model.get_input_embeddings().weight.shape[0]
    dec = Decoder(cfg, dtype=torch.float32)
    dec.load_hf_state_dict(ref.model.state_dict())
    ours = BlockDiffusionLM(dec, mask_id=0, ar_only=True)
    ids, labels, am, seg, rpos = _packed_batch()
    with torch.no_grad():
        r = ref(ids, labels, am, seg_id=seg)
        o = ours(ids, labels, am, seg_id=seg)
    assert o[1]["ntok"] == r[1]["ntok"]
    torch.testing.assert_close(o[0], r[0], rtol=1e-5, atol=1e-5)
