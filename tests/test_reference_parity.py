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
