"""GLM-OCR (GravityOCR's architecture) on CPU: the native decoder and image encoder vs transformers,
checkpoint names round trip, and the serving runtime (image prefill with 3-D RoPE, causal canvases)
vs the model's full-sequence statement."""
import pytest
import torch

from trida_stack_b200.data.images import mrope_position_ids
from trida_stack_b200.models.glm_ocr import GlmOcrDecoder, glm_ocr_config
from trida_stack_b200.serve import Runtime

IMG = 290


def tiny_hf(seed=0):
    from transformers.models.glm_ocr.configuration_glm_ocr import GlmOcrConfig
    from transformers.models.glm_ocr.modeling_glm_ocr import GlmOcrForConditionalGeneration
    torch.manual_seed(seed)
    cfg = GlmOcrConfig(
        text_config=dict(vocab_size=300, hidden_size=64, intermediate_size=96, num_hidden_layers=2,
                         num_attention_heads=4, num_key_value_heads=2, head_dim=16,
                         rope_parameters={"rope_type": "default", "rope_theta": 10000.0,
                                          "partial_rotary_factor": 0.5, "mrope_section": [1, 1, 2]}),
        vision_config=dict(depth=2, hidden_size=32, intermediate_size=48, num_heads=2, patch_size=4,
                           out_hidden_size=64, spatial_merge_size=2, temporal_patch_size=2),
        image_token_id=IMG)
    hf = GlmOcrForConditionalGeneration(cfg).float().eval()
    with torch.no_grad():
        for p in hf.parameters():
            p.add_(0.05 * torch.randn_like(p))
    return hf, cfg


def native(hf, cfg):
    dec = GlmOcrDecoder(glm_ocr_config(cfg.to_dict()), dtype=torch.float32)
    assert dec.load_hf_state_dict(hf.state_dict()) == []
    return dec


def _sample():
    grid = torch.tensor([[1, 4, 6]])
    px = torch.randn(24, 3 * 2 * 4 * 4)
    ids = torch.tensor([5, 6, 7] + [IMG] * 6 + [8, 9, 10, 11])
    return ids, grid, px


def test_native_glm_ocr_matches_transformers():
    hf, cfg = tiny_hf()
    dec = native(hf, cfg)
    assert set(dec.hf_state_dict()) == set(hf.state_dict())
    torch.manual_seed(1)
    ids, grid, px = _sample()
    with torch.no_grad():
        ref = hf(input_ids=ids[None], pixel_values=px, image_grid_thw=grid,
                 mm_token_type_ids=(ids == IMG).int()[None]).logits[0]
        feats = dec.visual(px, grid)
        torch.testing.assert_close(feats, hf.model.visual(px, grid_thw=grid).pooler_output, rtol=1e-5, atol=1e-5)
        ours = dec.forward_ref(ids, mrope_position_ids(ids, grid, IMG), feats)
    torch.testing.assert_close(ours, ref, rtol=1e-4, atol=1e-4)
    # q / k rotary rows are stored permuted; saving restores the checkpoint's order
    sd = dec.hf_state_dict()
    for k, v in hf.state_dict().items():
        torch.testing.assert_close(sd[k], v, msg=k)


def test_runtime_image_prefill_and_decode_match_statement():
    hf, cfg = tiny_hf()
    dec = native(hf, cfg)
    torch.manual_seed(2)
    ids, grid, px = _sample()
    feats = dec.visual(px, grid)
    rt = Runtime(dec, max_slots=2, max_len=128)
    s = rt.alloc()
    with torch.no_grad():
        last = rt.prefill([s], [ids.tolist()], vis=[(feats, mrope_position_ids(ids, grid, IMG))])
        more = torch.tensor([12, 13, 14, 15, 16])
        lg = rt.canvas([s], [more.tolist()], 5)
        rt.commit([s], [5])
        ids2 = torch.cat([ids, more])
        full = dec.forward_ref(ids2, mrope_position_ids(ids2, grid, IMG), feats)
    torch.testing.assert_close(last[0], full[len(ids) - 1], rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(lg[0], full[len(ids):], rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("pos_offset", [0, 1])
def test_ocr_self_spec_equals_causal_with_images(pos_offset):
    """An image request decoded by draft / verify rounds gives the causal decoder's greedy tokens
    (same RoPE layout on both sides, including GravityOCR's one-position offset)."""
    from trida_stack_b200.serve import Engine, Request, SamplingParams
    hf, cfg = tiny_hf()
    dec = native(hf, cfg)
    torch.manual_seed(4)
    ids, grid, px = _sample()
    outs = []
    for mode in ("causal", "draft-verify"):
        eng = Engine(Runtime(dec, max_slots=2, max_len=128), mask_id=299, mode=mode, block_size=6,
                     pos_offset=pos_offset)
        r = eng.submit(Request(ids.tolist(), 20, SamplingParams()))
        r.images = (px, grid)
        while not r.done:
            eng.step()
        outs.append(r.output)
    assert outs[0] == outs[1] and len(outs[0]) == 20
