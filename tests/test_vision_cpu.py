"""Vision-language (Qwen3.5 VL) support on CPU: vision tower and 3-D RoPE vs transformers, image
preprocessing vs transformers' processor, image-pad expansion / positions / packing, and the
two-stream objective with images (features reach every stream, only the merger trains)."""
import math
import random

import numpy as np
import pytest
import torch

from trida_stack_b200.data import images as I
from trida_stack_b200.data import sft
from trida_stack_b200.models import Decoder, ModelConfig
from trida_stack_b200.models.hybrid import HybridBlockDiffusionLM
from trida_stack_b200.models.vision import VisionConfig, VisionTower, mrope_angles

IMG = 290
VCFG = dict(depth=2, hidden_size=32, intermediate_size=48, num_heads=2, in_channels=3, patch_size=4,
            temporal_patch_size=2, spatial_merge_size=2, out_hidden_size=64, num_position_embeddings=16,
            hidden_act="gelu_pytorch_tanh")


def random_layout(rng, n_images, img=IMG):
    ids, grids = [], []
    for _ in range(n_images):
        ids += [rng.randint(0, 200) for _ in range(rng.randint(1, 12))]
        gh, gw = 2 * rng.randint(1, 5), 2 * rng.randint(1, 5)
        grids.append([1, gh, gw])
        ids += [img] * (gh * gw // 4)
    ids += [rng.randint(0, 200) for _ in range(rng.randint(1, 12))]
    return torch.tensor(ids), torch.tensor(grids, dtype=torch.long).reshape(-1, 3)


def test_mrope_positions_match_transformers_rope_index():
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5Config
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5Model
    cfg = Qwen3_5Config(text_config=dict(hidden_size=64, intermediate_size=64, num_hidden_layers=2,
                                         num_attention_heads=2, num_key_value_heads=1, head_dim=32, vocab_size=300,
                                         layer_types=["linear_attention", "full_attention"]),
                        vision_config=dict(depth=1, hidden_size=32, intermediate_size=32, num_heads=2,
                                           out_hidden_size=64),
                        image_token_id=IMG)
    model = Qwen3_5Model(cfg)
    rng = random.Random(0)
    for n_images in (0, 1, 2, 3):
        for _ in range(4):
            ids, grids = random_layout(rng, n_images)
            ref, _ = model.get_rope_index(ids[None], (ids == IMG).int()[None],
                                          image_grid_thw=grids if n_images else None)
            assert torch.equal(I.mrope_position_ids(ids, grids if n_images else None, IMG), ref[:, 0])


def test_text_mrope_angles_match_transformers_rotary():
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5TextConfig
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5TextRotaryEmbedding
    cfg = Qwen3_5TextConfig(hidden_size=64, num_attention_heads=2, head_dim=256, vocab_size=300,
                            rope_parameters={"rope_type": "default", "rope_theta": 1e7, "partial_rotary_factor": 0.25,
                                             "mrope_section": [11, 11, 10], "mrope_interleaved": True})
    rot = Qwen3_5TextRotaryEmbedding(cfg)
    rng = random.Random(1)
    ids, grids = random_layout(rng, 2)
    pos3 = I.mrope_position_ids(ids, grids, IMG)[:, None]                 # [3, 1, T]
    cos, sin = rot(torch.zeros(1, dtype=torch.float32), pos3)
    ang = mrope_angles(pos3.permute(1, 0, 2), 64, 1e7, (11, 11, 10))      # [1, T, 32]
    torch.testing.assert_close(torch.cat([ang, ang], -1).cos(), cos, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(torch.cat([ang, ang], -1).sin(), sin, rtol=1e-5, atol=1e-5)
    # all three axes equal -> plain 1-D RoPE angles
    p = torch.arange(50)
    a1 = mrope_angles(p.expand(1, 3, -1), 64, 1e7, (11, 11, 10))
    inv = 1.0 / (1e7 ** (torch.arange(0, 64, 2).float() / 64))
    torch.testing.assert_close(a1[0], p.float()[:, None] * inv)


def test_vision_tower_matches_transformers():
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5VisionConfig
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5VisionModel
    torch.manual_seed(0)
    hf = Qwen3_5VisionModel(Qwen3_5VisionConfig(**VCFG)).float().eval()
    with torch.no_grad():
        for p in hf.parameters():
            p.add_(0.05 * torch.randn_like(p))
    ours = VisionTower(VisionConfig.from_dict(VCFG), dtype=torch.float32)
    ours.load_state_dict(hf.state_dict())
    grid = torch.tensor([[1, 4, 6], [1, 2, 2], [1, 6, 4]])
    P = int(grid.prod(-1).sum())
    px = torch.randn(P, 3 * 2 * 4 * 4)
    with torch.no_grad():
        ref = hf(px, grid_thw=grid).pooler_output
        out = ours(px, grid)
    assert out.shape == (P // 4, 64)
    torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-4)


def test_image_processor_matches_transformers():
    from PIL import Image
    try:
        from transformers.models.qwen2_vl.image_processing_pil_qwen2_vl import Qwen2VLImageProcessorPil
    except ImportError:
        pytest.skip("transformers PIL image processor not available")
    kw = dict(patch_size=16, temporal_patch_size=2, merge_size=2, image_mean=[0.5, 0.5, 0.5],
              image_std=[0.5, 0.5, 0.5])
    hf = Qwen2VLImageProcessorPil(size={"shortest_edge": 64 * 64, "longest_edge": 256 * 256}, **kw)
    ours = I.ImageProcessor(min_pixels=64 * 64, max_pixels=256 * 256, **kw)
    rng = np.random.default_rng(0)
    imgs = [Image.fromarray(rng.integers(0, 255, (h, w, 3), dtype=np.uint8)) for h, w in
            ((100, 70), (300, 520), (32, 32), (64, 128))]
    ref = hf(images=imgs, return_tensors="pt")
    pv, grid = ours(imgs)
    assert torch.equal(grid, ref["image_grid_thw"].long())
    torch.testing.assert_close(pv, ref["pixel_values"].float(), rtol=1e-5, atol=1e-5)


def test_fit_size_bounds():
    for h, w in ((10, 10), (1000, 3000), (33, 47), (5000, 40)):
        a, b = I.fit_size(h, w, 32, 64 * 64, 512 * 512)
        assert a % 32 == 0 and b % 32 == 0 and 64 * 64 <= a * b <= 512 * 512


def test_image_refs_and_pad_expansion():
    msgs = [{"role": "user", "content": [{"type": "image", "image": "a.png"}, {"type": "text", "text": "x"},
                                         {"image_url": {"url": "data:b"}}]},
            {"role": "assistant", "content": "ok"},
            {"role": "user", "content": [{"type": "image", "image": "c.png"}]}]
    assert I.image_refs(msgs) == ["a.png", "data:b", "c.png"]
    with pytest.raises(ValueError):
        I.image_refs([{"role": "user", "content": [{"type": "video", "video": "v.mp4"}]}])
    assert I.expand_image_pads([1, IMG, 2, IMG, 3], IMG, [3, 2]) == [1, IMG, IMG, IMG, 2, IMG, IMG, 3]
    assert I.expand_image_pads([1, IMG, 2], IMG, [3, 2]) == [1, IMG, IMG, IMG, 2]


def _image_doc(rng, n_images, bd):
    ids, grids = random_layout(rng, n_images)
    labels = torch.full_like(ids, -100)
    labels[-3:] = ids[-3:]
    s = {"input_ids": ids, "labels": labels, "resp_block": torch.where(labels != -100, 0, -1),
         "turn_id": torch.where(labels != -100, 0, -1)}
    if n_images:
        P = int(grids.prod(-1).sum()) * 1
        s.update(pixel_values=torch.randn(P, 3 * 2 * 4 * 4), image_grid_thw=grids,
                 mrope_pos=I.mrope_position_ids(ids, grids, IMG))
    return sft.block_align_doc(s, bd, 0)


def test_packing_keeps_image_order_and_positions():
    rng = random.Random(3)
    bd = 8
    rows = [[_image_doc(rng, 1, bd), _image_doc(rng, 0, bd)], [_image_doc(rng, 2, bd)]]
    b = sft.pack_rows_multiturn(rows, 0, bd, None, 4096)
    B, L = b["input_ids"].shape
    assert b["mrope_pos"].shape == (B, 3, L)
    assert b["image_grid_thw"].shape[0] == 3
    n_tok = int((b["input_ids"] == IMG).sum())
    assert n_tok == int((b["image_grid_thw"].prod(-1) // 4).sum())
    # the text doc packed second in row 0 restarts at 0 on all three axes
    n0 = rows[0][0]["input_ids"].shape[0]
    n1 = rows[0][1]["input_ids"].shape[0]
    assert torch.equal(b["mrope_pos"][0, :, n0:n0 + n1], torch.arange(n1).expand(3, -1))
    # block-aligned pad continues the doc's positions
    d = rows[1][0]
    assert int(d["mrope_pos"][0, -1]) == int(d["mrope_pos"].max())


def tiny_vl(seed=0):
    cfg = ModelConfig.from_hf_dict({
        "model_type": "qwen3_5", "image_token_id": IMG, "tie_word_embeddings": True,
        "text_config": {"model_type": "qwen3_5_text", "vocab_size": 300, "hidden_size": 64, "intermediate_size": 128,
                        "num_hidden_layers": 4, "num_attention_heads": 2, "num_key_value_heads": 1,
                        "head_dim": 32, "linear_num_key_heads": 2, "linear_num_value_heads": 4,
                        "linear_key_head_dim": 16, "linear_value_head_dim": 16, "linear_conv_kernel_dim": 4,
                        "layer_types": ["linear_attention"] * 3 + ["full_attention"],
                        "rope_parameters": {"rope_theta": 1e4, "partial_rotary_factor": 0.5,
                                            "mrope_section": [3, 3, 2]}},
        "vision_config": VCFG})
    torch.manual_seed(seed)
    return Decoder(cfg, dtype=torch.float32)


def test_vl_checkpoint_names_round_trip():
    dec = tiny_vl()
    sd = dec.hf_state_dict()
    assert "model.visual.blocks.0.attn.qkv.weight" in sd and "model.visual.patch_embed.proj.weight" in sd
    assert "model.language_model.embed_tokens.weight" in sd and "model.embed_tokens.weight" not in sd
    dec2 = tiny_vl(seed=1)
    dec2.load_hf_state_dict(sd)
    for (n, a), (_, b) in zip(dec.named_parameters(), dec2.named_parameters()):
        assert torch.equal(a, b), n
    # the encoder is frozen, the merger trains
    assert not dec.visual.blocks[0].attn.qkv.weight.requires_grad
    assert dec.visual.merger.linear_fc1.weight.requires_grad


def test_two_stream_objective_with_images():
    rng = random.Random(5)
    bd = 8
    rows = [[_image_doc(rng, 1, bd)], [_image_doc(rng, 2, bd), _image_doc(rng, 0, bd)]]
    batch = sft.pack_rows_multiturn(rows, 0, bd, None, 4096)
    dec = tiny_vl()
    m = HybridBlockDiffusionLM(dec, mask_id=299, bd_size=bd, ar_loss_weight=1.0)
    m.train()
    groups = m.param_groups(projector_lr_scale=0.1)
    assert [g["lr_scale"] for g in groups] == [1.0, 0.1]
    assert all(".visual." not in n or ".merger." in n for n, p in m.named_parameters() if p.requires_grad)
    torch.manual_seed(0)
    loss, _ = m(**batch)
    loss.backward()
    assert math.isfinite(loss.item())
    assert dec.visual.merger.linear_fc2.weight.grad is not None
    assert dec.visual.blocks[0].attn.qkv.weight.grad is None
    # the features are read: other pixels give another loss (same noise)
    torch.manual_seed(0)
    b2 = dict(batch, pixel_values=batch["pixel_values"] + 1.0)
    with torch.no_grad():
        l2, _ = m(**b2)
    assert abs(l2.item() - loss.item()) > 1e-6


def test_text_only_rows_mrope_equals_1d_rope():
    dec = tiny_vl()
    m = HybridBlockDiffusionLM(dec, mask_id=299, bd_size=8, ar_loss_weight=1.0)
    ids = torch.randint(0, 280, (2, 32))
    labels = ids.clone()
    labels[:, :12] = -100
    with torch.no_grad():
        torch.manual_seed(1)
        a, _ = m(ids, labels, torch.ones_like(ids))
        torch.manual_seed(1)
        b, _ = m(ids, labels, torch.ones_like(ids), mrope_pos=torch.arange(32).expand(2, 3, -1))
    torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-6)


def test_compose_vl_checkpoint(tmp_path):
    import json

    from trida_stack_b200.checkpoint import read_hf_weights, write_hf_weights
    from trida_stack_b200.compose_vl import compose
    vl = tiny_vl(seed=2)
    vdir, tdir, odir = tmp_path / "vl", tmp_path / "text", tmp_path / "out"
    write_hf_weights(vl.hf_state_dict(), str(vdir))
    json.dump(vl.cfg.to_hf_dict(), open(vdir / "config.json", "w"))
    # a text-only checkpoint of the same backbone with a grown vocabulary
    tcfg = dict(vl.cfg.to_hf_dict()["text_config"], vocab_size=301, tie_word_embeddings=True)
    text = Decoder(ModelConfig.from_hf_dict(tcfg), dtype=torch.float32)
    write_hf_weights(text.hf_state_dict(), str(tdir))
    json.dump(tcfg, open(tdir / "config.json", "w"))
    compose(str(tdir), str(vdir), str(odir))
    cfg = ModelConfig.from_pretrained(str(odir))
    assert cfg.is_vl and cfg.vocab_size == 301
    dec = Decoder(cfg, dtype=torch.float32)
    dec.load_hf_state_dict(read_hf_weights(str(odir)))
    assert torch.equal(dec.embed, text.embed)
    assert torch.equal(dec.visual.merger.linear_fc1.weight, vl.visual.merger.linear_fc1.weight)
