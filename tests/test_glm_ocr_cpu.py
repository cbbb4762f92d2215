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


def test_glm_image_processor_matches_transformers():
    import numpy as np
    from PIL import Image

    from trida_stack_b200.data.images import ImageProcessor
    try:
        from transformers.models.glm4v.image_processing_pil_glm4v import Glm4vImageProcessorPil
    except ImportError:
        pytest.skip("transformers GLM-V PIL image processor not available")
    size = {"shortest_edge": 12544, "longest_edge": 28 * 28 * 2 * 600}
    hf = Glm4vImageProcessorPil(size=size, patch_size=14, temporal_patch_size=2, merge_size=2)
    ours = ImageProcessor(patch_size=14, temporal_patch_size=2, merge_size=2, min_pixels=size["shortest_edge"],
                          max_pixels=size["longest_edge"], image_mean=hf.image_mean, image_std=hf.image_std,
                          glm=True)
    rng = np.random.default_rng(0)
    imgs = [Image.fromarray(rng.integers(0, 255, (h, w, 3), dtype=np.uint8))
            for h, w in ((100, 70), (300, 900), (20, 64), (64, 128))]
    ref = hf(images=imgs, return_tensors="pt")
    pv, grid = ours(imgs)
    assert torch.equal(grid, ref["image_grid_thw"].long())
    torch.testing.assert_close(pv, ref["pixel_values"].float(), rtol=1e-5, atol=1e-5)


def _ckpt(tmp_path):
    """A tiny GravityOCR-layout checkpoint: config, weights, tokenizer, processor, block_diffusion.json."""
    import json as _json

    from helpers import make_tokenizer
    hf, cfg = tiny_hf()
    hf.save_pretrained(str(tmp_path))
    make_tokenizer(str(tmp_path), 300)
    _json.dump({"image_processor": {"image_processor_type": "Glm46VImageProcessor", "patch_size": 4,
                                    "temporal_patch_size": 2, "merge_size": 2,
                                    "size": {"shortest_edge": 64, "longest_edge": 2 * 24 * 24},
                                    "image_mean": [0.5, 0.5, 0.5], "image_std": [0.5, 0.5, 0.5]}},
               open(tmp_path / "processor_config.json", "w"))
    _json.dump({"bd_size": 5, "mask_id": 298, "ar_loss_weight": 1.0}, open(tmp_path / "block_diffusion.json", "w"))
    return str(tmp_path)


def test_ocr_server_self_spec_and_security(tmp_path, monkeypatch):
    import threading
    import time

    import requests
    import uvicorn

    import ocr_request
    import serve_gravityocr as S
    from trida_stack_b200.serve.ocr import build_ocr_app
    path = _ckpt(tmp_path)
    outs = {}
    for mode in ("causal", "self-spec"):
        args = S.parse_args([path, "--mode", mode, "--device", "cpu", "--dtype", "float32", "--max-running", "2",
                             "--context", "256", "--pos-offset", "0"])
        engine, tok, proc, eos = S.build(args)
        assert proc.glm and proc.patch_size == 4
        engine.start()
        import socket
        sk = socket.socket()
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
        sk.close()
        srv = uvicorn.Server(uvicorn.Config(build_ocr_app(engine, tok, proc, api_key="k3y", context=256, eos=()),
                                            host="127.0.0.1", port=port, log_level="error"))
        threading.Thread(target=srv.run, daemon=True).start()
        url = f"http://127.0.0.1:{port}"
        for _ in range(200):
            try:
                if requests.get(url + "/health", timeout=1).ok:
                    break
            except requests.ConnectionError:
                time.sleep(0.05)
        try:
            png, mime = ocr_request.synthetic_png("t1 t2")
            body = ocr_request.build_body(png, mime, "Text Recognition:", "glm-ocr", 12)
            assert requests.post(url + "/v1/chat/completions", json=body).status_code == 401
            r = ocr_request.send(body, url, 60, api_key="k3y")
            assert r["usage"]["completion_tokens"] == 12 and r["choices"][0]["finish_reason"] == "length"
            bad = dict(body)
            bad["messages"] = [{"role": "user", "content": [{"type": "image_url",
                                                             "image_url": {"url": "http://example.com/x.png"}}]}]
            rb = requests.post(url + "/v1/chat/completions", json=bad, headers={"Authorization": "Bearer k3y"})
            assert rb.status_code == 400
            outs[mode] = (r["choices"][0]["message"]["content"], r["usage"]["forwards"])
        finally:
            srv.should_exit = True
            engine.stop()
    # self-speculation reproduces causal decoding (greedy, same RoPE layout) in fewer forwards
    assert outs["self-spec"][0] == outs["causal"][0]
