"""Attach a Qwen3.5 vision tower to a text-only block-diffusion checkpoint (the reference's
``train/tools/compose_vl_checkpoint.py``).

A checkpoint trained from a text-only backbone holds ``model.*`` (+ ``lm_head.weight`` when untied).
The result is a ``Qwen3_5ForConditionalGeneration`` directory that the trainer loads for image+text
SFT: the text weights under ``model.language_model.*``, the untied LM head kept, the base VL
model's ``model.visual.*`` (encoder and merger) copied unchanged, its ``mtp.*`` dropped; the config
is the base VL config with ``text_config`` taken from the text checkpoint (so the grown vocabulary
with ``<|mask|>`` carries over) and the merger's output width set to the text hidden size.
Tokenizer files and ``block_diffusion.json`` come from the text checkpoint, the image processor
configs from the base VL model.

    python -m trida_stack_b200.compose_vl --text <ckpt> --vision <Qwen3.5 VL dir> --out <ckpt>-vl
"""
import argparse
import json
import os
import shutil

import torch

from .checkpoint import read_hf_weights, write_hf_weights

_TEXT_ONLY_KEYS = ("architectures", "transformers_version", "bos_token_id", "pad_token_id")
_FROM_TEXT = ("tokenizer.json", "tokenizer_config.json", "chat_template.jinja", "block_diffusion.json",
              "generation_config.json", "special_tokens_map.json", "vocab.json", "merges.txt")
_FROM_VISION = ("preprocessor_config.json", "video_preprocessor_config.json")


def compose(text_dir, vision_dir, out_dir):
    with open(os.path.join(text_dir, "config.json")) as f:
        text_cfg = json.load(f)
    with open(os.path.join(vision_dir, "config.json")) as f:
        vl_cfg = json.load(f)
    if "vision_config" in text_cfg:
        raise SystemExit(f"{text_dir} already has a vision_config")
    if "vision_config" not in vl_cfg:
        raise SystemExit(f"{vision_dir} has no vision_config")
    text = read_hf_weights(text_dir)
    lm_head = text.pop("lm_head.weight", None)
    out = {}
    for k, v in text.items():
        if not k.startswith("model."):
            raise SystemExit(f"unexpected text weight {k}")
        out["model.language_model." + k[len("model."):]] = v
    embed = out["model.language_model.embed_tokens.weight"]
    tied = lm_head is None or torch.equal(lm_head, embed)
    if not tied:
        out["lm_head.weight"] = lm_head
    visual = {k: v for k, v in read_hf_weights(vision_dir).items() if k.startswith("model.visual.")}
    for part in ("patch_embed", "blocks", "merger"):
        if not any(k.startswith(f"model.visual.{part}.") for k in visual):
            raise SystemExit(f"no model.visual.{part}.* weights in {vision_dir}")
    out.update(visual)
    tc = {k: v for k, v in text_cfg.items() if k not in _TEXT_ONLY_KEYS}
    tc["tie_word_embeddings"] = tied
    vl_cfg["text_config"] = tc
    vl_cfg["tie_word_embeddings"] = tied
    vl_cfg["architectures"] = ["Qwen3_5ForConditionalGeneration"]
    vl_cfg["vision_config"]["out_hidden_size"] = tc["hidden_size"]
    for k in ("bos_token_id", "pad_token_id"):
        if k in text_cfg:
            vl_cfg[k] = text_cfg[k]
    os.makedirs(out_dir, exist_ok=True)
    write_hf_weights(out, out_dir)
    with open(os.path.join(out_dir, "config.json"), "w") as f:
        json.dump(vl_cfg, f, indent=2)
    for src, names in ((text_dir, _FROM_TEXT), (vision_dir, _FROM_VISION)):
        for n in names:
            if os.path.exists(os.path.join(src, n)):
                shutil.copy(os.path.join(src, n), os.path.join(out_dir, n))
    return out_dir


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--text", required=True, help="text-only block-diffusion checkpoint")
    ap.add_argument("--vision", required=True, help="base Qwen3.5 vision-language model directory")
    ap.add_argument("--out", required=True)
    a = ap.parse_args()
    print(compose(a.text, a.vision, a.out))


if __name__ == "__main__":
    main()
