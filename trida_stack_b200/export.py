"""Decision checkpoint -> kev's full-weight serving layout.

A checkpoint saved by the trainer holds the text decoder (plain ``model.*`` names, or
``model.language_model.*`` plus a nested ``text_config`` for a vision-language checkpoint) and the
pointer head (``decision_head.pt`` or the legacy ``jev_head.pt``).  kev's loader wants a plain
Qwen3.5 text model directory and a ``head.pt`` whose keys it reads by name (the contract of the
reference's ``train/tools/export_decision_checkpoint.py``: ``base``, ``head``, ``head_dim``,
``weights`` = ``"full"``, ``weights_dtype``, ``temperature``, ``lora``, ``option_isolation``,
``special_embeddings``, ``holdout``, ``exported_from``).

This exporter streams the text tensors one at a time from the source shards into the repository's
own shard writer (``checkpoint.ShardWriter``), so peak host memory is one shard, and checks the
head against the backbone's hidden size before anything is written.

    python -m trida_stack_b200.export --ckpt <save_dir>/step_N --out <dir> [--temperature T]
"""
import argparse
import json
import os
import shutil

import torch

from .checkpoint import SHARD_BYTES, ShardWriter

# files a serving tokenizer may consist of; copied when present
TOKENIZER_FILES = ("tokenizer.json", "tokenizer_config.json", "chat_template.jinja", "special_tokens_map.json",
                   "vocab.json", "merges.txt")
HEAD_FILES = ("decision_head.pt", "jev_head.pt")
_DTYPE_NAMES = {torch.bfloat16: ("bf16", "bfloat16"), torch.float32: ("fp32", "float32"),
                torch.float16: ("fp16", "float16")}


class ExportError(ValueError):
    pass


def text_backbone(ckpt):
    """(flat text config for a ``Qwen3_5ForCausalLM``, name prefix of the text weights)."""
    with open(os.path.join(ckpt, "config.json")) as f:
        cfg = json.load(f)
    if "text_config" in cfg and "vision_config" in cfg:
        text, prefix = dict(cfg["text_config"]), "model.language_model."
    else:
        text, prefix = dict(cfg), "model."
    for k in ("torch_dtype", "vision_config", "text_config", "image_token_id", "video_token_id",
              "vision_start_token_id", "vision_end_token_id"):
        text.pop(k, None)
    text["architectures"] = ["Qwen3_5ForCausalLM"]
    text["model_type"] = "qwen3_5_text"
    return text, prefix


def load_head(ckpt, hidden):
    """The pointer head's state and projection width, checked against the backbone's hidden size."""
    path = next((os.path.join(ckpt, n) for n in HEAD_FILES if os.path.exists(os.path.join(ckpt, n))), None)
    if path is None:
        raise ExportError(f"no pointer head in {ckpt}: expected one of {', '.join(HEAD_FILES)}")
    blob = torch.load(path, map_location="cpu")
    state, width = blob["head"], int(blob["head_dim"])
    for proj in ("q", "k"):
        w = state.get(f"{proj}.weight")
        if w is None or tuple(w.shape) != (width, hidden):
            got = None if w is None else tuple(w.shape)
            raise ExportError(f"{os.path.basename(path)}: {proj}.weight is {got}, expected ({width}, {hidden})")
    return {k: v.float() for k, v in state.items()}, width


def _source_files(ckpt):
    """Weight files of the checkpoint, in index order when an index exists."""
    index = os.path.join(ckpt, "model.safetensors.index.json")
    if os.path.exists(index):
        with open(index) as f:
            names = dict.fromkeys(json.load(f)["weight_map"].values())
        return [os.path.join(ckpt, n) for n in names]
    return sorted(os.path.join(ckpt, n) for n in os.listdir(ckpt) if n.endswith(".safetensors"))


def text_tensors(ckpt, prefix):
    """(``model.*`` name, tensor) of every text weight, read lazily shard by shard."""
    from safetensors import safe_open
    for path in _source_files(ckpt):
        with safe_open(path, "pt") as src:
            for name in src.keys():
                if name.startswith(prefix):
                    yield "model." + name[len(prefix):], src.get_tensor(name)


def export(ckpt, out, temperature=1.0, max_shard_bytes=SHARD_BYTES):
    text_cfg, prefix = text_backbone(ckpt)
    head, width = load_head(ckpt, int(text_cfg["hidden_size"]))
    os.makedirs(out, exist_ok=True)
    writer = ShardWriter(out, max_shard_bytes)
    dtype = None
    for name, t in text_tensors(ckpt, prefix):
        if dtype is None:
            dtype = t.dtype
        writer.add(name, t)
    if writer.count == 0:
        raise ExportError(f"{ckpt} holds no text weights (looked for names starting with {prefix!r})")
    writer.close()
    short, long_name = _DTYPE_NAMES.get(dtype, (str(dtype).replace("torch.", ""),) * 2)
    text_cfg["dtype"] = long_name
    with open(os.path.join(out, "config.json"), "w") as f:
        json.dump(text_cfg, f, indent=2)
    for n in TOKENIZER_FILES:
        if os.path.exists(os.path.join(ckpt, n)):
            shutil.copy2(os.path.join(ckpt, n), os.path.join(out, n))
    torch.save({"base": os.path.abspath(out), "head": head, "head_dim": width, "weights": "full",
                "weights_dtype": short, "temperature": float(temperature), "lora": 0, "option_isolation": False,
                "special_embeddings": False, "holdout": [], "exported_from": os.path.abspath(ckpt)},
               os.path.join(out, "head.pt"))
    return out


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--ckpt", required=True, help="checkpoint directory written by the trainer")
    ap.add_argument("--out", required=True, help="output directory (created)")
    ap.add_argument("--temperature", type=float, default=1.0, help="softmax temperature stored in head.pt")
    a = ap.parse_args()
    export(a.ckpt, a.out, a.temperature)
    print(f"exported {a.ckpt} -> {a.out}")


if __name__ == "__main__":
    main()
