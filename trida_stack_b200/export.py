"""Export a decision-trained checkpoint to kev's full-weight layout (the reference's
``scripts/export_decision_checkpoint.py``): text backbone weights under ``model.*`` with a flat
Qwen3.5 text config, the tokenizer, and ``head.pt`` with kev's metadata (``weights="full"``, the
pointer head, ``head_dim``, ``weights_dtype``, ``temperature``).

    python -m trida_stack_b200.export --ckpt <save_dir>/step_N --out <dir> [--temperature T]
"""
import argparse
import glob
import json
import os
import shutil

import torch

TOKENIZER_FILES = ("tokenizer.json", "tokenizer_config.json", "chat_template.jinja", "special_tokens_map.json",
                   "vocab.json", "merges.txt")


def head_file(ckpt):
    for name in ("decision_head.pt", "jev_head.pt"):
        p = os.path.join(ckpt, name)
        if os.path.exists(p):
            return p
    raise FileNotFoundError(f"{ckpt} has no decision head (decision_head.pt or jev_head.pt)")


def export(ckpt, out, temperature=1.0):
    from safetensors import safe_open
    from safetensors.torch import save_file
    with open(os.path.join(ckpt, "config.json")) as f:
        cfg = json.load(f)
    head = torch.load(head_file(ckpt), map_location="cpu")
    nested = "text_config" in cfg and "vision_config" in cfg
    prefix = "model.language_model." if nested else "model."
    tensors = {}
    for f in sorted(glob.glob(os.path.join(ckpt, "*.safetensors"))):
        with safe_open(f, "pt") as s:
            for k in s.keys():
                if k.startswith(prefix):
                    tensors["model." + k[len(prefix):]] = s.get_tensor(k)
    if not tensors:
        raise SystemExit(f"no text weights under {prefix!r} in {ckpt}")
    dtype = next(iter(tensors.values())).dtype
    wd, dname = {torch.bfloat16: ("bf16", "bfloat16"), torch.float32: ("fp32", "float32")}[dtype]
    text_cfg = dict(cfg["text_config"]) if nested else dict(cfg)
    text_cfg.update(architectures=["Qwen3_5ForCausalLM"], model_type="qwen3_5_text", dtype=dname)
    text_cfg.pop("torch_dtype", None)
    os.makedirs(out, exist_ok=True)
    save_file(tensors, os.path.join(out, "model.safetensors"), metadata={"format": "pt"})
    with open(os.path.join(out, "config.json"), "w") as f:
        json.dump(text_cfg, f, indent=2)
    for name in TOKENIZER_FILES:
        if os.path.exists(os.path.join(ckpt, name)):
            shutil.copy2(os.path.join(ckpt, name), out)
    meta = {"base": os.path.abspath(out), "head": {k: v.float() for k, v in head["head"].items()},
            "head_dim": head["head_dim"], "weights": "full", "weights_dtype": wd, "temperature": float(temperature),
            "lora": 0, "option_isolation": False, "special_embeddings": False, "holdout": [],
            "exported_from": os.path.abspath(ckpt)}
    torch.save(meta, os.path.join(out, "head.pt"))
    return out


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--ckpt", required=True)
    ap.add_argument("--out", required=True)
    ap.add_argument("--temperature", type=float, default=1.0)
    a = ap.parse_args()
    export(a.ckpt, a.out, a.temperature)
    print(f"exported {a.ckpt} -> {a.out}")


if __name__ == "__main__":
    main()
