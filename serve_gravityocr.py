#!/usr/bin/env python3
"""Serve a GravityOCR (GLM-OCR block-diffusion) checkpoint: crop-level OCR over an OpenAI API.

    python serve_gravityocr.py /path/to/GravityOCR [--mode self-spec|causal] [--port 30000]

The native counterpart of the reference's ``inference/gravityocr/serve.sh``: ``self-spec`` (default)
decodes by draft / verify rounds over a window of ``--draft`` rows (the boundary token plus
``bd_size`` masks; ``bd_size`` and the mask id from the checkpoint's ``block_diffusion.json`` or
``$SELFSPEC_MASK_ID``), ``causal`` one token per forward.  Generated tokens sit ``--pos-offset``
RoPE positions after the causal layout (1 reproduces GravityOCR's published self-spec setting; 0 is
the causal layout).  Binds to 127.0.0.1 by default; the API key comes from ``$API_KEY`` or
``--api-key-file`` (never from the command line).  ``--random-init CONFIG_JSON`` serves random
weights of an architecture (smoke tests).
"""
import argparse
import json
import os
import sys


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("ckpt", nargs="?", default=os.environ.get("CKPT"))
    ap.add_argument("--mode", default="self-spec", choices=["self-spec", "causal"])
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=30000)
    ap.add_argument("--served-name", default="glm-ocr")
    ap.add_argument("--draft", type=int, default=None, help="draft window rows (default bd_size + 1)")
    ap.add_argument("--pos-offset", type=int, default=int(os.environ.get("SELFSPEC_POS_OFFSET", "1")))
    ap.add_argument("--context", type=int, default=16384)
    ap.add_argument("--max-running", type=int, default=16)
    ap.add_argument("--api-key-file", default=None)
    ap.add_argument("--device", default=None)
    ap.add_argument("--dtype", default="bfloat16", choices=["bfloat16", "float32"])
    ap.add_argument("--no-graphs", action="store_true")
    ap.add_argument("--random-init", default=None, help="serve random weights of this config.json")
    return ap.parse_args(argv)


def build(args):
    import torch

    from trida_stack_b200.data.images import ImageProcessor
    from trida_stack_b200.models.glm_ocr import GlmOcrDecoder, glm_ocr_config, load_glm_ocr
    from trida_stack_b200.serve import Engine, Runtime
    from trida_stack_b200.serve.ocr import mask_id_of, pick_eos
    dev = args.device or ("cuda" if torch.cuda.is_available() else "cpu")
    dtype = torch.bfloat16 if args.dtype == "bfloat16" else torch.float32
    tok = None
    if args.random_init:
        with open(args.random_init) as f:
            dec, bd = GlmOcrDecoder(glm_ocr_config(json.load(f)), dtype=dtype, device=dev), {}
    else:
        if not args.ckpt or not os.path.isdir(args.ckpt):
            raise SystemExit(f"checkpoint directory not found: {args.ckpt!r}")
        dec, bd = load_glm_ocr(args.ckpt, dev, dtype)
        from trida_stack_b200.models.build import load_tokenizer
        tok = load_tokenizer(args.ckpt)
    proc = (ImageProcessor.from_pretrained(args.ckpt, glm=True) if args.ckpt else None) or ImageProcessor(
        patch_size=14, temporal_patch_size=2, merge_size=2, min_pixels=12544, max_pixels=9633792,
        image_mean=(0.48145466, 0.4578275, 0.40821073), image_std=(0.26862954, 0.26130258, 0.27577711), glm=True)
    mask_id, src = (None, None)
    block = 32
    if args.mode == "self-spec":
        mask_id, src = mask_id_of(args.ckpt, dec.cfg.vocab_size) if not args.random_init else (
            dec.cfg.vocab_size - 1, "random-init")
        block = (args.draft - 1) if args.draft else int(bd.get("bd_size", 32))
        if bd.get("bd_size") and block != int(bd["bd_size"]):
            print(f"[gravityocr] warning: draft window {block + 1} != bd_size {bd['bd_size']} + 1", flush=True)
        print(f"[gravityocr] K={block + 1} mask_id={mask_id} (from {src}) bd_size={bd.get('bd_size')}", flush=True)
    rt = Runtime(dec, max_slots=args.max_running, max_len=args.context + block + 2, device=dev)
    graphs = str(dev).startswith("cuda") and not args.no_graphs
    engine = Engine(rt, mask_id=mask_id if mask_id is not None else dec.cfg.vocab_size - 1,
                    mode="draft-verify" if args.mode == "self-spec" else "causal", block_size=block,
                    max_running=args.max_running, graphs=graphs, pos_offset=args.pos_offset)
    return engine, tok, proc, pick_eos(args.ckpt, tok) if tok is not None else ()


def main(argv=None):
    args = parse_args(argv)
    key = os.environ.get("API_KEY")
    if args.api_key_file:
        with open(args.api_key_file) as f:
            key = f.read().strip()
    engine, tok, proc, eos = build(args)
    if tok is None:
        raise SystemExit("the HTTP server needs the checkpoint's tokenizer")
    from trida_stack_b200.serve.ocr import build_ocr_app
    import uvicorn
    engine.start()
    print(f"[serve] MODE={args.mode} HOST={args.host} PORT={args.port} SERVED_NAME={args.served_name} "
          f"CKPT={args.ckpt} auth={'on' if key else 'off'}", flush=True)
    uvicorn.run(build_ocr_app(engine, tok, proc, args.served_name, api_key=key, context=args.context, eos=eos),
                host=args.host, port=args.port, log_level="warning")
    return 0


if __name__ == "__main__":
    sys.exit(main())
