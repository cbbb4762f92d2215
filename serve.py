#!/usr/bin/env python3
"""Serve a Trida checkpoint over HTTP with the native engine (OpenAI-compatible + decisions).

    python serve.py [model] --mode {self-spec,causal,diffusion,decide} --port 30000 [--config decode.yaml]

Flags follow the reference launcher (``inference/zoro-1/serve.py:193-222``); model resolution:
positional > ``$TRIDA_DECIDE_MODEL`` (decide) > ``$TRIDA_MODEL``.  Checkpoints are local HF
directories (``config.json`` + safetensors [+ ``decision_head.pt`` / ``jev_head.pt``,
``temperature.json``, ``block_diffusion.json``]).  ``--random-init CONFIG_JSON`` serves a
random-initialised model of that architecture (smoke tests without weights).

Decode config (YAML, keys of ``configs/zoro1_self_spec_b15_g8.yaml``): ``block_size`` (canvas
rows, 2N-1; in ``diffusion`` mode the denoised block length), ``gen_block_size`` (N), ``mask_id``,
``temperature``, ``top_k``, ``top_p``; ``diffusion`` mode (pure block diffusion with the
LowConfidenceShift gate) also reads ``threshold`` and ``max_steps``.  Decode steps replay from
CUDA graphs for the ``--cuda-graph-bs`` batch sizes.  ``--tp N`` shards the model over N GPUs:
launch with ``torchrun --nproc-per-node N``; rank 0 serves HTTP and every rank steps the same
engine (requests are broadcast to the other ranks at each step).
"""
import argparse
import json
import os
import sys

MODES = ("self-spec", "causal", "diffusion", "decide")


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("model", nargs="?", default=None)
    ap.add_argument("--mode", default="self-spec", choices=MODES)
    ap.add_argument("--port", type=int, default=30000)
    ap.add_argument("--host", default="0.0.0.0")
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--mem-fraction", type=float, default=0.8)
    ap.add_argument("--max-running", type=int, default=32)
    ap.add_argument("--max-len", type=int, default=8192)
    ap.add_argument("--kv-pages", type=int, default=0,
                    help="full-attention KV pool in pages of 64 positions shared by all requests (0: enough for "
                         "every slot at --max-len)")
    ap.add_argument("--cuda-graph-bs", default="1 2 4 8")
    ap.add_argument("--dtype", default="bfloat16", choices=["bfloat16", "float32"])
    ap.add_argument("--config", default=None, help="decode YAML (block_size, gen_block_size, mask_id, ...)")
    ap.add_argument("--reasoning-parser", default="qwen3", choices=["qwen3", "deepseek-r1"])
    ap.add_argument("--log", default=None)
    ap.add_argument("--no-stats", action="store_true")
    ap.add_argument("--no-shape", action="store_true")
    ap.add_argument("--dry-run", action="store_true")
    ap.add_argument("--random-init", default=None, help="serve a random-init model of this config.json")
    ap.add_argument("--device", default=None)
    ap.add_argument("--no-graphs", action="store_true", help="launch decode steps eagerly (no CUDA graphs)")
    return ap.parse_args(argv)


def resolve_model(args):
    if args.model:
        return args.model
    if args.mode == "decide" and os.environ.get("TRIDA_DECIDE_MODEL"):
        return os.environ["TRIDA_DECIDE_MODEL"]
    return os.environ.get("TRIDA_MODEL")


def decode_config(path):
    if not path:
        return {}
    import yaml
    with open(path) as f:
        return yaml.safe_load(f) or {}


def build(args):
    """(engine, tokenizer, model name, decider) for the arguments."""
    import torch

    from trida_stack_b200.models import Decoder, ModelConfig
    from trida_stack_b200.models.build import MASK_TOKEN, load_decoder, load_tokenizer
    from trida_stack_b200.serve import Engine, Runtime
    dev = args.device or ("cuda" if torch.cuda.is_available() else "cpu")
    dtype = torch.bfloat16 if args.dtype == "bfloat16" else torch.float32
    path = resolve_model(args)
    tok = None
    if args.random_init:
        with open(args.random_init) as f:
            cfg = ModelConfig.from_hf_dict(json.load(f))
        dec = Decoder(cfg, dtype=dtype, device=dev)
        name = "random-init"
    else:
        if not path or not os.path.isdir(path):
            raise SystemExit(f"model directory not found: {path!r} (give a local checkpoint directory)")
        tok = load_tokenizer(path)
        if args.mode == "decide":
            dec = None          # the decision model below owns the decoder
        else:
            dec, _ = load_decoder(path, dev, dtype, tokenizer=tok, add_mask=args.mode != "causal")
        name = os.path.basename(os.path.normpath(path))
    dcfg = decode_config(args.config)
    mask_id = dcfg.get("mask_id")
    if mask_id is None and tok is not None:
        mask_id = tok.convert_tokens_to_ids(MASK_TOKEN)
    if mask_id is None and path and os.path.isfile(os.path.join(path, "block_diffusion.json")):
        with open(os.path.join(path, "block_diffusion.json")) as f:
            mask_id = json.load(f).get("mask_id")
    n = int(dcfg.get("gen_block_size", (int(dcfg.get("block_size", 7)) + 1) // 2))
    decider = None
    if args.mode == "decide":
        from trida_stack_b200.cli import build_parser
        from trida_stack_b200.models.build import build_model
        from trida_stack_b200.serve.decide import DecideEngine
        ns = build_parser().parse_args(["--model_id", path, "--ar_only", "--decision_data", "serving"])
        model = build_model(ns, torch.device(dev)).eval()
        decider = DecideEngine(model, tok, DecideEngine.temperatures_from(path))
        dec = model.decoder
    if mask_id is None:
        mask_id = dec.cfg.vocab_size - 1
    tp = None
    if args.tp > 1:
        import torch.distributed as dist

        from trida_stack_b200.serve.tp import TPContext, shard_decoder
        dec = shard_decoder(dec, dist.get_rank(), dist.get_world_size())
        tp = TPContext(max_rows=args.max_running * 64, hidden=dec.cfg.hidden_size)
    rt = Runtime(dec, max_slots=args.max_running, max_len=args.max_len, device=dev, tp=tp,
                 kv_pages=args.kv_pages or None)
    mode = args.mode if args.mode in ("self-spec", "diffusion") else "causal"
    graphs = dev.startswith("cuda") and not args.no_graphs
    engine = Engine(rt, mask_id=mask_id, mode=mode, n=n, max_running=args.max_running, graphs=graphs,
                    block_size=int(dcfg.get("block_size", 8)), threshold=float(dcfg.get("threshold", 0.9)),
                    max_steps=dcfg.get("max_steps"))
    if graphs:
        rt.use_graphs(tuple(int(b) for b in args.cuda_graph_bs.split()))
    if decider is not None:
        decider.gen_engine = engine      # reasoning-then-decide writes its reasoning with the same weights
    if not args.no_stats:
        engine.stats_interval = 10.0
    return engine, tok, name, decider


def _init_tp(args):
    """torchrun-launched TP ranks: NCCL for the shards' collectives, gloo for the request stream."""
    import datetime

    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world != args.tp:
        raise SystemExit(f"--tp {args.tp} needs torchrun --nproc-per-node {args.tp} (WORLD_SIZE={world})")
    if args.mode == "decide":
        raise SystemExit("decide mode runs on one GPU (--tp 1)")
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    args.device = f"cuda:{local}"
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    return dist.new_group(backend="gloo", timeout=datetime.timedelta(days=1))


class _Tee:
    """Write-through to the console and a log file (``--log``)."""

    def __init__(self, *streams):
        self.streams = streams

    def write(self, data):
        for s in self.streams:
            s.write(data)
            s.flush()
        return len(data)

    def flush(self):
        for s in self.streams:
            s.flush()

    def isatty(self):
        return False


def main(argv=None):
    args = parse_args(argv)
    if args.log:
        fh = open(args.log, "a", buffering=1)
        sys.stdout, sys.stderr = _Tee(sys.__stdout__, fh), _Tee(sys.__stderr__, fh)
    if args.dry_run:
        print(json.dumps({"model": resolve_model(args), "mode": args.mode, "port": args.port, "host": args.host,
                          "tp": args.tp, "config": decode_config(args.config)}))
        return 0
    ctrl = _init_tp(args) if args.tp > 1 else None
    engine, tok, name, decider = build(args)
    if tok is None:
        raise SystemExit("the HTTP server needs a tokenizer in the checkpoint directory")
    driver = None
    if ctrl is not None:
        from trida_stack_b200.serve.lockstep import LockstepDriver
        driver = LockstepDriver(engine, ctrl)
        if driver.rank != 0:
            driver.run_follower()       # steps in lock-step until rank 0 sends the stop flag
            return 0
    from trida_stack_b200.serve.server import build_app
    import uvicorn
    (driver or engine).start()
    app = build_app(engine, tok, name, decider)
    try:
        uvicorn.run(app, host=args.host, port=args.port, log_level="warning")
    finally:
        if driver is not None:
            driver.stop()
    return 0


if __name__ == "__main__":
    sys.exit(main())
