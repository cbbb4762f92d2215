"""Checkpoints in the reference layout (``train/checkpoint.py:14-105``):

    save_dir/step_N/
      config.json, model*.safetensors (+ model.safetensors.index.json)   HF-loadable weights
      tokenizer files (with <|mask|>)                                    when a tokenizer is attached
      block_diffusion.json  {bd_size, mask_id, ar_loss_weight}
      jev_head.pt           {"head": {q.weight, q.bias, k.weight, k.bias}, "head_dim"}   decision head
      train_state/ + train_state.json {global_step}                      with --save_optim_state

Weights are written by rank 0 in bf16 (fp32 masters are cast); the sharded optimizer state is
written with torch.distributed.checkpoint, one key set per rank, and restored only into a run with
the same world size (exact resume); otherwise ``--resume`` is a warm restart.  Every early exit is
decided identically on all ranks so the collective calls never diverge.
"""
import json
import os

import torch
import torch.distributed as dist

from .distributed import is_master, log

SHARD_BYTES = 5 * 1024 ** 3


def _barrier():
    if dist.is_available() and dist.is_initialized():
        dist.barrier()


class ShardWriter:
    """Streams (name, tensor) pairs into safetensors shards of at most ``max_shard_bytes`` (HF
    layout): one ``model.safetensors``, or numbered shards plus ``model.safetensors.index.json``.
    Only the shard being filled is held in host memory; full shards are written under temporary
    names and renamed once the shard count is known."""

    def __init__(self, out_dir, max_shard_bytes=SHARD_BYTES):
        self.out, self.max = out_dir, max_shard_bytes
        os.makedirs(out_dir, exist_ok=True)
        self.cur, self.size, self.done, self.count, self.total = {}, 0, [], 0, 0

    def add(self, name, tensor):
        t = tensor.detach().to("cpu").contiguous()
        nbytes = t.numel() * t.element_size()
        if self.cur and self.size + nbytes > self.max:
            self._flush()
        self.cur[name] = t
        self.size += nbytes
        self.count += 1
        self.total += nbytes

    def _flush(self):
        from safetensors.torch import save_file
        tmp = os.path.join(self.out, f".shard-{len(self.done):05d}.tmp")
        save_file(self.cur, tmp, metadata={"format": "pt"})
        self.done.append((tmp, list(self.cur)))
        self.cur, self.size = {}, 0

    def close(self):
        if self.cur or not self.done:
            self._flush()
        n = len(self.done)
        if n == 1:
            os.replace(self.done[0][0], os.path.join(self.out, "model.safetensors"))
            return
        weight_map = {}
        for i, (tmp, names) in enumerate(self.done):
            fname = f"model-{i + 1:05d}-of-{n:05d}.safetensors"
            os.replace(tmp, os.path.join(self.out, fname))
            weight_map.update(dict.fromkeys(names, fname))
        with open(os.path.join(self.out, "model.safetensors.index.json"), "w") as f:
            json.dump({"metadata": {"total_size": self.total}, "weight_map": weight_map}, f, indent=2)


def write_hf_weights(state, out_dir, max_shard_bytes=SHARD_BYTES):
    """Save ``state`` (name -> tensor) as safetensors shards + index (HF layout)."""
    w = ShardWriter(out_dir, max_shard_bytes)
    for name in state:
        w.add(name, state[name])
    w.close()


def read_hf_weights(path):
    """name -> tensor from every ``*.safetensors`` file of an HF model dir."""
    import glob
    from safetensors.torch import load_file
    files = sorted(glob.glob(os.path.join(path, "*.safetensors")))
    if not files:
        raise FileNotFoundError(f"no *.safetensors weights in {path}")
    sd = {}
    for f in files:
        sd.update(load_file(f))
    return sd


def save_hf(model, args, tag):
    out = os.path.join(args.save_dir, tag)
    if is_master():
        dec = model.decoder
        state = dec.hf_state_dict(dtype=torch.bfloat16)
        write_hf_weights(state, out)
        cfg = dec.cfg.to_hf_dict()
        cfg["dtype"] = "bfloat16"
        cfg.pop("torch_dtype", None)
        with open(os.path.join(out, "config.json"), "w") as f:
            json.dump(cfg, f, indent=2)
        if getattr(model, "tokenizer", None) is not None:
            model.tokenizer.save_pretrained(out)
        if getattr(model, "image_processor", None) is not None:
            model.image_processor.save_pretrained(out)
        head = getattr(model, "decision_head", None)
        if head is not None:
            torch.save({"head": {k: v.detach().to("cpu", torch.bfloat16 if v.is_floating_point() else v.dtype)
                                 for k, v in head.state_dict().items()},
                        "head_dim": head.q.out_features}, os.path.join(out, "jev_head.pt"))
        with open(os.path.join(out, "block_diffusion.json"), "w") as f:
            json.dump({"bd_size": model.bd_size, "mask_id": model.mask_id,
                       "ar_loss_weight": model.ar_loss_weight}, f, indent=2)
        log(f"[save] wrote {out}")
    _barrier()


def _optim_state(optim):
    sd = optim.state_dict()
    r = sd["rank"]
    flat = {"step": torch.tensor(sd["step"]), "world": torch.tensor(sd["world"])}
    for i, g in enumerate(sd["groups"]):
        flat[f"rank{r}.g{i}.m"] = g["m"]
        flat[f"rank{r}.g{i}.v"] = g["v"]
        if g["master"] is not None:
            flat[f"rank{r}.g{i}.master"] = g["master"]
    return flat


def save_train_state(model, optim, global_step, args, tag):
    if not args.save_optim_state:
        return
    import torch.distributed.checkpoint as dcp
    out = os.path.join(args.save_dir, tag)
    dcp.save({"optim": _optim_state(optim)}, checkpoint_id=os.path.join(out, "train_state"))
    if is_master():
        with open(os.path.join(out, "train_state.json"), "w") as f:
            json.dump({"global_step": global_step}, f)
    _barrier()


def load_train_state(model, optim, resume_dir):
    """Restore the optimizer + step when ``resume_dir`` has train state, else 0 (warm restart)."""
    verify_manifest(resume_dir)
    state_dir = os.path.join(resume_dir, "train_state")
    meta = os.path.join(resume_dir, "train_state.json")
    if not (os.path.isdir(state_dir) and os.path.exists(meta)):
        log(f"[resume] {resume_dir} has no optimizer state -> warm restart (fresh optimizer, step 0)")
        return 0
    import torch.distributed.checkpoint as dcp
    tmpl = _optim_state(optim)
    dcp.load({"optim": tmpl}, checkpoint_id=state_dir)
    sd = optim.state_dict()
    if int(tmpl["world"]) != sd["world"]:
        raise ValueError(f"train_state was written by {int(tmpl['world'])} ranks, this run has {sd['world']}")
    r = sd["rank"]
    for i, g in enumerate(sd["groups"]):
        g["m"].copy_(tmpl[f"rank{r}.g{i}.m"])
        g["v"].copy_(tmpl[f"rank{r}.g{i}.v"])
        if g["master"] is not None:
            g["master"].copy_(tmpl[f"rank{r}.g{i}.master"])
    optim.step_count = int(tmpl["step"])
    with open(meta) as f:
        gs = int(json.load(f)["global_step"])
    log(f"[resume] restored optimizer + global_step={gs} from {resume_dir}")
    return gs


MANIFEST = "manifest.json"


class CheckpointCorrupt(RuntimeError):
    pass


def _digest(path, chunk=1 << 24):
    import hashlib
    h = hashlib.sha256()
    with open(path, "rb") as f:
        while True:
            b = f.read(chunk)
            if not b:
                break
            h.update(b)
    return h.hexdigest()


def write_manifest(ckpt_dir):
    """Record size and SHA-256 of every file under ``ckpt_dir`` (written last, by one rank)."""
    files = {}
    for root, _, names in os.walk(ckpt_dir):
        for n in sorted(names):
            full = os.path.join(root, n)
            rel = os.path.relpath(full, ckpt_dir)
            if rel == MANIFEST:
                continue
            files[rel] = {"bytes": os.path.getsize(full), "sha256": _digest(full)}
    tmp = os.path.join(ckpt_dir, MANIFEST + ".tmp")
    with open(tmp, "w") as f:
        json.dump({"files": files}, f, indent=1)
    os.replace(tmp, os.path.join(ckpt_dir, MANIFEST))


def verify_manifest(ckpt_dir):
    """Raise ``CheckpointCorrupt`` if a file listed in the manifest is missing, truncated or altered;
    a checkpoint without a manifest (written by another tool) is accepted as is."""
    path = os.path.join(ckpt_dir, MANIFEST)
    if not os.path.exists(path):
        return False
    with open(path) as f:
        files = json.load(f)["files"]
    bad = []
    for rel, meta in files.items():
        full = os.path.join(ckpt_dir, rel)
        if not os.path.exists(full):
            bad.append(f"{rel}: missing")
        elif os.path.getsize(full) != meta["bytes"]:
            bad.append(f"{rel}: {os.path.getsize(full)} bytes, manifest says {meta['bytes']}")
        elif _digest(full) != meta["sha256"]:
            bad.append(f"{rel}: content differs from the manifest")
    if bad:
        raise CheckpointCorrupt(f"checkpoint {ckpt_dir} is damaged: " + "; ".join(bad[:8]))
    return True


def save_checkpoint(model, optim, global_step, args):
    """Weights first, then the optional optimizer state, on every rank in the same order; rank 0
    then writes the integrity manifest."""
    tag = f"step_{global_step}"
    ring = getattr(optim, "param_ring", None)
    if ring is not None:
        ring.materialize()      # full-shard weights: every rank gathers every layer for the save
    try:
        save_hf(model, args, tag)
    finally:
        if ring is not None:
            ring.release_all()
    save_train_state(model, optim, global_step, args, tag)
    _barrier()
    out = os.path.join(args.save_dir, tag) if getattr(args, "save_dir", None) else None
    if out and os.path.isdir(out) and is_master() and os.environ.get("TRIDA_CKPT_MANIFEST", "1") != "0":
        write_manifest(out)
    _barrier()
