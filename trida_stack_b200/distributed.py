"""Process-group setup and rank helpers (same surface as the reference's ``train/distributed.py``).

One process per GPU; NCCL over NVLink/NVSwitch for the bootstrap collectives and as the baseline
data path (the fused peer-memory path lives in ``parallel``).  The process group gets a short
timeout so a rank that never joins or dies turns into an error on the others instead of a hang.
"""
import datetime
import os

import torch
import torch.distributed as dist


def rank():
    return int(os.environ.get("RANK", 0))


def local_rank():
    return int(os.environ.get("LOCAL_RANK", 0))


def world_size():
    return int(os.environ.get("WORLD_SIZE", 1))


def is_master():
    return rank() == 0


def log(msg):
    if is_master():
        print(msg, flush=True)


def setup_distributed(args, backend=None, timeout_s=None):
    """Bind this rank to its GPU first, then start the process group with that device."""
    timeout = datetime.timedelta(seconds=timeout_s or int(os.environ.get("TRIDA_PG_TIMEOUT", 600)))
    if torch.cuda.is_available() and backend != "gloo":
        torch.cuda.set_device(local_rank())
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29517")
        os.environ.setdefault("RANK", "0")
        os.environ.setdefault("WORLD_SIZE", "1")
        if not dist.is_initialized():
            dist.init_process_group("nccl", device_id=torch.device(f"cuda:{local_rank()}"), timeout=timeout)
        dev = torch.device("cuda", torch.cuda.current_device())
    else:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29517")
        os.environ.setdefault("RANK", "0")
        os.environ.setdefault("WORLD_SIZE", "1")
        if not dist.is_initialized():
            dist.init_process_group("gloo", timeout=timeout)
        dev = torch.device("cpu")
    torch.manual_seed(args.seed)
    return dev


def shard_model(model, args):
    """Prepare the model for training.  Parameter/gradient sharding itself lives in the optimizer
    (flat buffers, ``parallel.zero``), so this only sets train mode and reports sizes."""
    model.train()
    n_train = sum(p.numel() for p in model.parameters() if p.requires_grad)
    n_all = sum(p.numel() for p in model.parameters())
    log(f"[model] {args.model_id} on {world_size()} ranks | {'fp32 master' if args.fp32_master else 'bf16'} weights "
        f"| trainable {n_train / 1e9:.2f}B of {n_all / 1e9:.2f}B params")
    return model
