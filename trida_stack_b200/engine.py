"""Training engine: one optimizer step = ``grad_accum`` micro-batches + sharded AdamW update.

``TrainEngine`` is the public per-step API (the training loop in ``train.py`` and ``bench.py`` both
drive it).  A micro-step moves a host batch to the device (pinned, non-blocking), runs the model's
fused forward/backward and leaves gradients in the flat fp32 buffers; the optimizer step reduces
them across ranks, clips on the device and applies AdamW -- no host synchronisation anywhere
except the one the model needs for its loss-row selection.
"""
import math

import torch

from .models.block_diffusion import bucketed_clean_len
from .parallel.zero import ShardedAdamW


def get_lr(it, max_lr, warmup, total, min_ratio):
    """Linear warm-up then cosine decay to ``min_ratio * max_lr`` (``train/optimizer.py:8-15``)."""
    if it < warmup:
        return max_lr * (it + 1) / max(1, warmup)
    if it >= total:
        return max_lr * min_ratio
    r = (it - warmup) / max(1, total - warmup)
    return max_lr * (min_ratio + (1.0 - min_ratio) * 0.5 * (1.0 + math.cos(math.pi * r)))


def host_rpad(labels, bd_size, buckets):
    """Region-B length of a single-row batch, computed on the host copy of the labels."""
    ans = labels != -100
    if not bool(ans.any()):
        return bucketed_clean_len(1, bd_size, buckets)
    L = labels.shape[1]
    first = torch.argmax(ans.int(), 1)
    last = L - 1 - torch.argmax(torch.flip(ans, [1]).int(), 1)
    return bucketed_clean_len(int((last - first + 1).max()), bd_size, buckets)


class TrainEngine:
    def __init__(self, model, lr=1e-5, betas=(0.9, 0.95), weight_decay=0.0, grad_clip=1.0, fp32_master=False,
                 warmup=50, max_steps=2000, lr_min_ratio=0.1, projector_lr_scale=0.1, decision_head_lr_scale=1.0,
                 device=None, comm="nccl", grad_stream=False, full_shard=False, keep_params=False):
        """``full_shard``: decoder-layer weights sharded across ranks and gathered per layer;
        ``keep_params`` keeps gathered weights from forward to backward; ``grad_stream``: fp32
        gradients of one layer at a time (a two-slot ring reduced under backward) instead of
        resident gradient buffers."""
        self.model = model
        self.device = device or next(model.parameters()).device
        groups = model.param_groups(projector_lr_scale=projector_lr_scale,
                                    decision_head_lr_scale=decision_head_lr_scale,
                                    per_layer=grad_stream or full_shard, stream=grad_stream)
        self.optim = ShardedAdamW(groups, lr=lr, betas=betas, weight_decay=weight_decay, fp32_master=fp32_master,
                                  device=self.device, comm=comm, full_shard=full_shard, keep_params=keep_params)
        model.param_ring = self.optim.param_ring

        self.lr, self.warmup, self.max_steps, self.lr_min_ratio = lr, warmup, max_steps, lr_min_ratio
        self.grad_clip = grad_clip

    # ------------------------------------------------------------------------------------------
    def to_device(self, batch):
        out = {}
        for k, v in batch.items():
            if torch.is_tensor(v):
                if v.device.type == "cpu" and self.device.type == "cuda" and not v.is_pinned():
                    v = v.pin_memory()
                out[k] = v.to(self.device, non_blocking=True)
            else:
                out[k] = v
        return out

    def micro_step(self, batch, scale=1.0, rpad=None):
        """Forward + backward of one host (or device) batch; returns (loss, logs) on the device."""
        extra = {} if rpad is None else {"rpad": rpad}
        m = self.model
        if ("seg_id" not in batch and "resp_block" not in batch and hasattr(m, "bd_size")
                and not getattr(m, "ar_only", False) and batch["labels"].device.type == "cpu"
                and rpad is None):
            extra["rpad"] = host_rpad(batch["labels"], m.bd_size, m.response_buckets)
        b = self.to_device(batch)
        kw = {k: b[k] for k in ("seg_id", "resp_pos", "resp_block", "turn_id", "pixel_values",
                                "image_grid_thw", "mrope_pos") if k in b}
        loss, logs = m(b["input_ids"], b["labels"], b["attention_mask"], **kw, **extra)
        (loss * scale).backward()
        return loss.detach(), logs

    def optimizer_step(self, global_step):
        lr = get_lr(global_step, self.lr, self.warmup, self.max_steps, self.lr_min_ratio)
        for g in self.optim.param_groups:
            g["lr"] = lr * g.get("lr_scale", 1.0)
        self.optim.reduce_gradients()
        gnorm = self.optim.clip_grad_norm_(self.grad_clip)
        self.optim.step()
        self.optim.zero_grad(set_to_none=True)
        return lr, gnorm

    def train_step(self, micro_batches, global_step):
        """One optimizer step over ``micro_batches``; returns (mean loss tensor, last logs, lr, gnorm)."""
        n = len(micro_batches)
        total = None
        logs = None
        for mb in micro_batches:
            loss, logs = self.micro_step(mb, scale=1.0 / n)
            total = loss if total is None else total + loss
        lr, gnorm = self.optimizer_step(global_step)
        return total / n, logs, lr, gnorm
