"""Optimizer construction, LR schedule and the per-step update (reference surface:
``train/optimizer.py:8-41``): AdamW(betas=(0.9, adam_beta2), weight_decay) over the model's
``param_groups`` (each tagged with ``lr_scale``), linear warm-up then cosine decay, global-norm
clipping.  On GPU the optimizer is the sharded flat-buffer AdamW (``parallel.zero``) whose norm,
clip coefficient and update stay on the device; any torch optimizer also works (CPU tests)."""
import torch

from .distributed import log
from .engine import get_lr
from .parallel.zero import ShardedAdamW

__all__ = ["get_lr", "build_optimizer", "apply_optimizer_step"]


def build_optimizer(args, model, device=None):
    """Sharded AdamW.  With several ranks the decoder layers are fully sharded (the reference's
    FSDP ``fully_shard`` per layer, ``train/distributed.py:32-59``): each rank keeps 1/world of
    every layer's bf16 weights and gathers a layer around its forward and backward;
    ``--fsdp_keep_params`` keeps the gathered weights from forward to backward
    (``reshard_after_forward=False``).  ``--shard zero2`` keeps replicated weights instead."""
    from .distributed import world_size
    full = getattr(args, "shard", "full") == "full" and world_size() > 1
    groups = model.param_groups(projector_lr_scale=args.projector_lr_scale,
                                decision_head_lr_scale=args.decision_head_lr_scale, per_layer=full,
                                stream=getattr(args, "grad_stream", False))
    opt = ShardedAdamW(groups, lr=args.lr, betas=(0.9, args.adam_beta2), weight_decay=args.weight_decay,
                       fp32_master=getattr(args, "fp32_master", False), device=device,
                       comm=getattr(args, "comm", "nccl"), full_shard=full,
                       keep_params=getattr(args, "fsdp_keep_params", False))
    model.param_ring = opt.param_ring
    for g, src in zip(opt.param_groups, groups):
        g.setdefault("lr_scale", src.get("lr_scale", 1.0))
    if len(groups) > 1:
        log(f"[optim] lr {args.lr:g} | " + " | ".join(f"group {i} x{g.get('lr_scale', 1.0):g}"
                                                       for i, g in enumerate(groups)))
    return opt


def apply_optimizer_step(model, optim, global_step, args):
    """Schedule the LR, reduce + clip gradients, update, clear gradients; returns (lr, grad norm)."""
    lr = get_lr(global_step, args.lr, args.warmup, args.max_steps, args.lr_min_ratio)
    for g in optim.param_groups:
        g["lr"] = lr * g.get("lr_scale", 1.0)
    if isinstance(optim, ShardedAdamW):
        optim.reduce_gradients()
        gnorm = optim.clip_grad_norm_(args.grad_clip)
    else:
        gnorm = torch.nn.utils.clip_grad_norm_(model.parameters(), args.grad_clip)
    optim.step()
    optim.zero_grad(set_to_none=True)
    return lr, gnorm
