"""Training loop (reference surface: ``train/train.py:31-172``).

Text, mixed (text + typed decisions) and decision-only loops with gradient accumulation; the
decision micro-batches close an optimizer step; counters (supervised / real / total tokens) are
summed across ranks for the periodic log; checkpoints every ``--save_every`` steps and at the end.
``set_requires_gradient_sync`` is forwarded when the model exposes it (the sharded optimizer
reduces gradients once per step anyway, which is the same schedule).
"""
import sys
import os
import time

import torch
import torch.distributed as dist

from .checkpoint import load_train_state, save_checkpoint
from .cli import build_parser
from .distributed import is_master, log, setup_distributed, world_size
from .optimizer import apply_optimizer_step, build_optimizer


def _sync(model, flag):
    fn = getattr(model, "set_requires_gradient_sync", None)
    if fn is not None:
        fn(flag)


def decision_micro_steps(model, decision_iter, args, dev, running):
    for j in range(args.decision_micro_per_step):
        jb = next(decision_iter)
        jb = {k: (v.to(dev, non_blocking=True) if torch.is_tensor(v) else v) for k, v in jb.items()}
        _sync(model, j == args.decision_micro_per_step - 1)
        jloss, jlogs = model(None, None, None, decision=jb)
        (args.decision_loss_weight * jloss / args.decision_micro_per_step).backward()
        running["decision"] += jloss.item() / args.decision_micro_per_step
        running["decision_acc"] += jlogs["decision_acc"] / args.decision_micro_per_step
        running["decision_q"] += jlogs["decision_questions"]
        running["decision_rec"] += len({q["variant"] for q in jb["questions"]})
        running["decision_tok"] += jlogs["decision_tokens"]


def _all_sum(vals, dev):
    t = torch.tensor(vals, dtype=torch.float64, device=dev)
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return t.tolist()


def _peak_mem():
    return torch.cuda.max_memory_allocated() / 1e9 if torch.cuda.is_available() else 0.0


def log_text_progress(args, dev, running, step, lr, gnorm, t0, run, decision_iter):
    n = args.grad_accum * args.log_every
    dt = max(time.time() - t0, 1e-9)
    g_ntok, g_seq, g_tot = _all_sum([running["ntok"], running["seqtok"], running["tottok"]], dev)
    mb = n * world_size()
    log(f"step {step:6d} | loss {running['loss'] / n:.4f} diff {running['diff'] / n:.4f} ar {running['ar'] / n:.4f} "
        f"| lr {lr:.2e} | gnorm {float(gnorm):.2f} | {n / dt:.2f} mb/s "
        f"| tot_tps {g_tot / dt:,.0f} seq_tps {g_seq / dt:,.0f} resp_tps {g_ntok / dt:,.0f} "
        f"| seqlen {g_seq / mb:,.0f} ntok {g_ntok / mb:,.0f} | mem {_peak_mem():.1f}GB"
        + (f" | decision {running['decision'] / args.log_every:.4f} acc {running['decision_acc'] / args.log_every:.3f}"
           if decision_iter is not None else ""))
    if run is not None:
        run.log({"loss": running["loss"] / n, "diff_loss": running["diff"] / n, "ar_loss": running["ar"] / n,
                 "lr": lr, "grad_norm": float(gnorm), "tot_tps": g_tot / dt, "seq_tps": g_seq / dt,
                 "resp_tps": g_ntok / dt}, step=step)


def log_decision_progress(args, dev, running, step, lr, gnorm, t0, run):
    dt = max(time.time() - t0, 1e-9)
    q, tok, rec = _all_sum([running["decision_q"], running["decision_tok"], running["decision_rec"]], dev)
    log(f"step {step:6d} | decision {running['decision'] / args.log_every:.4f} "
        f"acc {running['decision_acc'] / args.log_every:.3f} | lr {lr:.2e} | gnorm {float(gnorm):.2f} "
        f"| q/step {q / args.log_every:,.0f} rec/step {rec / args.log_every:,.0f} | decision_tps {tok / dt:,.0f}")
    if run is not None:
        run.log({"decision_loss": running["decision"] / args.log_every, "lr": lr, "grad_norm": float(gnorm)}, step=step)


def _fresh():
    return {"loss": 0.0, "diff": 0.0, "ar": 0.0, "ntok": 0, "seqtok": 0, "tottok": 0, "decision": 0.0,
            "decision_acc": 0.0, "decision_q": 0, "decision_rec": 0, "decision_tok": 0}


def run_training(args, dev, model, loaders, optim):
    """Resume if asked, train to ``max_steps``, save the final checkpoint.  With several ranks a
    heartbeat thread watches the others (``parallel.health``): a rank that fails tells the rest,
    and a rank that goes silent for ``$TRIDA_HEARTBEAT_TIMEOUT`` seconds (default 120) stops the
    others at their next step boundary instead of at the process-group timeout."""
    hb = None
    if world_size() > 1 and os.environ.get("TRIDA_HEARTBEAT", "1") != "0":
        from .parallel.health import Heartbeat
        hb = Heartbeat(timeout=float(os.environ.get("TRIDA_HEARTBEAT_TIMEOUT", "120"))).start()
    try:
        _run_training(args, dev, model, loaders, optim, hb)
    except BaseException as e:
        if hb is not None:
            hb.fail(f"{type(e).__name__}: {str(e)[:200]}")
        raise
    finally:
        if hb is not None:
            hb.stop()


def _boundary(hb, step, args):
    if hb is not None:
        hb.beat(step)
        hb.check()
    if step % args.log_every == 0:
        from .parallel.health import check_device
        check_device()


def _run_training(args, dev, model, loaders, optim, hb):
    from .distributed import rank as _rank
    from .utils.trace import StepTracer
    tracer = StepTracer(args.profile_start, args.profile_steps, args.profile_dir, _rank(), dev)
    loader, decision_iter = loaders.text, loaders.decision
    run = None
    if args.wandb and is_master():
        import wandb
        run = wandb.init(project=args.wandb_project, name=args.run_name, config=vars(args))
    step = load_train_state(model, optim, args.resume) if args.resume else args.start_step
    micro = 0
    running = _fresh()
    t0 = time.time()
    done = False
    while args.decision_only and not done:
        decision_micro_steps(model, decision_iter, args, dev, running)
        lr, gnorm = apply_optimizer_step(model, optim, step, args)
        step += 1
        _boundary(hb, step, args)
        if step % args.log_every == 0:
            log_decision_progress(args, dev, running, step, lr, gnorm, t0, run)
            running, t0 = _fresh(), time.time()
        if step % args.save_every == 0:
            save_checkpoint(model, optim, step, args)
        done = step >= args.max_steps
    while not done:
        for batch in loader:
            if batch is None:
                continue
            is_boundary = (micro + 1) % args.grad_accum == 0
            if micro % args.grad_accum == 0:
                tracer.begin(step)
            _sync(model, is_boundary and decision_iter is None)
            host_labels = batch["labels"]
            with tracer.phase("h2d"):
                dev_batch = {k: (v.to(dev, non_blocking=True) if torch.is_tensor(v) else v) for k, v in batch.items()}
            extra = {k: dev_batch[k] for k in ("seg_id", "resp_pos", "resp_block", "turn_id", "pixel_values",
                                              "image_grid_thw", "mrope_pos") if k in dev_batch}
            if (getattr(model, "bd_size", None) and not getattr(model, "ar_only", False) and "seg_id" not in batch
                    and "resp_block" not in batch and torch.is_tensor(host_labels) and host_labels.device.type == "cpu"):
                from .engine import host_rpad
                extra["rpad"] = host_rpad(host_labels, model.bd_size, model.response_buckets)
            with tracer.phase("forward"):
                loss, logs = model(dev_batch["input_ids"], dev_batch["labels"], dev_batch["attention_mask"], **extra)
            with tracer.phase("backward"):
                (loss / args.grad_accum).backward()
            running["loss"] += loss.item()
            running["diff"] += float(logs["diff_loss"])
            running["ar"] += float(logs["ar_loss"])
            running["ntok"] += int(logs["ntok"])
            running["seqtok"] += int(batch["attention_mask"].sum())
            running["tottok"] += int(batch["input_ids"].numel())
            micro += 1
            if not is_boundary:
                continue
            if decision_iter is not None:
                with tracer.phase("decision"):
                    decision_micro_steps(model, decision_iter, args, dev, running)
            with tracer.phase("optimizer"):
                lr, gnorm = apply_optimizer_step(model, optim, step, args)
            tracer.end(tokens=int(batch["input_ids"].numel()))
            step += 1
            _boundary(hb, step, args)
            if step % args.log_every == 0:
                log_text_progress(args, dev, running, step, lr, gnorm, t0, run, decision_iter)
                running, t0 = _fresh(), time.time()
            if step % args.save_every == 0:
                save_checkpoint(model, optim, step, args)
            if step >= args.max_steps:
                done = True
                break
    save_checkpoint(model, optim, step, args)
    if run is not None:
        run.finish()


def main(argv=None):
    args = build_parser().parse_args(argv)
    dev = setup_distributed(args)
    from .data.loaders import build_data_loaders
    from .models.build import build_model
    from .distributed import shard_model
    model = build_model(args, device=dev)
    shard_model(model, args)
    loaders = build_data_loaders(args, model)
    optim = build_optimizer(args, model, device=dev)
    run_training(args, dev, model, loaders, optim)
    dist.destroy_process_group()


if __name__ == "__main__":
    if any(a in ("-h", "--help") for a in sys.argv[1:]):
        build_parser().print_help()
        sys.exit(0)
    main()
