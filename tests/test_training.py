"""Training orchestration on CPU: loop schedule, sync pattern, resume, checkpoint order, CLI,
process-group setup order (same checks as the reference's train/test_training.py)."""
import itertools
from types import SimpleNamespace
from unittest.mock import Mock

import pytest
import torch

from trida_stack_b200 import checkpoint, distributed
from trida_stack_b200 import train as trainer
from trida_stack_b200.cli import build_parser
from trida_stack_b200.data.loaders import TrainingLoaders
from trida_stack_b200.engine import get_lr
from trida_stack_b200.optimizer import build_optimizer


class ToyModel(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.tensor(1.0))
        self.events = []

    def set_requires_gradient_sync(self, enabled):
        self.events.append(("sync", enabled))

    def forward(self, ids, labels, mask, *, decision=None, **kwargs):
        if decision is not None:
            self.events.append(("decision", None))
            return 2 * self.weight.square(), {"decision_acc": 1.0, "decision_questions": 1, "decision_tokens": 4}
        self.events.append(("text", kwargs))
        loss = self.weight.square()
        return loss, {"diff_loss": loss.detach(), "ar_loss": loss.detach(), "ntok": 2}


@pytest.mark.parametrize("mode", ["text", "mixed", "decision"])
@pytest.mark.parametrize("resume", [False, True])
def test_training_updates_sync_resume_and_checkpoint_boundaries(monkeypatch, mode, resume):
    args = build_parser().parse_args([])
    args.decision_only = mode == "decision"
    args.decision_micro_per_step = 2
    args.decision_loss_weight = 0.5
    args.grad_accum = 2
    args.grad_clip = 100
    args.lr = 0.1
    args.lr_min_ratio = 1
    args.warmup = 0
    args.max_steps = 3
    args.log_every = 1
    args.save_every = 2
    args.resume = "checkpoint" if resume else None
    model = ToyModel()
    optim = torch.optim.SGD(model.parameters(), lr=args.lr)
    batch = {k: torch.ones(1, 2, dtype=torch.long) for k in (
        "input_ids", "labels", "attention_mask", "seg_id", "resp_pos", "resp_block", "turn_id",
        "pixel_values", "image_grid_thw", "mrope_pos")}
    text = [None, batch, batch, batch] if mode != "decision" else None
    decision = itertools.repeat({"questions": [{"variant": 0}]}) if mode != "text" else None
    saved, logs = [], []

    def save(model, optimizer, step, args):
        assert model.weight.grad is None
        saved.append(step)

    load = Mock(return_value=1)
    monkeypatch.setattr(trainer, "load_train_state", load)
    monkeypatch.setattr(trainer, "save_checkpoint", save)
    monkeypatch.setattr(trainer, "log", logs.append)
    trainer.run_training(args, "cpu", model, TrainingLoaders(text, decision), optim)
    steps = 2 if resume else 3
    factor = 0.6 if mode == "mixed" else 0.8
    assert model.weight.item() == pytest.approx(factor ** steps, abs=1e-6)
    assert saved == [2, 3]
    assert len(logs) == steps
    assert [e[1] for e in model.events if e[0] == "sync"] == {
        "text": [False, True] * steps, "mixed": [False, False, False, True] * steps,
        "decision": [False, True] * steps}[mode]
    assert sum(e[0] == "text" for e in model.events) == (0 if mode == "decision" else 2 * steps)
    assert load.call_count == int(resume)


def test_lr_schedule_and_optimizer_groups():
    args = build_parser().parse_args(["--lr", "1e-3", "--decision_head_lr_scale", "5"])
    a = torch.nn.Parameter(torch.ones(10))
    b = torch.nn.Parameter(torch.ones(3))
    model = SimpleNamespace(param_groups=Mock(return_value=[{"params": [a], "lr_scale": 1.0},
                                                            {"params": [b], "lr_scale": 5.0}]))
    opt = build_optimizer(args, model, device=torch.device("cpu"))
    assert opt.defaults["betas"] == (0.9, args.adam_beta2)
    assert opt.param_groups[1]["lr_scale"] == 5.0
    assert get_lr(0, 1, 2, 10, 0.1) == 0.5
    assert get_lr(10, 1, 2, 10, 0.1) == 0.1


def test_checkpoint_saves_weights_before_optimizer(monkeypatch):
    events = []
    monkeypatch.setattr(checkpoint, "save_hf", lambda *a: events.append(("weights", a[-1])))
    monkeypatch.setattr(checkpoint, "save_train_state", lambda *a: events.append(("optimizer", a[-1])))
    checkpoint.save_checkpoint(None, None, 12, None)
    assert events == [("weights", "step_12"), ("optimizer", "step_12")]


def test_distributed_binds_gpu_before_process_group(monkeypatch):
    events = []
    monkeypatch.setenv("LOCAL_RANK", "2")
    monkeypatch.setattr(torch.cuda, "is_available", lambda: True)
    monkeypatch.setattr(torch.cuda, "set_device", lambda n: events.append(("device", n)))
    monkeypatch.setattr(distributed.dist, "is_initialized", lambda: False)
    monkeypatch.setattr(distributed.dist, "init_process_group",
                        lambda backend, device_id, timeout: events.append((backend, str(device_id))))
    monkeypatch.setattr(torch, "manual_seed", lambda seed: events.append(("seed", seed)))
    monkeypatch.setattr(torch.cuda, "current_device", lambda: 2)
    distributed.setup_distributed(SimpleNamespace(seed=42))
    assert events == [("device", 2), ("nccl", "cuda:2"), ("seed", 42)]


@pytest.mark.parametrize("suffix,value,expected", [
    ("data", "records.jsonl", "records.jsonl"), ("only", None, True), ("loss_weight", "0.5", 0.5),
    ("micro_per_step", "2", 2), ("max_tokens", "1024", 1024), ("max_state", "384", 384),
    ("head_dim", "32", 32), ("head_lr_scale", "5", 5.0)])
def test_cli_accepts_decision_flags_and_rejects_legacy(suffix, value, expected):
    p = build_parser()
    extra = [] if value is None else [value]
    assert getattr(p.parse_args([f"--decision_{suffix}", *extra]), f"decision_{suffix}") == expected
    with pytest.raises(SystemExit) as e:
        p.parse_args([f"--jev_{suffix}", *extra])
    assert e.value.code == 2


def test_help_is_torch_free():
    import subprocess
    import sys
    code = ("import sys; sys.argv=['train.py','--help']; import builtins; real=builtins.__import__\n"
            "def guard(n,*a,**k):\n    assert not n.startswith('torch'), n\n    return real(n,*a,**k)\n"
            "builtins.__import__=guard\nexec(open('train.py').read())")
    import os
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", code], cwd=root, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    assert "--model_id" in r.stdout


def test_streamed_layer_gradients_match_resident():
    """Per-layer gradient streaming (two-slot ring, reduce into the shard as each layer's backward
    ends) gives the same update as the resident full-gradient buffers."""
    import copy

    from helpers import make_tiny_qwen3  # noqa: F401  (fixture module on sys.path)
    from trida_stack_b200.engine import TrainEngine
    from trida_stack_b200.models import BlockDiffusionLM, Decoder, qwen3_config
    torch.manual_seed(0)
    cfg = qwen3_config(vocab_size=97, hidden_size=32, intermediate_size=64, num_layers=3, n_heads=2,
                       n_kv_heads=1, head_dim=16)
    dec = Decoder(cfg, dtype=torch.float32)
    outs = []
    for stream in (False, True):
        m = BlockDiffusionLM(copy.deepcopy(dec), mask_id=96, pad_id=95, bd_size=4, ar_loss_weight=1.0)
        m.train()
        eng = TrainEngine(m, lr=1e-2, warmup=0, max_steps=10, device=torch.device("cpu"), grad_stream=stream)
        g = torch.Generator().manual_seed(1)
        torch.manual_seed(5)                     # same noising draws in both runs
        for step in range(2):
            ids = torch.randint(0, 95, (2, 16), generator=g)
            labels = ids.clone()
            labels[:, :8] = -100
            eng.train_step([{"input_ids": ids, "labels": labels, "attention_mask": torch.ones_like(ids)}], step)
        outs.append([p.detach().clone() for p in m.parameters()])
    for a, b in zip(*outs):
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-6)


def test_step_tracer_and_request_trace(tmp_path, monkeypatch):
    """--profile_* window: one JSON line per traced step with per-phase times (phases repeated by
    gradient accumulation are summed); $TRIDA_TRACE_JSONL: one line per finished request."""
    import json as _json

    from trida_stack_b200.utils.trace import StepTracer
    tr = StepTracer(start=2, steps=2, out_dir=str(tmp_path / "prof"), rank=0, device="cpu")
    for step in range(6):
        tr.begin(step)
        for _ in range(2):
            with tr.phase("forward"):
                sum(range(1000))
            with tr.phase("backward"):
                sum(range(2000))
        tr.end(tokens=8)
    recs = [_json.loads(l) for l in open(tmp_path / "prof" / "rank0.jsonl")]
    assert [r["step"] for r in recs] == [2, 3]
    assert all(r["forward_ms"] > 0 and r["backward_ms"] > 0 and r["total_ms"] >= r["forward_ms"] for r in recs)
    monkeypatch.setenv("TRIDA_TRACE_JSONL", str(tmp_path / "req.jsonl"))
    from test_serve_cpu import tiny_dense

    from trida_stack_b200.serve import Engine, Runtime
    eng = Engine(Runtime(tiny_dense(), max_slots=2, max_len=128), mask_id=96, mode="self-spec", n=2)
    eng.generate([[1, 2, 3], [4, 5, 6, 7]], max_new_tokens=6)
    lines = [_json.loads(l) for l in open(tmp_path / "req.jsonl")]
    assert len(lines) == 2 and all(l["output_tokens"] == 6 and l["forwards"] > 0 for l in lines)


def test_kernel_breakdown_runs_and_reports(capsys):
    """``--kernel-breakdown``'s helper: profiles the given steps and prints one table (on a CPU-only
    machine it has no device kernels to list and returns no rows)."""
    from trida_stack_b200.utils.trace import kernel_breakdown
    calls = []
    rows = kernel_breakdown(lambda: calls.append(torch.ones(64).sum()), steps=3)
    assert len(calls) == 3
    assert "kernel breakdown" in capsys.readouterr().err
    assert all(0.0 <= r[0] <= 1.0 for r in rows)


def test_layer_checkpoint_and_offload_match_resident():
    """Recomputing every layer in backward (``--activation_checkpoint layer``), with or without
    ``--activation_offload``, gives the same update as keeping activations resident; ``auto``
    keeps them resident when they fit (always on the host)."""
    import copy

    from trida_stack_b200.engine import TrainEngine
    from trida_stack_b200.models import BlockDiffusionLM, Decoder, qwen3_config
    torch.manual_seed(0)
    cfg = qwen3_config(vocab_size=97, hidden_size=32, intermediate_size=64, num_layers=3, n_heads=2,
                       n_kv_heads=1, head_dim=16)
    dec = Decoder(cfg, dtype=torch.float32)
    outs = []
    for mode, offload in (("none", False), ("layer", False), ("layer", True), ("auto", True)):
        m = BlockDiffusionLM(copy.deepcopy(dec), mask_id=96, pad_id=95, bd_size=4, ar_loss_weight=1.0,
                             activation_checkpoint=mode, activation_offload=offload)
        m.train()
        eng = TrainEngine(m, lr=1e-2, warmup=0, max_steps=10, device=torch.device("cpu"))
        g = torch.Generator().manual_seed(1)
        torch.manual_seed(5)
        for step in range(2):
            ids = torch.randint(0, 95, (2, 16), generator=g)
            labels = ids.clone()
            labels[:, :8] = -100
            eng.train_step([{"input_ids": ids, "labels": labels, "attention_mask": torch.ones_like(ids)}], step)
        outs.append([p.detach().clone() for p in m.parameters()])
    for other in outs[1:]:
        for a, b in zip(outs[0], other):
            torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-6)
    args = build_parser().parse_args(["--model_id", "x", "--activation_offload", "--activation_checkpoint", "layer"])
    assert args.activation_offload and args.activation_checkpoint == "layer"
