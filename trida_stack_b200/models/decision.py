"""Decision pointer head and loss (reference: ``train/models/decision.py:15-48``).

``z = k(h_opt) . q(h_decide)[owner] / sqrt(dp)``; the loss is per-question CE (or soft-target CE),
averaged within each request variant, then across variants.  Parameter names ``q`` / ``k`` and the
checkpoint prefix ``jev_head.`` are kept so checkpoints and optimizer groups stay compatible.
"""
import math

import torch
import torch.nn as nn
import torch.nn.functional as F


class PointerHead(nn.Module):
    def __init__(self, d, dp=256):
        super().__init__()
        self.q, self.k = nn.Linear(d, dp), nn.Linear(d, dp)
        self.scale = 1.0 / math.sqrt(dp)

    def forward(self, h_decide, h_opts, owner):
        return (self.k(h_opts) * self.q(h_decide)[owner]).sum(-1) * self.scale


def decision_loss(z, batch):
    """(loss, accuracy over hard-label questions)."""
    per_variant = {}
    correct = hard = 0
    for q in batch["questions"]:
        lp = F.log_softmax(z[q["start"]:q["start"] + q["k"]].float(), -1)
        if q.get("target") is not None:
            loss = -(torch.tensor(q["target"], device=lp.device) * lp).sum()
        else:
            loss = -lp[q["label"]]
            correct += int(lp.argmax()) == q["label"]
            hard += 1
        per_variant.setdefault(q["variant"], []).append(loss)
    loss = torch.stack([torch.stack(v).mean() for v in per_variant.values()]).mean()
    return loss, (correct / hard if hard else float("nan"))
