"""Activation offload on the GPU: with every layer recomputed in backward, the checkpointed layer
inputs go to pinned host memory on a side stream and come back for the recompute.  The update must
equal the resident-checkpoint run's (same kernels, same bytes restored), and the pinned pool must
have held the layer inputs."""
import copy

import pytest
import torch


@pytest.mark.gpu
def test_activation_offload_matches_resident_checkpoint():
    from trida_stack_b200.engine import TrainEngine
    from trida_stack_b200.models import BlockDiffusionLM, Decoder, qwen3_config
    from trida_stack_b200.ops._ext import ext

    ext()
    torch.manual_seed(0)
    cfg = qwen3_config(vocab_size=4096, hidden_size=512, intermediate_size=1536, num_layers=3, n_heads=4,
                       n_kv_heads=2, head_dim=128)
    dec = Decoder(cfg, dtype=torch.bfloat16, device="cuda")
    results = []
    for offload in (False, True):
        m = BlockDiffusionLM(copy.deepcopy(dec), mask_id=4095, pad_id=4094, bd_size=32, ar_loss_weight=1.0,
                             activation_checkpoint="layer", activation_offload=offload)
        m.train()
        eng = TrainEngine(m, lr=1e-3, warmup=0, max_steps=10, device=torch.device("cuda"))
        g = torch.Generator().manual_seed(1)
        torch.manual_seed(7)
        losses = []
        for step in range(3):
            ids = torch.randint(0, 4094, (2, 1024), generator=g)
            labels = ids.clone()
            labels[:, :512] = -100
            loss, _, _, _ = eng.train_step([{"input_ids": ids, "labels": labels,
                                             "attention_mask": torch.ones_like(ids)}], step)
            losses.append(float(loss))
        torch.cuda.synchronize()
        results.append((losses, [p.detach().float().clone() for p in m.parameters()], m))
    (l0, p0, _), (l1, p1, m1) = results
    for a, b in zip(l0, l1):
        assert abs(a - b) <= 1e-3 * max(1.0, abs(a)), (l0, l1)
    for a, b in zip(p0, p1):
        assert (a - b).abs().max().item() <= 2e-2 * max(1.0, a.abs().max().item())
    pool = m1._offload_pool
    assert pool is not None
    pool.reclaim()
    # one [rows * 2 views * 1536 tokens, 512] bf16 input per layer went through the pool
    assert pool.nbytes() >= 2 * 2 * 1536 * 512 * 2
