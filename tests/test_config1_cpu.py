"""Benchmark config 1 on CPU (fp32): tiny Qwen3 (2 layers, hidden 128, 4/2 heads x 32, FFN 384,
vocab 1024 incl. <|mask|> = 1023), batch 2 of [prompt 64 | response 64], bd 16, AR weight 1.0,
AdamW lr 1e-4 wd 0.01, 10 steps, seed 0.

The loss curve of this framework's trainer must match the reference trainer's.  The reference's
block-diffusion path hard-wires flex-attention, which has no CPU backward; for this oracle its
BlockMask is replaced by the equivalent dense additive mask under HF eager attention (same rule,
from ``ops.reference.bd_allowed``).  World size 2 (gloo) is checked for rank consistency."""
import os

import pytest
import torch
import torch.multiprocessing as mp

from helpers import import_reference, make_tiny_qwen3, patch_flex_for_cpu, reference_available
from trida_stack_b200.models import BlockDiffusionLM, Decoder, ModelConfig
from trida_stack_b200.ops import reference as R
from trida_stack_b200.parallel.zero import ShardedAdamW

STEPS, LR, WD = 10, 1e-4, 0.01


def batches(n, seed=0):
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(n):
        ids = torch.randint(0, 1022, (2, 128), generator=g)
        labels = ids.clone()
        labels[:, :64] = -100
        out.append((ids, labels, torch.ones_like(ids)))
    return out


def dense_block_mask(seg, opos, rblk, x0_token_causal=False, within_block_causal=False):
    B, T = seg.shape
    z = torch.zeros_like(seg)
    meta = {"seg": seg, "opos": opos, "rblk": rblk, "segid": z, "view": z}
    ok = R.bd_allowed(meta, meta, x0_token_causal, within_block_causal, torch.eye(T, dtype=torch.bool))
    return torch.zeros(B, 1, T, T).masked_fill(~ok[:, None], torch.finfo(torch.float32).min)


def lr_at(it, warmup=50, total=2000, min_ratio=0.1):
    from trida_stack_b200.engine import get_lr
    return get_lr(it, LR, warmup, total, min_ratio)


@pytest.mark.skipif(not reference_available(), reason="reference not installed in baseline/_ref")
def test_config1_loss_curve_matches_reference(tmp_path):
    patch_flex_for_cpu()
    bd = import_reference()
    make_tiny_qwen3(str(tmp_path), seed=0)
    ref = bd.HFBlockDiffusion(model_id=str(tmp_path), bd_size=16, ar_loss_weight=1.0, dtype=torch.float32,
                              response_buckets=None)
    ref._build_block_mask = dense_block_mask
    ref._set_text_attn_impl("eager")
    ref.train()
    cfg = ModelConfig.from_pretrained(str(tmp_path))
    cfg.vocab_size = ref.model.get_input_embeddings().weight.shape[0]
    dec = Decoder(cfg, dtype=torch.float32)
    dec.load_hf_state_dict(ref.model.state_dict())
    ours = BlockDiffusionLM(dec, mask_id=ref.mask_id, bd_size=16, ar_loss_weight=1.0, response_buckets=None)
    ours.train()
    ropt = torch.optim.AdamW([p for p in ref.parameters() if p.requires_grad], lr=LR, betas=(0.9, 0.95),
                             weight_decay=WD)
    oopt = ShardedAdamW(ours.param_groups(), lr=LR, betas=(0.9, 0.95), weight_decay=WD,
                        device=torch.device("cpu"))
    data = batches(STEPS)
    lr_ref, lr_ours = [], []
    for step, (ids, labels, am) in enumerate(data):
        lr = lr_at(step)
        torch.manual_seed(1000 + step)
        lr_l, _ = ref(ids, labels, am)
        lr_l.backward()
        for g in ropt.param_groups:
            g["lr"] = lr
        torch.nn.utils.clip_grad_norm_(ref.parameters(), 1.0)
        ropt.step()
        ropt.zero_grad(set_to_none=True)
        torch.manual_seed(1000 + step)
        lo, _ = ours(ids, labels, am)
        lo.backward()
        for g in oopt.param_groups:
            g["lr"] = lr
        oopt.reduce_gradients()
        oopt.clip_grad_norm_(1.0)
        oopt.step()
        oopt.zero_grad()
        lr_ref.append(lr_l.item())
        lr_ours.append(lo.item())
    for a, b in zip(lr_ours, lr_ref):
        assert abs(a - b) <= 1e-4 * max(1.0, abs(b)), (lr_ours, lr_ref)


def _rank_main(rank, world, path, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.manual_seed(0)
    cfg = ModelConfig.from_pretrained(path)
    cfg.vocab_size = 1024
    dec = Decoder(cfg, dtype=torch.float32)
    torch.manual_seed(0)
    dec.reset_parameters()
    m = BlockDiffusionLM(dec, mask_id=1023, bd_size=16, ar_loss_weight=1.0, response_buckets=None)
    opt = ShardedAdamW(m.param_groups(), lr=LR, betas=(0.9, 0.95), weight_decay=WD, device=torch.device("cpu"))
    losses = []
    for step, (ids, labels, am) in enumerate(batches(4, seed=rank)):
        torch.manual_seed(50 + step + 100 * rank)
        loss, _ = m(ids[:1], labels[:1], am[:1])
        loss.backward()
        for g in opt.param_groups:
            g["lr"] = lr_at(step)
        opt.reduce_gradients()
        opt.clip_grad_norm_(1.0)
        opt.step()
        opt.zero_grad()
        losses.append(loss.item())
    flat = torch.cat([g.flat for g in opt.groups])
    gathered = [torch.zeros_like(flat) for _ in range(world)]
    dist.all_gather(gathered, flat)
    out[rank] = (losses, all(torch.equal(gathered[0], x) for x in gathered))
    dist.destroy_process_group()


def test_config1_world2_gloo_ranks_stay_in_sync(tmp_path):
    make_tiny_qwen3(str(tmp_path), seed=0)
    port = 29600 + os.getpid() % 300
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.spawn(_rank_main, args=(2, str(tmp_path), port, out), nprocs=2, join=True)
        res = dict(out)
    for r in range(2):
        losses, same = res[r]
        assert same, "sharded optimizer left ranks with different parameters"
        assert all(l == l and l < 20 for l in losses)


def _shard_main(rank, world, path, port, out):
    """Full-shard (per-layer weight shards gathered around each layer) against replicated weights
    with sharded optimizer state, on the same data: identical loss curves and final weights."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world)
    res = {}
    for mode in ("zero2", "full", "full_keep", "full_resident"):
        cfg = ModelConfig.from_pretrained(path)
        cfg.vocab_size = 1024
        dec = Decoder(cfg, dtype=torch.float32)
        torch.manual_seed(0)
        dec.reset_parameters()
        m = BlockDiffusionLM(dec, mask_id=1023, bd_size=16, ar_loss_weight=1.0, response_buckets=None)
        full = mode != "zero2"
        opt = ShardedAdamW(m.param_groups(per_layer=full, stream=mode != "full_resident"), lr=LR,
                           betas=(0.9, 0.95), weight_decay=WD,
                           device=torch.device("cpu"), full_shard=full, keep_params=mode == "full_keep")
        m.param_ring = opt.param_ring
        losses = []
        for step, (ids, labels, am) in enumerate(batches(4, seed=rank)):
            torch.manual_seed(50 + step + 100 * rank)
            loss, _ = m(ids[:1], labels[:1], am[:1])
            loss.backward()
            for g in opt.param_groups:
                g["lr"] = lr_at(step)
            opt.reduce_gradients()
            opt.clip_grad_norm_(1.0)
            opt.step()
            opt.zero_grad()
            losses.append(loss.item())
        if opt.param_ring is not None:
            opt.param_ring.materialize()
            res[mode + "_shard_sizes"] = [g.shard_param().numel() for g in opt.groups if g.full_shard]
        res[mode] = (losses, {n: p.detach().clone() for n, p in m.named_parameters()})
    out[rank] = res
    dist.destroy_process_group()


def test_config1_world2_full_shard_matches_replicated(tmp_path):
    make_tiny_qwen3(str(tmp_path), seed=0)
    port = 29300 + os.getpid() % 300
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.spawn(_shard_main, args=(2, str(tmp_path), port, out), nprocs=2, join=True)
        res = dict(out)
    for r in range(2):
        ref_losses, ref_params = res[r]["zero2"]
        for mode in ("full", "full_keep", "full_resident"):
            losses, params = res[r][mode]
            for a, b in zip(losses, ref_losses):
                assert abs(a - b) <= 1e-5 * max(1.0, abs(b)), (mode, losses, ref_losses)
            for n, p in params.items():
                torch.testing.assert_close(p, ref_params[n], rtol=1e-5, atol=1e-6, msg=f"{mode}: {n}")
        assert all(s > 0 for s in res[r]["full_shard_sizes"])   # every rank holds part of each layer
