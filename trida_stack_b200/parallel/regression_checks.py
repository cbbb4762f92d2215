"""Data-parallel regression checks for vision-language training (run on two or more ranks).

The reference keeps two 2-GPU FSDP checks for failure modes of sharded VL training
(``train/tools/vlm_fsdp_check.py``, ``train/tools/decision_fsdp_check.py``): a rank with an image
row and a rank with a text-only row must stay in lockstep (a rank that skips the vision tower's
collectives deadlocks the other), and in joint SFT + decision training the vision projector's
gradient, produced only by the SFT micro-step, must still reach the optimizer.  Both are checked
here on this package's engine (sharded flat buffers, fused or NCCL collectives):

``mixed``     rank 0 trains on image rows, the other ranks on text-only rows, ``--steps`` optimizer
              steps.  Passes when no collective times out, the projector moved, and every rank
              holds the same parameters after every step.
``decision``  every optimizer step is one SFT micro-step (rank 0 an image row, the others text-only)
              plus one typed-decision micro-step; passes when the projector moves every step on
              every rank and the ranks agree on the parameters.

    torchrun --nproc-per-node 2 -m trida_stack_b200.parallel.regression_checks mixed --ckpt <vl ckpt>
    torchrun --nproc-per-node 2 -m trida_stack_b200.parallel.regression_checks decision --tiny

``--tiny`` builds a small random VL hybrid in memory (no checkpoint); ``--cpu`` runs the ranks on
gloo.  Each rank prints one line per step; rank 0 prints PASS / FAIL and the exit code is 0 / 1.
"""
import argparse
import datetime
import os
import random
import sys
import zlib

import torch
import torch.distributed as dist

IMG = 290
BD = 8
REQUEST = {"state": "Customer writes: I was charged twice for my October invoice and want the duplicate refunded.",
           "questions": {
               "team": {"type": "choice", "instructions": "Which team should handle this?",
                        "criteria": {"billing": "payments and refunds", "tech": "product bugs", "sales": "new purchases"},
                        "label": "billing"},
               "urgent": {"type": "noul", "instructions": "Is this urgent?", "label": False}}}


def tiny_vl_decoder(seed=0):
    """A small random VL hybrid (3 gated-delta + 1 full-attention layer, 2-block ViT)."""
    from ..models import Decoder, ModelConfig
    cfg = ModelConfig.from_hf_dict({
        "model_type": "qwen3_5", "image_token_id": IMG, "tie_word_embeddings": True,
        "text_config": {"model_type": "qwen3_5_text", "vocab_size": 300, "hidden_size": 64, "intermediate_size": 128,
                        "num_hidden_layers": 4, "num_attention_heads": 2, "num_key_value_heads": 1, "head_dim": 32,
                        "linear_num_key_heads": 2, "linear_num_value_heads": 4, "linear_key_head_dim": 16,
                        "linear_value_head_dim": 16, "linear_conv_kernel_dim": 4,
                        "layer_types": ["linear_attention"] * 3 + ["full_attention"],
                        "rope_parameters": {"rope_theta": 1e4, "partial_rotary_factor": 0.5,
                                            "mrope_section": [3, 3, 2]}},
        "vision_config": {"depth": 2, "hidden_size": 32, "intermediate_size": 48, "num_heads": 2, "in_channels": 3,
                          "patch_size": 4, "temporal_patch_size": 2, "spatial_merge_size": 2,
                          "out_hidden_size": 64, "num_position_embeddings": 16,
                          "hidden_act": "gelu_pytorch_tanh"}})
    torch.manual_seed(seed)
    return Decoder(cfg, dtype=torch.float32)


def _doc(rng, with_image, vocab, img_id, patch_dim):
    """One block-aligned training document: text, optionally one image, a 3-token response."""
    from ..data import images as I
    from ..data import sft
    ids = [rng.randint(0, vocab - 20) for _ in range(rng.randint(4, 12))]
    grids = None
    if with_image:
        gh, gw = 2 * rng.randint(1, 3), 2 * rng.randint(1, 3)
        grids = torch.tensor([[1, gh, gw]])
        ids += [img_id] * (gh * gw // 4)
    ids += [rng.randint(0, vocab - 20) for _ in range(rng.randint(4, 12))]
    ids = torch.tensor(ids)
    labels = torch.full_like(ids, -100)
    labels[-3:] = ids[-3:]
    s = {"input_ids": ids, "labels": labels, "resp_block": torch.where(labels != -100, 0, -1),
         "turn_id": torch.where(labels != -100, 0, -1)}
    if with_image:
        s.update(pixel_values=torch.randn(int(grids.prod(-1).sum()), patch_dim), image_grid_thw=grids,
                 mrope_pos=I.mrope_position_ids(ids, grids, img_id))
    return sft.block_align_doc(s, BD, 0)


def sft_rows(with_image, seed, n, dec):
    from ..data import sft
    vc = dec.cfg.vision
    patch_dim = vc["in_channels"] * vc["temporal_patch_size"] * vc["patch_size"] ** 2
    rng = random.Random(seed)
    return [sft.pack_rows_multiturn([[_doc(rng, with_image, dec.cfg.vocab_size, dec.cfg.image_token_id, patch_dim)]],
                                    0, BD, None, 4096) for _ in range(n)]


def decision_batch(tok, dev):
    from ..data.decision import encode_rows, materialize, pack_decision, training_context
    jb = pack_decision([encode_rows(tok, materialize(REQUEST), **training_context())], tok)
    return {k: (v.to(dev) if torch.is_tensor(v) else v) for k, v in jb.items()}


class _WordTok:
    """Whitespace tokenizer over the tiny model's vocabulary with the decision control tokens."""

    def __init__(self, vocab):
        from ..data.decision import SPECIAL
        self.special = {t: vocab - 1 - i for i, t in enumerate(SPECIAL)}
        self.vocab = vocab
        self.pad_token_id = 0
        self.unk_token_id = None

    def convert_tokens_to_ids(self, t):
        return self.special.get(t)

    def __call__(self, text, add_special_tokens=False):
        class _E:
            pass
        e = _E()
        e.input_ids = [zlib.crc32(w.encode()) % (self.vocab - 40) for w in text.split()]
        return e


def _params_digest(model):
    v = torch.stack([p.detach().double().sum() for p in model.parameters()] +
                    [p.detach().double().abs().sum() for p in model.parameters()])
    return v


def run(check, steps, dev, ckpt=None):
    from ..engine import TrainEngine
    from ..models.hybrid import HybridBlockDiffusionLM
    rank, world = dist.get_rank(), dist.get_world_size()
    if ckpt:
        from ..models.build import load_decoder, load_tokenizer
        tok = load_tokenizer(ckpt)
        dec, _ = load_decoder(ckpt, dev, torch.bfloat16 if dev.type == "cuda" else torch.float32, tokenizer=tok)
    else:
        dec = tiny_vl_decoder().to(dev)
        tok = _WordTok(dec.cfg.vocab_size)
    if not dec.cfg.is_vl:
        raise SystemExit("the regression checks need a vision-language checkpoint")
    m = HybridBlockDiffusionLM(dec, mask_id=dec.cfg.vocab_size - 6, bd_size=BD, ar_loss_weight=1.0,
                               decision_head_dim=32 if check == "decision" else 0)
    if check == "decision":
        m.jev_head.to(dev)
    m.train()
    eng = TrainEngine(m, lr=1e-3, warmup=0, max_steps=100, device=dev, projector_lr_scale=1.0,
                      decision_head_lr_scale=10.0, comm="nccl" if dev.type != "cuda" else "fused")
    rows = sft_rows(rank == 0, seed=rank, n=steps, dec=dec)
    jb = decision_batch(tok, dev) if check == "decision" else None
    proj = list(dec.visual.merger.parameters())
    ok = True
    for step in range(steps):
        before = [p.detach().clone() for p in proj]
        torch.manual_seed(step)
        loss, _ = eng.micro_step(rows[step], scale=1.0)
        jloss = None
        if jb is not None:
            jloss, _ = m(None, None, None, decision=jb)
            jloss.backward()
        eng.optimizer_step(step)
        moved = sum(float((p.detach() - q).abs().sum()) for p, q in zip(proj, before))
        digest = _params_digest(m)
        gathered = [torch.zeros_like(digest) for _ in range(world)]
        dist.all_gather(gathered, digest)
        same = all(torch.allclose(g, gathered[0], rtol=1e-9, atol=0) for g in gathered)
        flag = torch.tensor([1.0 if (moved > 0 and same) else 0.0], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        ok &= bool(flag.item() > 0)
        kind = "images" if "pixel_values" in rows[step] else "text-only"
        print(f"rank {rank} step {step}: {kind} row, loss {float(loss.detach()):.4f}"
              + (f" decision {float(jloss.detach()):.4f}" if jloss is not None else "")
              + f" | projector moved {moved:.3e} | ranks agree {same}", flush=True)
    dist.barrier()
    return ok


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("check", choices=["mixed", "decision"])
    ap.add_argument("--ckpt", default=None, help="vision-language checkpoint directory")
    ap.add_argument("--tiny", action="store_true", help="a small random VL model built in memory")
    ap.add_argument("--steps", type=int, default=4)
    ap.add_argument("--cpu", action="store_true", help="gloo ranks on the host")
    a = ap.parse_args(argv)
    if not a.tiny and not a.ckpt:
        ap.error("give --ckpt or --tiny")
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if a.cpu or not torch.cuda.is_available():
        dev = torch.device("cpu")
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    else:
        dev = torch.device("cuda", local)
        torch.cuda.set_device(dev)
        # a regression fails fast instead of waiting out NCCL's default timeout
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        ok = run(a.check, a.steps, dev, a.ckpt)
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()
    if int(os.environ.get("RANK", "0")) == 0:
        print(f"{a.check} check: " + ("PASS" if ok else "FAIL"), flush=True)
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
