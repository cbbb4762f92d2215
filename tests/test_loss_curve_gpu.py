"""Loss curve of this framework's B200 trainer against the reference trainer on the same GPU.

One random HF Qwen3 initialisation (4 layers, hidden 512, 4 Q / 2 KV heads x 128, FFN 1536, vocab
2048 including <|mask|>) is loaded into the reference's ``HFBlockDiffusion`` (flex-attention block
mask, ``train/models/block_diffusion.py``) and into this package's ``BlockDiffusionLM`` running on
its sm_100a kernels through ``TrainEngine`` (the per-step API of ``train.py``).  Both train 10
optimizer steps on the same batches ([prompt 128 | response 128] x 2 rows, block 32, AR weight 1.0)
with the same noising seed per step (both draw the per-block rates and token draws with
``torch.rand`` on the device in the same order), bf16 weights, AdamW (beta2 0.95, clip 1.0) and
the reference's learning-rate schedule (``train/optimizer.py:8-15``).  Tokens come from the first
100 ids so the loss has something to learn; the two curves must agree to bf16 tolerance at every
step and both must fall.
"""
import pytest
import torch

from helpers import import_reference, make_tiny_qwen3, reference_available

STEPS, LR, WARMUP, WD = 10, 1e-3, 2, 0.01
PROMPT, RESP, BD, ROWS = 128, 128, 32, 2


def _batches(n, seed=0):
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(n):
        ids = torch.randint(0, 100, (ROWS, PROMPT + RESP), generator=g)
        labels = ids.clone()
        labels[:, :PROMPT] = -100
        out.append({"input_ids": ids, "labels": labels, "attention_mask": torch.ones_like(ids)})
    return out


@pytest.mark.gpu
@pytest.mark.skipif(not reference_available(), reason="reference not installed in baseline/_ref")
def test_loss_curve_matches_reference_on_gpu(tmp_path):
    from trida_stack_b200.engine import TrainEngine, get_lr
    from trida_stack_b200.models import BlockDiffusionLM, Decoder, ModelConfig
    from trida_stack_b200.ops._ext import ext

    ext()   # the CUDA path must be the one under test
    bd = import_reference()
    path = str(tmp_path)
    make_tiny_qwen3(path, vocab=2047, hidden=512, ffn=1536, layers=4, heads=4, kv=2, head_dim=128, seed=0)
    dev = torch.device("cuda")
    torch.manual_seed(0)
    ref = bd.HFBlockDiffusion(model_id=path, bd_size=BD, ar_loss_weight=1.0, dtype=torch.bfloat16,
                              response_buckets=None).to(dev)
    ref.train()
    cfg = ModelConfig.from_pretrained(path)
    cfg.vocab_size = ref.model.get_input_embeddings().weight.shape[0]
    assert cfg.vocab_size == 2048
    dec = Decoder(cfg, dtype=torch.bfloat16, device="cuda")
    dec.load_hf_state_dict({k: v.detach() for k, v in ref.model.state_dict().items()})
    ours = BlockDiffusionLM(dec, mask_id=ref.mask_id, bd_size=BD, ar_loss_weight=1.0, response_buckets=None)
    ours.train()
    engine = TrainEngine(ours, lr=LR, betas=(0.9, 0.95), weight_decay=WD, grad_clip=1.0, warmup=WARMUP,
                         max_steps=100, lr_min_ratio=0.1, device=dev)
    ropt = torch.optim.AdamW([p for p in ref.parameters() if p.requires_grad], lr=LR, betas=(0.9, 0.95),
                             weight_decay=WD)
    ref_losses, our_losses = [], []
    for step, b in enumerate(_batches(STEPS)):
        torch.manual_seed(1000 + step)
        rl, _ = ref(b["input_ids"].to(dev), b["labels"].to(dev), b["attention_mask"].to(dev))
        rl.backward()
        for g in ropt.param_groups:
            g["lr"] = get_lr(step, LR, WARMUP, 100, 0.1)
        torch.nn.utils.clip_grad_norm_(ref.parameters(), 1.0)
        ropt.step()
        ropt.zero_grad(set_to_none=True)
        torch.manual_seed(1000 + step)
        ol, _, _, _ = engine.train_step([b], step)
        ref_losses.append(float(rl.item()))
        our_losses.append(float(ol.item()))
    for a, r in zip(our_losses, ref_losses):
        assert abs(a - r) <= 2e-2 * max(1.0, abs(r)), (our_losses, ref_losses)
    assert ref_losses[-1] < ref_losses[0] - 0.5, ref_losses
    assert our_losses[-1] < our_losses[0] - 0.5, our_losses
