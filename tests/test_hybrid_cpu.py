"""Native Qwen3.5 hybrid decoder vs transformers' implementation, and the two-stream objective."""
import math

import pytest
import torch

from trida_stack_b200.models import Decoder, ModelConfig
from trida_stack_b200.models.hybrid import HybridBlockDiffusionLM
from trida_stack_b200.ops import gdn_reference as G


def tiny_qwen35(path=None, seed=0):
    from transformers.models.qwen3_5 import Qwen3_5ForCausalLM, Qwen3_5TextConfig
    torch.manual_seed(seed)
    cfg = Qwen3_5TextConfig(vocab_size=300, hidden_size=64, intermediate_size=128, num_hidden_layers=4,
                            num_attention_heads=2, num_key_value_heads=1, head_dim=32,
                            linear_num_key_heads=2, linear_num_value_heads=4, linear_key_head_dim=16,
                            linear_value_head_dim=16, linear_conv_kernel_dim=4, max_position_embeddings=2048,
                            layer_types=["linear_attention"] * 3 + ["full_attention"], tie_word_embeddings=True)
    m = Qwen3_5ForCausalLM(cfg).float().eval()
    with torch.no_grad():   # non-trivial norm / gate parameters so the offsets are exercised
        for n, p in m.named_parameters():
            if p.dim() == 1:
                p.add_(0.1 * torch.randn_like(p))
    if path is not None:
        m.save_pretrained(path)
    return m


def native_from(hf):
    cfg = ModelConfig.from_hf_dict(hf.config.to_dict())
    dec = Decoder(cfg, dtype=torch.float32)
    dec.load_hf_state_dict(hf.state_dict())
    return dec


def test_native_hybrid_matches_transformers_causal_logits():
    hf = tiny_qwen35()
    dec = native_from(hf)
    m = HybridBlockDiffusionLM(dec, mask_id=299, ar_only=True)
    ids = torch.randint(0, 299, (2, 40))
    with torch.no_grad():
        ref = hf(ids).logits
        actx = m._causal_rows(ids, None)
        h = dec(dec.embed_tokens(ids), actx)
        ours = (h @ dec.lm_weight.t()).view(2, 40, -1)
    torch.testing.assert_close(ours, ref, rtol=2e-4, atol=2e-4)


def test_hf_state_dict_round_trip_keeps_zero_centred_norms():
    hf = tiny_qwen35()
    dec = native_from(hf)
    sd = dec.hf_state_dict()
    ref = hf.state_dict()
    for k, v in sd.items():
        torch.testing.assert_close(v, ref[k].float(), msg=k)


def test_packed_causal_rows_isolate_documents():
    hf = tiny_qwen35()
    dec = native_from(hf)
    m = HybridBlockDiffusionLM(dec, mask_id=299, ar_only=True)
    ids = torch.randint(0, 299, (1, 48))
    seg = torch.tensor([[0] * 20 + [1] * 28])
    with torch.no_grad():
        h = dec(dec.embed_tokens(ids), m._causal_rows(ids, seg)).view(48, -1)
        h2 = dec(dec.embed_tokens(ids[:, 20:]), m._causal_rows(ids[:, 20:], None)).view(28, -1)
    torch.testing.assert_close(h[20:], h2, rtol=1e-4, atol=1e-4)


def test_two_stream_recurrence_semantics():
    """Noisy block k restarts from the clean state at the end of block k-1 and, in bidirectional
    mode, every token reads the block-end state; with identical streams and token-causal noisy
    read-out the noisy output equals the clean output."""
    torch.manual_seed(0)
    B, L, H, dk, dv, bd = 1, 16, 2, 8, 8, 4
    q = G.l2norm(torch.randn(B, 2 * L, H, dk))
    k = G.l2norm(torch.randn(B, 2 * L, H, dk))
    v = torch.randn(B, 2 * L, H, dv)
    g = -torch.rand(B, 2 * L, H)
    beta = torch.rand(B, 2 * L, H)
    same = [torch.cat([x[:, :L], x[:, :L]], 1) for x in (q, k, v, g, beta)]
    o = G.gdn_two_stream(*same, L=L, V=1, bd=bd, causal_noisy=True)
    torch.testing.assert_close(o[:, L:], o[:, :L], rtol=1e-5, atol=1e-5)
    ob = G.gdn_two_stream(q, k, v, g, beta, L=L, V=1, bd=bd, causal_noisy=False)
    oc = G.gdn_two_stream(q, k, v, g, beta, L=L, V=1, bd=bd, causal_noisy=True)
    # the last token of every noisy block reads the same state in both modes
    torch.testing.assert_close(ob[:, L + bd - 1::bd], oc[:, L + bd - 1::bd], rtol=1e-5, atol=1e-5)


def test_two_stream_objective_and_decision_backward():
    hf = tiny_qwen35()
    dec = native_from(hf)
    m = HybridBlockDiffusionLM(dec, mask_id=299, bd_size=8, ar_loss_weight=1.0, decision_head_dim=16,
                               pos_decay_gamma=4.0)
    ids = torch.randint(0, 298, (2, 32))
    labels = ids.clone()
    labels[:, :12] = -100
    torch.manual_seed(3)
    loss, logs = m(ids, labels, torch.ones_like(ids))
    loss.backward()
    assert math.isfinite(loss.item()) and logs["ntok"] == 2 * 20
    assert all(p.grad is not None for n, p in m.named_parameters() if not n.startswith("jev_head"))
    from trida_stack_b200.data.decision import pack_decision
    rows = [{"ids": list(range(5, 25)), "decide": 19, "opts": [8, 12, 16], "label": 1},
            {"ids": list(range(30, 45)), "decide": 14, "opts": [5, 9], "label": 0}]
    batch = pack_decision([rows], None)
    dl, dlog = m(None, None, None, decision=batch)
    dl.backward()
    assert m.jev_head.q.weight.grad is not None and math.isfinite(dl.item())


def test_block_bidirectional_reference_scan():
    """Single-stream block-bidirectional recurrence: one-token blocks reduce to the causal scan, and a
    block's read-out depends on later tokens of the same block but never on later blocks."""
    torch.manual_seed(0)
    B, T, H, d = 2, 12, 2, 8
    q, k = G.l2norm(torch.randn(B, T, H, d)), G.l2norm(torch.randn(B, T, H, d))
    v = torch.randn(B, T, H, d)
    g = -torch.rand(B, T, H)
    beta = torch.rand(B, T, H)
    o1, S1 = G.gdn_block_bidirectional(q, k, v, g, beta, torch.arange(T).expand(B, -1))
    oc, _ = G.gdn_causal(q, k, v, g, beta)
    torch.testing.assert_close(o1, oc, rtol=1e-5, atol=1e-5)
    blocks = (torch.arange(T) // 4).expand(B, -1)
    o4, S4 = G.gdn_block_bidirectional(q, k, v, g, beta, blocks)
    torch.testing.assert_close(S4, S1, rtol=1e-5, atol=1e-5)       # the exit state stays causal
    v2 = v.clone()
    v2[:, 6] += 1.0                                                # a token in block 1
    o5, _ = G.gdn_block_bidirectional(q, k, v2, g, beta, blocks)
    assert torch.allclose(o5[:, :4], o4[:, :4])                    # earlier block untouched
    assert not torch.allclose(o5[:, 4], o4[:, 4])                  # same block: read-out sees the future


def test_causal_mode_matches_reference(tmp_path):
    """``linear_block_mode="causal"``: the dense [S | x_t | x_0] row with the block-diffusion mask on
    the full-attention layers and region A / region B scanned as separate causal documents by the
    linear layers -- the same loss as the reference's HFBlockDiffusionHybrid (torch fallbacks, dense
    additive mask in place of flex-attention) on the same noise draws."""
    from helpers import import_reference, make_tokenizer, patch_flex_for_cpu, reference_available
    if not reference_available():
        pytest.skip("reference not installed in baseline/_ref")
    patch_flex_for_cpu()
    import_reference()
    from test_config1_cpu import dense_block_mask
    from train.models.hybrid import HFBlockDiffusionHybrid
    tiny_qwen35(str(tmp_path))
    make_tokenizer(str(tmp_path), 300)
    ref = HFBlockDiffusionHybrid(model_id=str(tmp_path), bd_size=8, ar_loss_weight=1.0, dtype=torch.float32,
                                 response_buckets=None, linear_block_mode="causal", attn_impl="eager",
                                 require_kernels=False)
    ref._build_block_mask = dense_block_mask
    ref.train()
    cfg = ModelConfig.from_pretrained(str(tmp_path))
    cfg.vocab_size = ref.model.get_input_embeddings().weight.shape[0]
    dec = Decoder(cfg, dtype=torch.float32)
    dec.load_hf_state_dict(ref.model.state_dict())
    ours = HybridBlockDiffusionLM(dec, mask_id=ref.mask_id, bd_size=8, ar_loss_weight=1.0, response_buckets=None,
                                  linear_block_mode="causal")
    ours.train()
    g = torch.Generator().manual_seed(5)
    ids = torch.randint(0, 298, (2, 48), generator=g)
    labels = ids.clone()
    labels[:, :24] = -100
    am = torch.ones_like(ids)
    torch.manual_seed(11)
    lr_, _ = ref(ids, labels, am)
    torch.manual_seed(11)
    lo, _ = ours(ids, labels, am)
    assert abs(lo.item() - lr_.item()) <= 2e-4 * max(1.0, abs(lr_.item())), (lo.item(), lr_.item())


def test_pointer_rows_in_two_stream_forward():
    """Pointer-head questions on some rows of a two-stream batch: the head's loss joins the row's
    block-diffusion loss in the same forward, and its gradient reaches the head and the stack."""
    hf = tiny_qwen35()
    m = HybridBlockDiffusionLM(native_from(hf), mask_id=299, bd_size=8, ar_loss_weight=1.0, decision_head_dim=16)
    ids = torch.randint(0, 298, (2, 32))
    labels = ids.clone()
    labels[:, :12] = -100
    L = 32
    pointer = {"decide": torch.tensor([1 * L + 30]), "opts": torch.tensor([1 * L + 14, 1 * L + 20, 1 * L + 26]),
               "owner": torch.tensor([0, 0, 0]), "weight": 0.5,
               "questions": [{"start": 0, "k": 3, "label": 2, "variant": 0}]}
    torch.manual_seed(4)
    base, _ = m(ids, labels, torch.ones_like(ids))
    torch.manual_seed(4)
    loss, logs = m(ids, labels, torch.ones_like(ids), pointer=pointer)
    loss.backward()
    torch.testing.assert_close(loss.detach(), base.detach() + 0.5 * logs["decision_loss"])
    assert m.jev_head.q.weight.grad is not None and m.jev_head.k.weight.grad.abs().sum() > 0
