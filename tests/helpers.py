"""Shared test fixtures: tiny HF checkpoints and the reference trainer (when installed)."""
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")


def reference_available():
    return os.path.isdir(os.path.join(REF, "train"))


def import_reference():
    if REF not in sys.path:
        sys.path.insert(0, REF)
    import train.models.block_diffusion as bd  # noqa: E402
    return bd


def make_tokenizer(path, n_tokens):
    """Word-level fast tokenizer with ``n_tokens`` entries (ids 0..n-1) and <|endoftext|> as pad."""
    from tokenizers import Tokenizer, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast
    vocab = {f"t{i}": i for i in range(n_tokens - 1)}
    vocab["<|endoftext|>"] = n_tokens - 1
    tok = Tokenizer(models.WordLevel(vocab=vocab, unk_token="<|endoftext|>"))
    tok.pre_tokenizer = pre_tokenizers.WhitespaceSplit()
    fast = PreTrainedTokenizerFast(tokenizer_object=tok, eos_token="<|endoftext|>", pad_token="<|endoftext|>")
    fast.save_pretrained(path)
    return fast


def make_tiny_qwen3(path, vocab=1023, hidden=128, ffn=384, layers=2, heads=4, kv=2, head_dim=32, seed=0,
                    tie=True, dtype=torch.float32):
    """Random-init HF Qwen3 checkpoint + tokenizer in ``path`` (config 1 of the benchmark spec)."""
    from transformers import Qwen3Config, Qwen3ForCausalLM
    torch.manual_seed(seed)
    cfg = Qwen3Config(vocab_size=vocab, hidden_size=hidden, intermediate_size=ffn, num_hidden_layers=layers,
                      num_attention_heads=heads, num_key_value_heads=kv, head_dim=head_dim, rms_norm_eps=1e-6,
                      rope_parameters={"rope_theta": 1e6, "rope_type": "default"}, tie_word_embeddings=tie,
                      max_position_embeddings=4096)
    model = Qwen3ForCausalLM(cfg).to(dtype)
    model.save_pretrained(path)
    make_tokenizer(path, vocab)
    return model


def patch_flex_for_cpu():
    """The reference builds its flex BlockMask with ``_compile=True``, which needs a working
    C++ inductor toolchain; for CPU forward-only checks build it eagerly instead."""
    import torch.nn.attention.flex_attention as fa
    orig = fa.create_block_mask
    if getattr(orig, "_trida_patched", False):
        return

    def eager(*a, **k):
        k["_compile"] = False
        return orig(*a, **k)
    eager._trida_patched = True
    fa.create_block_mask = eager
    # transformers wraps flex_attention in torch.compile; call the eager kernel instead
    import transformers.integrations.flex_attention as hf_fa

    def eager_flex(query, key, value, training=False, **kwargs):
        return fa.flex_attention(query, key, value, **kwargs)
    hf_fa.compile_friendly_flex_attention = eager_flex


def write_json(path, obj):
    with open(path, "w") as f:
        json.dump(obj, f)
