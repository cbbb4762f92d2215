"""SFT data pipeline (rendering, labels, packing invariants) and HF checkpoint round trips."""
import json
import os

import pytest
import torch

from helpers import make_tiny_qwen3
from trida_stack_b200.data import sft

TEMPLATE = ("{% for m in messages %}<|im_start|> {{ m['role'] }} {{ m['content'] }} <|im_end|> {% endfor %}"
            "{% if add_generation_prompt %}<|im_start|> assistant {% endif %}")


def chat_tokenizer(tmp_path, n=300):
    from tokenizers import Tokenizer, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast
    words = ["<|endoftext|>", "<|im_start|>", "<|im_end|>", "user", "assistant", "system", "tool"]
    vocab = {w: i for i, w in enumerate(words)}
    for i in range(n - len(words)):
        vocab[f"w{i}"] = len(vocab)
    tok = Tokenizer(models.WordLevel(vocab=vocab, unk_token="<|endoftext|>"))
    tok.pre_tokenizer = pre_tokenizers.WhitespaceSplit()
    fast = PreTrainedTokenizerFast(tokenizer_object=tok, eos_token="<|endoftext|>", pad_token="<|endoftext|>")
    fast.chat_template = TEMPLATE
    return fast


def conv(turns):
    msgs = [{"role": "system", "content": "w1 w2"}]
    for i, (u, a) in enumerate(turns):
        msgs += [{"role": "user", "content": u}, {"role": "assistant", "content": a}]
    return {"messages": msgs}


def test_build_sample_supervises_last_turn_only(tmp_path):
    tok = chat_tokenizer(tmp_path)
    s = sft.build_sample(tok, conv([("w3 w4", "w5 w6 w7"), ("w8", "w9 w10")]))
    ids, lab = s["input_ids"], s["labels"]
    sup = ids[lab != -100].tolist()
    assert tok.decode(sup).split() == ["w9", "w10", "<|im_end|>"]
    span = (lab != -100).nonzero().squeeze(1)
    assert span.numel() == span[-1] - span[0] + 1


def test_multiturn_labels_blocks_and_turns(tmp_path):
    tok = chat_tokenizer(tmp_path)
    s = sft.build_sample_multiturn(tok, conv([("w3", " ".join(f"w{i}" for i in range(20, 40))), ("w8", "w9")]), 8)
    assert set(s["turn_id"][s["labels"] != -100].tolist()) == {0, 1}
    rb = s["resp_block"][s["labels"] != -100]
    assert rb.min() == 0 and (rb[1:] >= rb[:-1]).all()
    assert ((s["resp_block"] >= 0) == (s["labels"] != -100)).all()


def test_pack_rows_isolation_and_positions(tmp_path):
    tok = chat_tokenizer(tmp_path)
    samples = [sft.build_sample(tok, conv([(f"w{3 + i}", f"w{50 + i} w{60 + i}")])) for i in range(5)]
    rows = sft.greedy_pack(samples, max_length=64)
    batch = sft.pack_rows_to_batch(rows, 0, None, 64)
    for b in range(batch["input_ids"].shape[0]):
        seg = batch["seg_id"][b]
        for k in seg.unique().tolist():
            if k < 0:
                continue
            m = seg == k
            assert batch["labels"][b][m][0] == -100
            rp = batch["resp_pos"][b][m]
            assert rp[rp >= 0].tolist() == list(range(int((rp >= 0).sum())))
    assert all(sum(sft.forward_cost(s) for s in r) <= 64 or len(r) == 1 for r in rows)


def test_stream_first_fit_properties():
    docs = [{"input_ids": torch.zeros(n, dtype=torch.long)} for n in [5, 9, 3, 7, 2, 8, 6, 1, 4]]
    rows = list(sft.stream_first_fit(iter(docs), max_length=10, buffer_size=3))
    flat = sorted(id(d) for r in rows for d in r)
    assert flat == sorted(id(d) for d in docs)              # every doc exactly once
    assert all(sum(d["input_ids"].shape[0] for d in r) <= 10 for r in rows)
    heads = [r[0] for r in rows]
    assert heads[0] is docs[0]
    with pytest.raises(ValueError):
        list(sft.stream_first_fit(iter([{"input_ids": torch.zeros(11)}]), max_length=10))
    with pytest.raises(ValueError):
        list(sft.stream_first_fit(iter(docs), max_length=10, buffer_size=0))


def test_block_align_and_multiturn_pack(tmp_path):
    tok = chat_tokenizer(tmp_path)
    docs = [sft.block_align_doc(sft.build_sample_multiturn(tok, conv([("w3", "w4 w5 w6")]), 8), 8, 0)
            for _ in range(3)]
    assert all(d["input_ids"].shape[0] % 8 == 0 for d in docs)
    batch = sft.pack_rows_multiturn([docs], 0, 8, None, 256)
    starts = [int(i) for i in torch.nonzero(batch["seg_id"][0][1:] != batch["seg_id"][0][:-1]).squeeze(1) + 1]
    assert all(s % 8 == 0 for s in starts)


def test_jsonl_stream_shards_disjointly(tmp_path):
    p = tmp_path / "d.jsonl"
    with open(p, "w") as f:
        for i in range(40):
            f.write(json.dumps({"messages": [{"role": "user", "content": f"w{i}"},
                                             {"role": "assistant", "content": "w1"}]}) + "\n")
        f.write("not json\n")
    seen = []
    for r in range(2):
        ds = sft.JsonlChatDataset([str(p)], rank=r, world=2, seed=0, shuffle_buffer=4)
        seen.append([x["messages"][0]["content"] for x in ds])
    assert len(seen[0]) == len(seen[1]) == 20
    assert not set(seen[0]) & set(seen[1])


def test_hf_checkpoint_round_trip(tmp_path):
    """save_hf writes a transformers-loadable checkpoint whose logits equal the native decoder's."""
    from types import SimpleNamespace

    from transformers import AutoModelForCausalLM

    from trida_stack_b200 import checkpoint
    from trida_stack_b200.models import BlockDiffusionLM, Decoder, ModelConfig
    src = tmp_path / "src"
    make_tiny_qwen3(str(src))
    cfg = ModelConfig.from_pretrained(str(src))
    dec = Decoder(cfg, dtype=torch.float32)
    torch.manual_seed(1)
    dec.reset_parameters()
    m = BlockDiffusionLM(dec, mask_id=cfg.vocab_size - 1, bd_size=16, ar_loss_weight=0.5)
    args = SimpleNamespace(save_dir=str(tmp_path / "out"), save_optim_state=False)
    checkpoint.save_hf(m, args, "step_3")
    out = tmp_path / "out" / "step_3"
    side = json.load(open(out / "block_diffusion.json"))
    assert side == {"bd_size": 16, "mask_id": cfg.vocab_size - 1, "ar_loss_weight": 0.5}
    hf = AutoModelForCausalLM.from_pretrained(str(out), dtype=torch.float32)
    ids = torch.randint(0, cfg.vocab_size, (1, 20))
    ref_logits = hf(ids).logits.float()
    from trida_stack_b200.models.block_diffusion import BlockDiffusionLM as _M  # noqa: F401
    from trida_stack_b200.ops import reference as R
    z = torch.zeros(1, 20, dtype=torch.int32)
    pos = torch.arange(20)[None]
    m2 = BlockDiffusionLM(Decoder(ModelConfig.from_pretrained(str(out)), dtype=torch.float32), mask_id=0)
    m2.decoder.load_hf_state_dict(checkpoint.read_hf_weights(str(out)))
    actx = m2.make_actx(torch.full((1, 20), R.SHARED), pos, z, z, z, pos, True)
    h = m2.decoder(m2.decoder.embed_tokens(ids), actx)
    ours = h @ m2.decoder.lm_weight.t()
    torch.testing.assert_close(ours, ref_logits[0], rtol=2e-2, atol=2e-2)


def test_sharded_optimizer_state_round_trip(tmp_path):
    from types import SimpleNamespace

    import torch.distributed as dist

    from trida_stack_b200 import checkpoint
    from trida_stack_b200.parallel.zero import ShardedAdamW
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT="29711", RANK="0", WORLD_SIZE="1")
    if not dist.is_initialized():
        dist.init_process_group("gloo", rank=0, world_size=1)
    p = torch.nn.Parameter(torch.randn(100))
    opt = ShardedAdamW([{"params": [p]}], lr=1e-2, device=torch.device("cpu"))
    p.main_grad.copy_(torch.randn(100))
    opt.clip_grad_norm_(1.0)
    opt.step()
    args = SimpleNamespace(save_dir=str(tmp_path), save_optim_state=True)
    checkpoint.save_train_state(None, opt, 7, args, "step_7")
    p2 = torch.nn.Parameter(p.detach().clone())
    opt2 = ShardedAdamW([{"params": [p2]}], lr=1e-2, device=torch.device("cpu"))
    step = checkpoint.load_train_state(None, opt2, str(tmp_path / "step_7"))
    assert step == 7 and opt2.step_count == 1
    torch.testing.assert_close(opt2.groups[0].m, opt.groups[0].m)
    torch.testing.assert_close(opt2.groups[0].v, opt.groups[0].v)


def test_compat_names_and_decision_export(tmp_path):
    import warnings

    import torch

    from test_hybrid_cpu import tiny_qwen35
    from trida_stack_b200.export import export
    with warnings.catch_warnings():
        warnings.simplefilter("ignore", DeprecationWarning)
        from trida_stack_b200 import hf_block_diffusion, hf_block_diffusion_hybrid, jev
    assert hf_block_diffusion.HFBlockDiffusion.__name__ == "BlockDiffusionLM"
    assert hf_block_diffusion_hybrid.HFBlockDiffusionHybrid.__name__ == "HybridBlockDiffusionLM"
    assert callable(jev.jev_loss)
    ck = tmp_path / "ck"
    tiny_qwen35(str(ck))
    torch.save({"head": {"q.weight": torch.zeros(8, 64), "q.bias": torch.zeros(8),
                         "k.weight": torch.zeros(8, 64), "k.bias": torch.zeros(8)}, "head_dim": 8},
               ck / "jev_head.pt")
    out = export(str(ck), str(tmp_path / "kev"), temperature=1.5)
    meta = torch.load(f"{out}/head.pt")
    assert meta["weights"] == "full" and meta["head_dim"] == 8 and meta["temperature"] == 1.5
    from safetensors import safe_open
    with safe_open(f"{out}/model.safetensors", "pt") as s:
        assert all(k.startswith("model.") for k in s.keys())


def test_decision_export_round_trip(tmp_path):
    """A tiny hybrid decoder saved with the trainer's own writer (several shards), plus a pointer head,
    exported and read back: the text weights and the head survive unchanged, the config is flat, and
    a head whose width does not match the backbone is refused before anything is written."""
    import json

    import pytest
    import torch

    from test_hybrid_cpu import tiny_qwen35
    from trida_stack_b200 import checkpoint
    from trida_stack_b200.export import ExportError, export
    src = tmp_path / "src"
    tiny_qwen35(str(src))
    sd = checkpoint.read_hf_weights(str(src))
    for f in src.glob("*.safetensors"):
        f.unlink()
    checkpoint.write_hf_weights(sd, str(src), max_shard_bytes=200_000)          # force several shards
    assert (src / "model.safetensors.index.json").exists()
    hidden = json.load(open(src / "config.json"))["hidden_size"]
    g = torch.Generator().manual_seed(0)
    head = {"q.weight": torch.randn(8, hidden, generator=g), "q.bias": torch.randn(8, generator=g),
            "k.weight": torch.randn(8, hidden, generator=g), "k.bias": torch.randn(8, generator=g)}
    torch.save({"head": head, "head_dim": 8}, src / "decision_head.pt")
    out = export(str(src), str(tmp_path / "kev"), temperature=0.7, max_shard_bytes=150_000)
    back = checkpoint.read_hf_weights(out)
    text = {("model." + k[len("model."):]): v for k, v in sd.items() if k.startswith("model.")}
    assert back.keys() == text.keys()
    for k in text:
        assert torch.equal(back[k], text[k]), k
    meta = torch.load(f"{out}/head.pt")
    assert set(meta) == {"base", "head", "head_dim", "weights", "weights_dtype", "temperature", "lora",
                         "option_isolation", "special_embeddings", "holdout", "exported_from"}
    assert meta["head_dim"] == 8 and meta["temperature"] == 0.7 and meta["weights"] == "full"
    for k, v in head.items():
        torch.testing.assert_close(meta["head"][k], v)
    cfg = json.load(open(f"{out}/config.json"))
    assert cfg["model_type"] == "qwen3_5_text" and cfg["architectures"] == ["Qwen3_5ForCausalLM"]
    bad = tmp_path / "bad"
    tiny_qwen35(str(bad))
    torch.save({"head": {**head, "k.weight": torch.zeros(8, hidden + 1)}, "head_dim": 8}, bad / "jev_head.pt")
    with pytest.raises(ExportError, match="k.weight"):
        export(str(bad), str(tmp_path / "kev_bad"))
    assert not (tmp_path / "kev_bad").exists()


def test_decision_text_format_is_stable():
    """The row text of requests (render / materialize / augmentation draws) equals the recorded
    golden output: it is the format released checkpoints were trained on."""
    import json
    import os
    import random

    from trida_stack_b200.data import decision as D
    gold = json.load(open(os.path.join(os.path.dirname(__file__), "fixtures", "decision_golden.json")))
    v = {"name": "x", "items": [1, {"a": 2, "b": [3, "four", None]}, [5, 6]], "flag": True, "none": None,
         "nested": {"deep": {"deeper": ["z", {"k": 1.5}]}}, "empty": {}, "elist": []}
    req = {"state": {"user": "alice", "history": ["a", "b"], "meta": {"age": 30}},
           "questions": {"q1": {"type": "choice", "instructions": {"task": "pick", "notes": ["n1"]},
                                "criteria": {"red": "warm colour", "blue": {"why": "cold"}, "green": None},
                                "label": "blue"},
                         "q2": {"type": "noul", "instructions": "yes or no?",
                                "criteria": {"true": "it is", "false": None}, "label": 1},
                         "q3": {"type": "score", "instructions": None, "criteria": ["low", {"mid": 2}, 3], "label": 2},
                         "q4": {"type": "choice", "instructions": "soft", "criteria": {"a": 1, "b": 2},
                                "label": "a", "target": {"a": 3, "b": 1}}}}
    assert D.render(v) == gold["render"]
    assert D.render([1, [2, 3], {"x": [4]}]) == gold["render_list"]
    assert json.loads(json.dumps(D.materialize(req))) == gold["materialize"]
    rng = random.Random(5)
    assert json.loads(json.dumps([D.materialize(x) for x in D.record_variants(req, rng, 1.0)])) == gold["variants"]


def test_epoch_sampler_shards_cover_each_epoch():
    from trida_stack_b200.data.sharding import EpochSampler
    n, nshard = 10, 4
    per = [EpochSampler(n, s, nshard, seed=3).epoch(0) for s in range(nshard)]
    assert all(len(p) == 3 for p in per)                     # ceil(10 / 4), equal for every shard
    assert set(i for p in per for i in p) == set(range(n))   # every record visited
    assert EpochSampler(n, 0, nshard, 3).epoch(1) != per[0]  # a fresh order each epoch
