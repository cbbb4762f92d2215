"""Device sampler of the sampled self-speculative step (csrc/sampler.cu).

Speculative sampling must leave the emitted tokens distributed as the target model's truncated
distribution whatever the draft distribution is: a batch of independent requests (one seed each)
draws drafts from q, verifies them against p, and the first emitted token's empirical distribution
must match p (and the draft's must match q, the acceptance rate sum_t min(p_t, q_t)).  The engine
runs sampled requests through it reproducibly from their seeds."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _trunc(logits, T, k, top_p):
    """The host statement of the truncated distribution (engine.truncated_probs)."""
    from trida_stack_b200.serve.engine import SamplingParams, truncated_probs
    return truncated_probs(logits, SamplingParams(temperature=T, top_k=k, top_p=top_p))


def test_speculative_sampling_preserves_target_distribution():
    from trida_stack_b200.ops._ext import ext
    C = ext()
    torch.manual_seed(0)
    B, V, n, T, k, top_p = 20000, 24, 2, 0.9, 16, 0.95
    K, blk = n - 1, 2 * n - 1
    dev = "cuda"
    L1 = torch.randn(blk, V) * 1.5       # draft step: rows 0 (clean) and 1 (draft)
    L2 = torch.randn(blk, V) * 1.5       # verify step: row 0 judges the draft
    q = _trunc(L1[1:2], T, k, top_p)[0]
    p = _trunc(L2[0:1], T, k, top_p)[0]
    slots = torch.arange(B, dtype=torch.int32, device=dev)
    ctr = torch.zeros(B + 1, dtype=torch.long, device=dev)
    q_idx = torch.full((B + 1, K, 64), -1, dtype=torch.int32, device=dev)
    q_prob = torch.zeros(B + 1, K, 64, device=dev)
    temp = torch.full((B,), T, device=dev)
    topk = torch.full((B,), k, dtype=torch.int32, device=dev)
    topp = torch.full((B,), top_p, device=dev)
    seed = torch.arange(B, dtype=torch.long, device=dev) * 7919 + 11

    def step(L, specs, has):
        vals, idx = torch.topk(L.to(dev)[None].expand(B, -1, -1).contiguous(), k, dim=-1)
        out = torch.empty(B, 3 + K, dtype=torch.int32, device=dev)
        C.spec_sample(vals.contiguous(), idx.contiguous(), temp, topk, topp, seed, ctr, slots, specs, has, q_idx,
                      q_prob, out, n)
        return out.cpu()

    none = torch.zeros(B, dtype=torch.int32, device=dev)
    o1 = step(L1, torch.zeros(B, K, dtype=torch.int32, device=dev), none)
    drafts = o1[:, 3]
    freq_q = torch.bincount(drafts.long(), minlength=V).float() / B
    assert (freq_q - q).abs().max().item() < 0.015, (freq_q, q)
    o2 = step(L2, drafts[:, None].to(torch.int32).to(dev).contiguous(), torch.ones(B, dtype=torch.int32, device=dev))
    acc, corr = o2[:, 0], o2[:, 1]
    first = torch.where(acc > 0, drafts, corr)
    assert bool(((acc > 0) | (corr >= 0)).all())
    freq_p = torch.bincount(first.long(), minlength=V).float() / B
    assert (freq_p - p).abs().max().item() < 0.015, (freq_p, p)
    rate = (acc > 0).float().mean().item()
    assert abs(rate - torch.minimum(p, q).sum().item()) < 0.015
    # the same seeds and counters reproduce the draws
    ctr.zero_()
    o1b = step(L1, torch.zeros(B, K, dtype=torch.int32, device=dev), none)
    assert torch.equal(o1b, o1)


def test_engine_sampled_self_spec_is_seeded():
    from trida_stack_b200.serve import Engine, Runtime
    from trida_stack_b200.serve.engine import SamplingParams
    from test_serve_gpu import _hybrid, _init
    dec = _init(_hybrid(128)).to("cuda", torch.bfloat16)
    torch.manual_seed(4)
    prompts = [torch.randint(0, 500, (24,)).tolist() for _ in range(5)]
    runs = []
    from trida_stack_b200.serve.engine import Request
    for _ in range(2):
        eng = Engine(Runtime(dec, max_slots=8, max_len=256), mask_id=511, mode="self-spec", n=4)
        sps = [SamplingParams(temperature=0.8, top_k=20, top_p=0.95, seed=100 + i) for i in range(4)] + \
              [SamplingParams()]                       # a greedy request in the same batch
        reqs = [eng.submit(Request(p, 40, sp)) for p, sp in zip(prompts, sps)]
        while not all(r.done for r in reqs):
            eng.step()
        assert all(len(r.output) == 40 for r in reqs)
        runs.append([r.output for r in reqs])
    assert runs[0] == runs[1]
    # the greedy request decodes as in an all-greedy batch of the same shape (argmax path)
    eng = Engine(Runtime(dec, max_slots=8, max_len=256), mask_id=511, mode="self-spec", n=4)
    greedy = eng.generate(prompts, max_new_tokens=40)
    assert greedy[4].output == runs[0][4]
