"""Self-distillation data for draft-aligned fine-tuning: regenerate every assistant turn of SFT
conversations with the model's own greedy causal decoding.

Reference behaviour: ``train/tools/draftalign/gen_selfdistill.py``.  The system / user / tool turns
and the tool schemas of each conversation are kept; the assistant turns are regenerated one after
another, each conditioned on the already regenerated earlier turns (what the verifier sees at
inference time).  Prompts are rendered to token ids with the trainer's own chat-template helper
(``data.sft.render``) and sent as token ids to the OpenAI-compatible ``/v1/completions`` endpoint of
one or more ``serve.py`` instances (``--mode causal``, greedy), so the served model reads exactly
the tokens it was trained on.

A conversation is dropped when a prompt is longer than ``--max-prompt`` tokens, when a turn runs
out of budget (``finish_reason == "length"``; the turn's head and tail go to ``OUT.truncated.jsonl``)
or when a request fails.  Every kept turn is checked by a round trip: the conversation re-rendered
with the new turn must start with the prompt ids followed by the generated ids (mismatches are
counted, not dropped).  Counters go to ``OUT.stats.json``.

    python -m trida_stack_b200.selfdistill --src DIR --out shard.jsonl --tokenizer CKPT \\
        --ports 30000 30001 [--stride 17 --offset 0 --count 20000 --max-tokens 16384]

Conversations are every ``--stride``-th line over ``DIR/chunk-*.jsonl`` (global line order), and
this shard takes ``[offset, offset + count)`` of them.
"""
import argparse
import asyncio
import glob
import json
import os
import sys
import time


def select_rows(src, stride, offset, count):
    """Every ``stride``-th conversation over the sorted chunk files, then ``[offset, offset + count)``."""
    k = taken = 0
    for path in sorted(glob.glob(os.path.join(src, "chunk-*.jsonl"))):
        with open(path, encoding="utf-8") as fh:
            for i, line in enumerate(fh):
                if i % stride:
                    continue
                if k >= offset:
                    if taken >= count:
                        return
                    taken += 1
                    yield json.loads(line)
                k += 1


class Distiller:
    def __init__(self, tok, ports, model="trida", max_tokens=16384, max_prompt=24000, ctx_len=32768, per_port=16,
                 timeout=3600.0, host="127.0.0.1", out=None):
        self.tok, self.ports, self.model = tok, list(ports), model
        self.max_tokens, self.max_prompt, self.ctx_len = max_tokens, max_prompt, ctx_len
        self.per_port, self.timeout, self.host, self.out = per_port, timeout, host, out
        self.stats = {"conv": 0, "kept": 0, "turns": 0, "truncated": 0, "long_prompt": 0, "roundtrip_mismatch": 0,
                      "errors": 0, "gen_tokens": 0}
        self._rr = 0

    def render(self, messages, tools, gen):
        from .data.sft import render
        try:
            return render(self.tok, messages, tools, gen, keep_all_reasoning=True), tools
        except Exception:          # a template that rejects the tool schemas renders without them
            return render(self.tok, messages, None, gen, keep_all_reasoning=True), None

    async def complete(self, sess, sems, prompt_ids):
        import aiohttp
        port = self.ports[self._rr % len(self.ports)]
        self._rr += 1
        budget = max(256, min(self.max_tokens, self.ctx_len - len(prompt_ids) - 16))
        body = {"model": self.model, "prompt": list(prompt_ids), "max_tokens": budget, "temperature": 0,
                "return_token_ids": True}
        async with sems[port]:
            async with sess.post(f"http://{self.host}:{port}/v1/completions", json=body,
                                 timeout=aiohttp.ClientTimeout(total=self.timeout)) as r:
                d = await r.json()
                if r.status != 200:
                    raise RuntimeError(str(d)[:200])
        c = d["choices"][0]
        return c["text"], c.get("finish_reason"), c.get("token_ids")

    async def conversation(self, sess, sems, row):
        from .data.sft import normalize_messages
        msgs = normalize_messages(row.get("messages") or [])
        tools = row.get("tools")
        turns = [i for i, m in enumerate(msgs) if m["role"] == "assistant"]
        if not turns:
            return None
        new = [dict(m) for m in msgs]
        for i in turns:
            prompt, used = self.render(new[:i], tools, True)
            if len(prompt) > self.max_prompt:
                self.stats["long_prompt"] += 1
                return None
            try:
                text, finish, gen_ids = await self.complete(sess, sems, prompt)
            except Exception as e:   # noqa: BLE001  (any failed request drops the conversation)
                self.stats["errors"] += 1
                self.stats.setdefault("error_samples", [])
                if len(self.stats["error_samples"]) < 5:
                    self.stats["error_samples"].append(str(e)[:160])
                return None
            if finish == "length":
                self.stats["truncated"] += 1
                if self.out:
                    with open(self.out + ".truncated.jsonl", "a", encoding="utf-8") as f:
                        f.write(json.dumps({"id": row.get("id"), "turn": i, "head": text[:300], "tail": text[-300:]},
                                           ensure_ascii=False) + "\n")
                return None
            text = text.split("<|im_end|>")[0]
            # the generation prompt of a thinking template ends inside an open <think> block
            new[i] = {"role": "assistant", "content": text if text.startswith("<think>") else "<think>\n" + text}
            self.stats["turns"] += 1
            self.stats["gen_tokens"] += len(gen_ids or [])
            try:
                full, _ = self.render(new[:i + 1], used, False)
                expect = list(prompt) + list(gen_ids if gen_ids else self.tok(text, add_special_tokens=False).input_ids)
                if full[:len(expect)] != expect:
                    self.stats["roundtrip_mismatch"] += 1
            except Exception:        # noqa: BLE001
                self.stats["roundtrip_mismatch"] += 1
        out = dict(row)
        out["messages"] = new
        out["meta"] = dict(row.get("meta") or {}, generated={"model": self.model, "max_tokens": self.max_tokens,
                                                              "greedy": True, "sequential_history": True})
        return out

    async def run(self, rows, fo):
        import aiohttp
        sems = {p: asyncio.Semaphore(self.per_port) for p in self.ports}
        t0 = time.time()
        pending = set()
        async with aiohttp.ClientSession() as sess:
            async def one(row):
                self.stats["conv"] += 1
                res = await self.conversation(sess, sems, row)
                if res is not None:
                    self.stats["kept"] += 1
                    fo.write(json.dumps(res, ensure_ascii=False) + "\n")
                if self.stats["conv"] % 200 == 0:
                    print(f"[{time.time() - t0:7.0f}s] {self.stats}", file=sys.stderr, flush=True)
            # turns of one conversation are sequential: keep many conversations in flight
            for row in rows:
                while len(pending) >= len(self.ports) * self.per_port * 2:
                    _, pending = await asyncio.wait(pending, return_when=asyncio.FIRST_COMPLETED)
                pending.add(asyncio.create_task(one(row)))
            if pending:
                await asyncio.gather(*pending)
        return self.stats


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--src", required=True, help="directory of chunk-*.jsonl SFT conversations")
    ap.add_argument("--out", required=True)
    ap.add_argument("--tokenizer", required=True, help="checkpoint directory whose chat template renders prompts")
    ap.add_argument("--ports", type=int, nargs="+", required=True)
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--model", default="trida")
    ap.add_argument("--stride", type=int, default=17)
    ap.add_argument("--offset", type=int, default=0)
    ap.add_argument("--count", type=int, default=20000)
    ap.add_argument("--max-tokens", type=int, default=16384)
    ap.add_argument("--max-prompt", type=int, default=24000)
    ap.add_argument("--ctx-len", type=int, default=32768, help="server context: max_tokens is clipped to it")
    ap.add_argument("--per-port", type=int, default=16)
    ap.add_argument("--timeout", type=float, default=3600.0)
    a = ap.parse_args(argv)
    from .models.build import load_tokenizer
    tok = load_tokenizer(a.tokenizer)
    d = Distiller(tok, a.ports, a.model, a.max_tokens, a.max_prompt, a.ctx_len, a.per_port, a.timeout, a.host, a.out)
    with open(a.out, "w", encoding="utf-8") as fo:
        stats = asyncio.run(d.run(select_rows(a.src, a.stride, a.offset, a.count), fo))
    print(json.dumps(stats), file=sys.stderr)
    with open(a.out + ".stats.json", "w") as f:
        json.dump(stats, f)
    return 0


if __name__ == "__main__":
    sys.exit(main())
