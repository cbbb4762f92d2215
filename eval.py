#!/usr/bin/env python3
"""Accuracy and throughput of a served model (the reference's ``inference/zoro-1/eval.py`` and the
fixed-output sweep ``vllm/tools/comprehensive_run/sweep_client.py``).

    python eval.py gsm8k --data gsm8k_test.jsonl [--num-problems 500] [--port 30000]
    python eval.py mmlu_pro --data mmlu_pro_test.jsonl --max-workers 64
    python eval.py sweep --data gsm8k_test.jsonl --concurrency 1 4 8 16 --max-tokens 512
    python eval.py merge results/a results/b            # shards written with --shard I/N

One endpoint per run (``serve.py``).  A task run reports, from the same requests: accuracy,
aggregate and per-request tokens/s, latency p50/p90, mean output length and, from the server's
own counters (``/v1/stats``, or a ``--server-log`` holding this server's, SGLang's or the vLLM
plugin's stats lines), tokens per forward.  Every request goes to ``<out>/requests.jsonl``, the
totals to ``<out>/summary.json``.  Sampling defaults are the self-spec serving setting
(temperature 1.0, top-p 0.95, top-k 20, thinking on).  ``sweep`` sends the GSM8K prompts with
``ignore_eos`` so every request generates exactly ``--max-tokens`` (greedy, thinking off) in strict
waves of ``--concurrency`` requests: a throughput benchmark, not a quality one.

Datasets are read from local files (no network): JSONL / JSON / Parquet with GSM8K's
``question`` / ``answer`` fields or MMLU-Pro's ``question`` / ``options`` / ``answer_index``
(``answer``); with the ``datasets`` package and hub access, the hub ids are used when ``--data`` is
omitted.  Scoring, prompts and the summary fields follow the reference so numbers compare.
"""
import argparse
import json
import random
import re
import statistics
import sys
import time
from concurrent.futures import ThreadPoolExecutor, as_completed
from pathlib import Path

LETTERS = "ABCDEFGHIJ"
SUBSAMPLE_SEED = 42
GSM8K_SUFFIX = "\nPlease reason step by step, and put your final answer within \\boxed{}."


# ------------------------------------------------------------------------------------ datasets
def read_records(path):
    p = Path(path)
    if p.suffix == ".parquet":
        import pyarrow.parquet as pq
        return pq.read_table(p).to_pylist()
    text = p.read_text()
    if p.suffix == ".json":
        data = json.loads(text)
        return data if isinstance(data, list) else data.get("data", [])
    return [json.loads(line) for line in text.splitlines() if line.strip()]


def _hub(name, *args, split="test"):
    try:
        from datasets import load_dataset
    except ImportError:
        raise SystemExit(f"give --data (a local file): the datasets package is not installed for {name}")
    return list(load_dataset(name, *args, split=split))


def gsm8k_load(path=None):
    rows = read_records(path) if path else _hub("openai/gsm8k", "main")
    return [(r["question"], str(r["answer"]).split("####")[-1].strip().replace(",", "")) for r in rows]


def gsm8k_prompt(q):
    return q + GSM8K_SUFFIX


def gsm8k_extract(c):
    boxed = re.findall(r"\\boxed\{([^}]+)\}", c)
    if boxed:
        return boxed[-1].replace(",", "").replace("$", "").replace("\\", "").strip()
    after = c.split("</think>")[-1] if "</think>" in c else c
    nums = re.findall(r"[\d,]+", after)
    return nums[-1].replace(",", "") if nums else "?"


def mmlu_load(path=None):
    rows = read_records(path) if path else _hub("TIGER-Lab/MMLU-Pro")
    out = []
    for r in rows:
        opts = r["options"]
        if isinstance(opts, str):
            opts = json.loads(opts)
        choices = "\n".join(f"{LETTERS[i]}. {o}" for i, o in enumerate(opts) if i < len(LETTERS))
        ai = r.get("answer_index")
        gold = LETTERS[ai] if isinstance(ai, int) else str(r["answer"])
        out.append((f'{r["question"]}\n\n{choices}', gold))
    return out


def mmlu_prompt(qc):
    return f'{qc}\n\nThink step by step, then give your answer as "The answer is (X)".'


def mmlu_extract(c):
    after = re.sub(r"^.*?</think>\s*", "", c, count=1, flags=re.DOTALL) if "</think>" in c else c[-500:]
    for pat in (r"[Aa]nswer is:?\s*\*{0,2}\(?([A-Ja-j])\)?\*{0,2}",
                r"\\boxed\{[^}]*?([A-Ja-j])[^A-Ja-j}]*\}",
                r"[Aa]nswer:?\s*\(?([A-Ja-j])\)?"):
        m = re.search(pat, after)
        if m:
            return m.group(1).upper()
    return "?"


TASKS = {
    "gsm8k": dict(load=gsm8k_load, prompt=gsm8k_prompt, extract=gsm8k_extract),
    "mmlu_pro": dict(load=mmlu_load, prompt=mmlu_prompt, extract=mmlu_extract),
}


# ------------------------------------------------------------------------------------ HTTP
def _post(url, body, timeout):
    import requests
    return requests.post(url, json=body, timeout=timeout).json()


def _get(url, timeout=10):
    import requests
    return requests.get(url, timeout=timeout).json()


def served_model_id(base):
    try:
        return _get(f"{base}/v1/models")["data"][0]["id"]
    except Exception as e:
        print(f"warning: could not read the model id from {base}/v1/models ({type(e).__name__}: {e}); "
              f"sending model='default'", file=sys.stderr, flush=True)
        return "default"


def run_one(base, model, spec, idx, item, args):
    prompt_text, gold = item
    body = {"model": model, "messages": [{"role": "user", "content": spec["prompt"](prompt_text)}],
            "max_tokens": args.max_tokens, "temperature": args.temperature, "top_p": args.top_p,
            "top_k": args.top_k, "presence_penalty": args.presence_penalty,
            "chat_template_kwargs": {"enable_thinking": args.think}}
    rec = {"idx": idx, "gold": gold, "pred": None, "correct": False, "prompt_tokens": 0, "completion_tokens": 0,
           "latency_s": 0.0, "finish_reason": None, "error": None}
    t0 = time.perf_counter()
    try:
        r = _post(f"{base}/v1/chat/completions", body, args.timeout)
        rec["latency_s"] = round(time.perf_counter() - t0, 3)
        if "choices" not in r:
            raise RuntimeError(str(r.get("error", r))[:300])
        c = r["choices"][0]["message"].get("content") or ""
        rec["finish_reason"] = r["choices"][0].get("finish_reason")
        rec["pred"] = spec["extract"](c)
        rec["correct"] = rec["pred"] == gold
        rec["prompt_tokens"] = r["usage"].get("prompt_tokens", 0)
        rec["completion_tokens"] = r["usage"]["completion_tokens"]
    except Exception as e:
        rec["latency_s"] = round(time.perf_counter() - t0, 3)
        rec["error"] = str(e)[:300]
    return rec


# ------------------------------------------------------------------------------------ summaries
def _quantile(lat, p):
    return lat[min(int(p * len(lat)), len(lat) - 1)] if lat else 0.0


def summarize(args, base, model, n, recs, el):
    ok = [r for r in recs if r["error"] is None]
    correct = sum(r["correct"] for r in recs)
    tokens = sum(r["completion_tokens"] for r in ok)
    lat = sorted(r["latency_s"] for r in ok)
    per_req = [r["completion_tokens"] / r["latency_s"] for r in ok if r["latency_s"] > 0]
    return {
        "task": args.task, "endpoint": base, "model": model, "n": n, "correct": correct,
        "num_problems": args.num_problems, "seed": SUBSAMPLE_SEED if args.num_problems else None,
        "shard": args.shard, "accuracy_pct": round(correct / n * 100, 2) if n else 0.0, "errors": n - len(ok),
        "wall_s": round(el, 1), "client_concurrency": args.max_workers,
        "tok_per_s_aggregate": round(tokens / el, 1) if el > 0 else 0.0,
        "tok_per_s_per_request": round(statistics.mean(per_req), 1) if per_req else 0.0,
        "latency_s": {"mean": round(statistics.mean(lat), 2) if lat else 0.0, "p50": _quantile(lat, 0.5),
                      "p90": _quantile(lat, 0.9), "max": lat[-1] if lat else 0.0},
        "completion_tokens_mean": round(tokens / max(len(ok), 1), 1),
        "truncated_pct": round(100 * sum(r["finish_reason"] == "length" for r in ok) / max(len(ok), 1), 1),
        "settings": {"max_tokens": args.max_tokens, "temperature": args.temperature, "top_p": args.top_p,
                     "top_k": args.top_k, "presence_penalty": args.presence_penalty, "thinking": args.think},
    }


def forward_counters(log_path=None, base=None):
    """(emitted tokens, forwards, source), cumulative since server start, or None.  Reads this
    server's ``/v1/stats`` first, else the last stats line of a server log (this engine's, SGLang's
    self-spec line or the vLLM plugin's DiffusionDecoding metrics)."""
    if base is not None:
        try:
            st = _get(f"{base}/v1/stats")
            return st["tokens"], st["forwards"], "server /v1/stats"
        except Exception:
            pass
    if not log_path:
        return None
    try:
        text = Path(log_path).read_text(errors="replace")
    except OSError:
        return None
    m = re.findall(r"\[trida-engine\][^\n]*?fwd=(\d+) tok=(\d+)", text)
    if m:
        return int(m[-1][1]), int(m[-1][0]), "trida engine stats line"
    m = re.findall(r"Committed: (\d+) tokens, Denoising steps: (\d+)", text)
    if m:   # committed drafts exclude the one bonus token every step emits
        fwd = sum(int(b) for _, b in m)
        return sum(int(a) for a, _ in m) + fwd, fwd, "vLLM DiffusionDecoding counters (+1 bonus token per step)"
    m = re.findall(r"\[HybridDiffusionSelfSpec\][^\n]*?fwd=(\d+)[^\n]*?tok/fwd=([\d.]+)", text)
    if m:
        fwd, tpf = int(m[-1][0]), float(m[-1][1])
        return round(fwd * tpf), fwd, "SGLang HybridDiffusionSelfSpec stats"
    return None


def tokens_per_forward(before, after):
    if after is None:
        return {"tok_per_fwd": None, "source": "no forward counter (no /v1/stats and no stats line in the log)"}
    tok0, fwd0 = (before[0], before[1]) if before else (0, 0)
    tok, fwd = after[0] - tok0, after[1] - fwd0
    if fwd <= 0:
        return {"tok_per_fwd": None, "source": f"{after[2]}: counter did not advance during the run"}
    return {"tok_per_fwd": round(tok / fwd, 3), "forwards": fwd, "committed_tokens": tok, "source": after[2]}


def merge(dirs):
    """One summary over shard result dirs; wall is the slowest shard, throughput sums the shards."""
    if not dirs:
        sys.exit("usage: eval.py merge <out-dir> [<out-dir> ...]")
    recs, sums = [], []
    for d in dirs:
        recs += [json.loads(line) for line in open(Path(d) / "requests.jsonl")]
        sums.append(json.loads((Path(d) / "summary.json").read_text()))
    ok = [r for r in recs if r["error"] is None]
    n, correct = len(recs), sum(r["correct"] for r in recs)
    lat = sorted(r["latency_s"] for r in ok)
    per_req = [r["completion_tokens"] / r["latency_s"] for r in ok if r["latency_s"] > 0]
    out = {"task": sums[0]["task"], "shards": len(dirs), "n": n, "correct": correct,
           "accuracy_pct": round(correct / n * 100, 2) if n else 0.0, "errors": n - len(ok),
           "wall_s": max(s["wall_s"] for s in sums),
           "tok_per_s_aggregate": round(sum(s["tok_per_s_aggregate"] for s in sums), 1),
           "tok_per_s_per_request": round(statistics.mean(per_req), 1) if per_req else 0.0,
           "latency_s": {"mean": round(statistics.mean(lat), 2) if lat else 0.0, "p50": _quantile(lat, 0.5),
                         "p90": _quantile(lat, 0.9), "max": lat[-1] if lat else 0.0},
           "completion_tokens_mean": round(sum(r["completion_tokens"] for r in ok) / max(len(ok), 1), 1),
           "truncated_pct": round(100 * sum(r.get("finish_reason") == "length" for r in ok) / max(len(ok), 1), 1),
           "settings": sums[0]["settings"]}
    fw = [s["forward"] for s in sums if s.get("forward", {}).get("tok_per_fwd")]
    if fw:
        tok, f_ = sum(f["committed_tokens"] for f in fw), sum(f["forwards"] for f in fw)
        out["forward"] = {"tok_per_fwd": round(tok / f_, 3), "forwards": f_, "committed_tokens": tok,
                          "source": fw[0]["source"]}
    print(json.dumps(out, indent=1))
    return out


# ------------------------------------------------------------------------------------ sweep
def sweep(args):
    """Fixed-output throughput in strict waves; one JSON line per concurrency level."""
    items = gsm8k_load(args.data)
    qs = [q + GSM8K_SUFFIX for q, _ in items[:args.limit + args.warmup]]
    base = f"http://{args.host}:{args.port}"
    model = served_model_id(base)
    url = f"{base}/v1/chat/completions"

    def one(q):
        body = {"model": model, "messages": [{"role": "user", "content": q}], "max_tokens": args.max_tokens,
                "ignore_eos": True, "temperature": 0, "top_p": 1.0, "chat_template_kwargs": {"enable_thinking": False}}
        t0 = time.perf_counter()
        try:
            d = _post(url, body, args.timeout)
        except Exception as e:
            return {"ok": False, "s": time.perf_counter() - t0, "tok": 0, "err": repr(e)[:200]}
        dt = time.perf_counter() - t0
        if "usage" not in d:
            return {"ok": False, "s": dt, "tok": 0, "err": str(d)[:200]}
        return {"ok": True, "s": dt, "tok": d["usage"]["completion_tokens"]}

    results = []
    for c in args.concurrency:
        with ThreadPoolExecutor(max_workers=c) as pool:
            if args.warmup:
                list(pool.map(one, qs[:args.warmup]))
            work = qs[args.warmup:]
            before = forward_counters(base=base)
            res, T0 = [], time.perf_counter()
            for i in range(0, len(work), c):
                res += list(pool.map(one, work[i:i + c]))
            wall = time.perf_counter() - T0
            after = forward_counters(base=base)
        ok = [r for r in res if r["ok"]]
        tok = sum(r["tok"] for r in ok)
        out = {"concurrency": c, "limit": len(work), "max_tokens": args.max_tokens, "n_ok": len(ok),
               "n_err": len(res) - len(ok), "wall_s": round(wall, 3), "tokens": tok,
               "tok_per_s": round(tok / wall, 2) if wall else 0.0,
               "per_req_tok_per_s": round(statistics.mean(r["tok"] / r["s"] for r in ok), 2) if ok else 0.0,
               "p50_latency_s": round(statistics.median(r["s"] for r in ok), 3) if ok else 0.0,
               "forward": tokens_per_forward(before, after), "errors": [r["err"] for r in res if not r["ok"]][:3]}
        print(json.dumps(out), flush=True)
        results.append(out)
    if args.save:
        Path(args.save).write_text(json.dumps(results, indent=1))
    return results


# ------------------------------------------------------------------------------------ main
def main(argv=None):
    argv = sys.argv[1:] if argv is None else argv
    if argv and argv[0] == "merge":
        return merge(argv[1:])
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("task", choices=list(TASKS) + ["sweep"])
    ap.add_argument("--data", default=None, help="local dataset file (jsonl / json / parquet)")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=30000)
    ap.add_argument("--num-problems", type=int, default=0, help="0 = full set; else a seeded subsample")
    ap.add_argument("--max-tokens", type=int, default=None)
    ap.add_argument("--temperature", type=float, default=1.0)
    ap.add_argument("--top-p", type=float, default=0.95)
    ap.add_argument("--top-k", type=int, default=20)
    ap.add_argument("--presence-penalty", type=float, default=0.0)
    ap.add_argument("--no-think", dest="think", action="store_false")
    ap.add_argument("--timeout", type=int, default=1800)
    ap.add_argument("--max-workers", type=int, default=64, help="client concurrency")
    ap.add_argument("--shard", default=None, metavar="I/N", help="only slice I of N (0-based)")
    ap.add_argument("--out", default=None, help="results dir (default results/<task>_<timestamp>)")
    ap.add_argument("--server-log", default=None, help="server log with stats lines (tokens per forward)")
    ap.add_argument("--concurrency", type=int, nargs="+", default=[8], help="sweep: wave sizes")
    ap.add_argument("--limit", type=int, default=64, help="sweep: timed requests per wave size")
    ap.add_argument("--warmup", type=int, default=2, help="sweep: untimed requests first")
    ap.add_argument("--save", default=None, help="sweep: write the results here")
    args = ap.parse_args(argv)
    if args.task == "sweep":
        args.max_tokens = args.max_tokens or 512
        return sweep(args)
    args.max_tokens = args.max_tokens or 8192
    spec = TASKS[args.task]
    items = spec["load"](args.data)
    if 0 < args.num_problems < len(items):
        rnd = random.Random(SUBSAMPLE_SEED)
        items = [items[i] for i in rnd.sample(range(len(items)), args.num_problems)]
    else:
        args.num_problems = 0
    if args.shard:
        try:
            i, n = (int(x) for x in args.shard.split("/"))
        except ValueError:
            ap.error(f"--shard must look like I/N (0-based), got {args.shard!r}")
        if n < 1 or not (0 <= i < n):
            ap.error(f"--shard I/N needs N >= 1 and 0 <= I < N, got {args.shard!r}")
        items = items[i::n]
    if not items:
        ap.error("no problems selected (check --num-problems / --shard / --data)")
    base = f"http://{args.host}:{args.port}"
    model = served_model_id(base)
    out = Path(args.out or f"results/{args.task}_{time.strftime('%Y%m%d-%H%M%S')}")
    out.mkdir(parents=True, exist_ok=True)
    print(f"{args.task}: {len(items)} problems -> {base} (model={model}, workers={args.max_workers}) -> {out}/",
          flush=True)
    before = forward_counters(args.server_log, base)
    t0 = time.time()
    recs = []
    with ThreadPoolExecutor(max_workers=args.max_workers) as pool, open(out / "requests.jsonl", "w") as fh:
        futs = [pool.submit(run_one, base, model, spec, i, it, args) for i, it in enumerate(items)]
        for k, f in enumerate(as_completed(futs), 1):
            rec = f.result()
            recs.append(rec)
            fh.write(json.dumps(rec) + "\n")
            if k % max(len(items) // 10, 1) == 0:
                print(f"  {k}/{len(items)}  acc={sum(r['correct'] for r in recs) / k * 100:.1f}%  "
                      f"({time.time() - t0:.0f}s)", flush=True)
    el = time.time() - t0
    summary = summarize(args, base, model, len(items), recs, el)
    if args.server_log:
        time.sleep(1)
    summary["forward"] = tokens_per_forward(before, forward_counters(args.server_log, base))
    (out / "summary.json").write_text(json.dumps(summary, indent=1))
    L = summary["latency_s"]
    print(f"\n{args.task}: {summary['correct']}/{len(items)} = {summary['accuracy_pct']:.2f}%   "
          f"errors={summary['errors']}   wall={el:.0f}s")
    print(f"  throughput : {summary['tok_per_s_aggregate']:.0f} tok/s aggregate (C={args.max_workers}), "
          f"{summary['tok_per_s_per_request']:.0f} tok/s per request")
    print(f"  latency    : p50 {L['p50']:.2f}s  p90 {L['p90']:.2f}s  mean {L['mean']:.2f}s   "
          f"(mean output {summary['completion_tokens_mean']:.0f} tokens, "
          f"{summary['truncated_pct']:.1f}% hit max_tokens={args.max_tokens})")
    fw = summary["forward"]
    print(f"  tok/forward: {fw['tok_per_fwd'] if fw['tok_per_fwd'] is not None else 'n/a'}   [{fw['source']}]")
    print(f"  -> {out}/summary.json, {out}/requests.jsonl")
    return summary


if __name__ == "__main__":
    main()
