#!/usr/bin/env python3
"""IFEval strict / loose accuracy of a served model (the reference's ``inference/zoro-1/eval_ifeval.py``).

    python eval_ifeval.py --data ifeval_input_data.jsonl --port 30000 [--num-problems 50]

``--data``: the IFEval records (JSONL with ``key``, ``prompt``, ``instruction_id_list``, ``kwargs``);
the checks are ``trida_stack_b200.evals.ifeval``.  Sampling defaults follow the reference
(temperature 1.0, top-p 0.95, top-k 20, presence penalty 1.5, thinking on).  Writes
``<out>/responses.jsonl`` and ``<out>/summary.json``.
"""
import argparse
import json
import sys
import time
from concurrent.futures import ThreadPoolExecutor, as_completed
from pathlib import Path


def run_one(base, ref, args):
    import requests
    body = {"model": "default", "messages": [{"role": "user", "content": ref["prompt"]}],
            "max_tokens": args.max_tokens, "temperature": args.temperature, "top_p": args.top_p,
            "top_k": args.top_k, "presence_penalty": args.presence_penalty,
            "chat_template_kwargs": {"enable_thinking": args.think}}
    try:
        r = requests.post(f"{base}/v1/chat/completions", json=body, timeout=args.timeout).json()
        return ref, r["choices"][0]["message"]["content"] or "", None
    except Exception as e:
        return ref, "", str(e)[:300]


def main(argv=None):
    from trida_stack_b200.evals.ifeval import aggregate, score_example
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--data", required=True, help="IFEval records (jsonl)")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=30000)
    ap.add_argument("--num-problems", type=int, default=0, help="0 = all (first N otherwise)")
    ap.add_argument("--max-tokens", type=int, default=8192)
    ap.add_argument("--temperature", type=float, default=1.0)
    ap.add_argument("--top-p", type=float, default=0.95)
    ap.add_argument("--top-k", type=int, default=20)
    ap.add_argument("--presence-penalty", type=float, default=1.5)
    ap.add_argument("--no-think", dest="think", action="store_false")
    ap.add_argument("--timeout", type=int, default=1800)
    ap.add_argument("--max-workers", type=int, default=64)
    ap.add_argument("--out", default=None)
    args = ap.parse_args(argv)
    refs = [json.loads(line) for line in open(args.data) if line.strip()]
    if args.num_problems:
        refs = refs[:args.num_problems]
    base = f"http://{args.host}:{args.port}"
    out = Path(args.out or f"results/ifeval_{time.strftime('%Y%m%d-%H%M%S')}")
    out.mkdir(parents=True, exist_ok=True)
    t0 = time.time()
    results, errors = [], 0
    with ThreadPoolExecutor(max_workers=args.max_workers) as pool, open(out / "responses.jsonl", "w") as fh:
        futs = [pool.submit(run_one, base, r, args) for r in refs]
        for f in as_completed(futs):
            ref, resp, err = f.result()
            errors += err is not None
            strict, loose = score_example(ref, resp)
            results.append((strict, loose))
            fh.write(json.dumps({"key": ref.get("key"), "response": resp, "error": err, "strict": strict,
                                 "loose": loose}) + "\n")
    summary = dict(aggregate(results), errors=errors, wall_s=round(time.time() - t0, 1), endpoint=base)
    (out / "summary.json").write_text(json.dumps(summary, indent=1))
    print(json.dumps(summary))
    return summary


if __name__ == "__main__":
    sys.exit(0 if main() else 1)
