#!/usr/bin/env python3
"""Function-calling accuracy (BFCL-style AST match) of a served model.

    python eval_fc.py --questions BFCL_v4_simple_python.json --answers possible_answer/BFCL_v4_simple_python.json \
        --port 30000 [--num-problems 50] [--out results/fc]

The question / answer files use the Berkeley Function-Calling Leaderboard layout (JSONL; several
categories may be concatenated); the reference runs that leaderboard's own package against its
server (``benchmark/bfcl_v4/run_eval.sh``).  Each question goes to ``/v1/chat/completions`` with the
functions as OpenAI ``tools`` (greedy, thinking off by default), and the returned ``tool_calls`` are
scored by ``trida_stack_b200.evals.function_call``.  Writes ``<out>/responses.jsonl`` and
``<out>/summary.json`` (overall and per-category accuracy).
"""
import argparse
import json
import sys
import time
from concurrent.futures import ThreadPoolExecutor, as_completed
from pathlib import Path


def run_one(base, case, args):
    import requests

    from trida_stack_b200.evals.function_call import to_openai_tools
    turns = case["question"]
    messages = [m for turn in turns for m in turn] if turns and isinstance(turns[0], list) else turns
    body = {"model": "default", "messages": messages, "tools": to_openai_tools(case["function"]),
            "max_tokens": args.max_tokens, "temperature": args.temperature,
            "chat_template_kwargs": {"enable_thinking": args.think}}
    try:
        r = requests.post(f"{base}/v1/chat/completions", json=body, timeout=args.timeout).json()
        return case, r["choices"][0]["message"], None
    except Exception as e:
        return case, None, str(e)[:300]


def load_jsonl(path):
    with open(path) as fh:
        text = fh.read().strip()
    if text.startswith("["):
        return json.loads(text)
    return [json.loads(line) for line in text.splitlines() if line.strip()]


def main(argv=None):
    from trida_stack_b200.evals.function_call import score_case, summarize
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--questions", required=True, nargs="+", help="question files (jsonl)")
    ap.add_argument("--answers", required=True, nargs="+", help="ground-truth files (jsonl)")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=30000)
    ap.add_argument("--num-problems", type=int, default=0, help="0 = all (first N otherwise)")
    ap.add_argument("--max-tokens", type=int, default=2048)
    ap.add_argument("--temperature", type=float, default=0.0)
    ap.add_argument("--think", action="store_true", help="enable the model's thinking block")
    ap.add_argument("--timeout", type=int, default=900)
    ap.add_argument("--max-workers", type=int, default=32)
    ap.add_argument("--out", default=None)
    args = ap.parse_args(argv)
    cases = [c for p in args.questions for c in load_jsonl(p)]
    answers = {a["id"]: a for p in args.answers for a in load_jsonl(p)}
    cases = [c for c in cases if c["id"] in answers]
    if args.num_problems:
        cases = cases[:args.num_problems]
    if not cases:
        print("no question has a ground-truth answer", file=sys.stderr)
        return 1
    base = f"http://{args.host}:{args.port}"
    out = Path(args.out or f"results/fc_{time.strftime('%Y%m%d-%H%M%S')}")
    out.mkdir(parents=True, exist_ok=True)
    t0 = time.time()
    results, errors = [], 0
    with ThreadPoolExecutor(max_workers=args.max_workers) as pool, open(out / "responses.jsonl", "w") as fh:
        for f in as_completed([pool.submit(run_one, base, c, args) for c in cases]):
            case, msg, err = f.result()
            errors += err is not None
            res = score_case(case, answers[case["id"]], msg)
            res["error"] = err
            res["content"] = (msg or {}).get("content")
            results.append(res)
            fh.write(json.dumps(res) + "\n")
    summary = summarize(results)
    summary.update(errors=errors, wall_s=round(time.time() - t0, 1))
    (out / "summary.json").write_text(json.dumps(summary, indent=2))
    print(json.dumps(summary))
    return 0


if __name__ == "__main__":
    sys.exit(main())
