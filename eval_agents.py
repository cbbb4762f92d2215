#!/usr/bin/env python3
"""Agentic evaluations against the OpenAI-compatible server (``trida_stack_b200.evals.agents``).

    # SWE-bench: instances JSONL (instance_id, repo, base_commit, problem_statement), local checkouts
    python eval_agents.py swebench --instances verified.jsonl --repos /data/repos --port 30000 \\
        --out predictions.jsonl [--test-cmd "pytest -x -q"] [--evaluate]
    # Terminal-Bench style task directories (task.yaml + run-tests.sh), inside a sandbox only
    python eval_agents.py terminal --tasks /sandbox/tasks --port 30000 --out results/terminal.json
    # tau2-bench / Ko-AgentBench with a replica pool started here (or --base-url of a running one)
    python eval_agents.py tau2 --model CKPT --gpus 8 --domains airline retail telecom
    python eval_agents.py koab --model CKPT --gpus 1 --koab-dir /path/to/Ko-AgentBench
    python eval_agents.py tau2 --summarize results.json

The harness commands need tau2-bench / Ko-AgentBench / the swebench harness installed; without them
the command lines are printed (``--dry-run`` prints them in any case).
"""
import argparse
import json
import os
import subprocess
import sys
from pathlib import Path


def _base(a):
    return a.base_url or f"http://{a.host}:{a.port}"


def cmd_swebench(a):
    from trida_stack_b200.evals import agents as A
    insts = [json.loads(ln) for ln in open(a.instances, encoding="utf-8") if ln.strip()]
    if a.limit:
        insts = insts[:a.limit]
    chat = A.ChatClient(_base(a), max_tokens=a.max_tokens, think=a.think)
    agent = A.PatchAgent(chat, rounds=a.rounds, files=a.files, test_cmd=a.test_cmd)
    n = A.write_predictions(insts, agent, a.repos, a.out, a.model_name)
    print(json.dumps({"instances": len(insts), "with_patch": n, "predictions": a.out}))
    ev = A.swebench_eval_command(a.out, a.dataset, a.workers)
    if a.evaluate and not a.dry_run:
        return subprocess.call(ev)
    print("evaluate with:", A.shell_line(ev))
    return 0


def cmd_terminal(a):
    from trida_stack_b200.evals import agents as A
    tasks = sorted(p for p in Path(a.tasks).iterdir() if p.is_dir())
    if a.limit:
        tasks = tasks[:a.limit]
    agent = A.TerminalAgent(A.ChatClient(_base(a), max_tokens=a.max_tokens, think=a.think), max_turns=a.max_turns)
    res = [A.run_task_dir(agent, str(t), timeout=a.cmd_timeout) for t in tasks]
    summary = {"tasks": len(res), "resolved": sum(r["resolved"] for r in res),
               "resolved_rate": sum(r["resolved"] for r in res) / max(len(res), 1), "results": res}
    if a.out:
        os.makedirs(os.path.dirname(a.out) or ".", exist_ok=True)
        json.dump(summary, open(a.out, "w"), indent=1)
    print(json.dumps({k: v for k, v in summary.items() if k != "results"}))
    return 0


def _with_pool(a, fn):
    from trida_stack_b200.evals import agents as A
    if a.base_url or a.dry_run:
        return fn(a.base_url or f"http://127.0.0.1:{a.port}")
    if not a.model:
        sys.exit("give --model (a checkpoint to serve) or --base-url of a running server")
    extra = a.serve_args.split() if a.serve_args else []
    with A.Pool(a.model, gpus=a.gpus, port=a.port, serve_args=extra, log_dir=a.log_dir) as base:
        return fn(base)


def cmd_tau2(a):
    from trida_stack_b200.evals import agents as A
    if a.summarize:
        print(json.dumps(A.summarize_tau2(a.summarize)))
        return 0

    def run(base):
        rc = 0
        for d in a.domains:
            cmd = A.tau2_command(d, f"{base}/v1", a.served, a.user_llm, a.trials, a.concurrency or a.gpus,
                                 a.max_tokens, num_tasks=a.num_tasks)
            print(A.shell_line(cmd), flush=True)
            if a.dry_run:
                continue
            rc |= subprocess.call(cmd, cwd=a.tau2_dir)
            res = Path(a.tau2_dir or ".") / "data" / "simulations" / f"trida_{d}" / "results.json"
            if res.is_file():
                print(d, json.dumps(A.summarize_tau2(res)), flush=True)
        return rc
    return _with_pool(a, run)


def cmd_koab(a):
    from trida_stack_b200.evals import agents as A

    def run(base):
        rc = 0
        for argv, env in A.koab_commands(f"{base}/v1", a.served, a.levels, a.judge, concurrency=a.concurrency or 8):
            print(A.shell_line(argv, env), flush=True)
            if not a.dry_run:
                rc |= subprocess.call(argv, cwd=a.koab_dir, env={**os.environ, **env})
        return rc
    return _with_pool(a, run)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    sub = ap.add_subparsers(dest="cmd", required=True)
    common = argparse.ArgumentParser(add_help=False)
    common.add_argument("--host", default="127.0.0.1")
    common.add_argument("--port", type=int, default=30000)
    common.add_argument("--base-url", default=None)
    common.add_argument("--max-tokens", type=int, default=2048)
    common.add_argument("--think", action="store_true", help="enable the chat template's thinking mode")
    common.add_argument("--dry-run", action="store_true")
    s = sub.add_parser("swebench", parents=[common])
    s.add_argument("--instances", required=True)
    s.add_argument("--repos", required=True, help="checkouts: <repos>/<instance_id> or <repos>/<owner>__<name>")
    s.add_argument("--out", default="predictions.jsonl")
    s.add_argument("--rounds", type=int, default=3)
    s.add_argument("--files", type=int, default=4)
    s.add_argument("--test-cmd", default=None)
    s.add_argument("--limit", type=int, default=0)
    s.add_argument("--model-name", default="trida")
    s.add_argument("--dataset", default="princeton-nlp/SWE-bench_Verified")
    s.add_argument("--workers", type=int, default=4)
    s.add_argument("--evaluate", action="store_true", help="run the swebench harness afterwards (Docker)")
    s.set_defaults(fn=cmd_swebench)
    t = sub.add_parser("terminal", parents=[common])
    t.add_argument("--tasks", required=True)
    t.add_argument("--out", default=None)
    t.add_argument("--limit", type=int, default=0)
    t.add_argument("--max-turns", type=int, default=30)
    t.add_argument("--cmd-timeout", type=int, default=180)
    t.set_defaults(fn=cmd_terminal)
    for name, fn in (("tau2", cmd_tau2), ("koab", cmd_koab)):
        h = sub.add_parser(name, parents=[common])
        h.add_argument("--model", default=None, help="checkpoint to serve on a replica pool started here")
        h.add_argument("--gpus", type=int, default=1)
        h.add_argument("--serve-args", default="", help="extra serve.py flags for every replica")
        h.add_argument("--log-dir", default=None)
        h.add_argument("--served", default="trida")
        h.add_argument("--concurrency", type=int, default=0)
        h.set_defaults(fn=fn)
        if name == "tau2":
            h.add_argument("--domains", nargs="+", default=["airline", "retail", "telecom"])
            h.add_argument("--user-llm", default="openrouter/openai/gpt-4o-mini")
            h.add_argument("--trials", type=int, default=1)
            h.add_argument("--num-tasks", type=int, default=0)
            h.add_argument("--tau2-dir", default=None)
            h.add_argument("--summarize", default=None, help="only summarise this results.json")
        else:
            h.add_argument("--levels", default="L1,L2,L3,L4,L5,L6,L7")
            h.add_argument("--judge", default="openrouter/openai/gpt-4.1-mini")
            h.add_argument("--koab-dir", default=None)
    a = ap.parse_args(argv)
    return a.fn(a)


if __name__ == "__main__":
    sys.exit(main())
