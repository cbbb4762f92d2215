"""Agentic evaluation drivers (trida_stack_b200/evals/agents.py) with a scripted chat model: the
SWE-bench patch agent on a scratch git repository (a wrong diff, its feedback, then a diff that
passes the tests), the terminal agent on a task directory, and the harness command lines."""
import json
import subprocess

import pytest

from trida_stack_b200.evals import agents as A


class Scripted:
    def __init__(self, answers):
        self.answers, self.seen = list(answers), []

    def __call__(self, messages):
        self.seen.append([dict(m) for m in messages])
        return self.answers.pop(0)


def _repo(tmp_path):
    root = tmp_path / "proj"
    root.mkdir()
    (root / "mathops.py").write_text("def add(a, b):\n    return a - b\n")
    (root / "other.py").write_text("X = 1\n")
    for cmd in (["init", "-q"], ["add", "."], ["-c", "user.email=a@b", "-c", "user.name=n", "commit", "-qm", "i"]):
        subprocess.run(["git", *cmd], cwd=root, check=True)
    return root


GOOD = """Here is the fix.
```diff
--- a/mathops.py
+++ b/mathops.py
@@ -1,2 +1,2 @@
 def add(a, b):
-    return a - b
+    return a + b
```"""
WRONG_CONTEXT = """```diff
--- a/mathops.py
+++ b/mathops.py
@@ -1,2 +1,2 @@
 def add(x, y):
-    return x - y
+    return x + y
```"""
FAILS_TESTS = """<think>maybe multiply</think>
--- a/mathops.py
+++ b/mathops.py
@@ -1,2 +1,2 @@
 def add(a, b):
-    return a - b
+    return a * b
"""


def test_extract_helpers():
    assert A.extract_diff(GOOD).startswith("--- a/mathops.py") and A.extract_diff(GOOD).endswith("+    return a + b\n")
    assert A.extract_diff(FAILS_TESTS).startswith("--- a/mathops.py")
    assert A.extract_diff("no patch here") == ""
    assert A.next_command("<think>ls?</think>\n```bash\nls -la\n```") == "ls -la"
    assert A.next_command("DONE") is None


def test_patch_agent_iterates_until_tests_pass(tmp_path):
    root = _repo(tmp_path)
    assert A.rank_files(str(root), "add(1, 2) in mathops returns -1")[0] == "mathops.py"
    chat = Scripted([WRONG_CONTEXT, FAILS_TESTS, GOOD])
    agent = A.PatchAgent(chat, rounds=3, test_cmd="python -c 'import mathops; assert mathops.add(1, 2) == 3'")
    diff = agent.solve({"problem_statement": "mathops.add(1, 2) returns -1"}, str(root))
    assert diff == A.extract_diff(GOOD)
    assert "def add(a, b)" in chat.seen[0][1]["content"]                    # the retrieved file is shown
    assert "git apply --check failed" in chat.seen[1][-1]["content"]
    assert "tests fail" in chat.seen[2][-1]["content"]
    assert (root / "mathops.py").read_text().endswith("a - b\n")          # the checkout is left untouched
    # predictions file in the harness layout
    out = tmp_path / "pred.jsonl"
    inst = {"instance_id": "proj", "repo": "o/proj", "base_commit": "HEAD", "problem_statement": "add is wrong"}
    n = A.write_predictions([inst], A.PatchAgent(Scripted([GOOD])), str(tmp_path), str(out), "m")
    row = json.loads(out.read_text())
    assert n == 1 and row["instance_id"] == "proj" and row["model_name_or_path"] == "m"
    assert row["model_patch"].startswith("--- a/mathops.py")


def test_terminal_agent_task_dir(tmp_path):
    task = tmp_path / "hello"
    task.mkdir()
    (task / "task.yaml").write_text("instruction: write hi into out.txt\n")
    (task / "run-tests.sh").write_text("grep -qx hi out.txt\n")
    chat = Scripted(["```bash\necho hi > out.txt\n```", "```bash\ncat out.txt\n```", "DONE"])
    res = A.run_task_dir(A.TerminalAgent(chat, max_turns=5), str(task), timeout=30)
    assert res == {"task": "hello", "resolved": True, "turns": 2}
    assert "hi" in chat.seen[2][-1]["content"] and "[exit 0]" in chat.seen[2][-1]["content"]
    assert not (task / "out.txt").exists()                                 # ran in a scratch copy
    res = A.run_task_dir(A.TerminalAgent(Scripted(["DONE"])), str(task), timeout=30)
    assert res["resolved"] is False


def test_harness_commands(tmp_path):
    cmd = A.tau2_command("retail", "http://h:1/v1", served="s", concurrency=4, num_tasks=5)
    assert cmd[:4] == ["tau2", "run", "--domain", "retail"]
    args = json.loads(cmd[cmd.index("--agent-llm-args") + 1])
    assert args["api_base"] == "http://h:1/v1" and args["temperature"] == 0.0
    assert cmd[cmd.index("--num-tasks") + 1] == "5" and cmd[cmd.index("--agent-llm") + 1] == "openai/s"
    res = tmp_path / "results.json"
    res.write_text(json.dumps({"simulations": [{"reward_info": {"reward": 1.0}}, {"reward_info": {"reward": 0.5}},
                                               {"reward_info": None}]}))
    s = A.summarize_tau2(res)
    assert s["sims"] == 3 and s["passed"] == 1 and abs(s["avg_reward"] - 0.5) < 1e-9
    (run, run_env), (score, score_env) = A.koab_commands("http://h:1/v1", date="20260101")
    assert run_env["OPENAI_API_BASE"] == "http://h:1/v1" and "OPENAI_API_BASE" not in score_env
    assert "--judge-models" in score and "--cache-mode" in run
    pool = A.Pool("ckpt", gpus=2, port=9000, serve_args=["--mode", "causal"])
    cmds = pool.commands()
    assert [c[1].get("CUDA_VISIBLE_DEVICES") for c in cmds[:2]] == ["0", "1"]
    assert "--upstreams" in cmds[2][0] and "http://127.0.0.1:9002" in cmds[2][0][-1]


def test_cli_dry_run(capsys):
    import importlib.util
    import pathlib
    spec = importlib.util.spec_from_file_location("eval_agents", pathlib.Path(__file__).parents[1] / "eval_agents.py")
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    assert m.main(["koab", "--dry-run", "--base-url", "http://x:2"]) == 0
    out = capsys.readouterr().out
    assert "OPENAI_API_BASE=http://x:2/v1" in out and "evaluate_model_run.py" in out
    with pytest.raises(SystemExit):
        m.main(["tau2"])                       # neither a model to serve nor a base URL
