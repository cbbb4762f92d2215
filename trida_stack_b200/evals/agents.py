"""Agentic evaluations over the OpenAI-compatible server: two agent loops of this package's own
(a SWE-bench patch agent and a terminal agent) and launchers for the external multi-turn harnesses.

Reference behaviour: ``benchmark/swe_bench/run_swebench.py`` and
``benchmark/terminal_bench/run_terminal_bench.py`` (scaffolds whose agent loops are left to be
written), ``benchmark/tau2/run_eval.sh`` and ``benchmark/ko_agentbench/run_eval.sh`` (a replica
pool behind one OpenAI base URL, the harness's LiteLLM ``openai/<name>`` agent pointed at it, then
a summary of its result files), ``benchmark/serving/pool.sh`` (replicas + router + chat self-check).

* ``PatchAgent``     SWE-bench: retrieves the repository files an issue names, asks the model for a
                     unified diff, checks it with ``git apply --check`` (and an optional test
                     command on a scratch worktree), feeds failures back for a bounded number of
                     rounds; ``write_predictions`` emits the harness's ``predictions.jsonl``.
* ``TerminalAgent``  Terminal-Bench style tasks: the model answers with one shell command per turn
                     (a fenced ``bash`` block) or ``DONE``; the command's output goes back as the next
                     user turn.  ``run_task_dir`` runs a task directory (``task.yaml`` instruction,
                     ``run-tests.sh`` check) in a scratch copy -- only inside a sandbox the caller
                     provides, since task commands are untrusted.
* ``tau2_command`` / ``koab_commands`` build the harness command lines; ``summarize_tau2`` reads
                     a tau2 ``results.json`` (simulations, average reward, pass@1).
* ``Pool``           starts N ``serve.py`` replicas (one per GPU) and the data-parallel router, and
                     waits until a chat completion answers.
"""
import json
import os
import re
import shlex
import shutil
import subprocess
import sys
import tempfile
import time
from pathlib import Path


class ChatClient:
    """``/v1/chat/completions`` of one base URL (greedy by default)."""

    def __init__(self, base, model="default", max_tokens=2048, temperature=0.0, timeout=1200.0, think=False):
        self.base, self.model, self.max_tokens = base.rstrip("/"), model, max_tokens
        self.temperature, self.timeout, self.think = temperature, timeout, think

    def __call__(self, messages):
        import requests
        body = {"model": self.model, "messages": messages, "max_tokens": self.max_tokens,
                "temperature": self.temperature, "chat_template_kwargs": {"enable_thinking": self.think}}
        r = requests.post(f"{self.base}/v1/chat/completions", json=body, timeout=self.timeout)
        r.raise_for_status()
        return r.json()["choices"][0]["message"].get("content") or ""


def _strip_think(text):
    return re.sub(r"<think>.*?</think>", "", text, flags=re.S).strip()


# ------------------------------------------------------------------------------------ SWE-bench
PATCH_SYSTEM = ("You fix bugs in a Python repository. Answer with one unified diff against the files shown "
                "(paths relative to the repository root, with --- a/ and +++ b/ headers) inside a ```diff block. "
                "Change only what the issue needs.")

_WORD = re.compile(r"[A-Za-z_][A-Za-z0-9_]{2,}")


def extract_diff(text):
    """The unified diff of a model answer: the last ```diff / ```patch block, else the text from the
    first ``diff --git`` or ``--- a/`` line; always ends with a newline ('' when there is none)."""
    text = _strip_think(text)
    blocks = re.findall(r"```(?:diff|patch)\s*\n(.*?)```", text, flags=re.S)
    if blocks:
        d = blocks[-1]
    else:
        m = re.search(r"^(diff --git |--- a/)", text, flags=re.M)
        if not m:
            return ""
        d = text[m.start():].split("```")[0]
    d = d.strip("\n")
    return d + "\n" if d else ""


def rank_files(root, problem, k=4, max_bytes=200_000, exts=(".py",)):
    """Repository files ranked by how many of the issue's identifiers they contain (file-name hits
    count triple); the lexical retrieval step that picks the context the model sees."""
    words = {w.lower() for w in _WORD.findall(problem)}
    scored = []
    for dp, dns, fns in os.walk(root):
        dns[:] = [d for d in dns if not d.startswith(".") and d not in ("node_modules", "__pycache__", "build")]
        for fn in fns:
            if not fn.endswith(exts):
                continue
            p = os.path.join(dp, fn)
            try:
                if os.path.getsize(p) > max_bytes:
                    continue
                body = open(p, encoding="utf-8", errors="replace").read()
            except OSError:
                continue
            toks = {w.lower() for w in _WORD.findall(body)}
            stem = {w.lower() for w in _WORD.findall(os.path.relpath(p, root))}
            s = len(words & toks) + 3 * len(words & stem)
            if s:
                scored.append((s, os.path.relpath(p, root)))
    scored.sort(key=lambda t: (-t[0], t[1]))
    return [p for _, p in scored[:k]]


def _git(cwd, *args, stdin=None, timeout=120):
    return subprocess.run(["git", *args], cwd=cwd, input=stdin, capture_output=True, text=True, timeout=timeout)


class PatchAgent:
    """Issue -> unified diff, checked by ``git apply --check`` and optionally by a test command run
    on a scratch copy of the checkout; failures go back to the model for up to ``rounds`` answers."""

    def __init__(self, chat, rounds=3, files=4, max_file_chars=12_000, test_cmd=None, test_timeout=900):
        self.chat, self.rounds, self.files, self.max_file_chars = chat, rounds, files, max_file_chars
        self.test_cmd, self.test_timeout = test_cmd, test_timeout

    def context(self, root, problem):
        parts = []
        for rel in rank_files(root, problem, self.files):
            body = open(os.path.join(root, rel), encoding="utf-8", errors="replace").read()
            if len(body) > self.max_file_chars:
                body = body[:self.max_file_chars] + "\n# ... (truncated)\n"
            parts.append(f"### {rel}\n```python\n{body}\n```")
        return "\n\n".join(parts)

    def check(self, root, diff):
        """(ok, feedback) of a candidate diff."""
        if not diff:
            return False, "No diff found in the answer. Reply with a ```diff block."
        r = _git(root, "apply", "--check", "-", stdin=diff)
        if r.returncode:
            return False, f"git apply --check failed:\n{(r.stderr or r.stdout)[-2000:]}"
        if not self.test_cmd:
            return True, ""
        with tempfile.TemporaryDirectory() as tmp:
            work = os.path.join(tmp, "w")
            shutil.copytree(root, work, symlinks=True)
            _git(work, "apply", "-", stdin=diff)
            try:
                t = subprocess.run(self.test_cmd, shell=True, cwd=work, capture_output=True, text=True,
                                   timeout=self.test_timeout)
            except subprocess.TimeoutExpired:
                return False, f"The tests timed out after {self.test_timeout} s."
            if t.returncode:
                return False, f"The patch applies but the tests fail:\n{(t.stdout + t.stderr)[-3000:]}"
        return True, ""

    def solve(self, instance, root):
        """The final diff for one instance ('' when no candidate applied)."""
        problem = instance["problem_statement"]
        msgs = [{"role": "system", "content": PATCH_SYSTEM},
                {"role": "user", "content": f"Issue:\n{problem}\n\nRelevant files:\n\n{self.context(root, problem)}"}]
        best = ""
        for _ in range(self.rounds):
            answer = self.chat(msgs)
            diff = extract_diff(answer)
            ok, fb = self.check(root, diff)
            if ok:
                return diff
            if diff and not best and "git apply" not in fb:
                best = diff                       # applies; tests failed -- kept if nothing better comes
            msgs += [{"role": "assistant", "content": answer}, {"role": "user", "content": fb}]
        return best


def checkout(instance, repos):
    """The working tree of an instance: ``repos/<instance_id>`` if present, else a clone of
    ``repos/<owner>__<name>`` checked out at ``base_commit`` in a scratch directory."""
    direct = Path(repos) / instance["instance_id"]
    if direct.is_dir():
        return str(direct), None
    src = Path(repos) / instance["repo"].replace("/", "__")
    if not src.is_dir():
        raise FileNotFoundError(f"no checkout for {instance['instance_id']} under {repos}")
    tmp = tempfile.mkdtemp(prefix="swe-")
    r = _git(tmp, "clone", "-q", "--no-checkout", str(src), "w", timeout=600)
    if r.returncode:
        raise RuntimeError(r.stderr)
    work = os.path.join(tmp, "w")
    r = _git(work, "checkout", "-q", instance["base_commit"])
    if r.returncode:
        raise RuntimeError(r.stderr)
    return work, tmp


def write_predictions(instances, agent, repos, out, model_name="trida"):
    """Solve every instance and write the harness's predictions file; returns the count with a patch."""
    n = 0
    with open(out, "w", encoding="utf-8") as fo:
        for inst in instances:
            root, tmp = checkout(inst, repos)
            try:
                patch = agent.solve(inst, root)
            finally:
                if tmp:
                    shutil.rmtree(tmp, ignore_errors=True)
            n += bool(patch)
            fo.write(json.dumps({"instance_id": inst["instance_id"], "model_name_or_path": model_name,
                                 "model_patch": patch}) + "\n")
    return n


def swebench_eval_command(predictions, dataset="princeton-nlp/SWE-bench_Verified", workers=4, run_id="trida"):
    """The official harness's evaluation (runs each instance's tests in Docker)."""
    return [sys.executable, "-m", "swebench.harness.run_evaluation", "--dataset_name", dataset,
            "--predictions_path", str(predictions), "--max_workers", str(workers), "--run_id", run_id]


# ------------------------------------------------------------------------------------ terminal
TERMINAL_SYSTEM = ("You operate a Linux shell to complete a task. Each reply is either exactly one command in a "
                   "```bash block, which is run and whose output you then see, or the single word DONE when the "
                   "task is complete.")


def next_command(text):
    """The command of a terminal-agent answer, or None for DONE / no command."""
    text = _strip_think(text)
    m = re.findall(r"```(?:bash|sh|shell)?\s*\n(.*?)```", text, flags=re.S)
    if m:
        cmd = m[-1].strip()
        return cmd or None
    return None


class LocalSession:
    """Commands run by ``bash -lc`` in one working directory (inside the caller's sandbox)."""

    def __init__(self, cwd, timeout=180, max_output=4000, env=None):
        self.cwd, self.timeout, self.max_output, self.env = cwd, timeout, max_output, env

    def run(self, cmd):
        try:
            r = subprocess.run(["bash", "-lc", cmd], cwd=self.cwd, capture_output=True, text=True,
                               timeout=self.timeout, env=self.env)
            out = (r.stdout + r.stderr)
            tail = f"\n[exit {r.returncode}]"
        except subprocess.TimeoutExpired as e:
            out = ((e.stdout or b"").decode(errors="replace") if isinstance(e.stdout, bytes) else (e.stdout or ""))
            tail = f"\n[timed out after {self.timeout} s]"
        if len(out) > self.max_output:
            out = out[:self.max_output // 2] + "\n...\n" + out[-self.max_output // 2:]
        return out + tail


class TerminalAgent:
    """One command per turn until the model says DONE or ``max_turns`` run out; returns the
    transcript as (command, output) pairs."""

    def __init__(self, chat, max_turns=30):
        self.chat, self.max_turns = chat, max_turns

    def perform_task(self, instruction, session):
        msgs = [{"role": "system", "content": TERMINAL_SYSTEM}, {"role": "user", "content": f"Task:\n{instruction}"}]
        log = []
        for _ in range(self.max_turns):
            answer = self.chat(msgs)
            cmd = next_command(answer)
            if cmd is None:
                if "DONE" in _strip_think(answer):
                    break
                msgs += [{"role": "assistant", "content": answer},
                         {"role": "user", "content": "Reply with one ```bash block or DONE."}]
                continue
            out = session.run(cmd)
            log.append((cmd, out))
            msgs += [{"role": "assistant", "content": answer}, {"role": "user", "content": f"Output:\n{out}"}]
        return log


def read_instruction(task_dir):
    """The instruction of a task directory (``task.yaml`` key ``instruction``, else ``instruction.md``)."""
    y = Path(task_dir) / "task.yaml"
    if y.is_file():
        import yaml
        d = yaml.safe_load(y.read_text()) or {}
        if d.get("instruction"):
            return d["instruction"]
    md = Path(task_dir) / "instruction.md"
    if md.is_file():
        return md.read_text()
    raise FileNotFoundError(f"{task_dir}: no task.yaml instruction or instruction.md")


def run_task_dir(agent, task_dir, timeout=180):
    """Run one task in a scratch copy of its directory; resolved when ``run-tests.sh`` exits 0
    afterwards.  Task commands are untrusted: call this only inside a sandbox."""
    with tempfile.TemporaryDirectory() as tmp:
        work = os.path.join(tmp, "task")
        shutil.copytree(task_dir, work, symlinks=True)
        sess = LocalSession(work, timeout=timeout)
        log = agent.perform_task(read_instruction(work), sess)
        test = os.path.join(work, "run-tests.sh")
        ok = False
        if os.path.isfile(test):
            r = subprocess.run(["bash", test], cwd=work, capture_output=True, text=True, timeout=timeout * 5)
            ok = r.returncode == 0
    return {"task": os.path.basename(os.path.normpath(task_dir)), "resolved": ok, "turns": len(log)}


# ------------------------------------------------------------------------------------ harness launchers
def tau2_command(domain, base_url, served="trida", user_llm="openrouter/openai/gpt-4o-mini", trials=1,
                 concurrency=8, max_tokens=2048, timeout=900, save_to=None, num_tasks=None, task_ids=None):
    """tau2-bench's ``tau2 run`` with the agent on this server (LiteLLM ``openai/`` provider, greedy,
    per-turn token cap so long reasoning does not fill the context) and the user simulator elsewhere."""
    agent_args = {"temperature": 0.0, "max_tokens": max_tokens, "api_base": base_url, "api_key": "EMPTY"}
    cmd = ["tau2", "run", "--domain", domain, "--agent-llm", f"openai/{served}", "--agent-llm-args",
           json.dumps(agent_args), "--user-llm", user_llm, "--user-llm-args", json.dumps({"temperature": 0.0}),
           "--num-trials", str(trials), "--max-concurrency", str(concurrency), "--timeout", str(timeout),
           "--save-to", save_to or f"trida_{domain}", "--auto-resume"]
    if num_tasks:
        cmd += ["--num-tasks", str(num_tasks)]
    if task_ids:
        cmd += ["--task-ids", str(task_ids)]
    return cmd


def summarize_tau2(path):
    """Simulations, average reward and pass@1 (reward >= 0.999) of a tau2 ``results.json``."""
    sims = json.load(open(path)).get("simulations", [])
    rewards = [float(((s.get("reward_info") or {}).get("reward")) or 0.0) for s in sims]
    n = len(rewards)
    passed = sum(r >= 0.999 for r in rewards)
    return {"sims": n, "avg_reward": sum(rewards) / n if n else 0.0, "pass@1": passed / n if n else 0.0,
            "passed": passed}


def koab_commands(base_url, served="trida", levels="L1,L2,L3,L4,L5,L6,L7", judge="openrouter/openai/gpt-4.1-mini",
                  date=None, concurrency=8, timeout=1200):
    """Ko-AgentBench's two stages: trajectories against this server (cache-backed tools), then the
    judge run.  Returns [(argv, extra env)]; only the first stage sees this server's base URL."""
    date = date or time.strftime("%Y%m%d")
    run = (["python", "run_benchmark_with_logging.py", "--levels", levels, "--model", f"openai/{served}",
            "--cache-mode", "read", "--timeout", str(timeout), "--concurrency", str(concurrency)],
           {"OPENAI_API_BASE": base_url, "OPENAI_API_KEY": "EMPTY"})
    score = (["python", "evaluate_model_run.py", "--date", date, "--model", f"openai/{served}", "--judge-models",
              judge, "--levels", levels, "--format", "all"], {})
    return [run, score]


# ------------------------------------------------------------------------------------ replica pool
class Pool:
    """N ``serve.py`` replicas (GPU i on port base_port + 1 + i) behind the data-parallel router on
    ``port``; ``start`` returns the router's base URL once a chat completion answers."""

    def __init__(self, model, gpus=1, port=8000, serve_args=(), log_dir=None, ready_timeout=1800):
        self.model, self.gpus, self.port, self.serve_args = model, gpus, port, list(serve_args)
        self.log_dir, self.ready_timeout = log_dir, ready_timeout
        self.procs = []

    def commands(self):
        root = Path(__file__).resolve().parents[2]
        ups = [f"http://127.0.0.1:{self.port + 1 + i}" for i in range(self.gpus)]
        cmds = []
        for i in range(self.gpus):
            cmds.append(([sys.executable, str(root / "serve.py"), self.model, "--port", str(self.port + 1 + i),
                          "--host", "127.0.0.1", *self.serve_args], {"CUDA_VISIBLE_DEVICES": str(i)}))
        cmds.append(([sys.executable, "-m", "trida_stack_b200.serve.router", "--host", "127.0.0.1", "--port",
                      str(self.port), "--upstreams", ",".join(ups)], {}))
        return cmds

    def start(self):
        for i, (argv, env) in enumerate(self.commands()):
            log = open(os.path.join(self.log_dir, f"pool_{i}.log"), "w") if self.log_dir else subprocess.DEVNULL
            self.procs.append(subprocess.Popen(argv, env={**os.environ, **env}, stdout=log, stderr=subprocess.STDOUT))
        base = f"http://127.0.0.1:{self.port}"
        chat = ChatClient(base, max_tokens=8, timeout=60)
        t0 = time.time()
        while time.time() - t0 < self.ready_timeout:
            if any(p.poll() is not None for p in self.procs):
                self.stop()
                raise RuntimeError("a pool process exited during start-up")
            try:
                chat([{"role": "user", "content": "Say OK."}])
                return base
            except Exception:      # noqa: BLE001  (not up yet)
                time.sleep(5)
        self.stop()
        raise TimeoutError("the pool did not answer a chat completion in time")

    def stop(self):
        for p in self.procs:
            if p.poll() is None:
                p.terminate()
        for p in self.procs:
            try:
                p.wait(timeout=30)
            except subprocess.TimeoutExpired:
                p.kill()
        self.procs = []

    def __enter__(self):
        return self.start()

    def __exit__(self, *exc):
        self.stop()


def shell_line(argv, env=None):
    """A copy-pasteable command line."""
    pre = " ".join(f"{k}={shlex.quote(v)}" for k, v in (env or {}).items())
    return (pre + " " if pre else "") + " ".join(shlex.quote(a) for a in argv)
