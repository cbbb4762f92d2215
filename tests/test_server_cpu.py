"""HTTP server (OpenAI-compatible + System One) over the native engine, on CPU."""
import json
import socket
import threading
import time

import pytest
import requests

from helpers import make_tokenizer
from test_hybrid_cpu import tiny_qwen35


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.fixture(scope="module")
def server(tmp_path_factory):
    import uvicorn

    import serve as serve_cli
    from trida_stack_b200.serve.server import build_app
    path = tmp_path_factory.mktemp("ckpt")
    tiny_qwen35(str(path))            # hybrid checkpoint (the decision head rides on the hybrid model)
    tok = make_tokenizer(str(path), 295)
    from trida_stack_b200.data.decision import SPECIAL
    tok.add_special_tokens({"additional_special_tokens": SPECIAL})   # ids 295..299
    tok.save_pretrained(str(path))
    args = serve_cli.parse_args([str(path), "--mode", "decide", "--device", "cpu", "--dtype", "float32",
                                 "--max-running", "4", "--max-len", "512"])
    engine, tok, name, decider = serve_cli.build(args)
    engine.start()
    port = _free_port()
    cfg = uvicorn.Config(build_app(engine, tok, name, decider), host="127.0.0.1", port=port, log_level="error")
    srv = uvicorn.Server(cfg)
    th = threading.Thread(target=srv.run, daemon=True)
    th.start()
    url = f"http://127.0.0.1:{port}"
    for _ in range(200):
        try:
            if requests.get(url + "/health", timeout=1).ok:
                break
        except requests.ConnectionError:
            time.sleep(0.05)
    yield url
    srv.should_exit = True
    engine.stop()


def test_models_and_health(server):
    assert requests.get(server + "/health").json()["status"] == "ok"
    data = requests.get(server + "/v1/models").json()["data"]
    assert data and data[0]["object"] == "model"


def test_completion_and_chat(server):
    r = requests.post(server + "/v1/completions", json={"prompt": "t1 t2 t3 t4", "max_tokens": 6}).json()
    assert r["usage"]["prompt_tokens"] == 4 and r["usage"]["completion_tokens"] <= 6
    assert r["choices"][0]["finish_reason"] in ("stop", "length")
    r = requests.post(server + "/v1/chat/completions",
                      json={"messages": [{"role": "user", "content": "t5 t6"}], "max_tokens": 5}).json()
    assert r["object"] == "chat.completion" and r["choices"][0]["message"]["role"] == "assistant"
    assert r["usage"]["completion_tokens"] <= 5


def test_chat_streaming(server):
    with requests.post(server + "/v1/chat/completions", stream=True,
                       json={"messages": [{"role": "user", "content": "t7"}], "max_tokens": 5, "stream": True}) as r:
        lines = [l for l in r.iter_lines(decode_unicode=True) if l]
    assert lines[-1] == "data: [DONE]"
    last = json.loads(lines[-2][6:])
    assert last["choices"][0]["finish_reason"] in ("stop", "length") and "usage" in last


def test_systemone_decisions_and_validation(server):
    body = {"model": "m", "state": {"user": "t1 t2"}, "questions": {
        "q1": {"type": "choice", "instructions": "pick", "criteria": {"a": "t3", "b": "t4", "c": "t5"}},
        "q2": {"type": "noul", "criteria": {"true": "t6", "false": "t7"}},
        "q3": {"type": "score", "criteria": ["low", "mid", "high"]}}}
    r = requests.post(server + "/v1/systemone", json=body)
    assert r.status_code == 200, r.text
    out = r.json()
    assert out["model"] and out["usage"]["input_tokens"] > 0 and out["usage"]["output_tokens"] == 0
    ans = out["answers"]
    assert ans["q1"]["type"] == "choice" and ans["q1"]["choice"] in ("a", "b", "c")
    assert abs(sum(ans["q1"]["probabilities"].values()) - 1) < 1e-3
    assert 0.0 <= ans["q1"]["confidence"] <= 1.0
    assert ans["q2"]["type"] == "noul" and 0.0 <= ans["q2"]["noul"] <= 1.0
    assert ans["q3"]["type"] == "score" and 0.0 <= ans["q3"]["score"] <= 2.0
    assert ans["q3"]["legend"] == {"0": "low", "1": "mid", "2": "high"}
    assert set(ans["q3"]["probabilities"]) == {"0", "1", "2"}
    # a sharper temperature keeps the choice and moves its probability away from uniform
    sharp = requests.post(server + "/v1/systemone", json={**body, "temperature": 0.05}).json()["answers"]
    assert sharp["q1"]["choice"] == ans["q1"]["choice"]
    assert sharp["q1"]["confidence"] >= ans["q1"]["confidence"] - 1e-4
    bad = requests.post(server + "/v1/systemone", json={"model": "m", "state": {}, "questions": {"q": {"type": "pick"}}})
    assert bad.status_code == 422
    assert bad.json()["detail"][0]["loc"][-1] == "type"
    assert requests.post(server + "/v1/systemone", json={k: v for k, v in body.items() if k != "model"}).status_code == 422
    assert requests.post(server + "/v1/systemone", json={**body, "max_reasoning_tokens": 0}).status_code == 422
    alias = requests.post(server + "/v1/decide", json={"request": {k: body[k] for k in ("state", "questions")}})
    assert alias.status_code == 200 and set(alias.json()["answers"]) == {"q1", "q2", "q3"}
    assert alias.headers.get("Deprecation") == "true"
    assert requests.post(server + "/v1/decide", json={"state": {}}).status_code == 400


def test_systemone_concurrent_requests_share_forwards_and_reason(server):
    """Concurrent requests are packed into shared forwards and answered as if scored alone;
    reasoning first writes text with the generation engine and reports how it was used."""
    from concurrent.futures import ThreadPoolExecutor
    bodies = [{"model": "m", "state": {"user": f"t{i} t{i + 1}"}, "questions": {
        "q": {"type": "choice", "criteria": {"a": "t3", "b": "t4"}},
        "n": {"type": "noul"}}} for i in range(6)]
    alone = [requests.post(server + "/v1/systemone", json=b).json()["answers"] for b in bodies]
    with ThreadPoolExecutor(6) as ex:
        together = [r.json()["answers"] for r in ex.map(lambda b: requests.post(server + "/v1/systemone", json=b),
                                                          bodies)]
    for a, b in zip(alone, together):
        assert a["q"]["choice"] == b["q"]["choice"]
        assert abs(a["n"]["noul"] - b["n"]["noul"]) < 1e-3
    r = requests.post(server + "/v1/systemone", json={**bodies[0], "reasoning": True, "max_reasoning_tokens": 4})
    assert r.status_code == 200, r.text
    out = r.json()
    assert "reasoning" in out and out["answers_source"] in ("direct", "reasoned")
    assert out["usage"]["output_tokens"] <= 4
    if out["answers_source"] == "direct":
        assert out["cut"] in ("length", "empty", "state_limit")


def test_eval_client_task_sweep_and_merge(server, tmp_path):
    """eval.py against the served engine: a local GSM8K file, the summary fields, tokens per forward
    from /v1/stats, the fixed-output sweep (ignore_eos) and shard merging."""
    import eval as E
    port = int(server.rsplit(":", 1)[1])
    data = tmp_path / "gsm8k.jsonl"
    data.write_text("\n".join(json.dumps({"question": f"t{i} t{i + 1}", "answer": f"x #### {i}"}) for i in range(4)))
    outs = []
    for shard in ("0/2", "1/2"):
        out = tmp_path / f"r{shard[0]}"
        s = E.main(["gsm8k", "--data", str(data), "--port", str(port), "--max-tokens", "6", "--max-workers", "2",
                    "--shard", shard, "--out", str(out)])
        assert s["n"] == 2 and s["errors"] == 0 and s["forward"]["tok_per_fwd"] is not None
        assert (out / "requests.jsonl").exists()
        outs.append(str(out))
    merged = E.merge(outs)
    assert merged["n"] == 4 and merged["shards"] == 2
    res = E.main(["sweep", "--data", str(data), "--port", str(port), "--concurrency", "1", "2", "--limit", "2",
                  "--warmup", "0", "--max-tokens", "5"])
    assert [r["concurrency"] for r in res] == [1, 2]
    assert all(r["n_ok"] == 2 and r["tokens"] == 10 for r in res)     # ignore_eos: exactly max_tokens each
    st = requests.get(server + "/v1/stats").json()
    assert st["forwards"] > 0 and st["tokens"] > 0


def test_router_fails_over_and_streams(server):
    """Data-parallel router: a dead replica is skipped, streamed answers pass through, stats add up."""
    import uvicorn

    from trida_stack_b200.serve.router import build_app
    dead = f"http://127.0.0.1:{_free_port()}"
    port = _free_port()
    srv = uvicorn.Server(uvicorn.Config(build_app([dead, server], timeout=60), host="127.0.0.1", port=port,
                                        log_level="error"))
    threading.Thread(target=srv.run, daemon=True).start()
    url = f"http://127.0.0.1:{port}"
    for _ in range(200):
        try:
            if requests.get(url + "/health", timeout=1).ok:
                break
        except requests.ConnectionError:
            time.sleep(0.05)
    try:
        for _ in range(3):
            r = requests.post(url + "/v1/chat/completions",
                              json={"messages": [{"role": "user", "content": "t5 t6"}], "max_tokens": 4}).json()
            assert r["object"] == "chat.completion"
        with requests.post(url + "/v1/chat/completions", stream=True,
                           json={"messages": [{"role": "user", "content": "t7"}], "max_tokens": 4,
                                 "stream": True}) as r:
            lines = [l for l in r.iter_lines(decode_unicode=True) if l]
        assert lines[-1] == "data: [DONE]"
        assert requests.get(url + "/v1/stats").json()["replicas"] == 1
        assert requests.get(url + "/v1/models").json()["data"]
    finally:
        srv.should_exit = True


def test_chat_with_tools_request_path(server):
    """The request ``eval_fc.py`` sends (functions as OpenAI tools, greedy) is served; a random tiny
    model emits no call, which scores as incorrect rather than failing."""
    from trida_stack_b200.evals.function_call import score_case, to_openai_tools
    funcs = [{"name": "lookup", "description": "find", "parameters": {
        "type": "dict", "properties": {"city": {"type": "string"}}, "required": ["city"]}}]
    r = requests.post(server + "/v1/chat/completions", json={
        "messages": [{"role": "user", "content": "t1 t2"}], "tools": to_openai_tools(funcs), "max_tokens": 4,
        "temperature": 0}).json()
    msg = r["choices"][0]["message"]
    res = score_case({"id": "simple_python_0", "function": funcs}, {"ground_truth": [{"lookup": {"city": ["x"]}}]},
                     msg)
    assert res["correct"] is False and res["category"] == "simple_python"


def test_decision_answer_shapes_and_confidence():
    from trida_stack_b200.serve.decide import confidence, systemone_response, to_answer, with_reasoning
    assert abs(confidence("choice", [0.5, 0.25, 0.25]) - 0.25) < 1e-9
    assert confidence("choice", [1 / 3] * 3) == 0.0 and confidence("choice", [1.0]) == 1.0
    assert confidence("score", [0.0, 1.0, 0.0]) == 1.0
    assert abs(confidence("score", [1 / 3] * 3)) < 1e-9
    q = {"qtype": "score", "options": ["low", "high"], "keys": ["0", "1"]}
    a = to_answer(q, [0.25, 0.75])
    assert a == {"type": "score", "score": 0.75, "legend": ["low", "high"], "confidence": 0.5,
                 "probabilities": {"0": 0.25, "1": 0.75}}
    assert to_answer({"qtype": "noul", "options": [], "keys": ["false", "true"]}, [0.3, 0.7]) == \
        {"type": "noul", "noul": 0.7}
    r = systemone_response({"answers": {"s": a}, "usage": {"input_tokens": 9}, "timing_ms": 1.0}, "m")
    assert r["answers"]["s"]["legend"] == {"0": "low", "1": "high"} and r["timing_ms"] == 1.0
    assert r["usage"] == {"input_tokens": 9, "output_tokens": 0}
    assert with_reasoning({"state": "x", "questions": {}}, "why")["state"] == {"situation": "x", "reasoning": "why"}
    assert with_reasoning({"state": {"a": 1}, "questions": {}}, "why")["state"] == {"a": 1, "reasoning": "why"}


CHAT_TEMPLATE = ("{% for m in messages %}<|im_start|>{{ m['role'] }}\n{{ m['content'] }}<|im_end|>\n{% endfor %}"
                 "{% if add_generation_prompt %}<|im_start|>assistant\n{% endif %}")


def test_selfdistill_regenerates_assistant_turns(server, tmp_path):
    """Self-distillation over the served engine: token-id prompts reach /v1/completions (a tiny random
    model runs out of budget, so those conversations are dropped as truncated), and with a stand-in
    completion every assistant turn is regenerated in order and round-trips."""
    import asyncio

    from trida_stack_b200.selfdistill import Distiller, select_rows
    from helpers import make_tokenizer
    tok = make_tokenizer(str(tmp_path / "tok"), 295)
    tok.chat_template = CHAT_TEMPLATE
    conv = {"id": "c", "messages": [{"role": "user", "content": "t1 t2"}, {"role": "assistant", "content": "t3"},
                                    {"role": "user", "content": "t4"}, {"role": "assistant", "content": "t5 t6"}]}
    src = tmp_path / "src"
    src.mkdir()
    (src / "chunk-000.jsonl").write_text("\n".join(json.dumps(dict(conv, id=str(i))) for i in range(6)) + "\n")
    rows = list(select_rows(str(src), 2, 1, 2))
    assert [r["id"] for r in rows] == ["2", "4"]
    port = int(server.rsplit(":", 1)[1])
    out = tmp_path / "o.jsonl"
    d = Distiller(tok, [port], max_tokens=4, ctx_len=64, per_port=2, out=str(out))
    d.max_tokens, d.ctx_len = 4, 64
    with open(out, "w") as fo:
        st = asyncio.run(d.run(rows, fo))
    assert st["conv"] == 2 and st["errors"] == 0 and st["kept"] + st["truncated"] == 2

    seen = []

    async def fake_complete(sess, sems, prompt_ids):
        seen.append(list(prompt_ids))
        text = f"t{7 + len(seen)} t9"
        return text, "stop", tok(text, add_special_tokens=False).input_ids
    d2 = Distiller(tok, [port], out=str(out))
    d2.complete = fake_complete
    with open(out, "w") as fo:
        st = asyncio.run(d2.run([conv], fo))
    res = json.loads(out.read_text().splitlines()[0])
    assert st["kept"] == 1 and st["turns"] == 2
    assert res["messages"][1]["content"].endswith("t8 t9") and res["messages"][3]["content"].endswith("t9 t9")
    assert res["messages"][2]["content"] == "t4"
    # the second prompt holds the regenerated first turn, not the original
    assert tok("t8", add_special_tokens=False).input_ids[0] in seen[1]
