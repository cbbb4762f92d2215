"""Function-calling AST scoring (BFCL layout) and the ``eval_fc.py`` client against a stub server."""
import json
import threading
from http.server import BaseHTTPRequestHandler, HTTPServer

from trida_stack_b200.evals.function_call import (calls_match, score_case, summarize, to_openai_tools,
                                                  value_matches)

FUNCS = [{"name": "calc.area", "description": "area", "parameters": {"type": "dict", "properties": {
    "base": {"type": "integer"}, "height": {"type": "float"}, "unit": {"type": "string"},
    "dims": {"type": "array", "items": {"type": "integer"}}}, "required": ["base", "height"]}},
    {"name": "lookup", "description": "find", "parameters": {"type": "dict", "properties": {
        "city": {"type": "string"}}, "required": ["city"]}}]
TRUTH = {"calc.area": {"base": [10], "height": [5.0], "unit": ["cm", ""], "dims": [[1, 2], ""]}}


def test_values_and_calls():
    assert value_matches(5, 5.0, {"type": "float"}) and not value_matches(5.5, 5, {"type": "integer"})
    assert value_matches("New York, NY", "new york ny") and not value_matches("Boston", "new york")
    assert value_matches([1, 2], [1, 2]) and not value_matches([2, 1], [1, 2])
    assert value_matches(True, True) and not value_matches(1, True)
    assert calls_match([("calc.area", {"base": 10, "height": 5})], [TRUTH], FUNCS, False)
    assert calls_match([("calc_area", {"base": 10, "height": 5, "unit": "CM"})], [TRUTH], FUNCS, False)
    assert not calls_match([("calc.area", {"base": 10})], [TRUTH], FUNCS, False)                 # required
    assert not calls_match([("calc.area", {"base": 10, "height": 5, "colour": "x"})], [TRUTH], FUNCS, False)
    assert not calls_match([("calc.area", {"base": 11, "height": 5})], [TRUTH], FUNCS, False)    # value
    assert not calls_match([("lookup", {"city": "x"})], [TRUTH], FUNCS, False)                   # name
    two = [{"lookup": {"city": ["Paris"]}}, {"lookup": {"city": ["Rome"]}}]
    assert calls_match([("lookup", {"city": "rome"}), ("lookup", {"city": "Paris"})], two, FUNCS, True)
    assert not calls_match([("lookup", {"city": "rome"})], two, FUNCS, True)
    assert not calls_match([("lookup", {"city": "Paris"}), ("lookup", {"city": "Paris"})], two, FUNCS, True)
    tools = to_openai_tools(FUNCS)
    assert tools[0]["function"]["parameters"]["type"] == "object"
    assert tools[0]["function"]["parameters"]["properties"]["height"]["type"] == "number"


def test_score_and_summary():
    case = {"id": "simple_python_3", "function": FUNCS}
    good = {"tool_calls": [{"function": {"name": "calc.area", "arguments": json.dumps({"base": 10, "height": 5})}}]}
    bad = {"tool_calls": [{"function": {"name": "calc.area", "arguments": "{not json"}}]}
    r1 = score_case(case, {"ground_truth": [TRUTH]}, good)
    r2 = score_case(dict(case, id="simple_python_4"), {"ground_truth": [TRUTH]}, bad)
    r3 = score_case(dict(case, id="multiple_1"), {"ground_truth": [TRUTH]}, {"content": "no call"})
    assert r1["correct"] and not r2["correct"] and not r3["correct"]
    s = summarize([r1, r2, r3])
    assert s["n"] == 3 and abs(s["accuracy"] - 1 / 3) < 1e-3
    assert s["categories"]["simple_python"] == {"accuracy": 0.5, "n": 2}


class _Stub(BaseHTTPRequestHandler):
    def do_POST(self):
        body = json.loads(self.rfile.read(int(self.headers["Content-Length"])))
        assert body["tools"][0]["type"] == "function"
        text = body["messages"][-1]["content"]
        calls = [] if "skip" in text else [{"id": "c0", "type": "function", "function": {
            "name": "lookup", "arguments": json.dumps({"city": text.split()[-1]})}}]
        msg = {"role": "assistant", "content": None if calls else "none", "tool_calls": calls or None}
        data = json.dumps({"choices": [{"message": msg, "finish_reason": "tool_calls"}]}).encode()
        self.send_response(200)
        self.send_header("Content-Type", "application/json")
        self.send_header("Content-Length", str(len(data)))
        self.end_headers()
        self.wfile.write(data)

    def log_message(self, *a):
        pass


def test_eval_fc_client_end_to_end(tmp_path):
    import eval_fc
    srv = HTTPServer(("127.0.0.1", 0), _Stub)
    threading.Thread(target=srv.serve_forever, daemon=True).start()
    qs = [{"id": f"simple_python_{i}", "question": [[{"role": "user", "content": f"weather in {c}"}]],
           "function": FUNCS} for i, c in enumerate(["Paris", "Rome", "skip"])]
    ans = [{"id": f"simple_python_{i}", "ground_truth": [{"lookup": {"city": [c]}}]}
           for i, c in enumerate(["Paris", "Oslo", "Rome"])]
    (tmp_path / "q.jsonl").write_text("\n".join(json.dumps(q) for q in qs))
    (tmp_path / "a.jsonl").write_text("\n".join(json.dumps(a) for a in ans))
    rc = eval_fc.main(["--questions", str(tmp_path / "q.jsonl"), "--answers", str(tmp_path / "a.jsonl"),
                       "--port", str(srv.server_address[1]), "--out", str(tmp_path / "out"), "--max-workers", "2"])
    srv.shutdown()
    assert rc == 0
    summary = json.loads((tmp_path / "out" / "summary.json").read_text())
    assert summary["n"] == 3 and abs(summary["accuracy"] - 1 / 3) < 1e-3 and summary["errors"] == 0
    rows = [json.loads(l) for l in open(tmp_path / "out" / "responses.jsonl")]
    assert sorted(r["correct"] for r in rows) == [False, False, True]
