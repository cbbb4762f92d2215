"""Function-calling accuracy by AST match (the scoring behind BFCL's non-live categories).

The reference drives the Berkeley Function-Calling Leaderboard package against its server
(``benchmark/bfcl_v4/run_eval.sh``, ``benchmark/bfcl_v4/trida_handler.py``); that package is not part
of this repository.  This module reads the same data layout and scores the model's OpenAI
``tool_calls`` itself:

* question file (JSONL): ``{"id", "question": [[{"role", "content"}, ...]], "function": [schema, ...]}``
  where a schema is ``{"name", "description", "parameters": {"type": "dict", "properties", "required"}}``;
* answer file (JSONL): ``{"id", "ground_truth": [{"<function name>": {"<arg>": [acceptable, ...]}}]}``.
  An empty string among the acceptable values marks the argument as optional.

A response is correct when its calls and the ground-truth calls can be paired one to one (any order
for ``parallel*`` ids, exactly one call otherwise) so that each pair has the same function name,
every required argument is present, no argument outside the schema appears, and every value matches
one acceptable value: numbers by value (an integer is accepted where a float is expected), strings
case-insensitively with whitespace and the punctuation ``,./-_*^`` removed, lists element by element
in order, dicts key by key.
"""
import json
import re

_STRIP = re.compile(r"[\s,./\-_*^]")


def to_openai_tools(functions):
    """BFCL function docs -> OpenAI ``tools`` (``"dict"`` schemas become JSON-schema objects)."""
    def fix(node):
        if isinstance(node, dict):
            out = {k: fix(v) for k, v in node.items()}
            if out.get("type") == "dict":
                out["type"] = "object"
            elif out.get("type") == "float":
                out["type"] = "number"
            elif out.get("type") == "tuple":
                out["type"] = "array"
            return out
        if isinstance(node, list):
            return [fix(v) for v in node]
        return node
    return [{"type": "function", "function": {"name": f["name"], "description": f.get("description", ""),
                                              "parameters": fix(f.get("parameters", {"type": "dict", "properties": {}}))}}
            for f in functions]


def _norm_str(s):
    return _STRIP.sub("", str(s)).casefold()


def value_matches(got, acc, schema=None):
    """One model value against one acceptable value (``schema``: the parameter's JSON schema)."""
    ptype = (schema or {}).get("type")
    if isinstance(acc, bool) or isinstance(got, bool):
        return isinstance(got, bool) and isinstance(acc, bool) and got == acc
    if isinstance(acc, (int, float)):
        if isinstance(got, str):
            try:
                got = float(got)
            except ValueError:
                return False
        if not isinstance(got, (int, float)):
            return False
        if ptype == "integer" and isinstance(got, float) and not got.is_integer():
            return False
        return abs(float(got) - float(acc)) <= 1e-9 * max(1.0, abs(float(acc)))
    if isinstance(acc, str):
        return isinstance(got, str) and _norm_str(got) == _norm_str(acc)
    if isinstance(acc, (list, tuple)):
        if not isinstance(got, (list, tuple)) or len(got) != len(acc):
            return False
        item = (schema or {}).get("items")
        return all(value_matches(g, a, item) for g, a in zip(got, acc))
    if isinstance(acc, dict):
        if not isinstance(got, dict) or set(got) != set(acc):
            return False
        props = (schema or {}).get("properties", {})
        # nested dict values in BFCL answers are themselves lists of acceptable values
        return all(any(value_matches(got[k], a, props.get(k)) for a in (v if isinstance(v, list) else [v]))
                   for k, v in acc.items())
    return got == acc


def call_matches(name, args, truth, functions):
    """One model call (``name``, parsed ``args``) against one ground-truth entry ``{fname: {arg: [..]}}``."""
    (tname, targs), = truth.items()
    if name != tname and name.replace("_", ".") != tname and name != tname.replace(".", "_"):
        return False
    schema = next((f.get("parameters", {}) for f in functions if f["name"] == tname), {})
    props, required = schema.get("properties", {}), set(schema.get("required", []))
    if not isinstance(args, dict) or any(k not in props for k in args):
        return False
    if any(k not in args for k in required):
        return False
    for k, acceptable in targs.items():
        if k not in args:
            if "" not in acceptable:
                return False
            continue
        if not any(value_matches(args[k], a, props.get(k)) for a in acceptable if a != ""):
            return False
    return True


def calls_match(calls, truths, functions, parallel):
    """``calls``: [(name, args)].  Order-free one-to-one pairing for parallel categories."""
    if len(calls) != len(truths) or (not parallel and len(calls) != 1):
        return False
    used = [False] * len(truths)

    def assign(i):
        if i == len(calls):
            return True
        for j, t in enumerate(truths):
            if not used[j] and call_matches(calls[i][0], calls[i][1], t, functions):
                used[j] = True
                if assign(i + 1):
                    return True
                used[j] = False
        return False
    return assign(0)


def parse_response_calls(message):
    """OpenAI ``message.tool_calls`` -> [(name, args)]; arguments that are not JSON objects score 0."""
    out = []
    for c in (message or {}).get("tool_calls") or []:
        fn = c.get("function", {})
        raw = fn.get("arguments", "{}")
        try:
            args = json.loads(raw) if isinstance(raw, str) else raw
        except json.JSONDecodeError:
            args = None
        out.append((fn.get("name", ""), args))
    return out


def category(case_id):
    """BFCL ids look like ``simple_python_12`` / ``parallel_multiple_3``: the prefix names the category."""
    return re.sub(r"_\d+$", "", case_id)


def score_case(case, answer, message):
    calls = parse_response_calls(message)
    parallel = category(case["id"]).startswith("parallel")
    ok = calls_match(calls, answer["ground_truth"], case["function"], parallel)
    return {"id": case["id"], "category": category(case["id"]), "correct": bool(ok),
            "calls": [{"name": n, "arguments": a} for n, a in calls]}


def summarize(results):
    by = {}
    for r in results:
        c = by.setdefault(r["category"], [0, 0])
        c[0] += int(r["correct"])
        c[1] += 1
    cats = {k: {"accuracy": round(v[0] / v[1], 4), "n": v[1]} for k, v in sorted(by.items())}
    n = sum(v[1] for v in by.values())
    return {"accuracy": round(sum(v[0] for v in by.values()) / n, 4) if n else None, "n": n, "categories": cats}
