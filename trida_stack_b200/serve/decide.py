"""Typed decisions (``--mode decide``): System One requests -> pointer-head answers.

A request ``{"state": any JSON, "questions": {qid: {"type": "noul" | "choice" | "score",
"instructions"?, "criteria"}}}`` becomes one causal row per question, rendered and tokenised
exactly as the decision training rows (``data.decision.encode_rows``):
``<state> state <q> instructions <opt> o1 </opt> ... <decide>``.  The pointer head scores every
``</opt>`` state against the ``<decide>`` state; ``softmax(z / T)`` gives the option
probabilities (T: the request's ``temperature``, else the checkpoint's ``temperature.json``).

Batching: the rows of every question of every request waiting at that moment are packed into ONE
document-isolated causal row (``data.decision.pack_decision``) and scored by one forward of the
decoder and one head call; a request never waits more than ``window_ms`` for others to join.

Reason, then decide (``reasoning: true``): the model first writes its reasoning about the
request (the serving engine's causal decoding, stopped at ``</think>`` or after
``max_reasoning_tokens``); the reasoning's conclusion is added to the state (trimmed from the front
to the state budget) and the decision rows are scored on that.  ``cut`` reports why the direct
answers were used instead: ``length`` (budget ran out), ``empty`` or ``state_limit``.

Wire contract (the reference's System One envelope and answer shapes,
``inference/zoro-1/decide_request.py:216-431``, ``decide_engine.py:162-200``,
``serve_decide.py:202-240``): ``noul`` answers are P(true); ``choice`` answers name the most
likely key with a confidence rescaled so that a uniform distribution is 0; ``score`` answers are
the expected level with a confidence of 1 minus the mean distance from the mode, relative to a
uniform distribution's.
"""
import json
import math
import os
import queue
import threading
import time

import torch

from ..data.decision import ContextOverflow, encode_rows, option_text, pack_decision, question_keys, render

QTYPES = ("noul", "choice", "score")
MAX_OPTIONS = 255
REQUEST_KEYS = {"state", "questions", "image", "min_image_pixels", "max_image_pixels"}
SYSTEMONE_EXTENSIONS = ("reasoning", "max_reasoning_tokens", "temperature")
MAX_REASONING_TOKENS = 8192
END_THINK = "</think>"
REASONING_INSTRUCTION = ("Think it through step by step: work out anything that needs calculating or checking, then "
                         "say which option you choose for each question.")


class RequestError(ValueError):
    """A malformed request; ``loc`` is the JSON path of the offending field."""

    def __init__(self, msg, loc=()):
        super().__init__(msg)
        self.loc = list(loc)

    def detail(self):
        return [{"loc": ["body"] + self.loc, "msg": str(self), "type": "value_error"}]


def _finite_positive(v):
    return not isinstance(v, bool) and isinstance(v, (int, float)) and math.isfinite(v) and v > 0


# ---------------------------------------------------------------------------------------------
# request
# ---------------------------------------------------------------------------------------------
def _question(qid, q):
    loc = ["questions", qid]
    if not isinstance(q, dict):
        raise RequestError("a question must be an object with a type and criteria", loc)
    qt = q.get("type")
    if qt not in QTYPES:
        raise RequestError(f"type must be one of {', '.join(QTYPES)}", loc + ["type"])
    crit = q.get("criteria")
    if qt == "noul":
        if crit is not None and (not isinstance(crit, dict) or set(crit) - {"true", "false"}):
            raise RequestError("noul criteria are optional and may only have 'true' and 'false'", loc + ["criteria"])
        crit = crit or {}
        options = [option_text("no", crit.get("false")), option_text("yes", crit.get("true"))]
    elif qt == "choice":
        if not isinstance(crit, dict) or not crit:
            raise RequestError("choice criteria must be a non-empty object {key: description}", loc + ["criteria"])
        options = [option_text(k, v) for k, v in crit.items()]
    else:
        if not isinstance(crit, list) or not crit:
            raise RequestError("score criteria must be a non-empty list of levels, lowest first", loc + ["criteria"])
        options = [render(x) for x in crit]
    if len(options) > MAX_OPTIONS:
        raise RequestError(f"{len(options)} options; at most {MAX_OPTIONS}", loc + ["criteria"])
    return {"instr": render(q.get("instructions")), "options": options, "qid": qid, "qtype": qt,
            "keys": question_keys(qt, crit if qt != "noul" else None), "label": 0, "criteria": crit}


def parse(body):
    """Validate a decision request; returns the materialised request (no labels)."""
    if not isinstance(body, dict):
        raise RequestError("a request must be an object with 'state' and 'questions'")
    unknown = set(body) - REQUEST_KEYS
    if unknown:
        raise RequestError(f"unknown request keys {sorted(unknown)}; allowed: {sorted(REQUEST_KEYS)}")
    if "state" not in body:
        raise RequestError("field required", ["state"])
    qs = body.get("questions")
    if not isinstance(qs, dict) or not qs:
        raise RequestError("questions must be a non-empty object", ["questions"])
    if body.get("image") is not None:
        raise RequestError("this server scores text decision rows; image states are not accepted", ["image"])
    return {"state": render(body["state"]), "questions": [_question(qid, q) for qid, q in qs.items()]}


def systemone_request(body, reasoning_token_limit=4096):
    """System One body -> (decision request, {extension: value}).  The body needs ``state``,
    ``model`` and ``questions``; unknown top-level keys are ignored; ``images`` takes at most one
    entry; the extensions ``reasoning`` (bool), ``max_reasoning_tokens`` (1 .. limit) and
    ``temperature`` (> 0) are checked here, null meaning unset."""
    if not isinstance(body, dict):
        raise RequestError("the body must be an object with 'state', 'model' and 'questions'")
    for key in ("state", "model", "questions"):
        if key not in body:
            raise RequestError("field required", [key])
    if not isinstance(body["model"], str) or not body["model"].strip():
        raise RequestError("'model' must be a non-empty string", ["model"])
    request = {k: body[k] for k in ("state", "questions", "min_image_pixels", "max_image_pixels") if k in body}
    images = body.get("images") or []
    if not isinstance(images, list):
        raise RequestError("'images' must be a list", ["images"])
    if len(images) > 1:
        raise RequestError(f"'images' has {len(images)} entries; at most one image per request", ["images"])
    if images:
        request["image"] = images[0].get("url") if isinstance(images[0], dict) else images[0]
    opts = {k: body[k] for k in SYSTEMONE_EXTENSIONS if body.get(k) is not None}
    if "reasoning" in opts and not isinstance(opts["reasoning"], bool):
        raise RequestError("'reasoning' must be true or false", ["reasoning"])
    b = opts.get("max_reasoning_tokens")
    if b is not None and (type(b) is not int or not 1 <= b <= reasoning_token_limit):
        raise RequestError(f"'max_reasoning_tokens' must be an integer from 1 to {reasoning_token_limit}",
                           ["max_reasoning_tokens"])
    if "temperature" in opts and not _finite_positive(opts["temperature"]):
        raise RequestError("'temperature' must be a finite number above 0", ["temperature"])
    return request, opts


# ---------------------------------------------------------------------------------------------
# answers
# ---------------------------------------------------------------------------------------------
def confidence(qtype, p):
    """1 for a certain answer, 0 for a uniform one.  Choice: (max p - 1/k) / (1 - 1/k).  Score: one
    minus the mean distance of the levels from the most likely level, divided by that distance for a
    uniform distribution (the mean distance of the levels from the middle)."""
    k = len(p)
    if k == 1:
        return 1.0
    if qtype == "score":
        mode = max(range(k), key=lambda i: p[i])
        spread = sum(abs(i - (k - 1) / 2) for i in range(k)) / k
        return max(0.0, 1.0 - sum(pi * abs(i - mode) for i, pi in enumerate(p)) / spread)
    return (max(p) - 1.0 / k) / (1.0 - 1.0 / k)


def to_answer(q, p):
    """Question + option probabilities -> the reported answer (values rounded to 4 places)."""
    r4 = lambda x: round(float(x), 4)   # noqa: E731
    if q["qtype"] == "noul":
        return {"type": "noul", "noul": r4(p[1])}
    if q["qtype"] == "choice":
        keys = q["keys"]
        return {"type": "choice", "choice": keys[max(range(len(p)), key=lambda i: p[i])],
                "confidence": r4(confidence("choice", p)), "probabilities": {k: r4(v) for k, v in zip(keys, p)}}
    return {"type": "score", "score": r4(sum(i * x for i, x in enumerate(p))), "legend": list(q["options"]),
            "confidence": r4(confidence("score", p)), "probabilities": {str(i): r4(v) for i, v in enumerate(p)}}


def systemone_response(result, model):
    """Decision result -> System One response: score legends become {"0": level, ...}; fields other
    than answers / usage (timing, reasoning) are kept."""
    def answer(a):
        if a.get("type") == "score" and isinstance(a.get("legend"), list):
            return {**a, "legend": {str(i): lv for i, lv in enumerate(a["legend"])}}
        return a
    usage = result.get("usage") or {}
    return {"model": model, "answers": {qid: answer(a) for qid, a in result["answers"].items()},
            "usage": {"input_tokens": int(usage.get("input_tokens", 0)),
                      "output_tokens": int(usage.get("output_tokens", 0))},
            **{k: v for k, v in result.items() if k not in ("answers", "usage", "model")}}


# ---------------------------------------------------------------------------------------------
# reason, then decide
# ---------------------------------------------------------------------------------------------
def reasoning_prompt(body):
    """The user message the model reasons about: the state, then each question with its options
    (yes / no, the choice keys, or the numbered levels), then the instruction to conclude."""
    parts = [render(body["state"])]
    for qid, q in body["questions"].items():
        lines = [f"Question ({qid}): {render(q.get('instructions')) or qid}"]
        if q["type"] == "noul":
            lines.append("Answer yes or no.")
        elif q["type"] == "choice":
            lines.append("Options:")
            lines += [f"- {k}: {render(v)}" if v not in (None, "") else f"- {k}" for k, v in q["criteria"].items()]
        else:
            lines.append("Levels, lowest first:")
            lines += [f"{i}. {render(v)}" for i, v in enumerate(q["criteria"])]
        parts.append("\n".join(lines))
    return "\n\n".join(parts + [REASONING_INSTRUCTION])


def with_reasoning(body, text):
    """The request with the reasoning added to its state (a dict state gains a ``reasoning`` key;
    any other state becomes ``{"situation": state, "reasoning": text}``)."""
    state = body["state"]
    state = {**state, "reasoning": text} if isinstance(state, dict) else {"situation": state, "reasoning": text}
    return {**body, "state": state}


def fit_reasoning(body, text, tok, max_state, max_branch):
    """The longest tail of ``text`` (prefixed with an ellipsis when cut) whose state still fits the
    row budget next to the longest question branch; "" when not even one token fits."""
    from ..data.decision import user_tokens
    req = parse(body)
    sid_budget = max_state - 1
    longest = 0
    for q in req["questions"]:
        branch = 2 + len(user_tokens(tok, q["instr"])) + sum(len(user_tokens(tok, o)) + 2 for o in q["options"])
        longest = max(longest, branch)
    room = min(sid_budget, max_branch - longest - 1)

    def fits(candidate):
        return len(user_tokens(tok, render(with_reasoning(body, candidate)["state"]))) <= room

    if fits(text):
        return text
    ids = user_tokens(tok, text)
    lo, hi = 0, len(ids) + 1
    while hi - lo > 1:                      # binary search on the number of tail tokens kept
        mid = (lo + hi) // 2
        if fits("…" + tok.decode(ids[-mid:])):
            lo = mid
        else:
            hi = mid
    return "…" + tok.decode(ids[-lo:]) if lo else ""


# ---------------------------------------------------------------------------------------------
# packed scoring + micro-batching
# ---------------------------------------------------------------------------------------------
class _Job:
    __slots__ = ("rows", "result", "error", "done")

    def __init__(self, rows):
        self.rows, self.result, self.error = rows, None, None
        self.done = threading.Event()


class DecideEngine:
    """Pointer-head decisions over one decoder, with requests packed into shared forwards.

    ``gen_engine`` (the serving engine over the same decoder) writes the reasoning of
    ``reasoning=True`` requests; without it such requests are rejected."""

    def __init__(self, model, tokenizer, temperatures=None, max_state=7552, max_branch=8192, gen_engine=None,
                 reasoning_token_limit=4096, reasoning_temperature=0.6, window_ms=2.0, max_batch_tokens=65536):
        if model.decision_head is None:
            raise ValueError("decide mode needs a checkpoint with a decision head (decision_head.pt)")
        from ..data.decision import SPECIAL
        missing = [t for t in SPECIAL if tokenizer.convert_tokens_to_ids(t) in (None, tokenizer.unk_token_id)]
        if missing:
            raise ValueError(f"tokenizer lacks the decision control tokens {missing}")
        if not 1 <= reasoning_token_limit <= MAX_REASONING_TOKENS:
            raise ValueError(f"reasoning_token_limit must be between 1 and {MAX_REASONING_TOKENS}")
        self.model, self.tok = model, tokenizer
        t = temperatures or {}
        self.text_T, self.image_T = float(t.get("text", 1.0)), float(t.get("image", 1.0))
        self.max_state, self.max_branch = max_state, max_branch
        self.gen_engine = gen_engine
        self.reasoning_token_limit = reasoning_token_limit
        self.reasoning_temperature = reasoning_temperature
        self.window = window_ms / 1e3
        self.max_batch_tokens = max_batch_tokens
        self.stats = {"forwards": 0, "requests": 0, "rows": 0}
        self._jobs = queue.Queue()
        self._thread = None
        self._lock = threading.Lock()

    @classmethod
    def temperatures_from(cls, path):
        """``temperature.json`` next to the checkpoint: {"text": T, "image": T}."""
        f = os.path.join(path, "temperature.json") if path else None
        if f and os.path.isfile(f):
            with open(f) as fh:
                return {k: float(v) for k, v in json.load(fh).items()}
        return None

    # ---- scoring ------------------------------------------------------------------------------
    @torch.no_grad()
    def score(self, row_lists):
        """Rows of several requests -> per request, the option logits of each question: one packed
        causal forward (every question row its own document) and one pointer-head call."""
        m = self.model
        dev = next(m.decoder.parameters()).device
        pk = pack_decision(row_lists, self.tok)
        ids = pk["input_ids"].to(dev)
        actx = m._causal_rows(ids, pk["seg_id"].to(dev))
        h = m.run_stack(m.decoder.embed_tokens(ids), actx)
        z = m.decision_head(h[pk["decide"].to(dev)], h[pk["opts"].to(dev)], pk["owner"].to(dev)).float().cpu()
        self.stats["forwards"] += 1
        self.stats["rows"] += sum(len(r) for r in row_lists)
        out = [[] for _ in row_lists]
        for q in pk["questions"]:
            out[q["variant"]].append(z[q["start"]:q["start"] + q["k"]])
        return out

    def _serve(self):
        while True:
            jobs = [self._jobs.get()]
            deadline = time.perf_counter() + self.window
            used = sum(len(r["ids"]) for r in jobs[0].rows)
            while used < self.max_batch_tokens:
                try:
                    j = self._jobs.get(timeout=max(0.0, deadline - time.perf_counter()))
                except queue.Empty:
                    break
                jobs.append(j)
                used += sum(len(r["ids"]) for r in j.rows)
            try:
                res = self.score([j.rows for j in jobs])
                for j, r in zip(jobs, res):
                    j.result = r
            except Exception as e:     # hand the failure to every caller of this batch
                for j in jobs:
                    j.error = e
            for j in jobs:
                j.done.set()

    def _score_one(self, rows):
        with self._lock:
            if self._thread is None:
                self._thread = threading.Thread(target=self._serve, daemon=True)
                self._thread.start()
        job = _Job(rows)
        self._jobs.put(job)
        job.done.wait()
        if job.error is not None:
            raise job.error
        return job.result

    def _encode(self, body):
        req = parse(body)
        try:
            rows = encode_rows(self.tok, req, self.max_state, self.max_branch)
        except ContextOverflow as e:
            raise RequestError(str(e), ["state"])
        return req, rows

    # ---- requests -----------------------------------------------------------------------------
    def decide(self, body, temperature=None, reasoning=False, max_reasoning_tokens=None):
        """Decision request -> {"answers": {qid: answer}, "usage", "timing_ms"} (+ "reasoning",
        "reasoning_ms", "reasoning_stats", "answers_source" and maybe "cut" when ``reasoning``)."""
        if temperature is not None and not _finite_positive(temperature):
            raise RequestError("temperature must be a finite number above 0", ["temperature"])
        t0 = time.perf_counter()
        req, rows = self._encode(body)
        extra = {}
        if reasoning:
            text, stats = self.reason(body, max_reasoning_tokens)
            extra = {"reasoning": text, "reasoning_stats": stats,
                     "reasoning_ms": round((time.perf_counter() - t0) * 1e3, 1)}
            if stats["finish_reason"] != "stop":
                extra["cut"] = "length"
            elif not text:
                extra["cut"] = "empty"
            else:
                fitted = fit_reasoning(body, text, self.tok, self.max_state, self.max_branch)
                extra["reasoning_trimmed"] = fitted != text
                if not fitted:
                    extra["cut"] = "state_limit"
                else:
                    req, rows = self._encode(with_reasoning(body, fitted))
            extra["answers_source"] = "direct" if "cut" in extra else "reasoned"
        T = float(temperature) if temperature is not None else self.text_T
        z = self._score_one(rows)
        self.stats["requests"] += 1
        answers = {q["qid"]: to_answer(q, torch.softmax(zq / T, -1).tolist()) for q, zq in zip(req["questions"], z)}
        usage = {"input_tokens": sum(len(r["ids"]) for r in rows),
                 "output_tokens": extra.get("reasoning_stats", {}).get("completion_tokens", 0)}
        return {"answers": answers, "usage": usage, "timing_ms": round((time.perf_counter() - t0) * 1e3, 1), **extra}

    def reason(self, body, max_new_tokens=None):
        """The model's reasoning about the request (sampled at the reasoning temperature, top-p 0.95,
        top-k 20, until ``</think>`` / end of turn or the budget) -> (text, stats)."""
        from .engine import Request, SamplingParams
        if self.gen_engine is None:
            raise RequestError("this server has no generation engine for reasoning", ["reasoning"])
        if max_new_tokens is None:
            max_new_tokens = self.reasoning_token_limit
        if type(max_new_tokens) is not int or not 1 <= max_new_tokens <= self.reasoning_token_limit:
            raise RequestError(f"max_reasoning_tokens must be between 1 and {self.reasoning_token_limit}",
                               ["max_reasoning_tokens"])
        from .server import render_chat
        text = render_chat(self.tok, [{"role": "user", "content": reasoning_prompt(body)}])
        ids = self.tok(text, add_special_tokens=False).input_ids
        stops = tuple(t for t in (self.tok.convert_tokens_to_ids(END_THINK), self.tok.convert_tokens_to_ids("<|im_end|>"))
                      if isinstance(t, int) and t >= 0 and t != self.tok.unk_token_id)
        sp = SamplingParams(temperature=self.reasoning_temperature, top_k=20, top_p=0.95)
        eng = self.gen_engine
        if eng._thread is not None:        # the server's engine loop is running: queue and wait
            r = eng.submit(Request(list(ids), max_new_tokens, sp, stops))
            r.done_event.wait()
        else:
            r = eng.generate([ids], max_new_tokens=max_new_tokens, sampling=sp, eos=stops)[0]
        out = [t for t in r.output if t not in stops]
        text = self.tok.decode(out).replace(END_THINK, "").strip()
        return text, {"finish_reason": r.finish_reason or "unknown", "prompt_tokens": len(ids),
                      "completion_tokens": len(r.output)}
