"""Typed decisions (``--mode decide``): System One requests -> pointer-head answers.

A request ``{"state": any JSON, "questions": {qid: {"type": "noul" | "choice" | "score",
"instructions"?, "criteria"}}}`` becomes one causal row per question, rendered and tokenised
exactly as the decision training rows (``data.decision.encode_rows``):
``<state> state <q> instructions <opt> o1 </opt> ... <decide>``.  One causal forward of the rows
gives the last-layer states at every ``</opt>`` and at ``<decide>``; the pointer head scores the
options, a per-type temperature (``temperature.json`` next to the checkpoint, default 1) scales
the scores and the softmax gives the answer.  Reference: ``inference/zoro-1/decide_request.py``
(validation / rendering), ``decide_engine.py:62-173`` (head read-out), ``serve_decide.py:202-240``
(HTTP shapes).
"""
import json
import os
import time

import torch

from ..data.decision import ContextOverflow, encode_rows, option_text, question_keys, render

QTYPES = ("noul", "choice", "score")
MAX_OPTIONS = 255


class RequestError(ValueError):
    """A malformed request; ``loc`` is the JSON path of the offending field."""

    def __init__(self, msg, loc=()):
        super().__init__(msg)
        self.loc = list(loc)

    def detail(self):
        return [{"loc": ["body"] + self.loc, "msg": str(self), "type": "value_error"}]


def parse(body):
    """Validate a System One body; returns the materialised request (no labels)."""
    if not isinstance(body, dict):
        raise RequestError("request body must be a JSON object")
    if "state" not in body:
        raise RequestError("field required", ["state"])
    qs = body.get("questions")
    if not isinstance(qs, dict) or not qs:
        raise RequestError("questions must be a non-empty object", ["questions"])
    out = []
    for qid, q in qs.items():
        loc = ["questions", qid]
        if not isinstance(q, dict):
            raise RequestError("a question must be an object", loc)
        qt = q.get("type")
        if qt not in QTYPES:
            raise RequestError(f"type must be one of {', '.join(QTYPES)}", loc + ["type"])
        crit = q.get("criteria")
        if qt == "noul":
            if crit is not None and (not isinstance(crit, dict) or set(crit) - {"true", "false"}):
                raise RequestError("noul criteria must be {'true': ..., 'false': ...}", loc + ["criteria"])
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
            raise RequestError(f"at most {MAX_OPTIONS} options", loc + ["criteria"])
        out.append({"instr": render(q.get("instructions")), "options": options, "qid": qid, "qtype": qt,
                    "keys": question_keys(qt, crit if qt != "noul" else None), "label": 0,
                    "criteria": crit})
    return {"state": render(body["state"]), "questions": out}


class DecideEngine:
    def __init__(self, model, tokenizer, temperatures=None, max_state=7552, max_branch=8192):
        """``model``: a BlockDiffusionLM / HybridBlockDiffusionLM with a decision head."""
        if model.decision_head is None:
            raise ValueError("decide mode needs a checkpoint with a decision head (decision_head.pt)")
        from ..data.decision import SPECIAL
        missing = [t for t in SPECIAL if tokenizer.convert_tokens_to_ids(t) in (None, tokenizer.unk_token_id)]
        if missing:
            raise ValueError(f"tokenizer lacks the decision control tokens {missing}")
        self.model, self.tok = model, tokenizer
        self.temps = {"noul": 1.0, "choice": 1.0, "score": 1.0}
        self.temps.update(temperatures or {})
        self.max_state, self.max_branch = max_state, max_branch

    @classmethod
    def temperatures_from(cls, path):
        f = os.path.join(path, "temperature.json") if path else None
        if f and os.path.isfile(f):
            with open(f) as fh:
                return {k: float(v) for k, v in json.load(fh).items()}
        return None

    @torch.no_grad()
    def decide(self, body):
        t0 = time.perf_counter()
        req = parse(body)
        try:
            rows = encode_rows(self.tok, req, self.max_state, self.max_branch)
        except ContextOverflow as e:
            raise RequestError(str(e), ["state"])
        m = self.model
        dev = next(m.decoder.parameters()).device
        answers, n_in = {}, 0
        for q, row in zip(req["questions"], rows):
            ids = torch.tensor([row["ids"]], device=dev)
            n_in += len(row["ids"])
            actx = m._causal_rows(ids, None) if hasattr(m, "_causal_rows") else None
            if actx is None:
                raise RuntimeError("model has no causal-row layout")
            h = m.decoder(m.decoder.embed_tokens(ids), actx).view(-1, m.decoder.cfg.hidden_size)
            z = m.decision_head(h[row["decide"]][None], h[row["opts"]], torch.zeros(len(row["opts"]), dtype=torch.long,
                                                                                   device=dev))
            z = z.float().reshape(-1) / self.temps.get(q["qtype"], 1.0)
            p = torch.softmax(z, -1).tolist()
            answers[q["qid"]] = self._answer(q, p)
        return {"answers": answers, "usage": {"input_tokens": n_in, "output_tokens": 0},
                "timing_ms": round((time.perf_counter() - t0) * 1e3, 2)}

    @staticmethod
    def _answer(q, p):
        best = max(range(len(p)), key=lambda i: p[i])
        if q["qtype"] == "noul":
            return {"noul": bool(best == 1), "confidence": p[best], "probabilities": {"false": p[0], "true": p[1]}}
        if q["qtype"] == "choice":
            keys = q["keys"]
            return {"choice": keys[best], "confidence": p[best], "probabilities": dict(zip(keys, p))}
        legend = [render(x) for x in q["criteria"]]
        return {"score": best, "confidence": p[best], "legend": legend, "probabilities": p}
