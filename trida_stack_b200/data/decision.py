"""Typed-decision data (kev scheme; reference: ``train/data/decision.py``).

A request is a ``state`` plus typed questions (``noul`` yes/no, ``choice``, ``score``).  Each question
becomes one causal row ``<state> state <q> instructions <opt> o1 </opt> ... <decide>`` whose
delimiters reuse five Qwen special tokens; the pointer head scores every ``</opt>`` hidden state
against the row's ``<decide>`` state.  Rows must be byte-identical to the serving encoder, so the
delimiter tokens, the none-of-the-above / distractor tables and the order of random draws in the
augmentation are part of the contract and are kept exactly; the code around them is this
package's own.  Batches pack whole request variants into one causal row of documents.
"""
import hashlib
import json
import os
import random
import re

import torch
from torch.utils.data import IterableDataset, get_worker_info

# delimiters: state, question, option open, option close, decide
SPECIAL = ["<|fim_prefix|>", "<|fim_middle|>", "<|box_start|>", "<|box_end|>", "<|fim_suffix|>"]
MAX_STATE, MAX_BRANCH = 384, 1024
MIN_PACK = 128
NONE_OPTIONS = [("other", "None of the above"), ("other", "A reason that fits none of the above"),
                ("none", "None of these"), ("other", "Something else"), ("not_listed", "Not listed here"),
                ("none_of_the_above", None), ("other", "A category that fits none of the above"),
                ("other", "None of the listed options apply"), ("unknown", "Cannot be determined from the options given"),
                ("other", "Other"), ("none", None), ("other", "An answer not covered by the other options"),
                ("no_match", "No option matches")]
DISTRACTORS = {"weather": "Bad weather caused it", "purple": "The colour purple", "pancakes": "A recipe for pancakes",
               "taxes": "Unrelated: quarterly tax filing"}
_CONTROL = re.compile(r"<\|([A-Za-z0-9_]+)\|>")


class ContextOverflow(ValueError):
    pass


def render(v, indent=0):
    """Text form of a str / number / list / dict value (field names kept as labels)."""
    pad = "  " * indent
    if v is None:
        return ""
    if isinstance(v, (str, int, float, bool)):
        return str(v)
    if isinstance(v, list):
        return "\n".join(f"{pad}- {render(x, indent + 1).lstrip()}" for x in v)
    lines = []
    for k, x in v.items():
        lines.append(f"{pad}{k}:\n{render(x, indent + 1)}" if isinstance(x, (dict, list)) else f"{pad}{k}: {render(x)}")
    return "\n".join(lines)


def option_text(name, desc):
    return name if desc is None or desc == "" else f"{name}: {render(desc)}"


def question_keys(qtype, criteria):
    if qtype == "choice":
        return list(criteria)
    if qtype == "noul":
        return ["false", "true"]
    return [str(i) for i in range(len(criteria))]


def materialize(req):
    """Labelled request -> {"state": text, "questions": [{instr, options, qid, qtype, keys, label, target?}]}."""
    out = []
    for qid, q in req["questions"].items():
        keys = question_keys(q["type"], q.get("criteria"))
        if q["type"] == "noul":
            crit = q.get("criteria") or {}
            options = [option_text("no", crit.get("false")), option_text("yes", crit.get("true"))]
        elif q["type"] == "choice":
            options = [option_text(k, v) for k, v in q["criteria"].items()]
        else:
            options = [render(x) for x in q["criteria"]]
        label = keys.index(q["label"]) if q["type"] == "choice" else int(q["label"])
        item = {"instr": render(q.get("instructions")), "options": options, "qid": qid, "qtype": q["type"],
                "keys": keys, "label": label}
        if q.get("target") is not None:
            t = [float(q["target"].get(k, 0.0)) for k in keys]
            tot = sum(t)
            if tot <= 0:
                raise ValueError(f"target for {qid} puts no mass on any option")
            item["target"] = [x / tot for x in t]
        out.append(item)
    return {"state": render(req["state"]), "questions": out}


def augment(req, rng, p_none=0.1, p_none_distract=0.12, p_distract=0.15):
    """Choice questions: always permute the options; with probability p_none replace the true
    option by a none-of-the-above option (which becomes the answer), with p_none_distract add a
    wrong none option, with p_distract add an irrelevant distractor.  Soft targets are only permuted."""
    out = {"state": req["state"], "questions": {}}
    for qid, q in req["questions"].items():
        if q["type"] != "choice":
            out["questions"][qid] = q
            continue
        crit, label = dict(q["criteria"]), q["label"]
        if q.get("target") is not None:
            order = list(crit)
            rng.shuffle(order)
            out["questions"][qid] = {**q, "criteria": {k: crit[k] for k in order}}
            continue
        r = rng.random()
        nones = [(k, v) for k, v in NONE_OPTIONS if k not in crit]
        distract = [k for k in DISTRACTORS if k not in crit]
        if len(crit) > 2 and r < p_none and nones:
            nk, nd = rng.choice(nones)
            crit.pop(label)
            crit[nk] = nd
            label = nk
        elif p_none <= r < p_none + p_none_distract and len(crit) < 255 and nones:
            nk, nd = rng.choice(nones)
            crit[nk] = nd
        elif p_none + p_none_distract <= r < p_none + p_none_distract + p_distract and len(crit) < 255 and distract:
            k = rng.choice(distract)
            crit[k] = DISTRACTORS[k]
        order = list(crit)
        rng.shuffle(order)
        out["questions"][qid] = {**q, "criteria": {k: crit[k] for k in order}, "label": label}
    return out


def none_pair(req, rng):
    """The same choice question with the true option present (a none option is wrong) and removed
    (that none option is right); [] when no choice question has >= 3 options and a hard label."""
    eligible = [(qid, q) for qid, q in req["questions"].items()
                if q["type"] == "choice" and len(q["criteria"]) >= 3 and q.get("target") is None]
    if not eligible:
        return []
    qid, q = rng.choice(eligible)
    nk, nd = rng.choice([o for o in NONE_OPTIONS if o[0] not in q["criteria"]] or [("none_of_these", None)])
    order = list(q["criteria"]) + [nk]
    rng.shuffle(order)
    present = {**q, "criteria": {k: (nd if k == nk else q["criteria"][k]) for k in order}}
    absent = {**present, "criteria": {k: v for k, v in present["criteria"].items() if k != q["label"]}, "label": nk}
    return [{"state": req["state"], "questions": {qid: present}}, {"state": req["state"], "questions": {qid: absent}}]


def record_variants(req, rng, p_none_pair=0.25):
    variants = [augment(req, rng)]
    if p_none_pair > 0 and rng.random() < p_none_pair:
        variants += none_pair(req, rng)
    return variants


def training_context(max_state=MAX_STATE):
    if max_state < MAX_STATE:
        raise ValueError(f"max_state must be >= {MAX_STATE}")
    return {"max_state": max_state, "max_branch": MAX_BRANCH + max_state - MAX_STATE}


def user_tokens(tok, text):
    """Tokenize caller text so it can never produce a control token (``<|x|>`` -> ``<¦x¦>``)."""
    return tok(_CONTROL.sub(r"<¦\1¦>", text), add_special_tokens=False).input_ids


def encode_rows(tok, rec, max_state=MAX_STATE, max_branch=MAX_BRANCH):
    """Record -> question rows {"ids", "decide", "opts", "label", "target"?}; the state is cut to
    ``max_state`` tokens, a branch over its budget raises ContextOverflow."""
    sid, qid, oid, cid, did = (tok.convert_tokens_to_ids(t) for t in SPECIAL)
    state = [sid] + user_tokens(tok, rec["state"])[: max_state - 1]
    rows = []
    for q in rec["questions"]:
        head = [qid] + user_tokens(tok, q["instr"])
        spans = [[oid] + user_tokens(tok, o) + [cid] for o in q["options"]]
        branch = head + [t for sp in spans for t in sp] + [did]
        if len(branch) > max_branch - len(state):
            raise ContextOverflow(f"branch too long: {len(branch)} tokens with a {len(state)}-token state")
        ends, pos = [], len(state) + len(head)
        for sp in spans:
            pos += len(sp)
            ends.append(pos - 1)
        row = {"ids": state + branch, "decide": len(state) + len(branch) - 1, "opts": ends, "label": q["label"]}
        if q.get("target") is not None:
            row["target"] = q["target"]
        rows.append(row)
    return rows


def load_decision_records(paths):
    files = []
    for p in paths:
        files += sorted(os.path.join(p, f) for f in os.listdir(p) if f.endswith(".jsonl")) if os.path.isdir(p) else [p]
    recs = []
    for f in files:
        with open(f, encoding="utf-8") as fh:
            for line in fh:
                if line.strip():
                    r = json.loads(line)
                    recs.append({"state": r["state"], "questions": r["questions"]})
    return recs


def _seed(*parts):
    return int.from_bytes(hashlib.sha256(":".join(map(str, parts)).encode()).digest()[:8], "little")


def pack_decision(variants, tok):
    """Variants (lists of rows) -> one packed causal row [1, T] (each question row a document)
    with flat <decide> / </opt> indices and the per-question loss bookkeeping."""
    ids, seg, decide, opts, owner, questions = [], [], [], [], [], []
    for vi, rows in enumerate(variants):
        for row in rows:
            base, qi = len(ids), len(questions)
            ids += row["ids"]
            seg += [qi] * len(row["ids"])
            decide.append(base + row["decide"])
            q = {"start": len(opts), "k": len(row["opts"]), "label": row["label"], "variant": vi}
            if "target" in row:
                q["target"] = row["target"]
            opts += [base + o for o in row["opts"]]
            owner += [qi] * len(row["opts"])
            questions.append(q)
    if len(ids) < MIN_PACK:
        pad = MIN_PACK - len(ids)
        ids += [getattr(tok, "pad_token_id", None) or 0] * pad
        seg += [len(questions)] * pad
    return {"input_ids": torch.tensor([ids]), "seg_id": torch.tensor([seg]), "decide": torch.tensor(decide),
            "opts": torch.tensor(opts), "owner": torch.tensor(owner), "questions": questions}


class DecisionRowDataset(IterableDataset):
    """Endless stream of decision micro-batches: each epoch reshuffles, re-augments every record
    (plus none pairs), encodes rows and packs whole variants up to ``max_tokens`` row tokens
    (longer variants alone, up to ``max_variant_tokens``).  Records are sharded by (rank, worker)."""

    def __init__(self, records, tokenizer, rank=0, world=1, seed=0, max_tokens=32768, max_state=7552,
                 p_none_pair=0.25, max_variant_tokens=None):
        self.records, self.tok, self.rank, self.world, self.seed = records, tokenizer, rank, world, seed
        self.max_tokens, self.ctx, self.p_none_pair = max_tokens, training_context(max_state), p_none_pair
        self.max_variant_tokens = max(max_tokens, max_variant_tokens or 0)
        self.skipped = 0

    def _variants(self, epoch, idx):
        rng = random.Random(_seed(self.seed, epoch, idx))
        for v in record_variants(self.records[idx], rng, self.p_none_pair):
            try:
                rows = encode_rows(self.tok, materialize(v), **self.ctx)
            except ContextOverflow:
                self.skipped += 1
                continue
            if sum(len(r["ids"]) for r in rows) > self.max_variant_tokens:
                self.skipped += 1
                continue
            yield rows

    def __iter__(self):
        info = get_worker_info()
        wid, nw = (info.id, info.num_workers) if info else (0, 1)
        shard, nshard = self.rank * nw + wid, self.world * nw
        n = len(self.records)
        if n == 0:
            raise ValueError("DecisionRowDataset has no records")
        epoch = 0
        while True:
            order = list(range(n))
            random.Random(_seed(self.seed, "order", epoch)).shuffle(order)
            batch, used, emitted = [], 0, False
            for idx in (order[i % n] for i in range(shard, max(n, nshard), nshard)):
                for rows in self._variants(epoch, idx):
                    t = sum(len(r["ids"]) for r in rows)
                    if t > self.max_tokens:
                        emitted = True
                        yield pack_decision([rows], self.tok)
                        continue
                    if batch and used + t > self.max_tokens:
                        emitted = True
                        yield pack_decision(batch, self.tok)
                        batch, used = [], 0
                    batch.append(rows)
                    used += t
            if batch:
                emitted = True
                yield pack_decision(batch, self.tok)
            if not emitted:
                raise RuntimeError(f"decision shard {shard}/{nshard} produced no micro-batch in epoch {epoch}")
            epoch += 1
