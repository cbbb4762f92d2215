"""Typed-decision data (kev scheme; reference: ``train/data/decision.py``).

A request is a ``state`` plus typed questions (``noul`` yes/no, ``choice``, ``score``).  Each question
becomes one causal row ``<state> state <q> instructions <opt> o1 </opt> ... <decide>`` whose
delimiters reuse five Qwen special tokens; the pointer head scores every ``</opt>`` hidden state
against the row's ``<decide>`` state.  Rows must be byte-identical to the serving encoder, so the
delimiter tokens, the none-of-the-above / distractor tables and the order of random draws in the
augmentation are part of the contract and are kept exactly; the code around them is this
package's own.  Batches pack whole request variants into one causal row of documents.
"""
import json
import os
import random
import re

import torch
from torch.utils.data import IterableDataset

from .sharding import EpochSampler, mix_seed, worker_shard

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


class _Text:
    """Text form of a JSON value inside a decision row: scalars as ``str()``, ``None`` as nothing,
    mappings as ``key: value`` lines (nested values on the following lines, two more spaces of
    indent), sequences as ``- item`` lines.  The exact text is part of the row format a released
    checkpoint was trained on, so it must not change."""

    @classmethod
    def of(cls, value, depth=0):
        if value is None:
            return ""
        if isinstance(value, (str, int, float, bool)):
            return str(value)
        lines = cls._seq(value, depth) if isinstance(value, list) else cls._map(value, depth)
        return "\n".join(lines)

    @classmethod
    def _seq(cls, items, depth):
        lead = "  " * depth + "- "
        return [lead + cls.of(x, depth + 1).lstrip() for x in items]

    @classmethod
    def _map(cls, mapping, depth):
        pad = "  " * depth
        out = []
        for key, x in mapping.items():
            nested = isinstance(x, (dict, list))
            out.append(f"{pad}{key}:\n{cls.of(x, depth + 1)}" if nested else f"{pad}{key}: {cls.of(x)}")
        return out


def render(v, indent=0):
    """Text of a value for a decision row (see ``_Text``)."""
    return _Text.of(v, indent)


def option_text(name, desc):
    """An option line: the key alone when it has no description, else ``key: description``."""
    has_desc = not (desc is None or desc == "")
    return f"{name}: {render(desc)}" if has_desc else name


def question_keys(qtype, criteria):
    """Option keys of a question, in row order (a yes/no question is ``false`` then ``true``)."""
    return {"choice": lambda: list(criteria), "noul": lambda: ["false", "true"]}.get(
        qtype, lambda: [str(i) for i in range(len(criteria))])()


def _options(q):
    """Option texts of a question, aligned with ``question_keys``."""
    kind, crit = q["type"], q.get("criteria")
    if kind == "noul":
        crit = crit or {}
        return [option_text(word, crit.get(key)) for word, key in (("no", "false"), ("yes", "true"))]
    if kind == "choice":
        return [option_text(k, d) for k, d in crit.items()]
    return [render(x) for x in crit]


def _soft_target(q, keys):
    """Normalised soft-label distribution over ``keys`` (None when the question has no target)."""
    tgt = q.get("target")
    if tgt is None:
        return None
    mass = [float(tgt.get(k, 0.0)) for k in keys]
    total = sum(mass)
    if not total > 0:
        raise ValueError(f"question {q.get('_id', '?')}: the soft target gives no option any weight")
    return [m / total for m in mass]


def materialize(req):
    """Labelled request -> {"state": text, "questions": [{instr, options, qid, qtype, keys, label, target?}]}."""
    questions = []
    for qid, q in req["questions"].items():
        keys = question_keys(q["type"], q.get("criteria"))
        label = keys.index(q["label"]) if q["type"] == "choice" else int(q["label"])
        item = {"instr": render(q.get("instructions")), "options": _options(q), "qid": qid, "qtype": q["type"],
                "keys": keys, "label": label}
        target = _soft_target({**q, "_id": qid}, keys)
        if target is not None:
            item["target"] = target
        questions.append(item)
    return {"state": render(req["state"]), "questions": questions}


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


def _encode_variant(tok, variant, ctx, max_tokens):
    """Row list of one augmented variant, or None when it does not fit the context budgets."""
    try:
        rows = encode_rows(tok, materialize(variant), **ctx)
    except ContextOverflow:
        return None
    return rows if sum(len(r["ids"]) for r in rows) <= max_tokens else None


def pack_by_budget(variants, max_tokens):
    """Group a stream of variants (row lists) into micro-batches of at most ``max_tokens`` row
    tokens, in arrival order; a variant larger than the budget becomes a micro-batch of its own."""
    group, used = [], 0
    for rows in variants:
        size = sum(len(r["ids"]) for r in rows)
        if size > max_tokens:
            yield [rows]
            continue
        if group and used + size > max_tokens:
            yield group
            group, used = [], 0
        group.append(rows)
        used += size
    if group:
        yield group


class DecisionRowDataset(IterableDataset):
    """Endless stream of packed decision micro-batches.

    Records are dealt to (rank x DataLoader worker) shards by ``sharding.EpochSampler`` (a fresh
    permutation every epoch, equal counts per shard); every visit re-augments the record with a
    generator seeded by (seed, epoch, record), encodes its variants, drops the ones over the
    context budgets (counted in ``skipped``) and ``pack_by_budget`` groups them into micro-batches
    of ``max_tokens`` row tokens (a larger variant, up to ``max_variant_tokens``, goes alone)."""

    def __init__(self, records, tokenizer, rank=0, world=1, seed=0, max_tokens=32768, max_state=7552,
                 p_none_pair=0.25, max_variant_tokens=None):
        if not records:
            raise ValueError("DecisionRowDataset needs at least one record")
        self.records, self.tok, self.rank, self.world, self.seed = records, tokenizer, rank, world, seed
        self.max_tokens, self.ctx, self.p_none_pair = max_tokens, training_context(max_state), p_none_pair
        self.max_variant_tokens = max(max_tokens, max_variant_tokens or 0)
        self.skipped = 0

    def _variants(self, indices, epoch):
        for idx in indices:
            rng = random.Random(mix_seed(self.seed, epoch, idx))
            for variant in record_variants(self.records[idx], rng, self.p_none_pair):
                rows = _encode_variant(self.tok, variant, self.ctx, self.max_variant_tokens)
                if rows is None:
                    self.skipped += 1
                else:
                    yield rows

    def __iter__(self):
        shard, nshard = worker_shard(self.rank, self.world)
        sampler = EpochSampler(len(self.records), shard, nshard, self.seed)
        epoch = 0
        while True:
            produced = False
            for group in pack_by_budget(self._variants(sampler.epoch(epoch), epoch), self.max_tokens):
                produced = True
                yield pack_decision(group, self.tok)
            if not produced:
                raise RuntimeError(f"decision shard {shard}/{nshard}: no record fits the budgets in epoch {epoch}")
            epoch += 1
