"""Chat SFT data: rendering, label masks, collators, packing and a sharded JSONL stream.

Behaviour follows the reference pipeline (``train/data/text_sft_data.py``):

* ``build_sample`` renders a conversation with the tokenizer's chat template and supervises the
  final assistant turn only (one contiguous response span); the prompt render must be an exact
  token prefix of the full render, otherwise the sample is dropped (``:211-263``).
* ``build_sample_multiturn`` supervises every assistant turn, locating each turn by incremental
  prefix renders and tagging tokens with a global response-block id and a turn ordinal
  (``:266-378``).
* Collators right-pad to a bucketed length; packers bin samples by *forward cost*
  (``n + 2 * n_response`` for block diffusion, ``n`` for pure AR) with first-fit and carry-over, and
  the multi-turn packer block-aligns documents so each starts on a ``bd_size`` boundary
  (``:470-818``).
* ``JsonlChatDataset`` streams local ``*.jsonl`` files sharded by (rank x DataLoader worker) with a
  bounded shuffle buffer whose seed advances every epoch (``:838-922``).

The implementation is this package's own; only the observable contract is shared so datasets and
launch scripts carry over unchanged.
"""
import glob
import json
import multiprocessing as mp
import os
import random

import torch
import torch.nn.functional as F
from torch.utils.data import IterableDataset, get_worker_info

from ..models.block_diffusion import bucketed_clean_len
from .images import expand_image_pads, image_pad_id, image_refs, mrope_position_ids, process_images

IGNORE = -100
_PASSTHROUGH_FIELDS = ("reasoning_content", "tool_calls", "tool_call_id", "name")


def normalize_messages(messages):
    """role/content (or from/value) dicts in the shape chat templates expect; keeps the fields
    templates consume (reasoning, tool calls) and drops everything else."""
    out = []
    for m in messages:
        content = m.get("content", m.get("value"))
        if content is None:
            content = ""
        if not isinstance(content, (str, list, dict)):
            content = str(content)
        msg = {"role": m.get("role") or m.get("from"), "content": content}
        msg.update({k: m[k] for k in _PASSTHROUGH_FIELDS if m.get(k)})
        out.append(msg)
    return out


def _ids_of(enc):
    if hasattr(enc, "input_ids"):
        enc = enc.input_ids
    elif isinstance(enc, dict):
        enc = enc["input_ids"]
    if enc and isinstance(enc[0], (list, tuple)):
        enc = enc[0]
    return [int(t) for t in enc]


def render(tokenizer, messages, tools, add_generation_prompt, keep_all_reasoning=False, image_counts=None):
    """Token ids of a chat-template render; each ``<|image_pad|>`` placeholder is expanded to its
    image's merged-patch count (a render with images but no counts raises)."""
    kw = {"keep_all_reasoning": keep_all_reasoning} if keep_all_reasoning else {}
    enc = tokenizer.apply_chat_template(messages, tools=tools, tokenize=True,
                                        add_generation_prompt=add_generation_prompt, **kw)
    ids = _ids_of(enc)
    pad = image_pad_id(tokenizer)
    if pad is not None and pad in ids:
        if image_counts is None:
            raise ValueError("conversation has images; only --pack --multiturn supports them")
        ids = expand_image_pads(ids, pad, image_counts)
    return ids


def _render_pair(tokenizer, example, fn):
    """Call ``fn(tools)`` with the example's tools, falling back to no tools -- the same mode is
    used for every render of one example so prefix boundaries stay comparable."""
    tools = example.get("tools")
    try:
        return fn(tools), tools
    except Exception:
        try:
            return fn(None), None
        except Exception:
            return None, None


def build_sample(tokenizer, example, keep_all_reasoning=False):
    """``{"input_ids", "labels"}`` supervising the last assistant turn, or None."""
    msgs = example.get("messages") or example.get("conversations")
    if not msgs:
        return None
    msgs = normalize_messages(msgs)
    last = max((i for i, m in enumerate(msgs) if m["role"] == "assistant"), default=None)
    if last is None:
        return None

    def both(tools):
        return (render(tokenizer, msgs[:last + 1], tools, False, keep_all_reasoning),
                render(tokenizer, msgs[:last], tools, True, keep_all_reasoning))

    pair, _ = _render_pair(tokenizer, example, both)
    if pair is None:
        return None
    full, prompt = pair
    if not full or len(prompt) >= len(full) or full[:len(prompt)] != prompt:
        return None
    ids = torch.tensor(full, dtype=torch.long)
    labels = ids.clone()
    labels[:len(prompt)] = IGNORE
    return {"input_ids": ids, "labels": labels}


def build_sample_multiturn(tokenizer, example, bd_size, keep_all_reasoning=False, image_processor=None,
                           max_image_pixels=1024 * 1024):
    """Every assistant turn supervised; adds ``resp_block`` (global block id, -1 off-response) and
    ``turn_id`` (assistant-turn ordinal, -1 off-response).  Turns that do not render as exact
    prefixes are left as conditioning.  A turn whose generation-prompt render does not match (e.g.
    an empty think block) is located by the ``<|im_start|>assistant\\n`` header instead.

    Conversations with image parts need ``image_processor`` (else they are skipped) and add
    ``pixel_values``, ``image_grid_thw`` and ``mrope_pos`` [3, T]; image tokens are never targets.
    ``example["max_image_pixels"]`` overrides the cap for that conversation."""
    msgs = example.get("messages") or example.get("conversations")
    if not msgs:
        return None
    msgs = normalize_messages(msgs)
    turns = [i for i, m in enumerate(msgs) if m["role"] == "assistant"]
    if not turns:
        return None
    try:
        refs = image_refs(msgs)
    except ValueError:
        return None
    counts = None
    if refs:
        if image_processor is None:
            return None
        cap = example.get("max_image_pixels") or max_image_pixels
        try:
            pixel_values, grid, counts = process_images(image_processor, refs, example.get("image_root"), cap)
        except Exception:
            return None

    def all_renders(tools):
        full = render(tokenizer, msgs, tools, False, keep_all_reasoning, counts)
        spans = [(render(tokenizer, msgs[:i], tools, True, keep_all_reasoning, counts),
                  render(tokenizer, msgs[:i + 1], tools, False, keep_all_reasoning, counts)) for i in turns]
        return full, spans

    res, tools = _render_pair(tokenizer, example, all_renders)
    if res is None:
        return None
    full, spans = res
    if not full:
        return None
    T = len(full)
    ids = torch.tensor(full, dtype=torch.long)
    labels = torch.full((T,), IGNORE, dtype=torch.long)
    resp_block = torch.full((T,), -1, dtype=torch.long)
    turn_id = torch.full((T,), -1, dtype=torch.long)
    header = None
    block = 0
    used = 0
    for j, (prefix, upto) in enumerate(spans):
        lo, hi = len(prefix), len(upto)
        if hi > T or full[:hi] != upto:
            continue
        if lo >= hi or full[:lo] != prefix:
            if header is None:
                header = tokenizer.encode("<|im_start|>assistant\n", add_special_tokens=False)
            try:
                base = render(tokenizer, msgs[:turns[j]], tools, False, keep_all_reasoning, counts)
            except Exception:
                continue
            lo = len(base) + len(header)
            if lo >= hi or full[:len(base)] != base or full[len(base):lo] != header:
                continue
        span = torch.arange(lo, hi)
        labels[span] = ids[span]
        turn_id[span] = j
        rb = torch.arange(hi - lo) // bd_size
        resp_block[span] = block + rb
        block += int(rb[-1]) + 1
        used += 1
    if counts:
        labels[ids == image_pad_id(tokenizer)] = IGNORE
    if used == 0 or int((labels != IGNORE).sum()) == 0:
        return None
    out = {"input_ids": ids, "labels": labels, "resp_block": resp_block, "turn_id": turn_id}
    if counts:
        out.update(pixel_values=pixel_values, image_grid_thw=grid,
                   mrope_pos=mrope_position_ids(ids, grid, image_pad_id(tokenizer), image_processor.merge_size))
    return out


def _pad_to(t, n, value):
    return F.pad(t, (0, n - t.shape[0]), value=value)


def _pad_id(tokenizer):
    return tokenizer.pad_token_id if tokenizer.pad_token_id is not None else tokenizer.eos_token_id


def n_supervised(s):
    return int((s["labels"] != IGNORE).sum())


class SftCollator:
    """Single-turn rows, filtered by length / response length, right-padded to a bucket."""

    def __init__(self, tokenizer, max_length=16384, max_response_length=4096,
                 length_buckets=(2048, 4096, 8192, 16384), keep_all_reasoning=False):
        self.tokenizer, self.pad_id = tokenizer, _pad_id(tokenizer)
        self.max_length, self.max_response_length = max_length, max_response_length
        self.length_buckets = tuple(length_buckets) if length_buckets else None
        self.keep_all_reasoning = keep_all_reasoning

    def build(self, ex):
        return build_sample(self.tokenizer, ex, keep_all_reasoning=self.keep_all_reasoning)

    def __call__(self, examples):
        kept = []
        for ex in examples:
            s = self.build(ex)
            if s is None or s["input_ids"].shape[0] > self.max_length or n_supervised(s) > self.max_response_length:
                continue
            kept.append(s)
        if not kept:
            return None
        L = min(bucketed_clean_len(max(s["input_ids"].shape[0] for s in kept), 1, self.length_buckets),
                self.max_length)
        return self.stack(kept, L)

    def stack(self, kept, L):
        return {"input_ids": torch.stack([_pad_to(s["input_ids"], L, self.pad_id) for s in kept]),
                "labels": torch.stack([_pad_to(s["labels"], L, IGNORE) for s in kept]),
                "attention_mask": torch.stack([_pad_to(torch.ones_like(s["input_ids"]), L, 0) for s in kept])}


class MultiTurnSftCollator(SftCollator):
    """Every assistant turn supervised, one conversation per row (adds resp_block / turn_id)."""

    def __init__(self, tokenizer, bd_size=32, **kw):
        super().__init__(tokenizer, **kw)
        self.bd_size = bd_size

    def build(self, ex):
        return build_sample_multiturn(self.tokenizer, ex, self.bd_size, keep_all_reasoning=self.keep_all_reasoning)

    def stack(self, kept, L):
        out = super().stack(kept, L)
        out["resp_block"] = torch.stack([_pad_to(s["resp_block"], L, -1) for s in kept])
        out["turn_id"] = torch.stack([_pad_to(s["turn_id"], L, -1) for s in kept])
        return out


# ------------------------------------------------------------------------------------------------
# packing
# ------------------------------------------------------------------------------------------------
def forward_cost(s, ar_only=False):
    """Forward tokens a sample adds to a packed row: region A plus the clean response copy
    (block diffusion), or just its tokens (pure AR)."""
    n = s["input_ids"].shape[0]
    return n if ar_only else n + 2 * n_supervised(s)


def greedy_pack(samples, max_length, max_segments=0, ar_only=False):
    rows, cur, cost = [], [], 0
    for s in samples:
        c = forward_cost(s, ar_only)
        if cur and (cost + c > max_length or (max_segments and len(cur) >= max_segments)):
            rows.append(cur)
            cur, cost = [], 0
        cur.append(s)
        cost += c
    if cur:
        rows.append(cur)
    return rows


def pack_rows_to_batch(rows, pad_id, length_buckets, max_length):
    """Concatenate each row's segments: ``seg_id`` = segment index (-1 pad), ``resp_pos`` =
    response-relative index (-1 off-response).  Every segment must begin with a prompt token so
    the shifted loss never crosses a document boundary."""
    L = min(bucketed_clean_len(max(sum(s["input_ids"].shape[0] for s in r) for r in rows), 1, length_buckets),
            max_length)
    cols = {k: [] for k in ("input_ids", "labels", "attention_mask", "seg_id", "resp_pos")}
    for row in rows:
        parts = {k: [] for k in cols}
        for k, s in enumerate(row):
            assert int(s["labels"][0]) == IGNORE, "packed segment must start with a prompt (label -100) token"
            n = s["input_ids"].shape[0]
            rp = torch.full((n,), -1, dtype=torch.long)
            ans = (s["labels"] != IGNORE).nonzero(as_tuple=True)[0]
            rp[ans] = torch.arange(ans.numel())
            parts["input_ids"].append(s["input_ids"])
            parts["labels"].append(s["labels"])
            parts["attention_mask"].append(torch.ones(n, dtype=torch.long))
            parts["seg_id"].append(torch.full((n,), k, dtype=torch.long))
            parts["resp_pos"].append(rp)
        fills = {"input_ids": pad_id, "labels": IGNORE, "attention_mask": 0, "seg_id": -1, "resp_pos": -1}
        for k in cols:
            cols[k].append(_pad_to(torch.cat(parts[k]), L, fills[k]))
    batch = {k: torch.stack(v) for k, v in cols.items()}
    docs = [s for row in rows for s in row]
    if any("mrope_pos" in s for s in docs):
        # 3-D positions [B, 3, L] restart per doc (text docs: arange on all axes; row pad 0); image
        # tensors concatenate in row-then-doc order = the order of their pad runs in input_ids
        mrope = torch.zeros(len(rows), 3, L, dtype=torch.long)
        for b, row in enumerate(rows):
            off = 0
            for s in row:
                n = s["input_ids"].shape[0]
                mrope[b, :, off:off + n] = s["mrope_pos"] if "mrope_pos" in s else torch.arange(n).expand(3, -1)
                off += n
        batch["mrope_pos"] = mrope
        batch["pixel_values"] = torch.cat([s["pixel_values"] for s in docs if "pixel_values" in s])
        batch["image_grid_thw"] = torch.cat([s["image_grid_thw"] for s in docs if "image_grid_thw" in s])
    return batch


class PackedSftCollator:
    """Build, filter and greedily pack a pull of examples into doc-isolated rows."""

    def __init__(self, tokenizer, max_length=16384, max_response_length=4096, length_buckets=(2048, 4096, 8192, 16384),
                 max_segments=0, max_packed_rows=0, keep_all_reasoning=False, ar_only=False):
        self.tokenizer, self.pad_id = tokenizer, _pad_id(tokenizer)
        self.max_length, self.max_response_length = max_length, max_response_length
        self.length_buckets = tuple(length_buckets) if length_buckets else None
        self.max_segments, self.max_packed_rows = max_segments, max_packed_rows
        self.keep_all_reasoning, self.ar_only = keep_all_reasoning, ar_only

    def __call__(self, examples):
        kept = [s for s in (build_sample(self.tokenizer, ex, keep_all_reasoning=self.keep_all_reasoning)
                            for ex in examples)
                if s is not None and forward_cost(s, self.ar_only) <= self.max_length
                and n_supervised(s) <= self.max_response_length]
        if not kept:
            return None
        rows = greedy_pack(kept, self.max_length, self.max_segments, self.ar_only)
        if self.max_packed_rows:
            rows = rows[:self.max_packed_rows]
        return pack_rows_to_batch(rows, self.pad_id, self.length_buckets, self.max_length)


def block_align_doc(s, bd_size, pad_id):
    """Right-pad a multi-turn doc to a multiple of ``bd_size`` (pad is non-response, off-turn)."""
    n = s["input_ids"].shape[0]
    extra = (-n) % bd_size
    if not extra:
        return s
    fills = {"input_ids": pad_id, "labels": IGNORE, "resp_block": -1, "turn_id": -1}
    out = dict(s)
    for k, v in fills.items():
        out[k] = _pad_to(s[k], n + extra, v)
    if "mrope_pos" in s:                   # the pad continues the doc's positions
        nxt = int(s["mrope_pos"].max()) + 1
        out["mrope_pos"] = torch.cat([s["mrope_pos"], torch.arange(nxt, nxt + extra).expand(3, -1)], 1)
    return out


def pack_rows_multiturn(rows, pad_id, bd_size, length_buckets, max_length):
    """Tensorize rows of block-aligned docs: input_ids, labels, attention_mask, seg_id, turn_id."""
    need = max(sum(s["input_ids"].shape[0] for s in r) for r in rows)
    L = min(bucketed_clean_len(need, bd_size, length_buckets), max_length)
    cols = {k: [] for k in ("input_ids", "labels", "attention_mask", "seg_id", "turn_id")}
    fills = {"input_ids": pad_id, "labels": IGNORE, "attention_mask": 0, "seg_id": -1, "turn_id": -1}
    for row in rows:
        parts = {k: [] for k in cols}
        for k, s in enumerate(row):
            n = s["input_ids"].shape[0]
            parts["input_ids"].append(s["input_ids"])
            parts["labels"].append(s["labels"])
            parts["attention_mask"].append(torch.ones(n, dtype=torch.long))
            parts["seg_id"].append(torch.full((n,), k, dtype=torch.long))
            parts["turn_id"].append(s["turn_id"])
        for k in cols:
            cols[k].append(_pad_to(torch.cat(parts[k]), L, fills[k]))
    batch = {k: torch.stack(v) for k, v in cols.items()}
    docs = [s for row in rows for s in row]
    if any("mrope_pos" in s for s in docs):
        # 3-D positions [B, 3, L] restart per doc (text docs: arange on all axes; row pad 0); image
        # tensors concatenate in row-then-doc order = the order of their pad runs in input_ids
        mrope = torch.zeros(len(rows), 3, L, dtype=torch.long)
        for b, row in enumerate(rows):
            off = 0
            for s in row:
                n = s["input_ids"].shape[0]
                mrope[b, :, off:off + n] = s["mrope_pos"] if "mrope_pos" in s else torch.arange(n).expand(3, -1)
                off += n
        batch["mrope_pos"] = mrope
        batch["pixel_values"] = torch.cat([s["pixel_values"] for s in docs if "pixel_values" in s])
        batch["image_grid_thw"] = torch.cat([s["image_grid_thw"] for s in docs if "image_grid_thw" in s])
    return batch


def stream_first_fit(docs, max_length, buffer_size=32, max_segments=0):
    """Buffered first-fit over a doc stream; every row starts with the oldest buffered doc, nothing
    is dropped, the buffer never exceeds ``buffer_size``, every row stays ``<= max_length``."""
    if buffer_size < 1:
        raise ValueError(f"buffer_size must be >= 1, got {buffer_size}")
    it = iter(docs)
    buf = []
    done = False

    def fill():
        nonlocal done
        while not done and len(buf) < buffer_size:
            try:
                buf.append(next(it))
            except StopIteration:
                done = True

    while True:
        fill()
        if not buf:
            return
        row = [buf.pop(0)]
        used = row[0]["input_ids"].shape[0]
        if used > max_length:
            raise ValueError(f"doc of {used} tokens does not fit alone in max_length={max_length}")
        while True:
            i = 0
            while i < len(buf) and not (max_segments and len(row) >= max_segments):
                n = buf[i]["input_ids"].shape[0]
                if used + n <= max_length:
                    row.append(buf.pop(i))
                    used += n
                else:
                    i += 1
            before = len(buf)
            fill()
            if len(buf) == before or (max_segments and len(row) >= max_segments):
                break
        yield row


class PackedRowDataset(IterableDataset):
    """Single-turn samples packed into ``<= max_length``-cost rows with carry-over."""

    def __init__(self, base, tokenizer, max_length=32768, max_response_length=32768, keep_all_reasoning=False,
                 max_segments=0, ar_only=False):
        self.base, self.tokenizer = base, tokenizer
        self.max_length, self.max_response_length = max_length, max_response_length
        self.keep_all_reasoning, self.max_segments, self.ar_only = keep_all_reasoning, max_segments, ar_only

    def __iter__(self):
        row, cost = [], 0
        for ex in self.base:
            s = build_sample(self.tokenizer, ex, keep_all_reasoning=self.keep_all_reasoning)
            if s is None:
                continue
            c = forward_cost(s, self.ar_only)
            if c > self.max_length or n_supervised(s) > self.max_response_length:
                continue
            if row and (cost + c > self.max_length or (self.max_segments and len(row) >= self.max_segments)):
                yield row
                row, cost = [], 0
            row.append(s)
            cost += c
        if row:
            yield row


class PackedMultiTurnRowDataset(IterableDataset):
    """Whole conversations (every turn supervised), block-aligned, packed by buffered first-fit."""

    def __init__(self, base, tokenizer, bd_size, max_length=32768, max_response_length=32768,
                 keep_all_reasoning=True, max_segments=0, buffer_size=32, image_processor=None,
                 max_image_pixels=1024 * 1024, **_ignored):
        self.base, self.tokenizer, self.pad_id = base, tokenizer, _pad_id(tokenizer)
        self.image_processor, self.max_image_pixels = image_processor, max_image_pixels
        self.bd_size, self.max_length, self.max_response_length = bd_size, max_length, max_response_length
        self.keep_all_reasoning, self.max_segments, self.buffer_size = keep_all_reasoning, max_segments, buffer_size
        self.stats = {}

    def _docs(self):
        st = self.stats = {"packed": 0, "too_long": 0, "response_too_long": 0, "unusable": 0}
        for ex in self.base:
            s = build_sample_multiturn(self.tokenizer, ex, self.bd_size, keep_all_reasoning=self.keep_all_reasoning,
                                       image_processor=self.image_processor, max_image_pixels=self.max_image_pixels)
            if s is None:
                st["unusable"] += 1
                continue
            s = block_align_doc(s, self.bd_size, self.pad_id)
            if s["input_ids"].shape[0] > self.max_length:
                st["too_long"] += 1
                continue
            if n_supervised(s) > self.max_response_length:
                st["response_too_long"] += 1
                continue
            st["packed"] += 1
            yield s

    def __iter__(self):
        yield from stream_first_fit(self._docs(), self.max_length, self.buffer_size, self.max_segments)


class StreamPackedCollator:
    def __init__(self, tokenizer, max_length=32768, length_buckets=(2048, 4096, 8192, 16384, 32768)):
        self.pad_id, self.max_length = _pad_id(tokenizer), max_length
        self.length_buckets = tuple(length_buckets) if length_buckets else None

    def __call__(self, rows):
        rows = [r for r in rows if r]
        return pack_rows_to_batch(rows, self.pad_id, self.length_buckets, self.max_length) if rows else None


class StreamPackedMultiTurnCollator:
    def __init__(self, tokenizer, bd_size, max_length=32768, length_buckets=(2048, 4096, 8192, 16384, 32768)):
        self.pad_id, self.bd_size, self.max_length = _pad_id(tokenizer), bd_size, max_length
        self.length_buckets = tuple(length_buckets) if length_buckets else None

    def __call__(self, rows):
        rows = [r for r in rows if r]
        return (pack_rows_multiturn(rows, self.pad_id, self.bd_size, self.length_buckets, self.max_length)
                if rows else None)


# ------------------------------------------------------------------------------------------------
# streaming JSONL
# ------------------------------------------------------------------------------------------------
def jsonl_paths(source):
    """Local ``*.jsonl`` files of a directory (sorted) or a single file."""
    if os.path.isdir(source):
        paths = sorted(glob.glob(os.path.join(source, "*.jsonl")))
        if not paths:
            raise FileNotFoundError(f"no .jsonl files in {source}")
        return paths
    if os.path.isfile(source):
        return [source]
    raise FileNotFoundError(f"{source} is neither a directory of *.jsonl files nor a file (no network here)")


class JsonlChatDataset(IterableDataset):
    """Streams chat records sharded by (rank x worker) line modulo, with a bounded shuffle buffer;
    each new iteration (epoch) draws a fresh shuffle seed through a fork-shared counter."""

    def __init__(self, paths, rank=0, world=1, seed=42, shuffle_buffer=10000):
        self.paths, self.rank, self.world, self.seed, self.shuffle_buffer = list(paths), rank, world, seed, shuffle_buffer
        self._epoch = mp.Value("i", 0)

    def __iter__(self):
        info = get_worker_info()
        wid, nw = (info.id, info.num_workers) if info else (0, 1)
        shard, nshard = self.rank * nw + wid, self.world * nw
        with self._epoch.get_lock():
            epoch = self._epoch.value
            self._epoch.value += 1
        rng = random.Random(self.seed + 1000 * epoch + shard)
        buf = []
        idx = 0
        for path in self.paths:
            with open(path) as f:
                for line in f:
                    take = idx % nshard == shard
                    idx += 1
                    if not take:
                        continue
                    try:
                        rec = json.loads(line)
                    except json.JSONDecodeError:
                        continue
                    msgs = rec.get("messages") or rec.get("conversations")
                    if not msgs:
                        continue
                    item = {"messages": msgs, "tools": rec.get("tools"),
                            "image_root": os.path.dirname(os.path.abspath(path)),
                            "max_image_pixels": rec.get("max_image_pixels")}
                    if self.shuffle_buffer <= 1:
                        yield item
                        continue
                    buf.append(item)
                    if len(buf) >= self.shuffle_buffer:
                        yield buf.pop(rng.randrange(len(buf)))
        rng.shuffle(buf)
        yield from buf
