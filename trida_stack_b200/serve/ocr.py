"""GravityOCR HTTP front end: OpenAI-compatible chat completions over image crops.

One layout region per request (``inference/gravityocr/README.md`` "Request format"): a user message
whose content holds the image as a ``data:`` URL and a task prompt (``Text Recognition:``,
``Table Recognition:``, ``Formula Recognition:``).  The server never fetches a URL or reads a file
named in a request (only ``data:`` URLs are accepted), binds to loopback unless told otherwise, and,
given a key, requires ``Authorization: Bearer <key>`` on every route but ``/health`` (compared in
constant time).  The prompt with its image tokens plus ``max_tokens`` must fit the context.
"""
import asyncio
import base64
import hmac
import io
import json
import time
import uuid

TASK_PROMPTS = {"text": "Text Recognition:", "table": "Table Recognition:", "formula": "Formula Recognition:"}


class OcrRequestError(ValueError):
    def __init__(self, msg, status=400):
        super().__init__(msg)
        self.status = status


def image_from_part(part):
    """PIL image of an ``image_url`` / ``image`` content part; only ``data:`` URLs are accepted."""
    from PIL import Image
    ref = part.get("image_url") or part.get("image")
    if isinstance(ref, dict):
        ref = ref.get("url")
    if not isinstance(ref, str) or not ref.startswith("data:"):
        raise OcrRequestError("images must be sent inline as data: URLs")
    try:
        raw = base64.b64decode(ref.split(",", 1)[1], validate=False)
        return Image.open(io.BytesIO(raw)).convert("RGB")
    except Exception as e:
        raise OcrRequestError(f"could not decode the image: {type(e).__name__}")


def split_content(messages):
    """(images, messages with each image part replaced by a bare image marker) in render order."""
    images, out = [], []
    for m in messages:
        c = m.get("content")
        if isinstance(c, list):
            parts = []
            for p in c:
                if isinstance(p, dict) and (p.get("type") in ("image_url", "image") or "image_url" in p):
                    images.append(image_from_part(p))
                    parts.append({"type": "image"})
                else:
                    parts.append(p)
            out.append(dict(m, content=parts))
        else:
            out.append(m)
    return images, out


def render_prompt(tok, messages, image_token_id, counts):
    """Token ids of the chat prompt with each image placeholder expanded to its merged-patch count."""
    from ..data.images import expand_image_pads
    if getattr(tok, "chat_template", None):
        ids = tok.apply_chat_template(messages, tokenize=True, add_generation_prompt=True)
        if hasattr(ids, "input_ids"):
            ids = ids.input_ids
        elif isinstance(ids, dict):
            ids = ids["input_ids"]
        ids = list(ids[0] if ids and isinstance(ids[0], list) else ids)
    else:                                   # template-less tokenizers: [image tokens] text
        ids = []
        for m in messages:
            c = m.get("content")
            for p in (c if isinstance(c, list) else [{"type": "text", "text": c or ""}]):
                if p.get("type") == "image":
                    ids.append(image_token_id)
                else:
                    ids += tok(p.get("text", ""), add_special_tokens=False).input_ids
    if ids.count(image_token_id) != len(counts):
        raise OcrRequestError(f"the prompt renders {ids.count(image_token_id)} image placeholders for "
                              f"{len(counts)} images")
    return expand_image_pads(ids, image_token_id, counts)


def build_ocr_app(engine, tok, processor, model_name="glm-ocr", api_key=None, context=16384, eos=()):
    from fastapi import FastAPI, Request as HTTPRequest
    from fastapi.responses import JSONResponse, StreamingResponse

    from .engine import Request, SamplingParams

    app = FastAPI()
    img_id = engine.rt.cfg.image_token_id
    merge = processor.merge_size if processor is not None else 2
    eos = tuple(eos) or tuple(t for t in (getattr(tok, "eos_token_id", None),) if isinstance(t, int))

    def authorized(http):
        if not api_key:
            return True
        h = http.headers.get("authorization", "")
        return h.startswith("Bearer ") and hmac.compare_digest(h[7:].encode(), api_key.encode())

    def deny():
        return JSONResponse({"error": {"message": "missing or wrong API key"}}, status_code=401)

    @app.get("/health")
    async def health():
        return {"status": "ok"}

    @app.get("/v1/models")
    async def models(http: HTTPRequest):
        if not authorized(http):
            return deny()
        return {"object": "list", "data": [{"id": model_name, "object": "model", "owned_by": "trida"}]}

    @app.get("/v1/stats")
    async def stats(http: HTTPRequest):
        if not authorized(http):
            return deny()
        st = dict(engine.stats)
        st.update(mode=engine.mode, tok_per_fwd=round(st["tokens"] / st["forwards"], 4) if st["forwards"] else None)
        return st

    def prepare(body):
        msgs = body.get("messages")
        if not isinstance(msgs, list) or not msgs:
            raise OcrRequestError("messages must be a non-empty list")
        images, msgs = split_content(msgs)
        if images and processor is None:
            raise OcrRequestError("this model takes no images")
        pv = grid = None
        counts = []
        if images:
            pv, grid = processor(images)
            counts = (grid.prod(-1) // merge ** 2).tolist()
        ids = render_prompt(tok, msgs, img_id, counts)
        max_tokens = int(body.get("max_tokens") or body.get("max_completion_tokens") or 4096)
        if len(ids) + max_tokens > context:
            raise OcrRequestError(f"{len(ids)} prompt tokens + max_tokens {max_tokens} exceed the context "
                                  f"of {context}")
        sp = SamplingParams(temperature=float(body.get("temperature", 0.0) or 0.0),
                            top_k=int(body.get("top_k", 20) or 0), top_p=float(body.get("top_p", 1.0) or 1.0),
                            seed=body.get("seed"))
        req = Request(ids, max_tokens, sp, () if body.get("ignore_eos") else eos)
        if images:
            req.images = (pv, grid)
        return req

    async def run(req, on_chunk=None):
        loop = asyncio.get_running_loop()
        q: asyncio.Queue = asyncio.Queue()
        req.on_tokens = lambda toks: loop.call_soon_threadsafe(q.put_nowait, toks)
        engine.submit(req)
        while True:
            toks = await q.get()
            if toks is None:
                return req
            if on_chunk is not None:
                await on_chunk(toks)

    @app.post("/v1/chat/completions")
    async def chat(http: HTTPRequest):
        if not authorized(http):
            return deny()
        try:
            body = await http.json()
            req = prepare(body)
        except OcrRequestError as e:
            return JSONResponse({"error": {"message": str(e)}}, status_code=e.status)
        except (ValueError, json.JSONDecodeError) as e:
            return JSONResponse({"error": {"message": f"bad request: {e}"}}, status_code=400)
        cid, created = f"chatcmpl-{uuid.uuid4().hex[:16]}", int(time.time())
        if body.get("stream"):
            async def gen():
                q: asyncio.Queue = asyncio.Queue()

                async def cb(toks):
                    await q.put(toks)

                task = asyncio.ensure_future(run(req, cb))
                while not (task.done() and q.empty()):
                    try:
                        toks = await asyncio.wait_for(q.get(), timeout=0.05)
                    except asyncio.TimeoutError:
                        continue
                    delta = {"content": tok.decode(toks, skip_special_tokens=True)}
                    yield "data: " + json.dumps({"id": cid, "object": "chat.completion.chunk", "created": created,
                                                 "model": model_name,
                                                 "choices": [{"index": 0, "delta": delta, "finish_reason": None}]}) + "\n\n"
                r = await task
                yield "data: " + json.dumps({"id": cid, "object": "chat.completion.chunk", "created": created,
                                             "model": model_name,
                                             "choices": [{"index": 0, "delta": {}, "finish_reason": r.finish_reason}],
                                             "usage": _usage(r)}) + "\n\n"
                yield "data: [DONE]\n\n"
            return StreamingResponse(gen(), media_type="text/event-stream")
        r = await run(req)
        return {"id": cid, "object": "chat.completion", "created": created, "model": model_name,
                "choices": [{"index": 0, "message": {"role": "assistant",
                                                     "content": tok.decode(r.output, skip_special_tokens=True)},
                             "finish_reason": r.finish_reason}],
                "usage": _usage(r)}

    return app


def _usage(r):
    return {"prompt_tokens": len(r.prompt), "completion_tokens": len(r.output),
            "total_tokens": len(r.prompt) + len(r.output), "forwards": r.forwards}


def synthetic_png(text, scale=2):
    """A small black-on-white PNG of ``text`` (for smoke tests without a sample image)."""
    from PIL import Image, ImageDraw
    w = max(64, 8 * len(text) + 16)
    img = Image.new("RGB", (w, 32), "white")
    ImageDraw.Draw(img).text((8, 10), text, fill="black")
    img = img.resize((w * scale, 32 * scale))
    buf = io.BytesIO()
    img.save(buf, format="PNG")
    return buf.getvalue()


def data_url(png_bytes, mime="image/png"):
    return f"data:{mime};base64," + base64.b64encode(png_bytes).decode()


def pick_eos(path, tok):
    """End-of-sequence ids: the checkpoint's generation config, else the tokenizer's."""
    import os
    ids = []
    gc = os.path.join(path, "generation_config.json") if path else None
    if gc and os.path.exists(gc):
        e = json.load(open(gc)).get("eos_token_id")
        ids = e if isinstance(e, list) else ([e] if isinstance(e, int) else [])
    if not ids and getattr(tok, "eos_token_id", None) is not None:
        ids = [tok.eos_token_id]
    return tuple(ids)


def mask_id_of(path, cfg_vocab):
    """The drafting mask id: ``$SELFSPEC_MASK_ID``, else ``block_diffusion.json``; no silent default."""
    import os
    env = os.environ.get("SELFSPEC_MASK_ID")
    if env:
        mid, src = int(env), "SELFSPEC_MASK_ID"
    else:
        side = os.path.join(path, "block_diffusion.json") if path else ""
        if not side or not os.path.exists(side):
            raise SystemExit("self-spec needs the mask id: block_diffusion.json in the checkpoint or $SELFSPEC_MASK_ID")
        mid, src = int(json.load(open(side))["mask_id"]), side
    if not 0 <= mid < cfg_vocab:
        raise SystemExit(f"mask id {mid} (from {src}) is outside the text vocabulary ({cfg_vocab})")
    return mid, src
