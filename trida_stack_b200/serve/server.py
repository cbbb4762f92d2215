"""OpenAI-compatible HTTP server over the native engine (and the decision engine in decide mode).

Endpoints (reference surface: ``inference/zoro-1/README.md:145-207``, ``serve_decide.py:1-25``):

  GET  /health, GET /v1/models
  POST /v1/chat/completions   streaming (SSE) or not; ``max_tokens``, ``temperature``, ``top_p``,
                              ``top_k``, ``chat_template_kwargs.enable_thinking``; the thinking is
                              returned as ``reasoning_content``; ``<tool_call>`` blocks of the
                              model's output become OpenAI ``tool_calls``; ``usage`` and
                              ``finish_reason`` ("stop" / "length" / "tool_calls")
  POST /v1/completions        plain prompt completion
  POST /v1/systemone          typed decisions (decide mode); 422 on malformed requests
  POST /v1/decide             deprecated alias: ``{"request": {...}}``

Generation runs on the engine's own thread; each request streams its tokens back through an
asyncio queue.
"""
import asyncio
import json
import re
import time
import uuid

END_THINK = "</think>"
_CALL = re.compile(r"<tool_call>\s*<function=([\w.-]+)>(.*?)</function>\s*</tool_call>", re.S)
_PARAM = re.compile(r"<parameter=([\w.-]+)>\n?(.*?)\n?</parameter>", re.S)
_CALL_JSON = re.compile(r"<tool_call>\s*(\{.*?\})\s*</tool_call>", re.S)


def parse_tool_calls(text, tools=None):
    """OpenAI tool calls from the model's ``<tool_call>`` blocks (XML-parameter form, or a JSON
    object ``{"name", "arguments"}``).  Parameters typed ``string`` by the tool schema stay text;
    any other value is read as JSON when it parses."""
    strings = {}
    for t in tools or []:
        f = t.get("function", t) if isinstance(t, dict) else {}
        props = (f.get("parameters") or {}).get("properties") or {}
        strings[f.get("name")] = {k for k, p in props.items() if isinstance(p, dict) and
                                  (p.get("type") == "string" or (isinstance(p.get("type"), list) and "string" in p["type"]))}
    calls = []
    for m in _CALL.finditer(text):
        args = {}
        for k, v in _PARAM.findall(m.group(2)):
            v = v.strip()
            if k in strings.get(m.group(1), ()):
                args[k] = v
                continue
            try:
                args[k] = json.loads(v)
            except ValueError:
                args[k] = v
        calls.append({"id": f"call_{uuid.uuid4().hex[:12]}", "type": "function",
                      "function": {"name": m.group(1), "arguments": json.dumps(args)}})
    for m in _CALL_JSON.finditer(text):
        try:
            obj = json.loads(m.group(1))
        except ValueError:
            continue
        calls.append({"id": f"call_{uuid.uuid4().hex[:12]}", "type": "function",
                      "function": {"name": obj.get("name"), "arguments": json.dumps(obj.get("arguments", {}))}})
    return calls


def split_turn(raw, thinking=True, truncated=False, tools=None):
    """Raw assistant text -> (reasoning, visible text, tool calls)."""
    if END_THINK in raw:
        reasoning, _, rest = raw.rpartition(END_THINK)
        reasoning = reasoning.replace("<think>", "").strip()
    elif thinking and truncated:
        reasoning, rest = raw.replace("<think>", ""), ""
    else:
        reasoning, rest = "", raw
    calls = parse_tool_calls(rest, tools) if tools else []
    if calls:
        rest = rest[:rest.find("<tool_call>")]
    return reasoning, rest.strip(), calls


def render_chat(tok, messages, tools=None, enable_thinking=True):
    if getattr(tok, "chat_template", None):
        kw = {"tools": tools} if tools else {}
        return tok.apply_chat_template(messages, tokenize=False, add_generation_prompt=True,
                                       enable_thinking=enable_thinking, **kw)
    parts = [f"<|im_start|>{m['role']}\n{m.get('content') or ''}<|im_end|>\n" for m in messages]
    return "".join(parts) + "<|im_start|>assistant\n"


def build_app(engine, tokenizer, model_name, decider=None):
    from fastapi import FastAPI, Request as HTTPRequest
    from fastapi.responses import JSONResponse, StreamingResponse

    from .decide import RequestError, systemone_request, systemone_response
    from .engine import Request, SamplingParams

    app = FastAPI()
    eos = tuple(t for t in {getattr(tokenizer, "eos_token_id", None),
                            tokenizer.convert_tokens_to_ids("<|im_end|>") if hasattr(tokenizer, "convert_tokens_to_ids") else None}
                if isinstance(t, int) and t >= 0)

    def sampling(body):
        return SamplingParams(temperature=float(body.get("temperature", 0.0) or 0.0),
                              top_k=int(body.get("top_k", 20) or 0), top_p=float(body.get("top_p", 1.0) or 1.0),
                              seed=body.get("seed"))

    async def run(ids, body, stream_cb=None):
        loop = asyncio.get_running_loop()
        q: asyncio.Queue = asyncio.Queue()
        req = Request(ids, int(body.get("max_tokens") or body.get("max_completion_tokens") or 512), sampling(body),
                      () if body.get("ignore_eos") else eos)
        req.on_tokens = lambda toks: loop.call_soon_threadsafe(q.put_nowait, toks)
        engine.submit(req)
        while True:
            toks = await q.get()
            if toks is None:
                break
            if stream_cb is not None:
                await stream_cb(req)
        return req

    @app.get("/health")
    async def health():
        return {"status": "ok"}

    @app.get("/v1/stats")
    async def stats():
        """Cumulative engine counters (forwards, emitted tokens, prefill tokens) and tokens per forward."""
        st = dict(engine.stats)
        st.update(mode=engine.mode, gen_block=engine.n, running=len(engine.running),
                  tok_per_fwd=round(st["tokens"] / st["forwards"], 4) if st["forwards"] else None)
        return st

    @app.get("/v1/models")
    async def models():
        return {"object": "list", "data": [{"id": model_name, "object": "model", "owned_by": "trida"}]}

    @app.post("/v1/completions")
    async def completions(http: HTTPRequest):
        body = await http.json()
        prompt = body.get("prompt", "")
        if isinstance(prompt, list) and all(isinstance(t, int) for t in prompt):
            ids = list(prompt)                    # token-id prompt (OpenAI completions allows it)
        else:
            ids = tokenizer(prompt, add_special_tokens=False).input_ids
        req = await run(ids, body)
        text = tokenizer.decode(req.output)
        choice = {"index": 0, "text": text, "finish_reason": req.finish_reason}
        if body.get("return_token_ids"):
            choice["token_ids"] = list(req.output)
        return {"id": f"cmpl-{uuid.uuid4().hex[:16]}", "object": "text_completion", "created": int(time.time()),
                "model": model_name, "choices": [choice],
                "usage": {"prompt_tokens": len(ids), "completion_tokens": len(req.output),
                          "total_tokens": len(ids) + len(req.output)}}

    @app.post("/v1/chat/completions")
    async def chat(http: HTTPRequest):
        body = await http.json()
        tools = body.get("tools")
        thinking = bool((body.get("chat_template_kwargs") or {}).get("enable_thinking", True))
        prompt = render_chat(tokenizer, body.get("messages", []), tools, thinking)
        ids = tokenizer(prompt, add_special_tokens=False).input_ids
        cid, created = f"chatcmpl-{uuid.uuid4().hex[:16]}", int(time.time())
        if not body.get("stream"):
            req = await run(ids, body)
            raw = tokenizer.decode(req.output)
            reasoning, text, calls = split_turn(raw, thinking, req.finish_reason == "length", tools)
            msg = {"role": "assistant", "content": text}
            if reasoning:
                msg["reasoning_content"] = reasoning
            finish = req.finish_reason
            if calls:
                msg["tool_calls"] = calls
                finish = "tool_calls"
            return {"id": cid, "object": "chat.completion", "created": created, "model": model_name,
                    "choices": [{"index": 0, "message": msg, "finish_reason": finish}],
                    "usage": {"prompt_tokens": len(ids), "completion_tokens": len(req.output),
                              "total_tokens": len(ids) + len(req.output)},
                    "forwards": req.forwards}

        async def gen():
            out_q: asyncio.Queue = asyncio.Queue()
            sent = {"n": 0}

            async def cb(req):
                text = tokenizer.decode(req.output)
                delta, sent["n"] = text[sent["n"]:], len(text)
                if delta:
                    await out_q.put(delta)

            task = asyncio.ensure_future(run(ids, body, cb))
            head = {"id": cid, "object": "chat.completion.chunk", "created": created, "model": model_name}
            yield "data: " + json.dumps({**head, "choices": [{"index": 0, "delta": {"role": "assistant"}}]}) + "\n\n"
            while not (task.done() and out_q.empty()):
                try:
                    d = await asyncio.wait_for(out_q.get(), timeout=0.05)
                except asyncio.TimeoutError:
                    continue
                yield "data: " + json.dumps({**head, "choices": [{"index": 0, "delta": {"content": d}}]}) + "\n\n"
            req = task.result()
            usage = {"prompt_tokens": len(ids), "completion_tokens": len(req.output),
                     "total_tokens": len(ids) + len(req.output)}
            yield "data: " + json.dumps({**head, "choices": [{"index": 0, "delta": {},
                                                            "finish_reason": req.finish_reason}], "usage": usage}) + "\n\n"
            yield "data: [DONE]\n\n"

        return StreamingResponse(gen(), media_type="text/event-stream")

    async def _decide(request, opts):
        return await asyncio.get_running_loop().run_in_executor(
            None, lambda: decider.decide(request, opts.get("temperature"), bool(opts.get("reasoning", False)),
                                         opts.get("max_reasoning_tokens")))

    def _no_decider():
        return JSONResponse({"detail": "decisions need --mode decide and a decision checkpoint"}, status_code=400)

    @app.post("/v1/systemone")
    async def systemone(http: HTTPRequest):
        if decider is None:
            return _no_decider()
        body = await http.json()
        try:
            request, opts = systemone_request(body, decider.reasoning_token_limit)
            out = await _decide(request, opts)
        except RequestError as e:
            return JSONResponse({"detail": e.detail()}, status_code=422)
        return systemone_response(out, model_name)

    @app.post("/v1/decide")
    async def decide_alias(http: HTTPRequest):
        """Deprecated: ``{"request": {...}, "reasoning"?, "temperature"?, "max_reasoning_tokens"?}`` ->
        the decision result itself (no System One envelope)."""
        if decider is None:
            return _no_decider()
        body = await http.json()
        headers = {"Deprecation": "true", "Link": '</v1/systemone>; rel="successor-version"'}
        if not isinstance(body, dict) or "request" not in body:
            return JSONResponse({"detail": 'body must be {"request": {...}, "reasoning"?: bool, "temperature"?: '
                                           'float, "max_reasoning_tokens"?: int}'}, status_code=400, headers=headers)
        opts = {k: body[k] for k in ("reasoning", "temperature", "max_reasoning_tokens") if body.get(k) is not None}
        try:
            out = await _decide(body["request"], opts)
        except RequestError as e:
            return JSONResponse({"detail": str(e)}, status_code=400, headers=headers)
        return JSONResponse(out, headers=headers)

    return app
