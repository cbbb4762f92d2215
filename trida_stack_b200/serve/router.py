"""Data-parallel serving front end: one OpenAI base URL in front of N replica servers (one
``serve.py`` per GPU or per TP group).  The reference's ``benchmark/serving/router.py`` cycles
round-robin with fail-over; this router sends each request to the replica with the fewest requests
in flight (round-robin among ties), fails over on connection errors, non-2xx answers or bodies
that are not JSON, passes streamed (``"stream": true``) responses through chunk by chunk, and sums
the replicas' ``/v1/stats`` counters.

    python -m trida_stack_b200.serve.router --port 8000 --upstreams http://127.0.0.1:8001,http://127.0.0.1:8002
"""
import argparse
import itertools
import json
import threading


def build_app(upstreams, timeout=1200.0):
    import httpx
    from fastapi import FastAPI, Request
    from fastapi.responses import JSONResponse, StreamingResponse

    app = FastAPI()
    client = httpx.AsyncClient(timeout=timeout)
    inflight = {u: 0 for u in upstreams}
    order = itertools.count()
    lock = threading.Lock()

    def ranked():
        """Upstreams by requests in flight, ties broken round-robin."""
        with lock:
            k = next(order)
            n = len(upstreams)
            return sorted(upstreams, key=lambda u: (inflight[u], (upstreams.index(u) - k) % n))

    def enter(u, d):
        with lock:
            inflight[u] += d

    @app.get("/health")
    async def health():
        return {"status": "ok", "upstreams": upstreams, "inflight": dict(inflight)}

    @app.get("/v1/models")
    async def models():
        for u in upstreams:
            try:
                r = await client.get(f"{u}/v1/models")
                return JSONResponse(r.json(), status_code=r.status_code)
            except Exception:
                continue
        return JSONResponse({"error": {"message": "no upstream answered"}}, status_code=502)

    @app.get("/v1/stats")
    async def stats():
        tot = {"forwards": 0, "tokens": 0, "prefill_tokens": 0, "replicas": 0}
        for u in upstreams:
            try:
                st = (await client.get(f"{u}/v1/stats")).json()
            except Exception:
                continue
            tot["replicas"] += 1
            for k in ("forwards", "tokens", "prefill_tokens"):
                tot[k] += int(st.get(k, 0))
        tot["tok_per_fwd"] = round(tot["tokens"] / tot["forwards"], 4) if tot["forwards"] else None
        return tot

    async def proxy(path, body):
        try:
            stream = bool(json.loads(body or b"{}").get("stream"))
        except ValueError:
            return JSONResponse({"error": {"message": "request body is not JSON"}}, status_code=400)
        last = None
        for up in ranked():
            enter(up, 1)
            try:
                if stream:
                    req = client.build_request("POST", f"{up}{path}", content=body,
                                               headers={"content-type": "application/json"})
                    r = await client.send(req, stream=True)
                    if r.status_code // 100 != 2:
                        await r.aclose()
                        last = f"{up}: HTTP {r.status_code}"
                        enter(up, -1)
                        continue

                    async def relay(r=r, up=up):
                        try:
                            async for chunk in r.aiter_raw():
                                yield chunk
                        finally:
                            await r.aclose()
                            enter(up, -1)
                    return StreamingResponse(relay(), media_type=r.headers.get("content-type", "text/event-stream"))
                r = await client.post(f"{up}{path}", content=body, headers={"content-type": "application/json"})
            except Exception as e:
                last = f"{up}: {type(e).__name__}: {e}"
                enter(up, -1)
                continue
            enter(up, -1)
            if r.status_code // 100 != 2:
                last = f"{up}: HTTP {r.status_code}"
                continue
            try:
                return JSONResponse(r.json(), status_code=200)
            except ValueError as e:
                last = f"{up}: bad JSON ({e})"
        return JSONResponse({"error": {"message": f"all upstreams failed: {last}"}}, status_code=502)

    for path in ("/v1/completions", "/v1/chat/completions", "/v1/systemone", "/v1/decide"):
        async def handler(request: Request, path=path):
            return await proxy(path, await request.body())
        app.add_api_route(path, handler, methods=["POST"])
    return app


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--host", default="0.0.0.0")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--upstreams", required=True, help="comma-separated base URLs of the replica servers")
    ap.add_argument("--timeout", type=float, default=1200.0)
    a = ap.parse_args(argv)
    import uvicorn
    ups = [u.strip().rstrip("/") for u in a.upstreams.split(",") if u.strip()]
    uvicorn.run(build_app(ups, a.timeout), host=a.host, port=a.port, log_level="warning")


if __name__ == "__main__":
    main()
