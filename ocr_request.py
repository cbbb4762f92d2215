#!/usr/bin/env python3
"""Send one image crop to a running GravityOCR server (``serve_gravityocr.py``) and print the text.

One layout region per request; pick the task that matches the crop (or give --prompt):

    --task text       Text Recognition:      plain text in reading order (default)
    --task table      Table Recognition:     the table as HTML
    --task formula    Formula Recognition:   the formula as LaTeX

    python ocr_request.py crop.png [--task table] [--url http://127.0.0.1:30000]
    python ocr_request.py --synthetic "Hello GravityOCR"      # renders the text into a PNG first

The image travels inside the request as a base64 data URL.  The bearer key is read from $API_KEY
only (command-line arguments are visible to other users); the request goes to --url and nowhere
else: redirects are refused and proxy variables ignored, so the key is never sent to another host.
Exit status 1 with a one-line message on an HTTP error, a connection failure, a timeout or a reply
without text.  Standard library only (Pillow only for --synthetic).
"""
import argparse
import base64
import io
import json
import os
import sys
import urllib.error
import urllib.request
from pathlib import Path

TASK_PROMPTS = {"text": "Text Recognition:", "table": "Table Recognition:", "formula": "Formula Recognition:"}
MIME = {".png": "image/png", ".jpg": "image/jpeg", ".jpeg": "image/jpeg", ".webp": "image/webp",
        ".bmp": "image/bmp", ".gif": "image/gif", ".tif": "image/tiff", ".tiff": "image/tiff"}


class _NoRedirect(urllib.request.HTTPRedirectHandler):
    def redirect_request(self, req, fp, code, msg, headers, newurl):
        raise urllib.error.HTTPError(req.full_url, code, f"redirect to {newurl} refused", headers, fp)


def synthetic_png(text):
    from PIL import Image, ImageDraw
    w = max(64, 8 * len(text) + 16)
    img = Image.new("RGB", (w, 32), "white")
    ImageDraw.Draw(img).text((8, 10), text, fill="black")
    buf = io.BytesIO()
    img.resize((2 * w, 64)).save(buf, format="PNG")
    return buf.getvalue(), "image/png"


def build_body(image_bytes, mime, prompt, model, max_tokens):
    url = f"data:{mime};base64," + base64.b64encode(image_bytes).decode()
    return {"model": model, "max_tokens": max_tokens, "temperature": 0,
            "messages": [{"role": "user", "content": [{"type": "image_url", "image_url": {"url": url}},
                                                      {"type": "text", "text": prompt}]}]}


def send(body, url, timeout, api_key=None):
    req = urllib.request.Request(url.rstrip("/") + "/v1/chat/completions", data=json.dumps(body).encode(),
                                 headers={"Content-Type": "application/json"}, method="POST")
    if api_key:
        req.add_header("Authorization", f"Bearer {api_key}")
    opener = urllib.request.build_opener(urllib.request.ProxyHandler({}), _NoRedirect())
    with opener.open(req, timeout=timeout) as r:
        return json.loads(r.read().decode())


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("image", nargs="?")
    ap.add_argument("--synthetic", default=None, metavar="TEXT")
    ap.add_argument("--task", choices=list(TASK_PROMPTS), default="text")
    ap.add_argument("--prompt", default=None)
    ap.add_argument("--url", default="http://127.0.0.1:30000")
    ap.add_argument("--model", default="glm-ocr")
    ap.add_argument("--max-tokens", type=int, default=4096)
    ap.add_argument("--timeout", type=float, default=300.0)
    a = ap.parse_args(argv)
    if a.synthetic is not None:
        data, mime = synthetic_png(a.synthetic)
    elif a.image:
        p = Path(a.image)
        if p.suffix.lower() not in MIME:
            print(f"error: unsupported image type {p.suffix!r}", file=sys.stderr)
            return 1
        data, mime = p.read_bytes(), MIME[p.suffix.lower()]
    else:
        print("error: give an image file or --synthetic TEXT", file=sys.stderr)
        return 1
    body = build_body(data, mime, a.prompt or TASK_PROMPTS[a.task], a.model, a.max_tokens)
    try:
        r = send(body, a.url, a.timeout, os.environ.get("API_KEY"))
        text = r["choices"][0]["message"]["content"]
    except urllib.error.HTTPError as e:
        print(f"error: HTTP {e.code}: {e.reason}", file=sys.stderr)
        return 1
    except (urllib.error.URLError, TimeoutError, OSError) as e:
        print(f"error: {e}", file=sys.stderr)
        return 1
    except (KeyError, IndexError, TypeError, ValueError):
        print("error: the reply has no choices[0].message.content", file=sys.stderr)
        return 1
    print(text)
    print(json.dumps(r.get("usage", {})), file=sys.stderr)
    return 0


if __name__ == "__main__":
    sys.exit(main())
