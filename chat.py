#!/usr/bin/env python3
"""Minimal OpenAI-compatible chat client for ``serve.py`` (reference: ``inference/zoro-1/chat.py``).

    python chat.py [--url http://127.0.0.1:30000] [--max-tokens 512] [--no-think] [--stream]
"""
import argparse
import json
import sys

import requests


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--url", default="http://127.0.0.1:30000")
    ap.add_argument("--max-tokens", type=int, default=512)
    ap.add_argument("--temperature", type=float, default=0.0)
    ap.add_argument("--no-think", action="store_true")
    ap.add_argument("--stream", action="store_true")
    args = ap.parse_args()
    model = requests.get(args.url + "/v1/models", timeout=10).json()["data"][0]["id"]
    history = []
    for line in sys.stdin if not sys.stdin.isatty() else iter(lambda: input("> "), None):
        line = line.strip()
        if not line:
            continue
        history.append({"role": "user", "content": line})
        body = {"model": model, "messages": history, "max_tokens": args.max_tokens, "temperature": args.temperature,
                "stream": args.stream, "chat_template_kwargs": {"enable_thinking": not args.no_think}}
        if args.stream:
            text = ""
            with requests.post(args.url + "/v1/chat/completions", json=body, stream=True) as r:
                for raw in r.iter_lines(decode_unicode=True):
                    if not raw or not raw.startswith("data: ") or raw == "data: [DONE]":
                        continue
                    d = json.loads(raw[6:])["choices"][0]["delta"].get("content", "")
                    text += d
                    print(d, end="", flush=True)
            print()
        else:
            r = requests.post(args.url + "/v1/chat/completions", json=body).json()
            msg = r["choices"][0]["message"]
            if msg.get("reasoning_content"):
                print("[thinking]", msg["reasoning_content"])
            text = msg.get("content") or ""
            print(text)
        history.append({"role": "assistant", "content": text})


if __name__ == "__main__":
    main()
