"""Native serving stack: slot runtime (KV / gated-delta caches, canvas step), self-speculative and
autoregressive engine, OpenAI-compatible HTTP server and the typed-decision engine."""
from .engine import Engine, Request, SamplingParams
from .runtime import Runtime

__all__ = ["Engine", "Request", "Runtime", "SamplingParams"]
