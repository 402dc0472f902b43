"""Serving engine: request scheduling, paged KV with radix prefix reuse, sampling."""
from .engine import Engine, Request
from .sampling import SamplingParams

__all__ = ["Engine", "Request", "SamplingParams"]
