"""OpenAI/Anthropic-compatible gateway with the agent-kernel floor, and its model backends."""
from .backend import EngineBackend, ReferenceBackend, UpstreamBackend
from .gateway import Gateway, create_app

__all__ = ["EngineBackend", "ReferenceBackend", "UpstreamBackend", "Gateway", "create_app"]
