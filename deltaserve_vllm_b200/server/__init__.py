"""HTTP serving: the engine loop thread and the FastAPI application."""

from .api import create_app
from .engine_thread import EngineThread

__all__ = ["create_app", "EngineThread"]
