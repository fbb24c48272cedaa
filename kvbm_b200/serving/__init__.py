"""Serving harness: the engine that drives the block manager's connector
(scheduler + model runner + connector hooks) and the P/D deployment built
on it."""

from .engine import DecodeBatch, EngineConfig, LLMEngine, Request, RequestStatus

__all__ = ["DecodeBatch", "EngineConfig", "LLMEngine", "Request", "RequestStatus"]
