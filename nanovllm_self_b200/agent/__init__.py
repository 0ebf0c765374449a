"""A small tool-using agent that drives the engine (or the P/D pool) as its LLM backend.

Reference: ``claude_self/`` (LangGraph agent with ``read_file`` / ``run_shell`` tools,
``ACTION:`` / ``FINAL:`` output protocol, prompt-memory trimming, and local, router-
scheduled and P/D-pool backends).  LangGraph is not available here; the same graph
``START -> bootstrap -> llm <-> tool -> final -> END`` is an explicit state machine.
"""
from .agent import Agent
from .backends import FakeBackend, LocalBackend, PDPoolBackend, ScheduledBackend
from .parser import parse_agent_output

__all__ = ["Agent", "FakeBackend", "LocalBackend", "ScheduledBackend", "PDPoolBackend", "parse_agent_output"]
