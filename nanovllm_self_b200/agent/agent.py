"""Agent loop: bootstrap -> llm <-> tool -> final (reference ``claude_self/agent.py:26-473``).

Each LLM call carries step metadata (``session_id``, ``step_id``, ``task_type``) so the
backends can use the session prefix cache and session-affine routing.
"""
from __future__ import annotations

import re

from .memory import trim_messages
from .parser import parse_agent_output
from .tools import make_tools

SYSTEM_PROMPT = (
    "You are a coding assistant with tools.\n"
    "To use a tool answer exactly:\nACTION: <read_file|run_shell>\nACTION_INPUT: <argument>\n"
    "When you know the answer, reply:\nFINAL: <answer>\n")


def build_prompt(messages: list) -> str:
    return "".join(f"{m['role'].upper()}: {m['content']}\n" for m in messages) + "ASSISTANT: "


class Agent:
    def __init__(self, backend, max_steps: int = 5, session_id: str | None = None, max_tokens: int = 128,
                 tools: dict | None = None, allowed_root: str = "."):
        self.backend = backend
        self.max_steps = max_steps
        self.max_tokens = max_tokens
        self.session_id = session_id or "agent-session-000000"
        self.tools = tools if tools is not None else make_tools(allowed_root)
        self.state: dict = {}
        self.trace: list = []

    # -------------------------------------------------------------- helpers
    @staticmethod
    def _extract_file_path(text: str):
        m = re.search(r"(/[\w\-. /]+\.py)\b", text)
        return m.group(1) if m else None

    def _task_type(self) -> str:
        msgs = self.state["messages"]
        if any(m["role"] == "tool" for m in msgs):
            return "tool_like"
        text = " ".join(m["content"] for m in msgs if m["role"] == "user").lower()
        if any(w in text for w in ("file", "code", "python", "search")):
            return "tool_like"
        return "simple_qa"

    def _metadata(self, prompt: str) -> dict:
        return {"session_id": self.session_id, "program_id": self.session_id, "step_id": self.state["step_id"],
                "task_type": self._task_type(), "prompt_chars": len(prompt)}

    # ---------------------------------------------------------------- nodes
    def _bootstrap(self, user_input: str) -> str:
        self.state = {"messages": [{"role": "system", "content": SYSTEM_PROMPT}, {"role": "user", "content": user_input}],
                      "step_id": 0, "executed": [], "final": None, "last_raw": None, "last_parsed": None}
        path = self._extract_file_path(user_input)
        if path and "read_file" in self.tools:
            # a file named in the request is read up front (one tool round trip saved)
            self._run_tool("read_file", path)
        return "llm"

    def _llm(self) -> str:
        if self.state["step_id"] >= self.max_steps:
            self.state["final"] = self.state["last_parsed"]["content"] if self.state["last_parsed"] and \
                self.state["last_parsed"]["type"] == "final" else "[agent] step limit reached"
            return "final"
        prompt = build_prompt(trim_messages(self.state["messages"]))
        raw = self.backend.generate_text(prompt, max_tokens=self.max_tokens, metadata=self._metadata(prompt))
        self.state["step_id"] += 1
        parsed = parse_agent_output(raw)
        self.state["last_raw"], self.state["last_parsed"] = raw, parsed
        self.trace.append({"step": self.state["step_id"], "raw": raw, "parsed": parsed})
        self.state["messages"].append({"role": "assistant", "content": raw})
        if parsed["type"] == "final":
            self.state["final"] = parsed["content"]
            return "final"
        key = (parsed["action"], parsed["action_input"])
        if key in self.state["executed"]:
            self.state["messages"].append({"role": "user", "content": "That tool call was already made; answer "
                                           "with FINAL: using its result."})
            return "llm"
        return "tool"

    def _run_tool(self, action: str, arg: str) -> None:
        fn = self.tools.get(action)
        result = fn(arg) if fn is not None else f"[agent] unknown tool: {action}"
        self.state["executed"].append((action, arg))
        self.state["messages"].append({"role": "tool", "content": f"TOOL_RESULT for {action}:\nINPUT: {arg}\n{result}"})

    def _tool(self) -> str:
        p = self.state["last_parsed"]
        self._run_tool(p["action"], p["action_input"])
        return "llm"

    def run(self, user_input: str) -> str:
        node = self._bootstrap(user_input)
        guard = 0
        while node != "final":
            node = self._llm() if node == "llm" else self._tool()
            guard += 1
            if guard > 4 * self.max_steps + 4:
                self.state["final"] = "[agent] loop guard tripped"
                break
        return self.state["final"] or ""
