"""Prompt memory trimming (reference ``claude_self/memory.py``): keep the newest messages
within a character budget, shorten long tool results in the middle, and keep only the
newest result of a repeated (tool, input) call."""
from __future__ import annotations


def shorten_text(text: str, max_chars: int) -> str:
    if len(text) <= max_chars:
        return text
    half = max_chars // 2
    return text[:half] + "\n\n...[truncated]...\n\n" + text[-half:]


def _tool_key(content: str):
    if not content.startswith("TOOL_RESULT for "):
        return None
    action = inp = None
    for ln in content.splitlines():
        if ln.startswith("TOOL_RESULT for "):
            action = ln[len("TOOL_RESULT for "):].strip().rstrip(":")
        elif ln.startswith("INPUT:"):
            inp = ln[len("INPUT:"):].strip()
    return None if action is None else (action, inp or "")


def trim_messages(messages: list, max_context_chars: int = 8000, max_tool_chars: int = 3000) -> list:
    kept, total, seen = [], 0, set()
    system = [m for m in messages[:1] if m["role"] == "system"]
    body = messages[len(system):]
    for m in reversed(body):
        content = shorten_text(m["content"], max_tool_chars) if m["role"] == "tool" else m["content"]
        if m["role"] == "tool":
            key = _tool_key(content)
            if key is not None:
                if key in seen:
                    continue
                seen.add(key)
        n = len(f"{m['role'].upper()}: {content}\n")
        if total + n > max_context_chars:
            break
        kept.append({"role": m["role"], "content": content})
        total += n
    return system + list(reversed(kept))
