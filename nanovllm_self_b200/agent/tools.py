"""Sandboxed agent tools (reference ``claude_self/tools.py``): ``read_file`` and an
allow-listed, keyword-filtered, time- and output-limited ``run_shell`` confined to a root."""
from __future__ import annotations

import shlex
import subprocess
from pathlib import Path

ALLOWED_COMMANDS = {"pwd", "ls", "cat", "head", "tail", "wc", "echo", "find", "grep", "rg"}
BLOCKED_KEYWORDS = {"rm", "mv", "cp", "sudo", "chmod", "chown", "kill", "pkill", "reboot", "shutdown", "mkfs", "dd",
                    "mount", "umount", "curl", "wget", "ssh", "scp", "git reset", "git clean"}


def read_file(path: str, max_chars: int = 4000, allowed_root: str | None = None) -> str:
    p = Path(path)
    if allowed_root is not None:
        try:
            p.resolve().relative_to(Path(allowed_root).resolve())
        except ValueError:
            return f"[read_file] outside the allowed root: {path}"
    if not p.exists():
        return f"[read_file] file not found: {path}"
    if not p.is_file():
        return f"[read_file] not a file: {path}"
    try:
        return p.read_text(encoding="utf-8")[:max_chars]
    except Exception as e:  # noqa: BLE001 - tool errors are reported to the model
        return f"[read_file] failed: {e}"


def run_shell(cmd: str, allowed_root: str = ".", timeout: int = 10, max_chars: int = 4000) -> str:
    cmd = cmd.strip()
    if not cmd:
        return "[run_shell] empty command"
    low = cmd.lower()
    for kw in BLOCKED_KEYWORDS:
        if (f" {kw} " in f" {low} ") or low.startswith(kw + " ") or low == kw:
            return f"[run_shell] blocked dangerous command: {kw}"
    if any(ch in cmd for ch in (";", "|", "&", ">", "<", "`", "$(")):
        return "[run_shell] shell operators are not allowed"
    try:
        parts = shlex.split(cmd)
    except ValueError as e:
        return f"[run_shell] failed to parse command: {e}"
    if not parts or parts[0] not in ALLOWED_COMMANDS:
        return f"[run_shell] command not allowed: {parts[0] if parts else ''}"
    root = Path(allowed_root)
    if not root.is_dir():
        return f"[run_shell] invalid allowed_root: {allowed_root}"
    try:
        r = subprocess.run(parts, capture_output=True, text=True, timeout=timeout, cwd=str(root))
    except subprocess.TimeoutExpired:
        return f"[run_shell] timed out after {timeout}s"
    out = (r.stdout or "") + (("\n[stderr]\n" + r.stderr) if r.stderr else "")
    return out[:max_chars] if out else f"[run_shell] exit code {r.returncode}, no output"


def make_tools(allowed_root: str = ".") -> dict:
    return {"read_file": lambda arg: read_file(arg, allowed_root=allowed_root),
            "run_shell": lambda arg: run_shell(arg, allowed_root=allowed_root)}
