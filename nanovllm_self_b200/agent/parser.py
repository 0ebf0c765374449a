"""Model-output protocol of the agent (reference ``claude_self/parser.py``).

``FINAL: <answer>`` ends the loop; ``ACTION: <tool>`` + ``ACTION_INPUT: <arg>`` requests a tool
call; anything else is treated as a final answer.  Small models often keep talking after
their answer, so a final answer is cut at the first continuation marker.
"""
from __future__ import annotations

STOP_MARKERS = ("\nWait,", "\nOkay,", "\nBut ", "\nHowever,", "\nACTION:", "\nACTION_INPUT:", "\nUSER:",
                "\nASSISTANT:", "\nTOOL:")
NO_ACTION = {"", "none", "null", "nil"}


def clean_final_content(text: str) -> str:
    out = text.strip()
    cut = min((i for i in (out.find(m) for m in STOP_MARKERS) if i != -1), default=-1)
    return out[:cut].strip() if cut != -1 else out


def parse_agent_output(text: str) -> dict:
    text = text.strip()
    i = text.find("FINAL:")
    if i != -1:
        return {"type": "final", "content": clean_final_content(text[i + len("FINAL:"):])}
    lines = text.splitlines()
    if lines and lines[0].strip() == "FINAL":
        return {"type": "final", "content": clean_final_content("\n".join(lines[1:]))}
    action = action_input = None
    for ln in lines:
        if ln.startswith("ACTION:"):
            action = ln[len("ACTION:"):].strip()
        elif ln.startswith("ACTION_INPUT:"):
            action_input = ln[len("ACTION_INPUT:"):].strip()
    if action is not None:
        if action.lower() in NO_ACTION:
            return {"type": "final", "content": text}
        return {"type": "action", "action": action, "action_input": action_input or ""}
    return {"type": "final", "content": clean_final_content(text)}
