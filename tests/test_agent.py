"""Agent loop with a scripted backend (the reference's only mock, ``claude_self/tests``) and with
the real engine (tiny CPU model) behind LocalBackend / ScheduledBackend."""
from nanovllm_self_b200 import LLM
from nanovllm_self_b200.agent import Agent, FakeBackend, LocalBackend, ScheduledBackend, parse_agent_output
from nanovllm_self_b200.agent.memory import trim_messages
from nanovllm_self_b200.agent.tools import read_file, run_shell


def test_tool_loop_action_then_final(tmp_path):
    f = tmp_path / "hello.txt"
    f.write_text("print('hi')\n")
    be = FakeBackend([f"ACTION: read_file\nACTION_INPUT: {f}", "FINAL: it prints hi\nWait, more"])
    agent = Agent(be, session_id="s-1", allowed_root=str(tmp_path))
    assert agent.run("what does the file do?") == "it prints hi"
    assert len(be.calls) == 2
    assert "TOOL_RESULT for read_file" in be.calls[1]["prompt"] and "print('hi')" in be.calls[1]["prompt"]
    md = be.calls[1]["metadata"]
    assert md["session_id"] == "s-1" and md["step_id"] == 1 and md["task_type"] == "tool_like"


def test_parser_protocol():
    assert parse_agent_output("FINAL: 42") == {"type": "final", "content": "42"}
    assert parse_agent_output("ACTION: run_shell\nACTION_INPUT: ls")["action_input"] == "ls"
    assert parse_agent_output("ACTION: none")["type"] == "final"
    assert parse_agent_output("just text\nOkay, also")["content"] == "just text"


def test_tools_are_sandboxed(tmp_path):
    (tmp_path / "a.txt").write_text("x")
    assert "a.txt" in run_shell("ls", allowed_root=str(tmp_path))
    assert "blocked" in run_shell("rm -rf /", allowed_root=str(tmp_path))
    assert "not allowed" in run_shell("python -c 1", allowed_root=str(tmp_path))
    assert "operators" in run_shell("ls; cat /etc/passwd", allowed_root=str(tmp_path))
    assert "outside" in read_file("/etc/hostname", allowed_root=str(tmp_path))


def test_memory_trims_and_dedups():
    msgs = [{"role": "system", "content": "S"}] + [
        {"role": "tool", "content": "TOOL_RESULT for read_file:\nINPUT: /a\n" + "x" * 5000} for _ in range(3)] + [
        {"role": "user", "content": "q"}]
    out = trim_messages(msgs, max_context_chars=4000, max_tool_chars=1000)
    assert out[0]["role"] == "system" and sum(m["role"] == "tool" for m in out) == 1


def test_real_engine_backends():
    llm = LLM("tiny", device="cpu", dtype="fp32", block_size=16, num_blocks=128, max_model_len=1024)
    agent = Agent(LocalBackend(llm), max_steps=2, max_tokens=8)
    assert isinstance(agent.run("hello"), str)
    sb = ScheduledBackend([llm, llm])
    Agent(sb, max_steps=2, max_tokens=4, session_id="sess").run("hi")
    assert sb.routes and all(r["session_id"] == "sess" for r in sb.routes)
