"""CLI commands that need no GPU: chat (scripted input), status against a
running server, diagnostics."""
import io
import json
import socket
import threading
import time
import types


def test_chat_loop_keeps_history():
    from swarmllm_b200.cli import chat_loop
    from swarmllm_b200.engine import EngineConfig, LLMEngine
    from swarmllm_b200.models.config import tiny_llama
    from swarmllm_b200.models.weights import RandomSource
    from swarmllm_b200.serve.tokenizer import ByteTokenizer
    cfg = tiny_llama()
    eng = LLMEngine.from_config(cfg, "cpu", EngineConfig(max_model_len=512, max_running=2,
                                                         max_step_tokens=512, prefill_chunk=512),
                                source=RandomSource(cfg, seed=1))
    seen = []
    orig = eng.generate

    def spy(prompts, sp):
        seen.append(len(prompts[0]))
        return orig(prompts, sp)
    eng.generate = spy
    args = types.SimpleNamespace(system="be brief", max_tokens=4, temperature=0.0)
    fout = io.StringIO()
    chat_loop(eng, ByteTokenizer(cfg.vocab), None, args, io.StringIO("hello\nagain\n\n"), fout)
    assert fout.getvalue().count("> ") == 3 and len(seen) == 2
    assert seen[1] > seen[0]            # the second turn carries the first


def test_status_of_running_server():
    import uvicorn

    from swarmllm_b200.cli import node_status
    from swarmllm_b200.serve.api import AsyncEngine, create_app
    from swarmllm_b200.serve.tokenizer import ByteTokenizer
    from test_api_ext import Scripted
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ae = AsyncEngine(Scripted("x"))
    app = create_app(ae, ByteTokenizer(512), "m", max_model_len=512)
    srv = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=port, log_level="error"))
    th = threading.Thread(target=srv.run, daemon=True)
    th.start()
    try:
        for _ in range(100):
            if srv.started:
                break
            time.sleep(0.05)
        st = node_status(f"http://127.0.0.1:{port}")
        assert st["status"]["model"] == "m" and st["ready"] == {"status": "ready"}
        down = node_status("http://127.0.0.1:9")         # nothing listens there
        assert "error" in down["status"]
    finally:
        srv.should_exit = True
        th.join(5)
        ae.shutdown()


def test_diagnostics_cpu():
    from swarmllm_b200.utils.diagnostics import collect
    d = collect()
    assert d["devices"] == [] or "name" in d["devices"][0]
    assert d["native_extensions"]["swarmllm_b200._native"]
    json.dumps(d)
