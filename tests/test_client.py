"""The Python client package against a live server (uvicorn on 127.0.0.1, the
CPU engine with a tiny random model): sync and asyncio clients, streaming,
errors in the OpenAI envelope, admin routes."""
import asyncio
import socket
import threading
import time

import pytest


@pytest.fixture(scope="module")
def server():
    import uvicorn

    from swarmllm_b200.engine import EngineConfig, LLMEngine
    from swarmllm_b200.models.config import tiny_llama
    from swarmllm_b200.serve.api import AsyncEngine, create_app
    from swarmllm_b200.serve.tokenizer import ByteTokenizer
    cfg = tiny_llama()
    eng = LLMEngine.from_config(cfg, "cpu", EngineConfig(max_model_len=512, max_running=4,
                                                        max_step_tokens=512, prefill_chunk=256))
    ae = AsyncEngine(eng)
    app = create_app(ae, ByteTokenizer(cfg.vocab), "tiny-llama", max_model_len=512)
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    srv = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=port, log_level="warning"))
    th = threading.Thread(target=srv.run, daemon=True)
    th.start()
    for _ in range(200):
        if srv.started:
            break
        time.sleep(0.05)
    yield f"http://127.0.0.1:{port}"
    srv.should_exit = True
    th.join(timeout=10)
    ae.shutdown()


def test_sync_client(server):
    from swarmllm_b200.client import ChatMessage, SwarmLLM, SwarmLLMError
    with SwarmLLM(server) as c:
        assert [m.id for m in c.models()] == ["tiny-llama"]
        r = c.chat("hello", max_tokens=8, temperature=0.0, ignore_eos=True)
        assert r.usage.completion_tokens == 8 and r.model == "tiny-llama"
        r2 = c.chat_completion([ChatMessage("user", "hello")], max_tokens=8, temperature=0.0,
                               ignore_eos=True)
        assert r2.content == r.content                      # greedy: the same reply
        text = "".join(c.chat("hello", stream=True, max_tokens=8, temperature=0.0,
                              ignore_eos=True))
        assert text == r.content                            # streamed deltas add up to it
        cp = c.completion("abc", max_tokens=5)
        assert cp.usage.completion_tokens <= 5 and cp.finish_reason in ("length", "stop")
        assert c.health() is not None and "tiny-llama" in str(c.status())
        assert "swarmllm" in c.metrics()
        with pytest.raises(SwarmLLMError) as e:
            c.chat("x" * 2000, max_tokens=400)               # past the 512-token window
        assert e.value.status_code == 400 and isinstance(e.value.message, str)
        assert isinstance(c.admin.stats(), dict)


def test_async_client(server):
    from swarmllm_b200.client import AsyncSwarmLLM

    async def go():
        async with AsyncSwarmLLM(server) as c:
            r = await c.chat("hello", max_tokens=6, temperature=0.0, ignore_eos=True)
            parts = [d async for d in c.chat_stream([{"role": "user", "content": "hello"}],
                                                    max_tokens=6, temperature=0.0,
                                                    ignore_eos=True)]
            return r, "".join(parts)
    r, streamed = asyncio.run(go())
    assert r.usage.completion_tokens == 6 and streamed == r.content
