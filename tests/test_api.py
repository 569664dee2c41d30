"""HTTP API on the CPU engine (tiny random model, byte tokenizer)."""
import json

import pytest


@pytest.fixture(scope="module")
def client():
    from fastapi.testclient import TestClient

    from swarmllm_b200.engine import EngineConfig, LLMEngine
    from swarmllm_b200.models.config import tiny_llama
    from swarmllm_b200.serve.api import AsyncEngine, create_app
    from swarmllm_b200.serve.tokenizer import ByteTokenizer
    cfg = tiny_llama()
    eng = LLMEngine.from_config(cfg, "cpu", EngineConfig(max_model_len=512, max_running=4,
                                                        max_step_tokens=512, prefill_chunk=256))
    ae = AsyncEngine(eng)
    app = create_app(ae, ByteTokenizer(cfg.vocab), "tiny-llama", max_model_len=512)
    with TestClient(app) as c:
        yield c
    ae.shutdown()


def test_chat_completion(client):
    r = client.post("/v1/chat/completions", json={
        "model": "tiny-llama", "messages": [{"role": "user", "content": "hello"}],
        "max_tokens": 8, "temperature": 0})
    assert r.status_code == 200, r.text
    j = r.json()
    assert j["object"] == "chat.completion"
    assert j["choices"][0]["finish_reason"] in ("length", "stop")
    assert j["usage"]["prompt_tokens"] > 0
    assert "x-swarmllm-ttft-ms" in r.headers


def test_chat_completion_stream(client):
    with client.stream("POST", "/v1/chat/completions", json={
            "model": "tiny-llama", "messages": [{"role": "user", "content": "hi"}],
            "max_tokens": 6, "temperature": 0.7, "seed": 3, "stream": True}) as r:
        assert r.status_code == 200
        lines = [l for l in r.iter_lines() if l.startswith("data: ")]
    assert lines[-1] == "data: [DONE]"
    chunks = [json.loads(l[6:]) for l in lines[:-1]]
    assert chunks[0]["choices"][0]["delta"].get("role") == "assistant"
    assert chunks[-1]["choices"][0]["finish_reason"] is not None


def test_completions_and_messages_and_models(client):
    r = client.post("/v1/completions", json={"prompt": [5, 6, 7, 8], "max_tokens": 4})
    assert r.status_code == 200 and r.json()["object"] == "text_completion"
    r = client.post("/v1/messages", json={"model": "x", "system": "be brief", "max_tokens": 4,
                                          "messages": [{"role": "user", "content": "yo"}]})
    assert r.status_code == 200 and r.json()["type"] == "message"
    r = client.get("/v1/models")
    assert r.json()["data"][0]["id"] == "tiny-llama"
    r = client.post("/v1/embeddings", json={"input": ["abc", "de"]})
    assert len(r.json()["data"]) == 2 and len(r.json()["data"][0]["embedding"]) == 256


def test_health_metrics_status(client):
    assert client.get("/health").json()["status"] == "ok"
    assert client.get("/health/ready").status_code == 200
    m = client.get("/metrics").text
    assert "swarmllm_inference_requests_total" in m and "swarmllm_kv_pages_free" in m
    for name in ("swarmllm_requests_running", "swarmllm_requests_waiting",
                 "swarmllm_prefix_cache_hit_tokens", "swarmllm_preemptions"):
        assert name in m, name
    assert "swarmllm_ready 1.0" in m
    s = client.get("/api/status").json()
    assert s["kv_pages"] > 0


def test_context_window_rejected(client):
    r = client.post("/v1/chat/completions", json={
        "messages": [{"role": "user", "content": "x"}], "max_tokens": 100000})
    assert r.status_code == 400


def test_tokenizers_roundtrip():
    from swarmllm_b200.serve.tokenizer import BPETokenizer, ByteTokenizer, _bytes_to_unicode
    bt = ByteTokenizer(1000)
    assert bt.decode(bt.encode("héllo wörld")) == "héllo wörld"
    b2u = _bytes_to_unicode()
    toks = [b2u[b] for b in range(256)] + ["he", "ll", "hell", "hello", "Ġw"]
    merges = ["h e", "l l", "he ll", "hell o", "Ġ w"]
    tk = BPETokenizer(toks, merges)
    ids = tk.encode("hello world", add_bos=False)
    assert tk.decode(ids) == "hello world"
    assert toks.index("hello") in ids


def test_prefix_snapshot_over_http(client):
    """Export the cached prefix of a completed prompt, then import it into a
    second server: the second server caches the pages."""
    from fastapi.testclient import TestClient

    from swarmllm_b200.engine import EngineConfig, LLMEngine
    from swarmllm_b200.models.config import tiny_llama
    from swarmllm_b200.serve.api import AsyncEngine, create_app
    from swarmllm_b200.serve.tokenizer import ByteTokenizer
    ids = list(range(5, 5 + 40))
    r = client.post("/v1/completions", json={"prompt": ids, "max_tokens": 2, "temperature": 0})
    assert r.status_code == 200
    r = client.post("/api/prefix/export", json={"tokens": ids})
    assert r.status_code == 200 and r.headers["x-swarmllm-prefix-tokens"] == "32"
    snap = r.content
    assert client.post("/api/prefix/import", content=snap).json()["imported_tokens"] == 0
    assert client.post("/api/prefix/import", content=b"garbage").status_code == 400
    cfg = tiny_llama()
    eng = LLMEngine.from_config(cfg, "cpu", EngineConfig(max_model_len=512, max_running=4,
                                                        max_step_tokens=512, prefill_chunk=256))
    ae = AsyncEngine(eng)
    with TestClient(create_app(ae, ByteTokenizer(cfg.vocab), "tiny-llama", max_model_len=512)) as c2:
        assert c2.post("/api/prefix/import", content=snap).json()["imported_tokens"] == 32
        assert c2.post("/api/prefix/export", json={"tokens": [9, 9, 9]}).status_code == 204
    ae.shutdown()
