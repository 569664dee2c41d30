"""Tool calling, the Responses API, the MCP server and the request guards.

The server logic is tested against a scripted engine whose output text is
fixed (through the byte tokenizer), so tool-call parsing and the event
sequences are exact; the real CPU engine is covered by test_api.py."""
import json
import time
import types

import pytest

from swarmllm_b200.serve.tools import (ToolSpec, content_prefix_len, parse_tool_calls,
                                       tools_from_openai)

WEATHER = ToolSpec("get_weather", "weather", {"type": "object", "properties": {
    "city": {"type": "string"}, "days": {"type": "integer"}}})
DATE = ToolSpec("date")


@pytest.mark.parametrize("text,want", [
    ('{"tool_calls": [{"name": "get_weather", "arguments": {"city": "Paris"}}]}',
     [("get_weather", {"city": "Paris"})]),
    ('Sure. {"tool_calls": [{"function": {"name": "date", "arguments": "{}"}}]}', [("date", {})]),
    ('<tool_call>\n{"name": "get_weather", "arguments": {"city": "Oslo"}}\n</tool_call>'
     '<tool_call>{"name":"date","arguments":{}}</tool_call>',
     [("get_weather", {"city": "Oslo"}), ("date", {})]),
    ('<tool_call>\n<function=get_weather>\n<parameter=city>\nRome\n</parameter>\n'
     '<parameter=days>\n3\n</parameter>\n</function>\n</tool_call>',
     [("get_weather", {"city": "Rome", "days": 3})]),
    ('[TOOL_CALLS][{"name": "date", "arguments": {}}]', [("date", {})]),
    ('[TOOL_CALLS]get_weather[ARGS]{"city": "Kyiv"}', [("get_weather", {"city": "Kyiv"})]),
    ('functools[{"name": "date", "arguments": {}}]', [("date", {})]),
    ('<|tool_calls|>[{"name": "date", "arguments": {}}]<|/tool_calls|>', [("date", {})]),
    ('<|python_tag|>{"name": "get_weather", "parameters": {"city": "Lima"}}',
     [("get_weather", {"city": "Lima"})]),
    ('{"name": "get_weather", "parameters": {"city": "Lima"}}', [("get_weather", {"city": "Lima"})]),
    ('```json\n{"tool_calls": [{"name": "date", "arguments": {}}]}\n```', [("date", {})]),
    ("The answer is {x} in math.", None),
    ('{"tool_calls": [{"name": "rm_rf", "arguments": {}}]}', None),     # undeclared tool
    ('{"tool_calls": [{"name": "date", "argum', None),                   # truncated
    ('{"name": "get_weather", "parameters": {"type": "object", "properties": {}}}', None),  # echo
])
def test_parse_tool_calls(text, want):
    r = parse_tool_calls(text, [WEATHER, DATE])
    if want is None:
        assert r is None
        return
    lead, calls = r
    assert [(c.name, json.loads(c.arguments)) for c in calls] == want
    assert len({c.id for c in calls}) == len(calls)


def test_content_prefix_len_streaming():
    assert content_prefix_len("Hello world") == 11
    assert content_prefix_len("Hello <tool") == 6
    assert content_prefix_len("Hello {") == 6
    assert content_prefix_len("x [TOOL") == 2
    assert content_prefix_len("ab`") == 2


def test_tools_from_openai_rejects_builtin():
    with pytest.raises(ValueError):
        tools_from_openai([{"type": "web_search"}])
    assert tools_from_openai([{"type": "function", "name": "f"}])[0].name == "f"


# --------------------------------------------------------------------------- scripted engine
class Scripted:
    """Engine stand-in: every request generates `script` (byte tokens, offset
    3, then EOS=2), one token per step."""

    def __init__(self, script: str, step_s: float = 0.0):
        self.script = [b + 3 for b in script.encode()] + [2]
        self.step_s = step_s
        self.reqs, self.traces, self.steps = {}, {}, 0
        self.lora_names = ["ad1"]
        self.loras = {}
        self.sched = types.SimpleNamespace(num_running=0, num_waiting=0)
        self.bm = types.SimpleNamespace(num_free=lambda: 10, num_pages=10, prefix_hit_tokens=0)
        self.prompts = []

    def add_request(self, ids, sp, request_id, lora=None):
        self.reqs[request_id] = [0, sp.max_tokens]
        self.loras[request_id] = lora
        self.prompts.append(ids)

    def has_work(self):
        return bool(self.reqs)

    def step(self):
        time.sleep(self.step_s)
        self.steps += 1
        out = []
        for rid, st in list(self.reqs.items()):
            tok = self.script[min(st[0], len(self.script) - 1)]
            st[0] += 1
            fin = st[0] >= st[1] or tok == 2
            out.append((rid, tok, fin))
            if fin:
                del self.reqs[rid]
        return out

    def abort(self, rid):
        self.reqs.pop(rid, None)

    def release(self, rid):
        pass


def _client(script, step_s=0.0, **kw):
    from fastapi.testclient import TestClient

    from swarmllm_b200.serve.api import AsyncEngine, create_app
    from swarmllm_b200.serve.tokenizer import ByteTokenizer
    eng = Scripted(script, step_s)
    ae = AsyncEngine(eng)
    app = create_app(ae, ByteTokenizer(512), "m", max_model_len=4096, **kw)
    return TestClient(app), ae, eng


TOOLS = [{"type": "function", "function": {"name": "get_weather", "description": "w",
                                           "parameters": WEATHER.parameters}}]
CALL = '{"tool_calls": [{"name": "get_weather", "arguments": {"city": "Paris"}}]}'


def test_chat_tool_call_and_stream():
    c, ae, eng = _client(CALL)
    with c:
        r = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "w?"}],
                                                 "tools": TOOLS, "max_tokens": 200})
        j = r.json()
        ch = j["choices"][0]
        assert ch["finish_reason"] == "tool_calls", j
        tc = ch["message"]["tool_calls"][0]
        assert tc["function"]["name"] == "get_weather"
        assert json.loads(tc["function"]["arguments"]) == {"city": "Paris"}
        assert j["usage"]["completion_tokens"] == len(CALL) + 1
        # the tool prompt reached the model
        assert b"get_weather" in bytes(t - 3 for t in eng.prompts[-1] if 3 <= t < 259)
        with c.stream("POST", "/v1/chat/completions", json={
                "messages": [{"role": "user", "content": "w?"}], "tools": TOOLS, "stream": True,
                "max_tokens": 200}) as s:
            chunks = [json.loads(l[6:]) for l in s.iter_lines() if l.startswith("data: {")]
        deltas = [x["choices"][0]["delta"] for x in chunks]
        assert not any(d.get("content") for d in deltas)       # the JSON never leaks as content
        assert any("tool_calls" in d for d in deltas)
        assert chunks[-1]["choices"][0]["finish_reason"] == "tool_calls"
        # tool_choice none: the JSON is plain content
        r = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "w?"}],
                                                 "tools": TOOLS, "tool_choice": "none", "max_tokens": 200})
        assert r.json()["choices"][0]["message"]["content"] == CALL
        # a follow-up turn carrying the call and its result renders
        r = c.post("/v1/chat/completions", json={"messages": [
            {"role": "user", "content": "w?"},
            {"role": "assistant", "content": None, "tool_calls": [tc]},
            {"role": "tool", "tool_call_id": tc["id"], "content": "sunny"}], "tools": TOOLS,
            "max_tokens": 200})
        assert r.status_code == 200
    ae.shutdown()


def test_anthropic_tool_use():
    c, ae, _ = _client(CALL)
    with c:
        r = c.post("/v1/messages", json={"max_tokens": 200, "messages": [{"role": "user", "content": "w"}],
                                         "tools": [{"name": "get_weather", "input_schema": WEATHER.parameters}]})
        j = r.json()
        assert j["stop_reason"] == "tool_use"
        blk = [b for b in j["content"] if b["type"] == "tool_use"][0]
        assert blk["name"] == "get_weather" and blk["input"] == {"city": "Paris"}
        with c.stream("POST", "/v1/messages", json={
                "max_tokens": 200, "stream": True, "messages": [{"role": "user", "content": "w"}],
                "tools": [{"name": "get_weather", "input_schema": WEATHER.parameters}]}) as s:
            evs = [json.loads(l[6:]) for l in s.iter_lines() if l.startswith("data: ")]
        kinds = [e["type"] for e in evs]
        assert kinds[0] == "message_start" and kinds[-1] == "message_stop"
        assert any(e.get("delta", {}).get("type") == "input_json_delta" for e in evs)
        assert [e for e in evs if e["type"] == "message_delta"][0]["delta"]["stop_reason"] == "tool_use"
    ae.shutdown()


def test_lora_selected_by_model_name():
    c, ae, eng = _client("hi")
    with c:
        c.post("/v1/chat/completions", json={"model": "m:ad1", "max_tokens": 4,
                                             "messages": [{"role": "user", "content": "x"}]})
        c.post("/v1/chat/completions", json={"model": "m", "max_tokens": 4,
                                             "messages": [{"role": "user", "content": "x"}]})
        assert list(eng.loras.values()) == ["ad1", None]
        assert [m["id"] for m in c.get("/v1/models").json()["data"]] == ["m", "m:ad1"]
    ae.shutdown()


# --------------------------------------------------------------------------- Responses API
def test_responses_basic_chain_and_items():
    c, ae, eng = _client("Hello there")
    with c:
        r = c.post("/v1/responses", json={"model": "m", "input": "hi", "instructions": "be nice",
                                          "max_output_tokens": 64})
        j = r.json()
        assert r.status_code == 200 and j["status"] == "completed", j
        assert j["output"][0]["type"] == "message"
        assert j["output"][0]["content"][0]["text"] == "Hello there" == j["output_text"]
        assert j["usage"]["output_tokens"] == len("Hello there") + 1
        rid = j["id"]
        assert c.get(f"/v1/responses/{rid}").json()["id"] == rid
        # chaining: the previous input and output are in the new prompt, its instructions are not
        r2 = c.post("/v1/responses", json={"input": [{"role": "user", "content": "again"}],
                                           "previous_response_id": rid, "max_output_tokens": 64})
        assert r2.status_code == 200
        prompt = bytes(t - 3 for t in eng.prompts[-1] if 3 <= t < 259).decode()
        assert "hi" in prompt and "Hello there" in prompt and "again" in prompt
        assert "be nice" not in prompt
        items = c.get(f"/v1/responses/{r2.json()['id']}/input_items?order=asc").json()
        assert items["data"][0]["type"] == "message" and not items["has_more"]
        # truncation -> incomplete
        r3 = c.post("/v1/responses", json={"input": "hi", "max_output_tokens": 3}).json()
        assert r3["status"] == "incomplete" and r3["incomplete_details"]["reason"] == "max_output_tokens"
        # store=false is not retrievable; delete works once
        r4 = c.post("/v1/responses", json={"input": "hi", "store": False, "max_output_tokens": 8}).json()
        assert c.get(f"/v1/responses/{r4['id']}").status_code == 404
        assert c.delete(f"/v1/responses/{rid}").json()["deleted"] is True
        assert c.delete(f"/v1/responses/{rid}").status_code == 404
        assert c.post("/v1/responses", json={"input": "x", "previous_response_id": rid}).status_code == 404
        assert c.post("/v1/responses", json={"input": "x", "tools": [{"type": "web_search"}]}).status_code == 400
    ae.shutdown()


def test_responses_stream_events_and_function_calls():
    c, ae, _ = _client(CALL)
    with c:
        with c.stream("POST", "/v1/responses", json={"input": "w?", "stream": True, "max_output_tokens": 200,
                                                     "tools": [{"type": "function", "name": "get_weather",
                                                                "parameters": WEATHER.parameters}]}) as s:
            evs = [json.loads(l[6:]) for l in s.iter_lines() if l.startswith("data: ")]
        kinds = [e["type"] for e in evs]
        assert kinds[:2] == ["response.created", "response.in_progress"]
        assert kinds[-1] == "response.completed"
        assert "response.function_call_arguments.done" in kinds
        assert [e["sequence_number"] for e in evs] == list(range(1, len(evs) + 1))
        out = evs[-1]["response"]["output"]
        assert out[-1]["type"] == "function_call" and json.loads(out[-1]["arguments"]) == {"city": "Paris"}
        # answer the call with function_call_output in a chained request
        r = c.post("/v1/responses", json={"previous_response_id": evs[-1]["response"]["id"],
                                          "max_output_tokens": 200, "input": [
            {"type": "function_call_output", "call_id": out[-1]["call_id"], "output": "sunny"}]})
        assert r.status_code == 200
    ae.shutdown()


def test_responses_background_replay_and_cancel():
    c, ae, _ = _client("abcdefghij" * 5, step_s=0.01)
    with c:
        r = c.post("/v1/responses", json={"input": "x", "background": True, "max_output_tokens": 30})
        assert r.status_code == 202 and r.headers["location"].endswith(r.json()["id"])
        rid = r.json()["id"]
        for _ in range(500):
            j = c.get(f"/v1/responses/{rid}").json()
            if j["status"] not in ("queued", "in_progress"):
                break
            time.sleep(0.01)
        assert j["status"] == "incomplete" and j["output_text"] == ("abcdefghij" * 3)
        with c.stream("GET", f"/v1/responses/{rid}?stream=true&starting_after=3") as s:
            evs = [json.loads(l[6:]) for l in s.iter_lines() if l.startswith("data: ")]
        assert evs[0]["sequence_number"] == 4 and evs[-1]["type"] == "response.incomplete"
        # cancel a long run
        r = c.post("/v1/responses", json={"input": "x", "background": True, "max_output_tokens": 3000})
        rid = r.json()["id"]
        time.sleep(0.05)
        assert c.post(f"/v1/responses/{rid}/cancel").json()["status"] == "cancelled"
        assert c.get(f"/v1/responses/{rid}").json()["status"] == "cancelled"
    ae.shutdown()


# --------------------------------------------------------------------------- MCP
def _rpc(c, method, params=None, rid=1):
    return c.post("/mcp", json={"jsonrpc": "2.0", "id": rid, "method": method, "params": params or {}})


def test_mcp_protocol():
    c, ae, _ = _client("ok")
    with c:
        j = _rpc(c, "initialize", {"protocolVersion": "2025-06-18"}).json()
        assert j["result"]["protocolVersion"] == "2025-06-18"
        assert _rpc(c, "initialize", {"protocolVersion": "1999-01-01"}).json()["result"]["protocolVersion"] == "2025-11-25"
        r = c.post("/mcp", json={"jsonrpc": "2.0", "method": "notifications/initialized"})
        assert r.status_code == 202 and r.content == b""
        names = [t["name"] for t in _rpc(c, "tools/list").json()["result"]["tools"]]
        assert {"chat", "models", "compare", "batch_prompts", "node_info"} <= set(names)
        res = _rpc(c, "tools/call", {"name": "chat", "arguments": {"prompt": "hi", "max_tokens": 8}}).json()
        assert res["result"]["content"][0]["text"] == "ok" and not res["result"]["isError"]
        res = _rpc(c, "tools/call", {"name": "batch_prompts", "arguments": {"tasks": [
            {"id": "a", "prompt": "1"}, {"id": "b", "prompt": "2", "model": "m:ad1"}]}}).json()
        assert [x["id"] for x in res["result"]["structuredContent"]["results"]] == ["a", "b"]
        res = _rpc(c, "tools/call", {"name": "compare", "arguments": {"prompt": "1"}}).json()
        assert len(res["result"]["structuredContent"]["results"]) == 2
        res = _rpc(c, "tools/call", {"name": "chat", "arguments": {"prompt": "1", "model": "nope"}}).json()
        assert res["result"]["isError"] is True
        assert _rpc(c, "tools/call", {"name": "nope"}).json()["error"]["code"] == -32602
        ls = _rpc(c, "resources/list").json()["result"]["resources"]
        assert {x["uri"] for x in ls} == {"swarmllm://status", "swarmllm://models", "swarmllm://peers"}
        rd = _rpc(c, "resources/read", {"uri": "swarmllm://models"}).json()["result"]["contents"][0]
        assert json.loads(rd["text"])["models"] == ["m", "m:ad1"]
        assert _rpc(c, "resources/read", {"uri": "x://y"}).json()["error"]["code"] == -32002
        assert _rpc(c, "bogus/method").json()["error"]["code"] == -32601
        bad = c.post("/mcp", content=b"{not json", headers={"content-type": "application/json"})
        assert bad.status_code == 400 and bad.json()["error"]["code"] == -32700 and bad.json()["id"] is None
        bad = c.post("/mcp", json=[{"jsonrpc": "2.0", "id": 1, "method": "ping"}])
        assert bad.json()["error"]["code"] == -32600
        assert c.get("/mcp").status_code == 405 and c.delete("/mcp").status_code == 200
    ae.shutdown()


# --------------------------------------------------------------------------- guards
def test_auth_cors_rate_limit_body_cap():
    c, ae, _ = _client("ok", api_key="sekrit", rpm=4, cors_origins=("https://app.example",))
    with c:
        assert c.get("/health").status_code == 200                      # exempt
        r = c.get("/v1/models")
        assert r.status_code == 401 and r.headers["x-content-type-options"] == "nosniff"
        assert c.get("/v1/models", headers={"Authorization": "Bearer wrong"}).status_code == 401
        assert c.get("/v1/models", headers={"authorization": "bearer sekrit"}).status_code == 200
        assert c.get("/v1/models", headers={"x-api-key": "sekrit"}).status_code == 200
        r = c.get("/v1/models", headers={"x-api-key": "sekrit"})   # 5th in the minute, failures count
        assert r.status_code == 429 and int(r.headers["retry-after"]) >= 1
        pre = c.options("/v1/chat/completions", headers={"Origin": "https://app.example",
                                                         "Access-Control-Request-Method": "POST"})
        assert pre.status_code == 204 and pre.headers["access-control-allow-origin"] == "https://app.example"
        assert c.options("/v1/models", headers={"Origin": "https://evil.example"}).status_code == 403
        big = c.post("/api/status", content=b"x", headers={"x-api-key": "sekrit",
                                                          "content-length": str(64 << 20)})
        assert big.status_code == 413
    ae.shutdown()


def test_rate_limiter_refill_and_isolation():
    from swarmllm_b200.serve.middleware import RateLimiter
    now = [0.0]
    rl = RateLimiter(60, clock=lambda: now[0])
    assert all(rl.acquire("a") == 0 for _ in range(60))
    assert rl.acquire("a") > 0 and rl.acquire("b") == 0
    now[0] += 1.0                      # one token a second at 60 rpm
    assert rl.acquire("a") == 0 and rl.acquire("a") > 0


def test_status_websocket_feed():
    c, ae, _ = _client("ok", api_key="k")
    with c:
        with c.websocket_connect("/api/admin/ws?n=2&token=k") as ws:
            a, b = ws.receive_json(), ws.receive_json()
        assert a["type"] == "status" and (a["seq"], b["seq"]) == (0, 1)
    ae.shutdown()


def test_admin_api(tmp_path):
    from fastapi.testclient import TestClient

    from swarmllm_b200.engine import EngineConfig, LLMEngine
    from swarmllm_b200.models.config import tiny_llama
    from swarmllm_b200.models.lora import LoraAdapter
    from swarmllm_b200.serve.api import AsyncEngine, create_app
    from swarmllm_b200.serve.tokenizer import ByteTokenizer
    cfg = tiny_llama()
    eng = LLMEngine.from_config(cfg, "cpu", EngineConfig(max_model_len=256, max_running=4,
                                                        max_step_tokens=256, prefill_chunk=256,
                                                        max_loras=1))
    toml = tmp_path / "c.toml"
    toml.write_text('[server]\nrpm = 77\ncors_origins = ["https://x.example"]\n')
    ae = AsyncEngine(eng)
    app = create_app(ae, ByteTokenizer(cfg.vocab), "tiny", max_model_len=256, api_key="k",
                     config_path=str(toml))
    h = {"x-api-key": "k"}
    with TestClient(app) as c:
        assert c.get("/api/admin/stats").status_code == 401
        c.post("/v1/completions", json={"prompt": [5, 6, 7], "max_tokens": 3}, headers=h)
        st = c.get("/api/admin/stats", headers=h).json()
        assert st["requests_completed"] >= 1 and st["tokens_generated"] >= 3
        assert set(c.get("/api/admin/performance", headers=h).json()["windows"]) == {"10", "60", "300"}
        cf = c.put("/api/admin/config", json={"rpm": 5}, headers=h).json()
        assert cf["server"]["rpm"] == 5 and cf["engine"]["max_running"] == 4
        assert c.put("/api/admin/config", json={"max_running": 9}, headers=h).status_code == 400
        cf = c.post("/api/admin/config/reload", headers=h).json()
        assert cf["server"]["rpm"] == 77 and cf["server"]["cors_origins"] == ["https://x.example"]
        pre = c.options("/v1/models", headers={"Origin": "https://x.example"})
        assert pre.status_code == 204       # the reloaded origin is live
        p = str(tmp_path / "ad.gguf")
        LoraAdapter.random(cfg, rank=4, seed=1).write_gguf(p)
        r = c.post("/api/admin/lora", json={"name": "ad", "path": p}, headers=h)
        assert r.status_code == 200 and "tiny:ad" in r.json()["models"]
        m = c.get("/api/admin/models", headers=h).json()
        assert m["lora_adapters"] == ["ad"] and m["layers"] == cfg.n_layers
        d = c.get("/api/admin/diagnostics", headers=h).json()
        assert d["native_extensions"]["swarmllm_b200._native"] and d["kv_cache"]["pages"] > 0
        assert c.get("/api/admin/responses", headers=h).json()["data"] == []
        ad = c.get("/api/admin/adapters", headers=h).json()
        assert ad["data"][0]["id"] == "ad" and ad["slots"] == 1
        assert c.get("/api/admin/models/tiny:ad", headers=h).json()["adapter"] == "ad"
        assert c.get("/api/admin/models/tiny/status", headers=h).json()["ready"] is True
        assert c.get("/api/admin/models/nope/status", headers=h).status_code == 404
        assert c.get("/api/admin/version", headers=h).json()["name"] == "swarmllm_b200"
        assert c.get("/api/admin/peers", headers=h).json()["peers"] == []
        assert c.get("/api/admin/schedule", headers=h).json()["max_running"] == 4
        assert c.get("/api/admin/swarm/capacity", headers=h).json()["kv_tokens"] > 0
        assert c.get("/api/admin/storage/breakdown", headers=h).status_code == 200
        assert c.post("/api/admin/shutdown", headers=h).status_code == 501    # no hook here
        # unload; the freed slot is reused by the next load
        r = c.delete("/api/admin/adapters/ad", headers=h)
        assert r.status_code == 200 and "tiny:ad" not in r.json()["models"]
        assert c.delete("/api/admin/adapters/ad", headers=h).status_code == 404
        assert c.post("/api/admin/adapters", json={"name": "ad2", "path": p}, headers=h).status_code == 200
        assert c.get("/api/admin/adapters", headers=h).json()["data"] == [
            {"id": "ad2", "slot": 0, "model": "tiny:ad2"}]
        r = c.post("/v1/completions", json={"prompt": [5, 6, 7], "max_tokens": 2, "model": "tiny:ad2"},
                   headers=h)
        assert r.status_code == 200
        called = []
        app.state.shutdown_hook = lambda: called.append(1)
        assert c.post("/api/admin/shutdown", headers=h).status_code == 200 and called
    eng.lora_of[999] = 0                       # a live request on the adapter's slot
    with pytest.raises(RuntimeError):
        eng.unload_lora("ad2")
    ae.shutdown()


def test_stalled_engine_withdraws_readiness():
    """A step that does not return for longer than stall_s takes /health/ready
    to 503; readiness comes back when the step returns."""
    import threading

    from fastapi.testclient import TestClient

    from swarmllm_b200.serve.api import AsyncEngine, create_app
    from swarmllm_b200.serve.tokenizer import ByteTokenizer
    gate = threading.Event()

    class Blocking(Scripted):
        def step(self):
            gate.wait(5.0)
            return super().step()

    eng = Blocking("ab")
    ae = AsyncEngine(eng, stall_s=0.2)
    app = create_app(ae, ByteTokenizer(512), "m", max_model_len=4096)
    with TestClient(app) as c:
        assert c.get("/health/ready").status_code == 200
        eng.add_request([5], types.SimpleNamespace(max_tokens=2), request_id=99)
        ae._wake.set()
        t0 = time.time()
        while c.get("/health/ready").status_code != 503:
            assert time.time() - t0 < 3, "stall not detected"
            time.sleep(0.05)
        assert ae.stalled() and c.get("/api/status").json()["ready"] is False
        gate.set()
        while c.get("/health/ready").status_code != 200:
            assert time.time() - t0 < 6, "readiness did not come back"
            time.sleep(0.05)
    ae.shutdown()


def test_penalties_reach_sampling_params():
    c, ae, eng = _client("hi")
    seen = []
    orig = eng.add_request

    def spy(ids, sp, request_id, lora=None):
        seen.append(sp)
        return orig(ids, sp, request_id, lora)
    eng.add_request = spy
    with c:
        r = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "x"}],
                                                 "max_tokens": 4, "frequency_penalty": 0.5,
                                                 "presence_penalty": 1.5})
        assert r.status_code == 200
    assert seen[-1].frequency_penalty == 0.5 and seen[-1].presence_penalty == 1.5
    ae.shutdown()


def test_logprobs_refused_not_ignored():
    c, ae, eng = _client("hi")
    with c:
        r = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "x"}],
                                                 "logprobs": True, "top_logprobs": 3})
        assert r.status_code == 400 and "logprobs" in r.text
        r = c.post("/v1/completions", json={"prompt": "x", "logprobs": 2, "max_tokens": 2})
        assert r.status_code == 400
        r = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "x"}],
                                                 "logprobs": False, "max_tokens": 2})
        assert r.status_code == 200
    ae.shutdown()


def test_n_choices_and_logit_bias_parameters():
    c, ae, eng = _client("hey")
    seen = []
    orig = eng.add_request

    def spy(ids, sp, request_id, lora=None):
        seen.append(sp)
        return orig(ids, sp, request_id, lora)
    eng.add_request = spy
    msgs = [{"role": "user", "content": "x"}]
    with c:
        r = c.post("/v1/chat/completions", json={"messages": msgs, "max_tokens": 8, "n": 3,
                                                 "temperature": 0.7, "seed": 10})
        j = r.json()
        assert r.status_code == 200 and [ch["index"] for ch in j["choices"]] == [0, 1, 2]
        assert all(ch["message"]["content"] == "hey" for ch in j["choices"])
        assert sorted(sp.seed for sp in seen[-3:]) == [10, 11, 12]
        assert j["usage"]["completion_tokens"] == 3 * 4
        r = c.post("/v1/completions", json={"prompt": "x", "max_tokens": 8, "n": 2})
        assert [ch["index"] for ch in r.json()["choices"]] == [0, 1]
        assert c.post("/v1/chat/completions", json={"messages": msgs, "n": 2, "stream": True}).status_code == 400
        assert c.post("/v1/chat/completions", json={"messages": msgs, "n": 0}).status_code == 400
        r = c.post("/v1/chat/completions", json={"messages": msgs, "max_tokens": 2,
                                                 "logit_bias": {"50": 5, "7": -300}})
        assert r.status_code == 200 and seen[-1].logit_bias == {50: 5.0, 7: -100.0}
        assert c.post("/v1/chat/completions", json={"messages": msgs,
                                                    "logit_bias": {"a": 1}}).status_code == 400
    ae.shutdown()


def test_model_retrieve_and_count_tokens():
    c, ae, eng = _client("x")
    with c:
        assert c.get("/v1/models/m").json()["id"] == "m"
        assert c.get("/v1/models/m:ad1").status_code == 200        # a LoRA adapter of the base
        assert c.get("/v1/models/other").status_code == 404
        r = c.post("/v1/messages/count_tokens", json={"model": "m", "system": "be brief",
                                                      "messages": [{"role": "user", "content": "hello"}]})
        n = r.json()["input_tokens"]
        r2 = c.post("/v1/messages/count_tokens", json={"model": "m",
                                                       "messages": [{"role": "user", "content": "hello"}]})
        assert r.status_code == 200 and n > r2.json()["input_tokens"] > 5
        assert c.post("/v1/messages/count_tokens", json={"messages": []}).status_code == 400
    ae.shutdown()


def test_completions_echo():
    c, ae, eng = _client("ok")
    with c:
        r = c.post("/v1/completions", json={"prompt": "say:", "max_tokens": 5, "echo": True})
        assert r.json()["choices"][0]["text"] == "say:ok"
        r = c.post("/v1/completions", json={"prompt": "say:", "max_tokens": 5})
        assert r.json()["choices"][0]["text"] == "ok"
    ae.shutdown()


def test_completions_stream_echo_and_prompt_batch():
    c, ae, eng = _client("ok")
    with c:
        r = c.post("/v1/completions", json={"prompt": "say:", "max_tokens": 5, "echo": True,
                                            "stream": True})
        chunks = [json.loads(l[6:]) for l in r.text.splitlines()
                  if l.startswith("data: ") and l != "data: [DONE]"]
        text = "".join(ch["choices"][0]["text"] for ch in chunks)
        assert chunks[0]["choices"][0]["text"] == "say:" and text == "say:ok"
        # a batch of prompts: one choice per prompt (x n), indexed prompt-major
        r = c.post("/v1/completions", json={"prompt": ["a:", "b:"], "max_tokens": 5,
                                            "echo": True, "n": 2})
        j = r.json()
        assert r.status_code == 200
        assert [ch["index"] for ch in j["choices"]] == [0, 1, 2, 3]
        assert [ch["text"] for ch in j["choices"]] == ["a:ok", "a:ok", "b:ok", "b:ok"]
        assert c.post("/v1/completions", json={"prompt": ["a", "b"], "stream": True}).status_code == 400
        assert c.post("/v1/completions", json={"prompt": 5}).status_code == 400
    ae.shutdown()


def test_unseeded_requests_draw_fresh_seeds():
    """Without a client seed every sampled request gets its own random seed,
    so two unseeded requests are not forced to sample identical tokens."""
    c, ae, eng = _client("hey")
    seen = []
    orig = eng.add_request

    def spy(ids, sp, *a, **kw):
        seen.append(sp)
        return orig(ids, sp, *a, **kw)
    eng.add_request = spy
    msgs = [{"role": "user", "content": "x"}]
    with c:
        for _ in range(2):
            assert c.post("/v1/chat/completions", json={"messages": msgs, "max_tokens": 2,
                                                        "temperature": 0.9}).status_code == 200
        assert seen[-1].seed != seen[-2].seed
        c.post("/v1/chat/completions", json={"messages": msgs, "max_tokens": 2, "seed": 7})
        assert seen[-1].seed == 7
        assert c.post("/v1/chat/completions", json={"messages": msgs, "seed": "x"}).status_code == 400
    ae.shutdown()


def test_api_key_rotation_and_ws_tickets(tmp_path):
    """Rotation takes effect with the next request and is written to the key
    file; a websocket ticket works once and the key never goes in the URL."""
    kf = tmp_path / "key"
    kf.write_text("k0\n")
    c, ae, _ = _client("ok", api_key_file=str(kf))
    H0 = {"Authorization": "Bearer k0"}
    with c:
        assert c.get("/api/admin/api-key").status_code == 401
        assert c.get("/api/admin/api-key", headers=H0).json()["api_key"] == "k0"
        new = c.post("/api/admin/api-key/rotate", headers=H0).json()["api_key"]
        assert len(new) == 64 and new != "k0"
        assert kf.read_text().strip() == new
        assert c.get("/v1/models", headers=H0).status_code == 401          # old key: out
        H1 = {"Authorization": f"Bearer {new}"}
        assert c.get("/v1/models", headers=H1).status_code == 200
        t = c.post("/api/admin/ws-ticket", headers=H1).json()["ticket"]
        with c.websocket_connect(f"/api/admin/ws?n=1&t={t}") as ws:
            assert ws.receive_json()["type"] == "status"
        import pytest as _pt
        from starlette.websockets import WebSocketDisconnect
        with _pt.raises(WebSocketDisconnect):                              # a ticket is single-use
            with c.websocket_connect(f"/api/admin/ws?n=1&t={t}") as ws:
                ws.receive_json()
    ae.shutdown()


def test_prune_history(tmp_path):
    import time as _t
    c, ae, _ = _client("ok")
    with c:
        store = c.app.state.response_store
        for i in range(5):
            store.put({"id": f"resp_{i}"}, [], [])
        with store.lock:   # age two of them by three days
            store.db.execute("UPDATE responses SET created = ? WHERE id IN ('resp_0', 'resp_1')",
                             (_t.time() - 3 * 86400,))
            store.db.commit()
        r = c.post("/api/admin/prune-history", json={"older_than_days": 2}).json()
        assert r == {"removed": 2, "left": 3}
        r = c.post("/api/admin/prune-history", json={"keep": 1}).json()
        assert r == {"removed": 2, "left": 1}
        assert c.post("/api/admin/prune-history", json={}).status_code == 400
        assert c.post("/api/admin/prune-history", json={"keep": -1}).status_code == 400
    ae.shutdown()
