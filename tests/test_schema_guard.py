"""JSON-Schema-constrained decoding (serve/schema_guard.py): what the
recogniser accepts and refuses, and schema-valid output from a constrained
random model through the HTTP API."""
import json

import pytest

from swarmllm_b200.serve.schema_guard import SchemaPrefix

PERSON = {"type": "object",
          "properties": {"name": {"type": "string"}, "age": {"type": "integer"},
                         "tags": {"type": "array", "items": {"enum": ["a", "b"]},
                                  "maxItems": 2},
                         "kind": {"anyOf": [{"type": "null"}, {"const": "x"}]}},
          "required": ["name", "age"], "additionalProperties": False}


def _ok(schema, text, done=None):
    s = SchemaPrefix(schema)
    good = s.feed(text)
    if done is not None and good:
        return s.done == done
    return good


@pytest.mark.parametrize("text", ['{"name":"x","age":3}', '{ "age" : 41 , "name" : "bo" }',
                                  '{\n "name": "x",\n "age": 3\n}',
                                  '{"name":"","age":0,"tags":["a","b"]}',
                                  '{"name":"q","age":-2,"kind":null}',
                                  '{"name":"q","age":5,"kind":"x"}'])
def test_accepts_valid(text):
    assert _ok(PERSON, text, done=True)
    json.loads(text)


@pytest.mark.parametrize("text", ['{"nam":', '{"name":1', '{"name":"x","age":3.5',
                                  '{"name":"x","age":3,"age"', '{"name":"x"}',
                                  '{"name":"x","age":3,"tags":["c"',
                                  '{"name":"x","age":3,"tags":["a","b","a"',
                                  '{"name":"x","age":3,"kind":"y"', '["a"]', '{"name":"x","zz"'])
def test_refuses_invalid(text):
    assert not _ok(PERSON, text)


def test_blank_runs_limited():
    assert not _ok(PERSON, " {")                   # nothing before the value
    assert not _ok(PERSON, '{  "name"')            # one blank between tokens
    assert _ok(PERSON, '{"name":"a  b"', None)      # strings keep theirs


def test_prefixes_and_dead_ends():
    # a valid prefix is taken and not yet done
    assert _ok(PERSON, '{"name":"x","ag', done=False)
    # every key used: no ',' (it could only lead to a dead end)
    full = '{"name":"x","age":1,"tags":[],"kind":null'
    assert _ok(PERSON, full) and not _ok(PERSON, full + ",")
    assert _ok({"type": "array", "minItems": 2, "items": {"type": "number"}}, "[1,2.5]", True)
    assert not _ok({"type": "array", "minItems": 2, "items": {"type": "number"}}, "[1]")
    # enum of numbers and nested alternatives
    assert _ok({"enum": [1, 12, "z"]}, "12", None)
    assert not _ok({"enum": [1, 12, "z"]}, "13")
    assert _ok({"oneOf": [{"type": "integer"}, {"type": "string"}]}, '"s"', True)


def test_constrained_api_output_matches_schema():
    from fastapi.testclient import TestClient

    from swarmllm_b200.engine import EngineConfig, LLMEngine
    from swarmllm_b200.models.config import tiny_llama
    from swarmllm_b200.serve.api import AsyncEngine, create_app
    from swarmllm_b200.serve.tokenizer import ByteTokenizer
    cfg = tiny_llama()
    eng = LLMEngine.from_config(cfg, "cpu", EngineConfig(max_model_len=1024, max_running=4,
                                                        max_step_tokens=1024, prefill_chunk=512))
    ae = AsyncEngine(eng)
    app = create_app(ae, ByteTokenizer(cfg.vocab), "tiny-llama", max_model_len=1024)
    schema = {"type": "object", "properties": {"ok": {"type": "boolean"},
                                               "n": {"enum": [1, 2, 3]}},
              "required": ["ok", "n"], "additionalProperties": False}
    try:
        with TestClient(app) as c:
            for seed in (1, 2, 3):
                r = c.post("/v1/chat/completions", json={
                    "messages": [{"role": "user", "content": "give json"}], "max_tokens": 120,
                    "temperature": 1.0, "seed": seed,
                    "response_format": {"type": "json_schema",
                                        "json_schema": {"name": "t", "schema": schema}}})
                assert r.status_code == 200, r.text
                text = r.json()["choices"][0]["message"]["content"]
                s = SchemaPrefix(schema)
                assert s.feed(text), text               # always a schema-valid prefix
                if r.json()["choices"][0]["finish_reason"] == "stop":
                    v = json.loads(text)
                    assert set(v) == {"ok", "n"} and isinstance(v["ok"], bool) and v["n"] in (1, 2, 3)
    finally:
        ae.shutdown()
