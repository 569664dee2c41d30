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


def test_regex_subset_matches_python_re():
    """The pattern NFA agrees with Python's re (fullmatch semantics via \\Z)
    on random strings, for anchored and unanchored patterns."""
    import random
    import re
    from swarmllm_b200.serve.regex_guard import FORMAT_PATTERNS, compile_pattern
    cases = [r"^\d{3}-\d{4}$", r"^[A-Z][a-z]+( [A-Z][a-z]+)*$", r"ab|cd", r"^(?:foo|bar)+baz?$",
             r"^[^@\s]+@[^@\s]+\.[a-z]{2,6}$", r"^x{2,4}y{0,}z?$", r"^[-+]?\d*\.?\d+$",
             r"colou?r", r"^\w+\s\w+$", r"^a.c$", r"^[\]a-]+$", r"^a{3}$"] + \
        list(FORMAT_PATTERNS.values())
    rng = random.Random(0)
    alphabet = "abcdxyzABZ0123456789-+.@ _:TZ]\n"
    for c in cases:
        p = compile_pattern(c)
        assert p is not None, c
        rx = re.compile(c[:-1] + r"\Z" if c.endswith("$") else c)
        for _ in range(1500):
            s = "".join(rng.choice(alphabet) for _ in range(rng.randint(0, 12)))
            assert p.fullmatch(s) == (rx.search(s) is not None), (c, s)
    for c in (r"(?=a)b", r"(a)\1", r"a^b", r"(ab", r"\bfoo"):
        assert compile_pattern(c) is None, c       # outside the subset: not enforced


def test_string_pattern_format_and_length():
    sch = {"type": "object", "properties": {
        "zip": {"type": "string", "pattern": "^[0-9]{5}$"},
        "day": {"type": "string", "format": "date"},
        "nick": {"type": "string", "minLength": 2, "maxLength": 3}},
        "required": ["zip"]}
    assert _ok(sch, '{"zip":"12345"}', done=True)
    assert not _ok(sch, '{"zip":"1234a')
    assert not _ok(sch, '{"zip":"1234"')              # closing quote before 5 digits
    assert not _ok(sch, '{"zip":"123456')
    assert _ok(sch, '{"zip":"00000","day":"2024-02-29"}', done=True)
    assert not _ok(sch, '{"zip":"00000","day":"2024-13')
    assert _ok(sch, '{"zip":"00000","nick":"ab"}', done=True)
    assert not _ok(sch, '{"zip":"00000","nick":"a"')
    assert not _ok(sch, '{"zip":"00000","nick":"abcd')
    # escapes count as the character they stand for
    assert _ok({"type": "string", "pattern": "^a\\nb$"}, '"a\\nb"', done=True)
    assert _ok({"type": "string", "pattern": "^\\u00e9$"}, '"\\u00e9"', done=True)
    assert not _ok({"type": "string", "maxLength": 1}, '"a\\')


def test_constrained_random_walk_respects_pattern():
    """Drawing characters at random among those the recogniser allows always
    ends in a string the pattern fully matches."""
    import random
    import re
    sch = {"type": "string", "pattern": "^(ab|c)+-[0-9]{2,3}$"}
    rng = random.Random(3)
    alphabet = list('abc-0123456789"x')
    for _ in range(30):
        s, text = SchemaPrefix(sch), ""
        while not s.done:
            allowed = [c for c in alphabet if s.copy().feed(c)]
            assert allowed, text
            c = rng.choice(allowed)
            assert s.feed(c)
            text += c
            assert len(text) < 200
        assert re.fullmatch("(ab|c)+-[0-9]{2,3}", json.loads(text))


def test_numeric_ranges():
    age = {"type": "integer", "minimum": 18, "maximum": 65}
    assert _ok(age, "18", None) and _ok(age, "65", None) and _ok(age, "40", None)
    assert not _ok(age, "7")                 # no completion of 7 is in [18, 65]... 70+ too big
    assert _ok(age, "1", None)                # 18, 19 still reachable
    assert not _ok(age, "-")
    assert not _ok(age, "66")
    arr = {"type": "array", "items": age}
    assert not _ok(arr, "[1]")               # "1" cannot end below the minimum
    assert _ok(arr, "[19,65]", True)
    p = {"type": "number", "exclusiveMinimum": 0, "maximum": 1}
    assert _ok(p, "0.5", None) and _ok(p, "1", None) and not _ok(p, "1.5")
    assert not _ok({"type": "array", "items": p}, "[0]")     # 0 itself is excluded
    assert _ok({"type": "array", "items": p}, "[0.25]", True)
    assert not _ok(p, "2")
    assert not _ok(p, "1e")                   # bounded numbers carry no exponent
    neg = {"type": "number", "minimum": -10, "maximum": -2}
    assert _ok(neg, "-3.5", None) and _ok(neg, "-10", None)
    assert _ok(neg, "-1", None)               # -10 is still reachable
    assert not _ok({"type": "array", "items": neg}, "[-1]")
    assert not _ok(neg, "-11") and not _ok(neg, "3")


def test_numeric_range_random_walk():
    """Characters drawn at random among the allowed ones always finish on an
    in-range number."""
    import random
    sch = {"type": "object", "properties": {"x": {"type": "number", "minimum": -2.5,
                                                  "exclusiveMaximum": 40}},
           "required": ["x"], "additionalProperties": False}
    rng = random.Random(5)
    alphabet = list('{}"x:-.0123456789e, ')
    for _ in range(40):
        s, text = SchemaPrefix(sch), ""
        while not s.done:
            allowed = [c for c in alphabet if s.copy().feed(c)]
            assert allowed, text
            c = rng.choice(allowed)
            assert s.feed(c)
            text += c
            assert len(text) < 300
        v = json.loads(text)["x"]
        assert -2.5 <= v < 40, text
