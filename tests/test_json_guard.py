"""JSON-constrained decoding: the incremental recogniser and the engine hook."""
import json

import pytest

from swarmllm_b200.serve.json_guard import JsonConstraint, JsonPrefix

VALID = ['{}', '{"a": 1}', '{"a": [1, 2.5, -3e-2, true, false, null, "x\\"y\\u00e9"], "b": {}}',
         '{"k": {"n": [[], [{}]], "z": 0}}', ' { "a" : "b" } ']
INVALID = ['[1]', '"s"', '{a: 1}', '{"a" 1}', '{"a": 01}', '{"a": 1,}', '{"a": tru}', '{"a": 1]',
           '{"a": "\\x"}', '{"a": .5}', '{}{}', '{"a": 1e}']


@pytest.mark.parametrize("text", VALID)
def test_valid_documents_accepted_and_done(text):
    p = JsonPrefix()
    assert p.feed(text) and p.done
    json.loads(text)


@pytest.mark.parametrize("text", INVALID)
def test_invalid_documents_refused(text):
    p = JsonPrefix()
    ok = p.feed(text)
    assert not (ok and p.done)


def test_prefixes_of_valid_documents_are_accepted():
    for text in VALID:
        for n in range(len(text)):
            p = JsonPrefix()
            assert p.feed(text[:n]), text[:n]
            assert not p.done or text[:n].strip() == text.strip()


def test_constraint_chooses_and_forces_eos():
    pieces = {3: '{', 4: '"a"', 5: ':', 6: '1', 7: '}', 8: 'x', 2: ''}
    c = JsonConstraint(lambda t: pieces.get(t, ""), eos_id=2)
    seq = []
    for drawn, cands in ((8, [8, 3]), (4, [4]), (8, [8, 5]), (6, [6]), (2, [2, 7]), (8, [8])):
        t = c.choose(drawn, cands)
        c.accept(t)
        seq.append(t)
    assert seq == [3, 4, 5, 6, 7, 2]                     # EOS refused before '}', forced after


def test_engine_output_is_json_prefix():
    import numpy as np

    from swarmllm_b200.engine import EngineConfig, LLMEngine, SamplingParams
    from swarmllm_b200.models.config import tiny_llama
    from swarmllm_b200.models.weights import RandomSource
    from swarmllm_b200.serve.tokenizer import ByteTokenizer
    cfg = tiny_llama()
    tok = ByteTokenizer(cfg.vocab)
    eng = LLMEngine.from_config(cfg, "cpu", EngineConfig(max_model_len=256, max_running=2,
                                                         max_step_tokens=256, prefill_chunk=256),
                                source=RandomSource(cfg, seed=2))
    prompt = tok.encode("give json")
    for temp in (0.0, 0.9):
        sp = SamplingParams(max_tokens=40, temperature=temp, seed=5, eos_token_id=tok.eos_id,
                            constraint=JsonConstraint(tok.token_str, tok.eos_id))
        out = eng.generate([prompt], sp)[0].token_ids
        text = tok.decode([t for t in out if t != tok.eos_id])
        assert text.lstrip().startswith("{") and JsonPrefix().feed(text), text
        if out and out[-1] == tok.eos_id:
            json.loads(text)


def test_api_attaches_json_constraint():
    from test_api_ext import _client
    c, ae, eng = _client("hi")
    seen = []
    orig = eng.add_request

    def spy(ids, sp, request_id, lora=None):
        seen.append(sp)
        return orig(ids, sp, request_id, lora)
    eng.add_request = spy
    with c:
        for rf in ({"type": "json_object"}, None):
            body = {"messages": [{"role": "user", "content": "x"}], "max_tokens": 3}
            if rf:
                body["response_format"] = rf
            assert c.post("/v1/chat/completions", json=body).status_code == 200
    assert isinstance(seen[0].constraint, JsonConstraint) and seen[1].constraint is None
    ae.shutdown()


def test_responses_text_format_attaches_constraint():
    from test_api_ext import _client
    c, ae, eng = _client("hi")
    seen = []
    orig = eng.add_request

    def spy(ids, sp, request_id, lora=None):
        seen.append(sp)
        return orig(ids, sp, request_id, lora)
    eng.add_request = spy
    with c:
        r = c.post("/v1/responses", json={"input": "x", "max_output_tokens": 3,
                                          "text": {"format": {"type": "json_schema", "name": "s",
                                                              "schema": {"type": "object"}}}})
        assert r.status_code == 200, r.text
    assert isinstance(seen[-1].constraint, JsonConstraint)
    ae.shutdown()


def test_constrained_tree_walk_equals_plain_constrained_decoding():
    """Speculative verify of a JSON reply: walking a draft tree with the
    constraint applied at each node commits exactly what step-by-step
    constrained decoding commits, while accepting drafted nodes."""
    import numpy as np
    import torch

    from swarmllm_b200.engine.sampling import SamplingParams, constrained_token
    from swarmllm_b200.engine.spec import walk_constrained
    from swarmllm_b200.utils.ext import native
    pieces = ['{', '}', '"a"', '"b"', ':', ', ', '1', '2', ' ', 'x', '[', ']', 'true', '"', 'ab']
    EOS = len(pieces)
    V = EOS + 1

    def piece(t):
        return pieces[t] if t < len(pieces) else ""

    def logits(prefix):  # a deterministic stand-in for the target model
        g = torch.Generator().manual_seed(hash(tuple(prefix)) % (2 ** 31))
        return torch.randn(V, generator=g)

    def choice(prefix):  # what plain constrained decoding commits after prefix
        c = JsonConstraint(piece, EOS)
        for t in prefix:
            c.accept(t)
        row = logits(prefix)
        return constrained_token(c, int(row.argmax()), row, EOS)

    plain = []
    while len(plain) < 40 and (not plain or plain[-1] != EOS):
        plain.append(choice(plain))

    rng = np.random.default_rng(0)
    c = JsonConstraint(piece, EOS)
    row = logits([])
    out = [constrained_token(c, int(row.argmax()), row, EOS)]
    p = SamplingParams(eos_token_id=EOS, constraint=c)
    accepted = 0
    while len(out) < 40 and out[-1] != EOS:
        tr = native().DraftTree(out[-1], 64)

        def prefix_of(node):
            par, tok, path = tr.parents(), tr.tokens(), []
            while node != 0:
                path.append(tok[node])
                node = par[node]
            return out + path[::-1]
        for _ in range(3):
            cand_t, cand_lp = [], []
            for node in tr.frontier():
                good = choice(prefix_of(node))
                other = int(rng.integers(0, V))
                first = good if rng.random() < 0.7 else other
                cand_t += [first, other if other != first else (first + 1) % V]
                cand_lp += [-0.1, -2.0]
            tr.expand(cand_t, cand_lp, 2, 2)
        n = len(tr)
        rows = [logits(prefix_of(i)) for i in range(n)]
        tgt = [int(r.argmax()) for r in rows]
        path, bonus = walk_constrained(tr, tgt, rows, p)
        accepted += len(path) - 1
        toks = tr.tokens()
        out += [toks[i] for i in path[1:]] + [bonus]
    if EOS in out:
        out = out[:out.index(EOS) + 1]
    assert out[:len(plain)] == plain[:len(out)]
    assert len(out) >= min(len(plain), 40) and accepted > 0
