"""Frequency / presence penalties (OpenAI semantics: completion tokens only,
subtracted from the raw logits before temperature)."""
import collections

import numpy as np
import torch


def _engine():
    from swarmllm_b200.engine import EngineConfig, LLMEngine
    from swarmllm_b200.models.config import tiny_llama
    from swarmllm_b200.models.weights import RandomSource
    cfg = tiny_llama()
    ec = EngineConfig(max_model_len=256, max_running=4, max_step_tokens=256, prefill_chunk=256)
    return LLMEngine.from_config(cfg, "cpu", ec, source=RandomSource(cfg, seed=5))


def test_penalty_table_and_host_sampler():
    from swarmllm_b200.engine.sampling import SamplingParams, penalty_table, sample_host
    p0 = SamplingParams()
    p1 = SamplingParams(frequency_penalty=0.5, presence_penalty=1.0)
    assert penalty_table([p0, p1], None) is None
    off, tok, val = penalty_table([p0, p1], [None, collections.Counter({3: 2, 7: 1})])
    assert off.tolist() == [0, 0, 2]
    assert dict(zip(tok.tolist(), val.tolist())) == {3: 2.0, 7: 1.5}
    logits = torch.zeros(2, 10)
    logits[:, 3] = 1.9                     # penalized below token 0 in row 1 only
    out = sample_host(logits, [p0, p1], [0, 0], [None, collections.Counter({3: 2})])
    assert out.tolist() == [3, 0]


def test_presence_penalty_stops_repeats_greedy():
    from swarmllm_b200.engine import SamplingParams
    eng = _engine()
    prompt = list(range(3, 40))
    plain = eng.generate([prompt], SamplingParams(max_tokens=40))[0].token_ids
    pen = eng.generate([prompt], SamplingParams(max_tokens=40, presence_penalty=1e4))[0].token_ids
    assert len(set(pen)) == len(pen)                       # never the same token twice
    assert len(set(plain)) < len(plain)                    # the random model does repeat
    assert pen[0] == plain[0]                              # nothing generated yet: same first token


def test_logit_bias_table_and_engine():
    from swarmllm_b200.engine.sampling import SamplingParams, penalty_table
    p = SamplingParams(logit_bias={5: 2.0, 9: -1.0})
    assert p.penalized
    off, tok, val = penalty_table([SamplingParams(), p], None)   # no history needed
    assert off.tolist() == [0, 0, 2] and dict(zip(tok.tolist(), val.tolist())) == {5: -2.0, 9: 1.0}
    q = SamplingParams(frequency_penalty=1.0, logit_bias={3: 0.5})
    off, tok, val = penalty_table([q], [collections.Counter({3: 2, 4: 1})])
    assert dict(zip(tok.tolist(), val.tolist())) == {3: 1.5, 4: 1.0}   # 2 * 1.0 - 0.5, 1 * 1.0
    from swarmllm_b200.engine import SamplingParams as SP
    eng = _engine()
    out = eng.generate([list(range(3, 20))], SP(max_tokens=6, logit_bias={42: 100.0}))[0].token_ids
    assert out == [42] * 6
