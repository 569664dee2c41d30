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
