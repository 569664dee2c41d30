"""Tree speculative decoding: output equals the target's greedy decoding; a
drafter identical to the target gets (almost) every drafted token accepted."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _cfg(layers=2, hidden=512):
    from swarmllm_b200.models.config import ModelConfig
    return ModelConfig(name="t", arch="llama", n_layers=layers, hidden=hidden, n_heads=8,
                       n_kv_heads=2, head_dim=64, ffn=1024, vocab=1024, weight_qtype="Q8_0",
                       embed_qtype="F16", output_qtype="Q8_0")


def _greedy_reference(cfg, seed, prompts, n):
    from swarmllm_b200.engine import EngineConfig, LLMEngine, SamplingParams
    from swarmllm_b200.models.weights import RandomSource
    eng = LLMEngine.from_config(cfg, DEV, EngineConfig(max_model_len=256, max_running=4,
                                                       max_step_tokens=128, prefill_chunk=128,
                                                       cuda_graphs=False),
                                source=RandomSource(cfg, seed=seed))
    return [o.token_ids for o in eng.generate(prompts, SamplingParams(max_tokens=n))]


@pytest.mark.parametrize("depth,width", [(4, 4), (3, 2)])
def test_tree_spec_matches_target_greedy(depth, width):
    from swarmllm_b200.engine.spec import TreeSpecDecoder
    from swarmllm_b200.models.llama import LlamaGPU
    from swarmllm_b200.models.weights import RandomSource
    cfg, dcfg = _cfg(), _cfg(layers=1, hidden=256)
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, cfg.vocab, n).tolist() for n in (9, 33, 20)]
    spec = TreeSpecDecoder(LlamaGPU(cfg, RandomSource(cfg, seed=7), DEV),
                           LlamaGPU(dcfg, RandomSource(dcfg, seed=9), DEV), depth=depth,
                           width=width, max_seqs=4, max_model_len=200, prefill_chunk=64)
    out = spec.generate(prompts, 14)
    ref = _greedy_reference(cfg, 7, prompts, 14)
    agree = np.mean([a == b for o, r in zip(out, ref) for a, b in zip(o, r)])
    assert agree >= 0.95, (agree, out, ref)
    assert all(len(o) == 14 for o in out)


def test_tree_spec_self_draft_accepts():
    from swarmllm_b200.engine.spec import TreeSpecDecoder
    from swarmllm_b200.models.llama import LlamaGPU
    from swarmllm_b200.models.weights import RandomSource
    cfg = _cfg()
    rng = np.random.default_rng(1)
    prompts = [rng.integers(0, cfg.vocab, 17).tolist(), rng.integers(0, cfg.vocab, 40).tolist()]
    spec = TreeSpecDecoder(LlamaGPU(cfg, RandomSource(cfg, seed=7), DEV),
                           LlamaGPU(cfg, RandomSource(cfg, seed=7), DEV), depth=4, width=3,
                           max_seqs=2, max_model_len=200, prefill_chunk=64)
    out = spec.generate(prompts, 21)
    st = spec.stats
    assert st.tokens_per_round >= 4.0, (st, out)
    ref = _greedy_reference(cfg, 7, prompts, 21)
    agree = np.mean([a == b for o, r in zip(out, ref) for a, b in zip(o, r)])
    assert agree >= 0.95, (agree, out, ref)
