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


@pytest.mark.parametrize("rows,V,k", [(1, 128256, 4), (4, 151936, 16), (300, 5000, 8), (7, 1000, 2)])
def test_tree_rank_matches_torch(rows, V, k):
    from swarmllm_b200.utils.ext import C
    torch.manual_seed(rows + k)
    logits = torch.randn(rows, V) * 4
    logits[0, 17] = logits[0, 23] = 50.0  # tie: lower id first
    ids = torch.zeros(rows * k, dtype=torch.int32, device=DEV)
    lp = torch.zeros(rows * k, dtype=torch.float32, device=DEV)
    ws = torch.zeros(int(C().tree_rank_ws_floats(rows, V, k)), dtype=torch.float32, device=DEV)
    for _ in range(2):
        C().tree_rank(logits.to(DEV), k, ids, lp, ws)
        torch.cuda.synchronize()
        ref_lp, ref_ix = torch.topk(torch.log_softmax(logits.double(), -1), k, dim=-1)
        got = ids.view(rows, k).cpu().long()
        assert torch.equal(got[1:], ref_ix[1:]) and torch.equal(got[0, 2:], ref_ix[0, 2:])
        assert ids.view(rows, k)[0, 0].item() == 17 and ids.view(rows, k)[0, 1].item() == 23
        assert torch.allclose(lp.view(rows, k).cpu().double(), ref_lp, atol=1e-4)


def test_ngram_spec_matches_target_greedy_and_accepts_repeats():
    from swarmllm_b200.engine.ngram_spec import NgramSpecDecoder
    from swarmllm_b200.models.llama import LlamaGPU
    from swarmllm_b200.models.weights import RandomSource
    cfg = _cfg()
    rng = np.random.default_rng(2)
    unit = rng.integers(0, cfg.vocab, 12).tolist()
    prompts = [unit * 4, rng.integers(0, cfg.vocab, 30).tolist()]
    spec = NgramSpecDecoder(LlamaGPU(cfg, RandomSource(cfg, seed=7), DEV), depth=5,
                            max_seqs=2, max_model_len=200, prefill_chunk=64)
    out = spec.generate(prompts, 24)
    ref = _greedy_reference(cfg, 7, prompts, 24)
    agree = np.mean([a == b for o, r in zip(out, ref) for a, b in zip(o, r)])
    assert agree >= 0.95, (agree, out, ref)
    assert all(len(o) == 24 for o in out)
    # a draft that would have been right anywhere must have been accepted somewhere
    from swarmllm_b200.engine.ngram_spec import ngram_draft
    right = any(ngram_draft(p + r[:i], 3, 1) == [r[i]]
                for p, r in zip(prompts, ref) for i in range(1, 24))
    assert spec.stats.accepted > 0 or not right, (spec.stats, out)
