"""Speculative serving through the engine API (SpecEngine): greedy and sampled
requests give what the plain engine gives (sampled: Philox-coupled noise, the
same seed and positions), several tokens commit per step with a drafter that
agrees with the target, end-of-sequence stops a request, and the HTTP layer
serves it."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _cfg(layers=2, hidden=512):
    from swarmllm_b200.models.config import ModelConfig
    return ModelConfig(name="t", arch="llama", n_layers=layers, hidden=hidden, n_heads=8,
                       n_kv_heads=2, head_dim=64, ffn=1024, vocab=1024, weight_qtype="Q4_K",
                       embed_qtype="F16", output_qtype="Q4_K")


def _ecfg(**kw):
    from swarmllm_b200.engine import EngineConfig
    return EngineConfig(max_model_len=256, max_running=4, max_step_tokens=128, prefill_chunk=64,
                        cuda_graphs=False, **kw)


def _plain(cfg, prompts, params):
    """The plain engine's tokens.  One or two decoding sequences run on the
    CUDA-core GEMV with int8 activations, while speculative verify steps (many
    rows) run the fp16 tensor-core GEMM; random-init models have near-tied
    logits everywhere, so the reference decodes at least three sequences (the
    extra ones are discarded) to stay on the same GEMM path."""
    from swarmllm_b200.engine import LLMEngine
    from swarmllm_b200.models.weights import RandomSource
    eng = LLMEngine.from_config(cfg, DEV, _ecfg(), source=RandomSource(cfg, seed=7))
    pad = [list(range(1, 9))] * max(0, 3 - len(prompts))
    return [o.token_ids for o in eng.generate(prompts + pad, params)][:len(prompts)]


def _spec(cfg, prompts, params, draft):
    from swarmllm_b200.engine.spec_engine import create_engine
    from swarmllm_b200.models.weights import RandomSource
    eng = create_engine(cfg, DEV, _ecfg(draft_model=draft, spec_depth=4, spec_width=3),
                        source=RandomSource(cfg, seed=7))
    outs = [o.token_ids for o in eng.generate(prompts, params)]
    return outs, eng


def _agree(a, b):
    return np.mean([x == y for o, r in zip(a, b) for x, y in zip(o, r)])


@pytest.mark.parametrize("temperature", [0.0, 0.8])
def test_spec_engine_self_draft_matches_plain_engine(temperature):
    from swarmllm_b200.engine import SamplingParams
    cfg = _cfg()
    rng = np.random.default_rng(2)
    prompts = [rng.integers(0, cfg.vocab, n).tolist() for n in (12, 40, 7)]
    sp = SamplingParams(max_tokens=20, temperature=temperature, top_k=40, seed=1234)
    want = _plain(cfg, prompts, sp)
    got, eng = _spec(cfg, prompts, sp, "self")
    assert all(len(o) == 20 for o in got)
    assert _agree(got, want) >= 0.95, (got, want)
    st = eng.dec.stats
    assert st.tokens_per_round >= 3.0, st       # the target drafting for itself is accepted


def test_spec_engine_ngram_and_eos():
    from swarmllm_b200.engine import SamplingParams
    cfg = _cfg()
    rng = np.random.default_rng(3)
    base = rng.integers(0, cfg.vocab, 10).tolist()
    prompts = [base * 4, rng.integers(0, cfg.vocab, 25).tolist()]
    sp = SamplingParams(max_tokens=16)
    want = _plain(cfg, prompts, sp)
    got, _ = _spec(cfg, prompts, sp, "ngram")
    assert _agree(got, want) >= 0.95, (got, want)
    # end of sequence: stop right after the first occurrence of a token the run produces
    eos = want[1][5]
    got, _ = _spec(cfg, prompts[1:], SamplingParams(max_tokens=16, eos_token_id=eos), "self")
    assert got[0][-1] == eos and len(got[0]) <= 6, got


def test_spec_engine_serves_http():
    from fastapi.testclient import TestClient
    from swarmllm_b200.engine.spec_engine import create_engine
    from swarmllm_b200.models.weights import RandomSource
    from swarmllm_b200.serve.api import AsyncEngine, create_app
    from swarmllm_b200.serve.tokenizer import ByteTokenizer
    cfg = _cfg()
    eng = create_engine(cfg, DEV, _ecfg(draft_model="self"), source=RandomSource(cfg, seed=7))
    ae = AsyncEngine(eng)
    app = create_app(ae, ByteTokenizer(cfg.vocab), "spec", max_model_len=256)
    with TestClient(app) as c:
        r = c.post("/v1/completions", json={"prompt": "hello", "max_tokens": 12, "ignore_eos": True})
        assert r.status_code == 200, r.text
        assert r.json()["usage"]["completion_tokens"] == 12
    ae.shutdown()


def test_spec_engine_swift_layer_skip():
    """The target drafting with a middle block of its layers skipped: output
    is the target's own."""
    from swarmllm_b200.engine import SamplingParams
    cfg = _cfg(layers=6)
    rng = np.random.default_rng(5)
    prompts = [rng.integers(0, cfg.vocab, n).tolist() for n in (15, 33)]
    sp = SamplingParams(max_tokens=16)
    want = _plain(cfg, prompts, sp)
    got, eng = _spec(cfg, prompts, sp, "swift:0.34")
    assert eng.dec.d.model.skipped == 2 and len(eng.dec.d.model.layers) == 4
    assert _agree(got, want) >= 0.95, (got, want)
