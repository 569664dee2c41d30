"""Next-token-prediction (MTP) block: loaded from the file's block after the
trunk, and a speculative greedy loop that drafts with it and verifies with the
trunk -- the output equals plain greedy decoding, for a dense trunk and for a
hybrid one whose recurrent state must not advance over rejected drafts."""
import dataclasses

import numpy as np
import pytest
import torch


def _dense():
    from swarmllm_b200.models.config import ModelConfig
    return ModelConfig(name="t-mtp", arch="qwen3", n_layers=2, hidden=256, n_heads=4, n_kv_heads=2,
                       head_dim=64, ffn=512, vocab=512, rope_neox=True, qk_norm=True,
                       weight_qtype="Q8_0", embed_qtype="F16", output_qtype="Q8_0", mtp_layers=1)


def _hybrid():
    from test_hybrid_cpu import tiny_hybrid
    return dataclasses.replace(tiny_hybrid(), arch="qwen35", n_experts=0, n_experts_used=0,
                               expert_ffn=0, shared_expert_ffn=0, mtp_layers=1)


def _greedy(model, prompt, n):
    from swarmllm_b200.models.llama import StepBatch
    from swarmllm_b200.ops.attention import PagedKVCache
    cfg = model.cfg
    kv = PagedKVCache(model.n_kv_layers, 16, cfg.n_kv_heads, cfg.head_dim, "cpu", dtype=torch.float32)
    spec = model.linear_state_spec()
    if spec:
        kv.add_linear_state(spec[0], 1, *spec[1:])
    bt = torch.arange(16, dtype=torch.int32)
    toks, out, p0 = list(prompt), [], 0
    for _ in range(n):
        t = len(toks) - p0
        pos = torch.arange(p0, p0 + t, dtype=torch.int32)
        ssm = torch.tensor([[0, t, 0, p0]], dtype=torch.int32) if model.n_lin_layers else None
        b = StepBatch(torch.tensor(toks[p0:], dtype=torch.int32), pos, pos, bt.repeat(t, 1), pos + 1,
                      torch.tensor([t - 1]), p0 + t, ssm_seqs=ssm)
        y = int(model.forward(b, kv)[-1].argmax())
        out.append(y)
        p0 = len(toks)
        toks.append(y)
    return out


@pytest.mark.parametrize("make", [_dense, _hybrid])
@pytest.mark.parametrize("depth", [1, 3])
def test_mtp_speculation_equals_greedy(make, depth):
    from swarmllm_b200.engine.mtp import MtpSpeculator
    from swarmllm_b200.models.llama import LlamaCPU
    from swarmllm_b200.models.weights import RandomSource
    cfg = make()
    src = RandomSource(cfg, seed=9)
    m = LlamaCPU(cfg, src, mtp=True)
    assert m.mtp is not None
    prompt = np.random.default_rng(3).integers(0, cfg.vocab, 11).tolist()
    want = _greedy(m, prompt, 14)
    spec = MtpSpeculator(m, depth=depth, max_len=128)
    got = spec.generate(prompt, 14)
    assert got == want
    st = spec.stats
    assert st.rounds >= 1 and st.drafted >= st.accepted and st.tokens_per_round >= 1.0


def test_mtp_block_in_the_file(tmp_path):
    """A written GGUF carries the block after the trunk (blk.{n_layers}) with
    its nextn tensors and the metadata key; the loader reads it back."""
    from swarmllm_b200.gguf.file import GGUFReader
    from swarmllm_b200.models.llama import LlamaCPU
    from swarmllm_b200.models.weights import GgufSource, write_random_gguf
    cfg = _hybrid()
    path = write_random_gguf(cfg, str(tmp_path / "m.gguf"), seed=1)
    r = GGUFReader(path)
    L = cfg.n_layers
    for n in ("nextn.eh_proj.weight", "nextn.enorm.weight", "nextn.hnorm.weight",
              "attn_q.weight", "post_attention_norm.weight"):
        assert f"blk.{L}.{n}" in r.tensors, n
    src = GgufSource(path)
    assert src.cfg.mtp_layers == 1
    m = LlamaCPU(src.cfg, src, mtp=True)
    assert m.mtp is not None and not m.mtp.linear


@pytest.mark.parametrize("make", [_dense, _hybrid])
def test_accepted_chains_commit_several_tokens(make, monkeypatch):
    """Drafts that the trunk agrees with (here: the true greedy tokens) are all
    kept, several tokens a round; a wrong token at a known place cuts the
    chain there, and the recurrent state is rewound."""
    from swarmllm_b200.engine.mtp import MtpSpeculator
    from swarmllm_b200.models.llama import LlamaCPU
    from swarmllm_b200.models.weights import RandomSource
    cfg = make()
    m = LlamaCPU(cfg, RandomSource(cfg, seed=4), mtp=True)
    prompt = np.random.default_rng(5).integers(0, cfg.vocab, 9).tolist()
    want = _greedy(m, prompt, 13)
    spec = MtpSpeculator(m, depth=4, max_len=128)
    real = spec._draft
    state = {"n": 1}                      # tokens committed so far (y counts)

    def oracle(lg, out, p_next):
        real(lg, out, p_next)             # the head still runs (its cache stays filled)
        k = p_next - len(prompt)          # index in `want` of the token at p_next
        d = want[k:k + spec.depth]
        if state["n"] == 1 and len(d) > 2:
            d = d[:2] + [(d[2] + 1) % cfg.vocab] + d[3:]   # one wrong guess in round 1
        state["n"] += 1
        return d
    monkeypatch.setattr(spec, "_draft", oracle)
    got = spec.generate(prompt, 13)
    assert got == want
    st = spec.stats
    # round 1 keeps the two tokens before the wrong one; the rest are all kept
    assert st.drafted - st.accepted == 2 and st.tokens_per_round > 2.0


def test_cli_generate_with_mtp(tmp_path, capsys):
    import json

    from swarmllm_b200.cli import main
    from swarmllm_b200.models.weights import write_random_gguf
    path = write_random_gguf(_dense(), str(tmp_path / "m.gguf"), seed=2)
    main(["generate", "--gguf", path, "--device", "cpu", "--ids", "5,6,7,8", "--max-tokens", "6"])
    plain = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    main(["generate", "--gguf", path, "--device", "cpu", "--ids", "5,6,7,8", "--max-tokens", "6",
          "--mtp-depth", "3"])
    spec = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert spec["token_ids"] == plain["token_ids"] and spec["mtp_rounds"] >= 1
