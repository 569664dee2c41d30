"""Block drafter (DFlash): the file format, the drafter forward over the
target's captured streams, and block speculation whose greedy output equals
plain decoding (dense and hybrid targets)."""
import numpy as np
import pytest

from test_mtp import _dense, _greedy, _hybrid


def _target(make, seed=9):
    from swarmllm_b200.models.llama import LlamaCPU
    from swarmllm_b200.models.weights import RandomSource
    cfg = make()
    return LlamaCPU(cfg, RandomSource(cfg, seed=seed))


@pytest.mark.parametrize("make", [_dense, _hybrid])
@pytest.mark.parametrize("causal", [False, True])
def test_block_speculation_equals_greedy(make, causal, tmp_path):
    from swarmllm_b200.engine.block_spec import BlockSpeculator
    from swarmllm_b200.models.dflash import DFlashDrafter, write_random_dflash
    m = _target(make)
    path = str(tmp_path / "block_drafter.gguf")
    dc = write_random_dflash(path, m.cfg, n_layers=2, block_size=5, causal=causal)
    d = DFlashDrafter(path, m)
    assert d.cfg.target_layers == dc.target_layers and d.cfg.causal == causal
    prompt = np.random.default_rng(1).integers(0, m.cfg.vocab, 10).tolist()
    want = _greedy(m, prompt, 12)
    spec = BlockSpeculator(m, d, max_len=128)
    assert spec.generate(prompt, 12) == want
    assert spec.stats.rounds >= 1 and d.n_ctx == len(prompt) + 12 - 1


@pytest.mark.parametrize("make", [_dense, _hybrid])
def test_kept_blocks_commit_several_tokens(make, tmp_path, monkeypatch):
    """Guesses the trunk agrees with are all kept: several tokens a round."""
    from swarmllm_b200.engine.block_spec import BlockSpeculator
    from swarmllm_b200.models.dflash import DFlashDrafter, write_random_dflash
    m = _target(make, seed=4)
    path = str(tmp_path / "d.gguf")
    write_random_dflash(path, m.cfg, n_layers=1, block_size=4)
    d = DFlashDrafter(path, m)
    prompt = np.random.default_rng(2).integers(0, m.cfg.vocab, 8).tolist()
    want = _greedy(m, prompt, 11)
    real = d.draft

    def oracle(last, start):
        real(last, start)                                  # the drafter still runs
        k = start - len(prompt) + 1                        # index in `want` of position start+1
        return want[k:k + d.cfg.block_size - 1]
    monkeypatch.setattr(d, "draft", oracle)
    spec = BlockSpeculator(m, d, max_len=128)
    assert spec.generate(prompt, 11) == want
    assert spec.stats.accepted == spec.stats.drafted and spec.stats.tokens_per_round > 3.0


def test_drafter_file_checks(tmp_path):
    from swarmllm_b200.models.dflash import DFlashDrafter, write_random_dflash
    m = _target(_dense)
    bad = str(tmp_path / "bad.gguf")
    write_random_dflash(bad, m.cfg, target_layers=(1, m.cfg.n_layers + 3))
    with pytest.raises(ValueError, match="target layers"):
        DFlashDrafter(bad, m)
    with pytest.raises(ValueError, match="mask token"):
        write_random_dflash(bad, m.cfg, mask_token=m.cfg.vocab + 5)
        DFlashDrafter(bad, m)


def test_cli_generate_with_block_drafter(tmp_path, capsys):
    import json

    from swarmllm_b200.cli import main
    from swarmllm_b200.models.dflash import write_random_dflash
    from swarmllm_b200.models.weights import GgufSource, write_random_gguf
    path = write_random_gguf(_dense(), str(tmp_path / "m.gguf"), seed=2)
    dpath = str(tmp_path / "block_drafter.gguf")
    write_random_dflash(dpath, GgufSource(path).cfg, block_size=4)
    args = ["generate", "--gguf", path, "--device", "cpu", "--ids", "5,6,7,8", "--max-tokens", "6"]
    main(args)
    plain = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    main(args + ["--block-drafter", dpath])
    spec = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert spec["token_ids"] == plain["token_ids"] and spec["rounds"] >= 1
