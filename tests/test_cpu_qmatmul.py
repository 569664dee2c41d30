"""Native CPU quantized matmul (csrc/native/cpu_qmatmul.cpp) against fp32.

The kernel quantizes the activations to int8 per 32 values and takes integer
dot products with the weights' codes; the oracle is the fp32 product of the
dequantized weights (gguf/quants.py) with (a) the exact activations, to bound
the int8 rounding error, and (b) the activations rounded the way the kernel
rounds them, which must match to fp32 accumulation order.
"""
import numpy as np
import pytest

from swarmllm_b200 import _native
from swarmllm_b200.gguf import quants as Q


def _round_like_kernel(x: np.ndarray) -> np.ndarray:
    T, K = x.shape
    b = x.reshape(T, K // 32, 32)
    amax = np.abs(b).max(-1, keepdims=True)
    inv = np.where(amax > 0, np.float32(127) / np.where(amax > 0, amax, 1), 0).astype(np.float32)
    q = np.rint(b * inv)
    return (q * (amax / np.float32(127))).reshape(T, K).astype(np.float32)


@pytest.mark.parametrize("qtype", [Q.Q4_K, Q.Q6_K, Q.Q8_0, Q.Q4_0, Q.IQ4_NL, Q.IQ4_XS,
                                   Q.MXFP4])
@pytest.mark.parametrize("T", [1, 3])
def test_cpu_qmatmul_matches_dequantized(qtype, T):
    rng = np.random.default_rng(qtype * 10 + T)
    rows, K = 48, 512
    w = Q.random_quantized(rows, K, qtype, rng=rng)
    wf = Q.dequantize(w, qtype, rows * K).reshape(rows, K)
    x = rng.standard_normal((T, K), dtype=np.float32)
    out = _native.cpu_qmatmul(w, qtype, rows, K, x)
    assert out.shape == (T, rows) and out.dtype == np.float32
    exact = x @ wf.T
    rounded = _round_like_kernel(x) @ wf.T
    scale = np.abs(exact).max()
    assert np.abs(out - rounded).max() <= 2e-5 * scale
    assert np.abs(out - exact).max() <= 2e-2 * scale


def test_cpu_qmatmul_rejects_bad_shapes():
    w = Q.random_quantized(4, 256, Q.Q4_K)
    with pytest.raises(ValueError):
        _native.cpu_qmatmul(w, Q.Q4_K, 4, 256, np.zeros((1, 128), np.float32))
    with pytest.raises(ValueError):
        _native.cpu_qmatmul(w, Q.F16, 4, 256, np.zeros((1, 256), np.float32))


def test_cpu_qmatmul_generic_path_agrees():
    """The portable path (forced by SWARMLLM_CPU_ISA=generic, read once per
    process) gives the same numbers as the one this CPU picks."""
    import os
    import subprocess
    import sys
    code = (
        "import numpy as np\n"
        "from swarmllm_b200 import _native\n"
        "from swarmllm_b200.gguf import quants as Q\n"
        "rng = np.random.default_rng(7)\n"
        "x = rng.standard_normal((5, 512), dtype=np.float32)\n"
        "outs = []\n"
        "for qt in (Q.Q4_K, Q.Q6_K, Q.Q8_0, Q.Q4_0, Q.IQ4_NL, Q.IQ4_XS, Q.MXFP4):\n"
        "    w = Q.random_quantized(40, 512, qt, rng=rng)\n"
        "    outs.append(_native.cpu_qmatmul(w, qt, 40, 512, x))\n"
        "np.save(__import__('sys').argv[1], np.stack(outs))\n"
        "print(_native.cpu_qmatmul_isa())\n")
    import tempfile
    with tempfile.TemporaryDirectory() as d:
        res = {}
        for isa in ("generic", "auto"):
            env = dict(os.environ)
            env.pop("SWARMLLM_CPU_ISA", None)
            if isa == "generic":
                env["SWARMLLM_CPU_ISA"] = "generic"
            f = os.path.join(d, isa + ".npy")
            r = subprocess.run([sys.executable, "-c", code, f], env=env, capture_output=True,
                               text=True, timeout=120)
            assert r.returncode == 0, r.stderr
            if isa == "generic":
                assert r.stdout.strip() == "generic"
            res[isa] = np.load(f)
        scale = np.abs(res["generic"]).max()
        assert np.abs(res["generic"] - res["auto"]).max() <= 1e-5 * scale


@pytest.mark.parametrize("qtype", [Q.Q8_0, Q.Q4_0, Q.IQ4_NL, Q.MXFP4])
def test_cpu_qmatmul_small_blocks_any_width(qtype):
    """32-value block formats take any K that is a multiple of 32 (the
    portable path runs when K is not a multiple of 256)."""
    rng = np.random.default_rng(9)
    rows, K = 24, 96
    w = Q.random_quantized(rows, K, qtype, rng=rng)
    wf = Q.dequantize(w, qtype, rows * K).reshape(rows, K)
    x = rng.standard_normal((2, K), dtype=np.float32)
    out = _native.cpu_qmatmul(w, qtype, rows, K, x)
    ref = _round_like_kernel(x) @ wf.T
    assert np.abs(out - ref).max() <= 2e-5 * np.abs(ref).max()


@pytest.mark.parametrize("qtype", [Q.Q4_K, Q.Q6_K, Q.Q8_0, Q.Q4_0, Q.IQ4_NL, Q.IQ4_XS, Q.MXFP4])
def test_cpu_dequant_matches_the_format(qtype):
    rng = np.random.default_rng(qtype)
    rows, K = 12, 512
    w = Q.random_quantized(rows, K, qtype, rng=rng)
    got = _native.cpu_dequant(w, qtype, rows, K)
    want = Q.dequantize(w, qtype, rows * K).reshape(rows, K)
    assert np.allclose(got, want, rtol=1e-6, atol=1e-7)


def test_prefill_rows_take_the_dequantized_gemm(monkeypatch):
    """From PREFILL_T rows on, _QWeight multiplies the dequantized slabs in
    fp32 (exact activations): equal to the fp32 product."""
    import torch

    from swarmllm_b200.models.llama import _QWeight
    rng = np.random.default_rng(2)
    rows, K = 300, 512
    w = Q.random_quantized(rows, K, Q.Q4_K, rng=rng)
    W = _QWeight(w, Q.Q4_K, rows, K)
    monkeypatch.setattr(_QWeight, "SLAB_FLOATS", 100 * K)     # several slabs
    x = torch.from_numpy(rng.standard_normal((_QWeight.PREFILL_T, K), dtype=np.float32))
    ref = x @ torch.from_numpy(Q.dequantize(w, Q.Q4_K, rows * K).reshape(rows, K)).T
    assert torch.allclose(W.mm(x), ref, atol=1e-4)
