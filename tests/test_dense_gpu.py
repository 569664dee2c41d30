"""Dense 16-bit tensor-core GEMM (dense_gemm_tc.cu) against an fp32 matmul."""
import numpy as np
import pytest
import torch

from swarmllm_b200.gguf import quants as Q

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _rel(a, b):
    return float((a.double() - b.double()).norm() / (b.double().norm() + 1e-30))


@pytest.mark.parametrize("rows,K,T", [(128, 128, 1), (384, 2880, 7), (200, 4096, 33),
                                      (1024, 2880, 64), (640, 1024, 300)])
@pytest.mark.parametrize("qt", [Q.F16, Q.BF16])
def test_dense_gemm_matches_fp32(rows, K, T, qt):
    from swarmllm_b200.ops.linear import GemmWorkspace, QLinear
    from swarmllm_b200.utils.ext import C
    rng = np.random.default_rng(rows + K + T)
    w = rng.standard_normal((rows, K), dtype=np.float32) * 0.05
    raw = Q.quantize(w, qt)
    lin = QLinear(torch.from_numpy(raw), qt, rows, K, DEV)
    assert lin.kind == "dense"
    ws = GemmWorkspace(DEV, max(T, 16), rows)
    x = torch.from_numpy(rng.standard_normal((T, K), dtype=np.float32)).half().to(DEV)
    g = lin(x, ws)
    out = torch.empty(T, rows, dtype=torch.float32, device=DEV)
    C().epi_copy(g, None, out)
    torch.cuda.synchronize()
    ws.check()
    wq = torch.from_numpy(Q.dequantize(raw, qt)).half().float()
    ref = x.float().cpu() @ wq.T
    assert _rel(out.cpu(), ref) < 1e-3


def test_dense_gemm_forced_sms_multi_segment():
    """Few CTAs: each one walks many tile segments (double-buffered accumulator)."""
    from swarmllm_b200.ops.linear import GemmWorkspace, QLinear
    from swarmllm_b200.utils.ext import C
    rng = np.random.default_rng(7)
    rows, K, T = 1024, 640, 40
    w = rng.standard_normal((rows, K), dtype=np.float32) * 0.05
    lin = QLinear(torch.from_numpy(Q.quantize(w, Q.F16)), Q.F16, rows, K, DEV)
    for sms in (3, 7, 16):
        ws = GemmWorkspace(DEV, T, rows, num_sms=sms)
        x = torch.from_numpy(rng.standard_normal((T, K), dtype=np.float32)).half().to(DEV)
        g = lin(x, ws)
        out = torch.empty(T, rows, dtype=torch.float32, device=DEV)
        C().epi_copy(g, None, out)
        torch.cuda.synchronize()
        ws.check()
        ref = x.float().cpu() @ torch.from_numpy(w).half().float().T
        assert _rel(out.cpu(), ref) < 1e-3, sms
