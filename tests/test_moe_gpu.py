"""MoE kernels (routing, dispatch, grouped tensor-core expert GEMMs, combine)
against a float32 PyTorch oracle built from the dequantized expert weights."""
import numpy as np
import pytest
import torch

from swarmllm_b200.gguf import quants as Q

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _experts(rng, E, rows, K, qt, std=0.05):
    w = (rng.standard_normal((E, rows, K), dtype=np.float32) * std)
    raw = np.stack([Q.quantize(w[e], qt) for e in range(E)])
    deq = np.stack([Q.dequantize(raw[e], qt) for e in range(E)]).astype(np.float32)
    return torch.from_numpy(raw), torch.from_numpy(deq)


def _oracle(x, ids, wts, gd, ud, dd, bg, bu, bd, act_kind, alpha, limit, xdt):
    """fp32 MoE with the GPU's routing; activations rounded like the kernels."""
    T, k = ids.shape
    xq = x.to(xdt).float()
    y = torch.zeros(T, dd.shape[1])
    for t in range(T):
        for j in range(k):
            e = int(ids[t, j])
            g = gd[e] @ xq[t] + (bg[e] if bg is not None else 0)
            u = ud[e] @ xq[t] + (bu[e] if bu is not None else 0)
            if act_kind == 0:
                h = torch.nn.functional.silu(g) * u
            else:
                g = torch.clamp(g, max=limit)
                u = torch.clamp(u, -limit, limit)
                h = g * torch.sigmoid(alpha * g) * (u + 1)
            h = h.to(xdt).float()
            o = dd[e] @ h + (bd[e] if bd is not None else 0)
            y[t] += wts[t, j] * o
    return y


def _rel(a, b):
    return float((a.double() - b.double()).norm() / (b.double().norm() + 1e-30))


@pytest.mark.parametrize("fmt,E,k,H,F,T,after,bias", [
    ("mxfp4", 8, 4, 320, 192, 1, True, True),      # partial last K unit on both GEMMs
    ("mxfp4", 8, 4, 320, 192, 37, True, True),
    ("mxfp4", 16, 2, 512, 256, 300, True, False),  # N=64/128 token tiles
    ("q4k", 16, 4, 512, 256, 5, False, False),
    ("q4k", 32, 8, 512, 256, 130, True, False),
])
def test_moe_ffn_matches_oracle(fmt, E, k, H, F, T, after, bias):
    from swarmllm_b200.ops.moe import MoeExperts, MoeWorkspace, moe_ffn
    rng = np.random.default_rng(E * 1000 + T)
    qt = Q.MXFP4 if fmt == "mxfp4" else Q.Q4_K
    graw, gd = _experts(rng, E, F, H, qt)
    uraw, ud = _experts(rng, E, F, H, qt)
    draw, dd = _experts(rng, E, H, F, qt)
    bg = bu = bd = None
    act_kind, alpha, limit = 0, 1.702, 7.0
    if bias:
        bg = torch.from_numpy(rng.standard_normal((E, F), dtype=np.float32) * 0.1)
        bu = torch.from_numpy(rng.standard_normal((E, F), dtype=np.float32) * 0.1)
        bd = torch.from_numpy(rng.standard_normal((E, H), dtype=np.float32) * 0.1)
        act_kind = 1
    ex = MoeExperts(graw, uraw, draw, qt, H, F, DEV, gate_b=bg, up_b=bu, down_b=bd,
                    act_kind=act_kind, alpha=alpha, limit=limit)
    wr = torch.from_numpy(rng.standard_normal((E, H), dtype=np.float32) * 0.1)
    br = torch.from_numpy(rng.standard_normal(E, dtype=np.float32) * 0.1) if bias else None
    nsm = torch.cuda.get_device_properties(0).multi_processor_count
    ws = MoeWorkspace(DEV, max(T, 8), H, F, E, k, ex.x_dtype, nsm)
    from swarmllm_b200.ops.linear import GemmWorkspace, QLinear
    router = QLinear(torch.from_numpy(Q.quantize(wr.numpy(), Q.F32)), Q.F32, E, H, DEV, f32_as_f16=True)
    gws = GemmWorkspace(DEV, max(T, 8), E)
    wr = wr.half().float()  # the router runs with fp16 weights
    x = torch.from_numpy(rng.standard_normal((T, H), dtype=np.float32)).half()
    resid0 = torch.from_numpy(rng.standard_normal((T, H), dtype=np.float32))
    for rep in range(2):  # second call reuses the zeroed counters
        resid = resid0.clone().to(DEV)
        moe_ffn(x.to(DEV), ex, router, br.to(DEV) if br is not None else None, ws, gws,
                resid, None, None, 1e-5, softmax_after_topk=after)
        torch.cuda.synchronize()
        ws.check()
        ids = ws.ids[:T * k].view(T, k).cpu()
        wts = ws.wts[:T * k].view(T, k).cpu()
        # routing: chosen experts are the top-k logits (up to near-ties)
        lg = x.float() @ wr.T + (br if br is not None else 0)
        srt = torch.sort(lg, dim=1, descending=True).values
        for t in range(T):
            thr = srt[t, k - 1] - 1e-3
            assert all(lg[t, int(e)] >= thr for e in ids[t]), (t, ids[t])
            assert len(set(ids[t].tolist())) == k
            p = torch.softmax(lg[t, ids[t].long()], 0) if after else torch.softmax(lg[t], 0)[ids[t].long()]
            assert torch.allclose(wts[t], p, atol=2e-4, rtol=1e-3)
        xdt = torch.bfloat16 if fmt == "mxfp4" else torch.float16
        y = _oracle(x.float(), ids, wts, gd, ud, dd, bg, bu, bd, act_kind, alpha, limit, xdt)
        got = resid.cpu() - resid0
        assert _rel(got, y) < 1e-2, (rep, _rel(got, y))
        assert int(ws.counts.abs().sum()) == 0


def test_moe_combine_norm_and_shared():
    """combine: weighted rows + sigmoid-gated shared expert + residual + RMSNorm."""
    from swarmllm_b200.ops.linear import GemmWorkspace, QLinear
    from swarmllm_b200.utils.ext import C
    rng = np.random.default_rng(3)
    T, k, H = 6, 3, 256
    rows = torch.from_numpy(rng.standard_normal((T * k, H), dtype=np.float32)).to(DEV)
    wts = torch.from_numpy(rng.random((T * k), dtype=np.float32)).to(DEV)
    resid0 = torch.from_numpy(rng.standard_normal((T, H), dtype=np.float32))
    x = torch.from_numpy(rng.standard_normal((T, 256), dtype=np.float32)).half().to(DEV)
    wsh = rng.standard_normal((H, 256), dtype=np.float32) * 0.05
    wg = rng.standard_normal((1, 256), dtype=np.float32) * 0.05
    ls = QLinear(torch.from_numpy(Q.quantize(wsh, Q.F32)), Q.F32, H, 256, DEV)
    lg = QLinear(torch.from_numpy(Q.quantize(wg, Q.F32)), Q.F32, 1, 256, DEV)
    gw = GemmWorkspace(DEV, 8, H)
    gw.dense(8 * H * 2)
    gw2 = GemmWorkspace(DEV, 8, H)
    gw2.dense(8 * H * 2)
    sh = ls(x, gw)
    shg = lg(x, gw2)
    norm = torch.from_numpy(rng.random(H, dtype=np.float32) + 0.5).to(DEV)
    out = torch.zeros(T, H, dtype=torch.float16, device=DEV)
    resid = resid0.clone().to(DEV)
    C().moe_combine(rows, wts, k, sh, shg, resid, norm, out, 1e-6)
    torch.cuda.synchronize()
    xf = x.float().cpu()
    gate = torch.sigmoid(xf @ torch.from_numpy(wg).T)
    v = (wts.cpu().view(T, k, 1) * rows.cpu().view(T, k, H)).sum(1) + gate * (xf @ torch.from_numpy(wsh).T)
    r = resid0 + v
    assert _rel(resid.cpu(), r) < 1e-5
    ref = r * torch.rsqrt(r.pow(2).mean(-1, keepdim=True) + 1e-6) * norm.cpu()
    assert _rel(out.float().cpu(), ref) < 2e-3
