"""Numerics of every sm_100a kernel against a plain PyTorch fp32 reference."""
import math

import numpy as np
import pytest
import torch

from swarmllm_b200.gguf import quants as Q

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def C():
    from swarmllm_b200.utils.ext import C as _C
    return _C()


# Q4_K at 1..2 tokens runs the CUDA-core GEMV on int8 activations (one scale
# per 32 values): ~0.5 % relative error from the activation rounding.
GEMV_I8_TOL = 1.2e-2


def q4k_tol(T):
    return GEMV_I8_TOL if T <= 2 else 3e-3


def rel_err(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / (b.norm() + 1e-30))


def _x(T, K, seed=0, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(T, K, generator=g) * scale).to(torch.float16)


@pytest.mark.parametrize("qt", [Q.Q4_0, Q.Q8_0, Q.Q4_K, Q.Q6_K, Q.IQ4_NL, Q.IQ4_XS, Q.MXFP4,
                                Q.F16, Q.BF16, Q.F32])
@pytest.mark.parametrize("T", [1, 5, 11])
def test_qmatmul_simt(qt, T):
    rows, K = 96, 512
    rng = np.random.default_rng(1)
    w = rng.standard_normal((rows, K), dtype=np.float32) * 0.02
    b = Q.quantize(w, qt)
    wd = torch.from_numpy(Q.dequantize(b, qt))
    x = _x(T, K)
    ref = x.float() @ wd.T
    out = torch.empty(T, rows, dtype=torch.float32, device=DEV)
    C().qmatmul_simt(torch.from_numpy(b).to(DEV), qt, rows, K, x.to(DEV), out)
    assert rel_err(out.cpu(), ref) < 1e-4


def _dense_from(g, T, rows):
    out = torch.empty(T, rows, dtype=torch.float32, device=DEV)
    C().epi_copy(g, None, out)
    return out


@pytest.mark.parametrize("rows,K", [(128, 256), (384, 1024), (1024, 4096), (256, 8192)])
@pytest.mark.parametrize("T", [1, 7, 16, 33, 64, 130, 256, 300])
def test_qgemm_q4k_tc(rows, K, T):
    rng = np.random.default_rng(rows + K)
    w = rng.standard_normal((rows, K), dtype=np.float32) * 0.02
    b = Q.quantize(w, Q.Q4_K)
    wd = torch.from_numpy(Q.dequantize(b, Q.Q4_K))
    x = _x(T, K, seed=T)
    ref = x.float() @ wd.T
    from swarmllm_b200.ops.linear import GemmWorkspace, QLinear
    ws = GemmWorkspace(DEV, max(T, 1), rows)
    lin = QLinear(b, Q.Q4_K, rows, K, DEV)
    assert lin.use_tc
    g = lin(x.to(DEV), ws)
    out = _dense_from(g, T, rows)
    torch.cuda.synchronize()
    ws.check()
    e = rel_err(out.cpu(), ref)
    assert e < q4k_tol(T), e


@pytest.mark.parametrize("rows,K", [(384, 1024), (1280, 8192)])
@pytest.mark.parametrize("T", [1, 2])
def test_qgemv_q4k_strided(rows, K, T):
    """Decode sizes run the CUDA-core GEMV; activations as a strided view."""
    from swarmllm_b200.ops.linear import GemmWorkspace, QLinear
    from swarmllm_b200.utils.ext import C
    assert T <= C().q4k_gemv_max_t()
    rng = np.random.default_rng(rows + 7 * T)
    w = rng.standard_normal((rows, K), dtype=np.float32) * 0.02
    b = Q.quantize(w, Q.Q4_K)
    wd = torch.from_numpy(Q.dequantize(b, Q.Q4_K))
    big = _x(T, K + 64, seed=3 * T) * 4.0
    x = big[:, 8:K + 8]                       # row stride K + 64, 16-byte aligned start
    ref = x.float() @ wd.T
    ws = GemmWorkspace(DEV, 3, rows)
    lin = QLinear(b, Q.Q4_K, rows, K, DEV)
    out = _dense_from(lin(big.to(DEV)[:, 8:K + 8], ws), T, rows)
    torch.cuda.synchronize()
    ws.check()
    assert rel_err(out.cpu(), ref) < q4k_tol(T)


@pytest.mark.parametrize("qt", [Q.Q4_0, Q.Q8_0, Q.Q6_K, Q.IQ4_NL, Q.IQ4_XS, Q.MXFP4])
def test_prefill_dequant_dense_path(qt):
    """Prefill-sized batches of types without their own tensor-core kernel:
    dequantize to fp16, then the dense tcgen05 GEMM."""
    from swarmllm_b200.ops.linear import DEQUANT_MIN_TOKENS, GemmWorkspace, QLinear
    rows, K, T = 640, 1024, max(DEQUANT_MIN_TOKENS, 100)
    rng = np.random.default_rng(qt)
    w = rng.standard_normal((rows, K), dtype=np.float32) * 0.02
    b = Q.quantize(w, qt)
    wd = torch.from_numpy(Q.dequantize(b, qt).reshape(rows, K))
    x = _x(T, K, seed=5)
    ref = x.float() @ wd.T
    lin = QLinear(b, qt, rows, K, DEV, force_simt=True)   # not the repacked tensor-core path
    ws = GemmWorkspace(DEV, T, rows)
    g = lin(x.to(DEV), ws)
    out = _dense_from(g, T, rows)
    torch.cuda.synchronize()
    ws.check()
    assert rel_err(out.cpu(), ref) < 3e-3


@pytest.mark.parametrize("qt,fmt", [(Q.Q6_K, 1), (Q.Q8_0, 2)])
def test_qfmt_repack_matches_host(qt, fmt):
    rows, K = 200, 768
    rng = np.random.default_rng(4)
    b = Q.quantize(rng.standard_normal((rows, K), dtype=np.float32) * 0.02, qt)
    rb = C().qfmt_row_bytes(fmt)
    dst = torch.full((256 * (K // 256) * rb,), 0xAB, dtype=torch.uint8, device=DEV)
    C().qfmt_repack(fmt, torch.from_numpy(b).to(DEV), rows, K, dst)
    host = (Q.q6k_repack_host if fmt == 1 else Q.q80_repack_host)(b, rows, K).reshape(-1)
    assert np.array_equal(dst.cpu().numpy(), host)


@pytest.mark.parametrize("qt,fmt", [(Q.Q6_K, 1), (Q.Q8_0, 2)])
@pytest.mark.parametrize("rows,K,T,sms", [(384, 1024, 1, 0), (384, 1024, 2, 0), (1024, 4096, 7, 0),
                                          (256, 8192, 33, 0), (640, 2048, 64, 0),
                                          (384, 1024, 130, 0), (1280, 2048, 1, 9),
                                          (1024, 2048, 40, 3), (512, 1024, 300, 4)])
def test_qgemm_tc_formats(qt, fmt, rows, K, T, sms):
    """Q6_K and Q8_0 on the repacked tensor-core GEMM (T > 2) and CUDA-core
    GEMV (T <= 2), against the fp32 product with the repacked weights."""
    from swarmllm_b200.ops.linear import GemmWorkspace, QLinear
    rng = np.random.default_rng(rows + K + T)
    b = Q.quantize(rng.standard_normal((rows, K), dtype=np.float32) * 0.02, qt)
    lin = QLinear(b, qt, rows, K, DEV)
    assert lin.kind == "q4k" and lin.fmt == fmt
    wd = torch.from_numpy(Q.repacked_dequant_host(
        (Q.q6k_repack_host if fmt == 1 else Q.q80_repack_host)(b, rows, K).reshape(-1),
        fmt, rows, K))
    x = _x(T, K, seed=T + 2) * 2.0
    ws = GemmWorkspace(DEV, T, rows, num_sms=sms or None)
    out = _dense_from(lin(x.to(DEV), ws), T, rows)
    torch.cuda.synchronize()
    ws.check()
    # 1..2 tokens: the GEMV's int8 activations
    tol = GEMV_I8_TOL if T <= 2 else 3e-3
    assert rel_err(out.cpu(), x.float() @ wd.T) < tol


def test_q4k_repack_matches_host():
    rows, K = 256, 512
    rng = np.random.default_rng(3)
    b = Q.quantize(rng.standard_normal((rows, K), dtype=np.float32) * 0.02, Q.Q4_K)
    dst = torch.empty(rows * (K // 256) * 144, dtype=torch.uint8, device=DEV)
    C().q4k_repack(torch.from_numpy(b).to(DEV), rows, K, dst)
    host = Q.q4k_repack_host(b, rows, K).reshape(-1)
    assert np.array_equal(dst.cpu().numpy(), host)


@pytest.mark.parametrize("rows,K,T,sms", [(1280, 2048, 1, 9), (1280, 2048, 33, 9),
                                          (1024, 2048, 1, 2), (1024, 2048, 17, 2), (1024, 2048, 1, 3),
                                          (1024, 2048, 40, 3), (1024, 2048, 130, 1),
                                          (128, 2048, 1, 1), (256, 2048, 5, 3), (384, 3072, 40, 7),
                                          (1024, 4096, 16, 5), (512, 1024, 300, 4),
                                          (256, 28672, 32, 148), (8192 // 8, 8192, 2, 148)])
def test_qgemm_tc_multi_unit_ctas(rows, K, T, sms):
    """Few CTAs: each processes many units and crosses tile boundaries."""
    rng = np.random.default_rng(rows * 7 + T)
    b = Q.quantize(rng.standard_normal((rows, K), dtype=np.float32) * 0.02, Q.Q4_K)
    wd = torch.from_numpy(Q.dequantize(b, Q.Q4_K))
    x = _x(T, K, seed=T + 1)
    from swarmllm_b200.ops.linear import GemmWorkspace, QLinear
    ws = GemmWorkspace(DEV, T, rows, num_sms=sms)
    lin = QLinear(b, Q.Q4_K, rows, K, DEV)
    g = lin(x.to(DEV), ws)
    out = _dense_from(g, T, rows)
    torch.cuda.synchronize()
    ws.check()
    assert rel_err(out.cpu(), x.float() @ wd.T) < q4k_tol(T)


def test_qgemm_tc_stream_k_many_segments():
    """K long enough that tiles split across several CTAs."""
    rows, K, T = 128, 256 * 96, 3
    rng = np.random.default_rng(5)
    b = Q.quantize(rng.standard_normal((rows, K), dtype=np.float32) * 0.02, Q.Q4_K)
    wd = torch.from_numpy(Q.dequantize(b, Q.Q4_K))
    x = _x(T, K, seed=9)
    from swarmllm_b200.ops.linear import GemmWorkspace, QLinear
    ws = GemmWorkspace(DEV, T, rows)
    g = QLinear(b, Q.Q4_K, rows, K, DEV)(x.to(DEV), ws)
    assert g.upc < g.ksb  # really split
    out = _dense_from(g, T, rows)
    assert rel_err(out.cpu(), x.float() @ wd.T) < 3e-3


# ----------------------------------------------------------------------------- epilogues
def _gemm_identity(vals):
    """GemmResult whose content equals `vals` [T, R] (F32 identity weight)."""
    T, R = vals.shape
    w = torch.eye(R, dtype=torch.float32)
    x = vals.to(torch.float16)
    out = torch.empty(T, R, dtype=torch.float32, device=DEV)
    g = C().qmatmul_simt(w.view(torch.uint8).reshape(-1).to(DEV), Q.F32, R, R, x.to(DEV), out)
    return g, x.float()


def test_epi_residual_rmsnorm():
    T, H = 5, 256
    g, v = _gemm_identity(torch.randn(T, H))
    res = torch.randn(T, H)
    w = torch.rand(H) + 0.5
    rd = res.clone().to(DEV)
    out = torch.empty(T, H, dtype=torch.float16, device=DEV)
    C().epi_residual_rmsnorm(g, rd, None, w.to(DEV), out, 1e-5)
    h = res + v
    ref = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + 1e-5) * w
    assert rel_err(rd.cpu(), h) < 1e-6
    assert rel_err(out.float().cpu(), ref) < 2e-3


# rope_dim 34 (odd half) takes the one-pair-per-thread path, the others the
# two-pairs-per-thread vector path; nq 6 leaves a partial 8-head group
@pytest.mark.parametrize("neox,rope_dim,nq", [(False, 64, 4), (True, 64, 4), (True, 32, 4),
                                              (False, 48, 6), (True, 34, 4), (False, 34, 6)])
def test_epi_rope_kv(neox, rope_dim, nq):
    T, nkv, d, ps = 6, 2, 64, 16
    R = (nq + 2 * nkv) * d
    g, v = _gemm_identity(torch.randn(T, R))
    pos = torch.tensor([0, 3, 17, 100, 4095, 9], dtype=torch.int32)
    slots = torch.tensor([5, 16, 33, 2, 40, 63], dtype=torch.int32)
    inv = 1.0 / (10000 ** (torch.arange(0, rope_dim, 2, dtype=torch.float64) / rope_dim))
    inv = inv.float()
    q = torch.empty(T, nq, d, dtype=torch.float16, device=DEV)
    kc = torch.zeros(4, nkv, ps, d, dtype=torch.float16, device=DEV)
    vc = torch.zeros_like(kc)
    C().epi_rope_kv(g, None, pos.to(DEV), slots.to(DEV), inv.to(DEV), nq, nkv, d, rope_dim, neox,
                    1.0, q, kc, vc, ps, None, None, 1e-6)
    x = v.view(T, nq + 2 * nkv, d)

    def rope(t):
        ang = pos.double()[:, None] * inv.double()[None]
        c, s = torch.cos(ang)[:, None], torch.sin(ang)[:, None]
        o = t.double().clone()
        if neox:
            a, b = t[..., :rope_dim // 2].double(), t[..., rope_dim // 2:rope_dim].double()
            o[..., :rope_dim // 2] = a * c - b * s
            o[..., rope_dim // 2:rope_dim] = b * c + a * s
        else:
            a, b = t[..., 0:rope_dim:2].double(), t[..., 1:rope_dim:2].double()
            o[..., 0:rope_dim:2] = a * c - b * s
            o[..., 1:rope_dim:2] = b * c + a * s
        return o
    qr = rope(x[:, :nq])
    kr = rope(x[:, nq:nq + nkv])
    assert rel_err(q.double().cpu(), qr) < 2e-3
    kc, vc = kc.cpu(), vc.cpu()
    for t in range(T):
        p, o = int(slots[t]) // ps, int(slots[t]) % ps
        assert rel_err(kc[p, :, o].double(), kr[t]) < 2e-3
        assert rel_err(vc[p, :, o].double(), x[t, nq + nkv:].double()) < 2e-3


@pytest.mark.parametrize("kind", [0, 1])
def test_epi_swiglu(kind):
    T, F = 3, 256
    g, v = _gemm_identity(torch.randn(T, 2 * F) * 3)
    out = torch.empty(T, F, dtype=torch.float16, device=DEV)
    C().epi_swiglu(g, None, F, kind, False, 1.702, 7.0, out)
    gg, uu = v[:, :F], v[:, F:]
    if kind == 0:
        ref = torch.nn.functional.silu(gg) * uu
    else:
        x = gg.clamp(max=7.0)
        u = uu.clamp(-7.0, 7.0)
        ref = x * torch.sigmoid(1.702 * x) * (u + 1)
    assert rel_err(out.float().cpu(), ref) < 2e-3


# ----------------------------------------------------------------------------- attention
def _attn_ref(q, K, V, bt, lens, ps, scale, window=0, sinks=None, tmask=None, tstart=None):
    T, nq, d = q.shape
    nkv = K.shape[1]
    rep = nq // nkv
    out = torch.zeros(T, nq, d, dtype=torch.float64)
    for t in range(T):
        L = int(lens[t])
        lo = max(0, L - window) if window else 0
        keys = torch.arange(lo, L)
        pg = bt[t].long()[keys // ps]
        kk = K[pg, :, keys % ps].double().repeat_interleave(rep, 1)
        vv = V[pg, :, keys % ps].double().repeat_interleave(rep, 1)
        s = torch.einsum("hd,nhd->hn", q[t].double(), kk) * scale
        if tmask is not None:
            vis = torch.tensor([(k < int(tstart[t])) or (k - int(tstart[t]) < 64 and
                               (int(tmask[t]) >> (k - int(tstart[t]))) & 1 == 1) for k in keys.tolist()])
            s = s.masked_fill(~vis[None], float("-inf"))
        if sinks is not None:
            s = torch.cat([s, sinks.double()[:, None]], 1)
        p = torch.softmax(s, -1)
        if sinks is not None:
            p = p[:, :-1]
        out[t] = torch.einsum("hn,nhd->hd", p, vv)
    return out


@pytest.mark.parametrize("force_simt", [False, True])
@pytest.mark.parametrize("d,nq,nkv", [(128, 64, 8), (128, 24, 8), (64, 64, 8), (256, 16, 2)])
@pytest.mark.parametrize("window,sinks", [(0, False), (128, True)])
def test_paged_decode_attention(d, nq, nkv, window, sinks, force_simt):
    from swarmllm_b200.ops.attention import AttentionWorkspace, paged_attention
    torch.manual_seed(0)
    ps, P = 16, 64
    lens = torch.tensor([1, 17, 300, 700], dtype=torch.int32)
    T = lens.numel()
    K = torch.randn(P, nkv, ps, d).half()
    V = torch.randn(P, nkv, ps, d).half()
    bt = torch.stack([torch.randperm(P)[:48] for _ in range(T)]).int()
    q = torch.randn(T, nq, d).half()
    sk = torch.randn(nq) if sinks else None
    scale = 1 / math.sqrt(d)
    ws = AttentionWorkspace(DEV, T, nq, nkv, d, 768)
    out = torch.empty(T, nq, d, dtype=torch.float16, device=DEV)
    paged_attention(q.to(DEV), K.to(DEV), V.to(DEV), bt.to(DEV), lens.to(DEV), ws, out, 768, scale,
                    window, sk.to(DEV) if sinks else None, force_simt=force_simt)
    torch.cuda.synchronize()
    assert int(ws.status[0]) == 0, ws.status.tolist()
    ref = _attn_ref(q, K, V, bt, lens, ps, scale, window, sk)
    assert rel_err(out.double().cpu(), ref) < 3e-3


@pytest.mark.parametrize("d,nq,nkv,window", [(128, 64, 8, 0), (128, 24, 8, 0), (64, 64, 8, 128),
                                             (256, 16, 2, 0)])
def test_attention_prefill_groups(d, nq, nkv, window):
    """Chunked prefill on the tensor-core path: rows of one sequence grouped
    128 // n_rep positions per CTA, causal lengths, a prefix already cached."""
    from swarmllm_b200.engine.runner import attention_groups
    from swarmllm_b200.ops.attention import AttentionWorkspace, paged_attention
    torch.manual_seed(2)
    ps, P = 16, 64
    prefix, chunk = 100, 150          # sequence 0: 100 cached + 150 new rows
    dec_len = 333                     # sequence 1: one decode row
    T = chunk + 1
    K = torch.randn(P, nkv, ps, d).half()
    V = torch.randn(P, nkv, ps, d).half()
    bt0 = torch.randperm(P)[:32].int()
    bt1 = torch.randperm(P)[:32].int()
    bt = torch.cat([bt0[None].repeat(chunk, 1), bt1[None]], 0)
    lens = torch.cat([torch.arange(prefix + 1, prefix + chunk + 1), torch.tensor([dec_len])]).int()
    q = torch.randn(T, nq, d).half()

    class _Plan:
        seq_start = np.array([0, chunk])
        seq_ntok = np.array([chunk, 1])
    r0, npos, ppg = attention_groups(_Plan, nq // nkv)
    ws = AttentionWorkspace(DEV, T, nq, nkv, d, 512)
    out = torch.empty(T, nq, d, dtype=torch.float16, device=DEV)
    paged_attention(q.to(DEV), K.to(DEV), V.to(DEV), bt.to(DEV), lens.to(DEV), ws, out, 512,
                    1 / math.sqrt(d), window,
                    groups=(torch.from_numpy(r0).to(DEV), torch.from_numpy(npos).to(DEV), ppg))
    torch.cuda.synchronize()
    assert int(ws.status[0]) == 0, ws.status.tolist()
    ref = _attn_ref(q, K, V, bt, lens, ps, 1 / math.sqrt(d), window)
    assert rel_err(out.double().cpu(), ref) < 3e-3


def test_paged_attention_tree_mask():
    from swarmllm_b200.ops.attention import AttentionWorkspace, paged_attention
    torch.manual_seed(1)
    d, nq, nkv, ps, P = 128, 16, 4, 16, 16
    T = 5
    base = 40
    lens = torch.full((T,), base + 5, dtype=torch.int32)
    tmask = torch.tensor([0b1, 0b11, 0b101, 0b1011, 0b10101], dtype=torch.int64)
    tstart = torch.full((T,), base, dtype=torch.int32)
    K = torch.randn(P, nkv, ps, d).half()
    V = torch.randn(P, nkv, ps, d).half()
    bt = torch.arange(P).int()[None].repeat(T, 1)
    q = torch.randn(T, nq, d).half()
    ws = AttentionWorkspace(DEV, T, nq, nkv, d, 64)
    out = torch.empty(T, nq, d, dtype=torch.float16, device=DEV)
    paged_attention(q.to(DEV), K.to(DEV), V.to(DEV), bt.to(DEV), lens.to(DEV), ws, out, 64,
                    1 / math.sqrt(d), tree_mask=tmask.to(DEV), tree_start=tstart.to(DEV))
    ref = _attn_ref(q, K, V, bt, lens, ps, 1 / math.sqrt(d), tmask=tmask, tstart=tstart)
    assert rel_err(out.double().cpu(), ref) < 3e-3


# ----------------------------------------------------------------------------- sampling
@pytest.mark.parametrize("rows,V", [(1, 201088), (3, 151936), (300, 9000), (2, 5000)])
def test_argmax_split_paths(rows, V):
    """Split (atomic 64-bit key) and single-CTA argmax: values, ties -> lowest
    index, all-negative rows, and back-to-back calls (keys reset)."""
    torch.manual_seed(rows)
    logits = -torch.rand(rows, V) * 5 - 1          # all negative
    logits[0, V // 3] = 2.0
    logits[0, V - 7] = 2.0                         # tie: lower index wins
    for _ in range(2):
        out = torch.empty(rows, dtype=torch.int32, device=DEV)
        val = torch.empty(rows, dtype=torch.float32, device=DEV)
        C().argmax(logits.to(DEV), out, val)
        torch.cuda.synchronize()
        assert torch.equal(out.cpu().long(), logits.argmax(-1))
        assert torch.equal(val.cpu(), logits.max(-1).values)


def test_argmax_and_sampling():
    from swarmllm_b200.engine.sampling import SamplingParams, sample_host
    torch.manual_seed(0)
    V = 50000
    logits = torch.randn(6, V) * 3
    out = torch.empty(6, dtype=torch.int32, device=DEV)
    C().argmax(logits.to(DEV), out, None)
    assert torch.equal(out.cpu().long(), logits.argmax(-1))
    params = [SamplingParams(temperature=0.8, seed=11), SamplingParams(temperature=1.0, top_k=20, seed=3),
              SamplingParams(temperature=0.7, top_p=0.9, seed=5), SamplingParams(temperature=0.0),
              SamplingParams(temperature=1.3, top_k=5, top_p=0.8, seed=99),
              SamplingParams(temperature=0.5, seed=123456789012)]
    pos = np.array([0, 5, 9, 3, 1000, 77], dtype=np.int32)
    dev_out = torch.empty(6, dtype=torch.int32, device=DEV)
    C().sample(logits.to(DEV), torch.tensor([p.temperature for p in params]).to(DEV),
               torch.tensor([p.top_k for p in params], dtype=torch.int32).to(DEV),
               torch.tensor([p.top_p for p in params]).to(DEV),
               torch.tensor([p.seed for p in params], dtype=torch.int64).to(DEV),
               torch.from_numpy(pos).to(DEV), dev_out)
    host = sample_host(logits, params, pos)
    assert dev_out.cpu().numpy().tolist() == host.tolist()


def test_philox_matches_host():
    from swarmllm_b200.engine.sampling import philox_uniform_host
    pos = torch.tensor([0, 7, 123456], dtype=torch.int32)
    out = torch.empty(3, 1000, dtype=torch.float32, device=DEV)
    C().philox_uniform(987654321, pos.to(DEV), 1000, out)
    for r in range(3):
        h = philox_uniform_host(987654321, int(pos[r]), np.arange(1000))
        assert np.array_equal(out[r].cpu().numpy(), h)


def test_apply_penalties_kernel():
    import collections
    from swarmllm_b200.engine.sampling import SamplingParams, penalty_table
    rows, V = 5, 3000
    logits = torch.randn(rows, V, device=DEV)
    ref = logits.clone().cpu()
    ps = [SamplingParams(frequency_penalty=0.3 * r, presence_penalty=0.5) for r in range(rows)]
    hist = [collections.Counter({(17 * r + 3 * i) % V: i + 1 for i in range(40 * r)})
            for r in range(rows)]
    off, tok, val = penalty_table(ps, hist)
    for r in range(rows):
        for t, c in hist[r].items():
            ref[r, t] -= c * ps[r].frequency_penalty + ps[r].presence_penalty
    C().apply_penalties(logits, *[torch.from_numpy(a).to(DEV) for a in (off, tok, val)])
    torch.cuda.synchronize()
    assert torch.allclose(logits.cpu(), ref, atol=1e-5)


@pytest.mark.parametrize("ties", [False, True])
def test_sampling_paths_match_host(ties):
    """Every sampling path (short-list top-k, mass radix select without top-k,
    top-k above the short-list size) draws the host sampler's token."""
    from swarmllm_b200.engine.sampling import SamplingParams, sample_host
    torch.manual_seed(1)
    V, R = 40000, 12
    logits = torch.randn(R, V) * 2.5
    if ties:
        logits = (logits * 2).round() / 2      # many equal logits at every cut
    ks = [0, 0, 7, 40, 2048, 3000, 0, 1, 50, 0, 100, 5000]
    ps = [0.5, 0.95, 1.0, 0.9, 0.7, 0.6, 0.99, 0.9, 0.3, 1.0, 1.0, 0.8]
    params = [SamplingParams(temperature=0.6 + 0.1 * r, top_k=ks[r], top_p=ps[r], seed=1000 + r)
              for r in range(R)]
    pos = np.arange(R, dtype=np.int32) * 31
    out = torch.empty(R, dtype=torch.int32, device=DEV)
    args = (logits.to(DEV), torch.tensor([p.temperature for p in params]).to(DEV),
            torch.tensor(ks, dtype=torch.int32).to(DEV), torch.tensor(ps).to(DEV),
            torch.tensor([p.seed for p in params], dtype=torch.int64).to(DEV),
            torch.from_numpy(pos).to(DEV), out)
    C().sample(*args)
    first = out.clone()
    C().sample(*args)
    assert torch.equal(first, out)             # bit-identical reruns
    host = sample_host(logits, params, pos)
    agree = (out.cpu().numpy() == host).mean()
    # float32 (device) and float64 (host) cumulative mass may straddle a cut
    assert agree >= (11 / 12 if ties else 1.0), (out.cpu().tolist(), host.tolist())


@pytest.mark.parametrize("T", [1, 40])
@pytest.mark.parametrize("kind", [0, 1])
def test_swiglu_on_stream_k_partials(T, kind):
    """SwiGLU epilogue (8-wide path) reading a Q4_K GEMM's stream-K partial
    sums, against the fp32 reference of GEMM + activation."""
    from swarmllm_b200.ops.linear import GemmWorkspace, QLinear
    F, K = 1280, 2048
    rng = np.random.default_rng(F + T + kind)
    w = rng.standard_normal((2 * F, K), dtype=np.float32) * 0.02
    b = Q.quantize(w, Q.Q4_K)
    wd = torch.from_numpy(Q.dequantize(b, Q.Q4_K))
    x = _x(T, K, seed=T)
    v = x.float() @ wd.T
    gg, uu = v[:, :F], v[:, F:]
    if kind == 0:
        ref = torch.nn.functional.silu(gg) * uu
    else:
        xg, u = gg.clamp(max=7.0), uu.clamp(-7.0, 7.0)
        ref = xg * torch.sigmoid(1.702 * xg) * (u + 1)
    lin = QLinear(b, Q.Q4_K, 2 * F, K, DEV)
    ws = GemmWorkspace(DEV, T, 2 * F)
    out = torch.empty(T, F, dtype=torch.float16, device=DEV)
    C().epi_swiglu(lin(x.to(DEV), ws), None, F, kind, False, 1.702, 7.0, out)
    torch.cuda.synchronize()
    ws.check()
    assert rel_err(out.float().cpu(), ref) < (1.5e-2 if T <= 2 else 4e-3)


@pytest.mark.parametrize("with_bias", [False, True])
def test_residual_rmsnorm_rows_path(with_bias):
    """Residual add + RMSNorm over >= 64 token rows (one CTA per row, 8-wide
    path) reading a Q4_K GEMM's stream-K partials, against fp32."""
    from swarmllm_b200.ops.linear import GemmWorkspace, QLinear
    T, H, K = 80, 1280, 2048
    rng = np.random.default_rng(7)
    w = rng.standard_normal((H, K), dtype=np.float32) * 0.02
    b = Q.quantize(w, Q.Q4_K)
    wd = torch.from_numpy(Q.dequantize(b, Q.Q4_K))
    x = _x(T, K, seed=3)
    res = torch.randn(T, H)
    bias = torch.randn(H) * 0.1 if with_bias else None
    nw = torch.rand(H) + 0.5
    h = res + x.float() @ wd.T + (bias if with_bias else 0)
    ref = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + 1e-5) * nw
    lin = QLinear(b, Q.Q4_K, H, K, DEV)
    ws = GemmWorkspace(DEV, T, H)
    rd = res.clone().to(DEV)
    out = torch.empty(T, H, dtype=torch.float16, device=DEV)
    C().epi_residual_rmsnorm(lin(x.to(DEV), ws), rd, bias.to(DEV) if with_bias else None,
                             nw.to(DEV), out, 1e-5)
    torch.cuda.synchronize()
    ws.check()
    assert rel_err(rd.cpu(), h) < 3e-3
    assert rel_err(out.float().cpu(), ref) < 4e-3


def test_delta_chunk_matches_recurrent():
    """Chunked gated delta rule (prefill) == the token-sequential recurrent
    kernel on the same inputs: two sequences (one fresh, one resuming a
    random state), partial last chunks; outputs and final states."""
    from swarmllm_b200.ops.linear import GemmWorkspace, QLinear
    torch.manual_seed(5)
    nk, nv, D, H = 2, 4, 128, 256
    seqs_l = [(0, 100, 0, 0), (100, 50, 1, 7)]
    T = 150
    C_ = (2 * nk + nv) * D
    qkv = torch.randn(T, C_, device=DEV)
    x = (torch.randn(T, H) * 0.5).half().to(DEV)
    wba = QLinear((torch.randn(2 * nv, H) * 0.05).half().view(torch.uint8).reshape(-1).numpy(),
                  Q.F16, 2 * nv, H, DEV)
    wz = QLinear((torch.randn(nv * D, H) * 0.05).half().view(torch.uint8).reshape(-1).numpy(),
                 Q.F16, nv * D, H, DEV)
    gba = wba(x, GemmWorkspace(DEV, T, 2 * nv))
    gz = wz(x, GemmWorkspace(DEV, T, nv * D))
    A = -torch.rand(nv, device=DEV) * 0.5
    dtb = torch.rand(nv, device=DEV)
    nw = (torch.rand(D) + 0.5).to(DEV)
    st0 = torch.zeros(3, nv, D, D, device=DEV)
    st0[1] = torch.randn(nv, D, D, device=DEV) * 0.05
    seqs = torch.tensor(seqs_l, dtype=torch.int32, device=DEV)
    st_r, st_c = st0.clone(), st0.clone()
    out_r = torch.zeros(T, nv * D, device=DEV).half()
    out_c = torch.zeros_like(out_r)
    oraw = torch.zeros(T, nv * D, device=DEV)
    C().delta_rule(qkv, nk, nv, D, gba, dtb, A, gz, nw, 1e-6, st_r, seqs, 2, out_r)
    C().delta_chunk(qkv, nk, nv, D, gba, dtb, A, gz, nw, 1e-6, st_c, seqs, 2, oraw, out_c)
    torch.cuda.synchronize()
    assert rel_err(out_c.float().cpu(), out_r.float().cpu()) < 3e-3
    for slot in (0, 1):
        assert rel_err(st_c[slot].cpu(), st_r[slot].cpu()) < 1e-3, slot
