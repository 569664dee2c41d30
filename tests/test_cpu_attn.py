"""Native CPU paged attention, SwiGLU tail and exp (csrc/native/cpu_attn.cpp)
against plain fp32 PyTorch."""
import numpy as np
import pytest
import torch

from swarmllm_b200 import _native


def _reference(q, K, V, bt, lens, scale, window=0, softcap=0.0, tree_start=None,
               tree_mask=None, sinks=None):
    N, nq, d = q.shape
    nkv, ps = K.shape[1], K.shape[2]
    rep = nq // nkv
    out = torch.zeros(N, nq, d)
    for t in range(N):
        Lt = int(lens[t])
        lo = max(0, Lt - window) if window else 0
        keys = torch.arange(lo, Lt)
        kp, ko = bt[t][keys // ps].long(), keys % ps
        kk = K[kp, :, ko, :].float().repeat_interleave(rep, 1)
        vv = V[kp, :, ko, :].float().repeat_interleave(rep, 1)
        s = torch.einsum("hd,nhd->hn", q[t], kk) * scale
        if softcap:
            s = softcap * torch.tanh(s / softcap)
        if tree_mask is not None:
            rel = keys - int(tree_start[t])
            m = int(tree_mask[t]) & ((1 << 64) - 1)
            vis = torch.tensor([r < 0 or (r < 64 and (m >> r) & 1 == 1) for r in rel.tolist()])
            s = s.masked_fill(~vis[None, :], float("-inf"))
        if sinks is not None:
            s = torch.cat([s, sinks[:, None]], 1)
        p = torch.softmax(s, -1)
        if sinks is not None:
            p = p[:, :-1]
        out[t] = torch.einsum("hn,nhd->hd", p, vv)
    return out


def _case(seed, dtype, N=5, nq=8, nkv=2, d=64, ps=16, max_len=700):
    g = torch.Generator().manual_seed(seed)
    pages_per = (max_len + ps - 1) // ps
    n_pages = N * pages_per + 3
    K = torch.randn(n_pages, nkv, ps, d, generator=g).to(dtype)
    V = torch.randn(n_pages, nkv, ps, d, generator=g).to(dtype)
    perm = torch.randperm(n_pages, generator=g)[: N * pages_per].view(N, pages_per).int()
    lens = torch.randint(1, max_len + 1, (N,), generator=g).int()
    lens[0] = max_len            # several 256-key chunks
    q = torch.randn(N, nq, d, generator=g)
    return q, K, V, perm, lens


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_cpu_attention_plain_and_gqa(dtype):
    q, K, V, bt, lens = _case(1, dtype)
    out = _native.cpu_paged_attention(q.numpy(), K.numpy(), V.numpy(), bt.numpy(), lens.numpy(),
                                      0.125)
    ref = _reference(q, K, V, bt, lens, 0.125)
    assert np.abs(out - ref.numpy()).max() < 2e-5 * 50


def test_cpu_attention_window_softcap_sinks():
    q, K, V, bt, lens = _case(2, torch.float16, nq=4, nkv=4)
    sinks = torch.randn(4)
    kw = dict(window=100, softcap=30.0)
    out = _native.cpu_paged_attention(q.numpy(), K.numpy(), V.numpy(), bt.numpy(), lens.numpy(),
                                      0.3, sinks=sinks.numpy(), **kw)
    ref = _reference(q, K, V, bt, lens, 0.3, sinks=sinks, **kw)
    assert np.abs(out - ref.numpy()).max() < 1e-4


def test_cpu_attention_tree_mask():
    q, K, V, bt, lens = _case(3, torch.float16, N=6, max_len=300)
    g = np.random.default_rng(3)
    tree_start = (lens.numpy() - g.integers(1, 40, size=6)).clip(0).astype(np.int32)
    masks = g.integers(0, 2 ** 62, size=6, dtype=np.int64)
    masks[1] = -1                     # every bit, the sign bit included
    out = _native.cpu_paged_attention(q.numpy(), K.numpy(), V.numpy(), bt.numpy(), lens.numpy(),
                                      0.125, tree_start=tree_start, tree_mask=masks)
    ref = _reference(q, K, V, bt, lens, 0.125, tree_start=torch.from_numpy(tree_start),
                     tree_mask=torch.from_numpy(masks))
    ok = ~torch.isnan(ref)
    assert np.abs(out[ok.numpy()] - ref[ok].numpy()).max() < 1e-4


def test_exp_approx_relative_error():
    x = np.linspace(-87, 88, 200001, dtype=np.float32)
    got = _native.exp_approx(x).astype(np.float64)
    want = np.exp(x.astype(np.float64))
    assert (np.abs(got - want) / want).max() < 5e-7
    assert _native.exp_approx(np.array([-200.0], np.float32))[0] == 0.0


@pytest.mark.parametrize("limit", [0.0, 7.0])
def test_cpu_silu_mul(limit):
    g = torch.randn(3, 1000) * 6
    u = torch.randn(3, 1000) * 6
    out = _native.cpu_silu_mul(g.numpy(), u.numpy(), limit, 1.702)
    if limit:
        gc, uc = torch.clamp(g, max=limit), torch.clamp(u, -limit, limit)
        ref = gc * torch.sigmoid(1.702 * gc) * (uc + 1)
    else:
        ref = torch.nn.functional.silu(g) * u
    assert np.abs(out - ref.numpy()).max() < 1e-5 * 50


def test_cpu_attention_reads_every_fp16_value():
    """Every fp16 bit pattern but inf/NaN (subnormals included) as a V row
    value comes back exactly through a one-key attention."""
    vals = np.arange(65536, dtype=np.uint32).astype(np.uint16).view(np.float16)
    vals = vals[np.isfinite(vals)]
    d = 64
    n = len(vals) // d
    V = vals[: n * d].reshape(n, 1, 1, d).copy()
    K = np.zeros_like(V)
    q = np.zeros((n, 1, d), np.float32)
    bt = np.arange(n, dtype=np.int32).reshape(n, 1)
    out = _native.cpu_paged_attention(q, K, V, bt, np.ones(n, np.int32), 1.0)
    assert np.array_equal(out.reshape(-1), V.reshape(-1).astype(np.float32))


@pytest.mark.parametrize("window,tree,sinks", [(0, False, False), (40, False, True), (0, True, False)])
def test_cpu_attention_prefill_blocks(window, tree, sinks):
    """Tokens of one sequence (one block table, causal lengths) share tasks in
    blocks of 16: per-token key ranges, windows, tree masks and sinks kept."""
    g = torch.Generator().manual_seed(5)
    T, nq, nkv, d, ps = 37, 8, 2, 64, 16
    pages = (T + ps - 1) // ps + 1
    K = torch.randn(pages, nkv, ps, d, generator=g).half()
    V = torch.randn(pages, nkv, ps, d, generator=g).half()
    bt = torch.randperm(pages, generator=g).int().repeat(T, 1)
    lens = torch.arange(1, T + 1, dtype=torch.int32)
    q = torch.randn(T, nq, d, generator=g)
    kw, ref_kw = {}, {}
    if window:
        kw["window"] = ref_kw["window"] = window
    if tree:
        ts = np.full(T, 30, np.int32)
        masks = np.random.default_rng(1).integers(0, 2 ** 20, size=T, dtype=np.int64) | 1
        kw.update(tree_start=ts, tree_mask=masks)
        ref_kw.update(tree_start=torch.from_numpy(ts), tree_mask=torch.from_numpy(masks))
    if sinks:
        sk = torch.randn(nq, generator=g)
        kw["sinks"], ref_kw["sinks"] = sk.numpy(), sk
    out = _native.cpu_paged_attention(q.numpy(), K.numpy(), V.numpy(), bt.numpy(), lens.numpy(),
                                      0.125, **kw)
    ref = _reference(q, K, V, bt, lens, 0.125, **ref_kw)
    ok = ~torch.isnan(ref)
    assert np.abs(out[ok.numpy()] - ref[ok].numpy()).max() < 1e-4
