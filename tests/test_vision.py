"""Vision input: the mmproj encoder and image rows spliced into prompts."""
import numpy as np
import pytest
import torch


def _img(seed, h=40, w=30):
    return np.random.default_rng(seed).integers(0, 256, (h, w, 3), dtype=np.uint8)


@pytest.mark.parametrize("projector,legacy", [("mlp", False), ("mlp", True), ("gemma3", False)])
def test_encoder_shapes_and_gguf_round_trip(tmp_path, projector, legacy):
    from swarmllm_b200.models.vision import VisionEncoder, write_random_mmproj
    p = str(tmp_path / "mm.gguf")
    write_random_mmproj(p, image_size=56, patch=14, hidden=32, heads=4, blocks=2, llm_hidden=48,
                        projector=projector, legacy_ffn=legacy)
    enc = VisionEncoder.from_gguf(p, 48)
    assert enc.ffn_swapped == legacy
    rows = enc.encode([_img(1), _img(2)])
    per = 16 if projector == "mlp" else 4        # 4x4 patches, or 2x2 squares of them
    assert rows.shape == (2 * per, 48) and enc.rows_per_image == per
    assert torch.isfinite(rows).all()
    assert not torch.allclose(rows[:per], rows[per:])   # two images, two row sets


def test_encoder_matches_plain_vit():
    """The encoder against a from-scratch restatement (CLS, pre-norm, blocks, MLP projector)."""
    import torch.nn.functional as F
    from swarmllm_b200.models.vision import VisionConfig, VisionEncoder
    rng = np.random.default_rng(0)
    H, P, S = 16, 8, 16
    t = lambda *s: rng.standard_normal(s).astype(np.float32) * 0.2
    ten = {"v.patch_embd.weight": t(H, 3, P, P), "v.class_embd": t(H), "v.position_embd.weight": t(5, H),
           "v.blk.0.ln1.weight": 1 + t(H), "v.blk.0.ln1.bias": t(H), "v.blk.0.ln2.weight": 1 + t(H),
           "v.blk.0.ln2.bias": t(H), "mm.0.weight": t(24, H), "mm.0.bias": t(24),
           "mm.2.weight": t(24, 24), "mm.2.bias": t(24)}
    for n in ("attn_q", "attn_k", "attn_v", "attn_out"):
        ten[f"v.blk.0.{n}.weight"], ten[f"v.blk.0.{n}.bias"] = t(H, H), t(H)
    ten["v.blk.0.ffn_up.weight"], ten["v.blk.0.ffn_up.bias"] = t(4 * H, H), t(4 * H)
    ten["v.blk.0.ffn_down.weight"], ten["v.blk.0.ffn_down.bias"] = t(H, 4 * H), t(H)
    enc = VisionEncoder(VisionConfig(S, P, H, 2, 1), ten, 24)
    img = _img(3, 16, 16)
    x = enc.preprocess(img)
    T = {k: torch.from_numpy(v) for k, v in ten.items()}
    h = torch.einsum("chw,dchw->d", x.unfold(1, P, P).unfold(2, P, P).permute(1, 2, 0, 3, 4)
                     .reshape(4, 3, P, P)[0], T["v.patch_embd.weight"])   # patch 0 only, as a spot check
    patches = x.unfold(1, P, P).unfold(2, P, P).permute(1, 2, 0, 3, 4).reshape(4, 3 * P * P)
    emb = patches @ T["v.patch_embd.weight"].reshape(H, -1).T
    assert torch.allclose(emb[0], h, atol=1e-5)
    z = torch.cat([T["v.class_embd"][None], emb]) + T["v.position_embd.weight"]
    def ln(v, n):
        return F.layer_norm(v, (H,), T[n + ".weight"], T[n + ".bias"], 1e-6)
    y = ln(z, "v.blk.0.ln1")
    q, k, v = (y @ T[f"v.blk.0.attn_{n}.weight"].T + T[f"v.blk.0.attn_{n}.bias"] for n in "qkv")
    q, k, v = (a.view(5, 2, 8).transpose(0, 1) for a in (q, k, v))
    a = torch.softmax(q @ k.transpose(1, 2) / np.sqrt(8), -1) @ v
    z = z + a.transpose(0, 1).reshape(5, H) @ T["v.blk.0.attn_out.weight"].T + T["v.blk.0.attn_out.bias"]
    y = ln(z, "v.blk.0.ln2")
    z = z + F.gelu(y @ T["v.blk.0.ffn_up.weight"].T + T["v.blk.0.ffn_up.bias"]) @ \
        T["v.blk.0.ffn_down.weight"].T + T["v.blk.0.ffn_down.bias"]
    ref = F.gelu(z[1:] @ T["mm.0.weight"].T + T["mm.0.bias"]) @ T["mm.2.weight"].T + T["mm.2.bias"]
    torch.testing.assert_close(enc.encode([img]), ref, rtol=1e-4, atol=1e-4)


def _engine(tmp_path, device="cpu"):
    from swarmllm_b200.engine import EngineConfig, LLMEngine
    from swarmllm_b200.models.config import tiny_llama
    from swarmllm_b200.models.vision import write_random_mmproj
    from swarmllm_b200.models.weights import RandomSource
    cfg = tiny_llama()
    p = str(tmp_path / "mm.gguf")
    write_random_mmproj(p, image_size=56, patch=14, hidden=32, heads=4, blocks=2,
                        llm_hidden=cfg.hidden)
    ec = EngineConfig(max_model_len=256, max_running=4, max_step_tokens=256, prefill_chunk=24,
                      graph_sizes=(1, 2, 4))
    eng = LLMEngine.from_config(cfg, device, ec, source=RandomSource(cfg, seed=5))
    eng.load_vision(p)
    return eng


def _gen(eng, ids, images, n=6):
    from swarmllm_b200.engine import SamplingParams
    rid = eng.add_request(ids, SamplingParams(max_tokens=n), images=images)
    out = []
    while eng.has_work():
        out += [t for r, t, _ in eng.step() if r == rid]
    eng.release(rid)
    return out


def test_engine_image_prompt(tmp_path):
    """Image rows change the output, repeat deterministically, survive chunked
    prefill (24-token chunks across the 16 image rows) and never leak through
    the prefix cache into another image's request."""
    from swarmllm_b200.models.vision import IMAGE_TOKEN
    eng = _engine(tmp_path)
    ids = [5, 6, 7, IMAGE_TOKEN, 8, 9, 10, 11, 12, 13, 14]
    a1 = _gen(eng, ids, [_img(1)])
    b1 = _gen(eng, ids, [_img(2)])
    a2 = _gen(eng, ids, [_img(1)])
    assert a1 == a2 and a1 != b1
    fresh = _engine(tmp_path)
    assert _gen(fresh, ids, [_img(2)]) == b1
    with pytest.raises(ValueError):
        _gen(eng, ids, [_img(1), _img(2)])


def test_engine_image_rows_equal_direct_embedding(tmp_path):
    """The spliced prompt equals running the model on embeddings where the
    image positions hold the encoder's rows."""
    from swarmllm_b200.models.llama import StepBatch
    from swarmllm_b200.models.vision import IMAGE_TOKEN
    from swarmllm_b200.ops.attention import PagedKVCache
    eng = _engine(tmp_path)
    img = _img(4)
    ids = [5, 6, IMAGE_TOKEN, 8, 9]
    out = _gen(eng, ids, [img], n=1)
    rows = eng.vision.encode([img])
    m = eng.model
    spliced = [5, 6] + [0] * rows.shape[0] + [8, 9]
    N = len(spliced)
    t = lambda a, dt=torch.int32: torch.as_tensor(np.asarray(a), dtype=dt)
    b = StepBatch(t(spliced), t(range(N)), t(range(N)), t(np.tile(np.arange(8), (N, 1))),
                  t(np.arange(N) + 1), t([N - 1], torch.int64), 256)
    b.embed_rows = t(range(2, 2 + rows.shape[0]))
    b.embed_vals = rows
    kv = PagedKVCache(m.cfg.n_layers, 8, m.cfg.n_kv_heads, m.cfg.head_dim, "cpu", dtype=torch.float32)
    logits = m.forward(b, kv)
    assert int(logits[0].argmax()) == out[0]


@pytest.mark.gpu
def test_gpu_engine_image_prompt_matches_cpu(tmp_path):
    from swarmllm_b200.models.vision import IMAGE_TOKEN
    ids = [5, 6, 7, IMAGE_TOKEN, 8, 9, 10]
    g = _gen(_engine(tmp_path, "cuda:0"), ids, [_img(1)], n=4)
    c = _gen(_engine(tmp_path, "cpu"), ids, [_img(1)], n=4)
    assert g[0] == c[0]


def _png(seed):
    import io

    from PIL import Image
    buf = io.BytesIO()
    Image.fromarray(_img(seed)).save(buf, format="PNG")
    return buf.getvalue()


def test_chat_api_with_image(tmp_path):
    import base64

    from fastapi.testclient import TestClient

    from swarmllm_b200.serve.api import AsyncEngine, create_app
    from swarmllm_b200.serve.tokenizer import ByteTokenizer
    eng = _engine(tmp_path)
    ae = AsyncEngine(eng)
    url = "data:image/png;base64," + base64.b64encode(_png(1)).decode()
    msg = lambda u: [{"role": "user", "content": [{"type": "text", "text": "what is this?"},
                                                   {"type": "image_url", "image_url": {"url": u}}]}]
    with TestClient(create_app(ae, ByteTokenizer(eng.cfg.vocab), "tiny", max_model_len=256)) as c:
        r = c.post("/v1/chat/completions", json={"messages": msg(url), "max_tokens": 4, "temperature": 0})
        assert r.status_code == 200, r.text
        n_text = r.json()["usage"]["prompt_tokens"]
        r0 = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "what is this?"}],
                                                  "max_tokens": 4, "temperature": 0})
        assert n_text == r0.json()["usage"]["prompt_tokens"] + 16   # + the image's 16 rows
        r = c.post("/v1/chat/completions", json={"messages": msg("http://example.com/x.png"), "max_tokens": 4})
        assert r.status_code == 400
        a = c.post("/v1/messages", json={"max_tokens": 4, "messages": [{"role": "user", "content": [
            {"type": "image", "source": {"type": "base64", "media_type": "image/png",
                                         "data": base64.b64encode(_png(2)).decode()}},
            {"type": "text", "text": "describe"}]}]})
        assert a.status_code == 200, a.text
        r = c.post("/v1/responses", json={"max_output_tokens": 4, "input": [{"role": "user", "content": [
            {"type": "input_text", "text": "hi"}, {"type": "input_image", "image_url": url}]}]})
        assert r.status_code == 200 and r.json()["status"] in ("completed", "incomplete"), r.text
    ae.shutdown()
