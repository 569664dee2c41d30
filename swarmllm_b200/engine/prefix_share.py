"""Prefix-KV snapshots: export the cached KV pages of a token prefix from one
engine and import them into another (another process, rank or node), so the
importer's next request with that prefix skips its prefill.

A snapshot holds the covered tokens (whole pages), the model's KV geometry and
the pages' K/V for every KV layer of the engine.  Import registers the pages
in the block manager's prefix cache (chained page hashes, as if a finished
request had produced them) and copies the data in; pages the importer already
caches are kept.  The byte form is a JSON header (geometry, dtype, tokens)
followed by the raw tensor, so it can go over any transport; `send_prefix` /
`recv_prefix` move it between torch.distributed ranks.

Hybrid models (linear-attention state) export nothing: their cached prefixes
also need the recurrent state saved at the prefix's end, which stays in the
engine's own state cache (engine/state_cache.py).

`save_prefix_cache` / `load_prefix_cache` persist the whole cache across
restarts: the snapshots of the engine's recent prompts in one file, stamped
with a digest of the package version, the model (name, size, weight file) and
the KV geometry.  A file whose stamp differs from the loading engine's is
discarded, since its pages would not match the new weights or layout.

Reference behaviour: KV snapshots keyed by block-hash chains and the
PrefixKvFetchReq / PrefixKvDataResp exchange between peers
(split/prefix_cache.rs:2359,2479; network/protocol/mod.rs:381-393).
"""
from __future__ import annotations

import hashlib
import json
import logging
import os
from dataclasses import dataclass

import numpy as np
import torch

_MAGIC = b"SWKV1\0"
_STORE_MAGIC = b"SWKVS1\0"
_log = logging.getLogger("swarmllm_b200.prefix")
_DTYPES = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}


@dataclass
class PrefixSnapshot:
    model: str
    tokens: list            # the covered tokens: n_pages * page_size of them
    page_size: int
    kv: torch.Tensor        # [n_kv_layers, 2, n_pages, n_kv, page_size, head_dim] (host)

    @property
    def n_pages(self) -> int:
        return int(self.kv.shape[2])

    def to_bytes(self) -> bytes:
        t = self.kv.contiguous()
        head = json.dumps({"model": self.model, "tokens": [int(x) for x in self.tokens],
                           "page_size": self.page_size, "shape": list(t.shape),
                           "dtype": str(t.dtype).replace("torch.", "")}).encode()
        raw = t.view(torch.uint8).numpy().tobytes()
        return _MAGIC + len(head).to_bytes(8, "little") + head + raw

    @classmethod
    def from_bytes(cls, b: bytes) -> "PrefixSnapshot":
        if not b.startswith(_MAGIC):
            raise ValueError("not a prefix snapshot")
        n = int.from_bytes(b[len(_MAGIC):len(_MAGIC) + 8], "little")
        o = len(_MAGIC) + 8
        h = json.loads(b[o:o + n].decode())
        dt = _DTYPES[h["dtype"]]
        arr = np.frombuffer(b[o + n:], dtype=np.uint8).copy()
        kv = torch.from_numpy(arr).view(dt).view(*h["shape"])
        return cls(h["model"], h["tokens"], h["page_size"], kv)


def export_prefix(engine, tokens) -> PrefixSnapshot | None:
    """Snapshot of the longest cached run of full pages of `tokens` (None if
    nothing is cached or the engine keeps no prefix cache)."""
    if not engine.ecfg.prefix_cache or getattr(engine, "state_cache", None) is not None:
        return None
    pages = np.asarray(engine.bm.cached_prefix_pages([int(x) for x in tokens]), dtype=np.int64)
    if len(pages) == 0:
        return None
    ps = engine.bm.page_size
    idx = torch.as_tensor(pages, device=engine.kv.data.device)
    kv = engine.kv.data.index_select(2, idx).to("cpu")
    return PrefixSnapshot(engine.cfg.name, [int(x) for x in tokens[: len(pages) * ps]], ps, kv)


def import_prefix(engine, snap: PrefixSnapshot) -> int:
    """Register the snapshot's pages in this engine's prefix cache; returns
    the number of tokens whose pages were newly imported."""
    if not engine.ecfg.prefix_cache or getattr(engine, "state_cache", None) is not None:
        raise RuntimeError("this engine keeps no importable prefix cache")
    d = engine.kv.data
    want = (d.shape[0], 2, snap.n_pages, d.shape[3], d.shape[4], d.shape[5])
    if snap.page_size != engine.bm.page_size or tuple(snap.kv.shape) != want:
        raise ValueError(f"snapshot geometry {tuple(snap.kv.shape)} does not fit this engine's "
                         f"KV cache {want}")
    if snap.model != engine.cfg.name:
        raise ValueError(f"snapshot of model {snap.model!r}, engine serves {engine.cfg.name!r}")
    dst = np.asarray(engine.bm.import_prefix_pages([int(x) for x in snap.tokens], snap.n_pages),
                     dtype=np.int64)
    src = np.nonzero(dst >= 0)[0]
    if len(src) == 0:
        return 0
    data = snap.kv.index_select(2, torch.as_tensor(src, dtype=torch.int64)).to(d.device, d.dtype)
    d.index_copy_(2, torch.as_tensor(dst[src], dtype=torch.int64, device=d.device), data)
    return int(len(src)) * snap.page_size


def send_prefix(snap: PrefixSnapshot | None, dst: int, group=None):
    """Send a snapshot (or "none") to rank `dst` (CPU tensors: gloo, or NCCL
    with CUDA tensors on both sides)."""
    import torch.distributed as dist
    b = snap.to_bytes() if snap is not None else b""
    dev = torch.device("cpu") if dist.get_backend(group) == "gloo" else torch.device("cuda")
    n = torch.tensor([len(b)], dtype=torch.int64, device=dev)
    dist.send(n, dst, group=group)
    if b:
        dist.send(torch.frombuffer(bytearray(b), dtype=torch.uint8).to(dev), dst, group=group)


def recv_prefix(src: int, group=None) -> PrefixSnapshot | None:
    import torch.distributed as dist
    dev = torch.device("cpu") if dist.get_backend(group) == "gloo" else torch.device("cuda")
    n = torch.zeros(1, dtype=torch.int64, device=dev)
    dist.recv(n, src, group=group)
    if int(n) == 0:
        return None
    buf = torch.empty(int(n), dtype=torch.uint8, device=dev)
    dist.recv(buf, src, group=group)
    return PrefixSnapshot.from_bytes(buf.cpu().numpy().tobytes())


# --------------------------------------------------------------------------- persistence
def build_stamp(engine) -> str:
    """Digest of what the cached KV depends on: package version, model
    identity (name, parameter count, weight file size and mtime) and the KV
    cache geometry and dtype."""
    from .. import __version__
    src = getattr(engine, "source_path", None)
    st = os.stat(src) if src and os.path.exists(src) else None
    d = engine.kv.data
    ident = {"v": __version__, "model": engine.cfg.name, "params": engine.cfg.param_count(),
             "source": os.path.abspath(src) if src else None,
             "size": st.st_size if st else None, "mtime": int(st.st_mtime) if st else None,
             "page": engine.bm.page_size, "kv": [int(x) for x in d.shape[:1] + d.shape[3:]],
             "dtype": str(d.dtype)}
    return hashlib.sha256(json.dumps(ident, sort_keys=True).encode()).hexdigest()[:32]


def _covering(prompts) -> list:
    """Drop prompts that are a prefix of another one (their pages are inside it)."""
    ps = sorted((tuple(int(x) for x in p) for p in prompts), key=len, reverse=True)
    out: list = []
    for p in ps:
        if not any(q[: len(p)] == p for q in out):
            out.append(p)
    return out


def save_prefix_cache(engine, path: str) -> int:
    """Write the cached prefixes of the engine's recent prompts to `path`
    (atomically); returns the number of tokens saved."""
    snaps = []
    for p in _covering(engine.recent_prompts()):
        s = export_prefix(engine, list(p))
        if s is not None:
            snaps.append(s.to_bytes())
    head = json.dumps({"stamp": build_stamp(engine), "sizes": [len(b) for b in snaps]}).encode()
    tmp = f"{path}.tmp"
    with open(tmp, "wb") as f:
        f.write(_STORE_MAGIC + len(head).to_bytes(8, "little") + head)
        for b in snaps:
            f.write(b)
    os.replace(tmp, path)
    return sum(PrefixSnapshot.from_bytes(b).n_pages for b in snaps) * engine.bm.page_size


def load_prefix_cache(engine, path: str) -> int:
    """Import a file written by save_prefix_cache; returns the tokens newly
    cached.  A missing file, a file of another build or model (stamp
    mismatch) or an unreadable one loads nothing."""
    if not os.path.exists(path):
        return 0
    with open(path, "rb") as f:
        b = f.read()
    if not b.startswith(_STORE_MAGIC):
        _log.warning("%s is not a prefix-cache file; ignored", path)
        return 0
    o = len(_STORE_MAGIC)
    n = int.from_bytes(b[o:o + 8], "little")
    head = json.loads(b[o + 8:o + 8 + n].decode())
    if head.get("stamp") != build_stamp(engine):
        _log.warning("%s was written by another build or model; discarded", path)
        return 0
    o += 8 + n
    total = 0
    for sz in head["sizes"]:
        total += import_prefix(engine, PrefixSnapshot.from_bytes(b[o:o + sz]))
        o += sz
    return total
