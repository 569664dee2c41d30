"""GGUF reading (native mmap reader) and writing (Python), plus the
reference's sharded checkpoint layout.

Writer: GGUF v3 (little-endian; strings are u64 length + bytes; metadata
values are typed; tensor data aligned to ``general.alignment``, 32 here).

Shard layout (reference ``src/model/shard.rs:65-73``,
``src/inference/shard_layout.rs:10-50``): a GGUF is split into
``gguf_header.bin`` (everything before the data section), layer-aligned
``shard_NNN.bin`` files holding tensor bytes, and ``manifest.json`` listing
each shard's tensors and a checksum.  ``ShardedGguf`` presents such a
directory as one virtual GGUF.  The checksum here is SHA-256 (the reference
uses BLAKE3, which is not available in this environment); the field is named
by algorithm so either can be verified.
"""
from __future__ import annotations

import hashlib
import json
import os
import struct
from dataclasses import dataclass
from typing import Any

import numpy as np

from . import quants as Q

GGUF_MAGIC = 0x46554747
ALIGN = 32

# metadata value types
U8, I8, U16, I16, U32, I32, F32T, BOOL, STR, ARR, U64, I64, F64T = range(13)


@dataclass
class TensorInfo:
    name: str
    shape: tuple  # numpy order (outer ... inner); GGUF dims are reversed
    qtype: int
    offset: int
    nbytes: int


class GGUFWriter:
    """Collect metadata + tensors, then ``write(path)``."""

    def __init__(self, arch: str):
        self.kv: list[tuple[str, int, Any, int]] = []
        self.tensors: list[tuple[str, tuple, int, np.ndarray]] = []
        self.add("general.architecture", arch)
        self.add("general.alignment", ALIGN, U32)

    def add(self, key: str, value: Any, vtype: int | None = None, elem_type: int | None = None):
        if vtype is None:
            if isinstance(value, bool):
                vtype = BOOL
            elif isinstance(value, int):
                vtype = U32 if 0 <= value < 2**32 else I64
            elif isinstance(value, float):
                vtype = F32T
            elif isinstance(value, str):
                vtype = STR
            elif isinstance(value, (list, tuple)):
                vtype = ARR
            else:
                raise TypeError(f"cannot infer GGUF type for {key}")
        if vtype == ARR and elem_type is None:
            v0 = value[0] if len(value) else 0
            elem_type = STR if isinstance(v0, str) else (F32T if isinstance(v0, float) else I32)
        self.kv = [kv for kv in self.kv if kv[0] != key]
        self.kv.append((key, vtype, value, elem_type or 0))

    def add_tensor(self, name: str, data: np.ndarray, qtype: int, shape: tuple):
        """`data`: uint8 block bytes (or raw float array for F32/F16); `shape` in
        numpy order [outer..., inner] of the logical tensor."""
        raw = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
        n = int(np.prod(shape))
        assert raw.size == Q.nbytes(qtype, n), (name, raw.size, Q.nbytes(qtype, n))
        self.tensors.append((name, tuple(int(s) for s in shape), qtype, raw))

    @staticmethod
    def _pack_str(s: str) -> bytes:
        b = s.encode("utf-8")
        return struct.pack("<Q", len(b)) + b

    def _pack_val(self, vtype: int, v: Any, elem_type: int = 0) -> bytes:
        fmt = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32T: "<f",
               U64: "<Q", I64: "<q", F64T: "<d"}
        if vtype in fmt:
            return struct.pack(fmt[vtype], v)
        if vtype == BOOL:
            return struct.pack("<B", 1 if v else 0)
        if vtype == STR:
            return self._pack_str(v)
        if vtype == ARR:
            out = struct.pack("<IQ", elem_type, len(v))
            if elem_type in fmt:
                return out + np.asarray(v, dtype=np.dtype(fmt[elem_type][1:]).newbyteorder("<")).tobytes()
            return out + b"".join(self._pack_val(elem_type, e) for e in v)
        raise TypeError(vtype)

    def header_bytes(self) -> tuple[bytes, list[TensorInfo]]:
        out = [struct.pack("<IIQQ", GGUF_MAGIC, 3, len(self.tensors), len(self.kv))]
        for key, vt, v, et in self.kv:
            out.append(self._pack_str(key) + struct.pack("<I", vt) + self._pack_val(vt, v, et))
        infos, off = [], 0
        for name, shape, qt, raw in self.tensors:
            dims = list(reversed(shape))
            out.append(self._pack_str(name) + struct.pack("<I", len(dims)) +
                       struct.pack(f"<{len(dims)}Q", *dims) + struct.pack("<IQ", qt, off))
            infos.append(TensorInfo(name, shape, qt, off, raw.size))
            off += (raw.size + ALIGN - 1) // ALIGN * ALIGN
        head = b"".join(out)
        pad = (-len(head)) % ALIGN
        return head + b"\0" * pad, infos

    def write(self, path: str):
        head, infos = self.header_bytes()
        with open(path, "wb") as f:
            f.write(head)
            for (_, _, _, raw), ti in zip(self.tensors, infos):
                f.write(raw.tobytes())
                f.write(b"\0" * ((-raw.size) % ALIGN))


class GGUFReader:
    """Read-only GGUF view: metadata dict and zero-copy tensor bytes (mmap)."""

    def __init__(self, path: str):
        from .. import _native
        self.path = path
        self._f = _native.GgufFile(path)
        self.metadata: dict = self._f.metadata()
        self.tensors: dict[str, TensorInfo] = {}
        for name, dims, qt, off, nb in self._f.tensors():
            self.tensors[name] = TensorInfo(name, tuple(reversed(dims)), qt, off, nb)

    def get(self, key: str, default=None):
        return self.metadata.get(key, default)

    def tensor_bytes(self, name: str) -> np.ndarray:
        return self._f.tensor_bytes(name)

    def tensor_float(self, name: str) -> np.ndarray:
        ti = self.tensors[name]
        return Q.dequantize(self.tensor_bytes(name), ti.qtype).reshape(ti.shape)


# --------------------------------------------------------------------------- shards
def _layer_of(name: str) -> int:
    parts = name.split(".")
    if len(parts) > 1 and parts[0] == "blk" and parts[1].isdigit():
        return int(parts[1])
    return -1


def write_sharded(src_path: str, out_dir: str, layers_per_shard: int = 4) -> dict:
    """Split a GGUF into gguf_header.bin + layer-aligned shard_NNN.bin + manifest.json."""
    r = GGUFReader(src_path)
    os.makedirs(out_dir, exist_ok=True)
    with open(src_path, "rb") as f:
        header = f.read(r._f.data_offset)
    with open(os.path.join(out_dir, "gguf_header.bin"), "wb") as f:
        f.write(header)
    groups: dict[int, list[str]] = {}
    for name in r.tensors:
        lay = _layer_of(name)
        key = -1 if lay < 0 else lay // layers_per_shard
        groups.setdefault(key, []).append(name)
    manifest = {"source": os.path.basename(src_path), "data_offset": r._f.data_offset,
                "checksum": "sha256", "shards": []}
    for i, key in enumerate(sorted(groups)):
        fname = f"shard_{i:03d}.bin"
        h = hashlib.sha256()
        entries, pos = [], 0
        with open(os.path.join(out_dir, fname), "wb") as f:
            for name in groups[key]:
                b = r.tensor_bytes(name).tobytes()
                f.write(b)
                h.update(b)
                entries.append({"name": name, "offset": r.tensors[name].offset,
                                "shard_offset": pos, "nbytes": len(b)})
                pos += len(b)
        layers = sorted({_layer_of(n) for n in groups[key] if _layer_of(n) >= 0})
        manifest["shards"].append({"file": fname, "sha256": h.hexdigest(), "tensors": entries,
                                   "layers": [layers[0], layers[-1]] if layers else []})
    with open(os.path.join(out_dir, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1)
    return manifest


class ShardedGguf:
    """A shard directory presented as one GGUF (metadata from the header file,
    tensor bytes from the shard files, each shard verified once on open)."""

    def __init__(self, shard_dir: str, verify: bool = True, layers: tuple[int, int] | None = None):
        self.dir = shard_dir
        with open(os.path.join(shard_dir, "manifest.json")) as f:
            self.manifest = json.load(f)
        # Parse the header by appending nothing: the native reader needs a whole
        # file, so a header-only view is read with tensor bounds unchecked.
        self.metadata, self.tensors = _parse_header_only(os.path.join(shard_dir, "gguf_header.bin"))
        self._where: dict[str, tuple[str, int, int]] = {}
        for sh in self.manifest["shards"]:
            if layers is not None and sh["layers"]:
                lo, hi = sh["layers"]
                if hi < layers[0] or lo > layers[1]:
                    continue
            path = os.path.join(shard_dir, sh["file"])
            if verify:
                h = hashlib.sha256()
                with open(path, "rb") as f:
                    for chunk in iter(lambda: f.read(1 << 24), b""):
                        h.update(chunk)
                if h.hexdigest() != sh["sha256"]:
                    raise IOError(f"shard {sh['file']} failed its checksum")
            for e in sh["tensors"]:
                self._where[e["name"]] = (path, e["shard_offset"], e["nbytes"])

    def get(self, key: str, default=None):
        return self.metadata.get(key, default)

    def tensor_bytes(self, name: str) -> np.ndarray:
        path, off, nb = self._where[name]
        return np.fromfile(path, dtype=np.uint8, count=nb, offset=off)

    def tensor_float(self, name: str) -> np.ndarray:
        ti = self.tensors[name]
        return Q.dequantize(self.tensor_bytes(name), ti.qtype).reshape(ti.shape)


def _parse_header_only(path: str) -> tuple[dict, dict[str, TensorInfo]]:
    """Pure-Python GGUF header parser (metadata + tensor table, no data)."""
    with open(path, "rb") as f:
        buf = f.read()
    pos = 0

    def rd(fmt):
        nonlocal pos
        v = struct.unpack_from(fmt, buf, pos)
        pos += struct.calcsize(fmt)
        return v[0]

    def rstr():
        n = rd("<Q")
        nonlocal pos
        s = buf[pos:pos + n].decode("utf-8", "replace")
        pos += n
        return s

    fmts = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32T: "<f",
            U64: "<Q", I64: "<q", F64T: "<d"}

    def rval(t):
        if t in fmts:
            return rd(fmts[t])
        if t == BOOL:
            return bool(rd("<B"))
        if t == STR:
            return rstr()
        if t == ARR:
            et, n = rd("<I"), rd("<Q")
            return [rval(et) for _ in range(n)]
        raise ValueError(t)

    assert rd("<I") == GGUF_MAGIC
    rd("<I")
    nt, nkv = rd("<Q"), rd("<Q")
    meta = {}
    for _ in range(nkv):
        k = rstr()
        meta[k] = rval(rd("<I"))
    tensors = {}
    for _ in range(nt):
        name = rstr()
        nd = rd("<I")
        dims = [rd("<Q") for _ in range(nd)]
        qt, off = rd("<I"), rd("<Q")
        shape = tuple(reversed(dims))
        tensors[name] = TensorInfo(name, shape, qt, off, Q.nbytes(qt, int(np.prod(shape))))
    return meta, tensors
