"""Quantized linear layers on the device.

``QLinear`` holds one (possibly row-concatenated) GGML-quantized weight
``[rows, K]`` and picks the kernel:

* Q4_K, Q6_K or Q8_0 with rows % 128 == 0 and K % 256 == 0: the tcgen05
  tensor-core GEMM (``qgemm_tc.cu``; at 1..2 tokens the CUDA-core GEMV of
  ``qgemv_q4k.cu``); the GGUF blocks are repacked on the device once at load
  into the format's tiled layout (``qfmt.cuh``) and dequantized in registers.
* F16 / BF16: the dense tcgen05 GEMM.
* anything else: the CUDA-core kernel over the GGUF block layout
  (``qmatmul_simt.cu``), writing a dense fp32 result.

Both return a ``GemmResult`` that the fused epilogue kernels consume.
Row concatenation is how q|k|v and gate|up become one GEMM each: GGML rows
are independent runs of blocks, so concatenating row bytes is exact.
"""
from __future__ import annotations

import numpy as np
import torch

from ..gguf import quants as Q
from ..utils.ext import C


def stream_k_floats(max_tokens: int, rows: int, num_sms: int) -> int:
    """fp32 floats of stream-K partial slots any GEMM of <= max_tokens rows x
    `rows` outputs needs: (tiles + CTAs) x tok_tile x 128, over every token tile."""
    need = 0
    for T in sorted({1, 16, 32, 64, 128, 256, max_tokens}):
        if T > max_tokens:
            continue
        n_tok = C().q4k_tc_plan(128, 256, T, num_sms)[0]
        tiles = (rows + 127) // 128 * ((T + n_tok - 1) // n_tok)
        need = max(need, (tiles + C().q4k_plan_max_ctas(T, num_sms)) * n_tok * 128)
    return need


# Quantized types without a tensor-core kernel of their own take the
# dequantize + dense GEMM path from this many tokens on (prefill).
DEQUANT_MIN_TOKENS = 64
_DEQUANT_TYPES = (Q.Q4_0, Q.Q8_0, Q.Q4_K, Q.Q6_K, Q.IQ4_NL, Q.IQ4_XS, Q.MXFP4)
_DQ_SCRATCH: dict = {}
# GGML type -> repacked tensor-core format (qfmt.cuh) and its bytes per row per 256 K
TC_FORMATS = {Q.Q4_K: (0, 144), Q.Q6_K: (1, 224), Q.Q8_0: (2, 272)}


def _dequant_scratch(device, n: int) -> torch.Tensor:
    """fp16 scratch of at least n values per device, shared by every layer
    (grows outside CUDA-graph capture only; prefill is not captured)."""
    key = str(device)
    buf = _DQ_SCRATCH.get(key)
    if buf is None or buf.numel() < n:
        buf = _DQ_SCRATCH[key] = torch.empty(n, dtype=torch.float16, device=device)
    return buf


class GemmWorkspace:
    """Scratch shared by every GEMM of one forward: the stream-K partial
    buffer, a dense fallback buffer and the kernel status word."""

    def __init__(self, device, max_tokens: int, max_rows: int, num_sms: int | None = None,
                 extra: tuple = ()):
        """Sized for every GEMM of up to `max_tokens` rows x `max_rows`
        outputs, plus each (tokens, rows) pair in `extra` (e.g. the LM head,
        which only sees the sampled rows)."""
        self.device = torch.device(device)
        props = torch.cuda.get_device_properties(self.device)
        self.num_sms = num_sms or props.multi_processor_count
        # Stream-K slots: (tiles + CTAs) x tok_tile x 128 floats, CTAs <= num_sms.
        need = max(stream_k_floats(mt, rows, self.num_sms)
                   for mt, rows in ((max_tokens, max_rows),) + tuple(extra))
        self.ws = torch.empty(int(need), dtype=torch.float32, device=self.device)
        self._dense = torch.empty(0, dtype=torch.float32, device=self.device)
        self.status = torch.zeros(8, dtype=torch.int32, device=self.device)
        self.max_tokens = max_tokens
        self.max_rows = max_rows

    def dense(self, n: int) -> torch.Tensor:
        """fp32 scratch of at least n floats for the CUDA-core GEMM (grows
        outside CUDA-graph capture only)."""
        if self._dense.numel() < n:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("GEMM scratch must be sized before CUDA-graph capture")
            self._dense = torch.empty(n, dtype=torch.float32, device=self.device)
        return self._dense

    def check(self):
        """Raise if a kernel wait timed out (status word set on the device)."""
        s = self.status.cpu().tolist()
        if s[0]:
            raise RuntimeError(f"GPU kernel reported a timed-out wait: code {s[0]} block {s[1]} "
                               f"detail {s[2]},{s[3]} parity {s[4]} thread {s[5]}")


class QLinear:
    def __init__(self, data, qtype: int, rows: int, K: int, device, bias: np.ndarray | None = None,
                 force_simt: bool = False, f32_as_f16: bool = False):
        """`f32_as_f16`: run an F32 matrix on the fp16 tensor-core GEMM (for
        small side projections -- routers, gates -- whose precision needs are
        met by fp16 weights with fp32 accumulation)."""
        self.qtype, self.rows, self.K = qtype, rows, K
        self.device = torch.device(device)
        raw = data if isinstance(data, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(data))
        raw = raw.reshape(-1).to(self.device, dtype=torch.uint8)
        self.kind = "simt"
        self.w16 = None
        self.packed = None
        self.raw = raw
        self.fmt = -1
        if not force_simt and qtype in TC_FORMATS and rows % 128 == 0 and K % 256 == 0:
            # kind "q4k" names the repacked tensor-core path for every format
            self.kind = "q4k"
            self.fmt, row_bytes = TC_FORMATS[qtype]
            self.packed = torch.empty(rows * (K // 256) * row_bytes, dtype=torch.uint8,
                                      device=self.device)
            C().qfmt_repack(self.fmt, raw, rows, K, self.packed)
            self.raw = None
        elif not force_simt and (qtype in (Q.F16, Q.BF16) or (qtype == Q.F32 and f32_as_f16)) \
                and K % 8 == 0:
            # 16-bit weights run on the dense tensor-core GEMM in fp16 (exact
            # for F16; BF16 rounds the mantissa, kept only when no weight
            # exceeds the fp16 range).
            dt = {Q.F16: torch.float16, Q.BF16: torch.bfloat16, Q.F32: torch.float32}[qtype]
            src = raw.view(dt).view(rows, K)
            if qtype == Q.F16 or float(src.float().abs().max()) < 60000.0:
                self.kind = "dense"
                self.w16 = src.to(torch.float16).contiguous()
                self.raw = None
        self.packed_b, self.fmt_b, self.split_tile = None, -1, 0
        self.use_tc = self.kind != "simt"
        self.bias = None
        if bias is not None:
            self.bias = torch.as_tensor(bias, dtype=torch.float32, device=self.device)

    @classmethod
    def from_parts(cls, parts, K: int, device) -> "QLinear":
        """One GEMM over row-concatenated tensors [(data, qtype, rows), ...].
        Parts of one type concatenate their bytes.  A leading Q4_K run and a
        trailing Q6_K run (a Q4_K_M checkpoint's q|k|v: v is Q6_K in some
        layers) become one mixed-format GEMM when the split falls on a 128-row
        tile; any other mix is dequantized to one fp16 weight."""
        types = [p[1] for p in parts]
        rows = sum(int(p[2]) for p in parts)
        dev = torch.device(device)
        as_dev = [p[0] if isinstance(p[0], torch.Tensor) else
                  torch.from_numpy(np.ascontiguousarray(p[0])) for p in parts]
        as_dev = [t.reshape(-1).to(dev, dtype=torch.uint8) for t in as_dev]
        if all(t == types[0] for t in types):
            return cls(torch.cat(as_dev), types[0], rows, K, dev)
        na = next(i for i, t in enumerate(types) if t != types[0])
        rows_a = sum(int(p[2]) for p in parts[:na])
        if (types[0] == Q.Q4_K and all(t == Q.Q6_K for t in types[na:]) and rows_a % 128 == 0
                and rows % 128 == 0 and K % 256 == 0):
            lin = cls(torch.cat(as_dev[:na]), Q.Q4_K, rows_a, K, dev)
            lin_b = cls(torch.cat(as_dev[na:]), Q.Q6_K, rows - rows_a, K, dev)
            lin.rows, lin.packed_b, lin.fmt_b = rows, lin_b.packed, lin_b.fmt
            lin.split_tile = rows_a // 128
            lin.qtype = -1      # mixed
            return lin
        w16 = torch.empty(rows, K, dtype=torch.float16, device=dev)
        r0 = 0
        for t, (_, qt, n) in zip(as_dev, parts):
            C().dequant_f16(t, qt, int(n), K, w16[r0:r0 + int(n)])
            r0 += int(n)
        return cls(w16.view(torch.uint8).reshape(-1), Q.F16, rows, K, dev)

    @property
    def nbytes(self) -> int:
        t = {"q4k": self.packed, "dense": self.w16, "simt": self.raw}[self.kind]
        extra = self.packed_b.numel() if self.packed_b is not None else 0
        return t.numel() * t.element_size() + extra

    def __call__(self, x: torch.Tensor, ws: GemmWorkspace, out: torch.Tensor | None = None):
        """GEMM result of x [T, K] (fp16).  `out` (fp32 [T, rows]) gives the
        CUDA-core path its own output instead of the workspace's dense buffer."""
        T = x.shape[0]
        if self.kind == "q4k":
            return C().qgemm_q4k_tc(self.packed, self.rows, self.K, x, ws.ws, ws.status, ws.num_sms,
                                    self.fmt, self.packed_b, self.fmt_b, self.split_tile)
        if self.kind == "dense":
            return C().dense_gemm_tc(self.w16, x, ws.ws, ws.status, ws.num_sms)
        if (T >= DEQUANT_MIN_TOKENS and self.qtype in _DEQUANT_TYPES and self.K % 8 == 0
                and not torch.cuda.is_current_stream_capturing()):
            # prefill-sized batch: dequantize once to fp16 and run the dense
            # tensor-core GEMM (the CUDA-core kernel re-reads the blocks per 8 tokens)
            w16 = _dequant_scratch(self.device, self.rows * self.K)[: self.rows * self.K]
            C().dequant_f16(self.raw, self.qtype, self.rows, self.K, w16)
            return C().dense_gemm_tc(w16.view(self.rows, self.K), x, ws.ws, ws.status, ws.num_sms)
        if out is None:
            out = ws.dense(T * self.rows)[: T * self.rows].view(T, self.rows)
        return C().qmatmul_simt(self.raw, self.qtype, self.rows, self.K, x, out)

    def reference(self, x: torch.Tensor, ws: GemmWorkspace):
        """Same product through the CUDA-core kernel (on-device oracle)."""
        raw = self.raw
        if raw is None:
            raise ValueError("reference() needs the GGUF-layout bytes (construct with force_simt)")
        out = torch.empty(x.shape[0], self.rows, dtype=torch.float32, device=self.device)
        return C().qmatmul_simt(raw, self.qtype, self.rows, self.K, x, out)


def concat_rows(parts: list[np.ndarray]) -> np.ndarray:
    """Concatenate quantized row blocks [rows_i, row_bytes] along rows."""
    return np.concatenate([np.asarray(p, dtype=np.uint8).reshape(p.shape[0], -1) for p in parts], 0)
