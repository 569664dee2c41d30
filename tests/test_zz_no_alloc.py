"""The allocation-free Q4_K GEMM entry point, called through its exported C
symbol, against the regular entry point.

The allocation-free entry point serves callers that may not allocate device
memory themselves (host frameworks that own all device memory, plug-ins
limited to the buffers they are handed); it keeps its scratch in a fixed
static device array.  This file is named so pytest collects it last, and it
must pass both alone in a fresh process and after the other tests.
"""
import ctypes
import glob
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _lib():
    import swarmllm_b200
    from swarmllm_b200.utils.ext import C
    C()  # loads the extension (and torch's libraries it links against) the usual way
    root = os.path.dirname(swarmllm_b200.__file__)
    so = sorted(glob.glob(os.path.join(root, "_C*.so")))
    assert so, "swarmllm_b200._C is not built"
    lib = ctypes.CDLL(so[0])  # same handle as the imported module: dlopen reuses it
    f = lib.swarm_q4k_gemm_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                  ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
    lib.swarm_q4k_gemm_noalloc_error.restype = ctypes.c_char_p
    lib.swarm_q4k_gemm_noalloc_error.argtypes = [ctypes.c_int]
    lib.swarm_q4k_gemm_noalloc_scratch_need.restype = ctypes.c_longlong
    lib.swarm_q4k_gemm_noalloc_scratch_need.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int]
    lib.swarm_q4k_gemm_noalloc_status.restype = ctypes.c_int
    lib.swarm_q4k_gemm_noalloc_status.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    return lib


def _status(lib, stream):
    """The status word of the last call (waits for the stream); 0 = output valid."""
    st = (ctypes.c_int * 8)()
    rc = lib.swarm_q4k_gemm_noalloc_status(ctypes.addressof(st), stream)
    return rc, list(st)


def _rel_err(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / (b.norm() + 1e-30))


def _regular(lin, ws, x):
    """The existing path: tensor-core GEMM into the workspace + logits-copy epilogue."""
    from swarmllm_b200.utils.ext import C
    g = lin(x, ws)
    out = torch.empty(x.shape[0], lin.rows, dtype=torch.float32, device=DEV)
    C().epi_copy(g, None, out)
    return out


# T = 1 and 2 take the CUDA-core GEMV branch of the entry point, 7 and 32 the
# tensor-core GEMM; both share the static partial sums and status word.
@pytest.mark.parametrize("rows,K,Ts", [(1024, 4096, (7, 32)), (512, 28672, (7, 32)),
                                       (1024, 4096, (1, 2)), (640, 8192, (2, 1))])
def test_noalloc_matches_regular_entry_point_twice(rows, K, Ts):
    from swarmllm_b200.gguf import quants as Q
    from swarmllm_b200.ops.linear import GemmWorkspace, QLinear
    torch.cuda.set_device(0)
    lib = _lib()
    rng = np.random.default_rng(rows + K + Ts[0])
    b = Q.quantize(rng.standard_normal((rows, K), dtype=np.float32) * 0.02, Q.Q4_K)
    lin = QLinear(b, Q.Q4_K, rows, K, DEV)
    ws = GemmWorkspace(DEV, 32, rows)
    stream = torch.cuda.current_stream().cuda_stream
    wd = torch.from_numpy(Q.dequantize(b, Q.Q4_K))
    for call, T in enumerate(Ts):  # two calls in a row with different inputs
        g = torch.Generator().manual_seed(100 + call)
        # the second call reads a row-strided input and writes a row-strided output
        xs, os_ = (K, rows) if call == 0 else (K + 64, rows + 32)
        xbuf = torch.randn(T, xs, generator=g).half().to(DEV)
        x = xbuf[:, :K]
        obuf = torch.full((T, os_), float("nan"), dtype=torch.float32, device=DEV)
        rc = lib.swarm_q4k_gemm_noalloc(lin.packed.data_ptr(), rows, K, xbuf.data_ptr(), xs, T,
                                        obuf.data_ptr(), os_, stream)
        assert rc == 0, lib.swarm_q4k_gemm_noalloc_error(rc).decode()
        rc, st = _status(lib, stream)
        assert rc == 0 and st[0] == 0, (rc, st)
        out = obuf[:, :rows]
        assert torch.isnan(obuf[:, rows:]).all()  # nothing written past each output row
        ref = _regular(lin, ws, x.contiguous())
        torch.cuda.synchronize()
        assert torch.isfinite(out).all()
        assert _rel_err(out.cpu(), ref.cpu()) < 3e-3, (call, T)
        # and against the dequantized fp32 product (1..2 tokens: the GEMV's
        # int8 activations add ~0.5 % relative error)
        tol = 1.2e-2 if T <= 2 else 3e-3
        assert _rel_err(out.cpu(), x.cpu().float() @ wd.T) < tol, (call, T)


def test_noalloc_rejects_oversized_problem():
    torch.cuda.set_device(0)
    lib = _lib()
    rows, K, T = 128256, 8192, 128   # partial sums far beyond the 16 MiB scratch
    need = lib.swarm_q4k_gemm_noalloc_scratch_need(rows, K, T)
    assert need > 16 * 1024 * 1024
    x = torch.zeros(T, K, dtype=torch.float16, device=DEV)
    out = torch.zeros(1, dtype=torch.float32, device=DEV)
    rc = lib.swarm_q4k_gemm_noalloc(ctypes.c_void_p(16), rows, K, x.data_ptr(), K, T,
                                    out.data_ptr(), rows, torch.cuda.current_stream().cuda_stream)
    assert rc == -10
    assert b"too large" in lib.swarm_q4k_gemm_noalloc_error(rc)
    assert lib.swarm_q4k_gemm_noalloc(ctypes.c_void_p(16), 100, K, x.data_ptr(), K, T,
                                      out.data_ptr(), rows, None) == -11
