"""Device-side bounded waits run out cleanly (one GPU, no fault, no hang).

Every cross-GPU wait in the kernels spins on a flag with a deadline; when the
deadline passes the kernel records an error code in a status word and
returns, so the context stays usable and the host can read what happened.
These tests make the waits run out on flags that nothing sets, with a 10 ms
deadline passed as a kernel argument, and check the status and that the
stream goes on working.  The tensor-parallel reduce kernel is also checked
numerically on a one-rank group against an fp32 reference."""
import socket
import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
TIMEOUT_NS = 10_000_000  # 10 ms


def test_flag_wait_times_out_and_stream_continues():
    from swarmllm_b200.utils.ext import C
    torch.cuda.set_device(0)
    flags = torch.zeros(4, dtype=torch.int32, device=DEV)   # nothing ever raises them
    ctl = torch.zeros(16, dtype=torch.int32, device=DEV)
    status = torch.zeros(8, dtype=torch.int32, device=DEV)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    C().flag_wait(flags.data_ptr(), 4, ctl, 2, status, 77, TIMEOUT_NS)
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    st = status.cpu().tolist()
    assert st[0] == 77, st                  # the wait gave up and said so
    assert 0.005 < dt < 0.5, dt             # after about the deadline, not the 1 s default
    # the stream and the context are still usable
    y = torch.arange(10, device=DEV, dtype=torch.float32).sum()
    assert float(y) == 45.0
    # a wait that gave up still consumed its epoch (every rank counts waits in
    # lockstep): the next wait passes once the flags reach epoch 2
    status.zero_()
    flags.fill_(2)
    C().flag_wait(flags.data_ptr(), 4, ctl, 2, status, 77, TIMEOUT_NS)
    torch.cuda.synchronize()
    assert status.cpu().tolist()[0] == 0


def _one_rank_group():
    import torch.distributed as dist
    if dist.is_initialized():
        return False
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1)
    return True


@pytest.mark.parametrize("one_hop", [False, True])
def test_tp_reduce_numerics_and_timeout_one_rank(one_hop):
    """Both reduce paths: the reduce-scatter + all-gather slices
    (tp_reduce_norm) and the one-hop local sum (tp_local_norm)."""
    import torch.distributed as dist
    from swarmllm_b200.gguf import quants as Q
    from swarmllm_b200.ops.linear import GemmWorkspace, QLinear, stream_k_floats
    from swarmllm_b200.parallel.tp import TpGroup
    torch.cuda.set_device(0)
    created = _one_rank_group()
    try:
        H, K, T = 1024, 512, 24
        rng = np.random.default_rng(3)
        wq = Q.quantize(rng.standard_normal((H, K), dtype=np.float32) * 0.05, Q.Q4_K)
        lin = QLinear(wq, Q.Q4_K, H, K, DEV)
        ws = GemmWorkspace(DEV, T, H)
        tp = TpGroup(0, 1, DEV, timeout_ns=TIMEOUT_NS)
        tp.LOCAL_ROWS = 10 ** 6 if one_hop else -1
        assert tp.local(T) == one_hop
        tp.setup(stream_k_floats(T, H, ws.num_sms), T, H)
        h = tp.h_view()
        h0 = torch.randn(T, H, device=DEV)
        h[:T].copy_(h0)
        x = torch.randn(T, K, device=DEV).half()
        bias = torch.randn(H, device=DEV) * 0.1
        nw = torch.rand(H, device=DEV) + 0.5
        out = torch.zeros(T, H, dtype=torch.float16, device=DEV)
        status = ws.status
        status.zero_()
        tp.begin_forward()
        g = tp.row_parallel(lin, x, status, ws.num_sms)
        tp.reduce_norm(g, bias, nw, out, 1e-5, status, ws.num_sms)
        torch.cuda.synchronize()
        assert status.cpu().tolist()[0] == 0
        wd = torch.from_numpy(Q.dequantize(wq, Q.Q4_K)).to(DEV)
        hr = h0 + x.float() @ wd.T + bias
        ref = hr * torch.rsqrt(hr.pow(2).mean(-1, keepdim=True) + 1e-5) * nw
        rel = float((out.float() - ref).norm() / ref.norm())
        assert rel < 2e-3, rel
        # Run the reduce of the same parity again: the GEMM-done epoch it now
        # waits for is never raised (no GEMM ran), so it must give up.
        tp.begin_forward()
        t0 = time.perf_counter()
        tp.reduce_norm(g, bias, nw, out, 1e-5, status, ws.num_sms)
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        st = status.cpu().tolist()
        assert st[0] == TpGroup.CODE_REDUCE, st
        assert dt < 0.5, dt
        assert float(torch.ones(4, device=DEV).sum()) == 4.0   # context still usable
        tp.close()
    finally:
        if created:
            dist.destroy_process_group()
