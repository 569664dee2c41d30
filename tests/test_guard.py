"""Canary-guarded buffers (CPU check of the helper itself)."""
import pytest
import torch


def test_guard_detects_writes_past_either_end():
    from swarmllm_b200.utils.guard import Guarded
    g = Guarded((3, 5), torch.float16, "cpu")
    g.t.fill_(1.0)
    assert g.check()
    g.raw[4096 + 30] = 0          # first byte after the 30-byte tensor
    with pytest.raises(AssertionError, match="after the buffer: byte offset 30"):
        g.check()
    g = Guarded((8,), torch.float32, "cpu")
    g.raw[4095] = 1               # last byte before it
    with pytest.raises(AssertionError, match="before the buffer: byte offset -1"):
        g.check()
