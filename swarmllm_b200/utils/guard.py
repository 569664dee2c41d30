"""Canary-guarded buffers for kernel tests: the tensor handed to a kernel sits
between two 4 KiB regions filled with a byte pattern, and `check()` reports
any byte of them that changed (a write past either end of the output).

Stands in for a memory checker where none can run: together with
bit-identical reruns it catches out-of-bounds stores and order-dependent
(racy) results.
"""
from __future__ import annotations

import math

import torch

CANARY = 0xA5
PAD_BYTES = 4096   # keeps the guarded tensor 4 KiB-aligned within its allocation


class Guarded:
    def __init__(self, shape, dtype, device, fill: float | None = 0.0):
        self.shape = tuple(shape)
        esize = torch.empty((), dtype=dtype).element_size()
        n = math.prod(self.shape)
        self.raw = torch.full((2 * PAD_BYTES + n * esize,), CANARY, dtype=torch.uint8, device=device)
        self.t = self.raw[PAD_BYTES:PAD_BYTES + n * esize].view(dtype).view(self.shape)
        if fill is not None:
            self.t.fill_(fill)

    def check(self):
        """Raise if a canary byte changed; name the first such byte's offset
        from the tensor (negative: before it)."""
        nb = self.t.numel() * self.t.element_size()
        head = self.raw[:PAD_BYTES]
        tail = self.raw[PAD_BYTES + nb:]
        for name, part, base in (("before", head, -PAD_BYTES), ("after", tail, nb)):
            bad = torch.nonzero(part != CANARY)
            if bad.numel():
                off = int(bad[0]) + base
                raise AssertionError(f"write {name} the buffer: byte offset {off} "
                                     f"({int(bad.numel())} bytes changed)")
        return True
