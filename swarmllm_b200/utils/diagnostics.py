"""Node diagnostics: software versions, GPUs (memory, SMs, and read-only NVML
clocks, power and temperature), the native extensions loaded, and -- given an
engine -- its KV cache.  Used by `GET /api/admin/diagnostics` and the CLI
`diagnostics` command.  Nothing here changes a device setting.

Reference behaviour: `swarmllm diagnostics` and the admin diagnostics view
(src/main.rs subcommands; src/api/admin.rs).
"""
from __future__ import annotations

import sys
import time


def collect(engine=None) -> dict:
    import torch
    out = {"python": sys.version.split()[0], "torch": torch.__version__,
           "cuda": torch.version.cuda, "time": time.time()}
    devs = []
    if torch.cuda.is_available():
        for i in range(torch.cuda.device_count()):
            p = torch.cuda.get_device_properties(i)
            free, total = torch.cuda.mem_get_info(i)
            d = {"index": i, "name": p.name, "sms": p.multi_processor_count,
                 "memory_total_gb": round(total / 2**30, 2), "memory_free_gb": round(free / 2**30, 2)}
            try:  # read-only NVML queries
                import pynvml
                pynvml.nvmlInit()
                h = pynvml.nvmlDeviceGetHandleByIndex(i)
                d["sm_clock_mhz"] = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                d["power_w"] = round(pynvml.nvmlDeviceGetPowerUsage(h) / 1000, 1)
                d["temperature_c"] = pynvml.nvmlDeviceGetTemperature(h, pynvml.NVML_TEMPERATURE_GPU)
            except Exception:
                pass
            devs.append(d)
    out["devices"] = devs
    mods = {}
    for name in ("swarmllm_b200._C", "swarmllm_b200._native"):
        mod = sys.modules.get(name)
        if mod is None:
            try:
                mod = __import__(name, fromlist=["_"])
            except ImportError:
                mod = None
        mods[name] = getattr(mod, "__file__", None) if mod else None
    out["native_extensions"] = mods
    if engine is not None:
        e = engine
        out["kv_cache"] = {"pages": e.bm.num_pages, "page_size": e.bm.page_size,
                           "free": e.bm.num_free(), "cached_pages": e.bm.num_cached_pages,
                           "bytes": int(e.kv.data.numel() * e.kv.data.element_size())}
        out["device"] = str(e.device)
    return out
