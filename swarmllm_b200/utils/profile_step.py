"""One eager engine step of a preset (reduced layer count) inside a
cudaProfilerStart/Stop range, for per-launch timing lists:

    ncu --profile-from-start off --metrics gpu__time_duration.sum \
        --clock-control none --csv --log-file launches.csv \
        python -m swarmllm_b200.utils.profile_step --model gpt-oss-120b-style --layers 4

--prefill profiles a prefill step of --prompt tokens instead of a decode step.
"""
import argparse, time
import numpy as np, torch
from swarmllm_b200.engine import EngineConfig, LLMEngine, SamplingParams
from swarmllm_b200.models.config import preset


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--model"); p.add_argument("--layers", type=int, default=4)
    p.add_argument("--batch", type=int, default=1); p.add_argument("--prompt", type=int, default=256)
    p.add_argument("--prefill", action="store_true", help="profile a prefill step instead")
    a = p.parse_args(argv)
    cfg = preset(a.model).scaled(n_layers=a.layers)
    dev = torch.device("cuda:0")
    ec = EngineConfig(max_model_len=a.prompt + 64, max_running=max(a.batch, 1), max_step_tokens=max(a.prompt, 64),
                      prefill_chunk=a.prompt, cuda_graphs=False)
    eng = LLMEngine.from_config(cfg, dev, ec, seed=1)
    rng = np.random.default_rng(0)
    sp = SamplingParams(max_tokens=32, ignore_eos=True)
    if a.prefill:
        for _ in range(2):
            r = eng.add_request(rng.integers(0, cfg.vocab, a.prompt).tolist(), SamplingParams(max_tokens=1, ignore_eos=True))
            eng.step(); eng.release(r)
        r = eng.add_request(rng.integers(0, cfg.vocab, a.prompt).tolist(), SamplingParams(max_tokens=1, ignore_eos=True))
        torch.cuda.synchronize(); torch.cuda.profiler.start(); t = time.perf_counter()
        eng.step(); torch.cuda.synchronize(); print("prefill ms", (time.perf_counter() - t) * 1e3)
        torch.cuda.profiler.stop()
    else:
        rids = [eng.add_request(rng.integers(0, cfg.vocab, a.prompt).tolist(), sp) for _ in range(a.batch)]
        while any(len(eng.output(r)) == 0 for r in rids):
            eng.step()
        for _ in range(3):
            eng.step()
        torch.cuda.synchronize(); torch.cuda.profiler.start(); t = time.perf_counter()
        eng.step(); torch.cuda.synchronize(); print("step ms", (time.perf_counter() - t) * 1e3)
        torch.cuda.profiler.stop()


if __name__ == "__main__":
    main()
