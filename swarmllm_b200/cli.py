"""Command line: ``python -m swarmllm_b200 <command>``.

  serve     OpenAI/Anthropic-compatible HTTP server on :8800 (reference: `swarmllm run`)
  generate  one-shot generation from token ids or text
  bench     single-GPU tokens/s over a preset (reference: `swarmllm bench`)
  info      model / GGUF summary
  shard     split a GGUF into the sharded checkpoint layout
  make-gguf write a random-init GGUF of a preset (test models)

Models: `--model <preset name>` (random-init weights of that architecture) or
`--gguf <file or shard dir>`.  Config overrides come from `--config file.toml`
and SWARMLLM_* environment variables (see utils/config.py).
"""
from __future__ import annotations

import argparse
import json
import sys
import time


def _engine(args):
    import torch

    from .engine import LLMEngine
    from .models.config import preset
    from .utils.config import load_engine_config
    ecfg = load_engine_config(args.config)
    if args.max_model_len:
        ecfg.max_model_len = args.max_model_len
    dev = args.device or ("cuda:0" if torch.cuda.is_available() else "cpu")
    if args.gguf:
        return LLMEngine.from_gguf(args.gguf, dev, ecfg)
    return LLMEngine.from_config(preset(args.model), dev, ecfg, seed=args.seed)


def _tokenizer(args, eng):
    from .serve.tokenizer import ByteTokenizer, from_gguf_metadata
    if args.gguf:
        from .gguf.file import GGUFReader
        import os
        md = GGUFReader(args.gguf).metadata if not os.path.isdir(args.gguf) else {}
        return from_gguf_metadata(md, eng.cfg.vocab), md.get("tokenizer.chat_template")
    return ByteTokenizer(eng.cfg.vocab), None


def main(argv=None):
    p = argparse.ArgumentParser(prog="swarmllm_b200")
    sub = p.add_subparsers(dest="cmd", required=True)
    for name in ("serve", "generate", "bench", "info"):
        s = sub.add_parser(name)
        s.add_argument("--model", default="llama-3.2-3b")
        s.add_argument("--gguf", default=None)
        s.add_argument("--device", default=None)
        s.add_argument("--config", default=None)
        s.add_argument("--seed", type=int, default=0)
        s.add_argument("--max-model-len", type=int, default=0)
        if name == "serve":
            s.add_argument("--host", default="0.0.0.0")
            s.add_argument("--port", type=int, default=8800)
        if name == "generate":
            s.add_argument("--prompt", default="Hello")
            s.add_argument("--ids", default=None, help="comma-separated token ids")
            s.add_argument("--max-tokens", type=int, default=32)
            s.add_argument("--temperature", type=float, default=0.0)
        if name == "bench":
            s.add_argument("--batch", type=int, default=8)
            s.add_argument("--prompt-len", type=int, default=512)
            s.add_argument("--gen", type=int, default=64)
    s = sub.add_parser("shard")
    s.add_argument("gguf")
    s.add_argument("out_dir")
    s.add_argument("--layers-per-shard", type=int, default=4)
    s = sub.add_parser("make-gguf")
    s.add_argument("--model", default="tiny-llama")
    s.add_argument("out")
    s.add_argument("--seed", type=int, default=0)
    args = p.parse_args(argv)

    if args.cmd == "shard":
        from .gguf.file import write_sharded
        m = write_sharded(args.gguf, args.out_dir, args.layers_per_shard)
        print(json.dumps({"shards": len(m["shards"])}))
        return
    if args.cmd == "make-gguf":
        from .models.config import preset
        from .models.weights import write_random_gguf
        write_random_gguf(preset(args.model), args.out, args.seed)
        print(args.out)
        return
    eng = _engine(args)
    if args.cmd == "info":
        print(json.dumps({"config": eng.cfg.to_dict(), "kv_pages": eng.bm.num_pages,
                          "params": eng.cfg.param_count()}, indent=1))
        return
    if args.cmd == "serve":
        from .serve.api import serve
        tok, tpl = _tokenizer(args, eng)
        serve(eng, tok, eng.cfg.name, args.host, args.port, arch=eng.cfg.arch, chat_template=tpl,
              max_model_len=eng.ecfg.max_model_len)
        return
    from .engine.sampling import SamplingParams
    if args.cmd == "generate":
        tok, _ = _tokenizer(args, eng)
        ids = [int(x) for x in args.ids.split(",")] if args.ids else tok.encode(args.prompt)
        out = eng.generate([ids], SamplingParams(max_tokens=args.max_tokens,
                                                 temperature=args.temperature))[0]
        print(json.dumps({"token_ids": out.token_ids, "text": tok.decode(out.token_ids),
                          "ttft_ms": out.trace.ttft * 1e3 if out.trace and out.trace.ttft else None}))
        return
    if args.cmd == "bench":
        import numpy as np
        rng = np.random.default_rng(0)
        prompts = [rng.integers(0, eng.cfg.vocab, args.prompt_len).tolist() for _ in range(args.batch)]
        t = time.perf_counter()
        outs = eng.generate(prompts, SamplingParams(max_tokens=args.gen, ignore_eos=True))
        dt = time.perf_counter() - t
        ntok = sum(len(o.token_ids) for o in outs)
        ttft = sorted(o.trace.ttft for o in outs if o.trace and o.trace.ttft)
        print(json.dumps({"tokens": ntok, "seconds": round(dt, 3), "tok_s": round(ntok / dt, 2),
                          "ttft_p50_ms": round(ttft[len(ttft) // 2] * 1e3, 2) if ttft else None}))


if __name__ == "__main__":
    main(sys.argv[1:])
