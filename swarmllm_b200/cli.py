"""Command line: ``python -m swarmllm_b200 <command>``.

  serve     OpenAI/Anthropic/Responses/MCP HTTP server on :8800 (reference: `swarmllm run`)
  generate  one-shot generation from token ids or text
  bench     single-GPU tokens/s over a preset (reference: `swarmllm bench`)
  chat      interactive chat with a local model (reference: `swarmllm chat`)
  info      model / GGUF summary
  status    a running node's status and readiness (reference: `swarmllm status`)
  diagnostics  GPUs, NVML readings (read-only), native extensions, versions
  test-split   the tiny Llama split over 2 CPU processes vs one (reference: `swarmllm test-split`)
  shard     split a GGUF into the sharded checkpoint layout
  make-gguf write a random-init GGUF of a preset (test models)

Models: `--model <preset name>` (random-init weights of that architecture) or
`--gguf <file or shard dir>`.  Config overrides come from `--config file.toml`
and SWARMLLM_* environment variables (see utils/config.py).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time


def _replica_set(args):
    """`serve --replicas N`: N whole-model engines in their own processes
    (GPU i each, or the host CPU) behind one front scheduler."""
    import torch

    from .models.config import preset
    from .parallel.replicas import ReplicaSet
    from .utils.config import load_engine_config
    if args.lora or args.mmproj or args.draft_model:
        raise SystemExit("--replicas does not combine with --lora, --mmproj or --draft-model")
    ecfg = load_engine_config(args.config)
    if args.max_model_len:
        ecfg.max_model_len = args.max_model_len
    dev = args.device or ("cuda" if torch.cuda.is_available() else "cpu")
    spec = {"device": "cuda" if dev.startswith("cuda") else "cpu", "ecfg": ecfg,
            "seed": args.seed}
    if args.gguf:
        from .models.weights import GgufSource
        spec["gguf"] = args.gguf
        cfg = GgufSource(args.gguf).cfg
    else:
        spec["preset"] = args.model
        cfg = preset(args.model)
    return ReplicaSet(cfg, spec, args.replicas)


def _engine(args):
    import torch
    if getattr(args, "replicas", 1) > 1:
        return _replica_set(args)

    from .engine import LLMEngine
    from .models.config import preset
    from .utils.config import load_engine_config
    ecfg = load_engine_config(args.config)
    if args.max_model_len:
        ecfg.max_model_len = args.max_model_len
    loras = [x.split("=", 1) for x in getattr(args, "lora", None) or []]
    if loras:
        ecfg.max_loras = max(ecfg.max_loras, len(loras))
    dev = args.device or ("cuda:0" if torch.cuda.is_available() else "cpu")
    if getattr(args, "draft_model", None):
        ecfg.draft_model = args.draft_model
        ecfg.spec_depth, ecfg.spec_width = args.spec_depth, args.spec_width
    if ecfg.draft_model:  # speculative serving (drafter preset / GGUF, "self" or "ngram")
        from .engine.spec_engine import create_engine
        src = None
        if args.gguf:
            from .models.weights import GgufSource
            src = GgufSource(args.gguf)
        cfg = src.cfg if src is not None else preset(args.model)
        eng = create_engine(cfg, dev, ecfg, source=src, seed=args.seed)
    elif args.gguf:
        eng = LLMEngine.from_gguf(args.gguf, dev, ecfg)
    else:
        eng = LLMEngine.from_config(preset(args.model), dev, ecfg, seed=args.seed)
    for name, path in loras:
        eng.load_lora(path, name)
    if getattr(args, "mmproj", None):
        eng.load_vision(args.mmproj)
    return eng


def _mtp_generate(eng, tok, ids, args) -> dict:
    """Greedy generation through the MTP or block-drafter speculator (CPU model)."""
    from .engine.mtp import MtpSpeculator
    from .models.llama import LlamaCPU
    if not isinstance(eng.model, LlamaCPU):
        raise SystemExit("--mtp-depth / --block-drafter run on the CPU model (--device cpu)")
    m = eng.model
    if args.block_drafter:
        from .engine.block_spec import BlockSpeculator
        from .models.dflash import DFlashDrafter
        d = DFlashDrafter(args.block_drafter, m)
        spec = BlockSpeculator(m, d, max_len=len(ids) + args.max_tokens + d.cfg.block_size + 16)
        toks = spec.generate(ids, args.max_tokens)
        st = spec.stats
        return {"token_ids": toks, "text": tok.decode(toks), "rounds": st.rounds,
                "acceptance": round(st.acceptance, 4),
                "tokens_per_round": round(st.tokens_per_round, 3)}
    if eng.cfg.mtp_layers < 1:
        raise SystemExit("--mtp-depth needs a model with a next-token-prediction block")
    if m.mtp is None:
        src = getattr(eng, "source", None)
        if src is None:
            from .models.weights import GgufSource, RandomSource
            src = GgufSource(args.gguf) if args.gguf else RandomSource(eng.cfg, seed=args.seed)
        m = LlamaCPU(eng.cfg, src, native=m.native, mtp=True)
    spec = MtpSpeculator(m, depth=args.mtp_depth,
                         max_len=len(ids) + args.max_tokens + args.mtp_depth + 16)
    toks = spec.generate(ids, args.max_tokens)
    st = spec.stats
    return {"token_ids": toks, "text": tok.decode(toks), "mtp_rounds": st.rounds,
            "mtp_acceptance": round(st.acceptance, 4),
            "tokens_per_round": round(st.tokens_per_round, 3)}


def _tokenizer(args, eng):
    from .serve.tokenizer import ByteTokenizer, from_gguf_metadata
    if args.gguf:
        from .gguf.file import GGUFReader
        import os
        md = GGUFReader(args.gguf).metadata if not os.path.isdir(args.gguf) else {}
        return from_gguf_metadata(md, eng.cfg.vocab), md.get("tokenizer.chat_template")
    return ByteTokenizer(eng.cfg.vocab), None


def node_status(url: str, api_key: str | None = None) -> dict:
    """GET a running node's /api/status and /health/ready."""
    import urllib.error
    import urllib.request
    hdr = {"Authorization": f"Bearer {api_key}"} if api_key else {}
    out = {"url": url}
    for key, path in (("status", "/api/status"), ("ready", "/health/ready")):
        try:
            with urllib.request.urlopen(urllib.request.Request(url.rstrip("/") + path, headers=hdr),
                                        timeout=5) as r:
                out[key] = json.loads(r.read().decode() or "null")
        except urllib.error.HTTPError as e:
            out[key] = {"http_status": e.code}
        except OSError as e:
            out[key] = {"error": str(e)}
    return out


def chat_loop(eng, tok, template, args, fin, fout):
    """Read user turns from `fin`, answer each with the full conversation so
    far; an empty line or EOF ends the session."""
    from .engine.sampling import SamplingParams
    from .serve.chat_template import render
    msgs = [{"role": "system", "content": args.system}] if args.system else []
    while True:
        fout.write("> ")
        fout.flush()
        line = fin.readline()
        if not line or not line.strip():
            return
        msgs.append({"role": "user", "content": line.rstrip("\n")})
        ids = tok.encode(render(msgs, eng.cfg.arch, template))
        sp = SamplingParams(max_tokens=args.max_tokens, temperature=args.temperature,
                            eos_token_id=getattr(tok, "eos_id", -1))
        out = eng.generate([ids], sp)[0].token_ids
        text = tok.decode([t for t in out if t != sp.eos_token_id])
        fout.write(text + "\n")
        msgs.append({"role": "assistant", "content": text})


def main(argv=None):
    p = argparse.ArgumentParser(prog="swarmllm_b200")
    sub = p.add_subparsers(dest="cmd", required=True)
    for name in ("serve", "generate", "bench", "info", "chat"):
        s = sub.add_parser(name)
        s.add_argument("--model", default="llama-3.2-3b")
        s.add_argument("--gguf", default=None)
        s.add_argument("--device", default=None)
        s.add_argument("--config", default=None)
        s.add_argument("--seed", type=int, default=0)
        s.add_argument("--max-model-len", type=int, default=0)
        s.add_argument("--lora", action="append", default=[], metavar="NAME=PATH",
                       help="LoRA adapter GGUF; requests select it with model NAME")
        s.add_argument("--mmproj", default=None, help="image encoder GGUF (vision input)")
        s.add_argument("--draft-model", default="",
                       help="speculative decoding: drafter preset or GGUF, 'self' or 'ngram'")
        s.add_argument("--spec-depth", type=int, default=4)
        s.add_argument("--spec-width", type=int, default=4)
        s.add_argument("--log-file", default=None, help="also log to this file (rotating, 50 MB x 3)")
        s.add_argument("--log-json", action="store_true", help="log one JSON object per line")
        s.add_argument("-v", "--verbose", action="count", default=0)
        if name == "serve":
            s.add_argument("--host", default="0.0.0.0")
            s.add_argument("--port", type=int, default=8800)
            s.add_argument("--api-key", default=os.environ.get("SWARMLLM_API_KEY"),
                           help="require this key (Bearer or x-api-key); default: open")
            s.add_argument("--api-key-file", default=os.environ.get("SWARMLLM_API_KEY_FILE"),
                           help="read the key from this file; a key rotated through "
                                "/api/admin/api-key/rotate is written back to it")
            s.add_argument("--cors-origin", action="append", default=[],
                           help="extra browser origin allowed besides localhost")
            s.add_argument("--rpm", type=int, default=0, help="requests a minute per client (0: off)")
            s.add_argument("--kv-persist", default=None,
                           help="file to load the prefix KV cache from at start and save it to at exit "
                                "(discarded when written by another build or model)")
            s.add_argument("--response-store", default=None,
                           help="SQLite file for stored /v1/responses (default: in memory)")
            s.add_argument("--replicas", type=int, default=1,
                           help="serve with N engine replicas (one per GPU, or N CPU processes) "
                                "behind one request router")
        if name == "generate":
            s.add_argument("--prompt", default="Hello")
            s.add_argument("--ids", default=None, help="comma-separated token ids")
            s.add_argument("--max-tokens", type=int, default=32)
            s.add_argument("--temperature", type=float, default=0.0)
            s.add_argument("--adapter", default=None, help="name of a --lora adapter to generate with")
            s.add_argument("--block-drafter", default=None,
                           help="CPU, greedy: a DFlash block drafter GGUF guessing a block a round, "
                                "verified by the model")
            s.add_argument("--mtp-depth", type=int, default=0,
                           help="CPU, greedy: draft this many tokens a round with the model's own "
                                "next-token-prediction block and verify them with the trunk")
        if name == "chat":
            s.add_argument("--max-tokens", type=int, default=256)
            s.add_argument("--temperature", type=float, default=0.7)
            s.add_argument("--system", default=None)
        if name == "bench":
            s.add_argument("--batch", type=int, default=8)
            s.add_argument("--prompt-len", type=int, default=512)
            s.add_argument("--gen", type=int, default=64)
    s = sub.add_parser("status")
    s.add_argument("--url", default="http://127.0.0.1:8800")
    s.add_argument("--api-key", default=os.environ.get("SWARMLLM_API_KEY"))
    sub.add_parser("diagnostics")
    s = sub.add_parser("test-split")
    s.add_argument("--world", type=int, default=2)
    s.add_argument("--native", action="store_true",
                   help="run both sides on the native CPU kernels")
    s = sub.add_parser("shard")
    s.add_argument("gguf")
    s.add_argument("out_dir")
    s.add_argument("--layers-per-shard", type=int, default=4)
    s = sub.add_parser("make-gguf")
    s.add_argument("--model", default="tiny-llama")
    s.add_argument("out")
    s.add_argument("--seed", type=int, default=0)
    args = p.parse_args(argv)

    if args.cmd == "status":
        print(json.dumps(node_status(args.url, args.api_key), indent=1))
        return
    if args.cmd == "diagnostics":
        from .utils.diagnostics import collect
        print(json.dumps(collect(), indent=1))
        return
    if args.cmd == "test-split":
        from .parallel.split_check import split_check
        r = split_check(world=args.world, native=args.native)
        r.pop("tokens")
        print(json.dumps(r))
        sys.exit(0 if r["ok"] else 1)
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
    from .utils.config import load_logging_settings
    from .utils.logsetup import get_logger, setup_logging
    lg = load_logging_settings(args.config)
    setup_logging(args.verbose, args.log_file or lg.get("file"), args.log_json or lg.get("json", False),
                  level=lg.get("level"))
    eng = _engine(args)
    if args.cmd == "info":
        print(json.dumps({"config": eng.cfg.to_dict(), "kv_pages": eng.bm.num_pages,
                          "params": eng.cfg.param_count()}, indent=1))
        return
    if args.cmd == "serve":
        from .serve.api import serve
        tok, tpl = _tokenizer(args, eng)
        log = get_logger("cli")
        kv_persist = args.kv_persist if hasattr(eng, "load_prefix_cache") else None
        if args.kv_persist and not kv_persist:
            log.warning("--kv-persist is ignored with --replicas")
        args.kv_persist = kv_persist
        if args.kv_persist and eng.ecfg.prefix_cache:
            log.info("prefix cache: %d tokens loaded from %s",
                     eng.load_prefix_cache(args.kv_persist), args.kv_persist)
        try:
            serve(eng, tok, eng.cfg.name, args.host, args.port, arch=eng.cfg.arch,
                  chat_template=tpl, max_model_len=eng.ecfg.max_model_len, api_key=args.api_key,
                  cors_origins=tuple(args.cors_origin), rpm=args.rpm,
                  store_path=args.response_store, config_path=args.config,
                  api_key_file=args.api_key_file)
        finally:
            if args.kv_persist and eng.ecfg.prefix_cache:
                log.info("prefix cache: %d tokens saved to %s",
                         eng.save_prefix_cache(args.kv_persist), args.kv_persist)
            if hasattr(eng, "close"):
                eng.close()
        return
    from .engine.sampling import SamplingParams
    if args.cmd == "chat":
        tok, tpl = _tokenizer(args, eng)
        chat_loop(eng, tok, tpl, args, sys.stdin, sys.stdout)
        return
    if args.cmd == "generate":
        tok, _ = _tokenizer(args, eng)
        ids = [int(x) for x in args.ids.split(",")] if args.ids else tok.encode(args.prompt)
        if args.mtp_depth or args.block_drafter:
            print(json.dumps(_mtp_generate(eng, tok, ids, args)))
            return
        sp = SamplingParams(max_tokens=args.max_tokens, temperature=args.temperature)
        rid = eng.add_request(ids, sp, lora=args.adapter) if args.adapter else eng.add_request(ids, sp)
        toks = []
        while eng.has_work():
            toks += [t for r, t, _ in eng.step() if r == rid]
        tr = eng.traces.get(rid)
        print(json.dumps({"token_ids": toks, "text": tok.decode(toks),
                          "ttft_ms": tr.ttft * 1e3 if tr is not None and tr.ttft else None}))
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
