"""Server CLI: ``python -m mlx_swift_lm_b200.server --model DIR [--host H] [--port P] ...``.

Flags mirror the reference's mlx-server (MLXLMServer/CLI/ServerConfiguration.swift:62-150):
--model/-m, --host, --port, --tool-call-parser, --reasoning-parser,
--embedding-model, --list-routes; each also reads B200LM_SERVER_<NAME>.
Extra engine flags: --max-concurrent, --max-model-len, --kv-fp8, --tp (tensor
parallel ranks when launched under torchrun), --random-config (serve a
random-weight model of a named shape, e.g. for load tests).
"""
from __future__ import annotations

import argparse
import os
import sys


def env(name, default=None):
    return os.environ.get("B200LM_SERVER_" + name.upper().replace("-", "_"), default)


def parse(argv=None):
    ap = argparse.ArgumentParser(prog="mlx_swift_lm_b200.server")
    ap.add_argument("--model", "-m", default=env("model"))
    ap.add_argument("--host", default=env("host", "127.0.0.1"))
    ap.add_argument("--port", type=int, default=int(env("port", "8080")))
    ap.add_argument("--tool-call-parser", default=env("tool_call_parser"))
    ap.add_argument("--reasoning-parser", default=env("reasoning_parser"))
    ap.add_argument("--embedding-model", default=env("embedding_model"))
    ap.add_argument("--list-routes", action="store_true")
    ap.add_argument("--max-concurrent", type=int, default=int(env("max_concurrent", "64")))
    ap.add_argument("--max-model-len", type=int, default=int(env("max_model_len", "8192")))
    ap.add_argument("--kv-fp8", action="store_true")
    ap.add_argument("--random-config", default=env("random_config"),
                    help="serve random weights of a named shape: tiny_qwen3 | qwen3_8b | ...")
    ap.add_argument("--device", default=env("device"))
    ap.add_argument("--data-parallel", type=int, default=int(env("data_parallel", "1")),
                    help="engine replicas, one per GPU (cuda:0..N-1), behind a load / prefix-affinity router")
    return ap.parse_args(argv)


def main(argv=None):
    args = parse(argv)
    from .app import ROUTES

    if args.list_routes:
        for m, p in ROUTES:
            print(f"{m:5s} {p}")
        return 0
    import torch
    import uvicorn

    from ..api.container import ModelContainer
    from ..engine.engine import EngineConfig
    from ..engine.scheduler import SchedulerConfig
    from .app import OpenAIService, build_app

    device = args.device or ("cuda" if torch.cuda.is_available() else "cpu")
    ecfg = EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=args.max_concurrent),
                        max_model_len=args.max_model_len, kv_fp8=args.kv_fp8, enable_prefix_cache=True,
                        use_cuda_graphs=device.startswith("cuda"))
    if args.random_config:
        from ..models import config as mcfg

        cfg = getattr(mcfg, args.random_config)()
        dt = torch.bfloat16 if device.startswith("cuda") else torch.float32
        container = ModelContainer.random(cfg, device, dt, engine_config=ecfg)
        container.model_id = args.random_config
    elif args.model:
        container = ModelContainer.load(args.model, device=device, engine_config=ecfg)
    else:
        print("either --model or --random-config is required", file=sys.stderr)
        return 2
    if args.data_parallel > 1:
        container.replicate([f"cuda:{i}" for i in range(1, args.data_parallel)], ecfg)
    embedder = None
    if args.embedding_model:
        from ..api.embed import Embedder

        embedder = Embedder.from_pretrained(args.embedding_model, device=device)
    svc = OpenAIService(container, tool_parser=args.tool_call_parser, reasoning_parser=args.reasoning_parser,
                        embedder=embedder)
    uvicorn.run(build_app(svc), host=args.host, port=args.port, log_level="info")
    return 0


if __name__ == "__main__":
    sys.exit(main())
