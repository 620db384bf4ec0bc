"""Launch a co-serving server from a sectioned YAML config.

    python -m deltaserve_vllm_b200.launch --config configs/llama3_8b.yaml
    python -m deltaserve_vllm_b200.launch --config ... --tp 2 --port 8001
    python -m deltaserve_vllm_b200.launch --config ... --dry-run

One process per GPU: with ``tensor_parallel_size`` > 1 the launcher re-runs
itself under ``torch.distributed.run`` (one rank per GPU, rendezvous on
127.0.0.1). Rank 0 builds the engine, profiles the step-time estimator, and
serves HTTP; every other rank builds its shard of the engine and replays rank
0's step plans until ``/shutdown``.

Same CLI surface as the reference launchers
(``scripts/launch_deltaserve.py:40-50``, ``eval-tp/launch_deltaserve.py:182-259``):
``--config``, ``--model``, ``--tp``, ``--port``, ``--start-finetuning``,
``--dry-run``; there is no separate vLLM process to wait for.
"""

from __future__ import annotations

import argparse
import dataclasses
import json
import os
import socket
import sys

from . import dprint


def build_engine(ecfg, ftcfg, rcfg, extras: dict, comm=None):
    """Engine with its tokenizer and the YAML's inference adapters loaded."""
    from .engine.llm_engine import CoServingEngine
    from .models.configs import resolve_arch
    from .utils.tokenizer import load_tokenizer

    arch = resolve_arch(ecfg.model)
    tok_path = ecfg.tokenizer or (ecfg.model if os.path.isdir(ecfg.model) else None)
    tok = load_tokenizer(tok_path, arch.vocab)
    adapters = {}
    for key, path in (extras.get("adapters") or {}).items():
        if not isinstance(path, str) or not os.path.isdir(path):
            raise FileNotFoundError(f"adapters.{key}: {path!r} is not a PEFT adapter directory")
        adapters[os.path.basename(os.path.normpath(path))] = {"path": path}
    eng = CoServingEngine(ecfg, ftcfg, rcfg, comm=comm, arch=arch, adapters=adapters, tokenizer=tok)
    if rcfg.enable_adapter_routing:
        from .adapters.routing import AdapterRouter
        eng.router = AdapterRouter(eng, rcfg)
    return eng


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def parse(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--config", required=True, help="sectioned YAML launch config")
    ap.add_argument("--model", default=None, help="override model.model")
    ap.add_argument("--tp", type=int, default=None, help="override tensor_parallel_size")
    ap.add_argument("--host", default=None, help="override server.host")
    ap.add_argument("--port", type=int, default=None, help="override server.port")
    ap.add_argument("--start-finetuning", action="store_true",
                    help="open finetuning admission once serving (as POST /start_finetuning)")
    ap.add_argument("--no-profile", action="store_true", help="skip the launch-time estimator profile")
    ap.add_argument("--dry-run", action="store_true",
                    help="print the resolved configuration and exit (no GPU, no model)")
    return ap.parse_args(argv)


def resolve(args):
    from .config_loader import load_yaml_config, split_config
    cfg = load_yaml_config(args.config)
    if args.model:
        cfg.setdefault("model", {})["model"] = args.model
    if args.tp:
        cfg.setdefault("parallel", {})["tensor_parallel_size"] = args.tp
    ecfg, ftcfg, rcfg, extras = split_config(cfg)
    server = extras.get("server") or {}
    host = args.host or server.get("host", "127.0.0.1")
    port = args.port or int(server.get("port", 8000))
    return ecfg, ftcfg, rcfg, extras, host, port


def main(argv=None) -> int:
    args = parse(argv)
    ecfg, ftcfg, rcfg, extras, host, port = resolve(args)
    if args.dry_run:
        print(json.dumps({"engine": dataclasses.asdict(ecfg), "finetune": dataclasses.asdict(ftcfg),
                          "adapter_routing": dataclasses.asdict(rcfg), "extras": extras,
                          "server": {"host": host, "port": port}}, indent=2, default=str))
        return 0
    tp = ecfg.tensor_parallel_size
    if tp > 1 and "WORLD_SIZE" not in os.environ:
        cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={tp}",
               "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
               "-m", "deltaserve_vllm_b200.launch", *(argv if argv is not None else sys.argv[1:])]
        dprint("launching", " ".join(cmd))
        os.execvp(cmd[0], cmd)
    import torch
    from .parallel.comm import init_tp

    comm = init_tp(timeout_s=600) if tp > 1 else None
    eng = build_engine(ecfg, ftcfg, rcfg, extras, comm)
    try:
        if not eng.is_driver:
            eng.follow()
            return 0
        if eng.ft_enabled and ftcfg.profile_on_launch and not args.no_profile:
            eng.profile_execution_model()
        elif eng.cuda:
            eng.warm_decode_graphs()
        if args.start_finetuning:
            eng.start_finetuning()
        import uvicorn
        from .server.api import create_app
        app = create_app(eng)
        server = uvicorn.Server(uvicorn.Config(app, host=host, port=port, log_level="warning"))
        app.state.server = server
        dprint(f"serving {ecfg.model} (TP={tp}) on http://{host}:{port}")
        server.run()
        eng.shutdown()
        return 0
    finally:
        eng.close()
        if comm is not None and torch.distributed.is_initialized():
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
