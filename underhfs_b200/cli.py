"""``underhfs`` command line (reference cli.py:30-320).

Kept commands and JSON keys: init, bench, doctor, test, train --smoke,
checkpoint {save-smoke, inspect, save-binary-smoke, inspect-binary},
dataset, serve {--smoke, --http-smoke}, export {manifest, onnx}.  Added:
``generate`` (greedy decoding with a byte tokenizer) and full ``train``
(``--model 125m|1.3b|7b`` on the CUDA engine, one process per GPU under
``python -m underhfs_b200.parallel.launch`` or torchrun).
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path

from underhfs_b200 import __version__


def _tiny_lm(args):
    from underhfs_b200.nn import TransformerLM

    return TransformerLM(vocab_size=args.vocab_size, max_seq_len=args.seq_len, features=args.features,
                         hidden_features=args.hidden_features, layers=args.layers)


def _tiny_meta(args) -> dict:
    return {"model": "TransformerLM", "vocab_size": args.vocab_size, "seq_len": args.seq_len,
            "features": args.features, "hidden_features": args.hidden_features, "layers": args.layers}


def _cmd_init(args) -> int:
    root = Path(args.path)
    root.mkdir(parents=True, exist_ok=True)
    (root / "underhfs.yaml").write_text("runtime:\n  device: cuda:0\n  dtype: bf16\n", encoding="utf-8")
    print(f"initialized {root}")
    return 0


def _cmd_bench(args) -> int:
    from underhfs_b200.benchmarks import run_benchmark_suite, run_memory_benchmark, run_microbenchmarks
    from underhfs_b200.cuda import allocator_stats, device_count, devices, is_available, memory_budgets, stream_stats
    from underhfs_b200.native import status

    st = status()
    results = run_microbenchmarks(size=args.size, iterations=args.iterations, warmup=args.warmup,
                                  include_cuda=not args.no_cuda)
    runtime = {}
    if st.cuda_enabled:
        try:
            runtime = {"allocator": allocator_stats(), "stream": stream_stats()}
        except RuntimeError:
            runtime = {}
    suite = None
    if args.suite:
        suite = run_benchmark_suite(size=max(2, min(args.size, 16)), iterations=max(1, min(args.iterations, 5)),
                                    warmup=max(0, min(args.warmup, 2)), include_cuda=not args.no_cuda,
                                    include_oracle=not args.no_oracle).to_dict()
    payload = {
        "underhfs": __version__, "suite": suite, "cuda_visible": is_available(), "cuda_device_count": device_count(),
        "cuda_devices": [d.to_dict() for d in devices()],
        "memory_budgets": {t.value: n for t, n in memory_budgets().items()}, "native_core": st.available,
        "native_reason": st.reason, "cuda_runtime": runtime, "results": [r.to_dict() for r in results],
        "memory": run_memory_benchmark().to_dict(),
    }
    print(json.dumps(payload, indent=2))
    return 0


def _cmd_doctor(_args) -> int:
    from underhfs_b200.diagnostics import doctor

    print(json.dumps(doctor().to_dict(), indent=2, default=str))
    return 0


TEST_MODULES = [
    "tests.test_tensor_autograd", "tests.test_nn_optim", "tests.test_runtime_surface",
    "tests.test_losses_serialization", "tests.test_transformer_lm", "tests.test_cli_train", "tests.test_benchmarks",
    "tests.test_text_generation", "tests.test_cli_fullstack", "tests.test_runtime_memory_planner",
    "tests.test_guardrails", "tests.test_native_contract", "tests.test_project_starters",
]


def _cmd_test(_args) -> int:
    import sys
    from pathlib import Path

    from underhfs_b200.testing import run_test_functions

    # the suite is the source tree's tests/ package: found from the current
    # directory (an installed console script's sys.path does not include it)
    # or next to a source checkout of this package
    for root in (Path.cwd(), Path(__file__).resolve().parents[1]):
        if (root / "tests" / "__init__.py").exists() and str(root) not in sys.path:
            sys.path.insert(0, str(root))
            break

    passed = run_test_functions(TEST_MODULES)
    for name in passed:
        print(f"{name} OK")
    print(f"{len(passed)} tests passed")
    return 0


def _cmd_train(args) -> int:
    if args.smoke:
        from underhfs_b200.functional import cross_entropy
        from underhfs_b200.optim import SGD
        from underhfs_b200.tensor import tensor

        model = _tiny_lm(args)
        opt = SGD(model.parameters(), lr=args.lr)
        ids = tensor([i % args.vocab_size for i in range(args.seq_len)])
        tg = tensor([(i + 1) % args.vocab_size for i in range(args.seq_len)])
        losses = []
        for _ in range(args.steps):
            opt.zero_grad()
            loss = cross_entropy(model(ids), tg)
            losses.append(loss.item())
            loss.backward()
            opt.step()
        print(json.dumps({"mode": "smoke", "steps": args.steps, "initial_loss": losses[0] if losses else None,
                          "final_loss": losses[-1] if losses else None, "losses": losses}, indent=2))
        return 0
    if not args.model:
        print("underhfs train needs --smoke or --model {125m,1.3b,7b}")
        return 2
    import torch

    from underhfs_b200.data import SyntheticTokens
    from underhfs_b200.train import TrainConfig, Trainer, build_model

    cfg = TrainConfig(model=args.model, batch=args.batch, seq_len=args.seq_len_train, lr=args.lr_train,
                      zero_stage=args.zero, cuda_graph=not args.no_graph, offload=args.offload,
                      context_parallel=getattr(args, "context_parallel", False))
    from underhfs_b200.distributed import policy_from_env
    from underhfs_b200.train import StepMeter

    pol = policy_from_env(zero_stage=cfg.zero_stage)
    if pol.world_size > 1:
        torch.cuda.set_device(pol.local_rank or 0)
    model = build_model(cfg, device=f"cuda:{pol.local_rank or 0}")
    spec = model.spec
    trainer = Trainer(model, cfg, policy=pol)
    # context parallelism: every rank draws the same sequences and trains on its shard
    data = SyntheticTokens(model.vocab_size, cfg.batch, cfg.seq_len, seed=cfg.seed,
                           rank=0 if cfg.context_parallel else pol.rank)
    host = torch.empty((2, cfg.batch, cfg.seq_len), dtype=torch.int64, pin_memory=True)
    tokens_per_step = cfg.batch * (cfg.seq_len if not cfg.context_parallel else cfg.seq_len // pol.world_size)
    meter = StepMeter(world=pol.world_size, tokens_per_rank=tokens_per_step,
                      flops_per_token=spec.train_flops_per_token(cfg.seq_len), peak_tflops=args.peak_tflops)
    losses, records = [], []
    for i in range(args.steps):
        meter.start()
        losses.append(trainer.step_from_host(data.next_host(host)))
        rec = meter.stop()  # device time of this step, max over ranks (a collective)
        rec.update(step=i, loss=losses[-1])
        records.append(rec)
        if pol.rank == 0 and args.log_every and (i % args.log_every == 0 or i == args.steps - 1):
            print(json.dumps(rec), flush=True)
    trainer.release()
    if pol.rank == 0:
        timed = records[1:] or records  # the first step includes capture / warm-up
        print(json.dumps({"mode": "train", "model": args.model, "world_size": pol.world_size, "steps": args.steps,
                          "zero_stage": cfg.zero_stage, "initial_loss": losses[0], "final_loss": losses[-1],
                          "losses": losses,
                          "tokens_per_s": sum(r["tokens_per_s"] for r in timed) / len(timed),
                          "max_memory_gb": max(r["max_memory_gb"] for r in records),
                          "mfu": sum(r["mfu"] for r in timed) / len(timed),
                          "peak_tflops": args.peak_tflops}, indent=2))
    return 0


def _cmd_checkpoint(args) -> int:
    from underhfs_b200.serialization import (load_binary_state_dict, load_checkpoint, save_binary_state_dict,
                                             save_checkpoint)

    path = Path(args.path)
    if args.action == "save-smoke":
        model = _tiny_lm(args)
        save_checkpoint(path, state=model.state_dict(), metadata=_tiny_meta(args))
        print(json.dumps({"saved": str(path), "parameters": len(model.state_dict())}, indent=2))
        return 0
    if args.action == "inspect":
        doc = load_checkpoint(path)
        print(json.dumps({"path": str(path), "metadata": doc["metadata"], "tensors": len(doc["state"])}, indent=2))
        return 0
    if args.action == "save-binary-smoke":
        model = _tiny_lm(args)
        save_binary_state_dict(path, model.state_dict(as_tensors=True))
        print(json.dumps({"saved": str(path), "format": "binary", "parameters": len(model.state_dict())}, indent=2))
        return 0
    if args.action == "inspect-binary":
        state = load_binary_state_dict(path)
        print(json.dumps({"path": str(path), "format": "binary", "tensors": len(state)}, indent=2))
        return 0
    print(f"unsupported checkpoint action: {args.action}")
    return 2


def _cmd_dataset(args) -> int:
    from underhfs_b200.datasets import inspect_text_dataset, write_sample_text_dataset

    report = write_sample_text_dataset(args.path) if args.sample else inspect_text_dataset(args.path)
    print(json.dumps(report.to_dict(), indent=2))
    return 0


def _byte_generator(max_new_tokens: int):
    from underhfs_b200.nn import TransformerLM
    from underhfs_b200.text import ByteTokenizer

    tok = ByteTokenizer()
    model = TransformerLM(vocab_size=256, max_seq_len=8, features=4, hidden_features=8, layers=1)
    return lambda prompt: tok.decode(model.generate(tok.encode(prompt), max_new_tokens))


def _cmd_serve(args) -> int:
    from underhfs_b200.serve import ServeConfig, serve, serve_http

    if not args.smoke and not args.http_smoke:
        print("underhfs serve currently supports --smoke and --http-smoke verification paths")
        return 2
    gen = _byte_generator(args.max_new_tokens)
    server = serve(lambda payload: gen(payload["prompt"]))
    if args.http_smoke:
        http = serve_http(lambda payload: {"text": server.predict(payload)}, ServeConfig(host=args.host, port=args.port))
        try:
            http.start()
            print(json.dumps({"url": http.url, "health": "/health", "predict": "/predict"}, indent=2))
        finally:
            http.close()
        return 0
    print(json.dumps({"prompt": args.prompt, "response": server.predict({"prompt": args.prompt})}, indent=2))
    return 0


def _cmd_generate(args) -> int:
    from underhfs_b200.nn import TransformerLM
    from underhfs_b200.serialization import load_binary_state_tensors
    from underhfs_b200.text import ByteTokenizer

    tok = ByteTokenizer()
    model = TransformerLM(vocab_size=256, max_seq_len=args.seq_len, features=args.features,
                          hidden_features=args.hidden_features, layers=args.layers)
    if args.checkpoint:
        model.load_state_dict(load_binary_state_tensors(args.checkpoint))
    if args.device.startswith("cuda"):
        model.to(args.device)
    out = model.generate(tok.encode(args.prompt), args.max_new_tokens)
    print(json.dumps({"prompt": args.prompt, "response": tok.decode(out), "tokens": [int(v) for v in out._storage]},
                     indent=2))
    return 0


def _cmd_export(args) -> int:
    from underhfs_b200.serialization import export_manifest, export_onnx

    model = _tiny_lm(args)
    inputs = {"token_ids": {"shape": [args.seq_len], "dtype": "int64"}}
    if args.format == "onnx":
        fmt = export_onnx(args.path, model_name="TransformerLM", state=model.state_dict(), inputs=inputs)
        print(json.dumps({"exported": args.path, "format": fmt, "model": "TransformerLM"}, indent=2))
        return 0
    export_manifest(args.path, model_name="TransformerLM", state=model.state_dict(), inputs=inputs)
    print(json.dumps({"exported": args.path, "format": "manifest", "model": "TransformerLM"}, indent=2))
    return 0


def _tiny_args(p: argparse.ArgumentParser, seq: int = 4) -> None:
    p.add_argument("--seq-len", type=int, default=seq)
    p.add_argument("--vocab-size", type=int, default=8)
    p.add_argument("--features", type=int, default=4)
    p.add_argument("--hidden-features", type=int, default=8)
    p.add_argument("--layers", type=int, default=1)


def main(argv: list[str] | None = None) -> int:
    parser = argparse.ArgumentParser(prog="underhfs")
    parser.add_argument("--version", action="version", version=f"underhfs {__version__}")
    sub = parser.add_subparsers(dest="command", required=True)

    p = sub.add_parser("init")
    p.add_argument("path", nargs="?", default=".")
    p.set_defaults(func=_cmd_init)

    p = sub.add_parser("bench")
    p.add_argument("--size", type=int, default=32)
    p.add_argument("--iterations", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--no-cuda", action="store_true")
    p.add_argument("--suite", action="store_true")
    p.add_argument("--no-oracle", action="store_true")
    p.set_defaults(func=_cmd_bench)

    sub.add_parser("doctor").set_defaults(func=_cmd_doctor)
    sub.add_parser("test").set_defaults(func=_cmd_test)

    p = sub.add_parser("train")
    p.add_argument("--smoke", action="store_true")
    p.add_argument("--steps", type=int, default=3)
    _tiny_args(p)
    p.add_argument("--lr", type=float, default=1e-3)
    p.add_argument("--model", choices=("125m", "1.3b", "7b"))
    p.add_argument("--batch", type=int, default=16)
    p.add_argument("--seq-len-train", type=int, default=1024)
    p.add_argument("--lr-train", type=float, default=3e-4)
    p.add_argument("--zero", type=int, default=0, choices=(0, 1, 2, 3))
    p.add_argument("--offload", choices=("auto", "host", "device"), default="auto",
                   help="ZeRO-3 Adam moments: the memory planner decides (auto), or force pinned host / device")
    p.add_argument("--no-graph", action="store_true")
    p.add_argument("--log-every", type=int, default=1, help="print a per-step JSON record every N steps (0: off)")
    p.add_argument("--peak-tflops", type=float, default=2250.0,
                   help="bf16 dense peak per GPU for the MFU column (default: B200 nominal 2250)")
    p.add_argument("--context-parallel", action="store_true",
                   help="shard every sequence over all ranks (zigzag) instead of giving each rank its own batch")
    p.set_defaults(func=_cmd_train)

    p = sub.add_parser("checkpoint")
    p.add_argument("action", choices=("save-smoke", "inspect", "save-binary-smoke", "inspect-binary"))
    p.add_argument("path")
    _tiny_args(p)
    p.set_defaults(func=_cmd_checkpoint)

    p = sub.add_parser("dataset")
    p.add_argument("path")
    p.add_argument("--sample", action="store_true")
    p.set_defaults(func=_cmd_dataset)

    p = sub.add_parser("serve")
    p.add_argument("--smoke", action="store_true")
    p.add_argument("--http-smoke", action="store_true")
    p.add_argument("--host", default="127.0.0.1")
    p.add_argument("--port", type=int, default=0)
    p.add_argument("--prompt", default="hi")
    p.add_argument("--max-new-tokens", type=int, default=2)
    p.set_defaults(func=_cmd_serve)

    p = sub.add_parser("generate")
    p.add_argument("--prompt", default="hi")
    p.add_argument("--max-new-tokens", type=int, default=8)
    p.add_argument("--checkpoint")
    p.add_argument("--device", default="cpu")
    p.add_argument("--seq-len", type=int, default=8)
    p.add_argument("--features", type=int, default=4)
    p.add_argument("--hidden-features", type=int, default=8)
    p.add_argument("--layers", type=int, default=1)
    p.set_defaults(func=_cmd_generate)

    p = sub.add_parser("export")
    p.add_argument("path")
    p.add_argument("--format", choices=("manifest", "onnx"), default="manifest")
    _tiny_args(p)
    p.set_defaults(func=_cmd_export)

    args = parser.parse_args(argv)
    return args.func(args)


if __name__ == "__main__":
    raise SystemExit(main())
