"""Headline benchmark: TransformerLM training tokens/s on 1..8 B200 (one process per GPU).

Workload (the data-parallel 125M configuration): TransformerLM d_model 768,
12 layers, 12 heads, MLP 3072, vocab 32000, tied embeddings, bf16 compute with
fp32 master weights, sequence 1024, micro-batch 16 per GPU (weak scaling),
FusedAdamW lr 3e-4, gradients all-reduced in 25 MB buckets overlapped with
backward.  Synthetic uniform token ids from a seed, random-init weights.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config NAME]

``--config tiny-cpu`` runs the CPU-fallback configuration instead (50 AdamW
steps of a d_model-64 model on 8 x 64 byte ids, checkpoint round trip,
greedy generation), which the reference's own runtime can also complete.

For N > 1 launch with torchrun (one rank per GPU); RANK / LOCAL_RANK /
WORLD_SIZE / MASTER_* come from the environment.  Rank 0 prints one JSON line.

Timing: W untimed warm-up steps, then exactly K steps between a barrier +
cuda.synchronize on both sides, timed with CUDA events on the launching
stream; the reported time is the max over ranks.  The per-step working set
(weights, fp32 gradients and moments, activations) is far larger than the
126 MB L2, so no explicit flush is done.  SM clocks and throttle reasons are
sampled with nvidia-smi during the timed region.  The end-to-end figure runs
the public ``Trainer.step_from_host`` API: each step copies its batch from
pinned host memory and reads the loss back to the host (with ``wait=False``
the host reads step i's loss while step i + 1 runs).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "TransformerLM train tokens/sec (device-timed, max over ranks) @1/2/4/8 B200"
MODEL = "125M TransformerLM (d_model 768, 12 layers, 12 heads, MLP 3072, vocab 32000, tied)"
SEQ, MICRO_BATCH = 1024, 16

# --config: the default is the headline data-parallel run; the others are the
# larger sharded configurations of the same model family.
CONFIGS = {
    "125m-ddp": dict(model="125m", batch=16, seq=1024, zero=0, desc=MODEL),
    "1.3b-zero2": dict(model="1.3b", batch=8, seq=2048, zero=2,
                       desc="1.3B TransformerLM (d_model 2048, 24 layers, 16 heads, MLP 8192, vocab 32000, tied)"),
    "7b-zero3": dict(model="7b", batch=2, seq=4096, zero=3,
                     desc="7B TransformerLM (d_model 4096, 32 layers, 32 heads, MLP 11008, vocab 32000, untied)"),
    # the CPU-fallback configuration: the one the reference's own runtime can
    # complete (pure Python, about 2.2-2.5 tokens/s on an 8-core host)
    # element-wise add / mul at 2^26, GEMM at 1024/4096/8192, collectives at N > 1
    "micro": dict(model=None, batch=0, seq=0, zero=0, desc="microbenchmarks"),
    "tiny-cpu": dict(model="tiny", batch=8, seq=64, zero=0, cpu=True,
                     desc="tiny TransformerLM (byte vocab 256, d_model 64, 2 blocks, 4 heads, MLP 256), CPU"),
}

TINY_STEPS = 50


def run_tiny_cpu(args) -> int:
    """CPU fallback: 50 AdamW steps (lr 1e-3, wd 0.01) on 8 x 64 uniform byte
    ids from seed 0, then a checkpoint round trip (.uhfsbin) and greedy
    generation of 32 bytes, through the public API.  Host wall-clock timing
    (no device); the round trip and generation are checked, not timed."""
    import torch

    from underhfs_b200.nn import CrossEntropyLoss, TransformerLM
    from underhfs_b200.optim import AdamW
    from underhfs_b200.serialization import load_binary_state_tensors, save_binary_state_dict
    from underhfs_b200.tensor import tensor

    steps = args.steps if args.steps_given else TINY_STEPS
    gen = torch.Generator().manual_seed(0)
    batches = [torch.randint(0, 256, (8, 65), generator=gen) for _ in range(args.warmup + steps)]
    model = TransformerLM(256, 64, 64, 256, 2, heads=4, seed=0)
    opt = AdamW(model.parameters(), lr=1e-3, weight_decay=0.01)
    loss_fn = CrossEntropyLoss()

    def step(b):
        opt.zero_grad()
        loss = loss_fn(model(tensor(b[:, :64])).reshape(8 * 64, 256), tensor(b[:, 1:].reshape(-1)))
        loss.backward()
        opt.step()
        return loss.item()

    for i in range(args.warmup):
        step(batches[i])
    t0 = time.perf_counter()
    losses = [step(batches[args.warmup + i]) for i in range(steps)]
    dt = time.perf_counter() - t0
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "tiny.uhfsbin")
        save_binary_state_dict(path, model.state_dict(as_tensors=True))
        again = TransformerLM(256, 64, 64, 256, 2, heads=4, seed=1)
        again.load_state_dict(load_binary_state_tensors(path))
        probe = tensor(batches[0][:1, :64])
        same = bool(torch.allclose(model(probe)._data.float(), again(probe)._data.float(), atol=1e-5))
    out = model.generate(tensor(batches[0][0, :16]), 32)
    tokens = 8 * 64 * steps
    print(json.dumps({
        "metric": "TransformerLM train tokens/sec (host wall clock, CPU fallback)", "value": tokens / dt,
        "unit": "tokens/s", "n_gpus": 0, "steps": steps, "warmup": args.warmup, "ms_per_step": 1e3 * dt / steps,
        "higher_is_better": True, "scaling": "none", "vs_baseline": None, "dtype": "fp64 (CPU tensors)",
        "data": "uniform byte ids in [0,256) from seed 0; random-init weights",
        "config": {"model": CONFIGS["tiny-cpu"]["desc"], "global_batch": 8, "seq_len": 64, "parallelism": "none",
                   "optimizer": "AdamW lr 1e-3 wd 0.01"},
        "first_loss": losses[0], "final_loss": losses[-1], "checkpoint_roundtrip_matches": same,
        "generated_tokens": int(out.shape[0]) - 16,
    }))
    return 0 if same else 1


def run_reference_tiny(args) -> int:
    """The same CPU configuration on the unmodified reference (baseline/_ref),
    through its public API in a subprocess rooted there (this repository's own
    ``underhfs`` package would otherwise shadow it).  Its TransformerLM has no
    batch dimension or heads, so the 8 sequences of a step are accumulated
    one by one before the optimizer step, single-head attention."""
    ref = ROOT / "baseline" / "_ref"
    if not (ref / "underhfs" / "__init__.py").exists():
        print(json.dumps({"impl": "reference", "unavailable": "reference not installed under baseline/_ref"}))
        return 0
    steps = args.steps if args.steps_given else 1
    code = f"""
import json, random, time
import underhfs
from underhfs.nn import TransformerLM
from underhfs.optim import AdamW
from underhfs.functional import cross_entropy
rng = random.Random(0)
model = TransformerLM(256, 64, 64, 256, 2)
opt = AdamW(model.parameters(), lr=1e-3, weight_decay=0.01)
t0 = time.perf_counter()
for _ in range({steps}):
    opt.zero_grad()
    for _ in range(8):
        ids = [rng.randrange(256) for _ in range(65)]
        loss = cross_entropy(model(underhfs.tensor(ids[:64])), underhfs.tensor(ids[1:]))
        loss.backward()
    opt.step()
dt = time.perf_counter() - t0
print(json.dumps({{"seconds": dt, "loss": loss.item()}}))
"""
    env = dict(os.environ, PYTHONPATH=str(ref))
    proc = subprocess.run([sys.executable, "-c", code], cwd=str(ref), env=env, capture_output=True, text=True)
    if proc.returncode != 0:
        print(json.dumps({"impl": "reference", "unavailable": "reference run failed: "
                          + (proc.stderr.strip().splitlines() or ["?"])[-1]}))
        return 0
    r = json.loads(proc.stdout.strip().splitlines()[-1])
    print(json.dumps({
        "impl": "reference", "metric": "TransformerLM train tokens/sec (host wall clock, CPU fallback)",
        "value": 8 * 64 * steps / r["seconds"], "unit": "tokens/s", "n_gpus": 0, "steps": steps, "warmup": 0,
        "ms_per_step": 1e3 * r["seconds"] / steps, "higher_is_better": True, "dtype": "Python float",
        "data": "uniform byte ids in [0,256) from a seed", "final_loss": r["loss"],
        "config": {"model": "reference TransformerLM(256, 64, 64, 256, 2), single head, 8 sequences accumulated "
                   "per step", "global_batch": 8, "seq_len": 64},
    }))
    return 0


def _clock_sampler(local_rank: int):
    fields = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    out = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
    try:
        proc = subprocess.Popen(["nvidia-smi", f"--id={local_rank}", f"--query-gpu={fields}", "--format=csv,noheader",
                                 "-lms", "200"], stdout=out, stderr=subprocess.DEVNULL)
    except (FileNotFoundError, OSError):
        return None, out.name
    return proc, out.name


def _clock_summary(path: str) -> dict:
    mhz, maxes, reasons = [], [], set()
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    for line in Path(path).read_text().splitlines():
        parts = [p.strip() for p in line.split(",")]
        if len(parts) < 9:
            continue
        try:
            mhz.append(float(parts[1].split()[0]))
            maxes.append(float(parts[2].split()[0]))
        except ValueError:
            continue
        for name, flag in zip(names, parts[5:9]):
            if flag.lower() == "active":
                reasons.add(name)
    if not mhz:
        return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
    return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": max(maxes), "reasons": sorted(reasons),
            "samples": len(mhz)}


def run_ours(args) -> int:
    import torch
    import torch.distributed as dist

    from underhfs_b200.data import SyntheticTokens
    from underhfs_b200.distributed import policy_from_env
    from underhfs_b200.ops._lib import core
    from underhfs_b200.train import TrainConfig, Trainer, build_model

    pol = policy_from_env(timeout_s=600.0)
    n = pol.world_size
    if n != args.gpus:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE={n}", file=sys.stderr)
    local = pol.local_rank or 0
    torch.cuda.set_device(local)
    cc = CONFIGS[args.config]
    if cc["zero"] == 3:
        return run_zero3(args, pol, cc)
    cfg = TrainConfig(model=cc["model"], batch=cc["batch"], seq_len=cc["seq"], lr=3e-4, bucket_mb=25.0,
                      cuda_graph=not args.no_graph, zero_stage=cc["zero"],
                      decoupled=True, weight_decay=0.0 if cc["zero"] == 0 else 0.1)
    model = build_model(cfg, device=f"cuda:{local}")
    trainer = Trainer(model, cfg, policy=pol)
    src = SyntheticTokens(model.vocab_size, cfg.batch, cfg.seq_len, seed=1234, rank=pol.rank)
    pool = [src.next_host().cuda() for _ in range(4)]

    def barrier():
        if n > 1:
            dist.barrier()

    # kernels of this library launched per training step (counted on one eager step)
    c = core()
    c.reset_launch_count()
    trainer.cfg.cuda_graph = False
    trainer.step(pool[0][0], pool[0][1])
    torch.cuda.synchronize()
    launches_per_step = c.launch_count()
    trainer.cfg.cuda_graph = not args.no_graph

    for i in range(args.warmup):
        trainer.step(pool[i % 4][0], pool[i % 4][1])
    torch.cuda.synchronize()
    barrier()

    sampler, clock_path = _clock_sampler(local)
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(args.steps):
        b = pool[i % 4]
        loss = trainer.step(b[0], b[1])
    end.record()
    torch.cuda.synchronize()
    barrier()
    if sampler is not None:
        sampler.terminate()
        sampler.wait()
    ms = start.elapsed_time(end)
    final_loss = float(loss.item())

    # end to end through the public API: pinned H2D of each batch + D2H of the loss
    host = torch.empty((2, cfg.batch, cfg.seq_len), dtype=torch.int64, pin_memory=True)
    src.next_host(host)
    trainer.step_from_host(host)
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    pending = None
    for _ in range(args.steps):
        # each step's loss is read on the host while the next step runs
        queued = trainer.step_from_host(host, wait=False)
        if pending is not None:
            pending.result()
        pending = queued
    pending.result()
    e2e_s = time.perf_counter() - t0
    barrier()

    stats = torch.tensor([ms, e2e_s], dtype=torch.float64, device="cuda")
    if n > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    ms_max, e2e_max = stats.tolist()
    clocks = _clock_summary(clock_path)
    trainer.release()
    tokens = n * cfg.batch * cfg.seq_len * args.steps
    if pol.rank == 0:
        line = {
            "metric": METRIC,
            "value": tokens / (ms_max / 1e3),
            "unit": "tokens/s",
            "n_gpus": n,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_max / args.steps,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic uniform token ids in [0,32000) from a fixed seed; random-init weights",
            "config": {"model": cc["desc"], "global_batch": n * cfg.batch, "micro_batch_per_gpu": cfg.batch,
                       "seq_len": cfg.seq_len, "parallelism": f"dp{n}" if cc["zero"] == 0 else f"zero{cc['zero']}-{n}",
                       "optimizer": (f"FusedAdamW lr 3e-4, betas (0.9, 0.95), eps 1e-8, weight decay "
                                     f"{cfg.weight_decay} (decoupled); fp32 master, one fused launch"
                                     if cc["zero"] == 0 else
                                     f"ZeRO-2 AdamW lr 3e-4, betas (0.9, 0.95), weight decay {cfg.weight_decay} "
                                     "(decoupled): fused NVLink reduce-scatter + AdamW + all-gather kernel"),
                       "grad_allreduce": ((f"fused NVLink two-shot kernel ({os.environ.get('UNDERHFS_DDP_WIRE', 'fp32')} "
                                           "on the wire), 25 MB buckets overlapped with backward")
                                          if cc["zero"] == 0 else "reduce-scatter fused with the AdamW update"),
                       "cuda_graph": not args.no_graph,
                       "l2": "no flush: per-step working set (weights, grads, moments, activations) >> 126 MB L2"},
            "clocks": clocks,
            "e2e": {"value": tokens / e2e_max, "unit": "tokens/s",
                    "h2d_bytes_per_step": host.numel() * host.element_size(), "d2h_bytes_per_step": 4,
                    "api": "underhfs_b200.train.Trainer.step_from_host(wait=False), each loss read while the next "
                           "step runs", "timer": "host wall clock, max over ranks"},
            "gpu_launches": launches_per_step * args.steps,
            "final_loss": final_loss,
        }
        print(json.dumps(line), flush=True)
    if n > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


REF_REASON = (
    "reference TransformerLM (src/underhfs/nn.py:287-334) is pure Python: every parameter is a Python float list, "
    "it has no batch dimension, no multi-head attention and no bf16 GEMM, and its modules have no device "
    "placement (only single tensors move to CUDA, and each CUDA op syncs back to a host list, tensor.py:401-405); "
    "one 16x1024-token step of the 125M model cannot complete"
)

# What the reference arm times, through the reference's own public API, in a
# subprocess rooted at baseline/_ref: building the stock modules of the
# headline model and running one TransformerBlock(768, 3072) forward on a short
# prefix of one sequence.  Each phase prints a JSON progress line, so what
# completed before the wall-time budget is reported even if the run is cut.
_REF_PROBE = """
import json, random, sys, time
budget_tokens = int(sys.argv[1])
from underhfs import tensor
from underhfs.nn import Embedding, TransformerBlock
def emit(**kw):
    print(json.dumps(kw), flush=True)
t = time.perf_counter()
block = TransformerBlock(768, 3072, causal=True)
emit(phase="build_block", seconds=time.perf_counter() - t, params=sum(p.numel() for p in block.parameters()))
t = time.perf_counter()
pos = Embedding(1024, 768)
emit(phase="build_position_embedding", seconds=time.perf_counter() - t, params=1024 * 768)
rng = random.Random(0)
x = tensor([[rng.uniform(-0.05, 0.05) for _ in range(768)] for _ in range(budget_tokens)])
t = time.perf_counter()
y = block(x)
emit(phase="block_forward", seconds=time.perf_counter() - t, tokens=budget_tokens)
t = time.perf_counter()
y.sum().backward()
emit(phase="block_backward", seconds=time.perf_counter() - t, tokens=budget_tokens)
"""


def run_reference(args) -> int:
    """The unmodified reference on the headline configuration, bounded in wall
    time (UNDERHFS_REF_BUDGET_S, default 90 s).  It cannot complete a step
    (REF_REASON), so the line is ``unavailable`` and carries what was measured:
    the reference's own time to build one 768/3072 block and the embedding
    tables, and one block's forward / backward on a 16-token prefix, plus a
    linear-in-tokens lower bound for one 16 x 1024-token step derived from them."""
    ref = ROOT / "baseline" / "_ref"
    rank = int(os.environ.get("RANK", "0"))
    if not (ref / "underhfs" / "__init__.py").exists():
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "reference not installed under baseline/_ref; "
                              + REF_REASON}))
        return 0
    if rank != 0:  # the reference has no data parallelism of its own: rank 0 measures
        return 0
    budget = float(os.environ.get("UNDERHFS_REF_BUDGET_S", "90"))
    probe_tokens = 16
    env = dict(os.environ, PYTHONPATH=str(ref))
    t0 = time.perf_counter()
    proc = subprocess.Popen([sys.executable, "-c", _REF_PROBE, str(probe_tokens)], cwd=str(ref), env=env,
                            stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)
    try:
        out, _err = proc.communicate(timeout=budget)
        finished = True
    except subprocess.TimeoutExpired:
        proc.kill()
        out, _err = proc.communicate()
        finished = False
    wall = time.perf_counter() - t0
    phases = {}
    for line in out.splitlines():
        try:
            rec = json.loads(line)
        except json.JSONDecodeError:
            continue
        phases[rec.pop("phase")] = rec
    measured = {"wall_budget_s": budget, "wall_s": round(wall, 2), "completed_phases": list(phases),
                "finished": finished, "phases": phases, "timer": "host wall clock (pure-Python reference)"}
    fwd, bwd = phases.get("block_forward"), phases.get("block_backward")
    if fwd and bwd:
        per_token_block = (fwd["seconds"] + bwd["seconds"]) / probe_tokens
        # 12 blocks x 16 x 1024 tokens, linear in tokens (attention is quadratic:
        # a lower bound); embeddings and the 32000-way head are left out
        step_lb = per_token_block * 12 * MICRO_BATCH * SEQ
        measured["step_seconds_lower_bound"] = step_lb
        measured["tokens_per_s_upper_bound"] = MICRO_BATCH * SEQ / step_lb
    build = phases.get("build_block")
    if build:
        measured["model_build_seconds_estimate"] = build["seconds"] * (
            (32000 * 768 + 12 * build["params"]) / build["params"])
    print(json.dumps({"impl": "reference", "unavailable": REF_REASON, "metric": METRIC,
                      "config": {"model": MODEL, "seq_len": SEQ, "micro_batch_per_gpu": MICRO_BATCH},
                      "measured": measured}))
    return 0


def run_torch_eager(args) -> int:
    """Comparison bar, clearly not this framework: the same 125M model in plain
    PyTorch -- fp32 parameters under bf16 autocast, torch.nn layers, torch's
    scaled_dot_product_attention (causal), torch.optim.AdamW(fused=True) and,
    for N > 1, torch DistributedDataParallel over NCCL with 25 MB buckets --
    timed exactly like ``--impl ours`` (CUDA events, max over ranks)."""
    import torch
    import torch.distributed as dist
    import torch.nn as tnn
    import torch.nn.functional as tF

    rank, n = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if n > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)
    V, T, F, Hd, L, H = 32000, SEQ, 768, 3072, 12, 12

    class Block(tnn.Module):
        def __init__(self):
            super().__init__()
            self.n1, self.n2 = tnn.RMSNorm(F, eps=1e-6), tnn.RMSNorm(F, eps=1e-6)
            self.qkv, self.proj = tnn.Linear(F, 3 * F), tnn.Linear(F, F)
            self.fc1, self.fc2 = tnn.Linear(F, Hd), tnn.Linear(Hd, F)

        def forward(self, x):
            B = x.shape[0]
            q, k, v = self.qkv(self.n1(x)).view(B, T, 3, H, F // H).permute(2, 0, 3, 1, 4)
            a = tF.scaled_dot_product_attention(q, k, v, is_causal=True).transpose(1, 2).reshape(B, T, F)
            x = x + self.proj(a)
            return x + self.fc2(tF.gelu(self.fc1(self.n2(x)), approximate="tanh"))

    class LM(tnn.Module):
        def __init__(self):
            super().__init__()
            self.tok, self.pos = tnn.Embedding(V, F), tnn.Embedding(T, F)
            self.blocks = tnn.ModuleList(Block() for _ in range(L))
            self.norm = tnn.RMSNorm(F, eps=1e-6)

        def forward(self, ids, tg):
            x = self.tok(ids) + self.pos.weight[: ids.shape[1]]
            for b in self.blocks:
                x = b(x)
            logits = self.norm(x) @ self.tok.weight.t()  # tied head
            return tF.cross_entropy(logits.float().view(-1, V), tg.view(-1))

    torch.manual_seed(0)
    model = LM().to(dev)
    with torch.no_grad():  # GPT-style init: N(0, 0.02) weights, zero biases
        for mod in model.modules():
            if isinstance(mod, (tnn.Linear, tnn.Embedding)):
                mod.weight.normal_(0.0, 0.02)
            if isinstance(mod, tnn.Linear) and mod.bias is not None:
                mod.bias.zero_()
    run = model
    if n > 1:
        run = tnn.parallel.DistributedDataParallel(model, device_ids=[local], bucket_cap_mb=25,
                                                   gradient_as_bucket_view=True)
    opt = torch.optim.AdamW(model.parameters(), lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.0, fused=True)
    gen = torch.Generator().manual_seed(1234 + rank)
    pool = [torch.randint(0, V, (2, MICRO_BATCH, T), generator=gen).to(dev) for _ in range(4)]

    def step(b):
        opt.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = run(b[0], b[1])
        loss.backward()
        opt.step()
        return loss

    for i in range(args.warmup):
        step(pool[i % 4])
    torch.cuda.synchronize()
    if n > 1:
        dist.barrier()
    sampler, clock_path = _clock_sampler(local)
    time.sleep(0.3)
    if n > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for i in range(args.steps):
        loss = step(pool[i % 4])
    t1.record()
    torch.cuda.synchronize()
    if sampler is not None:
        sampler.terminate()
        sampler.wait()
    ms = torch.tensor([t0.elapsed_time(t1)], dtype=torch.float64, device=dev)
    if n > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms.item())
    if rank == 0:
        tokens = n * MICRO_BATCH * T * args.steps
        print(json.dumps({
            "impl": "torch-eager", "metric": METRIC, "value": tokens / (ms / 1e3), "unit": "tokens/s", "n_gpus": n,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "dtype": "bf16 autocast (fp32 parameters)", "data": "synthetic uniform token ids",
            "config": {"model": MODEL, "global_batch": n * MICRO_BATCH, "seq_len": T, "parallelism": f"dp{n}",
                       "what": "plain PyTorch comparison bar: torch.nn + SDPA + fused torch AdamW + torch DDP/NCCL"},
            "clocks": _clock_summary(clock_path), "final_loss": float(loss.item())}), flush=True)
    if n > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_zero3(args, pol, cc) -> int:
    """7B-class ZeRO-3: sharded weights / grads / moments, per-layer gathers and
    reduce-scatter fused with AdamW (underhfs_b200.parallel.zero3)."""
    import torch
    import torch.distributed as dist

    from underhfs_b200.distributed import init_process_group
    from underhfs_b200.ops._lib import core
    from underhfs_b200.parallel.zero3 import Zero3LM
    from underhfs_b200.train import PRESETS

    n, local = pol.world_size, pol.local_rank or 0
    if n > 1:
        init_process_group(pol)
    spec = PRESETS[cc["model"]]
    # Adam moments: the memory planner decides from this GPU's free memory and
    # the step's activation estimate (--offload host / device forces it)
    offload = {"auto": "auto", "host": True, "device": False}[args.offload]
    z = Zero3LM(spec, rank=pol.rank, world=n, device=f"cuda:{local}", lr=3e-4, betas=(0.9, 0.95), eps=1e-8,
                weight_decay=0.1, decoupled=True, seed=1234, offload_moments=offload,
                activation_bytes=spec.activation_bytes(cc["batch"], cc["seq"]))
    planner_note = ("" if z.offload_placement is None else
                    f"; memory planner placed the moments in {z.offload_placement.tier.value} "
                    f"({z.offload_placement.reason})")
    gen = torch.Generator().manual_seed(1234 + pol.rank)
    pool = [torch.randint(0, spec.vocab_size, (2, cc["batch"], cc["seq"]), generator=gen).cuda() for _ in range(2)]

    def barrier():
        if n > 1:
            dist.barrier()

    c = core()
    c.reset_launch_count()
    z.train_step(pool[0][0], pool[0][1])
    torch.cuda.synchronize()
    launches_per_step = c.launch_count()
    for i in range(args.warmup):
        z.train_step(pool[i % 2][0], pool[i % 2][1])
    torch.cuda.synchronize()
    barrier()
    sampler, clock_path = _clock_sampler(local)
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(args.steps):
        loss = z.train_step(pool[i % 2][0], pool[i % 2][1])
    end.record()
    torch.cuda.synchronize()
    barrier()
    if sampler is not None:
        sampler.terminate()
        sampler.wait()
    ms = start.elapsed_time(end)
    final_loss = float(loss.item())
    host = torch.empty((2, cc["batch"], cc["seq"]), dtype=torch.int64, pin_memory=True)
    host.copy_(pool[0].cpu())
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        dev = host.to(f"cuda:{local}", non_blocking=True)
        float(z.train_step(dev[0], dev[1]).item())
    e2e_s = time.perf_counter() - t0
    barrier()
    stats = torch.tensor([ms, e2e_s], dtype=torch.float64, device="cuda")
    if n > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    ms_max, e2e_max = stats.tolist()
    clocks = _clock_summary(clock_path)
    tokens = n * cc["batch"] * cc["seq"] * args.steps
    if pol.rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": tokens / (ms_max / 1e3), "unit": "tokens/s", "n_gpus": n,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic uniform token ids in [0,32000) from a fixed seed; random-init weights",
            "config": {"model": cc["desc"], "global_batch": n * cc["batch"], "micro_batch_per_gpu": cc["batch"],
                       "seq_len": cc["seq"], "parallelism": f"zero3-{n}",
                       "optimizer": "ZeRO-3 AdamW lr 3e-4, betas (0.9, 0.95), weight decay 0.1 (decoupled): "
                                    "per-unit reduce-scatter fused with AdamW on owned rows"
                                    + ("; Adam moments in pinned host RAM, staged per unit" if z.offload
                                       else "; Adam moments on the device") + planner_note,
                       "param_gather": "per-unit push all-gather over NVLink, prefetched one unit ahead",
                       "cuda_graph": False,
                       "l2": "no flush: per-step working set >> 126 MB L2"},
            "clocks": clocks,
            "e2e": {"value": tokens / e2e_max, "unit": "tokens/s",
                    "h2d_bytes_per_step": host.numel() * host.element_size(), "d2h_bytes_per_step": 4,
                    "api": "underhfs_b200.parallel.zero3.Zero3LM.train_step", "timer": "host wall clock, max over ranks"},
            "gpu_launches": launches_per_step * args.steps, "final_loss": final_loss,
        }), flush=True)
    z.close()
    if n > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


_REF_MICRO = """
import json, statistics, sys, time
from underhfs import _core as core

iters, warm, with_coll = int(sys.argv[1]), int(sys.argv[2]), sys.argv[3] == "1"

def wall(fn):
    for _ in range(warm):
        fn()
    ts = []
    for _ in range(iters):
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
    return statistics.median(ts)

def emit(**kw):
    print(json.dumps(kw), flush=True)

if not with_coll:
    n = 1 << 26
    for cls, name, es in (("CudaTensorF32", "fp32", 4), ("CudaTensorF16", "fp16", 2), ("CudaTensorBF16", "bf16", 2)):
        C = getattr(core, cls)
        a, b = C([1.5] * n, [n]), C([2.5] * n, [n])
        for op in ("add", "mul"):
            f = getattr(a, op)
            t = wall(lambda: f(b))
            emit(op=op, dtype=name, numel=n, seconds=t, gbs=3 * n * es / t / 1e9)
        del a, b
    for m in (1024, 4096, 8192):
        a, b = core.CudaTensorF32([1.0] * (m * m), [m, m]), core.CudaTensorF32([0.5] * (m * m), [m, m])
        t = wall(lambda: a.matmul(b))
        emit(op="matmul", dtype="fp32", m=m, n=m, k=m, seconds=t, tflops=2.0 * m ** 3 / t / 1e12)
        del a, b
    from underhfs.benchmarks import run_microbenchmarks
    for r in run_microbenchmarks(size=32, iterations=iters, warmup=warm, include_cuda=True):
        emit(op="run_microbenchmarks", **r.to_dict())
else:
    rank, world, uid, max_bytes = int(sys.argv[4]), int(sys.argv[5]), sys.argv[6], int(sys.argv[7])
    if rank == 0:
        # NCCL's bootstrap root lives in the process that made the id: rank 0
        # makes it here and hands it to the others through the file named in uid
        import os
        tmp = uid + ".tmp"
        with open(tmp, "w") as f:
            f.write(core.nccl_create_unique_id_hex())
        os.replace(tmp, uid)
        uid = open(uid).read().strip()
    pg = core.NcclProcessGroup(rank, world, uid)
    nbytes = 1024
    while nbytes <= max_bytes:
        count = nbytes // 4 // world * world
        vec = [1.0] * count
        for op, fn in (("all_reduce_sum", lambda: pg.all_reduce_sum(vec)),
                       ("reduce_scatter", lambda: pg.reduce_scatter(vec)),
                       ("all_gather", lambda: pg.all_gather(vec[: count // world]))):
            pg.barrier()
            t = wall(fn)
            emit(op=op, bytes=count * 4, seconds=t, rank=rank)
        nbytes *= 4
"""


def run_reference_micro(args) -> int:
    """The reference's own microbenchmarks on its stock native module (the
    collectives/GEMM/elementwise configuration): CudaTensor{F32,F16,BF16}
    add / mul at 2^26 elements, the cublasSgemm matmul at 1024/4096/8192 and,
    with N > 1 ranks, NcclProcessGroup all_reduce_sum / reduce_scatter /
    all_gather from 1 KiB up (host vectors in and out, as its API takes
    them), plus its ``run_microbenchmarks`` suite.  Every op of that API
    synchronises its stream before returning, so the time is the host wall
    clock around the call (median).  Runs in a subprocess rooted at
    baseline/_ref; each rank's subprocess sees only its own GPU
    (CUDA_VISIBLE_DEVICES), since the reference selects no device itself.
    Reference: benchmarks.py:98-120, cuda/kernels.cu:428-500,
    cpp/nccl_runtime.cpp:120-170."""
    ref = ROOT / "baseline" / "_ref"
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if not (ref / "underhfs" / "__init__.py").exists():
        if rank == 0:
            print(json.dumps({"impl": "reference", "config": "micro",
                              "unavailable": "reference not installed under baseline/_ref"}))
        return 0
    env = dict(os.environ, PYTHONPATH=str(ref), CUDA_VISIBLE_DEVICES=str(local))
    iters, warm = (args.steps if args.steps_given else 10), args.warmup
    rows = []

    def run(argv, timeout):
        proc = subprocess.run([sys.executable, "-c", _REF_MICRO, *map(str, argv)], cwd=str(ref), env=env,
                              capture_output=True, text=True, timeout=timeout)
        out = [json.loads(l) for l in proc.stdout.splitlines() if l.startswith("{")]
        if proc.returncode != 0:
            out.append({"error": (proc.stderr.strip().splitlines() or ["?"])[-1]})
        return out

    if world == 1:  # the single-GPU ops; with N > 1 ranks only the collectives run
        rows += run([iters, warm, 0], 900)
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("gloo", timeout=__import__("datetime").timedelta(seconds=600))
        max_bytes = int(os.environ.get("UNDERHFS_REF_COLL_MAX_BYTES", str(64 << 20)))
        argv = [iters, warm, 1, rank, world]
        if rank == 0:
            # rank 0's subprocess creates the NCCL id (its bootstrap root must
            # stay alive) and writes it to a file; the id then goes to the
            # other ranks through the process group
            id_file = Path(tempfile.mkdtemp()) / "nccl_id"
            proc = subprocess.Popen([sys.executable, "-c", _REF_MICRO, *map(str, argv + [id_file, max_bytes])],
                                    cwd=str(ref), env=env, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)
            deadline = time.time() + 120
            while not id_file.exists() and proc.poll() is None and time.time() < deadline:
                time.sleep(0.05)
            uid = [id_file.read_text().strip() if id_file.exists() else ""]
            dist.broadcast_object_list(uid, src=0)
            try:
                out, err = proc.communicate(timeout=1800)
            except subprocess.TimeoutExpired:
                proc.kill()
                out, err = proc.communicate()
            coll = [json.loads(l) for l in out.splitlines() if l.startswith("{")]
            if proc.returncode != 0:
                coll.append({"error": (err.strip().splitlines() or ["?"])[-1]})
            import shutil

            shutil.rmtree(id_file.parent, ignore_errors=True)
        else:
            uid = [None]
            dist.broadcast_object_list(uid, src=0)
            coll = run(argv + [uid[0] or "missing", max_bytes], 1800) if uid[0] else [
                {"error": "rank 0 could not create an NCCL id"}]
        gathered = [None] * world
        dist.all_gather_object(gathered, coll)
        dist.destroy_process_group()
        if rank == 0:
            by_key = {}
            for per_rank in gathered:
                for r in per_rank:
                    if "op" in r:
                        k = (r["op"], r["bytes"])
                        by_key[k] = max(by_key.get(k, 0.0), r["seconds"])
                    else:
                        rows.append(r)
            for (op, nbytes), t in sorted(by_key.items()):
                # bus bandwidth over the full vector (the gathered output for all_gather)
                busbw = {"all_reduce_sum": 2.0 * (world - 1) / world}.get(op, (world - 1) / world)
                rows.append({"op": op, "dtype": "fp32", "bytes": nbytes, "n_gpus": world, "seconds": t,
                             "bus_gbs": busbw * nbytes / t / 1e9})
    if rank == 0:
        for r in rows:
            print(json.dumps(dict({"impl": "reference", "config": "micro",
                                   "timer": "host wall clock around the synchronous call, median"}, **r)))
    return 0


def run_micro(args) -> int:
    """This framework on the same microbenchmarks: element-wise add / mul at
    2^26 elements (fp32, fp16, bf16), GEMM at 1024/4096/8192 (the tcgen05
    bf16 GEMM, and the exact fp32 SIMT GEMM for a like-for-like fp32 row),
    device time with CUDA events (mean after warm-up; inputs larger than L2
    for the element-wise ops); with N > 1 ranks the collective sweep
    (P2P all-reduce / reduce-scatter / all-gather over NVLink against NCCL)."""
    import torch

    from underhfs_b200.ops import kernels as K

    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        from underhfs_b200.parallel import collective_bench

        return collective_bench.main(["--min-kib", "1", "--max-mib", "1024", "--step", "4"])
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    iters = args.steps if args.steps_given else 20

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(iters):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / 1e3 / iters

    n = 1 << 26
    for dtype, name in ((torch.float32, "fp32"), (torch.float16, "fp16"), (torch.bfloat16, "bf16")):
        a = torch.full((n,), 1.5, dtype=dtype, device=dev)
        b = torch.full((n,), 2.5, dtype=dtype, device=dev)
        for op, code in (("add", K.OP_ADD), ("mul", K.OP_MUL)):
            t = timed(lambda: K.ew_binary(code, a, b))
            print(json.dumps({"impl": "ours", "config": "micro", "op": op, "dtype": name, "numel": n, "seconds": t,
                              "gbs": 3 * n * a.element_size() / t / 1e9, "timer": "CUDA events"}))
        del a, b
    for m in (1024, 4096, 8192):
        for dtype, name, fn in ((torch.bfloat16, "bf16", K.matmul_bf16), (torch.float32, "fp32", K.matmul_f32)):
            a = torch.randn(m, m, device=dev).to(dtype)
            b = torch.randn(m, m, device=dev).to(dtype)
            t = timed(lambda: fn(a, b))
            print(json.dumps({"impl": "ours", "config": "micro", "op": "matmul", "dtype": name, "m": m, "n": m, "k": m,
                              "seconds": t, "tflops": 2.0 * m ** 3 / t / 1e12, "timer": "CUDA events"}))
    return 0


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=int(os.environ.get("WORLD_SIZE", "1")))
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=("ours", "reference", "torch-eager"), default="ours",
                    help="torch-eager: the labelled plain-PyTorch comparison bar (not this framework)")
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--offload", choices=("auto", "host", "device"), default="auto",
                    help="7b-zero3 Adam moments: the memory planner decides (auto) or force pinned host / device")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="125m-ddp",
                    help="125m-ddp is the headline run; the sharded configurations are measured the same way")
    args = ap.parse_args()
    args.steps_given = "--steps" in sys.argv
    if args.config == "micro":
        if "--warmup" not in sys.argv:
            args.warmup = 3
        return run_reference_micro(args) if args.impl == "reference" else run_micro(args)
    if args.config == "tiny-cpu":
        if "--warmup" not in sys.argv:
            args.warmup = 3
        return run_reference_tiny(args) if args.impl == "reference" else run_tiny_cpu(args)
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.impl == "torch-eager":
        return run_torch_eager(args)
    return run_ours(args)


if __name__ == "__main__":
    raise SystemExit(main())
