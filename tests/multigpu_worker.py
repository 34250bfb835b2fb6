"""Worker for tests/test_multigpu.py (one process per GPU, launched by torchrun).

    python -m torch.distributed.run --nproc-per-node 2 tests/multigpu_worker.py {allreduce|ddp|zero}

Exits 0 and prints "OK <case>" on rank 0 when the fused NVLink kernels agree
with NCCL / the single-buffer reference; any mismatch raises.
"""

from __future__ import annotations

import os
import sys
from datetime import timedelta
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))


def _setup():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", torch.cuda.current_device()))
    return rank, world


def case_allreduce(rank: int, world: int) -> None:
    from underhfs_b200.ops._lib import core
    from underhfs_b200.parallel.symmetric import SymmetricBuffer

    sym = SymmetricBuffer(64 << 20, rank=rank, world=world)
    buf = sym.tensor((64 << 20) // 4 - 1024, torch.float32)
    stream = torch.cuda.current_stream().cuda_stream
    for n in (4, 1000, 4096 * 1024 + 4, (25 << 20) // 4, (64 << 20) // 4 - 1024):
        gen = torch.Generator(device="cuda").manual_seed(1000 + rank * 7 + n % 97)
        x = torch.randn(n, device="cuda", generator=gen)
        buf[:n].copy_(x)
        ref = x.clone()
        dist.all_reduce(ref)
        ref /= world
        off = buf.data_ptr() - sym.heap.data_ptr(rank)
        for blocks in (8, 64):
            buf[:n].copy_(x)
            core().comm_allreduce_f32(sym.heap, off, n, 1.0 / world, blocks, stream)
            torch.cuda.synchronize()
            err = (buf[:n] - ref).abs().max().item()
            assert err < 1e-5 * max(1.0, ref.abs().max().item()), (n, blocks, err)
    st = core().device_status(True)
    assert st["code"] == 0, st


def _model(seed: int = 0, max_seq_len: int = 256):
    from underhfs_b200.nn import TransformerLM

    m = TransformerLM(vocab_size=1024, max_seq_len=max_seq_len, features=256, hidden_features=1024, layers=2, heads=4,
                      tied=True, init="normal", seed=seed)
    m.to(f"cuda:{torch.cuda.current_device()}", dtype="bf16")
    return m


def case_ddp(rank: int, world: int) -> None:
    from underhfs_b200.distributed import DistributedDataParallel, policy_from_env

    gen = torch.Generator().manual_seed(100 + rank)
    ids = torch.randint(0, 1024, (2, 256), generator=gen).cuda()
    tg = torch.roll(ids, -1, 1)
    ref_model = _model()
    ref_model.zero_grad()
    ref_model(ids, tg).backward()
    ref = ref_model.flat.grads.clone()
    dist.all_reduce(ref)
    ref /= world
    model = _model()
    ddp = DistributedDataParallel(model, policy_from_env(), bucket_mb=0.25)  # small buckets: many overlap launches
    for _ in range(2):  # second pass checks the epochs of reused buckets
        model.zero_grad()
        ddp(ids, tg).backward()
        ddp.synchronize_gradients()
        torch.cuda.synchronize()
        err = ((model.flat.grads - ref).abs().max() / ref.abs().max()).item()
        assert err < 1e-4, err
    # optimizer step split around the last (embedding) all-reduce: the same
    # weights as one step after every reduction.  The weight-gradient GEMMs
    # and the dQ accumulation add with fp32 atomics in a varying order, and a
    # last-bit change of an fp32 sum can flip a bf16 activation by one ulp, so
    # two identical runs differ slightly: the split run is compared with the
    # spread of two unsplit runs.  eps 1e-3 keeps Adam from turning that noise
    # into sign flips of near-zero updates.
    from underhfs_b200.optim import FusedAdamW

    outs = []
    for split in (False, False, True):
        m2 = _model()
        d2 = DistributedDataParallel(m2, policy_from_env(), bucket_mb=0.25)
        opt = FusedAdamW(m2.parameters(), lr=1e-3, betas=(0.9, 0.95), eps=1e-3, weight_decay=0.1, decoupled=True)
        for _ in range(2):
            m2.zero_grad()
            d2(ids, tg).backward()
            if split:
                boundary = d2.synchronize_gradients(defer_tail=True)
                assert boundary > 0  # the tied embedding is reduced last
                opt.step_split(boundary, d2.wait_gradients)
            else:
                d2.synchronize_gradients()
                opt.step()
        torch.cuda.synchronize()
        outs.append(m2.flat.master.clone())
    moved = (outs[0] - _model().flat.master).abs().max().item()  # how far two steps moved the weights
    spread = (outs[0] - outs[1]).abs().max().item()  # two unsplit runs
    diff = max((outs[2] - o).abs().max().item() for o in outs[:2])
    if rank == 0:
        print(f"split step: moved {moved:.3e}, unsplit spread {spread:.3e}, split diff {diff:.3e}", flush=True)
    assert diff <= 4.0 * spread + 1e-4 * moved, (diff, spread, moved)
    with ddp.no_sync():
        model.zero_grad()
        ddp(ids, tg).backward()
        ddp.synchronize_gradients()
    torch.cuda.synchronize()
    local = ((model.flat.grads - ref_model.flat.grads).abs().max() / ref_model.flat.grads.abs().max()).item()
    assert local < 1e-4, local  # no_sync keeps local gradients
    from underhfs_b200.ops._lib import core

    assert core().device_status(True)["code"] == 0


def case_ddp_wire(rank: int, world: int) -> None:
    """DDP with bf16 transport (UNDERHFS_DDP_WIRE=bf16): the averaged gradients
    match NCCL's fp32 all-reduce to bf16 rounding and are identical on every
    rank (replicas stay in step)."""
    os.environ["UNDERHFS_DDP_WIRE"] = "bf16"
    from underhfs_b200.distributed import DistributedDataParallel, policy_from_env

    gen = torch.Generator().manual_seed(700 + rank)
    ids = torch.randint(0, 1024, (2, 256), generator=gen).cuda()
    tg = torch.roll(ids, -1, 1)
    ref_model = _model()
    ref_model.zero_grad()
    ref_model(ids, tg).backward()
    ref = ref_model.flat.grads.clone()
    dist.all_reduce(ref)
    ref /= world
    model = _model()
    ddp = DistributedDataParallel(model, policy_from_env(), bucket_mb=0.25)
    assert ddp._bucketer.wire
    for _ in range(2):
        model.zero_grad()
        ddp(ids, tg).backward()
        ddp.synchronize_gradients()
        torch.cuda.synchronize()
        g = model.flat.grads[: ref.numel()]
        # each contribution and the result are rounded to bf16 (2^-9 relative)
        assert ((g - ref).norm() / ref.norm()).item() < 1e-2
        assert ((g - ref).abs().max() / ref.abs().max()).item() < 2e-2
        gathered = [torch.empty_like(g) for _ in range(world)]
        dist.all_gather(gathered, g)
        assert all(torch.equal(gathered[0], x) for x in gathered[1:]), "ranks disagree"
    from underhfs_b200.ops._lib import core

    assert core().device_status(True)["code"] == 0
    del os.environ["UNDERHFS_DDP_WIRE"]


def case_nvls(rank: int, world: int) -> None:
    """DDP gradients reduced in the NVSwitch (multimem) match NCCL's.

    A rank whose memory is bound to an NVLink multicast object must not die
    while a peer still uses it: every rank finishes its GPU work, the ranks
    agree on the outcome with a collective, release the buffers and meet at a
    barrier before either reports a failure."""
    import gc

    os.environ["UNDERHFS_NVLS"] = "1"
    from underhfs_b200.distributed import DistributedDataParallel, policy_from_env
    from underhfs_b200.ops._lib import core

    problems = []
    ddp = model = None
    try:
        gen = torch.Generator().manual_seed(400 + rank)
        ids = torch.randint(0, 1024, (2, 256), generator=gen).cuda()
        tg = torch.roll(ids, -1, 1)
        ref_model = _model()
        ref_model.zero_grad()
        ref_model(ids, tg).backward()
        ref = ref_model.flat.grads.clone()
        dist.all_reduce(ref)
        ref /= world
        model = _model()
        # from here on this rank's gradients may be bound to the multicast object
        ddp = DistributedDataParallel(model, policy_from_env(), bucket_mb=0.25)
        if ddp._bucketer.mc == 0:
            problems.append("no multicast address: NVLS not in use")
        else:
            for _ in range(2):
                model.zero_grad()
                ddp(ids, tg).backward()
                ddp.synchronize_gradients()
                torch.cuda.synchronize()
                err = ((model.flat.grads[: ref.numel()] - ref).abs().max() / ref.abs().max()).item()
                if not err < 1e-4:
                    problems.append(f"gradient error {err}")
        torch.cuda.synchronize()
        if core().device_status(True)["code"] != 0:
            problems.append("device status")
    except Exception as exc:  # recorded, never raised before the ranks agree
        problems.append(f"{type(exc).__name__}: {exc}")
    # every rank reaches the agreement, the release and the barrier, whatever
    # happened above, so no rank exits while a peer still uses its memory
    ok = torch.tensor([0 if problems else 1], device="cuda")
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)  # every rank learns the outcome
    del ddp, model
    gc.collect()
    torch.cuda.synchronize()
    dist.barrier()
    assert ok.item() == 1, (rank, problems)


def case_zero(rank: int, world: int) -> None:
    from underhfs_b200.optim import FusedAdamW, ZeroAwareAdamW, ZeroShard

    gen = torch.Generator().manual_seed(200 + rank)
    ids = torch.randint(0, 1024, (2, 256), generator=gen).cuda()
    tg = torch.roll(ids, -1, 1)
    # eps well above the gradient noise: AdamW's first steps move every weight by
    # ~lr * sign(g), so with eps=1e-8 a near-zero gradient whose fp32 sum order
    # differs (atomic weight-gradient accumulation) flips a whole 2*lr step
    kw = dict(lr=1e-2, betas=(0.9, 0.95), eps=1e-3, weight_decay=0.1, decoupled=True)
    ref_model = _model()
    ref_opt = FusedAdamW(ref_model.parameters(), **kw)
    model = _model()
    opt = ZeroAwareAdamW(model.parameters(), ZeroShard(rank, world), stage=2, **kw)
    for _ in range(3):
        ref_model.zero_grad()
        ref_model(ids, tg).backward()
        dist.all_reduce(ref_model.flat.grads)
        ref_model.flat.grads /= world
        ref_opt.step()
        model.zero_grad()
        model(ids, tg).backward()
        opt.step()
        torch.cuda.synchronize()
        a = model.flat.params.float()
        b = ref_model.flat.params.float()
        err = ((a - b).abs().max() / b.abs().max()).item()
        assert err < 2e-2, err
    # every rank holds identical full parameters after the fused all-gather
    p = model.flat.params.float().sum().reshape(1)
    allp = [torch.zeros_like(p) for _ in range(world)]
    dist.all_gather(allp, p)
    assert all(torch.equal(allp[0], q) for q in allp)


def case_zero3(rank: int, world: int) -> None:
    """ZeRO-3 (sharded weights, per-unit gather, RS fused with AdamW) against a
    replicated model with FusedAdamW on all-reduced gradients."""
    from underhfs_b200.nn import TransformerLM
    from underhfs_b200.optim import FusedAdamW
    from underhfs_b200.parallel.zero3 import Zero3LM

    kw = dict(lr=1e-2, betas=(0.9, 0.95), eps=1e-3, weight_decay=0.1, decoupled=True)
    for tied, fused, offload in ((True, True, False), (False, True, False), (True, False, False),
                                 (False, True, True)):
        cpu = TransformerLM(vocab_size=1024, max_seq_len=256, features=256, hidden_features=1024, layers=3, heads=4,
                            tied=tied, init="normal", seed=3)
        state = {n: p._data.detach().float().clone() for n, p in cpu.named_parameters()}
        ref = TransformerLM(vocab_size=1024, max_seq_len=256, features=256, hidden_features=1024, layers=3, heads=4,
                            tied=tied, init="normal", seed=3)
        ref.to(f"cuda:{torch.cuda.current_device()}", dtype="bf16")
        ref_opt = FusedAdamW(ref.parameters(), **kw)
        z = Zero3LM(cpu.spec, rank=rank, world=world, state=state, blocks=16, fused_gather=fused,
                    offload_moments=offload, **kw)
        assert z.fused == fused and z.offload == offload and (z.m.device.type == "cpu") == offload
        gen = torch.Generator().manual_seed(300 + rank)
        for _ in range(3):
            ids = torch.randint(0, 1024, (2, 256), generator=gen).cuda()
            tg = torch.roll(ids, -1, 1)
            ref.zero_grad()
            ref(ids, tg).backward()
            dist.all_reduce(ref.flat.grads)
            ref.flat.grads /= world
            ref_opt.step()
            loss = z.train_step(ids, tg)
        torch.cuda.synchronize()
        from underhfs_b200.ops._lib import core

        st = core().device_status(True)
        assert st["code"] == 0, st
        assert torch.isfinite(loss).item()
        full = z.full_state()
        for name, slot in ref.flat.by_name.items():
            a = full[name].reshape(-1)
            b = ref.flat.master[slot.offset: slot.offset + slot.numel].float().cpu()
            # floor the scale: k_proj.bias has an exactly-zero gradient (a per-row
            # shift of the scores) and stays at rounding-noise size
            err = ((a - b).abs().max() / b.abs().max().clamp_min(1e-3)).item()
            assert err < 2e-2, (tied, fused, offload, name, err)
        z.close()


def case_zero3_api(rank: int, world: int) -> None:
    """ZeRO-3 through the public surface: ZeroAwareAdamW(stage=3) on a
    TransformerLM (zero_grad / forward / backward / step) and Trainer with
    zero_stage=3, against the replicated model with FusedAdamW on all-reduced
    gradients."""
    from underhfs_b200.nn import TransformerLM
    from underhfs_b200.optim import FusedAdamW, ZeroAwareAdamW, ZeroShard

    kw = dict(lr=1e-2, betas=(0.9, 0.95), eps=1e-3, weight_decay=0.1, decoupled=True)
    dev = f"cuda:{torch.cuda.current_device()}"

    def model():
        m = TransformerLM(vocab_size=1024, max_seq_len=256, features=256, hidden_features=1024, layers=2, heads=4,
                          tied=True, init="normal", seed=9)
        return m.to(dev, dtype="bf16")

    ref = model()
    ref_opt = FusedAdamW(ref.parameters(), **kw)
    m = model()
    opt = ZeroAwareAdamW(m.parameters(), ZeroShard(rank, world), stage=3, offload="device", **kw)
    gen = torch.Generator().manual_seed(500 + rank)
    for _ in range(3):
        ids = torch.randint(0, 1024, (2, 256), generator=gen).cuda()
        tg = torch.roll(ids, -1, 1)
        ref.zero_grad()
        ref(ids, tg).backward()
        dist.all_reduce(ref.flat.grads)
        ref.flat.grads /= world
        ref_opt.step()
        opt.zero_grad()
        m(ids, tg).backward()
        opt.step()
    torch.cuda.synchronize()
    got, want = m.state_dict(as_tensors=True), ref.state_dict(as_tensors=True)
    for name in want:
        err = ((got[name] - want[name]).abs().max() / want[name].abs().max().clamp_min(1e-3)).item()
        assert err < 2e-2, (name, err)
    opt.zero3.close()

    from underhfs_b200.data import SyntheticTokens
    from underhfs_b200.distributed import policy_from_env
    from underhfs_b200.train import TrainConfig, Trainer, build_model

    cfg = TrainConfig(model="125m", batch=2, seq_len=256, zero_stage=3, weight_decay=0.1)
    tr = Trainer(build_model(cfg, device=dev), cfg, policy=policy_from_env(zero_stage=3))
    src = SyntheticTokens(32000, cfg.batch, cfg.seq_len, seed=3, rank=rank)
    host = torch.empty((2, cfg.batch, cfg.seq_len), dtype=torch.int64, pin_memory=True)
    src.next_host(host)  # one batch per rank, stepped on repeatedly: the loss must fall
    losses = [tr.step_from_host(host) for _ in range(4)]
    tr.release()
    assert all(l == l for l in losses) and losses[-1] < losses[0], losses


def case_native(rank: int, world: int) -> None:
    """The reference-style native NCCL group (host lists and device pointers),
    bootstrapped through UNDERHFS_NCCL_UNIQUE_ID or the torch store."""
    from underhfs_b200.distributed import native_nccl_group, policy_from_env

    g = native_nccl_group(policy_from_env())
    assert g.rank == rank and g.world_size == world
    out = g.all_reduce_sum([1.0 + rank, 2.0])
    assert out == [sum(1.0 + r for r in range(world)), 2.0 * world], out
    x = torch.full((1 << 20,), float(rank + 1), device="cuda")
    torch.cuda.synchronize()
    g.all_reduce_ptr(x.data_ptr(), x.numel(), 0, 0)
    torch.cuda.synchronize()
    assert torch.all(x == sum(r + 1 for r in range(world))).item()
    g.barrier()


def case_cp(rank: int, world: int) -> None:
    """Context parallelism: every rank holds a zigzag shard of the same
    sequences; the group-averaged loss and gradients match one rank running
    the whole sequences."""
    from underhfs_b200.parallel.context import enable_context_parallel, shard_sequence

    T = 1024
    gen = torch.Generator().manual_seed(300)
    ids = torch.randint(0, 1024, (2, T), generator=gen).cuda()
    tg = torch.roll(ids, -1, 1)
    ref_model = _model(max_seq_len=T)
    ref_model.zero_grad()
    ref_loss = ref_model(ids, tg)
    ref_loss.backward()
    ref = ref_model.flat.grads.clone()
    model = _model(max_seq_len=T)
    enable_context_parallel(model.engine, T)
    model.zero_grad()
    loss = model(shard_sequence(ids, rank, world), shard_sequence(tg, rank, world))
    loss.backward()
    torch.cuda.synchronize()
    g = model.flat.grads.clone()
    dist.all_reduce(g)
    g /= world
    lsum = torch.tensor([float(loss.item())], device="cuda")
    dist.all_reduce(lsum)
    lerr = abs(lsum.item() / world - ref_loss.item()) / abs(ref_loss.item())
    gerr = ((g - ref).abs().max() / ref.abs().max()).item()
    assert lerr < 2e-3 and gerr < 3e-2, (lerr, gerr)
    # the same through the public trainer: full sequences in, sharded per rank
    from underhfs_b200.distributed import policy_from_env
    from underhfs_b200.train import TrainConfig, Trainer

    cfg = TrainConfig(model="125m", batch=2, seq_len=T, context_parallel=True, cuda_graph=True)
    tmodel = _model(max_seq_len=T)
    trainer = Trainer(tmodel, cfg, policy=policy_from_env())
    assert trainer.cp is not None and not cfg.cuda_graph
    host = torch.stack([ids, tg]).cpu().pin_memory()
    first = trainer.step_from_host(host)
    for _ in range(3):
        last = trainer.step_from_host(host)
    assert last < first, (first, last)
    trainer.release()
    from underhfs_b200.ops._lib import core

    assert core().device_status(True)["code"] == 0


def main() -> int:
    case = sys.argv[1]
    rank, world = _setup()
    try:
        cases = {"allreduce": case_allreduce, "ddp": case_ddp, "zero": case_zero, "zero3": case_zero3, "zero3_api": case_zero3_api, "ddp_wire": case_ddp_wire,
                 "native": case_native, "cp": case_cp, "nvls": case_nvls}
        cases[case](rank, world)
        dist.barrier()
        if rank == 0:
            print(f"OK {case}", flush=True)
    finally:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
