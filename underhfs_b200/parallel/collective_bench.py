"""Collective sweep: this repo's NVLink kernels against NCCL, one process per GPU.

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        -m underhfs_b200.parallel.collective_bench [--min-kib 1] [--max-mib 1024] [--step 4]

For all-reduce, reduce-scatter and all-gather on fp32 and bf16 buffers of
1 KiB .. 1 GiB, each size is timed with CUDA events on the launching stream
(3 warm-ups, then a fixed number of back-to-back calls), the per-call time is
the maximum over ranks, and rank 0 prints one JSON line per (op, dtype, size,
implementation) plus a markdown table.  Bus bandwidth follows the usual
convention: all-reduce moves 2 (W-1)/W of the buffer per GPU, reduce-scatter
and all-gather (W-1)/W; the NVLink 5 reference is 900 GB/s per direction.

"ours" is the peer-load / peer-store kernel family of csrc/runtime/comm.cu over
a CUDA-IPC symmetric heap; "nccl" is torch.distributed with the NCCL backend on
ordinary tensors.  Results are checked against NCCL at every size.
Reference: the reference times its host-staged NCCL calls with a host clock
(src/underhfs/benchmarks.py:98-120, cpp/nccl_runtime.cpp:52-79).
"""

from __future__ import annotations

import argparse
import json
import os
from datetime import timedelta

import torch
import torch.distributed as dist

from underhfs_b200.ops._lib import core
from underhfs_b200.parallel.symmetric import SymmetricBuffer

LINK_GBS = 900.0


def _blocks(nbytes: int) -> int:
    """CTAs per collective launch: few for latency-bound sizes, many for peer-load bandwidth."""
    if nbytes <= 256 << 10:
        return 8
    if nbytes <= 4 << 20:
        return 64
    if nbytes <= 64 << 20:
        return 128
    return 256


def _time(fn, iters: int) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b) / iters], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--min-kib", type=int, default=1)
    ap.add_argument("--max-mib", type=int, default=1024)
    ap.add_argument("--step", type=int, default=4, help="size multiplier between points (2 = every power of two)")
    ap.add_argument("--ops", default="allreduce,reduce_scatter,allgather",
                    help="comma list of allreduce, allreduce_wire (fp32 over a bf16 wire), reduce_scatter, allgather")
    ap.add_argument("--fused-params", default="",
                    help="comma list of parameter counts (e.g. 125e6,1.3e9): time the fused ZeRO-2 step "
                         "(reduce-scatter + AdamW + all-gather) and report it against its roofline")
    args = ap.parse_args(argv)
    if args.fused_params:
        return fused_step_bench([int(float(v)) for v in args.fused_params.split(",")])

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", torch.cuda.current_device()))
    c = core()
    max_bytes = args.max_mib << 20
    sym = SymmetricBuffer(2 * max_bytes + (4 << 20), rank=rank, world=world)
    stream = torch.cuda.current_stream().cuda_stream
    sizes = []
    s = args.min_kib << 10
    while s <= max_bytes:
        sizes.append(s)
        s *= args.step
    rows = []
    gen = torch.Generator(device="cuda").manual_seed(1234 + rank)
    try:
        for dtype in (torch.float32, torch.bfloat16):
            bf16 = dtype == torch.bfloat16
            esize = 2 if bf16 else 4
            for nbytes in sizes:
                unit = 16 * world
                nbytes = max(unit, nbytes // unit * unit)
                n = nbytes // esize
                iters = max(5, min(100, (256 << 20) // nbytes))
                blocks = _blocks(nbytes)
                x = torch.randn(n, device="cuda", generator=gen).to(dtype)
                off_in, off_out = 0, max_bytes + (2 << 20)
                buf = sym.tensor(n, dtype, offset_bytes=off_in)
                out = sym.tensor(n, dtype, offset_bytes=off_out)
                for op in args.ops.split(","):
                    if op == "allreduce_wire" and bf16:
                        continue  # the wire variant reduces fp32 gradients
                    if op == "allreduce_wire":
                        # fp32 gradients over a bf16 wire; the staging span follows the data
                        ref = x.clone()
                        dist.all_reduce(ref)
                        buf.copy_(x)
                        c.comm_allreduce_f32_wire_bf16(sym.heap, off_in, off_out, n, 1.0, blocks, stream)
                        torch.cuda.synchronize()
                        err = (buf.float() - ref.float()).abs().max().item() / max(1.0, ref.float().abs().max().item())
                        t_ours = _time(lambda: c.comm_allreduce_f32_wire_bf16(sym.heap, off_in, off_out, n,
                                                                              1.0 / world, blocks, stream), iters)
                        nccl_t = x.clone()
                        t_nccl = _time(lambda: dist.all_reduce(nccl_t, op=dist.ReduceOp.AVG), iters)
                        factor = 2.0 * (world - 1) / world  # bus bytes counted at fp32 width
                    elif op == "allreduce":
                        ref = x.clone()
                        dist.all_reduce(ref)
                        buf.copy_(x)
                        fn = c.comm_allreduce_bf16 if bf16 else c.comm_allreduce_f32
                        fn(sym.heap, off_in, n, 1.0, blocks, stream)
                        torch.cuda.synchronize()
                        err = (buf.float() - ref.float()).abs().max().item() / max(1.0, ref.float().abs().max().item())
                        # timed calls average (scale 1/W) so repeated in-place reductions stay finite
                        t_ours = _time(lambda: fn(sym.heap, off_in, n, 1.0 / world, blocks, stream), iters)
                        nccl_t = x.clone()
                        t_nccl = _time(lambda: dist.all_reduce(nccl_t, op=dist.ReduceOp.AVG), iters)
                        factor = 2.0 * (world - 1) / world
                    elif op == "reduce_scatter":
                        ref = torch.empty(n // world, device="cuda", dtype=dtype)
                        dist.reduce_scatter_tensor(ref, x.clone())
                        buf.copy_(x)
                        c.comm_reduce_scatter(sym.heap, off_in, off_out, n, bf16, 1.0, blocks, stream)
                        torch.cuda.synchronize()
                        got = out[: n // world]
                        err = (got.float() - ref.float()).abs().max().item() / max(1.0, ref.float().abs().max().item())
                        t_ours = _time(lambda: c.comm_reduce_scatter(sym.heap, off_in, off_out, n, bf16, 1.0, blocks,
                                                                     stream), iters)
                        src = x.clone()
                        dst = torch.empty(n // world, device="cuda", dtype=dtype)
                        t_nccl = _time(lambda: dist.reduce_scatter_tensor(dst, src), iters)
                        factor = (world - 1) / world
                    else:  # allgather: rank r owns bytes [r*shard, (r+1)*shard)
                        shard = nbytes // world
                        shard_n = n // world
                        ref = torch.empty(n, device="cuda", dtype=dtype)
                        dist.all_gather_into_tensor(ref, x[:shard_n].contiguous())
                        buf.copy_(x)
                        buf[rank * shard_n:(rank + 1) * shard_n].copy_(x[:shard_n])
                        c.comm_allgather(sym.heap, off_in, shard, blocks, stream)
                        torch.cuda.synchronize()
                        err = (buf.float() - ref.float()).abs().max().item()
                        t_ours = _time(lambda: c.comm_allgather(sym.heap, off_in, shard, blocks, stream), iters)
                        part = x[:shard_n].contiguous()
                        gathered = torch.empty(n, device="cuda", dtype=dtype)
                        t_nccl = _time(lambda: dist.all_gather_into_tensor(gathered, part), iters)
                        factor = (world - 1) / world
                    st = c.device_status(True)
                    assert st["code"] == 0, st
                    tol = 2e-2 if (bf16 or op == "allreduce_wire") else 1e-5
                    assert err <= tol, (op, dtype, nbytes, err)
                    for impl, t in (("ours", t_ours), ("nccl", t_nccl)):
                        bus = nbytes * factor / (t * 1e-3) / 1e9
                        rows.append({"op": op, "dtype": "bf16" if bf16 else "fp32", "bytes": nbytes, "impl": impl,
                                     "n_gpus": world, "ms": t, "bus_gbs": bus, "frac_of_900": bus / LINK_GBS,
                                     "max_rel_err_vs_nccl": err})
                del x
        if rank == 0:
            for r in rows:
                print(json.dumps(r), flush=True)
            print(f"\n| op | dtype | size | ours ms | ours bus GB/s | NCCL ms | NCCL bus GB/s | ours / NCCL |")
            print("|---|---|---|---|---|---|---|---|")
            for i in range(0, len(rows), 2):
                o, n_ = rows[i], rows[i + 1]
                size = o["bytes"]
                label = f"{size >> 20} MiB" if size >= 1 << 20 else f"{size >> 10} KiB"
                print(f"| {o['op']} | {o['dtype']} | {label} | {o['ms']:.4f} | {o['bus_gbs']:.1f} | {n_['ms']:.4f} | "
                      f"{n_['bus_gbs']:.1f} | {n_['ms'] / o['ms']:.2f} |")
    finally:
        torch.cuda.synchronize()
        dist.barrier()
        sym.close()
        dist.destroy_process_group()
    return 0


PEER_GBS = 770.0   # measured peer copy per direction per GPU on this class of node
HBM_GBS = 6537.0   # measured device copy bandwidth (read + write)


def fused_step_bench(param_counts: list[int]) -> int:
    """The ZeRO-2 step kernel (rs_adamw_ag_kernel) on n fp32 gradients / bf16
    parameters in symmetric memory.  Per GPU and direction it moves
    (W-1)/W x 6n bytes over NVLink (fp32 shard reads + bf16 parameter pushes
    each way) and about 6n + 24n/W bytes of HBM (gradients and parameters, plus
    fp32 master / moments of the owned shard read and written); the roofline
    time is the larger of the two at the measured rates, and the line reports
    achieved / roofline."""
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", torch.cuda.current_device()))
    c = core()
    stream = torch.cuda.current_stream().cuda_stream
    try:
        for n in param_counts:
            unit = 8 * world
            n = (n + unit - 1) // unit * unit
            shard = n // world
            gsym = SymmetricBuffer(n * 4 + 4096, rank=rank, world=world)
            psym = SymmetricBuffer(n * 2 + 4096, rank=rank, world=world)
            grads = gsym.tensor(n, torch.float32, offset_bytes=0)
            params = psym.tensor(n, torch.bfloat16, offset_bytes=0)
            grads.normal_()
            params.zero_()
            master = torch.randn(shard, device="cuda") * 0.02
            m = torch.zeros(shard, device="cuda")
            v = torch.zeros(shard, device="cuda")
            step = torch.zeros((), dtype=torch.int32, device="cuda")
            blocks = 132

            def run():
                c.comm_rs_adamw_ag(gsym.heap, 0, psym.heap, 0, rank * shard, shard, master.data_ptr(), m.data_ptr(),
                                   v.data_ptr(), 1e-4, 0.9, 0.95, 1e-8, 0.1, 1.0 / world, True, step.data_ptr(),
                                   blocks, stream)

            ms = _time(run, 10)
            st = c.device_status(True)
            assert st["code"] == 0, st
            link_s = (world - 1) / world * 6.0 * n / (PEER_GBS * 1e9)
            hbm_s = (6.0 * n + 24.0 * n / world) / (HBM_GBS * 1e9)
            bound_ms = 1e3 * max(link_s, hbm_s)
            if rank == 0:
                print(json.dumps({"op": "zero2_rs_adamw_ag", "params": n, "n_gpus": world, "ms": ms,
                                  "roofline_ms": bound_ms, "bound": "nvlink" if link_s >= hbm_s else "hbm",
                                  "frac_of_roofline": bound_ms / ms}), flush=True)
            gsym.close()
            psym.close()
    finally:
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
