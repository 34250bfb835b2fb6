"""ZeRO-3 training of a TransformerLM: parameters, gradients and optimizer
state are all sharded; each unit's weights are gathered just before use.

A *unit* is the embedding tables, one transformer block, or the tail (final
norm and, untied, the head).  Rank r owns rows [r*N/W, (r+1)*N/W) of every
parameter matrix of every unit (a vector of length N counts as N x 1), so a
unit's all-gather is balanced over the ranks and every rank holds a slice of
every weight.  Per rank the model costs total/W of (bf16 weights + fp32
master + two fp32 moments), plus one gathered copy and one fp32 gradient
buffer for the embeddings, the tail, and a ring of two blocks.

Forward, per unit:  push all-gather of the unit's row segments into every
    rank's gather slot (csrc/runtime/comm.cu: gather_segments_kernel), then the
    usual engine kernels read the gathered weights.
Backward, per unit: weight gradients accumulate in fp32 into the unit's
    gradient slot (the same fused GEMM epilogues as the flat engine); then one
    kernel reduces every rank's gradients for the rows this rank owns and
    applies AdamW to the owned fp32 master / moments and bf16 shard
    (rs_adamw_segments_kernel).  Nothing is all-gathered after the update: the
    next forward gathers the new weights.

The two slots of the block ring are reused every second block; the gather
and reduce kernels open and close with a cross-rank barrier, so no rank
overwrites a slot a peer is still reading.

Moment offload: with ``offload_moments="auto"`` the memory planner
(runtime.MemoryPlanner.place_optimizer_state) decides from this GPU's free
memory, less the step's activation estimate, whether the two fp32 moments of
the shard stay in device memory or go to pinned host RAM; ``True`` / ``False``
force the choice.  Offloaded, the fp32 Adam moments of the shard
live in pinned host RAM.  A unit's moments (a contiguous shard range) are
copied into one of two device staging slots on a copy stream when the unit's
backward begins, the fused reduce-scatter + AdamW kernel updates them there,
and they are copied back right after it (on a second copy stream: the two
directions overlap), so the PCIe transfers overlap the backward of the
neighbouring units.  Device memory for the moments drops
from the whole shard to two units.

The reference has no ZeRO-3 (its ZeroAwareAdamW is a single-process stub,
optim.py:216-225).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from underhfs_b200.models.transformer import LMEngine, LMSpec, build_layout
from underhfs_b200.ops import kernels as K
from underhfs_b200.ops._lib import core
from underhfs_b200.parallel.symmetric import SymmetricBuffer
from underhfs_b200.utils import nvtx


def _round_up(n: int, a: int) -> int:
    return (n + a - 1) // a * a


@dataclass
class _Unit:
    key: object                      # "embed", block index, or "tail"
    lo: int                          # natural range in the flat layout
    hi: int
    slots: list = field(default_factory=list)
    segs: list = field(default_factory=list)  # (nat offset, shard offset, length) for this rank
    shard_lo: int = 0
    shard_len: int = 0

    @property
    def size(self) -> int:
        return _round_up(self.hi - self.lo, 64)


class Zero3Engine(LMEngine):
    """LMEngine whose weights / gradients are views into gather / gradient
    slots that Zero3LM fills and drains around every unit."""

    def __init__(self, spec: LMSpec, owner: "Zero3LM", *, causal: bool = True) -> None:
        if spec.head_dim not in (64, 128):
            raise ValueError("the flash-attention kernels support head_dim 64 or 128")
        self.spec = spec
        self.causal = causal
        self.grad_ready = None
        self._saved = None
        self.owner = owner
        F = spec.features
        self.blocks = []
        for i in range(spec.layers):
            pv, gv = owner.unit_views(i)
            p = f"blocks.{i}."

            def w(name, _pv=pv, _p=p):
                return _pv(_p + name)

            def g(name, _gv=gv, _p=p):
                return _gv(_p + name)

            blk = {
                "ln1": w("attn_norm.weight"), "g_ln1": g("attn_norm.weight"),
                "Wqkv": owner.group_view(i, p + "attn.q_proj.weight", 3 * F * F, False).view(3 * F, F),
                "gWqkv": owner.group_view(i, p + "attn.q_proj.weight", 3 * F * F, True).view(3 * F, F),
                "Wo": w("attn.out_proj.weight"), "gWo": g("attn.out_proj.weight"),
                "ln2": w("mlp_norm.weight"), "g_ln2": g("mlp_norm.weight"),
                "W1": w("mlp.net.0.weight"), "gW1": g("mlp.net.0.weight"),
                "W2": w("mlp.net.2.weight"), "gW2": g("mlp.net.2.weight"),
                "range": (0, 0),
            }
            if spec.bias:
                blk.update(
                    bqkv=owner.group_view(i, p + "attn.q_proj.bias", 3 * F, False),
                    gbqkv=owner.group_view(i, p + "attn.q_proj.bias", 3 * F, True),
                    bo=w("attn.out_proj.bias"), gbo=g("attn.out_proj.bias"),
                    b1=w("mlp.net.0.bias"), gb1=g("mlp.net.0.bias"),
                    b2=w("mlp.net.2.bias"), gb2=g("mlp.net.2.bias"))
            else:
                blk.update(bqkv=None, gbqkv=None, bo=None, gbo=None, b1=None, gb1=None, b2=None, gb2=None)
            self.blocks.append(blk)
        pe, ge = owner.unit_views("embed")
        self.E, self.gE = pe("token_embedding.weight"), ge("token_embedding.weight")
        self.P, self.gP = pe("position_embedding.weight"), ge("position_embedding.weight")
        pt, gt = owner.unit_views("tail")
        self.lnf, self.g_lnf = pt("norm.weight"), gt("norm.weight")
        self.Wh = self.E if spec.tied else pt("head.weight")
        self.gWh = self.gE if spec.tied else gt("head.weight")
        self.tail_range = (0, 0)
        self.embed_range = (0, 0)

    def unit_forward(self, unit) -> None:
        self.owner.gather(unit, prefetch_next=True, direction=1)

    def unit_backward_begin(self, unit) -> None:
        self.owner.backward_begin(unit)

    def unit_backward_end(self, unit) -> None:
        self.owner.backward_end(unit)


class Zero3LM:
    """Sharded TransformerLM for one rank of a ZeRO-3 job (one process per GPU)."""

    def __init__(self, spec: LMSpec, *, rank: int, world: int, device: str | torch.device = "cuda",
                 group=None, init: str = "normal", seed: int = 0, state: dict | None = None,
                 lr: float = 3e-4, betas: tuple[float, float] = (0.9, 0.95), eps: float = 1e-8,
                 weight_decay: float = 0.0, decoupled: bool = True, blocks: int = 128,
                 overlap: bool = True, fused_gather: bool = True, offload_moments: bool | str = False,
                 planner=None, activation_bytes: int = 0, hparams=None) -> None:
        self.spec = spec
        self.overlap = overlap
        self.fused = fused_gather
        # hparams: an object with lr / betas / eps / weight_decay / decoupled
        # (the optimizer that owns this runtime) read at every update, so
        # schedule changes on the optimizer take effect
        self.hparams = hparams
        self._await_step = False
        self.rank, self.world = rank, world
        self.device = torch.device(device)
        self.lr, self.betas, self.eps = lr, betas, eps
        self.weight_decay, self.decoupled = weight_decay, decoupled
        self.nblocks = blocks
        self.layout = build_layout(spec)
        self.by_name = {s.name: s for s in self.layout.slots}
        self.units: dict = {}
        self._build_units()
        self.offload_placement = None
        if offload_moments == "auto":
            from underhfs_b200.runtime import MemoryPlanner

            planner = planner or MemoryPlanner.for_device(self.device)
            # resident besides the moments: bf16 shard + fp32 master, the gather
            # and gradient slots (embed, tail, two blocks; 6 bytes per element)
            slots = (self.units["embed"].size + self.units["tail"].size
                     + 2 * max((self.units[i].size for i in range(spec.layers)), default=0))
            resident = 6 * self.shard_total + 6 * slots
            self.offload_placement = planner.place_optimizer_state(
                8 * self.shard_total, device_headroom=resident + int(activation_bytes))
            from underhfs_b200.cuda import MemoryTier

            offload_moments = self.offload_placement.tier is not MemoryTier.VRAM
        self.offload = bool(offload_moments)
        # shard storage (this rank's rows of every parameter)
        n = self.shard_total
        self.shard16 = torch.zeros(n, dtype=torch.bfloat16, device=self.device)
        self.master = torch.zeros(n, dtype=torch.float32, device=self.device)
        if self.offload:
            # moments in pinned host RAM, two device staging slots of [m | v] for the largest unit
            self.m = torch.zeros(n, dtype=torch.float32, pin_memory=True)
            self.v = torch.zeros(n, dtype=torch.float32, pin_memory=True)
            umax = _round_up(max(u.shard_len for u in self.units.values()), 64)
            self.stage = [torch.zeros(2, umax, dtype=torch.float32, device=self.device) for _ in range(2)]
            # host -> device and device -> host on separate streams: PCIe is full duplex
            self._copy = torch.cuda.Stream(device=self.device)
            self._copy_back = torch.cuda.Stream(device=self.device)
            self._staged: dict = {}       # unit key -> (slot, event: moments are on the device)
            self._slot_free = [None, None]  # event: the slot's moments are back in host RAM
            self._next_slot = 0
        else:
            self.m = torch.zeros_like(self.master)
            self.v = torch.zeros_like(self.master)
        self.step_t = torch.zeros((), dtype=torch.int32, device=self.device)
        self._init_shards(init, seed, state)
        # gather / gradient slots: embed, tail, two ring slots for blocks
        emb, tail = self.units["embed"].size, self.units["tail"].size
        blk = max(self.units[i].size for i in range(spec.layers)) if spec.layers else 0
        self.slot_off = {"embed": 0, "tail": emb, 0: emb + tail, 1: emb + tail + blk}
        total = emb + tail + 2 * blk
        # fused gathers: per slot (tail, ring 0, ring 1) one uint32 flag per 32
        # gathered rows of the unit's matrices, then one ready flag per rank
        self._plan_fused()
        self.flag_words = _round_up(self.max_chunks + world, 64)
        self.flag_off = {k: _round_up(total * 2, 256) + i * self.flag_words * 4
                         for i, k in enumerate(("tail", 0, 1))}
        gbytes = _round_up(total * 2, 256) + 3 * self.flag_words * 4
        self.gsym = SymmetricBuffer(gbytes + 4096, rank=rank, world=world, group=group)
        self.gradsym = SymmetricBuffer(total * 4 + 4096, rank=rank, world=world, group=group)
        self.gather_buf = self.gsym.tensor(total, torch.bfloat16, offset_bytes=0)
        self.grad_buf = self.gradsym.tensor(total, torch.float32, offset_bytes=0)
        self.gather_buf.zero_()
        self.grad_buf.zero_()
        self.gsym.tensor(3 * self.flag_words, torch.int32, offset_bytes=self.flag_off["tail"]).zero_()
        self.epoch = {"tail": 0, 0: 0, 1: 0}
        self.pending: dict = {}
        self._gathered: dict = {}
        if self.fused:
            torch.cuda.synchronize(self.device)
            K.set_b_gather(self._resolve_b)
        self.engine = Zero3Engine(spec, self)
        self.stream = lambda: torch.cuda.current_stream().cuda_stream

    # ------------------------------------------------------------ layout
    def _build_units(self) -> None:
        spec, W = self.spec, self.world
        order: list = ["embed"] + list(range(spec.layers)) + ["tail"]
        for key in order:
            if key == "embed":
                names = ["token_embedding.weight", "position_embedding.weight"]
            elif key == "tail":
                names = ["norm.weight"] + ([] if spec.tied else ["head.weight"])
            else:
                pre = f"blocks.{key}."
                names = [s.name for s in self.layout.slots if s.name.startswith(pre)]
            slots = [self.by_name[nm] for nm in names]
            lo = min(s.offset for s in slots)
            hi = max(s.offset + s.numel for s in slots)
            self.units[key] = _Unit(key, lo, hi, slots)
        cursor = 0
        for key in order:
            u = self.units[key]
            u.shard_lo = cursor
            for s in u.slots:
                rows = s.shape[0]
                cols = s.numel // rows
                if rows % W != 0 or (rows // W * cols) % 8 != 0:
                    raise ValueError(f"{s.name}: {rows} rows do not split into {W} shards of whole 16-byte vectors")
                ln = rows // W * cols
                u.segs.append((s.offset - u.lo + self.rank * ln, cursor, ln))
                cursor += ln
            u.shard_len = cursor - u.shard_lo
            if len(u.segs) > 16:
                raise ValueError(f"unit {key} has more than 16 parameter segments")
        self.shard_total = _round_up(max(cursor, 8), 64)

    def _init_shards(self, init: str, seed: int, state: dict | None) -> None:
        """Own rows of each parameter: from `state` (full tensors, e.g. a
        single-process model's state dict) or initialised on the device."""
        W, r = self.world, self.rank
        for u in self.units.values():
            for s, (nat, soff, ln) in zip(u.slots, u.segs):
                rows = s.shape[0]
                cols = s.numel // rows
                lo_row = r * (rows // W)
                if state is not None:
                    full = state[s.name].reshape(rows, cols).float()
                    part = full[lo_row: lo_row + rows // W].reshape(-1)
                elif s.name.endswith("norm.weight"):
                    part = torch.ones(ln)
                elif s.name.endswith(".bias"):
                    part = torch.zeros(ln)
                else:
                    std = 0.02
                    if s.name.endswith("out_proj.weight") or s.name.endswith("mlp.net.2.weight"):
                        std = 0.02 / math.sqrt(2 * self.spec.layers)
                    gen = torch.Generator(device=self.device).manual_seed(seed * 100003 + s.offset)
                    full_rows = torch.randn(rows // W, cols, generator=gen, device=self.device)
                    part = (full_rows * std).reshape(-1)
                self.master[soff: soff + ln].copy_(part.to(self.device, torch.float32))
        self.shard16.copy_(self.master)

    # ------------------------------------------------------ fused gather
    def _is_matrix(self, slot) -> bool:
        return len(slot.shape) == 2 and slot.shape[1] > 1

    def _plan_fused(self) -> None:
        """Flag numbering for the matrices of every fused unit (blocks, tail):
        chunk c of matrix m covers its gathered rows [32c, 32c+32)."""
        W = self.world
        self.flag_base: dict = {}
        self.max_chunks = 0
        for key, u in self.units.items():
            if key == "embed":
                continue
            n = 0
            for s in u.slots:
                if self._is_matrix(s):
                    if (s.shape[0] // W) % 32 != 0:
                        self.fused = False  # rows per rank must be whole 32-row chunks
                    self.flag_base[(key, s.name)] = n
                    n += s.shape[0] // 32
            self.max_chunks = max(self.max_chunks, n)

    def _gather_fused(self, key) -> None:
        with nvtx.nvtx_range(f"zero3/gather/{key}"):
            self._gather_fused_impl(key)

    def _gather_fused_impl(self, key) -> None:
        """Small parameters now (a barrier-bracketed gather kernel that also
        marks the unit boundary on every rank); the matrices are pushed by the
        first GEMM that reads them (gemm_ag)."""
        slot = self._slot_key(key)
        u = self.units[key]
        small = [list(sg) for s, sg in zip(u.slots, u.segs) if not self._is_matrix(s)]
        if small:
            core().comm_gather_segments(self.gsym.heap, self.slot_off[slot] * 2, self.shard16.data_ptr(), small,
                                        self.nblocks, self.stream())
        self.epoch[slot] += 1
        self.pending[slot] = key
        self._gathered[slot] = key

    def _resolve_b(self, b: torch.Tensor, b_mn: bool):
        """Gather arguments for a GEMM whose B operand lies in a fused slot."""
        base = self.gather_buf.data_ptr()
        off = (b.data_ptr() - base) // 2
        if off < 0 or off >= self.gather_buf.numel():
            return None
        for slot in ("tail", 0, 1):
            lo = self.slot_off[slot]
            key = self._gathered.get(slot)
            if key is None or not (lo <= off < lo + self.units[key].size):
                continue
            u = self.units[key]
            nat = off - lo
            name = next((s.name for s in u.slots if s.offset - u.lo == nat and self._is_matrix(s)), None)
            if name is None:
                return None
            segs = []
            if self.pending.get(slot) == key:
                W, r = self.world, self.rank
                for s, (snat, soff, ln) in zip(u.slots, u.segs):
                    if not self._is_matrix(s):
                        continue
                    rows = s.shape[0] // W
                    cols = s.numel // s.shape[0]
                    segs.append([self.shard16.data_ptr() + soff * 2, (lo + snat) * 2, rows, cols * 2,
                                 self.flag_base[(key, s.name)] + r * rows // 32])
                self.pending[slot] = None
            heap = self.gsym.heap
            data = [heap.data_ptr(p) for p in range(self.world)]
            flags = [heap.data_ptr(p) + self.flag_off[slot] for p in range(self.world)]
            return (self.world, self.rank, self.epoch[slot] & 0xFFFFFFFF, data, flags, segs,
                    self.flag_base[(key, name)], self.max_chunks)
        return None

    # ------------------------------------------------------------- views
    def _slot_key(self, key):
        return key if key in ("embed", "tail") else key % 2

    def unit_views(self, key):
        u = self.units[key]
        base = self.slot_off[self._slot_key(key)]

        def view(buf):
            def get(name):
                s = self.by_name[name]
                off = base + s.offset - u.lo
                return buf[off: off + s.numel].view(s.shape)
            return get

        return view(self.gather_buf), view(self.grad_buf)

    def group_view(self, key, first: str, numel: int, grad: bool) -> torch.Tensor:
        u = self.units[key]
        off = self.slot_off[self._slot_key(key)] + self.by_name[first].offset - u.lo
        buf = self.grad_buf if grad else self.gather_buf
        return buf[off: off + numel]

    # ------------------------------------------------- gather / reduce
    # With overlap (the default) gathers run one unit ahead and the fused
    # reduce-scatter + AdamW runs behind, both on a side stream, so NVLink
    # traffic overlaps the GEMMs of neighbouring units.  Events order every
    # slot reuse: a gather into a ring slot waits for the compute that last
    # read it, a gradient slot is zeroed only after its reduction finished.
    _FWD = "fwd"

    def _order(self):
        return ["embed"] + list(range(self.spec.layers)) + ["tail"]

    def _comm(self) -> torch.cuda.Stream:
        if getattr(self, "_comm_stream", None) is None:
            self._comm_stream = torch.cuda.Stream(device=self.device, priority=-1)
            self._events: dict = {}
        return self._comm_stream

    def _issue_gather(self, key, stream) -> None:
        slot = self._slot_key(key)
        u = self.units[key]
        core().comm_gather_segments(self.gsym.heap, self.slot_off[slot] * 2, self.shard16.data_ptr(),
                                    self._segs(u), self.nblocks, stream.cuda_stream)
        self._gathered[slot] = key

    def gather(self, key, prefetch_next: bool = False, direction: int = 1) -> None:
        """Make unit `key` resident in its slot; with overlap also start the
        gather of the unit that follows in `direction` (+1 forward, -1 backward)."""
        cur = torch.cuda.current_stream()
        slot = self._slot_key(key)
        if self.fused and key != "embed":
            ev = self._events.pop(("g", key), None) if getattr(self, "_events", None) else None
            if ev is not None:
                cur.wait_event(ev)
            if self._gathered.get(slot) != key:
                self._gather_fused(key)
            return
        if not self.overlap:
            if self._gathered.get(slot) != key:
                self._issue_gather(key, cur)
            return
        comm = self._comm()
        ev = self._events.pop(("g", key), None)
        if self._gathered.get(slot) != key:
            # not prefetched: gather now on the side stream and wait for it
            comm.wait_stream(cur)
            self._issue_gather(key, comm)
            ev = torch.cuda.Event()
            ev.record(comm)
        if ev is not None:
            cur.wait_event(ev)
        if prefetch_next:
            order = self._order()
            i = order.index(key) + direction
            if 0 <= i < len(order):
                nxt = order[i]
                nslot = self._slot_key(nxt)
                # fused units are gathered by their first GEMM, never ahead
                if self._gathered.get(nslot) != nxt and nxt != "embed" and not self.fused:
                    # everything issued so far (including the last reader of
                    # that slot) precedes the gather
                    comm.wait_stream(cur)
                    self._issue_gather(nxt, comm)
                    e2 = torch.cuda.Event()
                    e2.record(comm)
                    self._events[("g", nxt)] = e2

    def _segs(self, u: _Unit):
        return [list(sg) for sg in u.segs]

    # ------------------------------------------------------------ moment offload
    def _stage_moments(self, key) -> None:
        """Copy unit `key`'s moments host -> device staging slot (copy stream)."""
        if key in self._staged:
            return
        u = self.units[key]
        slot = self._next_slot
        self._next_slot ^= 1
        cs = self._copy
        if self._slot_free[slot] is not None:
            cs.wait_event(self._slot_free[slot])  # its previous unit's moments are back on the host
        lo, ln = u.shard_lo, u.shard_len
        with torch.cuda.stream(cs):
            self.stage[slot][0, :ln].copy_(self.m[lo: lo + ln], non_blocking=True)
            self.stage[slot][1, :ln].copy_(self.v[lo: lo + ln], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(cs)
        self._staged[key] = (slot, ev)

    def _moment_ptrs(self, key, stream: torch.cuda.Stream) -> tuple[int, int, int]:
        """(m, v) base pointers for the update kernel: shard offsets of this unit
        land in its staging slot."""
        self._stage_moments(key)
        slot, ev = self._staged[key]
        stream.wait_event(ev)
        lo = self.units[key].shard_lo
        return slot, self.stage[slot][0].data_ptr() - lo * 4, self.stage[slot][1].data_ptr() - lo * 4

    def _unstage_moments(self, key, slot: int, stream: torch.cuda.Stream) -> None:
        """After the update on `stream`: copy the unit's moments back to host RAM."""
        u = self.units[key]
        done = torch.cuda.Event()
        done.record(stream)
        cs = self._copy_back
        cs.wait_event(done)
        lo, ln = u.shard_lo, u.shard_len
        with torch.cuda.stream(cs):
            self.m[lo: lo + ln].copy_(self.stage[slot][0, :ln], non_blocking=True)
            self.v[lo: lo + ln].copy_(self.stage[slot][1, :ln], non_blocking=True)
        back = torch.cuda.Event()
        back.record(cs)
        self._slot_free[slot] = back
        del self._staged[key]

    def backward_begin(self, key) -> None:
        cur = torch.cuda.current_stream()
        if self.offload:
            self._stage_moments(key)
        if key == "tail":
            if self.hparams is not None:
                if self._await_step:
                    raise RuntimeError("ZeRO-3 applies the AdamW update inside backward(): call optimizer.step() "
                                       "after every backward (gradient accumulation is not available at stage 3)")
                self._await_step = True
            K.increment_(self.step_t)
            # the head gradient of a tied model lands in the embedding unit
            off = self.slot_off["embed"]
            self.grad_buf[off: off + self.units["embed"].size].zero_()
        if key != "embed":
            self.gather(key, prefetch_next=True, direction=-1)
            ev = self._events.pop(("r", self._slot_key(key)), None) if self.overlap else None
            if ev is not None:
                cur.wait_event(ev)  # the slot's previous reduction has read it on every rank
            off = self.slot_off[self._slot_key(key)]
            self.grad_buf[off: off + self.units[key].size].zero_()

    def backward_end(self, key) -> None:
        # a tied head's gradient is part of the embedding unit, reduced after
        # the embedding backward has added the lookup gradient
        self._reduce(key)
        if key == "embed" and self.overlap:
            torch.cuda.current_stream().wait_stream(self._comm())  # step boundary

    def _reduce(self, key) -> None:
        with nvtx.nvtx_range(f"zero3/rs_adamw/{key}"):
            self._reduce_impl(key)

    def _reduce_impl(self, key) -> None:
        hp = self.hparams if self.hparams is not None else self
        u = self.units[key]
        slot = self._slot_key(key)
        if self.overlap:
            comm = self._comm()
            comm.wait_stream(torch.cuda.current_stream())
            run = comm
        else:
            run = torch.cuda.current_stream()
        stream = run.cuda_stream
        if self.offload:
            mslot, m_ptr, v_ptr = self._moment_ptrs(key, run)
        else:
            m_ptr, v_ptr = self.m.data_ptr(), self.v.data_ptr()
        core().comm_rs_adamw_segments(
            self.gradsym.heap, self.slot_off[slot] * 4, self._segs(u), self.master.data_ptr(), m_ptr,
            v_ptr, self.shard16.data_ptr(), float(hp.lr), float(hp.betas[0]), float(hp.betas[1]),
            float(hp.eps), float(hp.weight_decay), float(1.0 / self.world), bool(hp.decoupled),
            self.step_t.data_ptr(), self.nblocks, stream)
        if self.offload:
            self._unstage_moments(key, mslot, run)
        if self.overlap:
            ev = torch.cuda.Event()
            ev.record(self._comm())
            self._events[("r", slot)] = ev
        # the updated shard invalidates every gathered copy of this unit
        for k, v in list(self._gathered.items()):
            if v == key:
                del self._gathered[k]

    # -------------------------------------------------------------- step
    def train_step(self, ids: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        """Forward, backward and the sharded AdamW update; returns the local loss."""
        loss, _ = self.engine.forward(ids, targets, fuse_loss_grad=True)
        self.engine.backward()
        return loss

    def full_state(self) -> dict:
        """Gather every parameter to full fp32 tensors (for checks and checkpoints)."""
        import torch.distributed as dist

        out = {}
        W = self.world
        for u in self.units.values():
            for s, (nat, soff, ln) in zip(u.slots, u.segs):
                part = self.master[soff: soff + ln].contiguous()
                parts = [torch.empty_like(part) for _ in range(W)]
                if W > 1:
                    dist.all_gather(parts, part)
                else:
                    parts = [part]
                out[s.name] = torch.cat(parts).reshape(s.shape).cpu()
        return out

    def step_done(self) -> None:
        """The owning optimizer's step(): the update already ran per unit during
        backward; this closes the step (the next backward may start)."""
        self._await_step = False

    def load_full_state(self, state: dict) -> None:
        """Overwrite this rank's shard (fp32 master and bf16 copy) from full
        parameter tensors keyed by name; moments are kept."""
        self._init_shards("normal", 0, state)
        self._gathered.clear()

    def close(self) -> None:
        if self.fused:
            K.set_b_gather(None)
        self.gsym.close()
        self.gradsym.close()
