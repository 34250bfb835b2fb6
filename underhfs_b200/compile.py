"""Compile reports: graph IR, guards, specialization cache, fusion plan.

Reference: compile.py:11-495.  The function always runs eagerly; afterwards
the op tape of its result (every Tensor op records ``_op`` / ``_prev``) is
turned into a ``GraphIR``, guards describe each tensor argument, elementwise
/ reduction / attention nodes are grouped, and the groups are lowered to
kernels of this build: ``native-cuda-fused`` (sm_100a elementwise / reduce
kernels), ``native-cuda-attention`` (fp32 attention kernel) or the eager
plan.  ``native_required`` / ``allow_fallback=False`` make a non-native group
an error.

On B200 the replacement for a tracing compiler is CUDA graph capture:
:func:`cuda_graph` records a step function once on a side stream and replays
it with one launch per call.
"""

from __future__ import annotations

from dataclasses import dataclass, field, replace
from enum import Enum
from functools import wraps
from typing import Any, Callable, TypeVar

Fn = TypeVar("Fn", bound=Callable)


class FusionKind(str, Enum):
    ELEMENTWISE = "elementwise"
    REDUCTION = "reduction"
    ATTENTION = "attention"


@dataclass
class CompilePolicy:
    enabled: bool = True
    partial_dynamic_shapes: bool = True
    guard_specialization: bool = True
    native_required: bool = False
    allow_fallback: bool = True
    fusion: tuple[FusionKind, ...] = field(
        default_factory=lambda: (FusionKind.ELEMENTWISE, FusionKind.REDUCTION, FusionKind.ATTENTION)
    )


GuardSignature = tuple[tuple[str, tuple[int, ...], str, str, str], ...]


@dataclass
class IRNode:
    name: str
    op: str
    inputs: tuple[str, ...]
    outputs: tuple[str, ...]
    shape: tuple[int, ...] = ()
    dtype: str = "unknown"
    device: str = "unknown"


@dataclass
class GraphIR:
    nodes: list[IRNode] = field(default_factory=list)

    def add(self, *, name: str, op: str, inputs: tuple[str, ...], outputs: tuple[str, ...],
            shape: tuple[int, ...] = (), dtype: str = "unknown", device: str = "unknown") -> None:
        self.nodes.append(IRNode(name, op, tuple(inputs), tuple(outputs), tuple(shape), dtype, device))

    def to_dict(self) -> dict[str, Any]:
        return {"nodes": [dict(vars(n)) for n in self.nodes]}


@dataclass(frozen=True)
class Guard:
    name: str
    shape: tuple[int, ...]
    dtype: str
    device: str
    layout: str

    def to_dict(self) -> dict[str, Any]:
        return dict(vars(self))


@dataclass(frozen=True)
class FusionGroup:
    kind: FusionKind
    nodes: tuple[str, ...]

    def to_dict(self) -> dict[str, Any]:
        return {"kind": self.kind.value, "nodes": list(self.nodes)}


@dataclass(frozen=True)
class CompiledKernel:
    name: str
    kind: FusionKind
    nodes: tuple[str, ...]
    backend: str
    executable: bool

    def dispatch(self, *inputs: Any, op: str | None = None, scale: float | None = None, causal: bool = False) -> Any:
        if not self.executable:
            raise RuntimeError(f"{self.name} is not executable for backend {self.backend}")
        if self.backend == "native-cuda-attention":
            return _run_attention(*inputs, scale=scale, causal=causal)
        if self.backend in ("native-cuda-fused", "eager-fused-plan"):
            return _run_fused(*inputs, op=op, native=self.backend == "native-cuda-fused")
        raise RuntimeError(f"{self.backend} dispatch is not implemented")

    def to_dict(self) -> dict[str, Any]:
        return {"name": self.name, "kind": self.kind.value, "nodes": list(self.nodes), "backend": self.backend,
                "executable": self.executable}


@dataclass(frozen=True)
class ExecutablePlan:
    graph: GraphIR
    kernels: tuple[CompiledKernel, ...]
    fallback_backend: str = "eager-python"

    def to_dict(self) -> dict[str, Any]:
        return {"graph": self.graph.to_dict(), "kernels": [k.to_dict() for k in self.kernels],
                "fallback_backend": self.fallback_backend}


@dataclass(frozen=True)
class CompileCacheInfo:
    hits: int = 0
    misses: int = 0
    specializations: int = 0

    def to_dict(self) -> dict[str, int]:
        return dict(vars(self))


@dataclass(frozen=True)
class CompileReport:
    policy: CompilePolicy
    graph: GraphIR
    guards: tuple[Guard, ...]
    fusion_groups: tuple[FusionGroup, ...]
    specialization_key: GuardSignature = ()
    cache_hit: bool = False
    cache_info: CompileCacheInfo = field(default_factory=CompileCacheInfo)
    plan: ExecutablePlan | None = None

    def to_dict(self) -> dict[str, Any]:
        p = self.policy
        return {
            "policy": {"enabled": p.enabled, "partial_dynamic_shapes": p.partial_dynamic_shapes,
                       "guard_specialization": p.guard_specialization, "native_required": p.native_required,
                       "allow_fallback": p.allow_fallback, "fusion": [k.value for k in p.fusion]},
            "graph": self.graph.to_dict(),
            "guards": [g.to_dict() for g in self.guards],
            "fusion_groups": [g.to_dict() for g in self.fusion_groups],
            "specialization_key": [
                {"name": n, "shape": s, "dtype": d, "device": dev, "layout": lay}
                for n, s, d, dev, lay in self.specialization_key
            ],
            "cache_hit": self.cache_hit,
            "cache_info": self.cache_info.to_dict(),
            "plan": None if self.plan is None else self.plan.to_dict(),
        }


@dataclass(frozen=True)
class CompileCacheEntry:
    signature: GuardSignature
    report: CompileReport
    hits: int = 0


def compile(function: Fn | None = None, *, policy: CompilePolicy | None = None):
    pol = policy or CompilePolicy()

    def decorate(fn: Fn) -> Fn:
        cache: dict[GuardSignature, CompileCacheEntry] = {}
        counters = {"hits": 0, "misses": 0}
        specialize = pol.enabled and pol.guard_specialization

        @wraps(fn)
        def run(*args: Any, **kwargs: Any) -> Any:
            key = _signature(args, kwargs)
            result = fn(*args, **kwargs)
            if specialize and key in cache:
                counters["hits"] += 1
                entry = cache[key]
                cache[key] = replace(entry, hits=entry.hits + 1)
                info = CompileCacheInfo(counters["hits"], counters["misses"], len(cache))
                report = replace(entry.report, cache_hit=True, cache_info=info)
            else:
                counters["misses"] += 1
                report = analyze_execution(result, args=args, kwargs=kwargs, policy=pol)
                n_spec = len(cache) + (1 if specialize else 0)
                report = replace(report, specialization_key=key, cache_hit=False,
                                 cache_info=CompileCacheInfo(counters["hits"], counters["misses"], n_spec))
                if specialize:
                    cache[key] = CompileCacheEntry(key, report)
            run._underhfs_last_compile_report = report
            run._underhfs_last_graph = report.graph
            return result

        run._underhfs_compile_policy = pol
        run._underhfs_last_compile_report = None
        run._underhfs_compile_cache = cache
        return run  # type: ignore[return-value]

    return decorate if function is None else decorate(function)


def _is_tensor(v: Any) -> bool:
    return hasattr(v, "shape") and hasattr(v, "dtype") and hasattr(v, "_prev")


def analyze_execution(result: Any, *, args: tuple = (), kwargs: dict | None = None,
                      policy: CompilePolicy | None = None) -> CompileReport:
    pol = policy or CompilePolicy()
    graph = GraphIR()
    names: dict[int, str] = {}

    def visit(t: Any) -> str | None:
        if not _is_tensor(t):
            return None
        if id(t) in names:
            return names[id(t)]
        name = f"t{len(names)}"
        names[id(t)] = name
        ins = tuple(n for n in (visit(p) for p in getattr(t, "_prev", ())) if n)
        graph.add(name=name, op=getattr(t, "_op", "") or "leaf", inputs=ins, outputs=(name,),
                  shape=tuple(t.shape), dtype=getattr(t.dtype, "value", "unknown"), device=str(t.device))
        return name

    outs = result if isinstance(result, (tuple, list)) else (
        tuple(result.values()) if isinstance(result, dict) else (result,))
    for item in outs:
        visit(item)
    guards = _guards(args, kwargs or {})
    groups = _fusion_groups(graph, pol)
    plan = lower_to_plan(graph, groups, policy=pol)
    if pol.native_required and any(not k.backend.startswith("native-") for k in plan.kernels):
        raise RuntimeError("compile native mode found unsupported fusion groups; fallback is disabled")
    return CompileReport(pol, graph, guards, groups, specialization_key=_to_signature(guards), plan=plan)


def explain(fn: Callable[..., Any], *args: Any, policy: CompilePolicy | None = None, **kwargs: Any) -> CompileReport:
    return analyze_execution(fn(*args, **kwargs), args=args, kwargs=kwargs, policy=policy)


def lower_to_plan(graph: GraphIR, fusion_groups: tuple[FusionGroup, ...], *,
                  policy: CompilePolicy | None = None) -> ExecutablePlan:
    pol = policy or CompilePolicy()
    kernels = []
    for i, group in enumerate(fusion_groups):
        backend = _backend_for(graph, group, pol)
        kernels.append(CompiledKernel(f"kernel_{i}_{group.kind.value}", group.kind, group.nodes, backend,
                                      backend != "unsupported-native"))
    if not pol.allow_fallback and any(not k.backend.startswith("native-") for k in kernels):
        raise RuntimeError("compile fallback is disabled, but a fusion group has no native backend")
    return ExecutablePlan(graph, tuple(kernels))


def _backend_for(graph: GraphIR, group: FusionGroup, pol: CompilePolicy) -> str:
    nodes = [n for n in graph.nodes if n.name in group.nodes]
    if not nodes:
        return "eager-fused-plan"
    on_cuda_fp32 = all(n.device.startswith("cuda") and n.dtype == "fp32" for n in nodes)
    strict = pol.native_required or not pol.allow_fallback
    if group.kind is FusionKind.ATTENTION:
        shapes = [n.shape for n in nodes if n.shape]
        if shapes and all(len(s) == 2 for s in shapes) and on_cuda_fp32:
            return "native-cuda-attention"
        return "unsupported-native" if strict else "eager-fused-plan"
    if on_cuda_fp32:
        return "native-cuda-fused"
    return "unsupported-native" if strict else "eager-fused-plan"


def _check_cuda_fp32(v: Any, what: str) -> None:
    if not _is_tensor(v):
        raise TypeError(f"{what} must be an underHFS Tensor")
    if str(v.device) != "cuda:0":
        raise ValueError(f"{what} must be on cuda:0")
    if getattr(v.dtype, "value", "") != "fp32":
        raise ValueError(f"{what} must be fp32")
    if getattr(v.layout, "value", "") != "dense":
        raise ValueError(f"{what} must be dense")


def _run_attention(*inputs: Any, scale: float | None, causal: bool) -> Any:
    if len(inputs) != 3:
        raise ValueError("native CUDA attention dispatch expects q, k, and v tensors")
    q, k, v = inputs
    for t, n in ((q, "q"), (k, "k"), (v, "v")):
        _check_cuda_fp32(t, n)
    if q.shape != k.shape or q.shape != v.shape or len(q.shape) != 2:
        raise ValueError("native CUDA attention dispatch expects q/k/v shape [tokens, features]")
    from underhfs_b200.ops import kernels as K
    from underhfs_b200.tensor import Tensor

    s = q.shape[1] ** -0.5 if scale is None else float(scale)
    out = K.attention_f32(q._data.detach(), k._data.detach(), v._data.detach(), s, causal)
    return Tensor._wrap(out, like=q, backend="native_cuda_attention", op="attention", parents=(q, k, v))


def _run_fused(*inputs: Any, op: str | None, native: bool) -> Any:
    if op not in ("add", "mul", "sum"):
        raise ValueError("fused dispatch supports op='add', op='mul', or op='sum'")
    if native:
        for i, t in enumerate(inputs):
            _check_cuda_fp32(t, f"input{i}")
    if op == "sum":
        if len(inputs) != 1:
            raise ValueError("fused sum dispatch expects one tensor")
        return inputs[0].sum()
    if len(inputs) != 2:
        raise ValueError(f"fused {op} dispatch expects two tensors")
    return inputs[0] + inputs[1] if op == "add" else inputs[0] * inputs[1]


def _guard(name: str, v: Any) -> Guard:
    return Guard(name, tuple(v.shape), getattr(v.dtype, "value", "unknown"), str(v.device),
                 getattr(getattr(v, "layout", None), "value", "unknown"))


def _guards(args: tuple, kwargs: dict) -> tuple[Guard, ...]:
    out = [_guard(f"arg{i}", a) for i, a in enumerate(args) if _is_tensor(a)]
    out += [_guard(k, v) for k, v in kwargs.items() if _is_tensor(v)]
    return tuple(out)


def _to_signature(guards: tuple[Guard, ...]) -> GuardSignature:
    return tuple((g.name, g.shape, g.dtype, g.device, g.layout) for g in guards)


def _signature(args: tuple, kwargs: dict) -> GuardSignature:
    return _to_signature(_guards(args, dict(sorted(kwargs.items()))))


_ELEMENTWISE = {"add", "sub", "mul", "div", "relu", "tanh", "exp", "log", "pow"}


def _fusion_groups(graph: GraphIR, pol: CompilePolicy) -> tuple[FusionGroup, ...]:
    groups: list[FusionGroup] = []
    if FusionKind.ELEMENTWISE in pol.fusion:
        ew = tuple(n.name for n in graph.nodes if n.op in _ELEMENTWISE)
        if len(ew) >= 2:
            groups.append(FusionGroup(FusionKind.ELEMENTWISE, ew))
    if FusionKind.REDUCTION in pol.fusion:
        red = tuple(n.name for n in graph.nodes if n.op in ("sum", "mean"))
        if red:
            groups.append(FusionGroup(FusionKind.REDUCTION, red))
    if FusionKind.ATTENTION in pol.fusion:
        ops = [n.op for n in graph.nodes]
        if ops.count("matmul") >= 2 and "softmax" in ops:
            groups.append(FusionGroup(FusionKind.ATTENTION,
                                      tuple(n.name for n in graph.nodes if n.op in ("matmul", "softmax"))))
    return tuple(groups)


class CudaGraphRunner:
    """Capture ``fn`` once (after ``warmup`` eager calls on a side stream) and
    replay it.  Inputs must be the same tensors (static addresses) each call;
    copy new data into them before ``__call__``."""

    def __init__(self, fn: Callable[[], Any], *, warmup: int = 2) -> None:
        import torch

        self.fn = fn
        self.graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(warmup):
                fn()
        torch.cuda.current_stream().wait_stream(side)
        with torch.cuda.graph(self.graph):
            self.output = fn()

    def __call__(self) -> Any:
        self.graph.replay()
        return self.output


def cuda_graph(fn: Callable[[], Any], *, warmup: int = 2) -> CudaGraphRunner:
    return CudaGraphRunner(fn, warmup=warmup)
