"""Memory tiers: a placement planner and the stores behind each tier.

Public surface of the reference (runtime.py:18-368 of the reference):
``MemoryPlanner`` (first-fit placement over the policy's tiers with an
oversubscription rule), ``OffloadExecutor`` (NVMe tensors as checksummed JSON
files, prefetch cache), ``NetworkOffloadServer`` / ``NetworkOffloadClient``
(the same tensors over HTTP) and ``planner_from_system``.  Record formats,
HTTP routes and the "checksum mismatch" / "not found" errors are kept so
files and servers interoperate.

Structure here:

* every tier is a :class:`TierStore` -- ``put(value) -> handle``,
  ``get(handle) -> Tensor``, ``drop(handle)``.  :class:`FileStore` (NVMe),
  :class:`NetworkOffloadClient` (network) and :class:`PinnedHostTier` (RAM:
  pinned host buffers moved with ``cudaMemcpyAsync`` on a side stream,
  ordered against compute by CUDA events) implement it;
* :class:`OffloadExecutor` routes a tensor to the store of the tier the
  planner chose and keeps the prefetch cache;
* :class:`MemoryPlanner` keeps one ledger entry per tier and, beyond
  tensor placement, answers the question the ZeRO-3 optimizer asks at
  construction: do the Adam moments of this rank's shard stay in device
  memory, or go to pinned host RAM (``place_optimizer_state``).
"""

from __future__ import annotations

import http.client
import json
from dataclasses import dataclass
from hashlib import sha256
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer
from pathlib import Path
from threading import Thread
from typing import Any, Callable, Protocol
from urllib.parse import urlsplit
from uuid import uuid4

import torch

from underhfs_b200.cuda import MemoryPolicy, MemoryTier, memory_budgets
from underhfs_b200.tensor import DType, Tensor, tensor

# bytes per element of every dtype the planner sizes (INT4 packs two per byte)
DTYPE_BYTES = {
    DType.FP32: 4, DType.FP16: 2, DType.BF16: 2, DType.FP8_E4M3: 1, DType.FP8_E5M2: 1, DType.INT8: 1, DType.INT4: 0.5,
}


@dataclass(frozen=True)
class Placement:
    tier: MemoryTier
    bytes: int
    reason: str


@dataclass(frozen=True)
class OffloadHandle:
    id: str
    tier: MemoryTier
    path: str
    bytes: int
    shape: tuple[int, ...]
    dtype: DType
    device: str
    sha256: str = ""
    cached: bool = False

    def to_dict(self) -> dict[str, Any]:
        out = {k: getattr(self, k) for k in ("id", "path", "bytes", "device", "sha256", "cached")}
        out.update(tier=self.tier.value, shape=list(self.shape), dtype=self.dtype.value)
        return out

    def with_cached(self, cached: bool) -> "OffloadHandle":
        return OffloadHandle(self.id, self.tier, self.path, self.bytes, self.shape, self.dtype, self.device,
                             self.sha256, cached)


# ------------------------------------------------------------------ planner
class MemoryPlanner:
    """Places byte counts on the tiers of a :class:`MemoryPolicy`.

    The ledger holds ``[capacity, used]`` per tier.  A request goes to the
    first tier, in policy order, whose free bytes cover it; when none does it
    is charged to the last tier if the policy allows offload (reason
    ``"oversubscribed-offload"``), otherwise ``MemoryError``."""

    def __init__(self, policy: MemoryPolicy, budgets: dict[MemoryTier, int]) -> None:
        self.policy = policy
        self._ledger: dict[MemoryTier, list[int]] = {t: [int(budgets.get(t, 0)), 0] for t in policy.tiers}

    @classmethod
    def for_device(cls, device: torch.device | str, policy: MemoryPolicy | None = None, *,
                   vram_fraction: float = 0.9, host_bytes: int | None = None) -> "MemoryPlanner":
        """Budgets of ONE GPU (its free memory now) plus host RAM: the planner a
        rank of a multi-GPU job uses for its own state."""
        policy = policy or MemoryPolicy(tiers=(MemoryTier.VRAM, MemoryTier.RAM))
        budgets = {t: 0 for t in policy.tiers}
        dev = torch.device(device)
        if dev.type == "cuda" and torch.cuda.is_available():
            free, _total = torch.cuda.mem_get_info(dev)
            budgets[MemoryTier.VRAM] = int(free * vram_fraction)
        if host_bytes is None:
            host_bytes = memory_budgets(vram_fraction=1.0).get(MemoryTier.RAM, 0)
        budgets[MemoryTier.RAM] = int(host_bytes)
        return cls(policy, budgets)

    def _free(self, tier: MemoryTier) -> int:
        cap, used = self._ledger[tier]
        return max(0, cap - used)

    def tensor_size_bytes(self, value: Tensor) -> int:
        return int(value.numel() * DTYPE_BYTES[value.dtype])

    def place_tensor(self, value: Tensor) -> Placement:
        return self.place_bytes(self.tensor_size_bytes(value))

    def place_bytes(self, size: int) -> Placement:
        if size < 0:
            raise ValueError("size must be non-negative")
        fits = [t for t in self.policy.tiers if self._free(t) >= size]
        if fits:
            self._ledger[fits[0]][1] += size
            return Placement(fits[0], size, "fits-budget")
        if not self.policy.allow_offload:
            raise MemoryError(f"tensor requires {size} bytes, but no configured tier has capacity")
        last = self.policy.tiers[-1]
        self._ledger[last][1] += size
        return Placement(last, size, "oversubscribed-offload")

    def reserve(self, tier: MemoryTier, size: int) -> None:
        """Charge bytes that are already placed (weights, activations) to a tier."""
        if tier in self._ledger:
            self._ledger[tier][1] += int(size)

    def release(self, placement: Placement) -> None:
        entry = self._ledger.get(placement.tier)
        if entry is not None:
            entry[1] = max(0, entry[1] - placement.bytes)

    def place_optimizer_state(self, size: int, *, device_headroom: int = 0) -> Placement:
        """Where optimizer state of ``size`` bytes lives: device memory when it
        fits next to ``device_headroom`` bytes kept free for the step's
        activations and buffers, else pinned host RAM (a RAM placement is
        what makes ZeRO-3 stream the moments over PCIe)."""
        if MemoryTier.VRAM in self._ledger and self._free(MemoryTier.VRAM) >= size + device_headroom:
            self._ledger[MemoryTier.VRAM][1] += size
            return Placement(MemoryTier.VRAM, size, "fits-device")
        if MemoryTier.RAM in self._ledger and (self._free(MemoryTier.RAM) >= size or self.policy.allow_offload):
            self._ledger[MemoryTier.RAM][1] += size
            return Placement(MemoryTier.RAM, size, "device-full-pinned-host")
        raise MemoryError(f"optimizer state of {size} bytes fits neither device memory nor host RAM")

    def snapshot(self) -> dict[str, dict[str, int]]:
        return {t.value: {"capacity_bytes": cap, "used_bytes": used, "available_bytes": max(0, cap - used)}
                for t, (cap, used) in self._ledger.items()}


def planner_from_system(policy: MemoryPolicy | None = None, *, vram_fraction: float = 0.9) -> MemoryPlanner:
    return MemoryPlanner(policy or MemoryPolicy(), budgets=memory_budgets(vram_fraction=vram_fraction))


# ------------------------------------------------------------- tier stores
class TierStore(Protocol):
    tier: MemoryTier

    def put(self, value: Tensor) -> OffloadHandle: ...

    def get(self, handle: OffloadHandle, device: str | None = None) -> Tensor: ...

    def drop(self, handle: OffloadHandle) -> None: ...


def _digest_of(data: Any) -> str:
    """sha256 of the canonical JSON of a tensor's nested value list."""
    return sha256(json.dumps(data, separators=(",", ":"), sort_keys=True).encode("utf-8")).hexdigest()


def _canonical(record: dict[str, Any]) -> bytes:
    return json.dumps(record, separators=(",", ":")).encode("utf-8")


@dataclass(frozen=True)
class _RecordFormat:
    """One self-describing tensor record format (file or wire)."""

    name: str    # value of the record's "format" field
    label: str   # how errors name it

    def encode(self, ident: str, value: Tensor) -> dict[str, Any]:
        data = value.detach().tolist()
        return {"format": self.name, "version": 1, "id": ident, "shape": list(value.shape),
                "dtype": value.dtype.value, "device": str(value.device), "data_sha256": _digest_of(data),
                "data": data}

    def decode(self, record: dict[str, Any], handle: OffloadHandle, device: str | None) -> Tensor:
        problems = (
            (record.get("format") != self.name, f"not an underhfs {self.label} tensor"),
            (record.get("version") != 1, f"unsupported {self.label} tensor version: {record.get('version')}"),
            (record.get("id", handle.id) != handle.id, f"{self.label} handle id mismatch"),
            (_digest_of(record.get("data")) != record.get("data_sha256"),
             f"{self.label} tensor data checksum mismatch"),
            (tuple(record.get("shape", ())) != tuple(handle.shape), f"{self.label} tensor shape mismatch"),
        )
        for bad, message in problems:
            if bad:
                raise ValueError(message)
        out = tensor(record["data"], dtype=handle.dtype)
        return out.to(device) if device is not None else out


FILE_RECORD = _RecordFormat("underhfs.offload-tensor", "offload")
WIRE_RECORD = _RecordFormat("underhfs.network-offload-tensor", "network offload")


class FileStore:
    """NVMe tier: one JSON record file per tensor under ``root``; the handle
    carries the sha256 of the file bytes, checked before decoding."""

    tier = MemoryTier.NVME

    def __init__(self, root: str | Path) -> None:
        self.root = Path(root)
        self.root.mkdir(parents=True, exist_ok=True)

    def put(self, value: Tensor) -> OffloadHandle:
        ident = uuid4().hex
        raw = _canonical(FILE_RECORD.encode(ident, value))
        path = self.root / f"{ident}.uhfsoffload.json"
        path.write_bytes(raw)
        return OffloadHandle(ident, self.tier, str(path), len(raw), tuple(value.shape), value.dtype,
                             str(value.device), sha256(raw).hexdigest())

    def get(self, handle: OffloadHandle, device: str | None = None) -> Tensor:
        raw = Path(handle.path).read_bytes()
        if handle.sha256 and sha256(raw).hexdigest() != handle.sha256:
            raise ValueError("offload file checksum mismatch")
        return FILE_RECORD.decode(json.loads(raw.decode("utf-8")), handle, device)

    def drop(self, handle: OffloadHandle) -> None:
        Path(handle.path).unlink(missing_ok=True)


class PinnedHostTier:
    """RAM tier as pinned host memory with asynchronous copies.

    Keyed buffers for the optimizer: ``offload(key, t)`` enqueues a
    device->host copy on the side stream after the compute stream's pending
    work; ``fetch(key, out)`` enqueues the host->device copy; ``wait(key)``
    makes the current stream wait for it.  Nothing blocks the host.  As a
    :class:`TierStore` (``put`` / ``get`` / ``drop``) it holds whole tensors.
    """

    tier = MemoryTier.RAM

    def __init__(self, device: torch.device | str = "cuda") -> None:
        self.device = torch.device(device)
        self.stream = torch.cuda.Stream(device=self.device) if self.device.type == "cuda" else None
        self._buffers: dict[str, torch.Tensor] = {}
        self._events: dict[str, torch.cuda.Event] = {}
        self._meta: dict[str, OffloadHandle] = {}

    def allocate(self, key: str, numel: int, dtype: torch.dtype = torch.float32) -> torch.Tensor:
        buf = torch.empty(numel, dtype=dtype, pin_memory=torch.cuda.is_available())
        self._buffers[key] = buf
        return buf

    def host(self, key: str) -> torch.Tensor:
        return self._buffers[key]

    def _async_copy(self, key: str, dst: torch.Tensor, src: torch.Tensor, device_side: torch.Tensor) -> None:
        if self.stream is None:
            dst.copy_(src)
            return
        ready = torch.cuda.Event()
        ready.record(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.stream):
            self.stream.wait_event(ready)
            dst.copy_(src, non_blocking=True)
            done = torch.cuda.Event()
            done.record(self.stream)
        device_side.record_stream(self.stream)
        self._events[key] = done

    def offload(self, key: str, src: torch.Tensor) -> None:
        if key not in self._buffers:
            self.allocate(key, src.numel(), src.dtype)
        self._async_copy(key, self._buffers[key], src.reshape(-1), src)

    def fetch(self, key: str, out: torch.Tensor) -> None:
        self._async_copy(key, out.reshape(-1), self._buffers[key], out)

    def wait(self, key: str) -> None:
        ev = self._events.get(key)
        if ev is not None:
            torch.cuda.current_stream(self.device).wait_event(ev)

    def bytes_resident(self) -> int:
        return sum(b.numel() * b.element_size() for b in self._buffers.values())

    # TierStore: whole tensors, synchronous at get()
    def put(self, value: Tensor) -> OffloadHandle:
        ident = uuid4().hex
        data = value._data.detach()
        self.offload(ident, data)
        h = OffloadHandle(ident, self.tier, f"pinned://{ident}", data.numel() * data.element_size(),
                          tuple(value.shape), value.dtype, str(value.device))
        self._meta[ident] = h
        return h

    def get(self, handle: OffloadHandle, device: str | None = None) -> Tensor:
        if handle.id not in self._buffers:
            raise KeyError(f"pinned tensor {handle.id} not found")
        ev = self._events.get(handle.id)
        if ev is not None:
            ev.synchronize()
        host = self._buffers[handle.id].reshape(handle.shape)
        out = Tensor._wrap(host.clone(), dtype=handle.dtype)
        return out.to(device) if device is not None else out

    def drop(self, handle: OffloadHandle) -> None:
        self._buffers.pop(handle.id, None)
        self._events.pop(handle.id, None)
        self._meta.pop(handle.id, None)


class OffloadExecutor:
    """Moves tensors to the store of a tier: NVMe files under ``root`` (or the
    policy's scratch path), the network client given as ``network``, pinned
    RAM given as ``host``.  ``prefetch_tensor`` loads a tensor ahead of use and
    returns its handle marked ``cached``."""

    def __init__(self, policy: MemoryPolicy, root: str | Path | None = None, *,
                 network: "NetworkOffloadClient | None" = None, host: PinnedHostTier | None = None) -> None:
        self.policy = policy
        self.root = Path(root or policy.scratch_path or ".underhfs-offload")
        self._stores: dict[MemoryTier, TierStore] = {MemoryTier.NVME: FileStore(self.root)}
        if network is not None:
            self._stores[MemoryTier.NETWORK] = network
        if host is not None:
            self._stores[MemoryTier.RAM] = host
        self._prefetched: dict[str, Tensor] = {}

    def _store(self, tier: MemoryTier) -> TierStore:
        store = self._stores.get(tier)
        if store is None:
            if tier is MemoryTier.NETWORK:
                raise RuntimeError("network offload requires a configured remote transport (pass network=...)")
            raise ValueError(f"no {tier.value} store configured on this executor")
        return store

    def offload_tensor(self, value: Tensor, tier: MemoryTier = MemoryTier.NVME) -> OffloadHandle:
        return self._store(tier).put(value)

    def offload_planned(self, value: Tensor, planner: MemoryPlanner) -> OffloadHandle | Placement:
        """Let the planner pick the tier; a VRAM placement leaves the tensor where it is."""
        placement = planner.place_tensor(value)
        if placement.tier is MemoryTier.VRAM:
            return placement
        return self.offload_tensor(value, placement.tier)

    def prefetch_tensor(self, handle: OffloadHandle) -> OffloadHandle:
        self._prefetched[handle.id] = self._store(handle.tier).get(handle)
        return handle.with_cached(True)

    def load_tensor(self, handle: OffloadHandle, *, device: str | None = None, use_cache: bool = True) -> Tensor:
        hit = self._prefetched.get(handle.id) if use_cache else None
        if hit is not None:
            return hit.detach().to(device or "cpu")
        return self._store(handle.tier).get(handle, device)

    def release(self, handle: OffloadHandle) -> None:
        self._prefetched.pop(handle.id, None)
        self._store(handle.tier).drop(handle)

    def cache_info(self) -> dict[str, int]:
        return {"prefetched_tensors": len(self._prefetched)}


# ------------------------------------------------------------ network tier
class NetworkOffloadServer:
    """In-memory tensor store over HTTP (threaded): ``GET /health``,
    ``GET /load/<id>``, ``POST /upload`` (a wire record, validated before it
    is stored), ``DELETE /release/<id>``.  Every reply is JSON; failures carry
    an ``"error"`` field and a 4xx status."""

    def __init__(self, host: str = "127.0.0.1", port: int = 0) -> None:
        self._store: dict[str, dict[str, Any]] = {}
        routes: dict[tuple[str, str], Callable[[str, bytes], tuple[int, Any]]] = {
            ("GET", "health"): lambda _arg, _body: (200, {"status": "ok", "tensors": len(self._store)}),
            ("GET", "load"): self._load,
            ("POST", "upload"): self._upload,
            ("DELETE", "release"): self._release,
        }
        self._server = ThreadingHTTPServer((host, port), _route_handler(routes))
        self.host, self.port = self._server.server_address[:2]
        self._thread: Thread | None = None

    @property
    def url(self) -> str:
        return f"http://{self.host}:{self.port}"

    def start(self) -> "NetworkOffloadServer":
        if self._thread is None:
            self._thread = Thread(target=self._server.serve_forever, daemon=True)
            self._thread.start()
        return self

    def close(self) -> None:
        self._server.shutdown()
        self._server.server_close()
        if self._thread is not None:
            self._thread.join(timeout=2.0)
            self._thread = None

    def _load(self, key: str, _body: bytes) -> tuple[int, Any]:
        rec = self._store.get(key)
        return (200, rec) if rec is not None else (404, {"error": f"tensor {key!r} not found"})

    def _upload(self, _arg: str, body: bytes) -> tuple[int, Any]:
        rec = json.loads(body.decode("utf-8")) if body else {}
        if rec.get("format") != WIRE_RECORD.name or rec.get("version") != 1:
            return 400, {"error": "not a network offload tensor record"}
        if _digest_of(rec.get("data")) != rec.get("data_sha256"):
            return 400, {"error": "uploaded tensor data checksum mismatch"}
        self._store[rec["id"]] = rec
        return 200, {"ok": True, "id": rec["id"]}

    def _release(self, key: str, _body: bytes) -> tuple[int, Any]:
        self._store.pop(key, None)
        return 200, {"ok": True, "id": key}


def _route_handler(routes):
    """Request handler class dispatching ``/<route>[/<arg>]`` through a table."""

    class RouteHandler(BaseHTTPRequestHandler):
        def log_message(self, *_args) -> None:
            return

        def _dispatch(self) -> None:
            parts = self.path.strip("/").split("/", 1)
            fn = routes.get((self.command, parts[0]))
            length = int(self.headers.get("Content-Length") or 0)
            body = self.rfile.read(length) if length else b""
            if fn is None:
                status, payload = 404, {"error": f"no route {self.command} {self.path} (not found)"}
            else:
                try:
                    status, payload = fn(parts[1] if len(parts) > 1 else "", body)
                except Exception as exc:  # a bad request must not kill the server thread
                    status, payload = 400, {"error": str(exc)}
            raw = json.dumps(payload).encode("utf-8")
            self.send_response(status)
            self.send_header("Content-Type", "application/json")
            self.send_header("Content-Length", str(len(raw)))
            self.end_headers()
            self.wfile.write(raw)

        do_GET = do_POST = do_DELETE = _dispatch

    return RouteHandler


class NetworkOffloadClient:
    """Network tier store: tensors uploaded to a :class:`NetworkOffloadServer`."""

    tier = MemoryTier.NETWORK

    def __init__(self, base_url: str, timeout: float = 5.0) -> None:
        self.base_url = base_url.rstrip("/")
        parts = urlsplit(self.base_url)
        self._host, self._port = parts.hostname or "127.0.0.1", parts.port or 80
        self.timeout = timeout

    def _call(self, method: str, route: str, body: bytes | None = None) -> Any:
        """One HTTP exchange; a non-2xx reply or an ``"error"`` field raises
        RuntimeError with the server's message."""
        conn = http.client.HTTPConnection(self._host, self._port, timeout=self.timeout)
        try:
            conn.request(method, route, body=body, headers={"Content-Type": "application/json"})
            resp = conn.getresponse()
            status, text = resp.status, resp.read().decode("utf-8")
        finally:
            conn.close()
        try:
            payload = json.loads(text) if text else {}
        except json.JSONDecodeError:
            payload = {"error": f"HTTP {status}: {text[:200]}"}
        if status >= 300 or (isinstance(payload, dict) and "error" in payload):
            message = payload.get("error") if isinstance(payload, dict) else None
            raise RuntimeError(message or f"HTTP {status}")
        return payload

    def put(self, value: Tensor) -> OffloadHandle:
        ident = uuid4().hex
        raw = _canonical(WIRE_RECORD.encode(ident, value))
        self._call("POST", "/upload", raw)
        return OffloadHandle(ident, self.tier, f"{self.base_url}/load/{ident}", len(raw), tuple(value.shape),
                             value.dtype, str(value.device), sha256(raw).hexdigest())

    def get(self, handle: OffloadHandle, device: str | None = None) -> Tensor:
        record = self._call("GET", f"/load/{handle.id}")
        if handle.sha256 and sha256(_canonical(record)).hexdigest() != handle.sha256:
            raise ValueError("network offload payload checksum mismatch")
        return WIRE_RECORD.decode(record, handle, device)

    def drop(self, handle: OffloadHandle) -> None:
        self._call("DELETE", f"/release/{handle.id}")

    # reference API names
    offload_tensor = put

    def load_tensor(self, handle: OffloadHandle, *, device: str | None = None) -> Tensor:
        return self.get(handle, device)

    release = drop
