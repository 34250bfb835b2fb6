"""Memory-tier planner and offload executors.

Reference: runtime.py:18-368 (first-fit tier planner, JSON NVMe offload with
sha256 checks, HTTP network offload).  Those keep their formats and
messages.  Added for B200: :class:`PinnedHostTier`, the RAM tier as real
pinned host buffers moved with ``cudaMemcpyAsync`` on a dedicated side
stream (ordered against compute with CUDA events), which the ZeRO optimizer
uses to keep Adam moments in host RAM while the GPUs compute.
"""

from __future__ import annotations

import json
from dataclasses import dataclass
from hashlib import sha256
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer
from pathlib import Path
from threading import Thread
from typing import Any
from urllib.error import HTTPError
from urllib.request import Request, urlopen
from uuid import uuid4

import torch

from underhfs_b200.cuda import MemoryPolicy, MemoryTier, memory_budgets
from underhfs_b200.tensor import DType, Tensor, tensor

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
        return {
            "id": self.id, "tier": self.tier.value, "path": self.path, "bytes": self.bytes,
            "shape": list(self.shape), "dtype": self.dtype.value, "device": self.device, "sha256": self.sha256,
            "cached": self.cached,
        }


@dataclass
class TierBudget:
    tier: MemoryTier
    capacity_bytes: int
    used_bytes: int = 0

    @property
    def available_bytes(self) -> int:
        return max(0, self.capacity_bytes - self.used_bytes)

    def reserve(self, size: int) -> bool:
        if size > self.available_bytes:
            return False
        self.used_bytes += size
        return True


class MemoryPlanner:
    """First-fit placement over the policy's tiers; oversubscribes the last
    tier when offload is allowed, raises MemoryError otherwise."""

    def __init__(self, policy: MemoryPolicy, budgets: dict[MemoryTier, int]) -> None:
        self.policy = policy
        self.budgets = {t: TierBudget(t, int(budgets.get(t, 0))) for t in policy.tiers}

    def tensor_size_bytes(self, value: Tensor) -> int:
        return int(value.numel() * DTYPE_BYTES[value.dtype])

    def place_tensor(self, value: Tensor) -> Placement:
        return self.place_bytes(self.tensor_size_bytes(value))

    def place_bytes(self, size: int) -> Placement:
        if size < 0:
            raise ValueError("size must be non-negative")
        for tier in self.policy.tiers:
            if self.budgets[tier].reserve(size):
                return Placement(tier, size, "fits-budget")
        if not self.policy.allow_offload:
            raise MemoryError(f"tensor requires {size} bytes, but no configured tier has capacity")
        last = self.policy.tiers[-1]
        self.budgets[last].used_bytes += size
        return Placement(last, size, "oversubscribed-offload")

    def snapshot(self) -> dict[str, dict[str, int]]:
        return {
            t.value: {"capacity_bytes": b.capacity_bytes, "used_bytes": b.used_bytes,
                      "available_bytes": b.available_bytes}
            for t, b in self.budgets.items()
        }


def _data_digest(data: Any) -> str:
    return sha256(json.dumps(data, separators=(",", ":"), sort_keys=True).encode("utf-8")).hexdigest()


class OffloadExecutor:
    """NVMe tier: one JSON file per tensor (format ``underhfs.offload-tensor`` v1)."""

    FORMAT = "underhfs.offload-tensor"

    def __init__(self, policy: MemoryPolicy, root: str | Path | None = None) -> None:
        self.policy = policy
        self.root = Path(root or policy.scratch_path or ".underhfs-offload")
        self.root.mkdir(parents=True, exist_ok=True)
        self._prefetch_cache: dict[str, Tensor] = {}

    def offload_tensor(self, value: Tensor, tier: MemoryTier = MemoryTier.NVME) -> OffloadHandle:
        if tier not in (MemoryTier.NVME, MemoryTier.NETWORK):
            raise ValueError("offload executor currently supports NVMe/network tiers")
        if tier is MemoryTier.NETWORK:
            raise RuntimeError("network offload requires a configured remote transport")
        ident = uuid4().hex
        data = value.detach().tolist()
        record = {
            "format": self.FORMAT, "version": 1, "id": ident, "shape": list(value.shape),
            "dtype": value.dtype.value, "device": str(value.device), "data_sha256": _data_digest(data), "data": data,
        }
        raw = json.dumps(record, separators=(",", ":")).encode("utf-8")
        path = self.root / f"{ident}.uhfsoffload.json"
        path.write_bytes(raw)
        return OffloadHandle(ident, tier, str(path), len(raw), value.shape, value.dtype, str(value.device),
                             sha256(raw).hexdigest())

    def prefetch_tensor(self, handle: OffloadHandle) -> OffloadHandle:
        self._prefetch_cache[handle.id] = self.load_tensor(handle, use_cache=False)
        return OffloadHandle(handle.id, handle.tier, handle.path, handle.bytes, handle.shape, handle.dtype,
                             handle.device, handle.sha256, cached=True)

    def load_tensor(self, handle: OffloadHandle, *, device: str | None = None, use_cache: bool = True) -> Tensor:
        if use_cache and handle.id in self._prefetch_cache:
            return self._prefetch_cache[handle.id].detach().to(device or "cpu")
        raw = Path(handle.path).read_bytes()
        if handle.sha256 and sha256(raw).hexdigest() != handle.sha256:
            raise ValueError("offload payload checksum mismatch")
        record = json.loads(raw.decode("utf-8"))
        if record.get("format") != self.FORMAT:
            raise ValueError("not an underhfs offload tensor")
        if record.get("version") != 1:
            raise ValueError(f"unsupported offload tensor version: {record.get('version')}")
        if record.get("id") != handle.id:
            raise ValueError("offload handle id mismatch")
        if _data_digest(record["data"]) != record.get("data_sha256"):
            raise ValueError("offload tensor data checksum mismatch")
        if tuple(record["shape"]) != handle.shape:
            raise ValueError("offload tensor shape mismatch")
        out = tensor(record["data"], dtype=handle.dtype)
        return out.to(device) if device is not None else out

    def release(self, handle: OffloadHandle) -> None:
        self._prefetch_cache.pop(handle.id, None)
        Path(handle.path).unlink(missing_ok=True)

    def cache_info(self) -> dict[str, int]:
        return {"prefetched_tensors": len(self._prefetch_cache)}


class PinnedHostTier:
    """RAM tier as pinned host memory with asynchronous copies.

    ``offload(t)`` enqueues a device->host copy on the side stream after the
    current compute stream's pending work; ``fetch(h, out)`` enqueues the
    host->device copy; ``wait(h)`` makes the current stream wait for it.
    Nothing blocks the host.
    """

    def __init__(self, device: torch.device | str = "cuda") -> None:
        self.device = torch.device(device)
        self.stream = torch.cuda.Stream(device=self.device)
        self._buffers: dict[str, torch.Tensor] = {}
        self._events: dict[str, torch.cuda.Event] = {}

    def allocate(self, key: str, numel: int, dtype: torch.dtype = torch.float32) -> torch.Tensor:
        buf = torch.empty(numel, dtype=dtype, pin_memory=True)
        self._buffers[key] = buf
        return buf

    def host(self, key: str) -> torch.Tensor:
        return self._buffers[key]

    def offload(self, key: str, src: torch.Tensor) -> None:
        if key not in self._buffers:
            self.allocate(key, src.numel(), src.dtype)
        dst = self._buffers[key]
        ready = torch.cuda.Event()
        ready.record(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.stream):
            self.stream.wait_event(ready)
            dst.copy_(src.reshape(-1), non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(self.stream)
        src.record_stream(self.stream)
        self._events[key] = ev

    def fetch(self, key: str, out: torch.Tensor) -> None:
        src = self._buffers[key]
        ready = torch.cuda.Event()
        ready.record(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.stream):
            self.stream.wait_event(ready)
            out.reshape(-1).copy_(src, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(self.stream)
        out.record_stream(self.stream)
        self._events[key] = ev

    def wait(self, key: str) -> None:
        ev = self._events.get(key)
        if ev is not None:
            torch.cuda.current_stream(self.device).wait_event(ev)

    def bytes_resident(self) -> int:
        return sum(b.numel() * b.element_size() for b in self._buffers.values())


# ------------------------------------------------------------ network tier
_NET_FORMAT = "underhfs.network-offload-tensor"


def _validate_network_payload(payload: dict[str, Any]) -> None:
    if payload.get("format") != _NET_FORMAT:
        raise ValueError("not an underhfs network offload tensor")
    if payload.get("version") != 1:
        raise ValueError(f"unsupported network offload tensor version: {payload.get('version')}")
    if _data_digest(payload["data"]) != payload.get("data_sha256"):
        raise ValueError("network offload tensor data checksum mismatch")


class NetworkOffloadServer:
    """Threaded HTTP tensor store: GET /health, GET /load/<id>, POST /upload, DELETE /release/<id>."""

    def __init__(self, host: str = "127.0.0.1", port: int = 0) -> None:
        self._store: dict[str, dict[str, Any]] = {}
        self._server = ThreadingHTTPServer((host, port), self._make_handler())
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

    def _make_handler(self):
        store = self._store

        class Handler(BaseHTTPRequestHandler):
            def log_message(self, *_a) -> None:
                return

            def _reply(self, payload: Any, status: int = 200) -> None:
                body = json.dumps(payload).encode("utf-8")
                self.send_response(status)
                self.send_header("Content-Type", "application/json")
                self.send_header("Content-Length", str(len(body)))
                self.end_headers()
                self.wfile.write(body)

            def do_GET(self) -> None:
                if self.path == "/health":
                    return self._reply({"status": "ok", "tensors": len(store)})
                if self.path.startswith("/load/"):
                    key = self.path.rsplit("/", 1)[-1]
                    if key in store:
                        return self._reply(store[key])
                return self._reply({"error": "not found"}, 404)

            def do_POST(self) -> None:
                if self.path != "/upload":
                    return self._reply({"error": "not found"}, 404)
                try:
                    n = int(self.headers.get("Content-Length", "0"))
                    payload = json.loads(self.rfile.read(n).decode("utf-8")) if n else {}
                    _validate_network_payload(payload)
                    store[payload["id"]] = payload
                    self._reply({"ok": True, "id": payload["id"]})
                except Exception as exc:  # noqa: BLE001
                    self._reply({"error": str(exc)}, 400)

            def do_DELETE(self) -> None:
                if not self.path.startswith("/release/"):
                    return self._reply({"error": "not found"}, 404)
                key = self.path.rsplit("/", 1)[-1]
                store.pop(key, None)
                self._reply({"ok": True, "id": key})

        return Handler


class NetworkOffloadClient:
    def __init__(self, base_url: str, timeout: float = 5.0) -> None:
        self.base_url = base_url.rstrip("/")
        self.timeout = timeout

    def offload_tensor(self, value: Tensor) -> OffloadHandle:
        ident = uuid4().hex
        data = value.detach().tolist()
        payload = {
            "format": _NET_FORMAT, "version": 1, "id": ident, "shape": list(value.shape), "dtype": value.dtype.value,
            "device": str(value.device), "data_sha256": _data_digest(data), "data": data,
        }
        raw = json.dumps(payload, separators=(",", ":")).encode("utf-8")
        self._request("/upload", method="POST", data=raw)
        return OffloadHandle(ident, MemoryTier.NETWORK, f"{self.base_url}/load/{ident}", len(raw), value.shape,
                             value.dtype, str(value.device), sha256(raw).hexdigest())

    def load_tensor(self, handle: OffloadHandle, *, device: str | None = None) -> Tensor:
        payload = self._request(f"/load/{handle.id}")
        raw = json.dumps(payload, separators=(",", ":")).encode("utf-8")
        if handle.sha256 and sha256(raw).hexdigest() != handle.sha256:
            raise ValueError("network offload payload checksum mismatch")
        _validate_network_payload(payload)
        if tuple(payload["shape"]) != handle.shape:
            raise ValueError("network offload tensor shape mismatch")
        out = tensor(payload["data"], dtype=handle.dtype)
        return out.to(device) if device is not None else out

    def release(self, handle: OffloadHandle) -> None:
        self._request(f"/release/{handle.id}", method="DELETE")

    def _request(self, path: str, *, method: str = "GET", data: bytes | None = None) -> Any:
        req = Request(f"{self.base_url}{path}", data=data, headers={"Content-Type": "application/json"},
                      method=method)
        try:
            with urlopen(req, timeout=self.timeout) as resp:
                payload = json.loads(resp.read().decode("utf-8"))
        except HTTPError as exc:
            body = exc.read().decode("utf-8")
            try:
                payload = json.loads(body)
            except json.JSONDecodeError:
                raise RuntimeError(f"HTTP {exc.code}: {body}") from exc
            if isinstance(payload, dict) and "error" in payload:
                raise RuntimeError(str(payload["error"])) from exc
            raise RuntimeError(f"HTTP {exc.code}") from exc
        if isinstance(payload, dict) and "error" in payload:
            raise RuntimeError(str(payload["error"]))
        return payload


def planner_from_system(policy: MemoryPolicy | None = None, *, vram_fraction: float = 0.9) -> MemoryPlanner:
    return MemoryPlanner(policy or MemoryPolicy(), budgets=memory_budgets(vram_fraction=vram_fraction))
