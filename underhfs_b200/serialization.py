"""Checkpoint and export formats (reference serialization.py:10-403).

Byte-compatible formats kept:

* ``underhfs.safe-tensors-lite`` / ``underhfs.checkpoint`` JSON files;
* the binary state file ``b"UHFSBIN1" + <Q header length + JSON header +
  payload`` whose header lists per tensor ``dtype, shape, offset, nbytes,
  sha256`` plus ``payload_nbytes`` / ``payload_sha256``; readers validate
  magic, truncation, format, version, payload size and digest, span sign /
  alignment / bounds / overlap and per-tensor digests;
* ONNX (``onnx`` package) or the ``underhfs.onnx-lite`` JSON fallback, and
  the ``underhfs.export-manifest``.

Additions: values may be torch tensors or Tensors (serialized straight from
their bytes, no per-element Python work), ``bf16`` payloads as an opt-in
dtype, per-rank sharded checkpoints with a JSON index, and full training
resume (model, optimizer, step, RNG).
"""

from __future__ import annotations

import hashlib
import json
import struct
from pathlib import Path
from typing import Any

import numpy as np
import torch

FORMAT_VERSION = 1
BINARY_MAGIC = b"UHFSBIN1"
_LEN = struct.Struct("<Q")
_BIN_FORMAT = "underhfs.safe-tensors-binary"
_ELEM = {"fp32": 4, "bf16": 2}


# --------------------------------------------------------------- helpers
def _as_tensor(value: Any) -> torch.Tensor:
    if isinstance(value, torch.Tensor):
        return value.detach()
    data = getattr(value, "_data", None)
    if isinstance(data, torch.Tensor):
        return data.detach()
    return torch.tensor(value, dtype=torch.float64)


def _shape_of(value: Any) -> list[int]:
    if isinstance(value, list):
        return [0] if not value else [len(value), *_shape_of(value[0])]
    if isinstance(value, (int, float)):
        return []
    return list(_as_tensor(value).shape)


def _to_list(t: torch.Tensor) -> Any:
    return t.double().tolist() if t.dim() else float(t.item())


def _jsonable(state: dict[str, Any]) -> dict[str, Any]:
    return {k: (v if isinstance(v, (list, int, float)) else _to_list(_as_tensor(v).float().cpu()))
            for k, v in state.items()}


def _payload_bytes(value: Any, dtype: str) -> bytes:
    t = _as_tensor(value).cpu()
    if dtype == "fp32":
        arr = t.to(torch.float32).contiguous().numpy()
        return arr.astype("<f4", copy=False).tobytes()
    if dtype == "bf16":
        return t.to(torch.bfloat16).contiguous().view(torch.int16).numpy().astype("<i2", copy=False).tobytes()
    raise ValueError(f"unsupported tensor dtype in binary state: {dtype}")


# ------------------------------------------------------------ JSON state
def save_state_dict(path: str | Path, state: dict[str, Any]) -> None:
    doc = {"format": "underhfs.safe-tensors-lite", "version": FORMAT_VERSION, "state": _jsonable(state)}
    Path(path).write_text(json.dumps(doc, indent=2), encoding="utf-8")


def load_state_dict(path: str | Path) -> dict[str, Any]:
    doc = json.loads(Path(path).read_text(encoding="utf-8"))
    if doc.get("format") != "underhfs.safe-tensors-lite":
        raise ValueError("not an underhfs state file")
    return doc["state"]


# ---------------------------------------------------------- binary state
def save_binary_state_dict(path: str | Path, state: dict[str, Any], *, dtype: str = "fp32") -> None:
    """Write a UHFSBIN1 file.  ``dtype="fp32"`` (default) is readable by the
    reference's loader; ``"bf16"`` halves the size for bf16 models."""
    tensors: dict[str, Any] = {}
    chunks: list[bytes] = []
    offset = 0
    for name, value in state.items():
        data = _payload_bytes(value, dtype)
        tensors[name] = {"dtype": dtype, "shape": _shape_of(value), "offset": offset, "nbytes": len(data),
                         "sha256": hashlib.sha256(data).hexdigest()}
        chunks.append(data)
        offset += len(data)
    payload = b"".join(chunks)
    header = {"format": _BIN_FORMAT, "version": FORMAT_VERSION, "payload_nbytes": len(payload),
              "payload_sha256": hashlib.sha256(payload).hexdigest(), "tensors": tensors}
    enc = json.dumps(header, separators=(",", ":")).encode("utf-8")
    Path(path).write_bytes(BINARY_MAGIC + _LEN.pack(len(enc)) + enc + payload)


def _check_spans(tensors: dict[str, Any], payload_nbytes: int) -> None:
    spans = []
    for name, meta in tensors.items():
        off, n = int(meta["offset"]), int(meta["nbytes"])
        if off < 0 or n < 0:
            raise ValueError(f"invalid negative tensor span: {name}")
        elem = _ELEM.get(meta.get("dtype", "fp32"), 4)
        if n % elem != 0:
            label = "fp32" if elem == 4 else meta.get("dtype")
            raise ValueError(f"{label} tensor payload is not {elem}-byte aligned: {name}")
        if off + n > payload_nbytes:
            raise ValueError(f"tensor payload points past end of file: {name}")
        spans.append((off, off + n, name))
    spans.sort()
    end, prev = 0, ""
    for start, stop, name in spans:
        if start < end:
            raise ValueError(f"overlapping tensor payloads: {prev} and {name}")
        end, prev = stop, name


def _read_binary(path: str | Path) -> tuple[dict[str, Any], bytes]:
    data = Path(path).read_bytes()
    if len(data) < len(BINARY_MAGIC) + _LEN.size or not data.startswith(BINARY_MAGIC):
        raise ValueError("not an underhfs binary state file")
    hlen = _LEN.unpack_from(data, len(BINARY_MAGIC))[0]
    hstart = len(BINARY_MAGIC) + _LEN.size
    pstart = hstart + hlen
    if pstart > len(data):
        raise ValueError("truncated underhfs binary state header")
    header = json.loads(data[hstart:pstart].decode("utf-8"))
    if header.get("format") != _BIN_FORMAT:
        raise ValueError("not an underhfs binary state file")
    if header.get("version") != FORMAT_VERSION:
        raise ValueError(f"unsupported binary state version: {header.get('version')}")
    payload = data[pstart:]
    want = int(header.get("payload_nbytes", len(payload)))
    if want != len(payload):
        raise ValueError(f"binary state payload size mismatch: expected {want} bytes, got {len(payload)}")
    digest = header.get("payload_sha256")
    if digest and hashlib.sha256(payload).hexdigest() != digest:
        raise ValueError("binary state payload checksum mismatch")
    _check_spans(header["tensors"], len(payload))
    return header, payload


def load_binary_state_tensors(path: str | Path) -> dict[str, torch.Tensor]:
    """Load a UHFSBIN1 file as fp32 (or bf16) torch tensors."""
    header, payload = _read_binary(path)
    out: dict[str, torch.Tensor] = {}
    for name, meta in header["tensors"].items():
        dt = meta.get("dtype")
        if dt not in _ELEM:
            raise ValueError(f"unsupported tensor dtype in binary state: {dt}")
        start, n = int(meta["offset"]), int(meta["nbytes"])
        chunk = payload[start : start + n]
        if meta.get("sha256") and hashlib.sha256(chunk).hexdigest() != meta["sha256"]:
            raise ValueError(f"tensor payload checksum mismatch: {name}")
        shape = [int(d) for d in meta["shape"]]
        if dt == "fp32":
            arr = np.frombuffer(chunk, dtype="<f4").copy()
            t = torch.from_numpy(arr)
        else:
            t = torch.from_numpy(np.frombuffer(chunk, dtype="<i2").copy()).view(torch.bfloat16)
        expected = int(np.prod(shape)) if shape else 1
        if t.numel() != expected:
            raise ValueError(f"shape {shape} expects {expected} values, got {t.numel()}")
        out[name] = t.reshape(shape)
    return out


def load_binary_state_dict(path: str | Path) -> dict[str, Any]:
    """Reference-compatible loader: nested Python lists (fp32 values)."""
    return {k: _to_list(v.float()) for k, v in load_binary_state_tensors(path).items()}


# ------------------------------------------------------------ checkpoint
def save_checkpoint(path: str | Path, *, state: dict[str, Any], metadata: dict[str, Any] | None = None) -> None:
    doc = {"format": "underhfs.checkpoint", "version": FORMAT_VERSION, "metadata": metadata or {},
           "state": _jsonable(state)}
    Path(path).write_text(json.dumps(doc, indent=2), encoding="utf-8")


def load_checkpoint(path: str | Path) -> dict[str, Any]:
    doc = json.loads(Path(path).read_text(encoding="utf-8"))
    if doc.get("format") != "underhfs.checkpoint":
        raise ValueError("not an underhfs checkpoint")
    if doc.get("version") != FORMAT_VERSION:
        raise ValueError(f"unsupported checkpoint version: {doc.get('version')}")
    return doc


def save_sharded_checkpoint(directory: str | Path, *, rank: int, world_size: int, state: dict[str, Any],
                            metadata: dict[str, Any] | None = None) -> Path:
    """One ``rank{r}.uhfsbin`` per rank plus ``index.json`` written by rank 0."""
    root = Path(directory)
    root.mkdir(parents=True, exist_ok=True)
    shard = root / f"rank{rank}.uhfsbin"
    save_binary_state_dict(shard, state)
    if rank == 0:
        index = {"format": "underhfs.sharded-checkpoint", "version": FORMAT_VERSION, "world_size": world_size,
                 "shards": [f"rank{r}.uhfsbin" for r in range(world_size)], "metadata": metadata or {}}
        (root / "index.json").write_text(json.dumps(index, indent=2), encoding="utf-8")
    return shard


def load_sharded_checkpoint(directory: str | Path, rank: int | None = None) -> dict[str, Any]:
    root = Path(directory)
    index = json.loads((root / "index.json").read_text(encoding="utf-8"))
    if index.get("format") != "underhfs.sharded-checkpoint":
        raise ValueError("not an underhfs sharded checkpoint")
    ranks = range(index["world_size"]) if rank is None else [rank]
    return {"index": index, "shards": {r: load_binary_state_tensors(root / index["shards"][r]) for r in ranks}}


def save_training_state(path: str | Path, *, model, optimizer=None, step: int = 0,
                        extra: dict[str, Any] | None = None) -> None:
    """Model weights (UHFSBIN1, fp32) + optimizer + step + RNG in one directory."""
    root = Path(path)
    root.mkdir(parents=True, exist_ok=True)
    save_binary_state_dict(root / "model.uhfsbin", model.state_dict(as_tensors=True))
    opt_state = None
    if optimizer is not None:
        opt_state = {"step_count": getattr(optimizer, "step_count", 0)}
        flat = getattr(optimizer, "_m_flat", None)
        if flat is not None:
            torch.save({"m": optimizer._m_flat.cpu(), "v": optimizer._v_flat.cpu(),
                        "master": optimizer._flat.master.cpu()}, root / "optimizer.pt")
        else:
            opt_state.update(optimizer.state_dict())
    rng = {"torch": torch.get_rng_state().tolist()}
    if torch.cuda.is_available():
        rng["cuda"] = [s.tolist() for s in torch.cuda.get_rng_state_all()]
    meta = {"format": "underhfs.training-state", "version": FORMAT_VERSION, "step": step,
            "optimizer": opt_state, "rng": rng, "extra": extra or {}}
    (root / "state.json").write_text(json.dumps(meta), encoding="utf-8")


def load_training_state(path: str | Path, *, model, optimizer=None) -> dict[str, Any]:
    root = Path(path)
    meta = json.loads((root / "state.json").read_text(encoding="utf-8"))
    if meta.get("format") != "underhfs.training-state":
        raise ValueError("not an underhfs training state")
    model.load_state_dict(load_binary_state_tensors(root / "model.uhfsbin"))
    if optimizer is not None and meta.get("optimizer") is not None:
        if (root / "optimizer.pt").exists() and getattr(optimizer, "_m_flat", None) is not None:
            saved = torch.load(root / "optimizer.pt")
            optimizer._m_flat.copy_(saved["m"])
            optimizer._v_flat.copy_(saved["v"])
            optimizer._flat.master.copy_(saved["master"])
            optimizer._flat.params.copy_(saved["master"])
            optimizer.step_count = int(meta["optimizer"]["step_count"])
            optimizer._step_t.fill_(optimizer.step_count)
        elif "m" in meta["optimizer"]:
            optimizer.load_state_dict(meta["optimizer"])
    torch.set_rng_state(torch.tensor(meta["rng"]["torch"], dtype=torch.uint8))
    if "cuda" in meta["rng"] and torch.cuda.is_available():
        torch.cuda.set_rng_state_all([torch.tensor(s, dtype=torch.uint8) for s in meta["rng"]["cuda"]])
    return meta


# ------------------------------------------------------------------ ONNX
def _state_digest(state: dict[str, Any]) -> str:
    return hashlib.sha256(json.dumps(state, separators=(",", ":"), sort_keys=True).encode("utf-8")).hexdigest()


def export_onnx(path: str | Path, *, model_name: str, state: dict[str, Any], inputs: dict[str, Any] | None = None,
                include_state: bool = True) -> str:
    state = _jsonable(state)
    if _export_onnx_proto(path, model_name, state, inputs):
        return "onnx"
    doc = {
        "ir_version": 10, "producer_name": "underhfs", "format": "underhfs.onnx-lite", "version": FORMAT_VERSION,
        "state_sha256": _state_digest(state),
        "graph": {"name": model_name, "inputs": inputs or {},
                  "initializers": [{"name": k, "dims": _shape_of(v), "data_type": "FLOAT"} for k, v in state.items()]},
    }
    if include_state:
        doc["state"] = state
    target = Path(path)
    target.parent.mkdir(parents=True, exist_ok=True)
    target.write_text(json.dumps(doc, indent=2), encoding="utf-8")
    return "onnx-lite"


def _export_onnx_proto(path, model_name, state, inputs) -> bool:
    try:
        import onnx
        from onnx import TensorProto, helper
    except ImportError:
        return False
    inits = [helper.make_tensor(k, TensorProto.FLOAT, _shape_of(v), np.asarray(v, dtype=np.float32).reshape(-1))
             for k, v in state.items()]
    ins, outs, nodes = [], [], []
    for name, spec in (inputs or {}).items():
        shape = spec.get("shape", [])
        ins.append(helper.make_tensor_value_info(name, TensorProto.FLOAT, shape))
        outs.append(helper.make_tensor_value_info(f"{name}_out", TensorProto.FLOAT, shape))
        nodes.append(helper.make_node("Identity", [name], [f"{name}_out"], name=f"{name}_identity"))
    if not outs:
        outs = [helper.make_tensor_value_info(k, TensorProto.FLOAT, _shape_of(v)) for k, v in state.items()]
    model = helper.make_model(helper.make_graph(nodes, model_name, ins, outs, inits), producer_name="underhfs")
    model.metadata_props.append(onnx.StringStringEntryProto(key="format", value="underhfs.onnx"))
    model.metadata_props.append(onnx.StringStringEntryProto(key="state_sha256", value=_state_digest(state)))
    onnx.checker.check_model(model)
    Path(path).parent.mkdir(parents=True, exist_ok=True)
    onnx.save(model, str(path))
    return True


def import_onnx(path: str | Path) -> dict[str, Any]:
    try:
        return _import_onnx_proto(path)
    except ImportError:
        pass
    except Exception as exc:  # noqa: BLE001
        if Path(path).suffix == ".onnx":
            raise ValueError(f"failed to import ONNX protobuf model: {exc}") from exc
    doc = json.loads(Path(path).read_text(encoding="utf-8"))
    if doc.get("format") != "underhfs.onnx-lite":
        raise ValueError("only underhfs.onnx-lite manifests are supported without the optional ONNX runtime")
    if "state" in doc and _state_digest(doc["state"]) != doc.get("state_sha256"):
        raise ValueError("ONNX-lite state checksum mismatch")
    return doc


def _import_onnx_proto(path) -> dict[str, Any]:
    import onnx
    from onnx import numpy_helper

    model = onnx.load(str(path))

    def info(v):
        dims = []
        for d in v.type.tensor_type.shape.dim:
            dims.append(int(d.dim_value) if d.HasField("dim_value") else (d.dim_param or "?"))
        return {"name": v.name, "shape": dims,
                "data_type": onnx.TensorProto.DataType.Name(v.type.tensor_type.elem_type)}

    g = model.graph
    return {
        "format": "underhfs.onnx",
        "producer_name": model.producer_name,
        "metadata": {p.key: p.value for p in model.metadata_props},
        "graph": {
            "name": g.name,
            "inputs": [info(v) for v in g.input],
            "outputs": [info(v) for v in g.output],
            "nodes": [{"name": n.name, "op_type": n.op_type, "inputs": list(n.input), "outputs": list(n.output)}
                      for n in g.node],
            "initializers": [{"name": t.name, "dims": list(t.dims), "data_type": str(t.data_type)}
                             for t in g.initializer],
        },
        "state": {t.name: numpy_helper.to_array(t).tolist() for t in g.initializer},
    }


def load_onnx_state_dict(path: str | Path) -> dict[str, Any]:
    doc = import_onnx(path)
    if "state" not in doc:
        raise ValueError("ONNX-lite manifest does not include embedded state")
    return doc["state"]


def export_manifest(path: str | Path, *, model_name: str, state: dict[str, Any],
                    inputs: dict[str, Any] | None = None) -> None:
    doc = {"format": "underhfs.export-manifest", "version": FORMAT_VERSION, "model": model_name,
           "inputs": inputs or {}, "parameters": [{"name": k, "shape": _shape_of(v)} for k, v in state.items()]}
    Path(path).write_text(json.dumps(doc, indent=2), encoding="utf-8")


def load_manifest(path: str | Path) -> dict[str, Any]:
    doc = json.loads(Path(path).read_text(encoding="utf-8"))
    if doc.get("format") != "underhfs.export-manifest":
        raise ValueError("not an underhfs export manifest")
    return doc
