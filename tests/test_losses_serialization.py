"""Losses, embedding/conv/attention gradients and the checkpoint formats."""

import json
import struct
from pathlib import Path

from underhfs import tensor
from underhfs.functional import cross_entropy, mse_loss
from underhfs.nn import Conv2d, Embedding, Linear, SelfAttention
from underhfs.serialization import (
    BINARY_MAGIC,
    export_onnx,
    import_onnx,
    load_binary_state_dict,
    load_onnx_state_dict,
    load_state_dict,
    save_binary_state_dict,
    save_state_dict,
)


def _close(a, b, tol=1e-6):
    if isinstance(a, dict):
        return a.keys() == b.keys() and all(_close(a[k], b[k], tol) for k in a)
    if isinstance(a, list):
        return len(a) == len(b) and all(_close(x, y, tol) for x, y in zip(a, b))
    return abs(a - b) <= tol


def _scratch(tmp_path, name):
    return Path(name) if tmp_path is None else Path(tmp_path) / name


def test_mse_gradient():
    x = tensor([[1.0, 2.0]], requires_grad=True)
    mse_loss(x, tensor([[0.0, 4.0]])).backward()
    assert x.grad.tolist() == [[1.0, -2.0]]


def test_cross_entropy_rows_of_gradient_sum_to_zero():
    logits = tensor([[2.0, 0.0, -1.0], [0.5, 1.0, -0.5]], requires_grad=True)
    cross_entropy(logits, tensor([0, 1])).backward()
    assert logits.grad.shape == logits.shape
    assert all(abs(sum(r)) < 1e-9 for r in logits.grad.tolist())


def test_embedding_scatter_add():
    emb = Embedding(4, 3)
    emb(tensor([1, 1, 2])).sum().backward()
    g = emb.weight.grad.tolist()
    assert g[0] == [0.0] * 3 and g[1] == [2.0] * 3 and g[2] == [1.0] * 3


def test_json_state_roundtrip(tmp_path=None):
    path = _scratch(tmp_path, "state.json")
    lin = Linear(2, 1)
    save_state_dict(path, lin.state_dict())
    assert load_state_dict(path) == lin.state_dict()


def test_binary_state_roundtrip_and_magic(tmp_path=None):
    path = _scratch(tmp_path, "state.uhfsbin")
    lin = Linear(2, 1)
    save_binary_state_dict(path, lin.state_dict())
    assert _close(load_binary_state_dict(path), lin.state_dict())
    assert path.read_bytes().startswith(b"UHFSBIN1")


def test_binary_state_detects_payload_corruption(tmp_path=None):
    path = _scratch(tmp_path, "corrupt.uhfsbin")
    save_binary_state_dict(path, Linear(2, 1).state_dict())
    raw = bytearray(path.read_bytes())
    raw[-1] ^= 0xFF
    path.write_bytes(bytes(raw))
    try:
        load_binary_state_dict(path)
    except ValueError as exc:
        assert "checksum mismatch" in str(exc)
    else:
        raise AssertionError("flipped payload byte must fail the digest check")


def test_binary_state_detects_overlapping_spans(tmp_path=None):
    path = _scratch(tmp_path, "overlap.uhfsbin")
    save_binary_state_dict(path, Linear(2, 1).state_dict())
    raw = path.read_bytes()
    hlen = struct.unpack_from("<Q", raw, len(BINARY_MAGIC))[0]
    hstart = len(BINARY_MAGIC) + 8
    header = json.loads(raw[hstart : hstart + hlen])
    names = list(header["tensors"])
    header["tensors"][names[1]]["offset"] = header["tensors"][names[0]]["offset"]
    enc = json.dumps(header, separators=(",", ":")).encode()
    path.write_bytes(BINARY_MAGIC + struct.pack("<Q", len(enc)) + enc + raw[hstart + hlen :])
    try:
        load_binary_state_dict(path)
    except ValueError as exc:
        assert "overlapping tensor payloads" in str(exc)
    else:
        raise AssertionError("overlapping spans must be rejected")


def test_binary_bf16_payload_roundtrip(tmp_path=None):
    import torch

    from underhfs.serialization import load_binary_state_tensors

    path = _scratch(tmp_path, "bf16.uhfsbin")
    w = torch.randn(4, 8)
    save_binary_state_dict(path, {"w": w}, dtype="bf16")
    back = load_binary_state_tensors(path)["w"]
    assert back.dtype == torch.bfloat16 and torch.equal(back, w.to(torch.bfloat16))


def test_onnx_export_import(tmp_path=None):
    path = _scratch(tmp_path, "model.onnx.json")
    lin = Linear(2, 1)
    fmt = export_onnx(path, model_name="Linear", state=lin.state_dict(), inputs={"x": {"shape": [1, 2]}})
    doc = import_onnx(path)
    assert fmt in ("onnx", "onnx-lite")
    assert doc["producer_name"] == "underhfs"
    assert doc["graph"]["name"] == "Linear"
    if fmt == "onnx-lite":
        assert doc["state_sha256"]
        assert load_onnx_state_dict(path) == lin.state_dict()


def test_conv2d_values_and_gradients():
    conv = Conv2d(1, 1, kernel_size=2, bias=True)
    conv.weight._storage = [1.0, 2.0, 3.0, 4.0]
    conv.bias._storage = [0.5]
    x = tensor([[[[1.0, 2.0], [3.0, 4.0]]]], requires_grad=True)
    y = conv(x)
    assert y.shape == (1, 1, 1, 1) and y.item() == 30.5
    y.sum().backward()
    assert x.grad.tolist() == [[[[1.0, 2.0], [3.0, 4.0]]]]
    assert conv.weight.grad.tolist() == [[[[1.0, 2.0], [3.0, 4.0]]]]
    assert conv.bias.grad.tolist() == [1.0]


def test_self_attention_backward():
    attn = SelfAttention(2)
    x = tensor([[1.0, 0.0], [0.0, 1.0]], requires_grad=True)
    attn(x).sum().backward()
    assert x.grad.shape == x.shape
    assert any(p.grad is not None for p in attn.parameters())
