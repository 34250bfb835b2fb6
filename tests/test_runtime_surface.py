"""Policies, capability matrix, compile reports, data/DDP/serving surfaces."""

import base64
import json
import os
import socket
import sys
from pathlib import Path
from tempfile import TemporaryDirectory
from urllib.request import Request, urlopen

from underhfs.compile import CompilePolicy, FusionGroup, FusionKind, GraphIR, compile, explain, lower_to_plan
from underhfs.cuda import MemoryPolicy, MemoryTier, RuntimePolicy, capability_matrix, require_kernel, supports_kernel
from underhfs.data import DataLoader, TensorDataset
from underhfs.distributed import DistributedDataParallel, DistributedPolicy, nccl_runtime_plan, process_group
from underhfs.native import status
from underhfs.nn import Linear
from underhfs.serve import (
    ServeConfig,
    ServingProtocol,
    StreamSourceKind,
    open_stream,
    protocol_capabilities,
    require_protocol,
    serve,
    serve_cpp,
    serve_cpp_manifest,
    serve_grpc,
    serve_grpc_manifest,
    serve_http,
    serve_protocol,
    serve_websocket,
    serve_websocket_loop,
)
from underhfs.tensor import DType, tensor


def test_policies_and_kernel_matrix():
    pol = RuntimePolicy(memory=MemoryPolicy(tiers=(MemoryTier.VRAM, MemoryTier.RAM, MemoryTier.NVME)))
    assert pol.memory.allow_offload and pol.memory.tiers[-1] is MemoryTier.NVME
    assert pol.precision.dtype == "bf16"
    assert supports_kernel("add", device="cpu", dtype=DType.FP32)
    assert any(c.op == "matmul" for c in capability_matrix())
    try:
        require_kernel("matmul", device="cuda", dtype=DType.INT4)
    except RuntimeError as exc:
        assert "does not have" in str(exc)
    else:
        raise AssertionError("int4 CUDA matmul does not exist")


def test_compile_decorator_report():
    @compile(policy=CompilePolicy(enabled=True))
    def f(x):
        return (x * x + x).sum()

    assert f._underhfs_compile_policy.enabled
    out = f(tensor([1.0, 2.0], requires_grad=True))
    rep = f._underhfs_last_compile_report
    assert out.item() == 8.0
    assert rep.guards[0].shape == (2,)
    assert any(n.op == "sum" for n in rep.graph.nodes)
    assert any(g.kind is FusionKind.ELEMENTWISE for g in rep.fusion_groups)


def test_explain_serializes():
    d = explain(lambda x: (x + x).relu(), tensor([-1.0, 2.0])).to_dict()
    assert d["guards"][0]["dtype"] == "fp32"
    assert d["graph"]["nodes"]
    assert d["plan"]["fallback_backend"] == "eager-python"


def test_lowering_to_eager_plan_is_executable():
    rep = explain(lambda x: (x * x + x).sum(), tensor([1.0, 2.0]))
    plan = lower_to_plan(rep.graph, rep.fusion_groups)
    assert any(k.executable for k in plan.kernels)
    assert plan.kernels[0].dispatch(tensor([1.0, 2.0]), tensor([3.0, 4.0]), op="add").tolist() == [4.0, 6.0]


def test_native_required_rejects_cpu_fallback():
    try:
        explain(lambda x: (x * x + x).sum(), tensor([1.0, 2.0]),
                policy=CompilePolicy(native_required=True, allow_fallback=False))
    except RuntimeError as exc:
        assert "unsupported fusion groups" in str(exc) or "fallback is disabled" in str(exc)
    else:
        raise AssertionError("native-only compile must reject CPU groups")


def _attention_graph(out_cols: int = 5) -> GraphIR:
    g = GraphIR()
    g.add(name="qk", op="matmul", inputs=("q", "k"), outputs=("qk",), shape=(3, 3), dtype="fp32", device="cuda:0")
    g.add(name="w", op="softmax", inputs=("qk",), outputs=("w",), shape=(3, 3), dtype="fp32", device="cuda:0")
    g.add(name="o", op="matmul", inputs=("w", "v"), outputs=("o",), shape=(3, out_cols), dtype="fp32",
          device="cuda:0")
    return g


def test_attention_group_lowers_to_native():
    plan = lower_to_plan(_attention_graph(), (FusionGroup(FusionKind.ATTENTION, ("qk", "w", "o")),),
                         policy=CompilePolicy(native_required=True, allow_fallback=False))
    assert plan.kernels[0].backend == "native-cuda-attention"


def test_native_attention_dispatch_on_gpu():
    if not status().cuda_enabled:
        return
    plan = lower_to_plan(_attention_graph(2), (FusionGroup(FusionKind.ATTENTION, ("qk", "w", "o")),),
                         policy=CompilePolicy(native_required=True, allow_fallback=False))
    q = tensor([[1.0, 0.0], [0.0, 1.0]]).cuda()
    v = tensor([[1.0, 2.0], [3.0, 4.0]]).cuda()
    out = plan.kernels[0].dispatch(q, q, v, scale=1.0)
    assert out.backend == "native_cuda_attention" and str(out.device) == "cuda:0"
    assert out.tolist()[0][0] > 1.0


def test_native_fused_dispatch_on_gpu():
    if not status().cuda_enabled:
        return
    x, y = tensor([1.0, 2.0]).cuda(), tensor([3.0, 4.0]).cuda()
    rep = explain(lambda a, b: (a + b) * (a + b), x, y)
    k = next(k for k in rep.plan.kernels if k.backend == "native-cuda-fused")
    out = k.dispatch(x, y, op="add")
    assert out.backend == "native_cuda" and out.tolist() == [4.0, 6.0]


def test_guard_specialization_cache():
    @compile(policy=CompilePolicy(enabled=True, guard_specialization=True))
    def f(x):
        return (x + x).sum()

    r1 = (f(tensor([1.0, 2.0])), f._underhfs_last_compile_report)
    r2 = (f(tensor([3.0, 4.0])), f._underhfs_last_compile_report)
    r3 = (f(tensor([[1.0], [2.0]])), f._underhfs_last_compile_report)
    assert [r[0].item() for r in (r1, r2, r3)] == [6.0, 14.0, 6.0]
    assert r1[1].cache_hit is False and r2[1].cache_hit is True
    assert (r2[1].cache_info.hits, r2[1].cache_info.misses, r2[1].cache_info.specializations) == (1, 1, 1)
    assert r3[1].cache_hit is False and r3[1].cache_info.specializations == 2


def test_single_rank_group_ddp_and_python_serving():
    assert list(DataLoader(TensorDataset([1, 2, 3]), batch_size=2)) == [[1, 2], [3]]
    ddp = DistributedDataParallel(Linear(1, 1))
    assert ddp.policy.world_size == 1
    g = process_group(DistributedPolicy())
    assert (g.rank, g.world_size, g.backend) == (0, 1, "nccl")
    assert g.all_reduce_sum(3) == 3
    assert g.broadcast("ok") == "ok"
    assert g.reduce_scatter(["only-rank"]) == "only-rank"
    assert g.all_gather("ok") == ["ok"]
    assert nccl_runtime_plan(DistributedPolicy(world_size=2)).to_dict()["backend"] == "nccl"
    if not status().nccl_enabled:
        try:
            process_group(DistributedPolicy(world_size=2))
        except RuntimeError as exc:
            assert "UNDERHFS_WITH_NCCL=ON" in str(exc)
        else:
            raise AssertionError("world_size > 1 without NCCL must fail")
    with ddp.no_sync():
        assert ddp.group.synchronized is False
    assert ddp.group.synchronized is True
    assert serve(lambda p: {"echo": p}).predict("ok") == {"echo": "ok"}
    assert serve_protocol(lambda p: p, ServingProtocol.PYTHON).predict("ok") == "ok"
    assert serve_websocket(lambda p: p["value"]).predict_frame('{"value":"ok"}') == '{"result": "ok"}'
    assert any(c.protocol is ServingProtocol.HTTP and c.available for c in protocol_capabilities())
    require_protocol(ServingProtocol.GRPC)
    assert serve_grpc_manifest().to_dict()["protocol"] == "grpc"
    assert serve_cpp_manifest().to_dict()["protocol"] == "cpp"


def test_launch_plan_names_existing_module():
    import importlib

    cmd = nccl_runtime_plan(DistributedPolicy(world_size=4)).launch_command
    assert importlib.import_module(cmd[2]) is not None


def test_grpc_roundtrip():
    try:
        srv = serve_grpc(lambda p: p["value"], ServeConfig(port=0)).start()
    except RuntimeError as exc:
        assert "grpcio" in str(exc)
        return
    try:
        import grpc

        with grpc.insecure_channel(f"{srv.host}:{srv.port}") as ch:
            call = ch.unary_unary("/underhfs.grpc.JsonPredictService/Predict")
            reply = call(json.dumps({"value": "ok"}).encode(), timeout=5)
        assert json.loads(reply.decode()) == {"result": "ok"}
    finally:
        srv.close()


def test_cpp_wrapper_speaks_json_lines():
    with TemporaryDirectory() as tmp:
        fake = Path(tmp) / "fake_serve.py"
        fake.write_text(
            "import json, sys\n"
            "for line in sys.stdin:\n"
            "    m = json.loads(line)\n"
            "    if m.get('op') == 'exit': break\n"
            "    if m.get('op') == 'health': print(json.dumps({'status': 'ok'}), flush=True); continue\n"
            "    if m.get('op') == 'predict': print(json.dumps({'result': m.get('payload')}), flush=True); continue\n"
            "    print(json.dumps({'error': 'unsupported op'}), flush=True)\n"
        )
        srv = serve_cpp([sys.executable, str(fake)])
        try:
            assert srv.request({"op": "health"}) == {"status": "ok"}
            assert srv.predict({"value": "ok"}) == {"value": "ok"}
        finally:
            srv.close()


def test_native_cpp_server_binary():
    from underhfs.serve import default_cpp_executable

    exe = default_cpp_executable()
    if not exe.exists():
        return
    srv = serve_cpp(exe)
    try:
        assert srv.request({"op": "health"}) == {"status": "ok"}
        assert srv.predict({"op": "inner", "x": [1, 2]}) == {"op": "inner", "x": [1, 2]}
    finally:
        srv.close()


def test_http_predict():
    srv = serve_http(lambda p: {"echo": p["value"]}, ServeConfig(port=0)).start()
    try:
        with urlopen(f"{srv.url}/health", timeout=5) as r:
            assert json.loads(r.read()) == {"status": "ok"}
        for route in ("/predict", "/v1/predict"):
            req = Request(f"{srv.url}{route}", data=json.dumps({"value": "ok"}).encode(),
                          headers={"Content-Type": "application/json"}, method="POST")
            with urlopen(req, timeout=5) as r:
                assert json.loads(r.read()) == {"result": {"echo": "ok"}}
    finally:
        srv.close()


def test_file_stream_chunks(tmp_path=None):
    path = Path(tmp_path or ".") / "stream.bin"
    path.write_bytes(b"abcdef")
    assert [f.data for f in open_stream(str(path), StreamSourceKind.FILE, chunk_bytes=2)] == [b"ab", b"cd", b"ef"]
    if tmp_path is None:
        path.unlink()


def _masked_text(text: str) -> bytes:
    data = text.encode()
    mask = b"\x05\x06\x07\x08"
    return bytes([0x81, 0x80 | len(data)]) + mask + bytes(b ^ mask[i % 4] for i, b in enumerate(data))


def _read_text(sock: socket.socket) -> str:
    head = sock.recv(2)
    n = head[1] & 0x7F
    if n == 126:
        n = int.from_bytes(sock.recv(2), "big")
    elif n == 127:
        n = int.from_bytes(sock.recv(8), "big")
    return sock.recv(n).decode()


def test_websocket_loop_predict():
    srv = serve_websocket_loop(lambda p: p["value"], ServeConfig(port=0)).start()
    try:
        with socket.create_connection((srv.host, srv.port), timeout=5) as s:
            key = base64.b64encode(os.urandom(16)).decode()
            s.sendall((f"GET / HTTP/1.1\r\nHost: {srv.host}\r\nUpgrade: websocket\r\nConnection: Upgrade\r\n"
                       f"Sec-WebSocket-Key: {key}\r\nSec-WebSocket-Version: 13\r\n\r\n").encode())
            assert "101 Switching Protocols" in s.recv(4096).decode(errors="ignore")
            s.sendall(_masked_text('{"value":"ok"}'))
            assert json.loads(_read_text(s)) == {"result": "ok"}
    finally:
        srv.close()


def test_to_cpu_dtype_and_cuda_contract():
    x = tensor([1.0, 2.0]).to(dtype=DType.FP16)
    assert x.dtype is DType.FP16 and str(x.cpu().device) == "cpu"
    if status().cuda_enabled:
        assert str(x.cuda().device) == "cuda:0"
    else:
        try:
            x.cuda()
        except RuntimeError as exc:
            assert "native core is unavailable" in str(exc) or "built without CUDA support" in str(exc)
        else:
            raise AssertionError(".cuda() without a device must fail loudly")
