"""Serving surfaces and stream sources (reference serve.py:18-571).

Protocols: in-process Python, JSON over HTTP (``/health``, ``/predict``,
``/v1/predict``), WebSocket text frames (RFC 6455 handshake and framing),
gRPC (generic handler ``/underhfs.grpc.JsonPredictService/Predict`` with JSON
bytes, needs ``grpcio``) and a native C++ JSON-lines process
(``underhfs_cpp_serve``, built from csrc/serve/serve_main.cpp).  Streams: file
chunks, OpenCV webcam, ffmpeg RTSP/HLS.
"""

from __future__ import annotations

import base64
import hashlib
import json
import socket
from concurrent import futures
from dataclasses import dataclass
from enum import Enum
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer
from pathlib import Path
from shutil import which
from subprocess import PIPE, Popen, TimeoutExpired
from threading import Thread
from typing import Any, Callable, Iterator, Sequence

Handler = Callable[[Any], Any]


class ServingProtocol(str, Enum):
    PYTHON = "python"
    HTTP = "http"
    WEBSOCKET = "websocket"
    GRPC = "grpc"
    CPP = "cpp"


class StreamSourceKind(str, Enum):
    FILE = "file"
    WEBCAM = "webcam"
    RTSP = "rtsp"
    HLS = "hls"
    WEBRTC = "webrtc"
    NETWORK = "network"


@dataclass(frozen=True)
class StreamFrame:
    index: int
    data: bytes
    source: str
    kind: StreamSourceKind

    def to_dict(self) -> dict[str, Any]:
        return {"index": self.index, "bytes": len(self.data), "source": self.source, "kind": self.kind.value}


@dataclass(frozen=True)
class ProtocolCapability:
    protocol: ServingProtocol
    available: bool
    transport: str
    reason: str = ""

    def to_dict(self) -> dict[str, Any]:
        return {"protocol": self.protocol.value, "available": self.available, "transport": self.transport,
                "reason": self.reason}


@dataclass
class ServeConfig:
    host: str = "127.0.0.1"
    port: int = 8765
    protocols: tuple[ServingProtocol, ...] = (ServingProtocol.PYTHON, ServingProtocol.HTTP, ServingProtocol.WEBSOCKET)


@dataclass
class ServingManifest:
    protocol: ServingProtocol
    entrypoint: str
    config: ServeConfig

    def to_dict(self) -> dict[str, Any]:
        return {"protocol": self.protocol.value, "entrypoint": self.entrypoint, "host": self.config.host,
                "port": self.config.port}


class PythonServer:
    def __init__(self, handler: Handler, config: ServeConfig | None = None) -> None:
        self.handler = handler
        self.config = config or ServeConfig()

    def predict(self, payload: Any) -> Any:
        return self.handler(payload)


class _Threaded:
    """start()/close() around a blocking serve loop on a daemon thread."""

    _thread: Thread | None = None

    def _run(self) -> None:  # pragma: no cover - overridden
        raise NotImplementedError

    def start(self):
        if self._thread is None:
            self._thread = Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def _join(self) -> None:
        if self._thread is not None:
            self._thread.join(timeout=2.0)
            self._thread = None


class JsonHTTPServer(_Threaded):
    def __init__(self, handler: Handler, config: ServeConfig | None = None) -> None:
        self.handler = handler
        self.config = config or ServeConfig()
        self._server = ThreadingHTTPServer((self.config.host, self.config.port), self._handler_class())
        self.host, self.port = self._server.server_address[:2]

    @property
    def url(self) -> str:
        return f"http://{self.host}:{self.port}"

    def _run(self) -> None:
        self._server.serve_forever()

    def close(self) -> None:
        self._server.shutdown()
        self._server.server_close()
        self._join()

    def _handler_class(self):
        predict = self.handler

        class H(BaseHTTPRequestHandler):
            def log_message(self, *_a) -> None:
                return

            def _json(self, obj: Any, code: int = 200) -> None:
                body = json.dumps(obj).encode("utf-8")
                self.send_response(code)
                self.send_header("Content-Type", "application/json")
                self.send_header("Content-Length", str(len(body)))
                self.end_headers()
                self.wfile.write(body)

            def do_GET(self) -> None:
                if self.path == "/health":
                    self._json({"status": "ok"})
                else:
                    self._json({"error": "not found"}, 404)

            def do_POST(self) -> None:
                if self.path not in ("/predict", "/v1/predict"):
                    return self._json({"error": "not found"}, 404)
                try:
                    n = int(self.headers.get("Content-Length", "0"))
                    payload = json.loads(self.rfile.read(n).decode("utf-8")) if n else {}
                    self._json({"result": predict(payload)})
                except Exception as exc:  # noqa: BLE001
                    self._json({"error": str(exc)}, 500)

        return H


class JsonWebSocketServer(PythonServer):
    def predict_frame(self, text_frame: str) -> str:
        return json.dumps({"result": self.predict(json.loads(text_frame))})


_WS_MAGIC = "258EAFA5-E914-47DA-95CA-C5AB0DC85B11"


def _ws_accept(key: str) -> str:
    return base64.b64encode(hashlib.sha1((key + _WS_MAGIC).encode("ascii")).digest()).decode("ascii")


def _read_n(sock: socket.socket, n: int) -> bytes | None:
    buf = bytearray()
    while len(buf) < n:
        part = sock.recv(n - len(buf))
        if not part:
            return None
        buf += part
    return bytes(buf)


def _ws_read_text(sock: socket.socket) -> str | None:
    head = _read_n(sock, 2)
    if head is None:
        return None
    opcode, masked, size = head[0] & 0x0F, bool(head[1] & 0x80), head[1] & 0x7F
    if opcode == 0x8:
        return None
    if opcode != 0x1:
        raise RuntimeError("only WebSocket text frames are supported")
    if size in (126, 127):
        ext = _read_n(sock, 2 if size == 126 else 8)
        if ext is None:
            return None
        size = int.from_bytes(ext, "big")
    mask = _read_n(sock, 4) if masked else bytes(4)
    data = _read_n(sock, size)
    if data is None or mask is None:
        return None
    if masked:
        data = bytes(b ^ mask[i & 3] for i, b in enumerate(data))
    return data.decode("utf-8")


def _ws_text_frame(text: str) -> bytes:
    data = text.encode("utf-8")
    n = len(data)
    if n < 126:
        head = bytes([0x81, n])
    elif n < 1 << 16:
        head = bytes([0x81, 126]) + n.to_bytes(2, "big")
    else:
        head = bytes([0x81, 127]) + n.to_bytes(8, "big")
    return head + data


class WebSocketPredictServer(JsonWebSocketServer, _Threaded):
    def __init__(self, handler: Handler, config: ServeConfig | None = None) -> None:
        super().__init__(handler, config)
        self._sock = socket.socket(socket.AF_INET, socket.SOCK_STREAM)
        self._sock.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
        self._sock.bind((self.config.host, self.config.port))
        self._sock.listen(16)
        self.host, self.port = self._sock.getsockname()[:2]
        self._closed = False

    @property
    def url(self) -> str:
        return f"ws://{self.host}:{self.port}"

    def _run(self) -> None:
        while not self._closed:
            try:
                conn, _ = self._sock.accept()
            except OSError:
                return
            Thread(target=self._client, args=(conn,), daemon=True).start()

    def _client(self, conn: socket.socket) -> None:
        with conn:
            request = conn.recv(4096).decode("utf-8", errors="ignore")
            key = ""
            for line in request.split("\r\n"):
                if line.lower().startswith("sec-websocket-key:"):
                    key = line.split(":", 1)[1].strip()
            if not key:
                return
            conn.sendall(("HTTP/1.1 101 Switching Protocols\r\nUpgrade: websocket\r\nConnection: Upgrade\r\n"
                          f"Sec-WebSocket-Accept: {_ws_accept(key)}\r\n\r\n").encode("ascii"))
            while not self._closed:
                text = _ws_read_text(conn)
                if text is None:
                    return
                conn.sendall(_ws_text_frame(self.predict_frame(text)))

    def close(self) -> None:
        self._closed = True
        try:
            self._sock.shutdown(socket.SHUT_RDWR)
        except OSError:
            pass
        self._sock.close()
        self._join()


class GrpcJsonPredictServer:
    SERVICE = "underhfs.grpc.JsonPredictService"

    def __init__(self, handler: Handler, config: ServeConfig | None = None) -> None:
        self.handler = handler
        self.config = config or ServeConfig()
        try:
            import grpc
        except ImportError as exc:
            raise RuntimeError("gRPC serving requires optional dependency grpcio") from exc
        self._server = grpc.server(futures.ThreadPoolExecutor(max_workers=4))
        self._server.add_generic_rpc_handlers((self._generic(grpc),))
        self.port = self._server.add_insecure_port(f"{self.config.host}:{self.config.port}")
        self.host = self.config.host
        self.url = f"grpc://{self.host}:{self.port}"
        self._started = False

    def _generic(self, grpc):
        handler = self.handler
        method = f"/{self.SERVICE}/Predict"

        def call(raw: bytes, _ctx) -> bytes:
            payload = json.loads(raw.decode("utf-8")) if raw else {}
            return json.dumps({"result": handler(payload)}).encode("utf-8")

        class Generic(grpc.GenericRpcHandler):
            def service(self, details):
                if details.method != method:
                    return None
                return grpc.unary_unary_rpc_method_handler(call, request_deserializer=None,
                                                           response_serializer=None)

        return Generic()

    def start(self) -> "GrpcJsonPredictServer":
        if not self._started:
            self._server.start()
            self._started = True
        return self

    def close(self) -> None:
        if self._started:
            self._server.stop(grace=0).wait(timeout=2.0)
            self._started = False

    def predict(self, payload: Any) -> Any:
        return self.handler(payload)


class CppJsonPredictServer:
    """JSON lines over stdin/stdout of a native process ({"op": ...} requests)."""

    def __init__(self, executable: str | Path | Sequence[str] | None = None) -> None:
        if isinstance(executable, Sequence) and not isinstance(executable, (str, bytes, Path)):
            self.command = [str(x) for x in executable]
        else:
            self.command = [str(executable or default_cpp_executable())]
        self.executable = self.command[0]
        self._proc: Popen | None = None

    def start(self) -> "CppJsonPredictServer":
        if self._proc is None:
            if not Path(self.executable).exists():
                raise RuntimeError(f"C++ serving executable not found: {self.executable}")
            self._proc = Popen(self.command, stdin=PIPE, stdout=PIPE, stderr=PIPE, text=True)
        return self

    def request(self, payload: dict[str, Any]) -> dict[str, Any]:
        self.start()
        assert self._proc is not None and self._proc.stdin and self._proc.stdout
        self._proc.stdin.write(json.dumps(payload, separators=(",", ":")) + "\n")
        self._proc.stdin.flush()
        line = self._proc.stdout.readline()
        if not line:
            raise RuntimeError("C++ serving process exited without a response")
        reply = json.loads(line)
        if "error" in reply:
            raise RuntimeError(str(reply["error"]))
        return reply

    def predict(self, payload: Any) -> Any:
        return self.request({"op": "predict", "payload": payload})["result"]

    def close(self) -> None:
        if self._proc is None:
            return
        try:
            if self._proc.stdin is not None:
                self._proc.stdin.write(json.dumps({"op": "exit"}) + "\n")
                self._proc.stdin.flush()
            self._proc.wait(timeout=2.0)
        except (BrokenPipeError, TimeoutExpired):
            self._proc.kill()
        finally:
            self._proc = None


def serve(handler: Handler, config: ServeConfig | None = None) -> PythonServer:
    return PythonServer(handler, config)


def serve_http(handler: Handler, config: ServeConfig | None = None) -> JsonHTTPServer:
    return JsonHTTPServer(handler, config)


def serve_websocket(handler: Handler, config: ServeConfig | None = None) -> JsonWebSocketServer:
    return JsonWebSocketServer(handler, config)


def serve_websocket_loop(handler: Handler, config: ServeConfig | None = None) -> WebSocketPredictServer:
    return WebSocketPredictServer(handler, config)


def serve_grpc(handler: Handler, config: ServeConfig | None = None) -> GrpcJsonPredictServer:
    return GrpcJsonPredictServer(handler, config)


def serve_grpc_manifest(config: ServeConfig | None = None) -> ServingManifest:
    return ServingManifest(ServingProtocol.GRPC, GrpcJsonPredictServer.SERVICE, config or ServeConfig())


def serve_cpp(executable: str | Path | Sequence[str] | None = None) -> CppJsonPredictServer:
    return CppJsonPredictServer(executable)


def serve_cpp_manifest(config: ServeConfig | None = None) -> ServingManifest:
    return ServingManifest(ServingProtocol.CPP, "underhfs_cpp_serve", config or ServeConfig())


def default_cpp_executable() -> Path:
    found = which("underhfs_cpp_serve")
    if found:
        return Path(found)
    here = Path(__file__).resolve().parent
    for cand in (here / "bin" / "underhfs_cpp_serve", here.parent / "build" / "native" / "underhfs_cpp_serve"):
        if cand.exists():
            return cand
    return here / "bin" / "underhfs_cpp_serve"


def _has_module(name: str) -> bool:
    try:
        __import__(name)
        return True
    except ImportError:
        return False


def protocol_capabilities() -> list[ProtocolCapability]:
    grpc_ok = _has_module("grpc")
    cpp = default_cpp_executable()
    return [
        ProtocolCapability(ServingProtocol.PYTHON, True, "in-process callable"),
        ProtocolCapability(ServingProtocol.HTTP, True, "standard-library JSON HTTP"),
        ProtocolCapability(ServingProtocol.WEBSOCKET, True, "standard-library WebSocket JSON server",
                           "text-frame predict loop"),
        ProtocolCapability(ServingProtocol.GRPC, True, "grpcio JSON predict service" if grpc_ok else "service manifest",
                           "grpcio runtime available" if grpc_ok else "install grpcio to enable the gRPC runtime"),
        ProtocolCapability(ServingProtocol.CPP, cpp.exists(), "native executable JSON stdin/stdout",
                           "C++ serving executable available" if cpp.exists()
                           else "build the native core to produce underhfs_cpp_serve"),
    ]


def require_protocol(protocol: ServingProtocol | str) -> None:
    want = ServingProtocol(protocol)
    for cap in protocol_capabilities():
        if cap.protocol is want:
            if cap.available:
                return
            raise RuntimeError(f"{want.value} serving is unavailable: {cap.reason}")
    raise RuntimeError(f"unknown serving protocol: {want.value}")


def serve_protocol(handler: Handler, protocol: ServingProtocol | str, config: ServeConfig | None = None):
    want = ServingProtocol(protocol)
    require_protocol(want)
    factory = {ServingProtocol.PYTHON: serve, ServingProtocol.HTTP: serve_http,
               ServingProtocol.WEBSOCKET: serve_websocket, ServingProtocol.GRPC: serve_grpc}.get(want)
    if factory is None:
        raise RuntimeError(f"{want.value} serving uses a native process wrapper instead of in-process prediction")
    return factory(handler, config)


def open_stream(source: str, kind: StreamSourceKind = StreamSourceKind.FILE, *,
                chunk_bytes: int = 4096) -> Iterator[StreamFrame]:
    if chunk_bytes <= 0:
        raise ValueError("chunk_bytes must be positive")
    if kind is StreamSourceKind.FILE:
        with Path(source).open("rb") as fh:
            i = 0
            while chunk := fh.read(chunk_bytes):
                yield StreamFrame(i, chunk, str(Path(source)), kind)
                i += 1
        return
    if kind is StreamSourceKind.WEBCAM:
        yield from _opencv_frames(source, kind, chunk_bytes)
        return
    if kind in (StreamSourceKind.RTSP, StreamSourceKind.HLS):
        yield from _ffmpeg_frames(source, kind, chunk_bytes)
        return
    if kind is StreamSourceKind.WEBRTC:
        raise RuntimeError("webrtc streaming requires an optional WebRTC transport adapter")
    raise RuntimeError(f"{kind.value} streaming requires a configured network transport")


def _ffmpeg_frames(source: str, kind: StreamSourceKind, chunk_bytes: int) -> Iterator[StreamFrame]:
    if which("ffmpeg") is None:
        raise RuntimeError(f"{kind.value} streaming requires ffmpeg on PATH")
    proc = Popen(["ffmpeg", "-hide_banner", "-loglevel", "error", "-i", source, "-f", "rawvideo", "-"],
                 stdout=PIPE, stderr=PIPE)
    assert proc.stdout is not None
    try:
        i = 0
        while chunk := proc.stdout.read(chunk_bytes):
            yield StreamFrame(i, chunk, source, kind)
            i += 1
    finally:
        proc.terminate()


def _opencv_frames(source: str, kind: StreamSourceKind, chunk_bytes: int) -> Iterator[StreamFrame]:
    try:
        import cv2
    except ImportError as exc:
        raise RuntimeError("webcam streaming requires opencv-python") from exc
    cap = cv2.VideoCapture(int(source) if source.isdigit() else source)
    if not cap.isOpened():
        raise RuntimeError(f"could not open OpenCV stream source: {source}")
    try:
        i = 0
        while True:
            ok, frame = cap.read()
            if not ok:
                break
            raw = frame.tobytes()
            for off in range(0, len(raw), chunk_bytes):
                yield StreamFrame(i, raw[off : off + chunk_bytes], source, kind)
                i += 1
    finally:
        cap.release()
