"""The stage server's side of a layer pipeline, and the coordinator's
connection to it, over a byte stream.

Restates rakkan-mesh's stage protocol (internal/llm/service.go):
  * frames: a 4-byte big-endian length, then the bytes (writeFrame /
    readFrame, service.go:671-691); requests and statuses are JSON
    (request 46-57, status 59-62; writeStatus / readStatus 693-715);
  * a connection opens one stage of one generation: {"op": "open", "model",
    "from", "to", "ctx"} -> status; then, until the coordinator closes it,
    {"op": "forward", "pos", "tokens"} and a frame of tokens·dim
    little-endian float32 activations -> status and a frame of the stage's
    output activations (Service.handle, service.go:722-823;
    llamaStage.forward, 186-199);
  * a forward outside the generation's positions is answered with an error
    status and the connection ends; an unknown op resets it.

The reference carries these frames over libp2p streams between mesh
nodes; here they run over a local TCP stream (the mesh transport, its
certificates, gas and the trust layer are not part of this path). The
server opens each stage with a caller-supplied function, in this package a
CUDA rk.Stage of the requested layer span; RemoteStage gives the
coordinator (coordinator.run_stage) the forward/close of such a stage.
"""
import json
import socket
import socketserver
import struct
import threading

import numpy as np

MAX_REQUEST = 64 << 10  # service.go:44


class FrameError(RuntimeError):
    pass


def _read_full(r, n):
    buf = bytearray()
    while len(buf) < n:
        chunk = r.read(n - len(buf))
        if not chunk:
            raise FrameError("stream closed")
        buf += chunk
    return bytes(buf)


def write_frame(w, b):
    w.write(struct.pack(">I", len(b)))
    w.write(b)
    w.flush()


def read_frame(r, limit):
    n = struct.unpack(">I", _read_full(r, 4))[0]
    if n > limit:
        raise FrameError(f"frame of {n} bytes exceeds {limit}")
    return _read_full(r, n)


def write_status(w, err=None):
    st = {"ok": err is None}
    if err is not None:
        st["error"] = str(err)
    write_frame(w, json.dumps(st, separators=(",", ":")).encode())


def read_status(r):
    st = json.loads(read_frame(r, MAX_REQUEST))
    if not st.get("ok"):
        raise RuntimeError(st.get("error", "stage error"))


def encode_acts(xs):
    """encodeActs (service.go:717): little-endian float32."""
    return np.ascontiguousarray(xs, dtype="<f4").tobytes()


def decode_acts(b, dim):
    """decodeActs (service.go:719), as rows of dim."""
    return np.frombuffer(b, dtype="<f4").astype(np.float32).reshape(-1, dim)


class StageHandle:
    """What open_stage returns: forward(xs [tokens][dim], pos) -> xs',
    close(), dim, and positions (the generation's context)."""

    def __init__(self, forward, close, dim, positions):
        self.forward, self.close, self.dim, self.positions = forward, close, dim, positions


def handle(rfile, wfile, open_stage, fail_next=None):
    """Service.handle (service.go:722-823) for one connection. open_stage(req)
    -> StageHandle for the open request's model, from, to and ctx; an
    exception becomes an error status. fail_next(shard), if given, is asked
    before each forward and, when true, drops the connection as a crashed
    node would (the reference's failNext, service.go:797-800)."""
    try:
        req = json.loads(read_frame(rfile, MAX_REQUEST))
    except (FrameError, ValueError):
        return
    if req.get("op") != "open":
        return
    try:
        stage = open_stage(req)
    except Exception as e:  # noqa: BLE001 (any failure is the coordinator's error)
        write_status(wfile, e)
        return
    shard = (req.get("model", ""), req.get("from", 0), req.get("to", 0))
    try:
        write_status(wfile, None)
        while True:
            try:
                req = json.loads(read_frame(rfile, MAX_REQUEST))
            except (FrameError, ValueError):
                return
            if req.get("op") != "forward":
                return
            pos, tokens = int(req.get("pos", 0)), int(req.get("tokens", 0))
            if tokens <= 0 or pos < 0 or pos + tokens > stage.positions:
                write_status(wfile, f"positions {pos}..{pos + tokens} outside the context of {stage.positions}")
                return
            try:
                raw = read_frame(rfile, 4 * tokens * stage.dim)  # payloadBytes, deepseek.go:100
            except FrameError:
                return
            if fail_next is not None and fail_next(shard):
                return  # a simulated crash: the stream just ends
            if len(raw) != 4 * tokens * stage.dim:
                write_status(wfile, "activations of the wrong size")
                return
            try:
                out = stage.forward(decode_acts(raw, stage.dim), pos)
            except Exception as e:  # noqa: BLE001
                write_status(wfile, e)
                return
            write_status(wfile, None)
            write_frame(wfile, encode_acts(out))
    finally:
        stage.close()


class StageServer:
    """A threaded TCP server running handle() per connection, on
    127.0.0.1 (port 0: any free port; .address after start())."""

    def __init__(self, open_stage, port=0, fail_next=None):
        outer = self

        class _H(socketserver.StreamRequestHandler):
            def handle(self):
                handle(self.rfile, self.wfile, open_stage, outer.fail_next)

        class _S(socketserver.ThreadingTCPServer):
            allow_reuse_address = True
            daemon_threads = True

        self.fail_next = fail_next
        self.srv = _S(("127.0.0.1", port), _H)
        self.address = self.srv.server_address
        self.thread = None

    def start(self):
        self.thread = threading.Thread(target=self.srv.serve_forever, daemon=True)
        self.thread.start()
        return self

    def serve_forever(self):
        self.srv.serve_forever()

    def stop(self):
        self.srv.shutdown()
        self.srv.server_close()


class RemoteStage:
    """The coordinator's connection to a stage on a server (the open and
    forward exchanges of runStage, generate.go:616-719): forward(xs, pos)
    sends the activations and returns the stage's output; any failure of the
    connection raises, which coordinator.run_stage takes as the node's."""

    def __init__(self, address, model, from_, to, ctx, dim, timeout=120.0):
        self.dim = dim
        self.sock = socket.create_connection(address, timeout=timeout)
        self.r = self.sock.makefile("rb")
        self.w = self.sock.makefile("wb")
        req = {"op": "open", "model": model, "from": from_, "to": to, "ctx": ctx}
        write_frame(self.w, json.dumps(req).encode())
        read_status(self.r)

    def forward(self, xs, pos):
        xs = np.ascontiguousarray(xs, dtype=np.float32).reshape(-1, self.dim)
        write_frame(self.w, json.dumps({"op": "forward", "pos": int(pos), "tokens": int(xs.shape[0])}).encode())
        write_frame(self.w, encode_acts(xs))
        read_status(self.r)
        return decode_acts(read_frame(self.r, 4 * xs.shape[0] * self.dim), self.dim)

    def close(self):
        for f in (self.r, self.w, self.sock):
            try:
                f.close()
            except OSError:
                pass


def cuda_stage_opener(dev, cfg, layers):
    """open_stage for a node holding a model's layers on a GPU (rk.Layer
    objects, e.g. from rk.layer_load_part): a request for layers
    [from, to) with context ctx opens an rk.Stage of those layers, its
    positions capped at the model's context as Service.handle caps them
    (service.go:755-758); ForwardMany runs on the stage (rk_stage_forward)."""
    import rkcuda as rk

    def open_stage(req):
        a, b = int(req.get("from", 0)), int(req.get("to", 0))
        if not (0 <= a < b <= len(layers)):
            raise ValueError(f"layers {a}..{b} not held here")
        positions = int(req.get("ctx") or 0)
        if positions <= 0 or positions > cfg.seq_len:
            positions = cfg.seq_len
        st = rk.Stage(dev, cfg, layers[a:b], positions)

        def forward(xs, pos):
            return st.forward(np.ascontiguousarray(xs, np.float32).ravel(), pos).reshape(-1, cfg.dim)

        return StageHandle(forward, st.free, cfg.dim, positions)

    return open_stage
