"""The stage protocol (internal/llm/service.go: frames 671-715, handle
722-823) between the coordinator and stage servers, host logic only: the
servers run fake stages whose output depends on every input they have
cached, so a failover whose replay missed or reordered an input changes the
tokens. A server that drops its connection mid-generation (the reference's
simulated crash, failNext) makes the coordinator move the stage to the
other server and replay its inputs; the tokens equal those of a run with no
failure."""
import json
import socket

import numpy as np
import pytest

import coordinator as co
import stage_server as ss
from test_coordinator_cpu import DIM, FakeStage, model

CTX = 32


def fake_open(calls):
    def open_stage(req):
        st = FakeStage(req["from"] // 3, calls)
        return ss.StageHandle(lambda xs, pos: st.forward(xs, pos), st.close, DIM, req.get("ctx") or CTX)
    return open_stage


def run_remote(fail_on=None):
    """Three stages over two servers; fail_on: (shard from, forward count)
    at which server A drops the stage's connection."""
    calls = [0]
    seen = {}

    def fail_next(shard):
        seen[shard] = seen.get(shard, 0) + 1
        return fail_on is not None and shard[1] == fail_on[0] and seen[shard] == fail_on[1]

    a = ss.StageServer(fake_open(calls), fail_next=fail_next).start()
    b = ss.StageServer(fake_open(calls)).start()
    servers = {0: a.address, 1: b.address}
    try:
        stages = [co.PlannedStage(3 * i, 3 * i + 3, 0, ss.RemoteStage(a.address, "m", 3 * i, 3 * i + 3, CTX, DIM))
                  for i in range(3)]

        def place(st, exclude):
            node = next((n for n in servers if n not in exclude), None)
            if node is None:
                return False
            st.node, st.conn = node, ss.RemoteStage(servers[node], "m", st.from_, st.to, CTX, DIM)
            return True

        embed, logits = model()
        out = co.generate(stages, embed, logits, [1, 7, 2, 9], 12, place, seq_len=CTX)
        for st in stages:
            st.conn.close()
        return out
    finally:
        a.stop()
        b.stop()


def test_remote_stages_match_local_and_fail_over():
    want, stats = run_remote()
    assert stats["failovers"] == 0 and len(want) == 12
    from test_coordinator_cpu import run
    local, _ = run()
    assert want == local
    # Server A drops the middle stage on its 5th forward (a decode pass).
    got, stats = run_remote(fail_on=(3, 5))
    assert got == want and stats["failovers"] == 1
    # ... and on its first (the prefill): no replay needed.
    got, stats = run_remote(fail_on=(6, 1))
    assert got == want and stats["failovers"] == 1


def test_protocol_checks():
    calls = [0]
    srv = ss.StageServer(fake_open(calls)).start()
    try:
        # A forward past the generation's positions: error status, then the stream ends.
        rs = ss.RemoteStage(srv.address, "m", 0, 3, 4, DIM)
        with pytest.raises(RuntimeError, match="outside the context"):
            rs.forward(np.zeros((5, DIM), np.float32), 0)
        rs.close()
        # Activations of the wrong size for the announced tokens.
        rs = ss.RemoteStage(srv.address, "m", 0, 3, CTX, DIM)
        ss.write_frame(rs.w, json.dumps({"op": "forward", "pos": 0, "tokens": 2}).encode())
        ss.write_frame(rs.w, np.zeros(DIM, np.float32).tobytes())
        with pytest.raises(RuntimeError, match="wrong size"):
            ss.read_status(rs.r)
        rs.close()
        # A first request that is not "open": the connection is dropped.
        s = socket.create_connection(srv.address)
        f = s.makefile("rwb")
        ss.write_frame(f, json.dumps({"op": "forward"}).encode())
        with pytest.raises(ss.FrameError):
            ss.read_frame(f, ss.MAX_REQUEST)
        s.close()
        # A frame over the request limit is refused by the reader.
        s = socket.create_connection(srv.address)
        f = s.makefile("rwb")
        f.write((ss.MAX_REQUEST + 1).to_bytes(4, "big"))
        f.flush()
        with pytest.raises(ss.FrameError):
            ss.read_frame(f, ss.MAX_REQUEST)
        s.close()
    finally:
        srv.stop()


def test_open_failure_is_a_status():
    def bad_open(req):
        raise ValueError("no such shard")
    srv = ss.StageServer(bad_open).start()
    try:
        with pytest.raises(RuntimeError, match="no such shard"):
            ss.RemoteStage(srv.address, "m", 0, 3, CTX, DIM)
    finally:
        srv.stop()
