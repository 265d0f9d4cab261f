"""The pipeline over stage servers in other processes, each serving CUDA
stages through the reference's stage protocol (internal/llm/service.go
handle 722-823): the coordinator (coordinator.generate) drives two servers
over local TCP streams; server A drops the second stage's connection on its
4th forward (a node lost mid-generation), the stage moves to server B and
its cache is rebuilt by replaying the inputs the coordinator kept. Tokens
and the last logits equal the CPU oracle's token-by-token decode bit for
bit."""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

import coordinator as co
import rk_oracle as ro
import rkcuda as rk
import stage_server as ss
import synth
from conftest import same_bits

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
CFG = dict(dim=256, hidden=384, layers=4, heads=4, kv_heads=2, vocab=64, seq_len=64, shared_classifier=1,
           head_dim=0, rope_theta=0.0, norm_eps=0.0, qkv_bias=0, qk_norm=0)
SEED = 17


def start_server(fail_after=0, fail_from=-1):
    p = subprocess.Popen([sys.executable, os.path.join(HERE, "stage_server_child.py"), "--config",
                          json.dumps(dict(CFG, dtype="q8_0")), "--seed", str(SEED), "--fail-after", str(fail_after),
                          "--fail-from", str(fail_from)],
                         stdout=subprocess.PIPE, text=True)
    line = p.stdout.readline()
    if not line:
        p.kill()
        raise RuntimeError("stage server did not start")
    return p, ("127.0.0.1", int(line))


def test_pipeline_over_stage_servers_with_failover(dev):
    c = synth.config("", "q8_0", **CFG)
    dm = synth.DeviceModel(dev, c, SEED, keep_host=True)
    om = ro.OracleModel(c, SEED, weights=dm.host_weights)
    pa, a = start_server(fail_after=4, fail_from=2)
    pb, b = start_server()
    servers = {0: a, 1: b}
    opened = []
    try:
        def connect(node, from_, to):
            rs = ss.RemoteStage(servers[node], "synthetic", from_, to, c.seq_len, c.dim)
            opened.append(rs)
            return rs

        stages = [co.PlannedStage(0, 2, 0, connect(0, 0, 2)), co.PlannedStage(2, 4, 0, connect(0, 2, 4))]

        def place(st, exclude):
            node = next((n for n in servers if n not in exclude), None)
            if node is None:
                return False
            st.node, st.conn = node, connect(node, st.from_, st.to)
            return True

        last = {}

        def logits_of(x):
            last["logits"] = dm.head.logits(x)
            return last["logits"]

        prompt, n = [3, 17, 5, 40, 9], 10
        embed = lambda toks: np.stack([rk.embed(dm.embed, int(t)) for t in toks])
        got, stats = co.generate(stages, embed, logits_of, prompt, n, place, seq_len=c.seq_len)
        want, want_logits = om.generate(prompt, n)
        assert got == [int(t) for t in want]
        assert stats["failovers"] == 1
        same_bits(last["logits"], want_logits[-1])
    finally:
        for rs in opened:
            rs.close()
        for p in (pa, pb):
            p.kill()
            p.wait()
        om.free()
        dm.free()
