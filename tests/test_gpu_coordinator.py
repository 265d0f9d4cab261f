"""The coordinator's pipeline loop over CUDA stages, with a stage's node
failing mid-generation (internal/llm/generate.go:511-586, runStage 616-719):
the replacement stage's cache is rebuilt by replaying the inputs the
coordinator kept, and the greedy tokens and last logits equal the oracle's
token-by-token decode bit for bit."""
import numpy as np
import pytest

import coordinator as co
import rk_oracle as ro
import rkcuda as rk
import synth
from conftest import same_bits

pytestmark = pytest.mark.gpu


def test_failover_on_gpu_stages(dev):
    c = synth.config("", "q8_0", dim=256, hidden=384, layers=4, heads=4, kv_heads=2, vocab=64, seq_len=64,
                     shared_classifier=1, head_dim=0, rope_theta=0.0, norm_eps=0.0, qkv_bias=0, qk_norm=0)
    dm = synth.DeviceModel(dev, c, 13, keep_host=True)
    om = ro.OracleModel(c, 13, weights=dm.host_weights)
    calls, opened = [0], []

    class GpuStage:
        """Layers [a, b) of the model in an rk.Stage; the node 'fails' on
        the listed call numbers (counted over all stages)."""

        def __init__(self, a, b, fail_calls=()):
            self.st = rk.Stage(dev, c, dm.layers[a:b], c.seq_len)
            self.fail_calls = set(fail_calls)
            opened.append(self)

        def forward(self, xs, pos):
            calls[0] += 1
            if calls[0] in self.fail_calls:
                raise RuntimeError(f"node lost at call {calls[0]}")
            return self.st.forward(np.ascontiguousarray(xs).ravel(), pos).reshape(-1, c.dim)

        def close(self):
            if self.st:
                self.st.free()
                self.st = None

    def place(st, exclude):
        st.node = max(exclude) + 1
        st.conn = GpuStage(st.from_, st.to)
        return True

    last = {}

    def logits_of(x):
        last["logits"] = dm.head.logits(x)
        return last["logits"]

    try:
        # The second stage's node is lost during the 4th decode pass (call 10).
        stages = [co.PlannedStage(0, 2, 0, GpuStage(0, 2)), co.PlannedStage(2, 4, 1, GpuStage(2, 4, {10}))]
        prompt, n = [3, 17, 5, 40, 9], 10
        embed = lambda toks: np.stack([rk.embed(dm.embed, int(t)) for t in toks])
        got, stats = co.generate(stages, embed, logits_of, prompt, n, place)
        want, want_logits = om.generate(prompt, n)
        assert got == [int(t) for t in want]
        assert stats["failovers"] == 1 and stats["passes"] == n
        same_bits(last["logits"], want_logits[-1])
    finally:
        for s in opened:
            s.close()
        om.free()
        dm.free()
