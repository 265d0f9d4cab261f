"""The coordinator's pipeline loop and stage failover (rakkan-mesh
internal/llm/generate.go:511-586 and runStage 616-719), host logic only:
stages here are fakes whose output depends on every input they have cached,
so a failover whose replay missed or reordered an input would change the
tokens. Runs without a GPU."""
import numpy as np
import pytest

import coordinator as co

DIM, VOCAB = 16, 40


class FakeStage:
    """out_p = x_p·(k+1) + ½·Σ_{q<=p} x_q over the cache of every position
    received; fails on the calls listed in fail_calls (a shared counter)."""

    def __init__(self, k, calls, fail_calls=()):
        self.k, self.cache, self.calls, self.fail_calls = k, [], calls, set(fail_calls)
        self.closed = False

    def forward(self, xs, pos):
        self.calls[0] += 1
        if self.calls[0] in self.fail_calls:
            raise RuntimeError(f"node lost at call {self.calls[0]}")
        del self.cache[pos:]
        if pos != len(self.cache):
            raise RuntimeError("cache gap")
        out = []
        for r in np.asarray(xs, np.float32).reshape(-1, DIM):
            self.cache.append(r.copy())
            acc = np.sum(np.stack(self.cache), axis=0, dtype=np.float32)
            out.append(np.float32(self.k + 1) * r + np.float32(0.5) * acc)
        return np.stack(out)

    def close(self):
        self.closed = True


def model(seed=3):
    rng = np.random.default_rng(seed)
    table = rng.standard_normal((VOCAB, DIM)).astype(np.float32) * 0.3
    wout = rng.standard_normal((VOCAB, DIM)).astype(np.float32)
    return (lambda toks: table[np.asarray(toks)]), (lambda x: wout @ x)


def pipeline(fails=None, spare_fails=()):
    """Three stages on nodes 0..2; placement opens a fresh stage on the
    lowest free node from 10 on. fails: {stage index: call numbers}."""
    calls = [0]
    fails = fails or {}
    stages = [co.PlannedStage(3 * i, 3 * i + 3, i, FakeStage(i, calls, fails.get(i, ()))) for i in range(3)]
    opened = []

    def place(st, exclude):
        node = 10
        while node in exclude or node in opened:
            node += 1
        opened.append(node)
        st.node, st.conn = node, FakeStage(st.from_ // 3, calls, spare_fails)
        return True

    return stages, place, calls


def run(fails=None, spare_fails=(), n=12):
    stages, place, calls = pipeline(fails, spare_fails)
    embed, logits = model()
    return co.generate(stages, embed, logits, [1, 7, 2, 9], n, place)


def test_failover_replays_the_stage_inputs():
    want, stats = run()
    assert stats == {"passes": 12, "tokens": 12, "failovers": 0}
    # Stage 1 fails on the 20th call overall (a decode pass); its
    # replacement gets the inputs so far replayed and the pass goes on.
    got, stats = run({1: {20}})
    assert got == want and stats["failovers"] == 1
    # A failure during the prefill needs no replay.
    got, stats = run({0: {1}})
    assert got == want and stats["failovers"] == 1
    # The replacement fails too, on its replay: the stage moves again.
    got, stats = run({2: {15}}, spare_fails={16})
    assert got == want and stats["failovers"] == 1


def test_a_stage_that_keeps_failing_is_an_error():
    stages, place, calls = pipeline()

    class Dead:
        def forward(self, xs, pos):
            raise RuntimeError("down")

        def close(self):
            pass

    def place_dead(st, exclude):
        st.node, st.conn = max(exclude) + 1, Dead()
        return True

    st = co.PlannedStage(0, 3, 0, Dead())
    with pytest.raises(co.StageError, match="layers 0..3"):
        co.run_stage(st, np.zeros((2, DIM), np.float32), 0, place_dead)


def test_rewind_and_position_checks():
    calls = [0]
    st = co.PlannedStage(0, 3, 0, FakeStage(0, calls))
    xs = np.random.default_rng(1).standard_normal((5, DIM)).astype(np.float32)
    first = co.run_stage(st, xs, 0, None)
    # A pass from an earlier position drops what the stage got from there on.
    again = co.run_stage(st, xs[3:], 3, None)
    assert np.array_equal(again, first[3:]) and len(st.inputs) == 5
    with pytest.raises(co.StageError, match="position 7 after 5"):
        co.run_stage(st, xs[:1], 7, None)


def test_first_max_is_the_samplers_rule():
    assert co.first_max([1.0, 3.0, 3.0, 2.0]) == 1
    assert co.first_max([np.nan, 5.0, 6.0]) == 0
    assert co.first_max([1.0, np.nan, 0.5]) == 0
    assert co.first_max([-np.inf, 2.0, np.nan, 2.0]) == 1


def test_generation_stops_at_the_context():
    """generate.go:442-450: a prompt that fills the context is refused, and
    max_tokens is clamped to the positions the stages hold, so the run ends
    cleanly instead of passing the context (which a stage refuses and the
    loop would take for a node failure)."""
    embed, logits = model()
    stages, place, calls = pipeline()
    with pytest.raises(ValueError, match="fills the context"):
        co.generate(stages, embed, logits, [1, 7, 2, 9], 5, place, seq_len=4)

    class Bounded(FakeStage):
        def forward(self, xs, pos):
            if pos + len(np.asarray(xs).reshape(-1, DIM)) > 10:
                raise RuntimeError("position past the context")
            return super().forward(xs, pos)

    calls = [0]
    stages = [co.PlannedStage(3 * i, 3 * i + 3, i, Bounded(i, calls)) for i in range(3)]
    got, stats = co.generate(stages, embed, logits, [1, 7, 2, 9], 100, place, seq_len=10)
    want, _ = run(n=6)
    assert len(got) == 6 and got == want and stats["failovers"] == 0
    # max_tokens <= 0 means every position left.
    calls = [0]
    stages = [co.PlannedStage(3 * i, 3 * i + 3, i, Bounded(i, calls)) for i in range(3)]
    got, _ = co.generate(stages, embed, logits, [1, 7, 2, 9], 0, place, seq_len=10)
    assert got == want
