"""rk_plan_stages (the layer pipeline's stage plan) against the reference's
own planStages cases (internal/llm/plan_test.go:8-54, 118-145) and against
the oracle restatement (oracle/plan_stages.py) on seeded random inputs. Host
code only: runs without a GPU.
"""
import numpy as np
import pytest

import plan_stages as ops
import rkcuda as rk


def lib_plan(cost, mem, speed, capacity, stages, free=None):
    """The library's spans as (from, to, node index)."""
    return [(a, b, n) for n, a, b in rk.plan_stages(cost, mem, speed, capacity, stages, free)]


def layer_nodes(spec):
    """plan_test.go's stageNode{speed, layers}: node i holds `layers` layers
    whatever they are (mem 1 per layer, capacity = layers)."""
    return [s for s, _ in spec], [l for _, l in spec]


# plan_test.go:9-13: cpu, tiny, gpu-small, gpu-big, in that order.
CPU, TINY, SMALL, BIG = 0, 1, 2, 3
NODES = [(10.0, 40), (30.0, 0), (60.0, 6), (100.0, 20)]


def test_reference_cases_automatic():
    speed, cap = layer_nodes(NODES)
    # plan_test.go:15-23: the fastest take what they hold, the CPU the rest.
    assert lib_plan([1] * 32, [1] * 32, speed, cap, 0) == [(0, 20, BIG), (20, 26, SMALL), (26, 32, CPU)]
    # plan_test.go:24-27: a model the big GPU holds alone.
    assert lib_plan([1] * 16, [1] * 16, speed, cap, 0) == [(0, 16, BIG)]
    # plan_test.go:28-31: too big for all of them.
    with pytest.raises(rk.RkError):
        lib_plan([1] * 100, [1] * 100, speed, cap, 0)


def test_reference_cases_staged():
    speed, cap = layer_nodes(NODES)
    # plan_test.go:33-40: two stages, split by speed within what they hold.
    assert lib_plan([1] * 16, [1] * 16, speed, cap, 2) == [(0, 10, BIG), (10, 16, SMALL)]
    # plan_test.go:41-45: every stage gets a layer, however slow its node.
    got = lib_plan([1] * 4, [1] * 4, [100.0, 0.01], [20, 10], 2)
    assert len(got) == 2 and got[1][2] == 1 and got[1][1] - got[1][0] == 1
    # plan_test.go:46-50: equal nodes share evenly.
    got = lib_plan([1] * 9, [1] * 9, [5.0] * 3, [99] * 3, 3)
    assert len(got) == 3 and got[0][1] == 3 and got[1][1] == 6
    # plan_test.go:51-54: more stages than layers: as many as there can be.
    assert len(lib_plan([1] * 2, [1] * 2, [5.0] * 3, [99] * 3, 5)) == 2


def test_reference_unequal_layers():
    # plan_test.go:118-145 (testShape: layer bytes, cache 1 per layer):
    # memory-bound automatic plan, and two equal stages balanced by bytes.
    layer = [10, 50, 10, 10, 50, 10]
    mem = [b + 1 for b in layer]
    assert lib_plan(layer, mem, [10.0, 5.0], [75, 80], 0) == [(0, 3, 0), (3, 6, 1)]
    assert lib_plan(layer, mem, [1.0, 1.0], [1000, 1000], 2) == [(0, 3, 0), (3, 6, 1)]


def oracle_plan(cost, mem, speed, capacity, stages, free):
    pre = np.concatenate([[0], np.cumsum(mem)])
    nodes = [(i, speed[i], free[i], (lambda c: lambda a, b: pre[b] - pre[a] <= c)(capacity[i]))
             for i in range(len(speed))]
    return ops.plan_stages(list(cost), nodes, stages)


@pytest.mark.parametrize("seed", range(40))
def test_matches_oracle_on_random_inputs(seed):
    rng = np.random.default_rng(seed)
    layers = int(rng.integers(1, 40))
    nodes = int(rng.integers(1, 9))
    cost = rng.integers(1, 1000, layers)
    mem = cost + rng.integers(0, 50, layers)
    speed = rng.choice([1.0, 2.5, 5.0, 10.0, 40.0], nodes)
    capacity = rng.integers(0, int(mem.sum()) + 1, nodes)
    free = rng.integers(0, 3, nodes)
    stages = int(rng.integers(-1, 10))
    try:
        want = oracle_plan(cost, mem, speed, capacity, stages, free)
    except ValueError:
        want = None
    if want is None:
        with pytest.raises(rk.RkError):
            lib_plan(cost, mem, speed, capacity, stages, free)
    else:
        assert lib_plan(cost, mem, speed, capacity, stages, free) == want
