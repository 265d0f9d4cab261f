"""A layer pipeline over two GPUs (rk_plan_stages + rk_pipeline_*) against
the CPU oracle running the whole model: the last rank's logits at every
step bit for bit, and the same greedy tokens on every rank. Each rank is a
child process on its own GPU holding the layers the plan gives it
(planStages, plan.go:122-207, equal speeds: bytes split evenly); the
activation passes by NCCL send/receive. Skipped on a box with one GPU.
"""
import numpy as np
import pytest

import rk_oracle as ro
import rkcuda as rk
import synth
from conftest import same_bits

pytestmark = pytest.mark.gpu

SEED = 20261204
PROMPT = [5, 77, 310, 42]
N_NEW = 6
CTX = 32


def _config(dtype):
    return synth.config("llama3-8b", dtype, layers=5, dim=512, hidden=1408, heads=8, kv_heads=4, vocab=4096,
                        seq_len=CTX)


def _spans(c, world):
    # Every layer reads the same bytes; the nodes are equal and hold it all.
    per = sum(synth.matrix_bytes(synth.mat_fmt(c, k), int(np.prod(synth.mat_shape(c, k)))) for k in synth.MATS)
    return rk.plan_stages([per] * c.layers, [per] * c.layers, [1.0] * world, [per * c.layers] * world, world)


def _rank(rank, world, gid, dtype, out):
    import os
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    try:
        c = _config(dtype)
        spans = _spans(c, world)
        node, first, end = spans[rank]
        assert node == rank
        dev = rk.Device(rank)
        grp = rk.Group(dev, world, rank, gid)
        pr = synth.PipelineRank(dev, c, SEED, grp, first, end, ctx=CTX)
        toks, logits = pr.generate(PROMPT, N_NEW)
        out.put((rank, toks, logits, (first, end)))
        pr.free()
        grp.free()
        dev.close()
    except Exception as e:
        out.put((rank, repr(e), None, None))


@pytest.mark.parametrize("dtype", ["q8_0", "q4_0"])
def test_pipeline_decode_matches_oracle(dtype):
    world = 2
    if rk.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    gid = rk.group_id()
    procs = [ctx.Process(target=_rank, args=(r, world, gid, dtype, out)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r, toks, logits, span = out.get(timeout=600)
        res[r] = (toks, logits, span)
    for p in procs:
        p.join(timeout=120)
    for r in range(world):
        assert not isinstance(res[r][0], str), res[r][0]
    # The plan gives each rank a contiguous part and covers every layer.
    assert res[0][2][0] == 0 and res[world - 1][2][1] == _config(dtype).layers
    om = ro.OracleModel(_config(dtype), SEED, ctx=CTX)
    want_toks, want_logits = om.generate(PROMPT, N_NEW)
    om.free()
    for r in range(world):
        assert list(res[r][0]) == list(want_toks)
    same_bits(res[world - 1][1], want_logits)
