"""Row sharding's host logic on the CPU (no GPU).

A product's output rows are computed from the whole input in the
reference's order, so splitting the rows over ranks and reassembling them
with an all-gather cannot change bits; the reference relies on the same
fact for its goroutine split (internal/num/matvec.go:384-400, tested by
TestMatVecSplitDoesNotChangeBits, num_test.go:61-81). These tests check the
shard plan the library and the synthetic model use (synth.shard_rows) and
run the split-and-gather with the oracle on two gloo ranks.
"""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import rk_oracle as ro
import synth


def _configs():
    for name in ("stories15M", "qwen2.5-0.5b", "llama3-8b", "qwen3-32b"):
        yield name, synth.config(name, "q8_0")


@pytest.mark.parametrize("name,c", list(_configs()), ids=lambda v: v if isinstance(v, str) else "")
def test_shard_plan_covers_rows_once(name, c):
    for G in (1, 2, 4, 8):
        try:
            parts = [synth.shard_rows(c, G, r) for r in range(G)]
        except ValueError:
            assert c.kv_heads % G or c.dim % G or c.hidden % G or c.vocab % G
            continue
        for k in synth.MATS + ("cls",):
            rows = c.vocab if k == "cls" else synth.mat_shape(c, k)[0]
            covered = np.zeros(rows, np.int32)
            for p in parts:
                r0, n = p[k]
                covered[r0:r0 + n] += 1
            assert (covered == 1).all(), (name, G, k)
        hs = synth.head_size(c)
        for r, p in enumerate(parts):
            # Whole kv heads, with their query heads, on each rank.
            assert p["wk"][0] % hs == 0 and p["wk"][1] % hs == 0
            assert p["wq"][0] // hs == (p["wk"][0] // hs) * (c.heads // c.kv_heads)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, rows, cols, fmt, errors):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import torch
        rng = np.random.default_rng(7)
        w32 = (rng.standard_normal(rows * cols) * 0.02).astype(np.float32)
        w, s = ro.quantize(fmt, w32)
        x = rng.standard_normal(cols).astype(np.float32)
        per = rows // world
        rb = (cols if fmt == ro.Q8_0 else cols // 2)
        mine = ro.matvec(fmt, w[rank * per * rb:(rank + 1) * per * rb], s[rank * per * cols // 32:(rank + 1) * per * cols // 32],
                         x, per, cols, threads=1)
        parts = [torch.empty(per, dtype=torch.float32) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(mine))
        got = torch.cat(parts).numpy()
        if rank == 0:
            want = ro.matvec(fmt, w, s, x, rows, cols, threads=1)
            if not (got.view(np.uint32) == want.view(np.uint32)).all():
                errors.put("sharded product differs from the whole one")
    except Exception as e:  # reported to the parent
        errors.put(repr(e))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_row_shards_gather_to_the_whole_product(fmt):
    f = {"q8_0": ro.Q8_0, "q4_0": ro.Q4_0}[fmt]
    ctx = mp.get_context("spawn")
    errors = ctx.Queue()
    mp.start_processes(_rank_main, args=(2, _free_port(), 512, 896, f, errors), nprocs=2, start_method="spawn")
    assert errors.empty(), errors.get()
