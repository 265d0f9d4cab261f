"""Row-sharded decode on 2, 4 and 8 GPUs (rk_group / rk_*_group) against the
CPU oracle: the same logits, bit for bit, and the same greedy tokens as the
reference path. Each rank is a child process on its own GPU; the shards
exchange activations as tagged words stored over NVLink (or NCCL all-gathers
where that is not possible). World sizes above the box's GPU count are
skipped.
"""
import numpy as np
import pytest

import rk_oracle as ro
import rkcuda as rk
import synth
from conftest import same_bits

pytestmark = pytest.mark.gpu

SEED = 20261203
PROMPT = [3, 141, 59, 265, 35, 897]
N_NEW = 6
CTX = 64


def _small(dtype, variant):
    # 8 kv heads: whole kv heads per rank up to 8 ranks.
    over = dict(layers=2, dim=1024, hidden=2816, heads=16, kv_heads=8, vocab=8192, seq_len=CTX)
    if variant == "qwen3":
        over.update(head_dim=128, qk_norm=1, rope_theta=1e6, norm_eps=1e-6, heads=16, kv_heads=8)
    if variant == "wide_hidden":
        # Hidden wider than a product's own quantizing prologue takes (as
        # Qwen3-32B's 25600): W2 quantizes its input in a separate launch
        # while the next layer's Q/K/V still gathers x as tagged words, which
        # W2's epilogue must store.
        over.update(hidden=16896)
    return synth.config("llama3-8b", dtype, **over)


def _rank(rank, world, gid, dtype, variant, out):
    import os
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    try:
        c = _small(dtype, variant)
        dev = rk.Device(rank)
        grp = rk.Group(dev, world, rank, gid)
        dm = synth.DeviceModel(dev, c, SEED, ctx=CTX, group=grp)
        toks, logits = dm.model.generate(np.array(PROMPT, np.int32), N_NEW, want_logits=True)
        out.put((rank, toks, logits, dm.stage.fused_gathers()))
        dm.free()
        grp.free()
        dev.close()
    except Exception as e:
        out.put((rank, repr(e), None, None))


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("variant", ["llama", "qwen3", "wide_hidden"])
@pytest.mark.parametrize("dtype", ["q8_0", "q4_0"])
def test_row_sharded_decode_matches_oracle(dtype, variant, world):
    if rk.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    gid = rk.group_id()
    procs = [ctx.Process(target=_rank, args=(r, world, gid, dtype, variant, out)) for r in range(world)]
    for p in procs:
        p.start()
    res, fused = {}, {}
    for _ in procs:
        r, toks, logits, f = out.get(timeout=600)
        res[r] = (toks, logits)
        fused[r] = f
    for p in procs:
        p.join(timeout=120)
    for r in range(world):
        assert not isinstance(res[r][0], str), res[r][0]
    om = ro.OracleModel(_small(dtype, variant), SEED, ctx=CTX)
    want_toks, want_logits = om.generate(PROMPT, N_NEW)
    om.free()
    for r in range(world):
        toks, logits = res[r]
        assert list(toks) == list(want_toks)
        same_bits(logits, want_logits)
    # The GPUs of one box reach each other over NVLink: the gathers are fused
    # unless the run asks for NCCL.
    import os
    want = 0 if os.environ.get("RK_GATHER") == "nccl" else 1
    assert all(fused[r] == want for r in range(world)), fused
