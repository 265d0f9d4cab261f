"""Decode steps deep into a filled KV cache, GPU against the CPU oracle, bit
for bit.

The stage's attention keeps the softmax sum and the value sums as serial
chains in position order (model.go:571-587, 640-654). At long contexts the
single softmax + value kernel splits the maximum and the exps over a
thread-block cluster (each CTA a chunk of the positions, exchanged through
distributed shared memory) and runs the chains from rotating registers, so
these cases reach many chunks, uneven last chunks and one or two chain warps
(heads per kv head x 8 chains). Both sides fill positions 0..P-1 of every
layer's cache with the same seeded values (rk_stage_fill_cache /
rko_stage_fill_cache), then decode positions P and P+1.
"""
import numpy as np
import pytest

import rk_oracle as ro
import synth
from conftest import same_bits

pytestmark = pytest.mark.gpu

# name: (config overrides, filled positions)
CASES = {
    # 4 query heads per kv head, head width 128: 32 chains, one warp.
    "gqa4_hs128": (dict(heads=8, kv_heads=2, head_dim=128), 4093),
    # One query head per kv head: 8 chains.
    "mha_hs64": (dict(heads=4, kv_heads=4, head_dim=64), 2050),
    # 7 query heads per kv head: 56 chains over two warps.
    "gqa7_hs64": (dict(heads=14, kv_heads=2, head_dim=64), 1531),
    # 8 per kv head: 64 chains over two chain warps.
    "gqa8_hs64": (dict(heads=16, kv_heads=2, head_dim=64), 1200),
}


@pytest.mark.parametrize("case", sorted(CASES))
def test_decode_after_long_cache(dev, case):
    over, filled = CASES[case]
    ctx = filled + 8
    c = synth.config("", "q8_0", dim=256, hidden=512, layers=2, vocab=64, seq_len=ctx, shared_classifier=1,
                     rope_theta=0.0, norm_eps=0.0, qkv_bias=0, qk_norm=0, **over)
    seed = 20261202
    dm = synth.DeviceModel(dev, c, seed, ctx=ctx, keep_host=True)
    try:
        om = ro.OracleModel(c, seed, ctx=ctx, weights=dm.host_weights)
        try:
            dm.stage.fill_cache(filled, seed)
            om.fill_cache(filled, seed)
            x = np.random.default_rng(seed).standard_normal(c.dim).astype(np.float32)
            for pos in (filled, filled + 1):
                y = dm.stage.forward(x, pos)
                yo = om.forward(x, pos)
                same_bits(y, yo)
                x = yo
        finally:
            om.free()
    finally:
        dm.free()
