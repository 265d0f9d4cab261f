"""Batched products of one Q8_0 or Q4_0 matrix with many input vectors (the
tensor core kernel behind ForwardMany) and whole batched prefills, against
the CPU oracle bit for bit.

The reference's ForwardMany (internal/llm/model.go:504-518) runs Forward
token by token, so every token's product is one MatVecQ8 (quant.go:167-181)
and every layer's arithmetic is Forward's. The batched kernel computes each
32-block's exact integer sum on the tensor cores and adds the blocks in
qrow's order on the CUDA cores; these cases cover row counts that are not a
multiple of 128, token counts that are not a multiple of a CTA's 16 or 32
tokens, both CTA widths, and the reference's awkward inputs (denormals,
-0, 1e-30; internal/gpu/gpu_test.go:35-48). The prefills cover two 64-token
submissions, a start position above 0, GQA, MHA, Qwen2's bias and Qwen3's
QK-norm with head width 128, in Q8_0, Q4_0 (expanded to int8 in shared
memory for the MMAs) and the mixed Q4_M model format (a launch per format).
"""
import numpy as np
import pytest

import rk_oracle as ro
import rkcuda as rk
import synth
from conftest import awkward, same_bits
from test_gpu_stage import oracle_weights, upload_layers

pytestmark = pytest.mark.gpu

# (rows, cols, tokens): 16-token CTAs unless rows/128 · tokens/32 fills the
# SMs, which (4864, 896, 160) does (38 · 5 CTAs of 32 tokens).
SHAPES = [(300, 896, 37), (128, 896, 16), (1000, 4864, 5), (4864, 896, 160), (7, 128, 70), (64, 256, 1),
          (384, 1024, 33)]


@pytest.mark.parametrize("fmt", [rk.FMT_Q8_0, rk.FMT_Q4_0], ids=["q8_0", "q4_0"])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_mulvec_many_matches_cpu(dev, shape, fmt):
    rows, cols, n = shape
    rng = np.random.default_rng(rows * 7 + cols + n)
    w = awkward(rng, rows * cols, 0.02)
    w[: cols * (rows // 3)][::97] = 0.0  # blocks with a zero weight
    if rows > 2:
        w[cols: 2 * cols] = 0.0  # a row of all-zero blocks (scale 0)
    xs = np.stack([awkward(rng, cols, 1.0) for _ in range(n)])
    if n > 2:
        xs[1] = 0.0  # an input whose every block quantizes to zero
        xs[2, :32] = 0.0
    q, s = ro.quantize(fmt, w)
    m = rk.Matrix(dev, rows, cols, fmt, q, s)
    try:
        got = m.mulvec_many(xs)
        for t in range(n):
            same_bits(got[t], ro.matvec(fmt, q, s, xs[t], rows, cols))
    finally:
        m.free()
    assert dev.used() == 0


def test_mulvec_many_other_formats(dev):
    """Matrices the batched kernel does not take (widths that are not
    multiples of 128, float formats) give the same bits through one product
    per vector."""
    rng = np.random.default_rng(3)
    for fmt, rows, cols in [(rk.FMT_Q4_0, 200, 160), (rk.FMT_Q8_0, 96, 96), (rk.FMT_F32, 40, 64)]:
        w = awkward(rng, rows * cols, 0.02)
        q, s = (w, None) if fmt == rk.FMT_F32 else ro.quantize(fmt, w)
        xs = np.stack([awkward(rng, cols, 1.0) for _ in range(5)])
        m = rk.Matrix(dev, rows, cols, fmt, q, s)
        try:
            got = m.mulvec_many(xs)
            for t in range(5):
                same_bits(got[t], ro.matvec(fmt, q, s, xs[t], rows, cols))
        finally:
            m.free()
    assert dev.used() == 0


VARIANTS = {
    "llama": {},
    "mha": dict(kv_heads=4),
    "qwen2": dict(qkv_bias=1, rope_theta=1e6, norm_eps=1e-6),
    "qwen3_hs128": dict(head_dim=128, qk_norm=1, rope_theta=1e6, norm_eps=1e-6),
    # Head width 32: batched products, attention token by token.
    "hs32": dict(heads=8, kv_heads=2, head_dim=32),
}


def prefill_config(dtype="q8_0", **over):
    base = dict(dim=256, hidden=384, layers=3, heads=4, kv_heads=2, vocab=50, seq_len=160, shared_classifier=1,
                head_dim=0, rope_theta=0.0, norm_eps=0.0, qkv_bias=0, qk_norm=0)
    base.update(over)
    return synth.config("", dtype, **base)


@pytest.mark.parametrize("dtype", ["q8_0", "q4_0", "q4_m"])
@pytest.mark.parametrize("variant", sorted(VARIANTS))
def test_batched_prefill_matches_cpu(dev, variant, dtype):
    c = prefill_config(dtype, **VARIANTS[variant])
    vs = 303
    om = ro.OracleModel(c, seed=17, vec_seed=vs)
    layers = upload_layers(dev, c, oracle_weights(om, c), vs)
    st = rk.Stage(dev, c, layers, c.seq_len)
    try:
        assert st.batched() == 1
        xs = np.random.default_rng(9).standard_normal((90, c.dim)).astype(np.float32)
        # 10 tokens, then 75 from position 10 (a 64-token submission and an
        # 11-token one), then single decode steps; the oracle goes token by
        # token.
        got = np.concatenate([st.forward(xs[:10].ravel(), 0).reshape(10, c.dim),
                              st.forward(xs[10:85].ravel(), 10).reshape(75, c.dim)])
        for t in range(85):
            same_bits(got[t], om.forward(xs[t], t))
        for t in range(85, 90):
            same_bits(st.forward(xs[t], t), om.forward(xs[t], t))
    finally:
        st.free()
        for l in layers:
            l.free()
        om.free()
    assert dev.used() == 0


def test_long_batched_prefill_matches_cpu(dev):
    """330 tokens in one call (six submissions, the last 10 tokens long):
    later submissions' attention spans hundreds of cached positions, in the
    batched attention's clusters, with 7 query heads per kv head."""
    c = prefill_config(heads=14, kv_heads=2, head_dim=64, dim=256, layers=2, seq_len=400)
    om = ro.OracleModel(c, seed=23)
    layers = upload_layers(dev, c, oracle_weights(om, c))
    st = rk.Stage(dev, c, layers, c.seq_len)
    try:
        assert st.batched() == 1
        xs = np.random.default_rng(29).standard_normal((332, c.dim)).astype(np.float32)
        got = st.forward(xs[:330].ravel(), 0).reshape(330, c.dim)
        for t in range(330):
            same_bits(got[t], om.forward(xs[t], t))
        for t in range(330, 332):
            same_bits(st.forward(xs[t], t), om.forward(xs[t], t))
    finally:
        st.free()
        for l in layers:
            l.free()
        om.free()
    assert dev.used() == 0


def test_unbatched_stages_report_it(dev):
    """A width that is not a multiple of 128 keeps the token-by-token path."""
    c = synth.config("", "q8_0", dim=96, hidden=224, layers=1, heads=4, kv_heads=2, vocab=50, seq_len=32,
                     shared_classifier=1, head_dim=0, rope_theta=0.0, norm_eps=0.0, qkv_bias=0, qk_norm=0)
    om = ro.OracleModel(c, seed=5)
    layers = upload_layers(dev, c, oracle_weights(om, c))
    st = rk.Stage(dev, c, layers, c.seq_len)
    try:
        assert st.batched() == 0
    finally:
        st.free()
        for l in layers:
            l.free()
        om.free()


@pytest.mark.parametrize("heads,kv_heads,fills,seq_len,dtype", [(8, 2, [0, 7, 64, 130, 33], 200, "q8_0"),
                                                                 (4, 4, [1500, 3, 777], 1600, "q8_0"),
                                                                 (14, 2, [250, 1, 99, 5], 300, "q8_0"),
                                                                 (8, 2, [0, 7, 64, 130, 33], 200, "q4_0"),
                                                                 (4, 4, [900, 3, 77], 1000, "q4_m")],
                         ids=["gqa4", "mha_long", "gqa7", "gqa4_q4_0", "mha_q4_m"])
def test_batched_decode_matches_cpu(dev, heads, kv_heads, fills, seq_len, dtype):
    """Several independent sequences decoded together (rk_stage_forward_batch):
    each sequence's cache is filled to its own length (up to 1500 positions),
    then three steps run for all of them at once, each at its own position,
    with 4, 1 and 7 query heads per kv head. Every sequence's activations
    equal its own oracle Stage's Forward, bit for bit."""
    c = prefill_config(dtype, heads=heads, kv_heads=kv_heads, head_dim=64, dim=256, layers=2, seq_len=seq_len,
                       qkv_bias=1)
    nseq, seed = len(fills), 41
    # One oracle Stage per sequence (the same seeded weights in each).
    oms = [ro.OracleModel(c, seed=31, vec_seed=5) for _ in range(nseq)]
    layers = upload_layers(dev, c, oracle_weights(oms[0], c), 5)
    st = rk.Stage(dev, c, layers, c.seq_len, nseq=nseq)
    try:
        st.fill_cache(max(fills), seed)
        for o, f in zip(oms, fills):
            o.fill_cache(f, seed)
        rng = np.random.default_rng(43)
        for step in range(3):
            xs = rng.standard_normal((nseq, c.dim)).astype(np.float32)
            pos = [f + step for f in fills]
            got = st.forward_batch(xs, pos)
            for q in range(nseq):
                same_bits(got[q], oms[q].forward(xs[q], pos[q]))
        # Fewer sequences than the stage holds: the first two only.
        xs = rng.standard_normal((2, c.dim)).astype(np.float32)
        got = st.forward_batch(xs, [f + 3 for f in fills[:2]])
        for q in range(2):
            same_bits(got[q], oms[q].forward(xs[q], fills[q] + 3))
    finally:
        st.free()
        for l in layers:
            l.free()
        for o in oms:
            o.free()
    assert dev.used() == 0
