"""Whole stages on the GPU against the CPU oracle, bit for bit.

Restates internal/llm/gpu_test.go:32-111 (TestGPUStagesMatchCPU): three
architecture variants (Qwen2's QKV bias; Qwen3's QK-norm with head width 32,
theta 1e6, eps 1e-6; no GQA) and the llama baseline, in f32, bf16, q8_0,
q4_0 and q4_m; a prefill of 70 tokens (more than one 64-token submission)
then 6 decode steps, activations compared at every position. Both the
reference-shaped Batch API (gpustage.go's recording) and rk_stage (the CUDA
graph path) are checked.
"""
import math

import numpy as np
import pytest

import rk_oracle as ro
import rkcuda as rk
import synth
from conftest import same_bits

pytestmark = pytest.mark.gpu

VARIANTS = {
    "llama": {},
    "qwen2": dict(qkv_bias=1, rope_theta=1e6, norm_eps=1e-6),
    "qwen3": dict(qk_norm=1, head_dim=32, rope_theta=1e6, norm_eps=1e-6),
    "mha": dict(kv_heads=4),
    # Widths that are not powers of two: Recip32(float32(n)) of the norms
    # then depends on every bit of the Newton iteration's constants.
    "odd": dict(dim=96, hidden=224, head_dim=24, qk_norm=1),
    # Head widths of the tiled scores kernel (64, 128), which also does the
    # bias / QK-norm / RoPE / cache-append work; seeded vectors.
    "qwen2_hs64": dict(dim=256, heads=4, kv_heads=2, qkv_bias=1, rope_theta=1e6, norm_eps=1e-6),
    "qwen3_hs128": dict(dim=256, heads=4, kv_heads=2, head_dim=128, qk_norm=1, rope_theta=1e6, norm_eps=1e-6),
}
VEC_SEED = {"qwen2_hs64": 101, "qwen3_hs128": 202}
DTYPES = ["f32", "bf16", "q8_0", "q4_0", "q4_m"]


def small_config(dtype, **over):
    base = dict(dim=64, hidden=160, layers=4, heads=4, kv_heads=2, vocab=50, seq_len=96, shared_classifier=1,
                head_dim=0, rope_theta=0.0, norm_eps=0.0, qkv_bias=0, qk_norm=0)
    base.update(over)
    return synth.config("", dtype, **base)


def oracle_weights(om, c):
    """The oracle model's arrays, keyed like OracleModel(weights=...)."""
    out = {}
    i = 0
    for l in range(c.layers):
        i += 1  # the layer's vector dict
        for k in synth.MATS:
            out[(l, k)] = om.keep[i]
            i += 1
    return out


def upload_layers(dev, c, weights, vec_seed=None):
    layers, keep = [], []
    for l in range(c.layers):
        hl, vec = synth.host_layer_vectors(c, None if vec_seed is None else vec_seed + l)
        for k in synth.MATS:
            w, s = weights[(l, k)]
            setattr(hl, k, rk.HostMatrix(synth.mat_fmt(c, k), w.ctypes.data, None if s is None else s.ctypes.data))
        keep.append((hl, vec))
        layers.append(rk.Layer(dev, c, host=(hl, vec)))
    return layers


def inputs(c, n, seed):
    rng = np.random.default_rng(seed)
    return rng.standard_normal((n, c.dim)).astype(np.float32)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("variant", sorted(VARIANTS))
def test_stage_matches_cpu(dev, variant, dtype):
    c = small_config(dtype, **VARIANTS[variant])
    vs = VEC_SEED.get(variant)
    om = ro.OracleModel(c, seed=11, vec_seed=vs)
    weights = oracle_weights(om, c)
    layers = upload_layers(dev, c, weights, vs)
    st = rk.Stage(dev, c, layers, c.seq_len)
    try:
        xs = inputs(c, 76, 5)
        # Prefill 70 tokens in one call (two 64-token submissions), then 6
        # decode steps; the oracle runs token by token (Stage.ForwardMany).
        got = st.forward(xs[:70].ravel(), 0).reshape(70, c.dim)
        for t in range(70):
            same_bits(got[t], om.forward(xs[t], t))
        for t in range(70, 76):
            same_bits(st.forward(xs[t], t), om.forward(xs[t], t))
    finally:
        st.free()
        for l in layers:
            l.free()
    assert dev.used() == 0


def record_token(b, c, g, layers, vecs, mats, pos):
    """gpustage.go:119-152 through the Batch API."""
    hs = synth.head_size(c)
    qd, kvd = c.heads * hs, c.kv_heads * hs
    eps = float(ro.lib().rko_eps(__import__("ctypes").byref(ro.to_config(c))))
    L = ro.lib()
    recip_dim, recip_head = L.rko_recip32(float(c.dim)), L.rko_recip32(float(hs))
    inv_sqrt = float(np.float32(1 / math.sqrt(hs)))
    half = hs // 2
    for li in range(c.layers):
        v, o = vecs[li], g["offs"]
        b.rmsnorm(v, g["x"], g["xb"], o["rms_att"], c.dim, 1, 0, recip_dim, eps)
        b.matvecs([mats[li]["wq"], mats[li]["wk"], mats[li]["wv"]], [g["q"], g["k"], g["v"]], g["xb"])
        if c.qkv_bias:
            b.addvec(v, g["q"], o["bq"], qd)
            b.addvec(v, g["k"], o["bk"], kvd)
            b.addvec(v, g["v"], o["bv"], kvd)
        if c.qk_norm:
            b.rmsnorm(v, g["q"], g["q"], o["q_norm"], hs, c.heads, hs, recip_head, eps)
            b.rmsnorm(v, g["k"], g["k"], o["k_norm"], hs, c.kv_heads, hs, recip_head, eps)
        b.rope(g["q"], g["k"], qd, kvd, hs, g["cos"] + pos * half, g["sin"] + pos * half)
        b.copy(g["k"], g["keys"][li] + pos * kvd, kvd)
        b.copy(g["v"], g["vals"][li] + pos * kvd, kvd)
        b.attention(g["q"], g["keys"][li], g["vals"][li], g["att"], g["ctx"], g["attOut"], pos + 1, c.heads,
                    c.kv_heads, hs, kvd, inv_sqrt)
        b.matvecs([mats[li]["wo"]], [g["xb2"]], g["attOut"])
        b.residual(g["x"], g["xb2"], c.dim, False)
        b.rmsnorm(v, g["x"], g["xb"], o["rms_ffn"], c.dim, 1, 0, recip_dim, eps)
        b.matvecs([mats[li]["w1"], mats[li]["w3"]], [g["hb"], g["hb2"]], g["xb"])
        b.silumul(g["hb"], g["hb2"], c.hidden)
        b.matvecs([mats[li]["w2"]], [g["xb"]], g["hb"])
        b.residual(g["x"], g["xb"], c.dim, True)


@pytest.mark.parametrize("dtype", ["f32", "bf16", "q8_0", "q4_m"])
@pytest.mark.parametrize("variant", ["qwen2", "qwen3", "mha"])
def test_batch_api_matches_cpu(dev, variant, dtype):
    """The Batch API driven exactly as gpustage.go drives gpu.Batch."""
    c = small_config(dtype, **VARIANTS[variant])
    om = ro.OracleModel(c, seed=13)
    weights = oracle_weights(om, c)
    hs = synth.head_size(c)
    qd, kvd, ctx = c.heads * hs, c.kv_heads * hs, c.seq_len
    at = [0]

    def alloc(n):
        o = at[0]
        at[0] += n
        return o

    g = {"x": alloc(c.dim), "xb": alloc(c.dim), "xb2": alloc(c.dim), "q": alloc(qd), "k": alloc(kvd),
         "v": alloc(kvd), "attOut": alloc(qd), "hb": alloc(c.hidden), "hb2": alloc(c.hidden),
         "att": alloc(c.heads * ctx), "ctx": ctx}
    widest = max(c.dim, qd, c.hidden)
    qx, xs_off = alloc(widest // 4), alloc(widest // 32)
    g["cos"], g["sin"] = alloc(ctx * (hs // 2)), alloc(ctx * (hs // 2))
    g["keys"], g["vals"] = [], []
    for _ in range(c.layers):
        g["keys"].append(alloc(ctx * kvd))
        g["vals"].append(alloc(ctx * kvd))
    arena = rk.Arena(dev, at[0], max(2 * 64 * c.dim, 2 * ctx * (hs // 2)))
    arena.set_quant_scratch(qx, xs_off)
    mats, vecs, order = [], [], []
    for l in range(c.layers):
        mats.append({k: rk.Matrix(dev, *synth.mat_shape(c, k), synth.mat_fmt(c, k), *weights[(l, k)])
                     for k in synth.MATS})
        vd = synth.layer_vectors(c)
        flat, offs = [], {}
        for name in ("rms_att", "rms_ffn", "bq", "bk", "bv", "q_norm", "k_norm"):
            if name in vd:
                offs[name] = len(flat)
                flat.extend(vd[name])
        g["offs"] = offs
        vecs.append(rk.Vectors(dev, np.array(flat, np.float32)))
    try:
        cos = np.empty(ctx * (hs // 2), np.float32)
        sin = np.empty_like(cos)
        ro.lib().rko_rope_table(__import__("ctypes").byref(ro.to_config(c)), ctx, ro._p(cos), ro._p(sin))
        b = arena.begin()
        b.write(g["cos"], cos)
        b.write(g["sin"], sin)
        b.submit()
        xs = inputs(c, 76, 6)
        outs = []
        # gpuStage.forward: batches of at most 64 tokens per submission.
        for start, n in ((0, 64), (64, 6)):
            b = arena.begin()
            reads = []
            for t in range(start, start + n):
                b.write(g["x"], xs[t])
                record_token(b, c, g, c.layers, vecs, mats, t)
                reads.append(b.read(g["x"], c.dim))
            b.submit()
            outs.extend(reads)
        for t in range(70, 76):
            b = arena.begin()
            b.write(g["x"], xs[t])
            record_token(b, c, g, c.layers, vecs, mats, t)
            outs.append(b.read(g["x"], c.dim))
            b.submit()
        for t in range(76):
            same_bits(outs[t], om.forward(xs[t], t))
    finally:
        for ms in mats:
            for m in ms.values():
                m.free()
        for v in vecs:
            v.free()
        arena.free()
    assert dev.used() == 0


def test_batch_errors_latch(dev):
    """A batch keeps its first error and returns it from Submit
    (batch.go:136-147, 333-343); out-of-range offsets are errors."""
    arena = rk.Arena(dev, 256, 64)
    try:
        b = arena.begin()
        b.write(250, np.zeros(16, np.float32))  # past the arena
        b.copy(0, 8, 8)
        with pytest.raises(rk.RkError):
            b.submit()
        b = arena.begin()
        b.write(0, np.zeros(100, np.float32))  # more than the staging holds
        with pytest.raises(rk.RkError):
            b.submit()
        m = rk.Matrix(dev, 4, 32, rk.FMT_Q8_0, np.zeros(128, np.int8), np.zeros(4, np.float32))
        b = arena.begin()
        b.matvecs([m], [64], 0)  # no quant scratch
        with pytest.raises(rk.RkError):
            b.submit()
        m.free()
    finally:
        arena.free()
    assert dev.used() == 0
