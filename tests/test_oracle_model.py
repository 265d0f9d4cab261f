"""The oracle's llama-family forward pass (CPU only).

TestForwardMatchesNaiveReference (internal/llm/model_test.go:191-212): the
stage agrees with an independent float64 forward to 1e-3 and on the argmax.
TestStagesComposeExactly (model_test.go:224-243): layers split into stages
give the bits of one stage.
"""
import ctypes as C

import numpy as np
import pytest

import rk_oracle as ro
import rkcuda as rk
import synth


def small_config(dtype="f32", **over):
    base = dict(dim=64, hidden=160, layers=4, heads=4, kv_heads=2, vocab=50, seq_len=64, shared_classifier=1,
                head_dim=0, rope_theta=0.0, norm_eps=0.0, qkv_bias=0, qk_norm=0)
    base.update(over)
    return synth.config("", dtype, **base)


VARIANTS = {
    "llama": {},
    "qwen2": dict(qkv_bias=1, rope_theta=1e6, norm_eps=1e-6),
    "qwen3": dict(qk_norm=1, head_dim=32, rope_theta=1e6, norm_eps=1e-6),
    "mha": dict(kv_heads=4),
}


def naive_forward(c, weights, toks):
    """float64 forward of the whole model over toks (positions 0..), from
    the float32 weights; returns the logits of every position."""
    hs = synth.head_size(c)
    qd, kvd = c.heads * hs, c.kv_heads * hs
    eps = float(np.float32(c.norm_eps if c.norm_eps > 0 else 1e-5))
    theta = c.rope_theta if c.rope_theta > 0 else 10000.0
    W = {k: v.astype(np.float64) for k, v in weights.items() if not isinstance(k, tuple)}
    L = {k: v.astype(np.float64) for k, v in weights.items() if isinstance(k, tuple)}
    keys = [np.zeros((len(toks), kvd)) for _ in range(c.layers)]
    vals = [np.zeros((len(toks), kvd)) for _ in range(c.layers)]

    def rms(x, w):
        return w * x / np.sqrt((x * x).mean() + eps)

    def rope(v, pos, n):
        v = v.copy()
        for i in range(0, n, 2):
            p = (i % hs) // 2
            a = pos * theta ** (-2 * p / hs)
            c0, s0 = np.cos(a), np.sin(a)
            v[i], v[i + 1] = v[i] * c0 - v[i + 1] * s0, v[i] * s0 + v[i + 1] * c0
        return v

    out = []
    for pos, t in enumerate(toks):
        x = W["embed"][t].copy()
        for l in range(c.layers):
            xb = rms(x, 1.0)
            q, k, v = (L[(l, m)].reshape(-1, c.dim) @ xb for m in ("wq", "wk", "wv"))
            if c.qk_norm:
                q = np.concatenate([rms(q[h:h + hs], 1.0) for h in range(0, qd, hs)])
                k = np.concatenate([rms(k[h:h + hs], 1.0) for h in range(0, kvd, hs)])
            q, k = rope(q, pos, qd), rope(k, pos, kvd)
            keys[l][pos], vals[l][pos] = k, v
            att = np.zeros(qd)
            mul = c.heads // c.kv_heads
            for h in range(c.heads):
                off = (h // mul) * hs
                s = keys[l][:pos + 1, off:off + hs] @ q[h * hs:(h + 1) * hs] / np.sqrt(hs)
                s = np.exp(s - s.max())
                s /= s.sum()
                att[h * hs:(h + 1) * hs] = s @ vals[l][:pos + 1, off:off + hs]
            x = x + L[(l, "wo")].reshape(c.dim, qd) @ att
            xb = rms(x, 1.0)
            g = L[(l, "w1")].reshape(c.hidden, c.dim) @ xb
            u = L[(l, "w3")].reshape(c.hidden, c.dim) @ xb
            x = x + L[(l, "w2")].reshape(c.dim, c.hidden) @ (g / (1 + np.exp(-g)) * u)
        out.append(W["embed"].reshape(c.vocab, c.dim) @ rms(x, 1.0))
    return np.array(out)


@pytest.mark.parametrize("variant", sorted(VARIANTS))
def test_forward_matches_naive_reference(variant):
    c = small_config("f32", **VARIANTS[variant])
    m = ro.OracleModel(c, seed=7)
    weights = {"embed": m.keep[-1][0].reshape(c.vocab, c.dim)}
    for l in range(c.layers):
        for k in synth.MATS:
            rows, cols = synth.mat_shape(c, k)
            weights[(l, k)] = ro.gen_normal(7, synth.tid(l, k), rows * cols, synth.WEIGHT_SCALE)
    toks = [3, 17, 42, 8, 0, 49, 21, 5]
    want = naive_forward(c, weights, toks)
    for pos, t in enumerate(toks):
        _, lg = m.step(t, pos)
        assert np.abs(lg - want[pos]).max() < 1e-3, (variant, pos)
        assert int(np.argmax(lg)) == int(np.argmax(want[pos]))


@pytest.mark.parametrize("dtype", ["f32", "bf16", "q8_0", "q4_0", "q4_m"])
def test_stages_compose_exactly(dtype):
    c = small_config(dtype)
    whole = ro.OracleModel(c, seed=3)
    # Two stages over layers [0, 2) and [2, 4), the same weights.
    cut = 2
    halves = []
    for lo, hi in ((0, cut), (cut, c.layers)):
        sub = ro.lib().rko_stage_new(C.byref(whole.c), C.byref(whole.layers, lo * C.sizeof(ro.Layer)), hi - lo,
                                     whole.ctx, 2)
        halves.append(sub)
    try:
        for pos, t in enumerate([1, 2, 3, 4, 5, 6]):
            x = whole.embed_token(t)
            a = whole.forward(x, pos)
            b = x.copy()
            for sub in halves:
                assert ro.lib().rko_stage_forward(sub, ro._p(b), pos) == 0
            assert (a.view(np.uint32) == b.view(np.uint32)).all()
    finally:
        for sub in halves:
            ro.lib().rko_stage_free(sub)


def test_config_validation_matches_reference():
    """Config.validate (model.go:115-131)."""
    good = small_config("q8_0")
    assert ro.lib().rko_config_validate(C.byref(ro.to_config(good))) == 0
    for bad in (dict(dim=0), dict(heads=3), dict(kv_heads=3), dict(dim=70, heads=5),
                dict(hidden=150), dict(norm_eps=2.0)):
        c = small_config("q8_0", **bad)
        assert ro.lib().rko_config_validate(C.byref(ro.to_config(c))) != 0, bad


def test_oracle_generator_is_deterministic_and_normal():
    a = ro.gen_normal(1, 2, 1 << 16, 1.0)
    b = ro.gen_normal(1, 2, 1 << 16, 1.0)
    assert (a.view(np.uint32) == b.view(np.uint32)).all()
    assert abs(a.mean()) < 0.02 and abs(a.std() - 1) < 0.02
    # Any offset reproduces the same elements.
    c = ro.gen_normal(1, 2, 1000, 1.0, offset=777)
    assert (c.view(np.uint32) == a[777:1777].view(np.uint32)).all()
