"""Models built from the reference's part bytes (LoadLayer / LoadEmbed /
LoadHead, shard.go:258-300, through rk_*_load_part) against the CPU oracle:
every step's logits bit for bit and the greedy tokens. The parts are made
by a restatement of EncodeLayer / EncodeHead (oracle/part_format.py) from
the oracle's own weights. Parts of the wrong size are refused.
"""
import numpy as np
import pytest

import part_format as pf
import rk_oracle as ro
import rkcuda as rk
import synth
from conftest import same_bits

pytestmark = pytest.mark.gpu

VARIANTS = {
    "llama": dict(shared_classifier=1),
    "qwen2_bias": dict(qkv_bias=1, rope_theta=1e6, norm_eps=1e-6, shared_classifier=1),
    "qwen3_qknorm_cls": dict(qk_norm=1, head_dim=32, shared_classifier=0),
}


@pytest.mark.parametrize("variant", sorted(VARIANTS))
@pytest.mark.parametrize("dtype", ["q8_0", "q4_0", "bf16", "f32", "q4_m"])
def test_model_from_parts_matches_oracle(dev, variant, dtype):
    base = dict(dim=64, hidden=160, layers=3, heads=4, kv_heads=2, vocab=50, seq_len=48, head_dim=0, rope_theta=0.0,
                norm_eps=0.0, qkv_bias=0, qk_norm=0)
    base.update(VARIANTS[variant])
    c = synth.config("", dtype, **base)
    seed, ctx = 31, 48
    om = ro.OracleModel(c, seed, ctx=ctx, vec_seed=700)
    keep = om.keep
    fmts = {k: synth.mat_fmt(c, k) for k in synth.MATS}
    ef = synth.embed_fmt(c)
    made = []
    try:
        layers, i = [], 0
        for _ in range(c.layers):
            vec, mats = keep[i], dict(zip(synth.MATS, keep[i + 1:i + 8]))
            i += 8
            part = pf.encode_layer(c, vec, mats, fmts)
            if not layers:
                for bad in (part[:-1], part + b"\0"):
                    with pytest.raises(rk.RkError) as e:
                        rk.layer_load_part(dev, c, bad)
                    assert e.value.code == rk.RK_ERR_ARGS
            layers.append(rk.layer_load_part(dev, c, part))
            made.append(layers[-1])
        ew, es = keep[i]
        embed = rk.embed_load_part(dev, c, pf.encode_matrix(ef, ew, es), ef)
        made.append(embed)
        cls = None if c.shared_classifier else keep[i + 1]
        head, wcls = rk.head_load_part(dev, c, pf.encode_head(c, om.rms_final, cls, ef), embed, ef)
        stage = rk.Stage(dev, c, layers, ctx)
        model = rk.Model(dev, embed, stage, head, c.vocab)
        made = [model, stage, head] + ([wcls] if wcls else []) + made
        prompt = np.array([3, 14, 15, 9], np.int32)
        toks, logits = model.generate(prompt, 5, want_logits=True)
        otoks, ologits = om.generate(prompt, 5)
        same_bits(logits, ologits)
        assert list(toks) == list(otoks)
    finally:
        om.free()
        for m in made:
            m.free()
    assert dev.used() == 0
