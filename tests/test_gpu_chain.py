"""The chained decode products (RK_CHAIN=1: after each layer's attention,
Wo, W1·W3, W2 and the next layer's Q/K/V in one persistent launch, each
product's output handed to the next as tagged words) against the CPU
oracle: every step's logits bit for bit and the greedy tokens, for a
Llama-style and a Qwen3-style model (QK-norm, head 128) in Q8_0 and Q4_0.
The variable is read when a stage records its decode step, so it is set
only while the model is built and run.
"""
import numpy as np
import pytest

import rk_oracle as ro
import synth
from conftest import same_bits

pytestmark = pytest.mark.gpu

PROMPT = np.array([7, 300, 12, 999, 45], np.int32)
N_NEW = 6


def _config(dtype, variant):
    over = dict(layers=3, dim=1024, hidden=2816, heads=16, kv_heads=4, vocab=4096, seq_len=64)
    if variant == "qwen3":
        over.update(head_dim=128, qk_norm=1, rope_theta=1e6, norm_eps=1e-6, kv_heads=8)
    return synth.config("llama3-8b", dtype, **over)


@pytest.mark.parametrize("variant", ["llama", "qwen3"])
@pytest.mark.parametrize("dtype", ["q8_0", "q4_0"])
def test_chained_decode_matches_oracle(dev, monkeypatch, dtype, variant):
    c = _config(dtype, variant)
    monkeypatch.setenv("RK_CHAIN", "1")
    dm = synth.DeviceModel(dev, c, 11, ctx=64, keep_host=True)
    try:
        toks, logits = dm.model.generate(PROMPT, N_NEW, want_logits=True)
        assert dm.stage.chained() == 1
        om = ro.OracleModel(c, 11, ctx=64, weights=dm.host_weights)
        try:
            want_toks, want_logits = om.generate(PROMPT, N_NEW)
        finally:
            om.free()
        for i in range(logits.shape[0]):
            same_bits(logits[i], want_logits[i])
        assert (toks == want_toks).all()
    finally:
        dm.free()
    assert dev.used() == 0
