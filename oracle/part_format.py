"""CPU restatement of the reference's part encoders (internal/llm/shard.go:
150-178 f32Bytes/appendMatrix, 242-253 EncodeLayer, 272-279 EncodeHead; the
embedding part is the table in its own type, shard.go:282-287). Test
infrastructure only: the GPU tests load the bytes it makes through the
library's rk_*_load_part and compare the model with the oracle.
"""
import numpy as np

import rk_oracle as ro


def encode_matrix(fmt, w, s):
    """appendMatrix (shard.go:165-183): quantized as the float32 scales then
    the values; bfloat16 and float32 as themselves; little-endian."""
    if fmt in (ro.Q8_0, ro.Q4_0):
        return np.ascontiguousarray(s, dtype="<f4").tobytes() + np.ascontiguousarray(w).view(np.uint8).tobytes()
    if fmt == ro.BF16:
        return np.ascontiguousarray(w, dtype="<u2").tobytes()
    return np.ascontiguousarray(w, dtype="<f4").tobytes()


def encode_layer(c, vec, mats, fmts):
    """EncodeLayer (shard.go:242-253) in Layer.tensors order (model.go:328-343).
    mats / fmts: {"wq": (w, s), ...} and their formats."""
    f32 = lambda a: np.ascontiguousarray(a, dtype="<f4").tobytes()
    out = [f32(vec["rms_att"])]
    out += [encode_matrix(fmts[k], *mats[k]) for k in ("wq", "wk", "wv", "wo")]
    out.append(f32(vec["rms_ffn"]))
    out += [encode_matrix(fmts[k], *mats[k]) for k in ("w1", "w2", "w3")]
    if c.qkv_bias:
        out += [f32(vec["bq"]), f32(vec["bk"]), f32(vec["bv"])]
    if c.qk_norm:
        out += [f32(vec["q_norm"]), f32(vec["k_norm"])]
    return b"".join(out)


def encode_head(c, rms_final, cls=None, cls_fmt=None):
    """EncodeHead (shard.go:272-279): RmsFinal, then the classifier unless
    it is shared."""
    b = np.ascontiguousarray(rms_final, dtype="<f4").tobytes()
    if not c.shared_classifier:
        b += encode_matrix(cls_fmt, *cls)
    return b
