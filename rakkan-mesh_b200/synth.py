"""Seeded synthetic models for the benchmark configurations.

The weights are random: every matrix is N(0, 0.02) from this project's
seeded generator (rk_matrix_generate: Box–Muller over splitmix64, element i
of tensor `tid`), quantized on the device to the model's format with the
reference's quantizers (num.QuantizeQ8 / QuantizeQ4). RMSNorm and QK-norm
weights are 1.0 and biases 0.0. The same (seed, tid) produce the same bytes
on the host, so a CPU reference can rebuild any model bit for bit.
"""
import ctypes as C

import numpy as np

import rkcuda as rk

# Model shapes (llm.Config fields, model.go:37-64).
CONFIGS = {
    # llama2.c stories15M (config 1): shared classifier, theta 1e4.
    "stories15M": dict(dim=288, hidden=768, layers=6, heads=6, kv_heads=6, vocab=32000, seq_len=256,
                       shared_classifier=1, head_dim=0, rope_theta=0.0, norm_eps=0.0, qkv_bias=0, qk_norm=0),
    # Qwen2.5-0.5B (config 3): QKV bias, head_dim 64, theta 1e6, eps 1e-6.
    "qwen2.5-0.5b": dict(dim=896, hidden=4864, layers=24, heads=14, kv_heads=2, vocab=151936, seq_len=768,
                         shared_classifier=1, head_dim=64, rope_theta=1e6, norm_eps=1e-6, qkv_bias=1, qk_norm=0),
    # Llama-3-8B (config 4): theta 5e5 (the published model's; BASELINE does not state it).
    "llama3-8b": dict(dim=4096, hidden=14336, layers=32, heads=32, kv_heads=8, vocab=128256, seq_len=4224,
                      shared_classifier=0, head_dim=0, rope_theta=5e5, norm_eps=1e-5, qkv_bias=0, qk_norm=0),
    # Qwen3-32B (config 5): QK-norm, head_dim 128, theta 1e6, eps 1e-6.
    "qwen3-32b": dict(dim=5120, hidden=25600, layers=64, heads=64, kv_heads=8, vocab=151936, seq_len=2560,
                      shared_classifier=0, head_dim=128, rope_theta=1e6, norm_eps=1e-6, qkv_bias=0, qk_norm=1),
}

DTYPES = {"f32": rk.DTYPE_F32, "bf16": rk.DTYPE_BF16, "q8_0": rk.DTYPE_Q8_0, "q4_0": rk.DTYPE_Q4_0,
          "q4_m": rk.DTYPE_Q4_M}

MATS = ("wq", "wk", "wv", "wo", "w1", "w2", "w3")
TID_EMBED = 0xE0000
TID_CLS = 0xC0000
WEIGHT_SCALE = 0.02


def tid(layer, kind):
    """Tensor id of a layer matrix (kind in MATS)."""
    return (layer << 4) | (MATS.index(kind) + 1)


def config(name, dtype="q8_0", **over):
    c = dict(CONFIGS[name]) if name in CONFIGS else {}
    c.update(over)
    c["dtype"] = DTYPES[dtype] if isinstance(dtype, str) else dtype
    return rk.Config(**c)


def head_size(c):
    return c.head_dim if c.head_dim > 0 else c.dim // c.heads


def mat_fmt(c, kind):
    """Config.matType (model.go:105-113) as a matrix format."""
    sensitive = kind in ("wv", "w2")
    return {rk.DTYPE_F32: rk.FMT_F32, rk.DTYPE_BF16: rk.FMT_BF16, rk.DTYPE_Q8_0: rk.FMT_Q8_0,
            rk.DTYPE_Q4_0: rk.FMT_Q4_0}.get(c.dtype, rk.FMT_Q8_0 if sensitive else rk.FMT_Q4_0)


def embed_fmt(c):
    """Config.embedType (model.go:96-101)."""
    return {rk.DTYPE_F32: rk.FMT_F32, rk.DTYPE_BF16: rk.FMT_BF16}.get(c.dtype, rk.FMT_Q8_0)


def mat_shape(c, kind):
    hs = head_size(c)
    q, kv, d, h = c.heads * hs, c.kv_heads * hs, c.dim, c.hidden
    return {"wq": (q, d), "wk": (kv, d), "wv": (kv, d), "wo": (d, q), "w1": (h, d), "w2": (d, h), "w3": (h, d)}[kind]


def shard_rows(c, nshards, shard):
    """Rows [row0, row0 + rows) of each layer matrix (and "cls", the
    classifier) that shard `shard` of `nshards` holds: whole query / kv heads
    of Wq, Wk, Wv; dim/G rows of Wo and W2; hidden/G rows of W1 and W3;
    vocab/G classifier rows (the layout rk_layer_*_shard checks)."""
    G, r, hs = nshards, shard, head_size(c)
    if c.kv_heads % G or c.dim % G or c.hidden % G or c.vocab % G:
        raise ValueError(f"cannot shard {c.kv_heads} kv heads / dim {c.dim} / hidden {c.hidden} / vocab {c.vocab} over {G}")
    q, kv, d, h = c.heads * hs // G, c.kv_heads * hs // G, c.dim // G, c.hidden // G
    return {"wq": (r * q, q), "wk": (r * kv, kv), "wv": (r * kv, kv), "wo": (r * d, d), "w1": (r * h, h),
            "w2": (r * d, d), "w3": (r * h, h), "cls": (r * (c.vocab // G), c.vocab // G)}


def layer_vectors(c, vec_seed=None):
    """RmsAtt, RmsFfn = 1; biases = 0; QNorm, KNorm = 1 (the benchmark's
    choice: BASELINE.json does not give vectors). With vec_seed the tests get
    seeded non-trivial vectors instead (norm weights 1 + N(0, 0.1), biases
    N(0, 0.1)), so that every vector's indexing shows in the bits."""
    hs = head_size(c)
    if vec_seed is None:
        one = lambda n: np.ones(n, np.float32)
        zero = lambda n: np.zeros(n, np.float32)
    else:
        rng = np.random.default_rng(vec_seed)
        one = lambda n: (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
        zero = lambda n: (0.1 * rng.standard_normal(n)).astype(np.float32)
    v = {"rms_att": one(c.dim), "rms_ffn": one(c.dim)}
    if c.qkv_bias:
        v.update(bq=zero(c.heads * hs), bk=zero(c.kv_heads * hs), bv=zero(c.kv_heads * hs))
    if c.qk_norm:
        v.update(q_norm=one(hs), k_norm=one(hs))
    return v


def host_layer_vectors(c, vec_seed=None):
    v = layer_vectors(c, vec_seed)
    hl = rk.HostLayer()
    for k, a in v.items():
        setattr(hl, k, a.ctypes.data)
    return hl, v


def to_bf16(f):
    """num.ToBF16 (matvec.go:23-29) on float32 arrays."""
    b = np.ascontiguousarray(f, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(f)
    if nan.any():
        r[nan] = ((b[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def generate_matrix(dev, rows, cols, fmt, seed, t, part=None):
    """The seeded rows x cols tensor t; part=(row0, n) generates only rows
    [row0, row0 + n) (a shard)."""
    row0, n = part if part else (0, rows)
    if fmt == rk.FMT_BF16:
        w = rk.generate_normal(dev, seed, t, row0 * cols, n * cols, WEIGHT_SCALE)
        return rk.Matrix(dev, n, cols, fmt, to_bf16(w))
    if part:
        return rk.Matrix.generate_rows(dev, rows, row0, n, cols, fmt, seed, t, WEIGHT_SCALE)
    return rk.Matrix.generate(dev, rows, cols, fmt, seed, t, WEIGHT_SCALE)


class DeviceModel:
    """A whole synthetic model on one device: embed, stage of all layers,
    head and the greedy decode loop (rk_model)."""

    def __init__(self, dev, c, seed, ctx=None, keep_host=False, group=None, nseq=1):
        """keep_host: also download every matrix (host_weights, keyed like
        the oracle's OracleModel(weights=...)) before the layers own them.
        group: an rk.Group; this process then holds its row shard of every
        layer and of the classifier (shard_rows) and decodes collectively."""
        self.c, self.dev, self.seed = c, dev, seed
        self.ctx = ctx or c.seq_len
        self.layers = []
        self.host_weights = {} if keep_host else None
        G, r = (group.nranks, group.rank) if group else (1, 0)
        parts = shard_rows(c, G, r) if group else {}
        for l in range(c.layers):
            mats = [generate_matrix(dev, *mat_shape(c, k), mat_fmt(c, k), seed, tid(l, k), parts.get(k)) for k in MATS]
            if keep_host:
                for k, m in zip(MATS, mats):
                    self.host_weights[(l, k)] = m.download()
            self.layers.append(rk.Layer(dev, c, mats=mats, vectors=host_layer_vectors(c),
                                        shard=(G, r) if group else None))
        ef = embed_fmt(c)
        self.embed = generate_matrix(dev, c.vocab, c.dim, ef, seed, TID_EMBED)
        if group:
            t = TID_EMBED if c.shared_classifier else TID_CLS
            self.wcls = generate_matrix(dev, c.vocab, c.dim, ef, seed, t, parts["cls"])
        else:
            self.wcls = self.embed if c.shared_classifier else generate_matrix(dev, c.vocab, c.dim, ef, seed, TID_CLS)
        if keep_host:
            self.host_weights["embed"] = self.embed.download()
            self.host_weights["cls"] = self.wcls.download()
        self.stage = rk.Stage(dev, c, self.layers, self.ctx, group=group, nseq=nseq)
        self.head = rk.Head(dev, c, np.ones(c.dim, np.float32), self.wcls, group=group)
        self.model = rk.Model(dev, self.embed, self.stage, self.head, c.vocab)

    def weight_bytes(self):
        """Algorithmic bytes of the weights one decode step reads (matBytes,
        model.go:269-279, for every layer matrix and the classifier)."""
        total = 0
        for l in range(self.c.layers):
            for k in MATS:
                rows, cols = mat_shape(self.c, k)
                total += matrix_bytes(mat_fmt(self.c, k), rows * cols)
        total += matrix_bytes(embed_fmt(self.c), self.c.vocab * self.c.dim)
        return total

    def free(self):
        self.model.free()
        self.head.free()
        self.stage.free()
        for l in self.layers:
            l.free()
        if self.wcls is not self.embed:
            self.wcls.free()
        self.embed.free()


def matrix_bytes(fmt, n):
    """matBytes (model.go:269-279)."""
    return {rk.FMT_BF16: 2 * n, rk.FMT_Q8_0: n + (n // 32) * 4, rk.FMT_Q4_0: n // 2 + (n // 32) * 4}.get(fmt, 4 * n)


class PipelineRank:
    """Rank `group.rank`'s part of a layer pipeline of a synthetic model:
    layers [first, end) (their weights those of the whole model's layers
    first..end-1, so the oracle's single model matches), the embedding table
    on the first rank and the head on the last (rk.Pipeline)."""

    def __init__(self, dev, c, seed, group, first, end, ctx=None):
        self.c, self.dev = c, dev
        self.ctx = ctx or c.seq_len
        self.layers = []
        for l in range(first, end):
            mats = [generate_matrix(dev, *mat_shape(c, k), mat_fmt(c, k), seed, tid(l, k)) for k in MATS]
            self.layers.append(rk.Layer(dev, c, mats=mats, vectors=host_layer_vectors(c)))
        self.stage = rk.Stage(dev, c, self.layers, self.ctx)
        ef = embed_fmt(c)
        first_rank, last_rank = group.rank == 0, group.rank == group.nranks - 1
        self.embed = generate_matrix(dev, c.vocab, c.dim, ef, seed, TID_EMBED) if first_rank else None
        self.wcls, self.head = None, None
        if last_rank:
            if c.shared_classifier:
                self.wcls = self.embed if first_rank else generate_matrix(dev, c.vocab, c.dim, ef, seed, TID_EMBED)
            else:
                self.wcls = generate_matrix(dev, c.vocab, c.dim, ef, seed, TID_CLS)
            self.head = rk.Head(dev, c, np.ones(c.dim, np.float32), self.wcls)
        self.pipeline = rk.Pipeline(group, self.embed, self.stage, self.head, c.vocab)

    def generate(self, prompt, n_new):
        """The greedy loop (generate.go:522-585) over the pipeline: tokens,
        and on the last rank every step's logits."""
        toks, logits = [], []
        steps = len(prompt) + n_new - 1
        nxt = 0
        for i in range(steps):
            tok = int(prompt[i]) if i < len(prompt) else nxt
            nxt, lg = self.pipeline.step(tok, i)
            if lg is not None:
                logits.append(lg)
            if i >= len(prompt) - 1:
                toks.append(nxt)
        return np.array(toks[:n_new], np.int32), (np.stack(logits) if logits else None)

    def free(self):
        self.pipeline.free()
        if self.head:
            self.head.free()
        self.stage.free()
        for l in self.layers:
            l.free()
        for m in {id(x): x for x in (self.embed, self.wcls) if x is not None}.values():
            m.free()
