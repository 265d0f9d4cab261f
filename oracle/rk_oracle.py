"""ctypes binding of the CPU oracle (librk_oracle.so, rk_oracle.c).

TEST INFRASTRUCTURE ONLY: the checker the CUDA backend is compared against
(tests/, __graft_entry__.smoke() and bench.py's CPU baseline). The product
library never imports or calls this module.
"""
import ctypes as C
import os
import subprocess
import sys
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "librk_oracle.so")
sys.path.insert(0, os.path.join(HERE, "..", "rakkan-mesh_b200"))
import synth  # noqa: E402  (tensor ids and shapes of the synthetic models)
import rkcuda as rk  # noqa: E402  (only for its Config / format constants)

F32, BF16, Q8_0, Q4_0 = 0, 1, 2, 3
DT_F32, DT_I8, DT_I32 = 0, 1, 2


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)


class Config(C.Structure):
    _fields_ = [("dim", C.c_int), ("hidden", C.c_int), ("layers", C.c_int), ("heads", C.c_int),
                ("kv_heads", C.c_int), ("vocab", C.c_int), ("seq_len", C.c_int), ("shared_classifier", C.c_int),
                ("head_dim", C.c_int), ("rope_theta", C.c_double), ("norm_eps", C.c_double), ("qkv_bias", C.c_int),
                ("qk_norm", C.c_int), ("dtype", C.c_int)]


class Mat(C.Structure):
    _fields_ = [("fmt", C.c_int), ("rows", C.c_int), ("cols", C.c_int), ("w", C.c_void_p), ("scales", C.c_void_p)]


class Layer(C.Structure):
    _fields_ = [("rms_att", C.c_void_p), ("rms_ffn", C.c_void_p), ("bq", C.c_void_p), ("bk", C.c_void_p),
                ("bv", C.c_void_p), ("q_norm", C.c_void_p), ("k_norm", C.c_void_p)] + [
                   (n, Mat) for n in ("wq", "wk", "wv", "wo", "w1", "w2", "w3")]


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        vp, i, i64, f, d, u64 = C.c_void_p, C.c_int, C.c_int64, C.c_float, C.c_double, C.c_uint64
        sig = {
            "rko_canonical": (f, [f]), "rko_exp32": (f, [f]), "rko_exp": (d, [d]), "rko_log": (d, [d]),
            "rko_log32": (f, [f]), "rko_log1p32": (f, [f]), "rko_log1p": (d, [d]), "rko_sincos": (None, [d, vp, vp]),
            "rko_pow2": (f, [i]), "rko_scale2": (f, [f, i]), "rko_recip32": (f, [f]), "rko_rsqrt32": (f, [f]),
            "rko_gomax32": (f, [f, f]), "rko_dot": (f, [vp, vp, i]), "rko_dot32": (f, [vp, vp, i]),
            "rko_dotbf16": (f, [vp, vp, i]), "rko_bf16": (f, [C.c_uint16]), "rko_to_bf16": (C.c_uint16, [f]),
            "rko_quantize_q8": (None, [vp, i64, vp, vp]), "rko_quantize_q4": (None, [vp, i64, vp, vp]),
            "rko_dequant_q8": (None, [vp, i64, vp, vp]), "rko_dequant_q4": (None, [vp, i64, vp, vp]),
            "rko_block_sums_q8": (None, [vp, vp, i, vp]), "rko_block_sums_q4": (None, [vp, vp, i, vp]),
            "rko_qrow": (f, [vp, vp, vp, i]), "rko_matvec": (None, [i, vp, i, i, vp, vp, vp, i]),
            "rko_tensor_matmul": (i, [i, i, i, i, i, vp, vp, vp, i]), "rko_config_validate": (i, [vp]),
            "rko_head_size": (i, [vp]), "rko_eps": (f, [vp]), "rko_rmsnorm": (None, [vp, vp, vp, i, f]),
            "rko_softmax": (None, [vp, i]), "rko_silu": (f, [f]), "rko_rope_table": (None, [vp, i, vp, vp]),
            "rko_argmax": (i, [vp, i]), "rko_stage_new": (vp, [vp, vp, i, i, i]), "rko_stage_free": (None, [vp]),
            "rko_stage_forward": (i, [vp, vp, i]), "rko_stage_fill_cache": (None, [vp, i, u64]), "rko_embed": (None, [vp, vp, i, vp]),
            "rko_head_logits": (None, [vp, vp, vp, vp, vp, i]), "rko_splitmix64": (u64, [u64]),
            "rko_gen_normal": (None, [u64, u64, i64, i64, f, vp]), "rko_transcendental_stream": (None, [vp]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a):
    return a.ctypes.data_as(C.c_void_p)


THREADS = max(1, min(64, os.cpu_count() or 1))


def _parallel(n, chunk, fn):
    """Runs fn(lo, hi) over [0, n) in chunks on threads (ctypes releases the GIL)."""
    spans = [(lo, min(n, lo + chunk)) for lo in range(0, n, chunk)]
    idx = [0]
    lock = threading.Lock()

    def worker():
        while True:
            with lock:
                if idx[0] >= len(spans):
                    return
                lo, hi = spans[idx[0]]
                idx[0] += 1
            fn(lo, hi)

    ts = [threading.Thread(target=worker) for _ in range(min(THREADS, len(spans)))]
    for t in ts:
        t.start()
    for t in ts:
        t.join()


def gen_normal(seed, tid, n, scale, offset=0):
    out = np.empty(n, dtype=np.float32)
    base = out.ctypes.data

    def fn(lo, hi):
        lib().rko_gen_normal(seed, tid, offset + lo, hi - lo, scale, C.c_void_p(base + 4 * lo))

    _parallel(n, 1 << 20, fn)
    return out


def quantize(fmt, w):
    w = np.ascontiguousarray(w, dtype=np.float32)
    n = w.size
    s = np.empty(n // 32, dtype=np.float32)
    if fmt == Q8_0:
        q = np.empty(n, dtype=np.int8)
        wb, qb, sb = w.ctypes.data, q.ctypes.data, s.ctypes.data

        def fn(lo, hi):
            lib().rko_quantize_q8(C.c_void_p(wb + 4 * 32 * lo), 32 * (hi - lo), C.c_void_p(qb + 32 * lo),
                                  C.c_void_p(sb + 4 * lo))

        _parallel(n // 32, 1 << 16, fn)
    else:
        # QuantizeQ4 over the whole tensor as one range (the reference's
        # stale-block rule depends on range boundaries; finite weights never
        # hit it, so splitting is safe for them).
        q = np.empty(n // 2, dtype=np.uint8)
        wb, qb, sb = w.ctypes.data, q.ctypes.data, s.ctypes.data
        if np.isfinite(w).all():
            def fn(lo, hi):
                lib().rko_quantize_q4(C.c_void_p(wb + 4 * 32 * lo), 32 * (hi - lo), C.c_void_p(qb + 16 * lo),
                                      C.c_void_p(sb + 4 * lo))

            _parallel(n // 32, 1 << 14, fn)
        else:
            lib().rko_quantize_q4(_p(w), n, _p(q), _p(s))
    return q, s


def matvec(fmt, w, scales, x, rows, cols, threads=THREADS):
    out = np.empty(rows, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    lib().rko_matvec(fmt, _p(out), rows, cols, _p(w), None if scales is None else _p(scales), _p(x), threads)
    return out


def tensor_matmul(a, b, transposed, threads=THREADS):
    if a.dtype == np.float32:
        dt, ot = DT_F32, np.float32
    elif a.dtype == np.int8:
        dt, ot = DT_I8, np.int32
    else:
        return None
    m, k = a.shape
    n = b.shape[0] if transposed else b.shape[1]
    c = np.empty((m, n), dtype=ot)
    rc = lib().rko_tensor_matmul(dt, 1 if transposed else 0, m, k, n, _p(np.ascontiguousarray(a)),
                                 _p(np.ascontiguousarray(b)), _p(c), threads)
    return c if rc == 0 else None


def to_config(c):
    """An oracle Config from the product's rk.Config (same fields)."""
    return Config(**{f: getattr(c, f) for f, _ in Config._fields_})


class OracleModel:
    """The synthetic model of synth.py rebuilt on the host, run by the CPU
    restatement (Stage.Forward / Head.Logits / argmax)."""

    def __init__(self, c, seed, ctx=None, weights=None, threads=THREADS, vec_seed=None):
        self.c = to_config(c)
        self.pc = c
        self.ctx = ctx or c.seq_len
        self.threads = threads
        self.keep = []
        self.layers = (Layer * c.layers)()
        for l in range(c.layers):
            vec = synth.layer_vectors(c, None if vec_seed is None else vec_seed + l)
            self.keep.append(vec)
            L = self.layers[l]
            for k, a in vec.items():
                setattr(L, k, a.ctypes.data)
            for k in synth.MATS:
                rows, cols = synth.mat_shape(c, k)
                fmt = synth.mat_fmt(c, k)
                w, s = weights[(l, k)] if weights else self._make(fmt, rows, cols, seed, synth.tid(l, k))
                self.keep.append((w, s))
                setattr(L, k, Mat(fmt, rows, cols, w.ctypes.data, None if s is None else s.ctypes.data))
        ef = synth.embed_fmt(c)
        ew, es = weights["embed"] if weights else self._make(ef, c.vocab, c.dim, seed, synth.TID_EMBED)
        self.embed = Mat(ef, c.vocab, c.dim, ew.ctypes.data, None if es is None else es.ctypes.data)
        self.keep.append((ew, es))
        if c.shared_classifier:
            self.wcls = self.embed
        else:
            cw, cs = weights["cls"] if weights else self._make(ef, c.vocab, c.dim, seed, synth.TID_CLS)
            self.keep.append((cw, cs))
            self.wcls = Mat(ef, c.vocab, c.dim, cw.ctypes.data, None if cs is None else cs.ctypes.data)
        self.rms_final = np.ones(c.dim, np.float32)
        self.stage = lib().rko_stage_new(C.byref(self.c), self.layers, c.layers, self.ctx, threads)
        if not self.stage:
            raise ValueError("invalid config")

    @staticmethod
    def _make(fmt, rows, cols, seed, tid):
        w = gen_normal(seed, tid, rows * cols, synth.WEIGHT_SCALE)
        if fmt == F32:
            return w, None
        if fmt == BF16:
            return synth.to_bf16(w), None
        return quantize(fmt, w)

    def fill_cache(self, positions, seed):
        lib().rko_stage_fill_cache(self.stage, positions, seed)

    def embed_token(self, tok):
        x = np.empty(self.c.dim, np.float32)
        lib().rko_embed(C.byref(self.c), C.byref(self.embed), tok, _p(x))
        return x

    def forward(self, x, pos):
        x = np.ascontiguousarray(x, dtype=np.float32).copy()
        rc = lib().rko_stage_forward(self.stage, _p(x), pos)
        assert rc == 0
        return x

    def logits(self, x):
        out = np.empty(self.c.vocab, np.float32)
        lib().rko_head_logits(C.byref(self.c), _p(self.rms_final), C.byref(self.wcls), _p(x), _p(out), self.threads)
        return out

    def step(self, tok, pos):
        lg = self.logits(self.forward(self.embed_token(tok), pos))
        return int(lib().rko_argmax(_p(lg), lg.size)), lg

    def generate(self, prompt, n_new):
        """Greedy decode as rk_model_generate: logits of every step."""
        toks, logits = [], []
        tok = int(prompt[0])
        steps = len(prompt) + n_new - 1
        for i in range(steps):
            if i < len(prompt):
                tok = int(prompt[i])
            nxt, lg = self.step(tok, i)
            logits.append(lg)
            if i >= len(prompt) - 1:
                toks.append(nxt)
            tok = nxt
        return np.array(toks, np.int32), np.stack(logits)

    def free(self):
        if self.stage:
            lib().rko_stage_free(self.stage)
            self.stage = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass
