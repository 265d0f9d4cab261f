"""ctypes binding of librakkan_cuda.so (include/rakkan_cuda.h).

The Python side of the C ABI: what a Go cgo shim would call, written as
thin classes over numpy arrays. There is no fallback: if the CUDA library
cannot be loaded or a call fails, an RkError is raised.
"""
import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "librakkan_cuda.so")

RK_OK, RK_ERR_ARGS, RK_ERR_TOO_BIG = 0, -1, -3
RK_ERR_CUDA, RK_ERR_NOMEM, RK_ERR_TIMEOUT, RK_ERR_STATE = -10, -11, -12, -13
RK_ERR_BLOB = -5
FMT_F32, FMT_BF16, FMT_Q8_0, FMT_Q4_0 = 0, 1, 2, 3
DTYPE_F32, DTYPE_BF16, DTYPE_Q8_0, DTYPE_Q4_0, DTYPE_Q4_M = 0, 1, 2, 3, 4
TENSOR_F32, TENSOR_I8, TENSOR_I32 = 0, 1, 2
RK_BENCH_FLUSH, RK_BENCH_FUSED = 1, 2
MAX_COLS, MAX_ROWS = 1 << 18, 1 << 20
NOALLOC_MAX_COLS = 32768

# Every symbol include/rakkan_cuda.h declares.
EXPORTS = [
    "rk_last_error", "rk_version", "rk_device_count", "rk_device_get_info", "rk_device_best", "rk_device_open",
    "rk_device_close", "rk_device_used", "rk_device_wait_selftest", "rk_matrix_upload", "rk_matrix_free", "rk_matrix_bytes", "rk_same_device",
    "rk_matrix_mulvec", "rk_matrix_mulvec_many", "rk_mulvecs", "rk_matrix_mulvec_noalloc", "rk_vectors_upload", "rk_vectors_free", "rk_arena_new",
    "rk_arena_set_quant_scratch", "rk_arena_bytes", "rk_arena_free", "rk_batch_begin", "rk_batch_write",
    "rk_batch_read", "rk_batch_matvecs", "rk_batch_quantize", "rk_batch_rmsnorm", "rk_batch_addvec", "rk_batch_rope",
    "rk_batch_copy", "rk_batch_attention", "rk_batch_residual", "rk_batch_silumul", "rk_batch_submit",
    "rk_config_validate", "rk_layer_upload", "rk_layer_from_device", "rk_layer_free", "rk_stage_new", "rk_stage_free",
    "rk_stage_positions", "rk_stage_forward", "rk_stage_batched", "rk_stage_new_batch", "rk_stage_forward_batch", "rk_head_new", "rk_head_free", "rk_head_logits", "rk_embed", "rk_sample_argmax",
    "rk_model_new", "rk_model_free", "rk_model_step", "rk_model_generate", "rk_tensor_matmul",
    "rk_tensor_matmul_device", "rk_matrix_generate", "rk_matrix_download", "rk_generate_normal", "rk_quantize",
    "rk_bench_matvec", "rk_bench_matvec_many", "rk_bench_tensor", "rk_bench_model", "rk_group_id", "rk_group_new", "rk_group_free",
    "rk_group_size", "rk_group_all_gather", "rk_layer_upload_shard", "rk_layer_from_device_shard",
    "rk_stage_new_group", "rk_head_new_group", "rk_matrix_generate_rows", "rk_stage_fused_gathers", "rk_stage_chained", "rk_model_kernel_count", "rk_model_profile", "rk_stage_fill_cache", "rk_stage_fill_cache_from",
    "rk_plan_stages", "rk_pipeline_new", "rk_pipeline_free", "rk_pipeline_step", "rk_bench_pipeline",
    "rk_tensor_add", "rk_tensor_scale", "rk_tensor_relu", "rk_tensor_softmax", "rk_tensor_quantize", "rk_tensor_argmax",
    "rk_layer_load_part", "rk_embed_load_part", "rk_head_load_part", "rk_matmul_bf16", "rk_measure_speed",
    "rk_tensors_new", "rk_tensors_free", "rk_tensors_used", "rk_tensors_from_memory", "rk_tensors_from_blob",
    "rk_tensors_to_memory", "rk_tensors_dim", "rk_tensors_release", "rk_tensors_matmul", "rk_tensors_add",
    "rk_tensors_scale", "rk_tensors_relu", "rk_tensors_softmax", "rk_tensors_quantize", "rk_tensors_argmax",
]


class RkError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"rakkan_cuda error {code}: {msg}")
        self.code = code


class DeviceInfo(C.Structure):
    _fields_ = [("index", C.c_int), ("name", C.c_char * 256), ("memory", C.c_int64), ("sm_count", C.c_int),
                ("cc_major", C.c_int), ("cc_minor", C.c_int), ("exact", C.c_int)]


class Config(C.Structure):
    """llm.Config (model.go:37-64)."""
    _fields_ = [("dim", C.c_int), ("hidden", C.c_int), ("layers", C.c_int), ("heads", C.c_int),
                ("kv_heads", C.c_int), ("vocab", C.c_int), ("seq_len", C.c_int), ("shared_classifier", C.c_int),
                ("head_dim", C.c_int), ("rope_theta", C.c_double), ("norm_eps", C.c_double), ("qkv_bias", C.c_int),
                ("qk_norm", C.c_int), ("dtype", C.c_int)]


class Profile(C.Structure):
    _fields_ = [("step_ms", C.c_float), ("matvec_ms", C.c_float), ("matvec_bytes", C.c_double),
                ("matvec_launches", C.c_int), ("launches", C.c_int)]


class HostMatrix(C.Structure):
    _fields_ = [("fmt", C.c_int), ("w", C.c_void_p), ("scales", C.c_void_p)]


class HostLayer(C.Structure):
    _fields_ = [("rms_att", C.c_void_p), ("rms_ffn", C.c_void_p), ("bq", C.c_void_p), ("bk", C.c_void_p),
                ("bv", C.c_void_p), ("q_norm", C.c_void_p), ("k_norm", C.c_void_p)] + [
                   (n, HostMatrix) for n in ("wq", "wk", "wv", "wo", "w1", "w2", "w3")]


_lib = None


def lib():
    """The loaded library (raises if it is missing: no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RkError(RK_ERR_CUDA, f"{LIB_PATH} is not built (run rakkan-mesh_b200/build.py)")
        L = C.CDLL(LIB_PATH)
        vp, i, i64, f, u64 = C.c_void_p, C.c_int, C.c_int64, C.c_float, C.c_uint64
        sig = {
            "rk_last_error": (C.c_char_p, []), "rk_version": (C.c_char_p, []),
            "rk_device_count": (i, [vp]), "rk_device_get_info": (i, [i, vp]), "rk_device_best": (i, [vp]),
            "rk_device_open": (i, [i, vp]), "rk_device_close": (None, [vp]), "rk_device_used": (i64, [vp]), "rk_device_wait_selftest": (i, [vp, i64]),
            "rk_matrix_upload": (i, [vp, i, i, i, vp, vp, vp]), "rk_matrix_free": (None, [vp]),
            "rk_matrix_bytes": (i64, [vp]), "rk_same_device": (i, [vp, vp]),
            "rk_matrix_mulvec": (i, [vp, vp, vp]), "rk_matrix_mulvec_many": (i, [vp, i, vp, vp]), "rk_mulvecs": (i, [i, vp, vp, vp]),
            "rk_matrix_mulvec_noalloc": (i, [vp, vp, vp, vp]),
            "rk_vectors_upload": (i, [vp, vp, i64, vp]), "rk_vectors_free": (None, [vp]),
            "rk_arena_new": (i, [vp, i64, i64, vp]), "rk_arena_set_quant_scratch": (None, [vp, i64, i64]),
            "rk_arena_bytes": (i64, [vp]), "rk_arena_free": (None, [vp]), "rk_batch_begin": (i, [vp, vp]),
            "rk_batch_write": (None, [vp, i64, vp, i64]), "rk_batch_read": (None, [vp, i64, vp, i64]),
            "rk_batch_matvecs": (None, [vp, i, vp, vp, i64]), "rk_batch_quantize": (None, [vp, i64, i]),
            "rk_batch_rmsnorm": (None, [vp, vp, i64, i64, i64, i, i, i, f, f]),
            "rk_batch_addvec": (None, [vp, vp, i64, i64, i]),
            "rk_batch_rope": (None, [vp, i64, i64, i, i, i, i64, i64]),
            "rk_batch_copy": (None, [vp, i64, i64, i]),
            "rk_batch_attention": (None, [vp, i64, i64, i64, i64, i, i64, i, i, i, i, i, f]),
            "rk_batch_residual": (None, [vp, i64, i64, i, i]), "rk_batch_silumul": (None, [vp, i64, i64, i]),
            "rk_batch_submit": (i, [vp]), "rk_config_validate": (i, [vp]),
            "rk_layer_upload": (i, [vp, vp, vp, vp]),
            "rk_layer_from_device": (i, [vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp]),
            "rk_layer_free": (None, [vp]), "rk_stage_new": (i, [vp, vp, vp, i, i, vp]),
            "rk_stage_free": (None, [vp]), "rk_stage_positions": (i, [vp]), "rk_stage_forward": (i, [vp, vp, i, i]), "rk_stage_batched": (i, [vp]), "rk_stage_new_batch": (i, [vp, vp, vp, i, i, i, vp]), "rk_stage_forward_batch": (i, [vp, vp, vp, i]),
            "rk_head_new": (i, [vp, vp, vp, vp, vp]), "rk_head_free": (None, [vp]),
            "rk_head_logits": (i, [vp, vp, vp]), "rk_embed": (i, [vp, i, vp]),
            "rk_sample_argmax": (i, [vp, vp, i, vp]),
            "rk_model_new": (i, [vp, vp, vp, vp, vp]), "rk_model_free": (None, [vp]),
            "rk_model_step": (i, [vp, i, i, vp, vp]), "rk_model_generate": (i, [vp, vp, i, i, vp, vp]),
            "rk_tensor_matmul": (i, [vp, i, i, i, i, i, vp, vp, vp]),
            "rk_tensor_matmul_device": (i, [vp, i, i, i, i, i, vp, vp, vp]),
            "rk_matrix_generate": (i, [vp, i, i, i, u64, u64, f, vp]), "rk_matrix_download": (i, [vp, vp, vp]),
            "rk_generate_normal": (i, [vp, u64, u64, i64, i64, f, vp]), "rk_quantize": (i, [vp, i, vp, i64, vp, vp]),
            "rk_bench_matvec": (i, [vp, i, i, vp]), "rk_bench_matvec_many": (i, [vp, i, i, i, vp]), "rk_bench_model": (i, [vp, i, i, vp]),
            "rk_bench_tensor": (i, [vp, i, i, i, i, i, i, i, vp]),
            "rk_group_id": (i, [vp]), "rk_group_new": (i, [vp, i, i, vp, vp]), "rk_group_free": (None, [vp]),
            "rk_group_size": (i, [vp, vp, vp]), "rk_group_all_gather": (i, [vp, vp, i64]),
            "rk_layer_upload_shard": (i, [vp, vp, i, i, vp, vp]),
            "rk_layer_from_device_shard": (i, [vp, vp, i, i, vp, vp, vp, vp, vp, vp, vp, vp, vp]),
            "rk_stage_new_group": (i, [vp, vp, vp, i, i, vp, vp]),
            "rk_head_new_group": (i, [vp, vp, vp, vp, vp, vp]), "rk_stage_fused_gathers": (i, [vp]), "rk_stage_chained": (i, [vp]),
            "rk_matrix_generate_rows": (i, [vp, i, i, i, i, i, u64, u64, f, vp]),
            "rk_model_kernel_count": (i, [vp, vp]), "rk_model_profile": (i, [vp, i, i, vp]),
            "rk_stage_fill_cache": (i, [vp, i, u64]), "rk_stage_fill_cache_from": (i, [vp, i, u64, i]),
            "rk_plan_stages": (i, [vp, vp, i, vp, vp, vp, i, i, vp, vp, vp, vp]),
            "rk_pipeline_new": (i, [vp, vp, vp, vp, vp]), "rk_pipeline_free": (None, [vp]),
            "rk_pipeline_step": (i, [vp, i, i, vp, vp]), "rk_bench_pipeline": (i, [vp, i, i, vp]),
            "rk_tensor_add": (i, [vp, i, i, i, vp, vp, i, vp]), "rk_tensor_scale": (i, [vp, i, i, i, vp, f, vp]),
            "rk_tensor_relu": (i, [vp, i, i, i, vp, vp]), "rk_tensor_softmax": (i, [vp, i, i, i, vp, vp]),
            "rk_tensor_quantize": (i, [vp, i, i, i, vp, f, vp]), "rk_tensor_argmax": (i, [vp, i, i, i, vp, vp]),
            "rk_tensors_new": (i, [vp, i64, vp]), "rk_tensors_free": (None, [vp]), "rk_tensors_used": (i64, [vp]),
            "rk_tensors_from_memory": (i, [vp, vp, i, i, i]), "rk_tensors_from_blob": (i, [vp, vp, i64, i64, i, i, i]),
            "rk_tensors_to_memory": (i64, [vp, i, vp, i64]), "rk_tensors_dim": (i, [vp, i, i]),
            "rk_tensors_release": (i, [vp, i]), "rk_tensors_matmul": (i, [vp, i, i, i]), "rk_tensors_add": (i, [vp, i, i]),
            "rk_tensors_scale": (i, [vp, i, f]), "rk_tensors_relu": (i, [vp, i]), "rk_tensors_softmax": (i, [vp, i]),
            "rk_tensors_quantize": (i, [vp, i, f]), "rk_tensors_argmax": (i, [vp, i, vp, i64]),
            "rk_layer_load_part": (i, [vp, vp, vp, i64, vp]), "rk_embed_load_part": (i, [vp, vp, vp, i64, vp]),
            "rk_head_load_part": (i, [vp, vp, vp, i64, vp, vp, vp]),
            "rk_matmul_bf16": (i, [vp, i, vp, vp]), "rk_measure_speed": (i, [vp, vp]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _check(rc):
    if rc != RK_OK:
        raise RkError(rc, lib().rk_last_error().decode())
    return rc


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def device_count():
    n = C.c_int()
    _check(lib().rk_device_count(C.byref(n)))
    return n.value


def row_bytes(fmt, cols):
    return {FMT_F32: 4 * cols, FMT_BF16: 2 * cols, FMT_Q8_0: cols, FMT_Q4_0: cols // 2}[fmt]


def weight_dtype(fmt):
    return {FMT_F32: np.float32, FMT_BF16: np.uint16, FMT_Q8_0: np.int8, FMT_Q4_0: np.uint8}[fmt]


class Device:
    """gpu.Device (device.go:204-345)."""

    def __init__(self, index=0):
        self.h = C.c_void_p()
        _check(lib().rk_device_open(index, C.byref(self.h)))
        info = DeviceInfo()
        _check(lib().rk_device_get_info(index, C.byref(info)))
        self.info = info

    def used(self):
        return lib().rk_device_used(self.h)

    def close(self):
        if self.h:
            lib().rk_device_close(self.h)
            self.h = C.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


class Matrix:
    """gpu.Matrix (device.go:544-793)."""

    def __init__(self, dev, rows, cols, fmt, w=None, scales=None, handle=None):
        self.dev, self.rows, self.cols, self.fmt = dev, rows, cols, fmt
        if handle is not None:
            self.h = handle
            return
        w = np.ascontiguousarray(w)
        assert w.nbytes == rows * row_bytes(fmt, cols), "weights of the wrong size"
        s = None if scales is None else np.ascontiguousarray(scales, dtype=np.float32)
        self.h = C.c_void_p()
        _check(lib().rk_matrix_upload(dev.h, rows, cols, fmt, _ptr(w), _ptr(s), C.byref(self.h)))

    @classmethod
    def generate(cls, dev, rows, cols, fmt, seed, tid, scale):
        h = C.c_void_p()
        _check(lib().rk_matrix_generate(dev.h, rows, cols, fmt, seed, tid, scale, C.byref(h)))
        return cls(dev, rows, cols, fmt, handle=h)

    @classmethod
    def generate_rows(cls, dev, rows_total, row0, rows, cols, fmt, seed, tid, scale):
        """Rows [row0, row0+rows) of the generated rows_total x cols tensor."""
        h = C.c_void_p()
        _check(lib().rk_matrix_generate_rows(dev.h, rows_total, row0, rows, cols, fmt, seed, tid, scale, C.byref(h)))
        return cls(dev, rows, cols, fmt, handle=h)

    def download(self):
        w = np.empty(self.rows * row_bytes(self.fmt, self.cols) // np.dtype(weight_dtype(self.fmt)).itemsize,
                     dtype=weight_dtype(self.fmt))
        s = np.empty(self.rows * self.cols // 32, dtype=np.float32) if self.fmt in (FMT_Q8_0, FMT_Q4_0) else None
        _check(lib().rk_matrix_download(self.h, _ptr(w), _ptr(s)))
        return w, s

    def bytes(self):
        return lib().rk_matrix_bytes(self.h)

    def mulvec(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty(self.rows, dtype=np.float32)
        _check(lib().rk_matrix_mulvec(self.h, _ptr(out), _ptr(x)))
        return out

    def mulvec_many(self, xs):
        """W·x for every row x of xs [n][cols] (one MatVecQ8 each), in one
        pass over the weights when the batched kernel takes the matrix."""
        xs = np.ascontiguousarray(xs, dtype=np.float32).reshape(-1, self.cols)
        out = np.empty((xs.shape[0], self.rows), dtype=np.float32)
        _check(lib().rk_matrix_mulvec_many(self.h, xs.shape[0], _ptr(out), _ptr(xs)))
        return out

    def bench(self, iters=20, flush=True, fused=False):
        """Mean kernel time (ms) of one matvec; `fused` quantizes the input
        inside the kernel as the decode step does."""
        ms = C.c_float()
        flags = (RK_BENCH_FLUSH if flush else 0) | (RK_BENCH_FUSED if fused else 0)
        _check(lib().rk_bench_matvec(self.h, iters, flags, C.byref(ms)))
        return ms.value

    def bench_many(self, n, iters=20, flush=True):
        """Mean kernel time (ms) of one batched product with n vectors."""
        ms = C.c_float()
        _check(lib().rk_bench_matvec_many(self.h, n, iters, RK_BENCH_FLUSH if flush else 0, C.byref(ms)))
        return ms.value

    def free(self):
        if self.h:
            lib().rk_matrix_free(self.h)
            self.h = C.c_void_p()


def mulvecs(ms, x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    outs = [np.empty(m.rows, dtype=np.float32) for m in ms]
    hs = (C.c_void_p * len(ms))(*[m.h for m in ms])
    ps = (C.c_void_p * len(ms))(*[o.ctypes.data for o in outs])
    _check(lib().rk_mulvecs(len(ms), hs, ps, _ptr(x)))
    return outs


class Vectors:
    def __init__(self, dev, v):
        v = np.ascontiguousarray(v, dtype=np.float32)
        self.h = C.c_void_p()
        _check(lib().rk_vectors_upload(dev.h, _ptr(v), v.size, C.byref(self.h)))

    def free(self):
        if self.h:
            lib().rk_vectors_free(self.h)
            self.h = C.c_void_p()


class Arena:
    """gpu.Arena (batch.go:12-71)."""

    def __init__(self, dev, words, staging_words):
        self.h = C.c_void_p()
        _check(lib().rk_arena_new(dev.h, words, staging_words, C.byref(self.h)))

    def set_quant_scratch(self, qx_off, xs_off):
        lib().rk_arena_set_quant_scratch(self.h, qx_off, xs_off)

    def begin(self):
        return Batch(self)

    def free(self):
        if self.h:
            lib().rk_arena_free(self.h)
            self.h = C.c_void_p()


class Batch:
    """gpu.Batch (batch.go:113-349); reads land in numpy arrays at submit."""

    def __init__(self, arena):
        self.h = C.c_void_p()
        self._keep = []
        _check(lib().rk_batch_begin(arena.h, C.byref(self.h)))

    def write(self, off, data):
        data = np.ascontiguousarray(data, dtype=np.float32)
        lib().rk_batch_write(self.h, off, _ptr(data), data.size)

    def read(self, off, n):
        dst = np.empty(n, dtype=np.float32)
        self._keep.append(dst)
        lib().rk_batch_read(self.h, off, _ptr(dst), n)
        return dst

    def matvecs(self, ms, out_offs, in_off):
        hs = (C.c_void_p * len(ms))(*[m.h for m in ms])
        offs = (C.c_int64 * len(ms))(*out_offs)
        lib().rk_batch_matvecs(self.h, len(ms), hs, offs, in_off)

    def quantize(self, in_off, n):
        lib().rk_batch_quantize(self.h, in_off, n)

    def rmsnorm(self, vecs, in_off, out_off, w_off, n, segs, stride, recip_n, eps):
        lib().rk_batch_rmsnorm(self.h, vecs.h, in_off, out_off, w_off, n, segs, stride, recip_n, eps)

    def addvec(self, vecs, out_off, v_off, n):
        lib().rk_batch_addvec(self.h, vecs.h, out_off, v_off, n)

    def rope(self, q, k, q_dim, kv_dim, hs, cos_off, sin_off):
        lib().rk_batch_rope(self.h, q, k, q_dim, kv_dim, hs, cos_off, sin_off)

    def copy(self, src, dst, n):
        lib().rk_batch_copy(self.h, src, dst, n)

    def attention(self, q, keys, vals, att, att_stride, out, positions, heads, kv_heads, hs, kv_dim, inv_sqrt):
        lib().rk_batch_attention(self.h, q, keys, vals, att, att_stride, out, positions, heads, kv_heads, hs, kv_dim,
                                 inv_sqrt)

    def residual(self, x, y, n, canonical):
        lib().rk_batch_residual(self.h, x, y, n, 1 if canonical else 0)

    def silumul(self, a, b, n):
        lib().rk_batch_silumul(self.h, a, b, n)

    def submit(self):
        h, self.h = self.h, C.c_void_p()
        _check(lib().rk_batch_submit(h))


def group_id():
    """A fresh group id (bytes) for Group on every rank."""
    buf = (C.c_ubyte * 128)()
    _check(lib().rk_group_id(buf))
    return bytes(buf)


class Group:
    """Rank `rank` of `nranks` GPUs sharing row-sharded stages (NCCL)."""

    def __init__(self, dev, nranks, rank, gid):
        self.h = C.c_void_p()
        self.nranks, self.rank = nranks, rank
        buf = (C.c_ubyte * 128).from_buffer_copy(gid)
        _check(lib().rk_group_new(dev.h, nranks, rank, buf, C.byref(self.h)))

    def all_gather(self, buf_dev_ptr, count):
        _check(lib().rk_group_all_gather(self.h, C.c_void_p(buf_dev_ptr), count))

    def free(self):
        if self.h:
            lib().rk_group_free(self.h)
            self.h = C.c_void_p()


class Layer:
    """llm.Layer on a device (model.go:282-387); shard=(n, r) for rank r's
    rows of n (rk_layer_*_shard)."""

    def __init__(self, dev, cfg, host=None, mats=None, vectors=None, shard=None):
        self.h = C.c_void_p()
        n, r = shard if shard else (1, 0)
        if host is not None:
            hl, keep = host
            self._keep = keep
            _check(lib().rk_layer_upload_shard(dev.h, C.byref(cfg), n, r, C.byref(hl), C.byref(self.h)))
        else:
            hl, keep = vectors
            self._keep = keep
            _check(lib().rk_layer_from_device_shard(dev.h, C.byref(cfg), n, r, C.byref(hl), *[m.h for m in mats],
                                                    C.byref(self.h)))
            for m in mats:
                m.h = C.c_void_p()  # owned by the layer now

    def free(self):
        if self.h:
            lib().rk_layer_free(self.h)
            self.h = C.c_void_p()


class Stage:
    """llm.Stage on a device (model.go:446-613)."""

    def __init__(self, dev, cfg, layers, ctx, group=None, nseq=1):
        hs = (C.c_void_p * max(1, len(layers)))(*[l.h for l in layers])
        self.h = C.c_void_p()
        self.dim = cfg.dim
        if nseq > 1:
            _check(lib().rk_stage_new_batch(dev.h, C.byref(cfg), hs, len(layers), ctx, nseq, C.byref(self.h)))
        elif group is None:
            _check(lib().rk_stage_new(dev.h, C.byref(cfg), hs, len(layers), ctx, C.byref(self.h)))
        else:
            _check(lib().rk_stage_new_group(dev.h, C.byref(cfg), hs, len(layers), ctx, group.h, C.byref(self.h)))

    def positions(self):
        return lib().rk_stage_positions(self.h)

    def fused_gathers(self):
        """1 when a sharded stage exchanges activations by NVLink stores and
        flags inside its kernels, 0 for NCCL all-gathers (or unsharded)."""
        return lib().rk_stage_fused_gathers(self.h)

    def chained(self):
        """1 when the recorded decode step runs each layer's products after
        the attention as one chained launch, 0 for a launch per product."""
        return lib().rk_stage_chained(self.h)

    def forward_batch(self, xs, positions):
        """One decode step of several sequences: row q of xs is sequence q's
        activation at positions[q] (a stage made with nseq > 1)."""
        xs = np.ascontiguousarray(xs, dtype=np.float32).reshape(-1, self.dim).copy()
        pos = np.ascontiguousarray(positions, dtype=np.int32)
        assert pos.size == xs.shape[0]
        _check(lib().rk_stage_forward_batch(self.h, _ptr(xs), _ptr(pos), xs.shape[0]))
        return xs

    def batched(self):
        """1 when forward() of several tokens runs the products batched on
        the tensor cores (an unsharded, all-Q8_0 stage of 128-multiple
        widths), else 0."""
        return lib().rk_stage_batched(self.h)

    def fill_cache(self, positions, seed, first_layer=0):
        """A seeded synthetic context in every layer's caches (positions
        rows); first_layer: the whole model's index of the stage's first
        layer (a pipeline rank's stage), so its caches match that model's."""
        _check(lib().rk_stage_fill_cache_from(self.h, positions, seed, first_layer))

    def forward(self, xs, pos):
        xs = np.ascontiguousarray(xs, dtype=np.float32).copy()
        tokens = xs.size // self.dim
        _check(lib().rk_stage_forward(self.h, _ptr(xs), pos, tokens))
        return xs

    def free(self):
        if self.h:
            lib().rk_stage_free(self.h)
            self.h = C.c_void_p()


class Head:
    def __init__(self, dev, cfg, rms_final, wcls, group=None):
        rms = np.ascontiguousarray(rms_final, dtype=np.float32)
        self.vocab = cfg.vocab
        self.h = C.c_void_p()
        if group is None:
            _check(lib().rk_head_new(dev.h, C.byref(cfg), _ptr(rms), wcls.h, C.byref(self.h)))
        else:
            _check(lib().rk_head_new_group(dev.h, C.byref(cfg), _ptr(rms), wcls.h, group.h, C.byref(self.h)))

    def logits(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty(self.vocab, dtype=np.float32)
        _check(lib().rk_head_logits(self.h, _ptr(x), _ptr(out)))
        return out

    def free(self):
        if self.h:
            lib().rk_head_free(self.h)
            self.h = C.c_void_p()


def sample_argmax(dev, logits):
    """Sampler.Sample at temperature 0 (sample.go:26-53), on the device."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    idx = C.c_int()
    _check(lib().rk_sample_argmax(dev.h, _ptr(logits), logits.size, C.byref(idx)))
    return idx.value


def embed(table, token):
    x = np.empty(table.cols, dtype=np.float32)
    _check(lib().rk_embed(table.h, token, _ptr(x)))
    return x


class Model:
    """Embed -> stage -> head -> greedy sample, all on one device."""

    def __init__(self, dev, embed_table, stage, head, vocab):
        self.vocab = vocab
        self.h = C.c_void_p()
        _check(lib().rk_model_new(dev.h, embed_table.h, stage.h, head.h, C.byref(self.h)))

    def step(self, token, pos, want_logits=True):
        logits = np.empty(self.vocab, dtype=np.float32) if want_logits else None
        nxt = C.c_int()
        _check(lib().rk_model_step(self.h, token, pos, _ptr(logits), C.byref(nxt)))
        return nxt.value, logits

    def generate(self, prompt, n_new, want_logits=False):
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        toks = np.empty(max(n_new, 1), dtype=np.int32)
        steps = prompt.size + n_new - 1
        logits = np.empty((steps, self.vocab), dtype=np.float32) if want_logits else None
        _check(lib().rk_model_generate(self.h, _ptr(prompt), prompt.size, n_new, _ptr(toks), _ptr(logits)))
        return toks[:n_new], logits

    def bench(self, pos, iters):
        ms = C.c_float()
        _check(lib().rk_bench_model(self.h, pos, iters, C.byref(ms)))
        return ms.value

    def profile(self, pos, iters):
        p = Profile()
        _check(lib().rk_model_profile(self.h, pos, iters, C.byref(p)))
        return p

    def kernel_count(self):
        n = C.c_int()
        _check(lib().rk_model_kernel_count(self.h, C.byref(n)))
        return n.value

    def free(self):
        if self.h:
            lib().rk_model_free(self.h)
            self.h = C.c_void_p()


def matmul_bf16(w, x):
    """MatMulBF16 (matvec.go:124-147) with a bfloat16 Matrix w: [n, w.rows]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty((x.shape[0], w.rows), np.float32)
    _check(lib().rk_matmul_bf16(w.h, x.shape[0], _ptr(x), _ptr(out)))
    return out


def measure_speed(dev):
    """MeasureSpeed (speed.go:16-47): GB/s of bfloat16 weights."""
    v = C.c_double()
    _check(lib().rk_measure_speed(dev.h, C.byref(v)))
    return v.value


def _part_buf(part):
    part = bytes(part)
    return C.create_string_buffer(part, len(part)), len(part)


def layer_load_part(dev, cfg, part):
    """LoadLayer (shard.go:258-269) + Layer.toDevice: a Layer from a part's bytes."""
    buf, n = _part_buf(part)
    layer = Layer.__new__(Layer)
    layer.h = C.c_void_p()
    _check(lib().rk_layer_load_part(dev.h, C.byref(cfg), buf, n, C.byref(layer.h)))
    return layer


def embed_load_part(dev, cfg, part, fmt):
    """LoadEmbed (shard.go:282-287): the embedding table as a Matrix."""
    buf, n = _part_buf(part)
    h = C.c_void_p()
    _check(lib().rk_embed_load_part(dev.h, C.byref(cfg), buf, n, C.byref(h)))
    return Matrix(dev, cfg.vocab, cfg.dim, fmt, handle=h)


def head_load_part(dev, cfg, part, embed, fmt):
    """LoadHead (shard.go:292-300): (Head, its own classifier Matrix or None)."""
    buf, n = _part_buf(part)
    h, w = C.c_void_p(), C.c_void_p()
    _check(lib().rk_head_load_part(dev.h, C.byref(cfg), buf, n, embed.h if embed else None, C.byref(w), C.byref(h)))
    head = Head.__new__(Head)
    head.vocab, head.h = cfg.vocab, h
    return head, (Matrix(dev, cfg.vocab, cfg.dim, fmt, handle=w) if w.value else None)


def plan_stages(cost, mem, speed, capacity, stages, free_mem=None):
    """planStages (plan.go:122-207) through rk_plan_stages: a list of
    (node, first layer, end layer) spans."""
    cost = np.ascontiguousarray(cost, dtype=np.int64)
    mem = np.ascontiguousarray(mem, dtype=np.int64)
    speed = np.ascontiguousarray(speed, dtype=np.float64)
    capacity = np.ascontiguousarray(capacity, dtype=np.int64)
    free = None if free_mem is None else np.ascontiguousarray(free_mem, dtype=np.int64)
    room = max(1, len(speed))
    node, first, end = (np.zeros(room, np.int32) for _ in range(3))
    n = C.c_int(room)
    _check(lib().rk_plan_stages(_ptr(cost), _ptr(mem), cost.size, _ptr(speed), _ptr(capacity), _ptr(free), speed.size,
                                stages, C.byref(n), _ptr(node), _ptr(first), _ptr(end)))
    return [(int(node[i]), int(first[i]), int(end[i])) for i in range(n.value)]


class Pipeline:
    """One rank's part of a layer pipeline over a Group: the first rank
    passes the embedding table, the last the head (rk_pipeline_*)."""

    def __init__(self, group, embed_table, stage, head, vocab):
        self.vocab = vocab
        self.last = group.rank == group.nranks - 1
        self.h = C.c_void_p()
        _check(lib().rk_pipeline_new(group.h, embed_table.h if embed_table else None, stage.h,
                                     head.h if head else None, C.byref(self.h)))

    def step(self, token, pos, want_logits=True):
        logits = np.empty(self.vocab, dtype=np.float32) if want_logits and self.last else None
        nxt = C.c_int()
        _check(lib().rk_pipeline_step(self.h, token, pos, _ptr(logits), C.byref(nxt)))
        return nxt.value, logits

    def bench(self, pos, iters):
        ms = C.c_float()
        _check(lib().rk_bench_pipeline(self.h, pos, iters, C.byref(ms)))
        return ms.value

    def free(self):
        if self.h:
            lib().rk_pipeline_free(self.h)
            self.h = C.c_void_p()


def _tdtype(a):
    return {np.dtype(np.float32): TENSOR_F32, np.dtype(np.int8): TENSOR_I8, np.dtype(np.int32): TENSOR_I32}[a.dtype]


def tensor_add(dev, a, b):
    """rakkan_tensor_v1 add: a [rows, cols] + b [rows or 1, cols]."""
    a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
    c = np.empty_like(a)
    _check(lib().rk_tensor_add(dev.h, _tdtype(a), a.shape[0], a.shape[1], _ptr(a), _ptr(b), b.shape[0], _ptr(c)))
    return c


def tensor_scale(dev, a, k):
    a = np.ascontiguousarray(a)
    c = np.empty(a.shape, np.float32)
    _check(lib().rk_tensor_scale(dev.h, _tdtype(a), a.shape[0], a.shape[1], _ptr(a), k, _ptr(c)))
    return c


def tensor_relu(dev, a):
    a = np.ascontiguousarray(a)
    c = np.empty_like(a)
    _check(lib().rk_tensor_relu(dev.h, _tdtype(a), a.shape[0], a.shape[1], _ptr(a), _ptr(c)))
    return c


def tensor_softmax(dev, a):
    a = np.ascontiguousarray(a)
    c = np.empty(a.shape, np.float32)
    _check(lib().rk_tensor_softmax(dev.h, _tdtype(a), a.shape[0], a.shape[1], _ptr(a), _ptr(c)))
    return c


def tensor_quantize(dev, a, k):
    a = np.ascontiguousarray(a)
    c = np.empty(a.shape, np.int8)
    _check(lib().rk_tensor_quantize(dev.h, _tdtype(a), a.shape[0], a.shape[1], _ptr(a), k, _ptr(c)))
    return c


def tensor_argmax(dev, a):
    a = np.ascontiguousarray(a)
    out = np.empty(a.shape[0], np.int32)
    _check(lib().rk_tensor_argmax(dev.h, _tdtype(a), a.shape[0], a.shape[1], _ptr(a), _ptr(out)))
    return out


def tensor_matmul(dev, a, b, transposed):
    """rakkan_tensor_v1 matmul (transposed=False) / matmul_t (True)."""
    if a.dtype == np.float32 and b.dtype == np.float32:
        dt, out_t = TENSOR_F32, np.float32
    elif a.dtype == np.int8 and b.dtype == np.int8:
        dt, out_t = TENSOR_I8, np.int32
    elif a.dtype == np.int32 and b.dtype == np.int32:
        dt, out_t = TENSOR_I32, np.int32
    else:
        raise RkError(RK_ERR_ARGS, "dtype mismatch")
    m, k = a.shape
    n = b.shape[0] if transposed else b.shape[1]
    kb = b.shape[1] if transposed else b.shape[0]
    if kb != k:
        raise RkError(RK_ERR_ARGS, "shape mismatch")
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    c = np.empty((m, n), dtype=out_t)
    _check(lib().rk_tensor_matmul(dev.h, dt, 1 if transposed else 0, m, k, n, _ptr(a), _ptr(b), _ptr(c)))
    return c


def bench_tensor(dev, dtype, transposed, m, k, n, iters=20, flush=True):
    """Mean device time (ms) of one tensor matmul on device-resident inputs."""
    ms = C.c_float()
    _check(lib().rk_bench_tensor(dev.h, dtype, 1 if transposed else 0, m, k, n, iters,
                                 RK_BENCH_FLUSH if flush else 0, C.byref(ms)))
    return ms.value


def generate_normal(dev, seed, tid, offset, n, scale):
    out = np.empty(n, dtype=np.float32)
    _check(lib().rk_generate_normal(dev.h, seed, tid, offset, n, scale, _ptr(out)))
    return out


def quantize(dev, fmt, w):
    w = np.ascontiguousarray(w, dtype=np.float32)
    q = np.empty(w.size if fmt == FMT_Q8_0 else w.size // 2, dtype=np.int8 if fmt == FMT_Q8_0 else np.uint8)
    s = np.empty(w.size // 32, dtype=np.float32)
    _check(lib().rk_quantize(dev.h, fmt, _ptr(w), w.size, _ptr(q), _ptr(s)))
    return q, s


class Tensors:
    """rakkan_tensor_v1's tensor table on a device (rk_tensors_*): handles of
    device-resident tensors; the calls return a handle, or raise RkError
    with the reference's error code (RK_ERR_ARGS / TOO_BIG / BLOB)."""

    DTYPES = {np.dtype(np.float32): TENSOR_F32, np.dtype(np.int8): TENSOR_I8, np.dtype(np.int32): TENSOR_I32}
    NP = {TENSOR_F32: np.float32, TENSOR_I8: np.int8, TENSOR_I32: np.int32}

    def __init__(self, dev, budget):
        self.dev = dev
        self.h = C.c_void_p()
        _check(lib().rk_tensors_new(dev.h, budget, C.byref(self.h)))

    @staticmethod
    def _h(rc):
        if rc < 0:
            raise RkError(rc, lib().rk_last_error().decode())
        return rc

    def from_memory(self, a):
        a = np.ascontiguousarray(a)
        rows, cols = a.shape if a.ndim == 2 else (1, a.size)
        return self._h(lib().rk_tensors_from_memory(self.h, _ptr(a), self.DTYPES[a.dtype], rows, cols))

    def from_blob(self, blob, offset, dtype, rows, cols):
        blob = np.frombuffer(bytes(blob), np.uint8) if not isinstance(blob, np.ndarray) else blob
        return self._h(lib().rk_tensors_from_blob(self.h, _ptr(blob), blob.nbytes, offset, dtype, rows, cols))

    def dims(self, t):
        return tuple(self._h(lib().rk_tensors_dim(self.h, t, w)) for w in range(3))

    def to_numpy(self, t):
        rows, cols, dt = self.dims(t)
        out = np.empty((rows, cols), self.NP[dt])
        got = lib().rk_tensors_to_memory(self.h, t, _ptr(out), out.nbytes)
        self._h(got)
        assert got == out.nbytes
        return out

    def matmul(self, a, b, transposed=False):
        return self._h(lib().rk_tensors_matmul(self.h, a, b, 1 if transposed else 0))

    def add(self, a, b):
        return self._h(lib().rk_tensors_add(self.h, a, b))

    def scale(self, a, k):
        return self._h(lib().rk_tensors_scale(self.h, a, k))

    def relu(self, a):
        return self._h(lib().rk_tensors_relu(self.h, a))

    def softmax(self, a):
        return self._h(lib().rk_tensors_softmax(self.h, a))

    def quantize(self, a, k):
        return self._h(lib().rk_tensors_quantize(self.h, a, k))

    def argmax(self, a):
        rows = self.dims(a)[0]
        out = np.empty(rows, np.int32)
        self._h(lib().rk_tensors_argmax(self.h, a, _ptr(out), out.nbytes))
        return out

    def release(self, t):
        self._h(lib().rk_tensors_release(self.h, t))

    def used(self):
        return lib().rk_tensors_used(self.h)

    def free(self):
        if self.h:
            lib().rk_tensors_free(self.h)
            self.h = C.c_void_p()
