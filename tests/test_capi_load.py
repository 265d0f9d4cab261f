"""The C-ABI library loads and exports every symbol include/rakkan_cuda.h
declares (CPU only: no compute calls)."""
import ctypes as C
import os
import re

import rkcuda as rk

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "rakkan_cuda.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(rk_[a-z0-9_]+)\s*\(", src)))


def test_header_declarations_are_exported():
    lib = C.CDLL(rk.LIB_PATH)
    names = declared_symbols()
    assert len(names) > 50
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_the_header():
    assert sorted(rk.EXPORTS) == declared_symbols()


def test_error_string_and_version_without_gpu():
    L = rk.lib()
    assert L.rk_version().startswith(b"rakkan-cuda")
    assert isinstance(L.rk_last_error(), bytes)
    # Argument checks fail before touching a device.
    assert L.rk_tensor_matmul(None, rk.TENSOR_F32, 0, 1, 1, 1, None, None, None) == rk.RK_ERR_ARGS
    assert L.rk_config_validate(None) == rk.RK_ERR_ARGS


def test_device_count_without_gpu_is_zero_or_more():
    n = C.c_int(-1)
    assert rk.lib().rk_device_count(C.byref(n)) == rk.RK_OK
    assert n.value >= 0


def test_batched_entry_points_check_arguments_without_gpu():
    """The batched prefill / batched decode entry points refuse bad
    arguments before they touch a device."""
    L = rk.lib()
    assert L.rk_matrix_mulvec_many(None, 4, None, None) == rk.RK_ERR_ARGS
    assert L.rk_bench_matvec_many(None, 4, 1, 0, None) == rk.RK_ERR_ARGS
    assert L.rk_stage_batched(None) == 0
    out = C.c_void_p()
    assert L.rk_stage_new_batch(None, None, None, 0, 16, 0, C.byref(out)) == rk.RK_ERR_ARGS
    assert L.rk_stage_new_batch(None, None, None, 0, 16, 4, C.byref(out)) == rk.RK_ERR_ARGS
    assert L.rk_stage_forward_batch(None, None, None, 2) == rk.RK_ERR_ARGS
    assert b"argument" in L.rk_last_error() or b"sequence" in L.rk_last_error()
