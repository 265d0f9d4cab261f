"""Test configuration: the `gpu` marker, import paths, shared fixtures.

`-m "not gpu"` runs on any host: the CPU oracle against the reference's
known answers, host logic, and that the CUDA library loads and exports its
C ABI. `-m gpu` needs a B200: parity of the CUDA kernels with the oracle.
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "rakkan-mesh_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def dev():
    import rkcuda as rk
    if rk.device_count() == 0:
        raise RuntimeError("no CUDA device: the gpu tests need a B200")
    d = rk.Device(0)
    yield d
    d.close()


def same_bits(got, want):
    """Bit equality of float32 arrays, counting any two NaNs as equal (NaN
    payloads are not part of the reference's cross-architecture contract;
    it canonicalises them where results leave a computation)."""
    got = np.ascontiguousarray(got, dtype=np.float32)
    want = np.ascontiguousarray(want, dtype=np.float32)
    assert got.shape == want.shape, (got.shape, want.shape)
    gb, wb = got.view(np.uint32), want.view(np.uint32)
    bad = (gb != wb) & ~(np.isnan(got) & np.isnan(want))
    if bad.any():
        i = int(np.flatnonzero(bad)[0])
        raise AssertionError(f"{int(bad.sum())} of {got.size} differ; first at {i}: got {got.flat[i]!r} "
                             f"(0x{int(gb.flat[i]):08x}), want {want.flat[i]!r} (0x{int(wb.flat[i]):08x})")


def awkward(rng, n, scale):
    """Normal values plus the cases that tell exact arithmetic apart, in the
    proportions of the reference's `awkward` (internal/gpu/gpu_test.go:35-48):
    1/40 each denormals, -0, 1e-30."""
    v = (rng.standard_normal(n) * scale).astype(np.float32)
    k = rng.integers(0, 40, n)
    den = rng.integers(0, 1 << 23, n, dtype=np.uint32).view(np.float32)
    v[k == 0] = den[k == 0]
    v[k == 1] = np.float32(-0.0)
    v[k == 2] = np.float32(1e-30)
    return v
