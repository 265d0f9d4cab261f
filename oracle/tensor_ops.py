"""CPU restatement of rakkan_tensor_v1's element and row operations
(internal/sandbox/tensor.go:341-476). Test infrastructure only: the tests
pin it against the reference's own cases (tensor_test.go:97-143) and check
the library's rk_tensor_* against it; nothing in the library calls it.

float32 arithmetic is numpy's, one IEEE rounding per operation as Go's
float32 operations are; Exp32 is the C oracle's (num.go:76-97).
"""
import numpy as np

import rk_oracle

CANON_NAN = np.uint32(0x7FC00000).view(np.float32)


def canonical(x):
    """num.Canonical: every NaN becomes 0x7fc00000."""
    x = np.array(x, dtype=np.float32, copy=True)
    x[np.isnan(x)] = CANON_NAN
    return x


def add(a, b):  # tensor.go:341-363
    if b.shape[0] == 1 and a.shape[0] != 1:
        b = np.broadcast_to(b, a.shape)
    if a.dtype == np.float32:
        return canonical(a + b)
    with np.errstate(over="ignore"):
        return (a.astype(np.int64) + b.astype(np.int64)).astype(np.uint32).view(np.int32)  # int32 wraps


def scale(a, k):  # tensor.go:365-383
    v = a.astype(np.float32)  # float32(int32) rounds to nearest even
    return canonical(v * np.float32(k))


def relu(a):  # tensor.go:385-406
    if a.dtype == np.float32:
        out = np.zeros_like(a)
        pos = a > 0
        out[pos] = a[pos]
        out[np.isnan(a)] = CANON_NAN
        return out
    return np.where(a > 0, a, 0).astype(np.int32)


def softmax(a):  # tensor.go:408-433
    exp32 = rk_oracle.lib().rko_exp32
    out = np.empty_like(a)
    for r in range(a.shape[0]):
        row = a[r]
        mx = row[0]
        for v in row[1:]:
            if v > mx:
                mx = v
        s = np.float32(0)
        for i, v in enumerate(row):
            out[r, i] = exp32(float(np.float32(v - mx)))
            s = np.float32(s + out[r, i])
        out[r] = canonical(out[r] / s)
    return out


def quantize(a, k):  # tensor.go:435-450
    with np.errstate(invalid="ignore", over="ignore", divide="ignore"):
        q = np.rint(a / np.float32(k))  # float32 division, then RoundToEven
        out = np.zeros(a.shape, np.int8)
        ok = ~np.isnan(q)  # Go's int8(NaN) is 0 on amd64
        out[ok] = np.clip(q[ok], -127, 127).astype(np.int8)
    return out


def argmax(a):  # tensor.go:452-476
    out = np.zeros(a.shape[0], np.int32)
    for r in range(a.shape[0]):
        best = 0
        for j in range(1, a.shape[1]):
            if a[r, j] > a[r, best]:
                best = j
        out[r] = best
    return out
