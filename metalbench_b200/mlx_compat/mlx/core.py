"""``mlx.core`` subset on numpy (see package docstring)."""
from __future__ import annotations

import numpy as np

float32 = np.float32
float16 = np.float16
int32 = np.int32
uint32 = np.uint32
array_t = np.ndarray


def array(x, dtype=None):
    return np.asarray(x, dtype=dtype if dtype is not None else np.float32)


def eval(*xs):  # MLX is lazy; numpy is eager, nothing to do.
    return None


def synchronize(*_a, **_k):
    return None


def matmul(a, b):
    return np.matmul(a, b)


def transpose(a, axes=None):
    """MLX default reverses all axes, like numpy. The result is materialised
    (a contiguous copy) so a timed reference call does the data movement."""
    return np.ascontiguousarray(np.transpose(a, axes))


def mean(a, axis=None, keepdims=False):
    return np.mean(a, axis=axis, keepdims=keepdims, dtype=a.dtype)


def var(a, axis=None, keepdims=False, ddof=0):
    return np.var(a, axis=axis, keepdims=keepdims, ddof=ddof, dtype=a.dtype)


def rsqrt(a):
    return (1.0 / np.sqrt(a)).astype(np.asarray(a).dtype)


def sqrt(a):
    return np.sqrt(a)


def cos(a):
    return np.cos(a)


def sin(a):
    return np.sin(a)


def exp(a):
    return np.exp(a)


def arange(*args, dtype=None):
    return np.arange(*args, dtype=dtype if dtype is not None else np.int32)


def stack(arrays, axis=0):
    return np.stack(arrays, axis=axis)


def concatenate(arrays, axis=0):
    return np.concatenate(arrays, axis=axis)


def repeat(a, repeats, axis=None):
    """Each element repeated ``repeats`` times consecutively (like numpy)."""
    return np.repeat(a, repeats, axis=axis)


def softmax(a, axis=-1):
    m = np.max(a, axis=axis, keepdims=True)
    e = np.exp(a - m)
    return e / np.sum(e, axis=axis, keepdims=True)


def conv2d(x, w, stride=1, padding=0, dilation=1, groups=1):
    """NHWC input, OHWI weight, cross-correlation (MLX convention)."""
    assert dilation == 1 and groups == 1, "shim supports dilation=1, groups=1"
    N, H, W, C = x.shape
    Co, KH, KW, _ = w.shape
    xp = np.pad(x, ((0, 0), (padding, padding), (padding, padding), (0, 0)))
    H2 = (H + 2 * padding - KH) // stride + 1
    W2 = (W + 2 * padding - KW) // stride + 1
    out = np.zeros((N, H2, W2, Co), dtype=x.dtype)
    for r in range(KH):
        for s in range(KW):
            p = xp[:, r:r + stride * (H2 - 1) + 1:stride, s:s + stride * (W2 - 1) + 1:stride, :]
            out += np.einsum("nhwc,oc->nhwo", p, w[:, r, s, :])
    return out


class _Random:
    """Seeded normal generator. MLX's own RNG stream is not reproduced: both
    sides of every comparison consume the same bytes instead."""

    def __init__(self):
        self._rng = np.random.default_rng(0)

    def seed(self, s):
        self._rng = np.random.default_rng(int(s))

    def normal(self, shape, dtype=np.float32):
        return self._rng.standard_normal(shape).astype(dtype)

    def uniform(self, low=0.0, high=1.0, shape=(), dtype=np.float32):
        return self._rng.uniform(low, high, shape).astype(dtype)


random = _Random()


def swapaxes(a, axis1, axis2):
    """Materialised like ``transpose``."""
    return np.ascontiguousarray(np.swapaxes(a, axis1, axis2))


def where(cond, x, y):
    return np.where(cond, x, y)


def maximum(a, b):
    return np.maximum(a, b)


def astype(a, dtype):
    return np.asarray(a).astype(dtype)
