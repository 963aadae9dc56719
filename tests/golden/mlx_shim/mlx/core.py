"""Minimal ``mlx.core`` API on NumPy for running the reference's CPU path.

Only the operations that ``mlx_foveated.py``, ``turbo_quantize.py`` and
``turbo_constants.py`` call are provided.  MLX and NumPy 2 share the relevant
semantics: Python scalars are weakly typed, ``round`` is half-to-even, and
float->int casts truncate.  ``fast.scaled_dot_product_attention`` is NOT
MLX's kernel: it is a float32 softmax attention written here, so outputs of
``attend`` produced through it pin the reference's dequant/concat/GQA logic,
not MLX's SDPA arithmetic.
"""
import numpy as np

float16 = np.float16
float32 = np.float32
bfloat16 = np.float32
uint8 = np.uint8
uint16 = np.uint16
uint32 = np.uint32
int32 = np.int32
int64 = np.int64
bool_ = np.bool_


class _ArrayMeta(type):
    def __instancecheck__(cls, obj):
        return isinstance(obj, np.ndarray)


class array(metaclass=_ArrayMeta):
    """``mx.array(x, dtype)`` builds a numpy array; isinstance checks see ndarrays."""

    def __new__(cls, x, dtype=None):
        return np.array(x, dtype=dtype)


def eval(*args):
    return None


def where(c, a, b):
    return np.where(c, a, b)


def zeros_like(x):
    return np.zeros_like(x)


def ones_like(x):
    return np.ones_like(x)


def zeros(shape, dtype=np.float32):
    return np.zeros(shape, dtype=dtype)


def full(shape, val, dtype=None):
    return np.full(shape, val, dtype=dtype)


def arange(*a, dtype=None):
    return np.arange(*a, dtype=dtype if dtype is not None else np.int32)


def concatenate(xs, axis=0):
    return np.concatenate(xs, axis=axis)


def stack(xs, axis=0):
    return np.stack(xs, axis=axis)


def broadcast_to(x, shape):
    return np.broadcast_to(x, shape)


def take_along_axis(x, idx, axis):
    return np.take_along_axis(x, idx.astype(np.int64), axis=axis)


def expand_dims(x, axis):
    return np.expand_dims(x, axis)


def squeeze(x, axis=None):
    return np.squeeze(x, axis=axis)


def min(x, axis=None, keepdims=False):
    return np.min(x, axis=axis, keepdims=keepdims)


def max(x, axis=None, keepdims=False):
    return np.max(x, axis=axis, keepdims=keepdims)


def sum(x, axis=None, keepdims=False):
    return np.sum(x, axis=axis, keepdims=keepdims, dtype=x.dtype if x.dtype.kind == "f" else None)


def mean(x, axis=None, keepdims=False):
    return np.mean(x, axis=axis, keepdims=keepdims, dtype=x.dtype)


def sqrt(x):
    return np.sqrt(x)


def maximum(a, b):
    return np.maximum(a, b)


def clip(x, lo, hi):
    return np.clip(x, lo, hi)


def round(x, decimals=0):
    return np.round(x, decimals)


def abs(x):
    return np.abs(x)


def repeat(x, n, axis):
    return np.repeat(x, n, axis=axis)


def any(x):
    return np.any(x)


def all(x):
    return np.all(x)


def argmax(x, axis=None):
    return np.argmax(x, axis=axis)


def array_equal(a, b):
    return np.array_equal(a, b)


def allclose(a, b, rtol=1e-5, atol=1e-8):
    return np.allclose(a, b, rtol=rtol, atol=atol)


def logsumexp(x, axis=None, keepdims=False):
    m = np.max(x, axis=axis, keepdims=True)
    r = m + np.log(np.sum(np.exp(x - m), axis=axis, keepdims=True))
    return r if keepdims else np.squeeze(r, axis=axis)


class _Fast:
    @staticmethod
    def scaled_dot_product_attention(q, k, v, *, scale, mask=None, **kw):
        qf = q.astype(np.float32)
        s = np.einsum("bhqd,bhkd->bhqk", qf, k.astype(np.float32)) * np.float32(scale)
        s = s - s.max(axis=-1, keepdims=True)
        p = np.exp(s)
        p = p / p.sum(axis=-1, keepdims=True)
        return np.einsum("bhqk,bhkd->bhqd", p, v.astype(np.float32)).astype(q.dtype)


fast = _Fast()
