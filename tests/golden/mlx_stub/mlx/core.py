"""Numpy-backed stub of the parts of mlx.core the reference touches."""
import ml_dtypes
import numpy as np

from oracle import affine as _aff

uint32 = np.uint32
uint16 = np.uint16
bfloat16 = ml_dtypes.bfloat16
float16 = np.float16
float32 = np.float32
array = np.ndarray


def _array(x, dtype=None):
    return np.array(x, dtype=dtype)


globals()["array"] = _array


def zeros(shape, dtype=np.float32):
    return np.zeros(shape, dtype=dtype)


def eval(*args, **kw):  # noqa: A001 - mirrors mx.eval
    return None


def async_eval(*args, **kw):
    return None


def expand_dims(a, axis):
    return np.expand_dims(a, axis)


def take(a, idx, axis=None):
    return np.take(a, np.asarray(idx).astype(np.int64), axis=axis)


def concatenate(xs, axis=0):
    return np.concatenate(xs, axis=axis)


def stack(xs, axis=0):
    return np.stack(xs, axis=axis)


def argpartition(a, kth, axis=-1):
    return np.argpartition(a, kth, axis=axis)


def take_along_axis(a, idx, axis):
    return np.take_along_axis(a, np.asarray(idx).astype(np.int64), axis=axis)


def gather_qmm(x, w, scales, biases, rhs_indices=None, transpose=True,
               group_size=64, bits=4, mode="affine"):
    assert transpose and mode == "affine"
    x = np.asarray(x)
    idx = np.asarray(rhs_indices).astype(np.int64)
    batch = np.broadcast_shapes(x.shape[:-2], idx.shape)
    xb = np.broadcast_to(x, batch + x.shape[-2:])
    ib = np.broadcast_to(idx, batch)
    out = np.zeros(batch + (x.shape[-2], w.shape[-2]), dtype=np.float32)
    cache = {}
    s16 = np.asarray(scales).view(np.uint16)
    b16 = np.asarray(biases).view(np.uint16)
    for pos in np.ndindex(*batch):
        e = int(ib[pos])
        if e not in cache:
            cache[e] = _aff.dequant(w[e], s16[e], b16[e], bits, group_size)
        xs = np.asarray(xb[pos], dtype=np.float32)
        out[pos] = _aff.qmv(xs, cache[e])
    return out.astype(ml_dtypes.bfloat16)
