import ml_dtypes
import numpy as np

from oracle import affine as _aff


def swiglu(gate, x):
    g = np.asarray(gate, dtype=np.float32)
    u = np.asarray(x, dtype=np.float32)
    return _aff.swiglu(g, u).astype(ml_dtypes.bfloat16)
