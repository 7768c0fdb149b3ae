"""numpy stand-in for jax.numpy.  Elementwise functions are
numpy's own; contractions run in float64 and are rounded to the JAX result
type (float32 unless every operand is bfloat16)."""
import ml_dtypes as _ml
import numpy as _np
from numpy import *  # noqa: F401,F403  (elementwise maths, shapes, creation)

bfloat16 = _ml.bfloat16
float32 = _np.float32
int32 = _np.int32
bool_ = _np.bool_
ndarray = _np.ndarray


def _jax_float_result(*arrays):
    """JAX's float promotion with 64-bit types disabled: bf16 with bf16 stays
    bf16, anything with a 32- or 64-bit float is float32."""
    dts = {_np.dtype(a.dtype) for a in arrays}
    if dts == {_np.dtype(bfloat16)}:
        return bfloat16
    return _np.float32


def contract(subscripts, operands, preferred_element_type=None):
    ops = [_np.asarray(o) for o in operands]
    out = preferred_element_type or _jax_float_result(*ops)
    r = _np.einsum(subscripts, *[o.astype(_np.float64) for o in ops], optimize=True)
    return _np.asarray(r).astype(out)


def einsum(subscripts, *operands, precision=None, preferred_element_type=None, **_kw):
    """jnp.einsum: a full-precision contraction (JAX on CPU computes fp32
    contractions at fp32 for every `precision`)."""
    return contract(subscripts, operands, preferred_element_type)


def dot(a, b, precision=None, preferred_element_type=None):
    a, b = _np.asarray(a), _np.asarray(b)
    if a.ndim != 2 or b.ndim != 2:
        raise NotImplementedError("the stand-in's jnp.dot covers 2-D operands only")
    return contract("ij,jk->ik", (a, b), preferred_element_type)


def arange(*args, dtype=None, **kw):
    r = _np.arange(*args, dtype=dtype, **kw)
    if dtype is None and r.dtype == _np.int64:
        r = r.astype(_np.int32)
    return r
