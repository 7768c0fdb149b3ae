"""numpy stand-in for the `jax` names the reference's jnp GLA code uses
(test infrastructure: only tests/golden/make_ref_golden.py imports it, to run
the reference's jnp code unchanged where JAX is not installed)."""
import numpy as _np

from . import lax, numpy  # noqa: F401
from . import experimental  # noqa: F401
from . import random  # noqa: F401

Array = _np.ndarray


def jit(fn=None, **_kw):
    """Identity: the stand-in runs everything eagerly."""
    if fn is None:
        return lambda f: f
    return fn


def devices():
    return []


def default_backend():
    return "cpu"
