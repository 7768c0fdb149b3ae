"""Placeholder for jax.experimental.pallas: the reference modules import it at
module level but the jnp reference functions never call it."""
from . import tpu  # noqa: F401


def __getattr__(name):
    raise AttributeError(f"pallas.{name} is not provided by the numpy stand-in")
