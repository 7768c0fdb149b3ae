"""Placeholder for jax.experimental.pallas.tpu (see pallas/__init__.py)."""


def __getattr__(name):
    raise AttributeError(f"pallas.tpu.{name} is not provided by the numpy stand-in")
