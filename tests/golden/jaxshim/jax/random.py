"""Placeholder: the golden generator draws its inputs with torch, never with
jax.random (JAX's PRNG streams are not reproduced)."""


def __getattr__(name):
    raise AttributeError(f"jax.random.{name} is not provided by the numpy stand-in")
