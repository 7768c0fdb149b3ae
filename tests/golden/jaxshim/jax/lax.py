"""numpy stand-in for the jax.lax names the reference's jnp GLA code uses:
Precision, dot_general, scan, iota."""
import string

import numpy as _np

from . import numpy as _jnp


class Precision:
    DEFAULT = "default"
    HIGH = "high"
    HIGHEST = "highest"


def dot_general(lhs, rhs, dimension_numbers, precision=None, preferred_element_type=None):
    """General contraction: output dims are the batch dims (in lhs order),
    then lhs's free dims, then rhs's free dims, as in jax.lax.dot_general."""
    (lc, rc), (lb, rb) = dimension_numbers
    lhs, rhs = _np.asarray(lhs), _np.asarray(rhs)
    letters = iter(string.ascii_letters)
    ls = [next(letters) for _ in range(lhs.ndim)]
    rs = [None] * rhs.ndim
    for a, b in zip(lc, rc):
        rs[b] = ls[a]
    for a, b in zip(lb, rb):
        rs[b] = ls[a]
    for i in range(rhs.ndim):
        if rs[i] is None:
            rs[i] = next(letters)
    batch = [ls[a] for a in lb]
    lfree = [ls[i] for i in range(lhs.ndim) if i not in lc and i not in lb]
    rfree = [rs[i] for i in range(rhs.ndim) if i not in rc and i not in rb]
    sub = "".join(ls) + "," + "".join(rs) + "->" + "".join(batch + lfree + rfree)
    return _jnp.contract(sub, (lhs, rhs), preferred_element_type)


def _leaves(tree):
    if tree is None:
        return [], lambda leaves: None
    if isinstance(tree, (tuple, list)):
        parts = [_leaves(t) for t in tree]
        counts = [len(p[0]) for p in parts]

        def rebuild(leaves, parts=parts, counts=counts, kind=type(tree)):
            out, i = [], 0
            for (_, rb), c in zip(parts, counts):
                out.append(rb(leaves[i:i + c]))
                i += c
            return kind(out)
        return [l for p in parts for l in p[0]], rebuild
    return [tree], lambda leaves: leaves[0]


def scan(f, init, xs, length=None, reverse=False, unroll=1):
    """carry, ys = scan(f, init, xs): the sequential loop over xs's leading
    axis; ys are stacked in xs's order (also when reverse=True)."""
    leaves, rebuild = _leaves(xs)
    n = length if length is not None else len(leaves[0])
    order = range(n - 1, -1, -1) if reverse else range(n)
    carry, ys = init, [None] * n
    for i in order:
        carry, y = f(carry, rebuild([l[i] for l in leaves]))
        ys[i] = y
    yl0, yrebuild = _leaves(ys[0])
    stacked = [_np.stack([_leaves(y)[0][j] for y in ys]) for j in range(len(yl0))]
    return carry, yrebuild(stacked)


def iota(dtype, size):
    return _np.arange(size, dtype=dtype)
