"""CPU oracle for the chunked Gated Linear Attention forward (numpy, fp32).

TEST INFRASTRUCTURE ONLY.  Imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / reference arm as the checker; never by the product
path (glaucis_b200/).

What it restates (fp32 throughout, the reference's Precision.HIGHEST):
  * g_cumsum: per-head constant gate g_gamma -> g_gamma * (1..C) within each
    chunk (KE/examples/kernels/chunk_gla_ref.py:109-111); per-key gate g ->
    chunk-local cumsum of g (gk semantics of
    KE/upstream/fused_chunk_simple_gla/common_chunk_h.py:385-387, :330-334).
  * state scan: h_0 = h0 (or 0), state stored BEFORE each chunk's update,
    h <- h * e^{G_last} + (k * e^{G_last - G})^T v (chunk_gla_ref.py:23-55,
    common_chunk_h.py:275-360 gk branch :330-334, h0 :348-350, ht :356-358).
  * intra-chunk A = (q e^G)(k e^-G)^T * scale (chunk_gla_ref.py:58-77).
  * o = scale (q e^G) h_n + tril(A) v, mask including the diagonal
    (chunk_gla_ref.py:80-99).
A second, independent restatement (`naive_recurrence`) runs the token-level
recurrence S_t = diag(e^{g_t}) S_{t-1} + k_t^T v_t, o_t = scale q_t S_t; the
tests pin the chunked oracle against it.

Parity status: UNPINNED against the reference itself: JAX is not installed
here, so chunk_gla_ref.py cannot be executed and the reference holds no golden
vectors.  Pinned instead against the naive recurrence (an exact algebraic
identity), the g_gamma <-> per-key-gate equivalence, the reference's CPU smoke
shape/finiteness checks (KE/tests/test_chunk_gla.py:81-95) and committed
fixtures in tests/golden/.
"""
from __future__ import annotations

import numpy as np


def g_cumsum_from(g: np.ndarray | None, g_gamma: np.ndarray | None, B: int, T: int, H: int,
                  K: int, C: int) -> np.ndarray:
    NT = T // C
    if g_gamma is not None:
        pos = np.tile(np.arange(1, C + 1, dtype=np.float32), NT).reshape(1, T, 1, 1)
        return np.broadcast_to(np.asarray(g_gamma, np.float32).reshape(1, 1, H, 1) * pos,
                               (B, T, H, K)).astype(np.float32)
    gc = np.asarray(g, np.float32).reshape(B, NT, C, H, K)
    return np.cumsum(gc, axis=2, dtype=np.float32).reshape(B, T, H, K)


def chunk_gla_fwd(q, k, v, g=None, g_gamma=None, h0=None, scale=None, chunk_size=64,
                  return_states=False):
    """Returns (o fp32 [B,T,H,V], ht fp32 [B,H,K,V]) (+ h_all [B,NT,H,K,V])."""
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    v = np.asarray(v, np.float32)
    B, T, H, K = q.shape
    V = v.shape[-1]
    C = chunk_size
    NT = T // C
    if scale is None:
        scale = K ** -0.5
    scale = np.float32(scale)
    gcs = g_cumsum_from(g, g_gamma, B, T, H, K, C)

    qc = q.reshape(B, NT, C, H, K)
    kc = k.reshape(B, NT, C, H, K)
    vc = v.reshape(B, NT, C, H, V)
    gc = gcs.reshape(B, NT, C, H, K)

    # state scan (states before each chunk)
    h = np.zeros((B, H, K, V), np.float32) if h0 is None else np.asarray(h0, np.float32).copy()
    h_all = np.empty((B, NT, H, K, V), np.float32)
    for n in range(NT):
        h_all[:, n] = h
        glast = gc[:, n, -1]                                          # [B,H,K]
        kd = kc[:, n] * np.exp(glast[:, None] - gc[:, n])             # [B,C,H,K]
        h = h * np.exp(glast)[..., None] + np.einsum("bchk,bchv->bhkv", kd, vc[:, n])
    ht = h

    # intra-chunk attention and output
    qg = qc * np.exp(gc)
    kg = kc * np.exp(-gc)
    A = np.einsum("bnihk,bnjhk->bnhij", qg, kg) * scale                # [B,NT,H,C,C]
    A = A * np.tril(np.ones((C, C), np.float32))
    o_inter = scale * np.einsum("bnchk,bnhkv->bnchv", qg, h_all)
    o_intra = np.einsum("bnhij,bnjhv->bnihv", A, vc)
    o = (o_inter + o_intra).reshape(B, T, H, V).astype(np.float32)
    if return_states:
        return o, ht, h_all
    return o, ht


def chunk_gla_fwd_intermediates(q, k, g=None, g_gamma=None, scale=None, chunk_size=64):
    """The first two outputs of the reference's chunk_gla_fwd: g_cumsum fp32
    [B,T,H,K] and the intra-chunk A = (q e^G)(k e^-G)^T * scale fp32 [B,T,H,C]
    over the full C x C square (the causal mask is applied only when o is
    formed), chunk_gla_ref.py:58-77, :102-117."""
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    B, T, H, K = q.shape
    C = chunk_size
    NT = T // C
    if scale is None:
        scale = K ** -0.5
    gcs = g_cumsum_from(g, g_gamma, B, T, H, K, C)
    gc = gcs.reshape(B, NT, C, H, K)
    qg = q.reshape(B, NT, C, H, K) * np.exp(gc)
    kg = k.reshape(B, NT, C, H, K) * np.exp(-gc)
    A = np.einsum("bnihk,bnjhk->bnihj", qg, kg) * np.float32(scale)
    return gcs, A.reshape(B, T, H, C).astype(np.float32)


def naive_recurrence(q, k, v, g=None, g_gamma=None, h0=None, scale=None, chunk_size=64):
    """Token-level recurrence in float64 (small sizes only).  The per-head
    gate contributes g_gamma per token; the per-key gate g[t] per token."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    B, T, H, K = q.shape
    V = v.shape[-1]
    if scale is None:
        scale = K ** -0.5
    if g_gamma is not None:
        gt = np.broadcast_to(np.asarray(g_gamma, np.float64).reshape(1, 1, H, 1), (B, T, H, K))
    else:
        gt = np.asarray(g, np.float64)
    S = np.zeros((B, H, K, V)) if h0 is None else np.asarray(h0, np.float64).copy()
    o = np.empty((B, T, H, V))
    for t in range(T):
        S = S * np.exp(gt[:, t])[..., None] + k[:, t, :, :, None] * v[:, t, :, None, :]
        o[:, t] = scale * np.einsum("bhk,bhkv->bhv", q[:, t], S)
    return o, S
