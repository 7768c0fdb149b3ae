"""CPU oracle for the backward of the chunked GLA forward.

TEST INFRASTRUCTURE ONLY.  Imported by tests/ as the checker; never by the
product path (glaucis_b200/).

What it restates: the gradients of o (and of the final state) with respect to
q, k, v and h0 for the GLA recurrence that the forward computes,
    h_t = diag(exp(g_t)) h_{t-1} + k_t^T v_t,    o_t = scale * q_t h_t,
with g_t the per-key log-gate (or the per-head constant g_gamma), which is the
quantity the reference's backward returns (KE/examples/kernels/chunk_gla.py
:281-305 reverse dh scan, :313-426 fused dq/dk/dv; custom_vjp :434-456 returns
dq, dk, dv; the gate is not differentiated).  Computed by reverse-mode
automatic differentiation (torch, float64, CPU) through the token-level
recurrence, so it does not share the chunked formulas the kernels use; the
forward recurrence itself is pinned against the chunked oracle in
tests/test_oracle_gla.py.

Parity status: UNPINNED against the reference itself (JAX absent; no golden
vectors).  The reference's own check is the scalar loss of value_and_grad
(KE/examples/chunk_gla.yaml:22, atol 10.0).
"""
from __future__ import annotations

import numpy as np
import torch


def gla_bwd_reference(q, k, v, do, g=None, g_gamma=None, h0=None, scale=None, dht=None):
    """float64 gradients (dq, dk, dv, dh0) of sum(o * do) (+ sum(ht * dht))
    for q, k [B,T,H,K], v [B,T,H,V], g [B,T,H,K] or g_gamma [H], h0 [B,H,K,V]."""
    t64 = lambda a: torch.from_numpy(np.asarray(a, np.float64).copy())
    Q, Kt, Vt = t64(q).requires_grad_(True), t64(k).requires_grad_(True), t64(v).requires_grad_(True)
    B, T, H, K = Q.shape
    V = Vt.shape[-1]
    if scale is None:
        scale = K ** -0.5
    if g_gamma is not None:
        G = t64(g_gamma).reshape(1, 1, H, 1).expand(B, T, H, K)
    else:
        G = t64(g)
    S0 = torch.zeros((B, H, K, V), dtype=torch.float64) if h0 is None else t64(h0)
    S0 = S0.requires_grad_(True)
    S = S0
    outs = []
    for t in range(T):
        S = S * torch.exp(G[:, t])[..., None] + Kt[:, t, :, :, None] * Vt[:, t, :, None, :]
        outs.append(scale * torch.einsum("bhk,bhkv->bhv", Q[:, t], S))
    o = torch.stack(outs, dim=1)
    loss = (o * t64(do)).sum()
    if dht is not None:
        loss = loss + (S * t64(dht)).sum()
    dq, dk, dv, dh0 = torch.autograd.grad(loss, (Q, Kt, Vt, S0))
    return dq.numpy(), dk.numpy(), dv.numpy(), dh0.numpy()
