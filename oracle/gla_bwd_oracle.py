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

chunk_gla_bwd restates the reference's chunked backward in numpy fp32:
the reverse state-gradient scan (KE/examples/kernels/chunk_gla_ref.py
:118-143; dh_all[n] is the gradient of the state after chunk n) and the
per-chunk dq / dk / dv (:146-199), with the per-head decay exp(g_gamma C)
generalised to the per-key e^{G_last} as in the forward's per-key gate, plus
the final-state gradient dht and dh0 (the scan's last value).  It is checked
against gla_bwd_reference (independent derivation) in tests/test_oracle_gla.py.

Parity status: UNPINNED against the reference itself (JAX absent; no golden
vectors).  The reference's own check is the scalar loss of value_and_grad
(KE/examples/chunk_gla.yaml:22, atol 10.0).
"""
from __future__ import annotations

import numpy as np
import torch

from oracle.gla_oracle import chunk_gla_fwd, g_cumsum_from


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


def chunk_gla_bwd(q, k, v, do, g=None, g_gamma=None, h0=None, scale=None, chunk_size=64,
                  dht=None):
    """fp32 (dq, dk, dv, dh0) by the reference's chunked formulas."""
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    v = np.asarray(v, np.float32)
    do = np.asarray(do, np.float32)
    B, T, H, K = q.shape
    V = v.shape[-1]
    C = chunk_size
    NT = T // C
    if scale is None:
        scale = K ** -0.5
    scale = np.float32(scale)
    _, _, h_all = chunk_gla_fwd(q, k, v, g=g, g_gamma=g_gamma, h0=h0, scale=scale, chunk_size=C,
                                return_states=True)
    gc = g_cumsum_from(g, g_gamma, B, T, H, K, C).reshape(B, NT, C, H, K)
    qc, kc = q.reshape(B, NT, C, H, K), k.reshape(B, NT, C, H, K)
    vc, doc = v.reshape(B, NT, C, H, V), do.reshape(B, NT, C, H, V)
    gn = gc[:, :, -1]                                                  # [B,NT,H,K]
    # reverse scan: dh_all[:, n] = dL/d(state after chunk n)  (ref :127-143)
    dh = np.zeros((B, H, K, V), np.float32) if dht is None else np.asarray(dht, np.float32).copy()
    dh_all = np.empty((B, NT, H, K, V), np.float32)
    for n in range(NT - 1, -1, -1):
        dh_all[:, n] = dh
        q_hat = qc[:, n] * np.exp(gc[:, n]) * scale                    # [B,C,H,K]
        dh = dh * np.exp(gn[:, n])[..., None] + np.einsum("bchk,bchv->bhkv", q_hat, doc[:, n])
    dh0 = dh
    mask = np.tril(np.ones((C, C), np.float32))
    # per-chunk gradients (ref :161-197)
    A = np.einsum("bnihk,bnjhk->bnihj", qc * np.exp(gc), kc * np.exp(-gc)) * scale
    A = A * mask[None, None, :, None, :]
    dA = np.einsum("bnihv,bnjhv->bnihj", doc, vc) * scale * mask[None, None, :, None, :]
    dv = (np.einsum("bnihj,bnihv->bnjhv", A, doc)
          + np.einsum("bnchk,bnhkv->bnchv", kc * np.exp(gn[:, :, None] - gc), dh_all))
    dq = (np.exp(gc) * np.einsum("bnihj,bnjhk->bnihk", dA, kc * np.exp(-gc))
          + scale * np.exp(gc) * np.einsum("bnchv,bnhkv->bnchk", doc, h_all))
    dk = (np.exp(-gc) * np.einsum("bnihj,bnihk->bnjhk", dA, qc * np.exp(gc))
          + np.exp(gn[:, :, None] - gc) * np.einsum("bnchv,bnhkv->bnchk", vc, dh_all))
    return (dq.reshape(B, T, H, K).astype(np.float32), dk.reshape(B, T, H, K).astype(np.float32),
            dv.reshape(B, T, H, V).astype(np.float32), dh0.astype(np.float32))
