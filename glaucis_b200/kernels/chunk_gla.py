"""Chunked GLA (Gated Linear Attention) for B200 (sm_100a) -- template for evolutionary optimization.

Chunked GLA forward fused into one tcgen05 kernel (gated QK^T, causal mask,
intra-chunk PV and the inter-chunk state recurrence), g_gamma (per-head
constant gate) mode as in KE/examples/kernels/chunk_gla.py, whose entry
points it keeps: `_make_test_data`, `chunk_gla_fwd`, `chunk_gla`,
`optimized_compute(B, T, H, K, V, chunk_size)`.

optimized_compute runs the forward and the backward (reverse state-gradient
scan + chunk-parallel dq/dk/dv kernel) and returns the scalar loss o.sum(),
as the reference's value_and_grad does; mode="fwd" runs the forward only.
"""

import torch

from glaucis_b200 import ops


def _make_test_data(B, T, H, K, V, chunk_size, seed=42):
    """Deterministic (q, k, v bf16 N(0,1), g_gamma = -|N(0,1)| * 0.1 fp32) on cuda."""
    gen = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn((B, T, H, K), generator=gen, device="cuda").to(torch.bfloat16)
    k_arr = torch.randn((B, T, H, K), generator=gen, device="cuda").to(torch.bfloat16)
    v = torch.randn((B, T, H, V), generator=gen, device="cuda").to(torch.bfloat16)
    g_gamma = -torch.randn((H,), generator=gen, device="cuda").abs() * 0.1
    return q, k_arr, v, g_gamma


# EVOLVE-BLOCK-START
def chunk_gla_fwd(q, k, v, g_gamma, scale, chunk_size):
    """Chunked GLA forward -> (g_cumsum, A, h, o); the fused kernel keeps
    g_cumsum, A and h on chip, so those are None."""
    return ops.chunk_gla_fwd(q, k, v, g_gamma, scale, chunk_size)


def chunk_gla(q, k, v, g_gamma, scale, chunk_size):
    """Chunked GLA output o (bf16), differentiable in q, k, v."""
    return ops.chunk_gla(q, k, v, g_gamma, scale, chunk_size)


def optimized_compute(B=2, T=4096, H=16, K=128, V=128, chunk_size=64, mode="fwd_bwd"):
    """Forward + backward chunked GLA (gradients of q, k, v computed, as the
    reference's value_and_grad); returns the loss scalar o.sum()."""
    q, k_arr, v, g_gamma = _make_test_data(B, T, H, K, V, chunk_size)
    scale = K ** -0.5
    if mode == "fwd":
        return chunk_gla(q, k_arr, v, g_gamma, scale, chunk_size).float().sum().cpu()
    for t in (q, k_arr, v):
        t.requires_grad_(True)
    loss = chunk_gla(q, k_arr, v, g_gamma, scale, chunk_size).float().sum()
    loss.backward()
    return loss.detach().cpu()
# EVOLVE-BLOCK-END
