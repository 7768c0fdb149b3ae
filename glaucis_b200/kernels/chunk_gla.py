"""Chunked GLA (Gated Linear Attention) for B200 (sm_100a) -- template for evolutionary optimization.

Chunked GLA forward fused into one tcgen05 kernel (gated QK^T, causal mask,
intra-chunk PV and the inter-chunk state recurrence), g_gamma (per-head
constant gate) mode as in KE/examples/kernels/chunk_gla.py, whose entry
points it keeps: `_make_test_data`, `chunk_gla_fwd`, `chunk_gla`,
`optimized_compute(B, T, H, K, V, chunk_size)`.

optimized_compute runs the FORWARD pass and returns the scalar loss o.sum();
the reference template also runs the backward, not built on B200 yet.
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
    """Chunked GLA forward output o (bf16)."""
    _, _, _, o = chunk_gla_fwd(q, k, v, g_gamma, scale, chunk_size)
    return o


def optimized_compute(B=2, T=4096, H=16, K=128, V=128, chunk_size=64):
    """Forward chunked GLA; returns the loss scalar o.sum()."""
    q, k_arr, v, g_gamma = _make_test_data(B, T, H, K, V, chunk_size)
    scale = K ** -0.5
    o = chunk_gla(q, k_arr, v, g_gamma, scale, chunk_size)
    return o.float().sum().cpu()
# EVOLVE-BLOCK-END
