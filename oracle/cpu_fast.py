"""BLAS-backed CPU restatements (torch on the host cores) of the same two
forwards as gmm_oracle.py / gla_oracle.py, used as the timed CPU baseline.

TEST INFRASTRUCTURE ONLY (bench.py's CPU-baseline / reference arm and the
tests that pin these against the numpy oracles); never part of the product
path.

* gmm_fp8_blockwise: absmax 1x128 / 128x128 quantisation (torch's
  float8_e4m3fn cast, pinned bit-for-bit against gmm_oracle.f32_to_e4m3 in
  tests), then one fp32 GEMM per group on the dequantised operands.  Scaling
  each operand block by its scale before the GEMM is the same sum as the
  per-K-block promotion of KE/examples/kernels/gmm_fp8_blockwise.py:109-119
  (only the fp32 summation order differs).
* chunk_gla_fwd: the chunked recurrence of gla_oracle.chunk_gla_fwd
  (KE/examples/kernels/chunk_gla_ref.py:23-117 with the per-key gate of
  KE/upstream/fused_chunk_simple_gla/common_chunk_h.py:330-334) with batched
  fp32 matmuls.
"""
from __future__ import annotations

import torch

TILE = 128
E4M3_MAX = 448.0


def _scale(amax: torch.Tensor) -> torch.Tensor:
    return torch.where(amax > 0, amax / E4M3_MAX, torch.ones_like(amax))


def quant_act_1x128(x: torch.Tensor):
    M, K = x.shape
    blk = x.float().reshape(M, K // TILE, TILE)
    s = _scale(blk.abs().amax(dim=-1))
    q = (blk / s[..., None]).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)
    return q.reshape(M, K), s


def quant_w_128x128(w: torch.Tensor):
    G, K, N = w.shape
    blk = w.float().reshape(G, K // TILE, TILE, N // TILE, TILE)
    s = _scale(blk.abs().amax(dim=(2, 4)))
    q = (blk / s[:, :, None, :, None]).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)
    return q.reshape(G, K, N), s


def dequant_act(q: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    M, K = q.shape
    return (q.float().reshape(M, K // TILE, TILE) * s[..., None]).reshape(M, K)


def dequant_w(q: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    G, K, N = q.shape
    b = q.float().reshape(G, K // TILE, TILE, N // TILE, TILE) * s[:, :, None, :, None]
    return b.reshape(G, K, N)


def gmm_fp8_blockwise(lhs: torch.Tensor, rhs: torch.Tensor, group_sizes) -> torch.Tensor:
    """bf16 lhs [M,K], bf16 rhs [G,K,N], sizes [G] -> fp32 [M,N]."""
    a_q, a_s = quant_act_1x128(lhs)
    b_q, b_s = quant_w_128x128(rhs)
    a = dequant_act(a_q, a_s)
    out = torch.zeros((lhs.shape[0], rhs.shape[-1]), dtype=torch.float32)
    off = 0
    for g, m in enumerate(int(x) for x in group_sizes):
        if m:
            b = dequant_w(b_q[g:g + 1], b_s[g:g + 1])[0]
            torch.matmul(a[off:off + m], b, out=out[off:off + m])
        off += m
    return out


def chunk_gla_fwd(q, k, v, g=None, g_gamma=None, h0=None, scale=None, chunk_size=64):
    """fp32 tensors [B,T,H,K/V] -> (o [B,T,H,V], ht [B,H,K,V])."""
    q, k, v = q.float(), k.float(), v.float()
    B, T, H, K = q.shape
    V = v.shape[-1]
    C = chunk_size
    NT = T // C
    scale = K ** -0.5 if scale is None else scale
    if g_gamma is not None:
        pos = torch.arange(1, C + 1, dtype=torch.float32).repeat(NT).reshape(1, T, 1, 1)
        gc = (g_gamma.float().reshape(1, 1, H, 1) * pos).expand(B, T, H, K)
    else:
        gc = g.float().reshape(B, NT, C, H, K).cumsum(dim=2).reshape(B, T, H, K)
    # [B,H,NT,C,D]
    r = lambda x, D: x.reshape(B, NT, C, H, D).permute(0, 3, 1, 2, 4)
    qc, kc, vc, gcc = r(q, K), r(k, K), r(v, V), r(gc, K)
    glast = gcc[:, :, :, -1]                                    # [B,H,NT,K]
    qg = qc * torch.exp(gcc)
    kg = kc * torch.exp(-gcc)
    kd = kc * torch.exp(glast[:, :, :, None] - gcc)
    S = kd.transpose(-1, -2) @ vc                               # [B,H,NT,K,V] chunk updates
    h = torch.zeros((B, H, K, V)) if h0 is None else h0.float().clone()
    states = torch.empty((B, H, NT, K, V))
    dec = torch.exp(glast)
    for n in range(NT):
        states[:, :, n] = h
        h = h * dec[:, :, n, :, None] + S[:, :, n]
    A = (qg @ kg.transpose(-1, -2)) * scale
    A = torch.tril(A)
    o = scale * (qg @ states) + A @ vc                          # [B,H,NT,C,V]
    o = o.permute(0, 2, 3, 1, 4).reshape(B, T, H, V)
    return o, h
