"""Seeded synthetic workloads for the grouped FP8 matmul and the GLA forward.

The Glaucis templates draw their inputs with JAX PRNG keys
(KE/examples/kernels/gmm_fp8_blockwise.py:39-49, chunk_gla.py:29-37); JAX is
not available, so the same distributions are drawn with torch / numpy
generators and the same tensors are handed to the kernel and to the CPU
oracle.  Shapes and value distributions of the benchmark workloads:

  gmm_small          G=8,   M=2048,  K=1024, N=1024, group sizes ~ multinomial
  gmm_moe_up         G=128, M=32768 (4096 tokens x top-8), K=7168, N=2048,
                     Zipf(1.2)-skewed top-8 routing, the G/32 lowest-ranked
                     experts switched off (empty groups)
  gmm_dense_expert   G=8,   M=65536, K=4096, N=14336, uniform random sizes
                     with one empty group
  gla_b8_t4096       B=8, T=4096,  H=16, K=V=128, C=64, per-key gate, h0 = 0
  gla_b1_t32768      B=1, T=32768, H=32, K=V=128, C=64, per-key gate, h0 ~ N(0, 0.1)

lhs ~ N(0,1) bf16, rhs ~ N(0,0.02) bf16; q, k, v ~ N(0,1) bf16;
g = logsigmoid(N(0,1)) / 16 fp32.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import numpy as np
import torch


@dataclass(frozen=True)
class GMMConfig:
    name: str
    G: int
    M: int
    K: int
    N: int
    routing: str            # "multinomial" | "zipf_topk" | "uniform_one_empty" | "equal"
    topk: int = 8
    zipf: float = 1.2
    rhs_std: float = 0.02

    @property
    def flops(self) -> float:
        return 2.0 * self.M * self.K * self.N


@dataclass(frozen=True)
class GLAConfig:
    name: str
    B: int
    T: int
    H: int
    K: int = 128
    V: int = 128
    C: int = 64
    h0_std: float = 0.0
    gate: str = "per_key"   # "per_key" | "gamma"


GMM_CONFIGS = {
    "gmm_small": GMMConfig("gmm_small", G=8, M=2048, K=1024, N=1024, routing="multinomial"),
    "gmm_moe_up": GMMConfig("gmm_moe_up", G=128, M=32768, K=7168, N=2048, routing="zipf_topk"),
    "gmm_dense_expert": GMMConfig("gmm_dense_expert", G=8, M=65536, K=4096, N=14336,
                                  routing="uniform_one_empty"),
}

GLA_CONFIGS = {
    "gla_b8_t4096": GLAConfig("gla_b8_t4096", B=8, T=4096, H=16),
    "gla_b1_t32768": GLAConfig("gla_b1_t32768", B=1, T=32768, H=32, h0_std=0.1),
}


def routing_desc(cfg: GMMConfig) -> str:
    """One-line statement of how the group sizes of `cfg` are drawn."""
    if cfg.routing == "zipf_topk":
        off = max(1, cfg.G // 32)
        return (f"{cfg.M // cfg.topk} tokens x top-{cfg.topk} distinct experts, p(e) ~ "
                f"rank^-{cfg.zipf} over a seeded expert permutation, the {off} lowest-ranked "
                f"experts switched off (p = 0) so that {off} groups are empty")
    if cfg.routing == "uniform_one_empty":
        return ("seeded uniform-random composition of M (sorted cut points), one random group "
                "emptied and its rows spread over the others")
    if cfg.routing == "multinomial":
        return f"multinomial(M, uniform 1/{cfg.G})"
    return cfg.routing


# ---------------------------------------------------------------------------
# Group sizes
# ---------------------------------------------------------------------------
def group_sizes(routing: str, G: int, M: int, seed: int = 0, topk: int = 8,
                zipf: float = 1.2) -> np.ndarray:
    """int32 [G] summing to M."""
    rng = np.random.default_rng(seed)
    if routing == "equal":
        base = M // G
        s = np.full(G, base, np.int64)
        s[-1] = M - base * (G - 1)
    elif routing == "multinomial":
        s = rng.multinomial(M, np.full(G, 1.0 / G))
    elif routing == "zipf_topk":
        # Each of M/topk tokens picks topk distinct experts without replacement,
        # p(e) ~ rank(e)^-zipf over a seeded permutation of the experts
        # (Gumbel top-k == successive sampling without replacement).  The
        # G/32 lowest-ranked experts are switched off (p = 0) so that some
        # groups are empty, as the workload specifies.
        tokens = M // topk
        perm = rng.permutation(G)
        ranks = np.arange(1, G + 1, dtype=np.float64)
        w = ranks ** (-zipf)
        w[G - max(1, G // 32):] = 0.0
        p = np.empty(G)
        p[perm] = w / w.sum()
        with np.errstate(divide="ignore"):
            keys = np.log(p)[None, :] + rng.gumbel(size=(tokens, G))
        choice = np.argpartition(-keys, topk - 1, axis=1)[:, :topk]
        s = np.bincount(choice.ravel(), minlength=G)
    elif routing == "uniform_one_empty":
        cuts = np.sort(rng.integers(0, M + 1, size=G - 1))
        s = np.diff(np.concatenate([[0], cuts, [M]]))
        z = int(rng.integers(0, G))
        extra = int(s[z])
        s[z] = 0
        others = [i for i in range(G) if i != z]
        for j, i in enumerate(others):
            s[i] += extra // len(others) + (1 if j < extra % len(others) else 0)
    else:
        raise ValueError(f"unknown routing {routing!r}")
    s = s.astype(np.int32)
    assert int(s.sum()) == M
    return s


# ---------------------------------------------------------------------------
# Tensors
# ---------------------------------------------------------------------------
def _gen(device, seed):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def make_gmm_inputs(cfg: GMMConfig, device="cuda", seed: int = 0):
    """Returns (lhs bf16 [M,K], rhs bf16 [G,K,N], group_sizes int32 [G] on device)."""
    gen = _gen(device, seed)
    lhs = torch.randn((cfg.M, cfg.K), generator=gen, device=device, dtype=torch.float32)
    lhs = lhs.to(torch.bfloat16)
    rhs = torch.empty((cfg.G, cfg.K, cfg.N), device=device, dtype=torch.bfloat16)
    for gi in range(cfg.G):  # per group keeps the fp32 temporary small
        rhs[gi] = (torch.randn((cfg.K, cfg.N), generator=gen, device=device,
                               dtype=torch.float32) * cfg.rhs_std).to(torch.bfloat16)
    sizes = group_sizes(cfg.routing, cfg.G, cfg.M, seed=seed, topk=cfg.topk, zipf=cfg.zipf)
    return lhs, rhs, torch.from_numpy(sizes).to(device)


def make_gla_inputs(cfg: GLAConfig, device="cuda", seed: int = 0):
    """Returns dict(q, k, v bf16 [B,T,H,*]; g fp32 [B,T,H,K] or g_gamma fp32 [H];
    h0 fp32 [B,H,K,V] or None)."""
    gen = _gen(device, seed)
    shp = (cfg.B, cfg.T, cfg.H)
    q = torch.randn(shp + (cfg.K,), generator=gen, device=device).to(torch.bfloat16)
    k = torch.randn(shp + (cfg.K,), generator=gen, device=device).to(torch.bfloat16)
    v = torch.randn(shp + (cfg.V,), generator=gen, device=device).to(torch.bfloat16)
    out = dict(q=q, k=k, v=v, g=None, g_gamma=None, h0=None)
    if cfg.gate == "per_key":
        out["g"] = torch.nn.functional.logsigmoid(
            torch.randn(shp + (cfg.K,), generator=gen, device=device)) / 16.0
    else:
        out["g_gamma"] = -torch.randn((cfg.H,), generator=gen, device=device).abs() * 0.1
    if cfg.h0_std > 0:
        out["h0"] = torch.randn((cfg.B, cfg.H, cfg.K, cfg.V), generator=gen,
                                device=device) * cfg.h0_std
    return out


# ---------------------------------------------------------------------------
# Roofline accounting of the GLA kernels
# ---------------------------------------------------------------------------
def gla_flops(B: int, T: int, H: int, K: int = 128, V: int = 128, C: int = 64) -> float:
    """Algorithmic FLOPs of the forward: per token-head 2CK (QK^T) + 2CV (A.V)
    + 2KV (q.h) + 2KV (k^T v state update)."""
    return float(B) * T * H * (2 * C * K + 2 * C * V + 2 * K * V + 2 * K * V)


def gla_bytes(B: int, T: int, H: int, K: int = 128, V: int = 128, per_key_gate: bool = True,
              has_h0: bool = False, has_ht: bool = True) -> float:
    """Algorithmic HBM bytes of the forward: q, k, v (bf16) + g (fp32, per-key
    gate) + o (bf16) per token-head, plus the final (and initial) state per
    sequence."""
    per_tok = 2 * K + 2 * K + 2 * V + (4 * K if per_key_gate else 0) + 2 * V
    state = 4 * K * V * (int(has_h0) + int(has_ht))
    return float(B) * T * H * per_tok + float(B) * H * state


def gla_bwd_flops(B: int, T: int, H: int, K: int = 128, V: int = 128, C: int = 64) -> float:
    """Algorithmic FLOPs of the backward per token-head: the scan's Qs^T do
    (2KV) and the gradient kernel's A, dA (2CK + 2CV), do h^T and v E^T
    (2 x 2KV), dP Kg and dP^T Qs (2 x 2CK), P^T do (2CV), Kg E (2KV)."""
    return float(B) * T * H * (2 * K * V + 2 * C * K + 2 * C * V + 4 * K * V + 4 * C * K
                               + 2 * C * V + 2 * K * V)


def gla_bwd_bytes(B: int, T: int, H: int, K: int = 128, V: int = 128, C: int = 64,
                  per_key_gate: bool = True, fused_minimum: bool = False) -> float:
    """HBM bytes of the backward per token-head.  The two-kernel design: the
    reverse scan reads q, do (bf16) and g, and writes E (bf16 [K, V] per
    chunk); the gradient kernel reads q, k, v, do, g, h and E and writes dq,
    dk, dv.  fused_minimum: one pass that keeps E on chip (reads q, k, v,
    do, g, h; writes dq, dk, dv)."""
    g = 4 * K if per_key_gate else 0
    state = 2 * K * V / C  # one bf16 [K, V] tile per chunk, per token
    grads_rd = 2 * K + 2 * K + 2 * V + 2 * V + g + state
    grads_wr = 2 * K + 2 * K + 2 * V
    if fused_minimum:
        per_tok = grads_rd + grads_wr
    else:
        per_tok = (2 * K + 2 * V + g + state) + (grads_rd + state + grads_wr)
    return float(B) * T * H * per_tok

