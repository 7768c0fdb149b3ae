"""Generates the committed golden fixtures (tests/golden/*.npz) from seeded
inputs with the CPU oracles.  The reference (JAX + qwix + tokamax on TPU)
cannot run in this environment, so these fixtures pin the oracle and the
GPU kernels against a fixed record rather than against reference output.

    python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import gla_oracle, gmm_oracle  # noqa: E402


def bf16_round(x):
    """fp32 -> bf16 bit pattern (uint16), round to nearest even."""
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def gmm_case():
    rng = np.random.default_rng(1234)
    G, M, K, N = 4, 200, 256, 128
    sizes = np.array([70, 0, 129, 1], np.int32)          # empty group, partial tiles
    lhs = bf16_round(rng.standard_normal((M, K)).astype(np.float32))
    rhs = bf16_round((rng.standard_normal((G, K, N)) * 0.02).astype(np.float32))
    lhs[3, :128] = 0                                     # an all-zero 1x128 block
    lf = gmm_oracle.bf16_bits_to_f32(lhs)
    rf = gmm_oracle.bf16_bits_to_f32(rhs)
    a_q, a_s = gmm_oracle.quant_act_1x128(lf)
    b_q, b_s = gmm_oracle.quant_w_128x128(rf)
    out = gmm_oracle.gmm_fwd(a_q, a_s, b_q, b_s, sizes)
    np.savez_compressed(os.path.join(HERE, "gmm_small_ragged.npz"), lhs_bf16=lhs, rhs_bf16=rhs,
                        group_sizes=sizes, a_q=a_q, a_s=a_s, b_q=b_q, b_s=b_s, out=out)


def gla_case():
    rng = np.random.default_rng(4321)
    B, T, H, K, V = 1, 128, 1, 128, 128
    q = bf16_round(rng.standard_normal((B, T, H, K)).astype(np.float32))
    k = bf16_round(rng.standard_normal((B, T, H, K)).astype(np.float32))
    v = bf16_round(rng.standard_normal((B, T, H, V)).astype(np.float32))
    x = rng.standard_normal((B, T, H, K))
    g = (-np.logaddexp(0.0, -x) / 16.0).astype(np.float32)   # logsigmoid(x)/16
    h0 = (rng.standard_normal((B, H, K, V)) * 0.1).astype(np.float32)
    f = gmm_oracle.bf16_bits_to_f32
    o, ht = gla_oracle.chunk_gla_fwd(f(q), f(k), f(v), g=g, h0=h0, scale=K ** -0.5)
    np.savez_compressed(os.path.join(HERE, "gla_per_key_h0.npz"), q_bf16=q, k_bf16=k, v_bf16=v,
                        g=g, h0=h0, o=o, ht=ht)


if __name__ == "__main__":
    gmm_case()
    gla_case()
    print("wrote", sorted(f for f in os.listdir(HERE) if f.endswith(".npz")))
