"""CPU oracle for the block-wise FP8 grouped matmul forward (numpy).

TEST INFRASTRUCTURE ONLY.  Imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / reference arm as the checker; never by the product
path (glaucis_b200/).

What it restates
  * qwix absmax block quantisation as called by the Glaucis template
    (KE/examples/kernels/gmm_fp8_blockwise.py:84-91 activations, 1x128 tiles
    along K; :100-107 weights, 128x128 tiles over (K, N) per group; qtype
    float8_e4m3fn, scale dtype f32).  qwix is not vendored in the reference
    (unpinned PyPI `qwix`, .github/ci/kernel-eval-gmm-job.yaml:36); its
    published algorithm is scale = absmax/qmax, q = cast(x / scale).
  * tokamax's ragged `gmm` forward (un-vendored `git+.../tokamax`, no commit,
    kernel-eval-gmm-job.yaml:37) as used at gmm_fp8_blockwise.py:109-119 and
    gmm_fp8_blockwise_ref.py:67-77: rows [off_g, off_g + size_g) of lhs times
    rhs[g], off_g the exclusive prefix sum of group_sizes, each 128-deep K
    block's fp32 partial product promoted by a_scale[m, kb] * b_scale[g, kb, nb]
    and accumulated in fp32 (the "dequantised fp32 reference").

Parity status: UNPINNED against the reference itself.  JAX, qwix and tokamax
are not installed and the reference's GMM runs only as a TPU Pallas kernel
(gmm_fp8_blockwise_ref.py:67-77, interpret=False), and the reference holds no
golden vectors.  Pinned instead: (1) the e4m3 cast bit-for-bit against
torch.float8_e4m3fn (an independent implementation of the same OCP format);
(2) scale shapes and the forward relative-error bound vs. a bf16 matmul that
the reference's own tests assert (KE/tests/standalone_gmm_fp8_blockwise_test.py
:287-316 and :365-370); (3) committed fixtures in tests/golden/.
Documented choices where qwix's exact behaviour is unknown: an all-zero block
gets scale 1.0 (q = 0); the cast saturates to +-448 (values never exceed 448
by more than rounding since |x/s| <= 448 up to one ulp).
"""
from __future__ import annotations

import numpy as np

E4M3_MAX = 448.0
TILE = 128


# ---------------------------------------------------------------------------
# e4m3fn (1 sign, 4 exponent bits with bias 7, 3 mantissa bits; no infinity,
# 0x7f / 0xff NaN; largest finite 448, smallest subnormal 2^-9)
# ---------------------------------------------------------------------------
def f32_to_e4m3(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even cast to e4m3fn bytes, saturating to +-448."""
    x = np.asarray(x, dtype=np.float32)
    sign = np.signbit(x).astype(np.uint8) << np.uint8(7)
    a = np.abs(x).astype(np.float64)
    nan = np.isnan(a)
    a = np.where(nan, 0.0, a)
    _, e = np.frexp(a)                      # a = m * 2**e, m in [0.5, 1)
    E = np.maximum(e - 1, -6)               # binade, clamped to the subnormal one
    quantum = np.ldexp(1.0, E - 3)          # 3 mantissa bits
    v = np.minimum(np.rint(a / quantum) * quantum, E4M3_MAX)   # rint: ties to even
    sub = v < 2.0 ** -6
    code_sub = np.rint(v / 2.0 ** -9).astype(np.int64)          # 0..8 (8 == 2^-6 == 0x08)
    mm, ee = np.frexp(np.where(sub, 1.0, v))
    code_norm = ((ee - 1 + 7) << 3) | np.rint((mm * 2.0 - 1.0) * 8.0).astype(np.int64)
    code = np.where(sub, code_sub, code_norm).astype(np.uint8)
    code = np.where(nan, np.uint8(0x7F), code)
    return (code | sign).astype(np.uint8)


def _e4m3_table() -> np.ndarray:
    b = np.arange(256, dtype=np.int64)
    s = (b >> 7) & 1
    e = (b >> 3) & 0xF
    m = b & 7
    val = np.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * np.ldexp(1.0, e - 7))
    val = np.where((e == 15) & (m == 7), np.nan, val)
    return np.where(s == 1, -val, val).astype(np.float32)


E4M3_TABLE = _e4m3_table()


def e4m3_to_f32(q: np.ndarray) -> np.ndarray:
    return E4M3_TABLE[np.asarray(q, dtype=np.uint8)]


def bf16_bits_to_f32(u16: np.ndarray) -> np.ndarray:
    return (np.asarray(u16, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------------------
# Quantisers
# ---------------------------------------------------------------------------
def _scale(amax: np.ndarray) -> np.ndarray:
    amax = amax.astype(np.float32)
    return np.where(amax > 0, amax / np.float32(E4M3_MAX), np.float32(1.0)).astype(np.float32)


def quant_act_1x128(x: np.ndarray):
    """x fp32 (bf16 values) [M, K] -> (q uint8 [M, K], s fp32 [M, K/128]).
    Follows gmm_fp8_blockwise.py:84-91 (channelwise axis 0, 128-tiles on axis 1)."""
    x = np.asarray(x, dtype=np.float32)
    M, K = x.shape
    blk = x.reshape(M, K // TILE, TILE)
    s = _scale(np.abs(blk).max(axis=-1))
    q = f32_to_e4m3(blk / s[..., None]).reshape(M, K)
    return q, s


def quant_w_128x128(w: np.ndarray):
    """w fp32 (bf16 values) [G, K, N] -> (q uint8 [G, K, N], s fp32 [G, K/128, N/128]).
    Follows gmm_fp8_blockwise.py:100-107 (channelwise axis 0, 128-tiles on 1, 2)."""
    w = np.asarray(w, dtype=np.float32)
    G, K, N = w.shape
    blk = w.reshape(G, K // TILE, TILE, N // TILE, TILE)
    s = _scale(np.abs(blk).max(axis=(2, 4)))
    q = f32_to_e4m3(blk / s[:, :, None, :, None]).reshape(G, K, N)
    return q, s


# ---------------------------------------------------------------------------
# Grouped matmul
# ---------------------------------------------------------------------------
def group_offsets(group_sizes: np.ndarray) -> np.ndarray:
    gs = np.asarray(group_sizes, dtype=np.int64)
    return np.concatenate([[0], np.cumsum(gs)])


def gmm_group_rows(a_q_rows, a_s_rows, b_q_g, b_s_g) -> np.ndarray:
    """Rows of one group: sum over 128-deep K blocks of the fp32 partial
    product times a_s[m, kb] * b_s[g, kb, n // 128], accumulated in fp32."""
    a = e4m3_to_f32(a_q_rows)                               # [R, K]
    b = e4m3_to_f32(b_q_g)                                  # [K, N]
    a_s_rows = np.asarray(a_s_rows, np.float32)
    b_s_g = np.asarray(b_s_g, np.float32)
    R, K = a.shape
    N = b.shape[1]
    acc = np.zeros((R, N), dtype=np.float32)
    for kb in range(K // TILE):
        part = a[:, kb * TILE:(kb + 1) * TILE] @ b[kb * TILE:(kb + 1) * TILE]
        sc = a_s_rows[:, kb][:, None] * np.repeat(b_s_g[kb], TILE)[None, :]
        acc += part * sc.astype(np.float32)
    return acc


def gmm_fwd(a_q, a_s, b_q, b_s, group_sizes, rows=None) -> np.ndarray:
    """out fp32 [M, N]; rows past sum(group_sizes) are zero.

    `rows` optionally restricts the computation to a sorted subset of row
    indices (returns [len(rows), N]) for sampled checks at full size.
    """
    M, K = a_q.shape
    G, _, N = b_q.shape
    off = group_offsets(group_sizes)
    sel = np.arange(M) if rows is None else np.asarray(rows, dtype=np.int64)
    out = np.zeros((len(sel), N), dtype=np.float32)
    gid = np.searchsorted(off, sel, side="right") - 1      # group of each selected row
    for g in range(G):
        idx = np.nonzero(gid == g)[0]
        if idx.size == 0:
            continue
        r = sel[idx]
        out[idx] = gmm_group_rows(a_q[r], np.asarray(a_s)[r], b_q[g], np.asarray(b_s)[g])
    return out


def gmm_bf16_reference(lhs: np.ndarray, rhs: np.ndarray, group_sizes) -> np.ndarray:
    """Unquantised grouped matmul (fp32 math on the bf16 values): the
    comparison point of KE/tests/standalone_gmm_fp8_blockwise_test.py:365-370."""
    M, _ = lhs.shape
    off = group_offsets(group_sizes)
    out = np.zeros((M, rhs.shape[-1]), dtype=np.float32)
    for g in range(rhs.shape[0]):
        out[off[g]:off[g + 1]] = lhs[off[g]:off[g + 1]] @ rhs[g]
    return out


def gmm_fp8_blockwise(lhs: np.ndarray, rhs: np.ndarray, group_sizes) -> np.ndarray:
    """End-to-end forward: quantise both operands then grouped matmul (fp32 out),
    KE/examples/kernels/gmm_fp8_blockwise_ref.py:37-78 forward."""
    a_q, a_s = quant_act_1x128(lhs)
    b_q, b_s = quant_w_128x128(rhs)
    return gmm_fwd(a_q, a_s, b_q, b_s, group_sizes)


def gemm_flops(group_sizes, K: int, N: int) -> float:
    return 2.0 * float(np.sum(np.asarray(group_sizes, dtype=np.int64))) * K * N
