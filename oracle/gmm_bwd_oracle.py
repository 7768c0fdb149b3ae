"""CPU oracle for the backward of the block-wise FP8 grouped matmul (numpy).

TEST INFRASTRUCTURE ONLY.  Imported by tests/ as the checker; never by the
product path (glaucis_b200/).

What it restates (KE/examples/kernels/gmm_fp8_blockwise.py:123-169, the
custom-VJP backward of the Glaucis template, with the residuals of the forward
at :80-120):
  * lhs_t = quantize(lhs^T, channelwise_axes=[0], tiled_axes={1: 128}) (:92-99):
    one fp32 scale per (column k of lhs, 128-row block of M).  Restated here
    untransposed: quant_col_128x1(lhs) -> q [M, K], s [M/128, K], with
    lhs_t.qvalue = q.T and lhs_t.scale = s.T.
  * dlhs_dout = quantize(grad, channelwise_axes=[0], tiled_axes={1: 128})
    (:128-134): the forward's 1x128 activation quantiser applied to grad [M, N].
  * drhs_dout = quantize(grad, channelwise_axes=[1], tiled_axes={0: 128})
    (:135-141): quant_col_128x1(grad) -> scales [M/128, N].
  * dlhs = gmm(dlhs_dout, rhs, transpose_rhs=True) (:143-153):
    dlhs[m, k] = sum over 128-wide N blocks nb of ds[m, nb] * b_s[g, k/128, nb]
    times the fp32 partial sum_{n in nb} dq[m, n] b_q[g, k, n], g the group of m.
  * drhs = tgmm(lhs_t, drhs_dout, group_sizes) (:155-165): per group g,
    drhs[g, k, n] = sum over the global 128-row blocks mb that the group's rows
    touch of ls[mb, k] * ds[mb, n] times sum_{m in group g and block mb}
    lq[m, k] dq[m, n]; empty groups give zeros.
  tokamax's gmm/tgmm are not vendored (git+.../tokamax with no commit,
  .github/ci/kernel-eval-gmm-job.yaml:37); the promotion per 128-deep
  reduction block in fp32 is the same rule as the forward's.

Parity status: UNPINNED against the reference itself (JAX / qwix / tokamax
are absent and the reference's kernels run only on TPU); the reference's own
backward check is a relative error below 0.5 against the unquantised
gradient (KE/tests/standalone_gmm_fp8_blockwise_test.py:388-401), which the
tests here also assert.  Requires M % 128 == 0 (the 128-row tiling of grad).
"""
from __future__ import annotations

import numpy as np

from oracle.gmm_oracle import (TILE, _scale, e4m3_to_f32, f32_to_e4m3, group_offsets,
                               quant_act_1x128, quant_w_128x128)


def quant_col_128x1(x: np.ndarray):
    """x fp32 (bf16 values) [M, C], M % 128 == 0 -> (q uint8 [M, C],
    s fp32 [M/128, C]): one scale per 128-row block of each column."""
    x = np.asarray(x, dtype=np.float32)
    M, C = x.shape
    blk = x.reshape(M // TILE, TILE, C)
    s = _scale(np.abs(blk).max(axis=1))                     # [M/128, C]
    q = f32_to_e4m3(blk / s[:, None, :]).reshape(M, C)
    return q, s


def gmm_dlhs(dq, ds, b_q, b_s, group_sizes) -> np.ndarray:
    """dlhs fp32 [M, K] from dout quantised 1x128 along N (dq [M, N], ds
    [M, N/128]) and the forward's weight QArray (b_q [G, K, N], b_s
    [G, K/128, N/128]); rows past sum(group_sizes) are zero."""
    M, N = dq.shape
    G, K, _ = b_q.shape
    off = group_offsets(group_sizes)
    out = np.zeros((M, K), dtype=np.float32)
    a = e4m3_to_f32(dq)
    ds = np.asarray(ds, np.float32)
    for g in range(G):
        r0, r1 = int(off[g]), int(off[g + 1])
        if r1 <= r0:
            continue
        b = e4m3_to_f32(b_q[g])                              # [K, N]
        acc = np.zeros((r1 - r0, K), dtype=np.float32)
        for nb in range(N // TILE):
            part = a[r0:r1, nb * TILE:(nb + 1) * TILE] @ b[:, nb * TILE:(nb + 1) * TILE].T
            sc = ds[r0:r1, nb][:, None] * np.repeat(np.asarray(b_s[g][:, nb], np.float32), TILE)[None, :]
            acc += part * sc.astype(np.float32)
        out[r0:r1] = acc
    return out


def tgmm(lq, ls, dq, ds, group_sizes, groups=None) -> np.ndarray:
    """drhs fp32 [G, K, N] (or only the listed `groups`, same shape with the
    others left zero) from lhs and dout quantised in 128x1 column blocks."""
    M, K = lq.shape
    N = dq.shape[1]
    G = len(group_sizes)
    off = group_offsets(group_sizes)
    out = np.zeros((G, K, N), dtype=np.float32)
    la, da = e4m3_to_f32(lq), e4m3_to_f32(dq)
    ls, ds = np.asarray(ls, np.float32), np.asarray(ds, np.float32)
    for g in (range(G) if groups is None else groups):
        r0, r1 = int(off[g]), int(off[g + 1])
        acc = np.zeros((K, N), dtype=np.float32)
        for mb in range(r0 // TILE, (r1 + TILE - 1) // TILE if r1 > r0 else r0 // TILE):
            lo, hi = max(r0, mb * TILE), min(r1, (mb + 1) * TILE)
            part = la[lo:hi].T @ da[lo:hi]                   # [K, N]
            acc += part * (ls[mb][:, None] * ds[mb][None, :]).astype(np.float32)
        out[g] = acc
    return out


def gmm_fp8_blockwise_bwd(lhs, rhs, group_sizes, grad):
    """(dlhs [M, K], drhs [G, K, N]) in fp32 from bf16-valued fp32 inputs,
    following KE/examples/kernels/gmm_fp8_blockwise.py:123-169."""
    lq, ls = quant_col_128x1(lhs)
    b_q, b_s = quant_w_128x128(rhs)
    dq1, ds1 = quant_act_1x128(grad)
    dq2, ds2 = quant_col_128x1(grad)
    return gmm_dlhs(dq1, ds1, b_q, b_s, group_sizes), tgmm(lq, ls, dq2, ds2, group_sizes)


def gmm_bwd_unquantised(lhs, rhs, group_sizes, grad):
    """Exact gradients of sum-free gmm (fp32 math): the comparison point of
    KE/tests/standalone_gmm_fp8_blockwise_test.py:388-401."""
    off = group_offsets(group_sizes)
    G = rhs.shape[0]
    dlhs = np.zeros_like(lhs, dtype=np.float32)
    drhs = np.zeros_like(rhs, dtype=np.float32)
    for g in range(G):
        r0, r1 = int(off[g]), int(off[g + 1])
        dlhs[r0:r1] = grad[r0:r1] @ rhs[g].T
        drhs[g] = lhs[r0:r1].T @ grad[r0:r1]
    return dlhs, drhs
