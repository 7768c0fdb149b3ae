"""Torch-facing ops over the C ABI.  Tensors must live on a CUDA device; every
op launches on the current stream and never falls back to another backend.

Op names and argument meaning mirror the Glaucis kernel templates
(KE/examples/kernels/gmm_fp8_blockwise.py, KE/examples/kernels/chunk_gla.py).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import _lib

FP8 = torch.float8_e4m3fn
TILE = 128


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _need_cuda(*ts: Optional[torch.Tensor]) -> None:
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("glaucis_b200 ops take CUDA tensors (no CPU path)")
        if not t.is_contiguous():
            raise ValueError("glaucis_b200 ops take contiguous tensors")


# ---------------------------------------------------------------------------
# Block-wise FP8 quantisers
# ---------------------------------------------------------------------------
def _out(t: Optional[torch.Tensor], shape, dtype, device, name: str) -> torch.Tensor:
    """A preallocated contiguous output of the given shape / dtype, or a new one."""
    if t is None:
        return torch.empty(shape, dtype=dtype, device=device)
    if tuple(t.shape) != tuple(shape) or t.dtype != dtype or not t.is_contiguous() or t.device != device:
        raise ValueError(f"{name} must be a contiguous {dtype} tensor of shape {tuple(shape)} on {device}")
    return t


def quant_act_1x128(x: torch.Tensor, q: Optional[torch.Tensor] = None,
                    s: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """bf16 [M, K] -> (e4m3 [M, K], fp32 scales [M, K/128]); `q` / `s` may be
    given as preallocated outputs.

    Replaces qwix.pallas.quantize(lhs, channelwise_axes=[0], tiled_axes={1: 128},
    absmax, fp32 scale) at KE/examples/kernels/gmm_fp8_blockwise.py:84-91.
    """
    _need_cuda(x)
    if x.dtype != torch.bfloat16 or x.dim() != 2:
        raise ValueError("quant_act_1x128 expects a 2-D bf16 tensor")
    M, K = x.shape
    q = _out(q, (M, K), FP8, x.device, "q")
    s = _out(s, (M, K // TILE), torch.float32, x.device, "s")
    lib = _lib.load()
    _lib.check(lib.gl_quant_act_1x128(x.data_ptr(), M, K, q.data_ptr(), s.data_ptr(), None,
                                      _stream()), "gl_quant_act_1x128")
    return q, s


def quant_w_128x128(w: torch.Tensor, q: Optional[torch.Tensor] = None,
                    s: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """bf16 [G, K, N] -> (e4m3 [G, K, N], fp32 scales [G, K/128, N/128]);
    `q` / `s` may be given as preallocated outputs.

    Replaces qwix.pallas.quantize(rhs, channelwise_axes=[0],
    tiled_axes={1: 128, 2: 128}) at KE/examples/kernels/gmm_fp8_blockwise.py:100-107.
    """
    _need_cuda(w)
    if w.dtype != torch.bfloat16 or w.dim() != 3:
        raise ValueError("quant_w_128x128 expects a 3-D bf16 tensor")
    G, K, N = w.shape
    q = _out(q, (G, K, N), FP8, w.device, "q")
    s = _out(s, (G, K // TILE, N // TILE), torch.float32, w.device, "s")
    lib = _lib.load()
    _lib.check(lib.gl_quant_w_128x128(w.data_ptr(), G, K, N, q.data_ptr(), s.data_ptr(), None,
                                      _stream()), "gl_quant_w_128x128")
    return q, s


# ---------------------------------------------------------------------------
# Grouped matmul
# ---------------------------------------------------------------------------
def gmm_fp8_fwd(a_q: torch.Tensor, a_s: torch.Tensor, b_q: torch.Tensor, b_s: torch.Tensor,
                group_sizes: torch.Tensor, out_dtype: torch.dtype = torch.float32,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Grouped matmul on pre-quantised operands (QArray-equivalent inputs).

    Replaces tokamax pallas_mosaic_tpu_kernel.gmm(lhs=QArray, rhs=QArray,
    group_sizes, out_dtype, transpose_rhs=False) at
    KE/examples/kernels/gmm_fp8_blockwise.py:109-119.  Rows at or beyond
    sum(group_sizes) are zero.
    """
    _need_cuda(a_q, a_s, b_q, b_s, group_sizes)
    M, K = a_q.shape
    G, K2, N = b_q.shape
    if K2 != K:
        raise ValueError(f"K mismatch: lhs {K} vs rhs {K2}")
    if group_sizes.dtype != torch.int32 or group_sizes.numel() != G:
        raise ValueError("group_sizes must be int32 [G]")
    if out_dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("out_dtype must be bf16 or fp32")
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=a_q.device)
    code = _lib.GL_OUT_F32 if out.dtype == torch.float32 else _lib.GL_OUT_BF16
    lib = _lib.load()
    _lib.check(lib.gl_gmm_fp8_fwd(a_q.data_ptr(), a_s.data_ptr(), b_q.data_ptr(), b_s.data_ptr(),
                                  group_sizes.data_ptr(), G, M, K, N, out.data_ptr(), code, None,
                                  _stream()), "gl_gmm_fp8_fwd")
    return out


def _zero_tail_rows(out: torch.Tensor, group_sizes: torch.Tensor) -> None:
    # Rows past sum(group_sizes) belong to no group: zero them on the device
    # without a host round trip.
    M = out.shape[0]
    total = group_sizes.sum()
    rows = torch.arange(M, device=out.device)
    out.masked_fill_((rows >= total).unsqueeze(1), 0)


def gmm_fp8_blockwise(lhs: torch.Tensor, rhs: torch.Tensor, group_sizes: torch.Tensor,
                      tiling: tuple = (256, 512, 256, 256, 512, 128, 1024, 512, 128),
                      out_dtype: torch.dtype = torch.float32,
                      zero_unassigned_rows: bool = True) -> torch.Tensor:
    """Forward of the Glaucis `gmm_fp8_blockwise(lhs, rhs, group_sizes, tiling)`
    (KE/examples/kernels/gmm_fp8_blockwise.py:53-120): quantise lhs 1x128 and
    rhs 128x128 to e4m3 with fp32 absmax scales, then the grouped matmul with
    per-K-block fp32 promotion.  `tiling` is accepted for signature
    compatibility; the B200 kernel's tiles are fixed (128x256x128).
    """
    del tiling
    if torch.is_grad_enabled() and (lhs.requires_grad or rhs.requires_grad):
        # differentiable path: backward = gmm_fp8_blockwise_bwd
        return _GmmFp8Blockwise.apply(lhs, rhs, group_sizes, out_dtype)
    a_q, a_s = quant_act_1x128(lhs)
    b_q, b_s = quant_w_128x128(rhs)
    out = gmm_fp8_fwd(a_q, a_s, b_q, b_s, group_sizes, out_dtype=out_dtype)
    if zero_unassigned_rows:
        _zero_tail_rows(out, group_sizes)
    return out


# ---------------------------------------------------------------------------
# Grouped matmul backward (KE/examples/kernels/gmm_fp8_blockwise.py:123-169)
# ---------------------------------------------------------------------------
def gmm_fp8_fwd_scatter(a_q: torch.Tensor, a_s: torch.Tensor, b_q: torch.Tensor, b_s: torch.Tensor,
                        group_sizes: torch.Tensor, outs, row_offset: int,
                        out_dtype: torch.dtype = torch.bfloat16) -> None:
    """gmm_fp8_fwd whose output rows go to row `row_offset` + m of every
    buffer in `outs` (tensors on this device, or integer device addresses of
    peer-mapped buffers such as shard.PeerBuffers.ptrs), each holding at
    least row_offset + M rows of N elements of `out_dtype`.  Used to assemble
    an expert-sharded output on every rank inside the matmul's epilogue; the
    caller synchronises the ranks after it."""
    _need_cuda(a_q, a_s, b_q, b_s, group_sizes)
    M, K = a_q.shape
    G, K2, N = b_q.shape
    if K2 != K:
        raise ValueError(f"K mismatch: a {K} vs b {K2}")
    ptrs = [o.data_ptr() if isinstance(o, torch.Tensor) else int(o) for o in outs]
    for o in outs:
        if isinstance(o, torch.Tensor) and (o.dtype != out_dtype or o.dim() != 2 or o.shape[1] != N
                                            or o.shape[0] < row_offset + M or not o.is_contiguous()):
            raise ValueError(f"each output must be a contiguous {out_dtype} [>= row_offset + M, N] tensor")
    import ctypes
    arr = (ctypes.c_void_p * len(ptrs))(*ptrs)
    code = _lib.GL_OUT_F32 if out_dtype == torch.float32 else _lib.GL_OUT_BF16
    _lib.check(_lib.load().gl_gmm_fp8_fwd_scatter(a_q.data_ptr(), a_s.data_ptr(), b_q.data_ptr(),
                                                  b_s.data_ptr(), group_sizes.data_ptr(), G, M, K, N,
                                                  ctypes.cast(arr, ctypes.c_void_p), len(ptrs),
                                                  int(row_offset), code, None, _stream()),
               "gl_gmm_fp8_fwd_scatter")


def quant_col_128x1(x: torch.Tensor, q: Optional[torch.Tensor] = None,
                    s: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """bf16 [M, C] (M, C multiples of 128) -> (e4m3 [M, C], fp32 scales
    [M/128, C]): one absmax scale per 128 rows of a column.  Replaces
    qpl.quantize(grad, channelwise_axes=[1], tiled_axes={0: 128}) (:135-141)
    and, untransposed, the lhs_t quantisation of the forward (:92-99)."""
    _need_cuda(x)
    if x.dtype != torch.bfloat16 or x.dim() != 2:
        raise ValueError("quant_col_128x1 expects a 2-D bf16 tensor")
    M, C = x.shape
    q = _out(q, (M, C), FP8, x.device, "q")
    s = _out(s, (M // TILE, C), torch.float32, x.device, "s")
    lib = _lib.load()
    _lib.check(lib.gl_quant_col_128x1(x.data_ptr(), M, C, q.data_ptr(), s.data_ptr(), None,
                                      _stream()), "gl_quant_col_128x1")
    return q, s


def gmm_fp8_dlhs(dq: torch.Tensor, ds: torch.Tensor, b_q: torch.Tensor, b_s: torch.Tensor,
                 group_sizes: torch.Tensor, out_dtype: torch.dtype = torch.bfloat16,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """dlhs [M, K] = dout x rhs^T per group from dout quantised 1x128 along N
    (quant_act_1x128 of grad [M, N]) and the forward's weight QArray; replaces
    tokamax gmm(..., transpose_rhs=True) (:143-153).  Rows at or beyond
    sum(group_sizes) are left as they are in `out` (zeroed when allocated)."""
    _need_cuda(dq, ds, b_q, b_s, group_sizes)
    M, N = dq.shape
    G, K, N2 = b_q.shape
    if N2 != N:
        raise ValueError(f"N mismatch: dout {N} vs rhs {N2}")
    if out is None:
        out = torch.zeros((M, K), dtype=out_dtype, device=dq.device)
    code = _lib.GL_OUT_F32 if out.dtype == torch.float32 else _lib.GL_OUT_BF16
    lib = _lib.load()
    _lib.check(lib.gl_gmm_fp8_dlhs(dq.data_ptr(), ds.data_ptr(), b_q.data_ptr(), b_s.data_ptr(),
                                   group_sizes.data_ptr(), G, M, K, N, out.data_ptr(), code, None,
                                   _stream()), "gl_gmm_fp8_dlhs")
    return out


def tgmm_fp8(lq: torch.Tensor, ls: torch.Tensor, dq: torch.Tensor, ds: torch.Tensor,
             group_sizes: torch.Tensor, out_dtype: torch.dtype = torch.bfloat16,
             out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """drhs [G, K, N] = per group lhs^T x dout over the group's rows, both
    quantised by quant_col_128x1; replaces tokamax tgmm (:155-165).  Empty
    groups give zeros."""
    _need_cuda(lq, ls, dq, ds, group_sizes)
    M, K = lq.shape
    N = dq.shape[1]
    G = group_sizes.numel()
    if group_sizes.dtype != torch.int32:
        raise ValueError("group_sizes must be int32")
    if out is None:
        out = torch.empty((G, K, N), dtype=out_dtype, device=lq.device)
    code = _lib.GL_OUT_F32 if out.dtype == torch.float32 else _lib.GL_OUT_BF16
    lib = _lib.load()
    _lib.check(lib.gl_tgmm_fp8(lq.data_ptr(), ls.data_ptr(), dq.data_ptr(), ds.data_ptr(),
                               group_sizes.data_ptr(), G, M, K, N, out.data_ptr(), code, None,
                               _stream()), "gl_tgmm_fp8")
    return out


def gmm_fp8_blockwise_bwd(lhs: torch.Tensor, rhs: torch.Tensor, group_sizes: torch.Tensor,
                          grad: torch.Tensor, rhs_q: Optional[Tuple[torch.Tensor, torch.Tensor]] = None
                          ) -> Tuple[torch.Tensor, torch.Tensor]:
    """(dlhs, drhs) of `gmm_fp8_blockwise(lhs, rhs, group_sizes)` for the
    output gradient `grad` [M, N] (KE/examples/kernels/gmm_fp8_blockwise.py
    :123-169): dout quantised 1x128 along N for dlhs and 128x1 along M for
    drhs, lhs quantised 128x1 along M, the forward's weight QArray (passed as
    `rhs_q` or recomputed).  dlhs has lhs's dtype, drhs rhs's (bf16)."""
    if grad.dtype != torch.bfloat16:
        grad = grad.to(torch.bfloat16)
    grad = grad.contiguous()
    b_q, b_s = rhs_q if rhs_q is not None else quant_w_128x128(rhs)
    dq1, ds1 = quant_act_1x128(grad)
    dlhs = gmm_fp8_dlhs(dq1, ds1, b_q, b_s, group_sizes, out_dtype=lhs.dtype)
    del dq1, ds1
    lq, ls = quant_col_128x1(lhs)
    dq2, ds2 = quant_col_128x1(grad)
    drhs = tgmm_fp8(lq, ls, dq2, ds2, group_sizes, out_dtype=rhs.dtype)
    return dlhs, drhs


class _GmmFp8Blockwise(torch.autograd.Function):
    """custom-VJP pair of the template (gmm_fp8_blockwise.py:71-78)."""

    @staticmethod
    def forward(ctx, lhs, rhs, group_sizes, out_dtype):
        a_q, a_s = quant_act_1x128(lhs)
        b_q, b_s = quant_w_128x128(rhs)
        out = gmm_fp8_fwd(a_q, a_s, b_q, b_s, group_sizes, out_dtype=out_dtype)
        _zero_tail_rows(out, group_sizes)
        ctx.save_for_backward(lhs, rhs, group_sizes, b_q, b_s)
        return out

    @staticmethod
    def backward(ctx, grad):
        lhs, rhs, group_sizes, b_q, b_s = ctx.saved_tensors
        dlhs, drhs = gmm_fp8_blockwise_bwd(lhs, rhs, group_sizes, grad, rhs_q=(b_q, b_s))
        return dlhs, drhs, None, None


_SIDE_STREAMS = {}


def _side_streams(device: torch.device):
    """Three per-device streams (copy-in, compute, copy-out) for the host op."""
    key = device.index if device.index is not None else torch.cuda.current_device()
    if key not in _SIDE_STREAMS:
        with torch.cuda.device(key):
            _SIDE_STREAMS[key] = (torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream())
    return _SIDE_STREAMS[key]


def _plan_chunks(sizes, chunks: int, min_rows: int = 1024):
    """Row ranges [r0, r1) of about equal size over the assigned rows, each
    with the index of its first group and its per-group row counts (a group
    may be split between consecutive chunks)."""
    import numpy as np
    sizes = np.asarray(sizes, dtype=np.int64)
    off = np.concatenate([[0], np.cumsum(sizes)])
    total = int(off[-1])
    n = max(1, min(chunks, total // min_rows if total >= min_rows else 1))
    bounds = [total * i // n for i in range(n + 1)]
    plan = []
    for r0, r1 in zip(bounds[:-1], bounds[1:]):
        if r1 <= r0:
            continue
        g_a = int(np.searchsorted(off, r0, side="right") - 1)
        g_b = int(np.searchsorted(off, r1, side="left") - 1)
        g_a = max(g_a, 0)
        sub = [max(0, min(int(off[g + 1]), r1) - max(int(off[g]), r0)) for g in range(g_a, g_b + 1)]
        plan.append((r0, r1, g_a, sub))
    return plan, total


def gmm_fp8_blockwise_host(lhs: torch.Tensor, rhs: torch.Tensor, group_sizes: torch.Tensor,
                           out: Optional[torch.Tensor] = None,
                           out_dtype: torch.dtype = torch.bfloat16,
                           chunks: int = 16, min_chunk_rows: int = 1024) -> torch.Tensor:
    """`gmm_fp8_blockwise` for activations that arrive in host memory (the
    serving case): `lhs` bf16 [M, K] in pinned host memory, `rhs` bf16
    [G, K, N] on the GPU (the weights), `group_sizes` int32 [G] (host or
    device); returns `out` [M, N] in pinned host memory (allocated when not
    given).  The activation rows go to the device in `chunks` row ranges on a
    copy stream (ranges of at least `min_chunk_rows` rows) while the ranges
    already there are quantised and multiplied on
    a compute stream, and finished output rows go back on a third stream, so
    the PCIe transfers overlap the kernels.  The work is ordered after the
    current stream and the current stream waits for all of it: the result is
    valid once the current stream has been synchronised.  Same numbers as
    `gmm_fp8_blockwise` (row ranges are computed by the same kernel).
    """
    if lhs.is_cuda or not lhs.is_pinned():
        raise ValueError("lhs must be a pinned host tensor")
    _need_cuda(rhs)
    if lhs.dtype != torch.bfloat16 or rhs.dtype != torch.bfloat16 or lhs.dim() != 2 or rhs.dim() != 3:
        raise ValueError("lhs bf16 [M, K] and rhs bf16 [G, K, N] expected")
    M, K = lhs.shape
    G, K2, N = rhs.shape
    if K2 != K:
        raise ValueError(f"K mismatch: lhs {K} vs rhs {K2}")
    if group_sizes.dtype != torch.int32 or group_sizes.numel() != G:
        raise ValueError("group_sizes must be int32 [G]")
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, pin_memory=True)
    elif out.is_cuda or not out.is_pinned() or tuple(out.shape) != (M, N) or out.dtype != out_dtype:
        raise ValueError("out must be a pinned host tensor [M, N] of out_dtype")
    sizes = group_sizes.cpu().numpy()
    if (sizes < 0).any() or int(sizes.sum()) > M:
        raise ValueError("group_sizes must be non-negative with sum <= M")
    plan, total = _plan_chunks(sizes, chunks, min_chunk_rows)
    if total < M:
        out[total:].zero_()  # rows that belong to no group
    if total == 0:
        return out
    dev = rhs.device
    s_in, s_c, s_out = _side_streams(dev)
    cur = torch.cuda.current_stream(dev)
    start = cur.record_event()
    for st in (s_in, s_c, s_out):
        st.wait_event(start)
    tab = torch.zeros((len(plan), G), dtype=torch.int32, pin_memory=True)
    for c, (_, _, _, sub) in enumerate(plan):
        tab[c, :len(sub)] = torch.tensor(sub, dtype=torch.int32)
    lhs_d = torch.empty((M, K), dtype=torch.bfloat16, device=dev)
    a_q = torch.empty((M, K), dtype=FP8, device=dev)
    a_s = torch.empty((M, K // TILE), dtype=torch.float32, device=dev)
    out_d = torch.empty((M, N), dtype=out_dtype, device=dev)
    with torch.cuda.stream(s_in):
        tab_d = tab.to(dev, non_blocking=True)
    tab_ready = s_in.record_event()
    with torch.cuda.stream(s_c):
        b_q, b_s = quant_w_128x128(rhs)
        s_c.wait_event(tab_ready)
    for c, (r0, r1, g_a, sub) in enumerate(plan):
        g_b = g_a + len(sub)
        with torch.cuda.stream(s_in):
            lhs_d[r0:r1].copy_(lhs[r0:r1], non_blocking=True)
            landed = s_in.record_event()
        with torch.cuda.stream(s_c):
            s_c.wait_event(landed)
            quant_act_1x128(lhs_d[r0:r1], a_q[r0:r1], a_s[r0:r1])
            gmm_fp8_fwd(a_q[r0:r1], a_s[r0:r1], b_q[g_a:g_b], b_s[g_a:g_b], tab_d[c, :len(sub)],
                        out=out_d[r0:r1])
            done = s_c.record_event()
        with torch.cuda.stream(s_out):
            s_out.wait_event(done)
            out[r0:r1].copy_(out_d[r0:r1], non_blocking=True)
    # keep the device buffers alive for the side streams, then join them
    for t in (lhs_d, a_q, a_s, out_d, tab_d, b_q, b_s):
        for st in (s_in, s_c, s_out):
            t.record_stream(st)
    for st in (s_in, s_c, s_out):
        cur.wait_stream(st)
    return out


# ---------------------------------------------------------------------------
# Chunked GLA forward
# ---------------------------------------------------------------------------
class GLAForward(tuple):
    """Result of chunk_gla_fwd, unpackable as the reference's
    (g_cumsum, A, h, o).  The fused kernel keeps g_cumsum and A on chip, so
    those entries are None unless asked for with output_intermediates=True
    (then fp32 [B, T, H, K] and fp32 [B, T, H, 64], from a separate kernel);
    h (the bf16 state before every chunk, [B, T/64, H, K, V]) is returned
    when asked for with output_states=True, else None; the final state is
    `.ht`."""

    def __new__(cls, o: torch.Tensor, ht: Optional[torch.Tensor], h: Optional[torch.Tensor] = None,
                g_cumsum: Optional[torch.Tensor] = None, A: Optional[torch.Tensor] = None):
        self = tuple.__new__(cls, (g_cumsum, A, h, o))
        self.ht = ht
        return self

    @property
    def g_cumsum(self) -> Optional[torch.Tensor]:
        return self[0]

    @property
    def A(self) -> Optional[torch.Tensor]:
        return self[1]

    @property
    def o(self) -> torch.Tensor:
        return self[3]

    @property
    def h(self) -> Optional[torch.Tensor]:
        return self[2]


def _gla_check(q, k, v, g_gamma, g, h0):
    _need_cuda(q, k, v, g_gamma, g, h0)
    B, T, H, K = q.shape
    V = v.shape[-1]
    for name, t in (("q", q), ("k", k), ("v", v)):
        if t.dtype != torch.bfloat16:
            raise ValueError(f"{name} must be bf16")
    if g is not None and (g.dtype != torch.float32 or tuple(g.shape) != (B, T, H, K)):
        raise ValueError("g must be fp32 [B, T, H, K]")
    if g_gamma is not None and (g_gamma.dtype != torch.float32 or g_gamma.numel() != H):
        raise ValueError("g_gamma must be fp32 [H]")
    if h0 is not None and (h0.dtype != torch.float32 or tuple(h0.shape) != (B, H, K, V)):
        raise ValueError("h0 must be fp32 [B, H, K, V]")
    return B, T, H, K, V


def chunk_gla_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                  g_gamma: Optional[torch.Tensor], scale: float, chunk_size: int = 64, *,
                  g: Optional[torch.Tensor] = None, h0: Optional[torch.Tensor] = None,
                  output_final_state: bool = False, output_states: bool = False,
                  output_intermediates: bool = False, exact_intra: bool = True,
                  o: Optional[torch.Tensor] = None,
                  ht: Optional[torch.Tensor] = None,
                  h: Optional[torch.Tensor] = None) -> GLAForward:
    """Chunked GLA forward (KE/examples/kernels/chunk_gla.py:258-273), fused
    into one kernel.  Either the per-head constant gate `g_gamma` [H] (the
    reference template's mode) or the per-key log-gate `g` [B, T, H, K] (raw,
    chunk-local cumsum taken in-kernel; semantics of
    KE/upstream/fused_chunk_simple_gla/common_chunk_h.py:330-334) is used.
    output_states=True also returns the per-chunk states h (bf16), the
    residual of the backward.  output_intermediates=True also returns
    g_cumsum (fp32 [B, T, H, K]) and the unmasked intra-chunk A (fp32
    [B, T, H, 64]) as the reference's first two outputs, computed by a
    separate fp32 kernel (one more pass over q, k and g).
    exact_intra=True (the default) feeds tril(A) to the intra-chunk product
    as a bf16 hi + lo pair (A to ~2^-17 relative, the fp32 A of the
    template's output kernel, chunk_gla.py:208-212); exact_intra=False
    rounds it to bf16 once (the operand precision of the reference jnp
    oracle's einsum at TPU default precision, chunk_gla_ref.py:96-97),
    about 10 % faster.  o, ht and h may be given
    preallocated.
    """
    B, T, H, K, V = _gla_check(q, k, v, g_gamma, g, h0)
    if o is None:
        o = torch.empty((B, T, H, V), dtype=torch.bfloat16, device=q.device)
    if output_final_state and ht is None:
        ht = torch.empty((B, H, K, V), dtype=torch.float32, device=q.device)
    lib = _lib.load()
    # Few (batch, head) pairs: the library splits the sequence and needs a
    # workspace for the per-segment states (0 bytes otherwise).
    ws_bytes = lib.gl_chunk_gla_fwd_workspace_bytes(B, T, H, K, V, chunk_size)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device) if ws_bytes else None
    if output_states:
        h = _out(h, (B, T // chunk_size, H, K, V), torch.bfloat16, q.device, "h")
    flags = 0 if exact_intra else _lib.GL_GLA_BF16_INTRA
    _lib.check(lib.gl_chunk_gla_fwd_ex(q.data_ptr(), k.data_ptr(), v.data_ptr(), _ptr(g),
                                       _ptr(g_gamma), _ptr(h0), float(scale), B, T, H, K, V,
                                       chunk_size, o.data_ptr(), _ptr(ht),
                                       h.data_ptr() if output_states else None, _ptr(ws), ws_bytes,
                                       flags, None, _stream()),
               "gl_chunk_gla_fwd_states" if output_states else "gl_chunk_gla_fwd")
    g_cumsum = A = None
    if output_intermediates:
        g_cumsum = torch.empty((B, T, H, K), dtype=torch.float32, device=q.device)
        A = torch.empty((B, T, H, chunk_size), dtype=torch.float32, device=q.device)
        _lib.check(lib.gl_chunk_gla_fwd_intermediates(q.data_ptr(), k.data_ptr(), _ptr(g),
                                                      _ptr(g_gamma), float(scale), B, T, H, K,
                                                      chunk_size, g_cumsum.data_ptr(), A.data_ptr(),
                                                      None, _stream()),
                   "gl_chunk_gla_fwd_intermediates")
    return GLAForward(o, ht if output_final_state else None, h, g_cumsum, A)


def chunk_gla_fwd_scatter(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                          g_gamma: Optional[torch.Tensor], scale: float, chunk_size: int = 64, *,
                          outs, g: Optional[torch.Tensor] = None, h0: Optional[torch.Tensor] = None,
                          ht: Optional[torch.Tensor] = None, exact_intra: bool = True) -> None:
    """chunk_gla_fwd whose output o is stored into every buffer of `outs`
    (tensors on this device, or integer device addresses of peer-mapped
    buffers such as shard.PeerBuffers.ptrs plus an offset), each holding o's
    layout [B, T, H, V] bf16.  Used to assemble a head-sharded forward on
    every rank inside the kernel; the caller synchronises the ranks after it.
    ht (fp32 [B, H, K, V]) receives the final state when given."""
    B, T, H, K, V = _gla_check(q, k, v, g_gamma, g, h0)
    ptrs = [o.data_ptr() if isinstance(o, torch.Tensor) else int(o) for o in outs]
    for o in outs:
        if isinstance(o, torch.Tensor) and (o.dtype != torch.bfloat16 or tuple(o.shape) != (B, T, H, V)
                                            or not o.is_contiguous()):
            raise ValueError("each output must be a contiguous bf16 [B, T, H, V] tensor")
    if ht is not None and (ht.dtype != torch.float32 or tuple(ht.shape) != (B, H, K, V)):
        raise ValueError("ht must be fp32 [B, H, K, V]")
    lib = _lib.load()
    ws_bytes = lib.gl_chunk_gla_fwd_workspace_bytes(B, T, H, K, V, chunk_size)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device) if ws_bytes else None
    import ctypes
    arr = (ctypes.c_void_p * len(ptrs))(*ptrs)
    flags = 0 if exact_intra else _lib.GL_GLA_BF16_INTRA
    _lib.check(lib.gl_chunk_gla_fwd_scatter(q.data_ptr(), k.data_ptr(), v.data_ptr(), _ptr(g),
                                            _ptr(g_gamma), _ptr(h0), float(scale), B, T, H, K, V,
                                            chunk_size, ctypes.cast(arr, ctypes.c_void_p), len(ptrs),
                                            _ptr(ht), _ptr(ws), ws_bytes, flags, None, _stream()),
               "gl_chunk_gla_fwd_scatter")


def chunk_gla_bwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, do: torch.Tensor,
                  h: torch.Tensor, g_gamma: Optional[torch.Tensor], scale: float,
                  chunk_size: int = 64, *, g: Optional[torch.Tensor] = None,
                  dht: Optional[torch.Tensor] = None, output_dh0: bool = False,
                  dq: Optional[torch.Tensor] = None, dk: Optional[torch.Tensor] = None,
                  dv: Optional[torch.Tensor] = None, workspace: Optional[torch.Tensor] = None
                  ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, Optional[torch.Tensor]]:
    """Backward of chunk_gla_fwd: (dq, dk, dv, dh0) for the output gradient
    `do` (and the final-state gradient `dht`), from the forward's per-chunk
    states `h` (chunk_gla_fwd(..., output_states=True).h).  Replaces _bwd of
    KE/examples/kernels/chunk_gla.py:446-453 (reverse dh scan :281-305, fused
    dq/dk/dv :313-426); the gate gets no gradient, as there.  dq, dk, dv and
    the uint8 `workspace` (chunk_gla_bwd_workspace_bytes) may be given
    preallocated."""
    B, T, H, K, V = _gla_check(q, k, v, g_gamma, g, dht)
    _need_cuda(do, h)
    if do.dtype != torch.bfloat16 or tuple(do.shape) != (B, T, H, V):
        raise ValueError("do must be bf16 [B, T, H, V]")
    if h.dtype != torch.bfloat16 or tuple(h.shape) != (B, T // chunk_size, H, K, V):
        raise ValueError("h must be bf16 [B, T/chunk, H, K, V]")
    lib = _lib.load()
    dq = _out(dq, q.shape, torch.bfloat16, q.device, "dq")
    dk = _out(dk, k.shape, torch.bfloat16, q.device, "dk")
    dv = _out(dv, v.shape, torch.bfloat16, q.device, "dv")
    dh0 = torch.empty((B, H, K, V), dtype=torch.float32, device=q.device) if output_dh0 else None
    ws_bytes = lib.gl_chunk_gla_bwd_workspace_bytes(B, T, H, K, V, chunk_size)
    if ws_bytes == 0:
        raise ValueError("gl_chunk_gla_bwd: unsupported shape")
    if workspace is None:
        workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
    elif workspace.dtype != torch.uint8 or workspace.numel() < ws_bytes or not workspace.is_cuda:
        raise ValueError(f"workspace must be a CUDA uint8 tensor of at least {ws_bytes} bytes")
    ws = workspace
    _lib.check(lib.gl_chunk_gla_bwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), _ptr(g), _ptr(g_gamma),
                                    h.data_ptr(), do.data_ptr(), _ptr(dht), float(scale), B, T, H, K,
                                    V, chunk_size, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
                                    _ptr(dh0), ws.data_ptr(), ws.numel(), None, _stream()),
               "gl_chunk_gla_bwd")
    return dq, dk, dv, dh0


def chunk_gla_bwd_workspace_bytes(B: int, T: int, H: int, K: int = 128, V: int = 128,
                                  chunk_size: int = 64) -> int:
    """Device workspace chunk_gla_bwd needs for this shape on the current device."""
    return int(_lib.load().gl_chunk_gla_bwd_workspace_bytes(B, T, H, K, V, chunk_size))


class _ChunkGLA(torch.autograd.Function):
    """custom-VJP pair of the template (chunk_gla.py:434-456): the forward
    keeps q, k, v, the gate and the per-chunk states; the backward returns
    dq, dk, dv (and dh0 when h0 is given)."""

    @staticmethod
    def forward(ctx, q, k, v, g_gamma, g, h0, scale, chunk_size, exact_intra):
        res = chunk_gla_fwd(q, k, v, g_gamma, scale, chunk_size, g=g, h0=h0, output_states=True,
                            exact_intra=exact_intra)
        ctx.save_for_backward(q, k, v, g_gamma, g, res.h)
        ctx.scale, ctx.chunk_size, ctx.has_h0 = scale, chunk_size, h0 is not None
        return res.o

    @staticmethod
    def backward(ctx, do):
        q, k, v, g_gamma, g, h = ctx.saved_tensors
        dq, dk, dv, dh0 = chunk_gla_bwd(q, k, v, do.to(torch.bfloat16).contiguous(), h, g_gamma,
                                        ctx.scale, ctx.chunk_size, g=g, output_dh0=ctx.has_h0)
        return dq, dk, dv, None, None, dh0, None, None, None


def chunk_gla(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g_gamma: Optional[torch.Tensor],
              scale: float, chunk_size: int = 64, *, g: Optional[torch.Tensor] = None,
              h0: Optional[torch.Tensor] = None, exact_intra: bool = True) -> torch.Tensor:
    """`chunk_gla(q, k, v, g_gamma, scale, chunk_size)`
    (KE/examples/kernels/chunk_gla.py:434-456): returns o (bf16),
    differentiable in q, k, v (and h0) when any of them requires grad.
    exact_intra as in chunk_gla_fwd."""
    if torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in (q, k, v, h0)):
        return _ChunkGLA.apply(q, k, v, g_gamma, g, h0, scale, chunk_size, exact_intra)
    return chunk_gla_fwd(q, k, v, g_gamma, scale, chunk_size, g=g, h0=h0, exact_intra=exact_intra).o


def device_status() -> int:
    """Synchronises the current stream and returns (and clears) the library's
    device error word: 0 when no kernel reported a problem."""
    return _lib.device_status(_stream())
