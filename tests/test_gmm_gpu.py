"""Parity of the sm_100a grouped FP8 matmul and its quantisers against the CPU
oracle, through the C ABI (glaucis_b200.ops is a thin ctypes wrapper).

The launcher reads GLAUCIS_GMM_VARIANT at every call, so each test runs once
per kernel variant.

Tolerances: quantisers are bit-exact (bytes and fp32 scales).  The matmul is
checked element-wise with |gpu - ref| <= 1e-2 * |ref| + 1e-3 * rms(ref), i.e.
within rtol 1e-2 of the dequantised fp32 reference (the atol term only covers
entries that cancel to ~0, where fp32 summation order dominates).
"""
import os

import numpy as np
import pytest
import torch

from glaucis_b200 import configs, ops
from oracle import gmm_oracle as O
from tests.helpers import assert_close, rel_fro

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
RTOL, ATOL_FRAC = 1e-2, 1e-3
VARIANTS = ["256", "128", "pair"]


@pytest.fixture(autouse=True, params=VARIANTS)
def kernel_variant(request, monkeypatch):
    """Every matmul test runs on each kernel variant: the 1-SM kernel with
    256- and 128-column tiles and the CTA-pair kernel (256 x 256 tiles)."""
    monkeypatch.setenv("GLAUCIS_GMM_VARIANT", request.param)
    return request.param


def _np_bytes(t):
    return t.view(torch.uint8).cpu().numpy()


def _gmm_case(cuda, G, M, K, N, sizes, seed=0, out_dtype=torch.bfloat16, zero_block=False):
    g = torch.Generator().manual_seed(seed)
    lhs = torch.randn((M, K), generator=g).to(torch.bfloat16)
    rhs = (torch.randn((G, K, N), generator=g) * 0.02).to(torch.bfloat16)
    if zero_block:
        lhs[min(1, M - 1), :128] = 0
    gs = torch.tensor(sizes, dtype=torch.int32)
    a_q, a_s = ops.quant_act_1x128(lhs.to(cuda))
    b_q, b_s = ops.quant_w_128x128(rhs.to(cuda))
    out = ops.gmm_fp8_fwd(a_q, a_s, b_q, b_s, gs.to(cuda), out_dtype=out_dtype)
    assert ops.device_status() == 0
    oa_q, oa_s = O.quant_act_1x128(lhs.float().numpy())
    ob_q, ob_s = O.quant_w_128x128(rhs.float().numpy())
    assert np.array_equal(_np_bytes(a_q), oa_q), "activation e4m3 bytes differ"
    assert np.array_equal(a_s.cpu().numpy(), oa_s), "activation scales differ"
    assert np.array_equal(_np_bytes(b_q), ob_q), "weight e4m3 bytes differ"
    assert np.array_equal(b_s.cpu().numpy(), ob_s), "weight scales differ"
    ref = O.gmm_fwd(oa_q, oa_s, ob_q, ob_s, gs.numpy())
    total = int(sum(sizes))
    got = out.float().cpu().numpy()
    assert_close(got[:total], ref[:total], RTOL, ATOL_FRAC, what=f"gmm G={G} M={M} K={K} N={N}")
    return got, ref


def test_quant_act_bit_exact(cuda):
    g = torch.Generator().manual_seed(1)
    x = torch.randn((333, 1024), generator=g) * torch.logspace(-3, 2, 1024)[None, :]
    x[5, 128:256] = 0
    x[7, 0] = 1e30
    x = x.to(torch.bfloat16)
    q, s = ops.quant_act_1x128(x.to(cuda))
    rq, rs = O.quant_act_1x128(x.float().numpy())
    assert np.array_equal(_np_bytes(q), rq)
    assert np.array_equal(s.cpu().numpy(), rs)


def test_quant_w_bit_exact(cuda):
    g = torch.Generator().manual_seed(2)
    w = (torch.randn((3, 256, 384), generator=g) * 0.02).to(torch.bfloat16)
    w[1, :128, 128:256] = 0
    q, s = ops.quant_w_128x128(w.to(cuda))
    rq, rs = O.quant_w_128x128(w.float().numpy())
    assert np.array_equal(_np_bytes(q), rq)
    assert np.array_equal(s.cpu().numpy(), rs)


def test_gmm_single_group_single_tile(cuda):
    _gmm_case(cuda, 1, 128, 128, 256, [128])


def test_gmm_small_config(cuda):
    cfg = configs.GMM_CONFIGS["gmm_small"]
    sizes = configs.group_sizes(cfg.routing, cfg.G, cfg.M, seed=0).tolist()
    _gmm_case(cuda, cfg.G, cfg.M, cfg.K, cfg.N, sizes, seed=0)


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_gmm_ragged_empty_partial(cuda, out_dtype):
    # empty groups (first, middle, last), 1-row groups, partial tiles, a
    # group spanning several tiles, N % 256 == 128, sum(sizes) < M
    sizes = [0, 1, 300, 0, 129, 127, 2, 0]
    _gmm_case(cuda, len(sizes), 600, 384, 384, sizes, seed=3, out_dtype=out_dtype,
              zero_block=True)


def test_gmm_pair_tile_edges(cuda):
    # 256-row tiles: a group of exactly 128 rows (second CTA of a pair has no
    # valid row), 255 / 257 rows (second CTA partial / a 1-row second tile),
    # several 256-row tiles, and N = 640 (the last 256-column tile is half
    # outside the weight matrix).
    sizes = [128, 256, 257, 255, 0, 512, 384]
    _gmm_case(cuda, len(sizes), 1800, 256, 640, sizes, seed=5)


def test_gmm_golden_fixture(cuda):
    d = np.load(os.path.join(GOLDEN, "gmm_small_ragged.npz"))
    lhs = torch.from_numpy(d["lhs_bf16"].view(np.int16)).view(torch.bfloat16)
    rhs = torch.from_numpy(d["rhs_bf16"].view(np.int16)).view(torch.bfloat16)
    gs = torch.from_numpy(d["group_sizes"]).to(cuda)
    a_q, a_s = ops.quant_act_1x128(lhs.to(cuda))
    b_q, b_s = ops.quant_w_128x128(rhs.to(cuda))
    assert np.array_equal(_np_bytes(a_q), d["a_q"]) and np.array_equal(a_s.cpu().numpy(), d["a_s"])
    assert np.array_equal(_np_bytes(b_q), d["b_q"]) and np.array_equal(b_s.cpu().numpy(), d["b_s"])
    out = ops.gmm_fp8_fwd(a_q, a_s, b_q, b_s, gs, out_dtype=torch.float32)
    total = int(d["group_sizes"].sum())
    assert_close(out.cpu().numpy()[:total], d["out"][:total], RTOL, ATOL_FRAC, what="golden")


def test_gmm_public_op_matches_oracle_end_to_end(cuda):
    cfg = configs.GMMConfig("t", G=5, M=700, K=512, N=512, routing="multinomial")
    lhs, rhs, gs = configs.make_gmm_inputs(cfg, device="cpu", seed=7)
    got = ops.gmm_fp8_blockwise(lhs.to(cuda), rhs.to(cuda), gs.to(cuda))
    assert got.dtype == torch.float32 and got.shape == (700, 512)
    ref = O.gmm_fp8_blockwise(lhs.float().numpy(), rhs.float().numpy(), gs.numpy())
    assert_close(got.cpu().numpy(), ref, RTOL, ATOL_FRAC, what="gmm_fp8_blockwise")
    bf = O.gmm_bf16_reference(lhs.float().numpy(), rhs.float().numpy(), gs.numpy())
    assert rel_fro(got.cpu().numpy(), bf) < 0.15


def test_gmm_every_group_empty(cuda):
    # no rows in any group: no tiles; the public op returns an all-zero output
    lhs = torch.randn((256, 256)).to(torch.bfloat16).to(cuda)
    rhs = (torch.randn((3, 256, 384)) * 0.02).to(torch.bfloat16).to(cuda)
    gs = torch.zeros(3, dtype=torch.int32, device=cuda)
    out = ops.gmm_fp8_blockwise(lhs, rhs, gs)
    assert ops.device_status() == 0
    assert out.shape == (256, 384) and torch.count_nonzero(out) == 0


def test_gmm_tail_rows_zero_in_public_op(cuda):
    lhs = torch.randn((300, 256)).to(torch.bfloat16).to(cuda)
    rhs = (torch.randn((2, 256, 256)) * 0.02).to(torch.bfloat16).to(cuda)
    gs = torch.tensor([100, 150], dtype=torch.int32, device=cuda)
    out = ops.gmm_fp8_blockwise(lhs, rhs, gs)
    assert torch.count_nonzero(out[250:]) == 0


@pytest.mark.parametrize("chunks", [1, 3, 7])
def test_gmm_host_pipeline_matches_device_op(cuda, chunks):
    # Activations in pinned host memory, streamed in row chunks (groups split
    # between chunks, an empty group, rows past sum(group_sizes)): the result
    # is the device op's result bit for bit.
    g = torch.Generator().manual_seed(11)
    G, M, K, N = 6, 3000, 256, 384
    sizes = [700, 0, 1100, 64, 900, 100]          # sum 2864 < M
    lhs = torch.randn((M, K), generator=g).to(torch.bfloat16)
    rhs = (torch.randn((G, K, N), generator=g) * 0.02).to(torch.bfloat16).to(cuda)
    gs = torch.tensor(sizes, dtype=torch.int32)
    ref = ops.gmm_fp8_blockwise(lhs.to(cuda), rhs, gs.to(cuda), out_dtype=torch.bfloat16)
    out = ops.gmm_fp8_blockwise_host(lhs.pin_memory(), rhs, gs, chunks=chunks, min_chunk_rows=128)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    assert out.is_pinned() and not out.is_cuda
    assert torch.equal(out, ref.cpu())


def test_gmm_bad_group_sizes_set_error_word(cuda):
    # The kernel validates group_sizes on the device and reports through the
    # error word instead of reading out of bounds.
    a_q = torch.zeros((256, 128), dtype=torch.float8_e4m3fn, device=cuda)
    a_s = torch.ones((256, 1), dtype=torch.float32, device=cuda)
    b_q = torch.zeros((2, 128, 256), dtype=torch.float8_e4m3fn, device=cuda)
    b_s = torch.ones((2, 1, 2), dtype=torch.float32, device=cuda)
    for bad in ([200, 100], [-1, 10]):
        gs = torch.tensor(bad, dtype=torch.int32, device=cuda)
        ops.gmm_fp8_fwd(a_q, a_s, b_q, b_s, gs)
        assert ops.device_status() == 2
    gs = torch.tensor([100, 100], dtype=torch.int32, device=cuda)
    ops.gmm_fp8_fwd(a_q, a_s, b_q, b_s, gs)
    assert ops.device_status() == 0


@pytest.mark.parametrize("name", ["gmm_moe_up", "gmm_dense_expert"])
def test_gmm_full_size_sampled_rows(cuda, name):
    # Full benchmark shapes on the GPU; the oracle recomputes a sample of rows
    # that covers the first / last row of every group and random interior rows.
    cfg = configs.GMM_CONFIGS[name]
    lhs, rhs, gs = configs.make_gmm_inputs(cfg, device=cuda, seed=0)
    a_q, a_s = ops.quant_act_1x128(lhs)
    b_q, b_s = ops.quant_w_128x128(rhs)
    del rhs
    out = ops.gmm_fp8_fwd(a_q, a_s, b_q, b_s, gs, out_dtype=torch.bfloat16)
    assert ops.device_status() == 0
    sizes = gs.cpu().numpy()
    off = O.group_offsets(sizes)
    rng = np.random.default_rng(0)
    rows = set(rng.integers(0, cfg.M, 96).tolist())
    for g in range(cfg.G):
        if sizes[g]:
            rows.update([int(off[g]), int(off[g + 1] - 1)])
    rows = np.array(sorted(rows))
    gid = np.searchsorted(off, rows, side="right") - 1
    rows_t = torch.from_numpy(rows).to(cuda)
    got = out[rows_t].float().cpu().numpy()
    aq_rows = _np_bytes(a_q[rows_t])
    as_rows = a_s[rows_t].cpu().numpy()
    b_s_n = b_s.cpu().numpy()
    for g in np.unique(gid):
        sel = np.nonzero(gid == g)[0]
        ref = O.gmm_group_rows(aq_rows[sel], as_rows[sel], _np_bytes(b_q[int(g)]), b_s_n[g])
        assert_close(got[sel], ref, RTOL, ATOL_FRAC, what=f"{name} group {g}")


def test_gmm_scatter_writes_every_output_at_the_row_offset(cuda):
    # the epilogue that assembles an expert-sharded output on every rank:
    # here two local buffers stand in for the ranks' buffers
    cfg = configs.GMMConfig("t", G=5, M=640, K=512, N=384, routing="uniform_one_empty")
    lhs, rhs, gs = configs.make_gmm_inputs(cfg, device=cuda, seed=11)
    a_q, a_s = ops.quant_act_1x128(lhs)
    b_q, b_s = ops.quant_w_128x128(rhs)
    want = ops.gmm_fp8_fwd(a_q, a_s, b_q, b_s, gs, out_dtype=torch.bfloat16)
    off = 256
    outs = [torch.full((off + cfg.M + 128, cfg.N), 7.0, dtype=torch.bfloat16, device=cuda) for _ in range(2)]
    ops.gmm_fp8_fwd_scatter(a_q, a_s, b_q, b_s, gs, [outs[0], outs[1].data_ptr()], off)
    assert ops.device_status() == 0
    rows = int(gs.sum().item())
    for o in outs:
        assert torch.equal(o[off:off + rows], want[:rows])
        assert bool((o[:off] == 7.0).all()) and bool((o[off + rows:] == 7.0).all())


@pytest.mark.parametrize("K,N", [(384, 384), (3072, 256), (3200, 640)])
def test_gmm_bf16_output_is_the_rounded_fp32_output(cuda, K, N):
    # The bf16 output of a call is the fp32 accumulator rounded once, however
    # it leaves the kernel: with short reductions (up to 24 K blocks) whole
    # 32-row warp slices go through shared memory and TMA stores, partial
    # slices (the last rows of a group) and fp32 outputs are stored directly.
    # Both dtypes of the forward and of dlhs must agree bit for bit.
    sizes = [0, 1, 31, 32, 33, 300, 0, 129, 127, 64, 96, 2]
    G, M = len(sizes), 1100
    g = torch.Generator().manual_seed(21)
    lhs = torch.randn((M, K), generator=g).to(torch.bfloat16).to(cuda)
    rhs = (torch.randn((G, K, N), generator=g) * 0.02).to(torch.bfloat16).to(cuda)
    dout = torch.randn((M, N), generator=g).to(torch.bfloat16).to(cuda)
    gs = torch.tensor(sizes, dtype=torch.int32, device=cuda)
    a_q, a_s = ops.quant_act_1x128(lhs)
    b_q, b_s = ops.quant_w_128x128(rhs)
    d_q, d_s = ops.quant_act_1x128(dout)
    total = sum(sizes)
    for name, fn in (("forward", lambda dt: ops.gmm_fp8_fwd(a_q, a_s, b_q, b_s, gs, out_dtype=dt)),
                     ("dlhs", lambda dt: ops.gmm_fp8_dlhs(d_q, d_s, b_q, b_s, gs, out_dtype=dt))):
        o16 = fn(torch.bfloat16)
        o32 = fn(torch.float32)
        assert ops.device_status() == 0
        assert torch.equal(o16[:total], o32[:total].to(torch.bfloat16)), name


def test_gmm_many_small_groups(cuda):
    # 700 groups of 0-24 rows (a third of them empty): one tile per non-empty
    # group, most of each tile padding, the tile table near its 1024-group
    # limit, several tiles per CTA
    rng = np.random.default_rng(77)
    sizes = [int(x) if rng.random() > 0.33 else 0 for x in rng.integers(1, 25, size=700)]
    _gmm_case(cuda, len(sizes), sum(sizes) + 5, 256, 384, sizes, seed=77)


@pytest.mark.parametrize("seed", range(6))
def test_gmm_random_ragged_shapes(cuda, seed):
    # Seeded random problems: group counts from 1 to 40 with empty groups and
    # groups of 1-300 rows, unassigned tail rows, K and N from 128 to 640,
    # bf16 or fp32 output.
    rng = np.random.default_rng(100 + seed)
    G = int(rng.integers(1, 41))
    sizes = [int(x) if rng.random() > 0.25 else 0 for x in rng.integers(1, 301, size=G)]
    M = max(1, sum(sizes) + int(rng.integers(0, 200)))
    K = 128 * int(rng.integers(1, 6))
    N = 128 * int(rng.integers(1, 6))
    out_dtype = torch.float32 if seed % 2 else torch.bfloat16
    _gmm_case(cuda, G, M, K, N, sizes, seed=seed, out_dtype=out_dtype)
