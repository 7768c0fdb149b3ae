"""Parity of the grouped-matmul backward (dlhs and drhs kernels, the 128x1
column quantiser, the autograd path of gmm_fp8_blockwise) against the CPU
oracle (oracle/gmm_bwd_oracle.py), through the C ABI.

Tolerances: the quantiser is bit-exact; dlhs and drhs element-wise within
|gpu - ref| <= 1e-2 * |ref| + 1e-3 * rms(ref) of the dequantised fp32
reference (as the forward), computed in fp32 and compared on the fp32
outputs; the bf16 outputs of the public op are checked with the bf16
rounding added.  Against the unquantised gradient the reference's own bound
(relative error < 0.5, KE/tests/standalone_gmm_fp8_blockwise_test.py:388-401)
is asserted too.
"""
import numpy as np
import pytest
import torch

from glaucis_b200 import ops
from oracle import gmm_bwd_oracle as B
from oracle import gmm_oracle as O
from tests.helpers import assert_close, rel_fro

pytestmark = pytest.mark.gpu
RTOL, ATOL_FRAC = 1e-2, 1e-3


def _bytes(t):
    return t.view(torch.uint8).cpu().numpy()


def _inputs(G, M, K, N, seed):
    g = torch.Generator().manual_seed(seed)
    lhs = torch.randn((M, K), generator=g).to(torch.bfloat16)
    rhs = (torch.randn((G, K, N), generator=g) * 0.02).to(torch.bfloat16)
    grad = torch.randn((M, N), generator=g).to(torch.bfloat16)
    return lhs, rhs, grad


def test_quant_col_bit_exact(cuda):
    g = torch.Generator().manual_seed(3)
    x = torch.randn((384, 256), generator=g) * torch.logspace(-3, 2, 256)[None, :]
    x[:128, 5] = 0          # an all-zero block
    x[200, 7] = 1e30
    x = x.to(torch.bfloat16)
    q, s = ops.quant_col_128x1(x.to(cuda))
    assert ops.device_status() == 0
    rq, rs = B.quant_col_128x1(x.float().numpy())
    assert np.array_equal(_bytes(q), rq)
    assert np.array_equal(s.cpu().numpy(), rs)


def test_quant_col_bit_exact_more_tiles(cuda):
    # 8 x 6 tiles: per-column maxima over 128 rows, scales shared by the
    # column owners, a block small enough for the plain-division path
    # (scale < 2^-64), a block of negative zeros, huge and tiny columns
    g = torch.Generator().manual_seed(11)
    x = torch.randn((1024, 768), generator=g) * torch.logspace(-4, 3, 768)[None, :]
    x[128:256, 9] = torch.randn(128, generator=g) * 1e-30
    x[256:384, 11] = -0.0
    x[512:640, 700:704] *= 1e20
    x = x.to(torch.bfloat16)
    q, s = ops.quant_col_128x1(x.to(cuda))
    assert ops.device_status() == 0
    rq, rs = B.quant_col_128x1(x.float().numpy())
    assert np.array_equal(_bytes(q), rq)
    assert np.array_equal(s.cpu().numpy(), rs)


@pytest.mark.parametrize("sizes,N", [([100, 0, 300, 128, 100], 384), ([512], 256), ([0, 0, 640], 512)])
def test_dlhs_matches_oracle(cuda, sizes, N):
    G, M, K = len(sizes), 640, 384
    lhs, rhs, grad = _inputs(G, M, K, N, seed=1)
    gs = torch.tensor(sizes, dtype=torch.int32)
    b_q, b_s = ops.quant_w_128x128(rhs.to(cuda))
    dq, ds = ops.quant_act_1x128(grad.to(cuda))
    out = ops.gmm_fp8_dlhs(dq, ds, b_q, b_s, gs.to(cuda), out_dtype=torch.float32)
    assert ops.device_status() == 0
    ref = B.gmm_dlhs(_bytes(dq), ds.cpu().numpy(), _bytes(b_q), b_s.cpu().numpy(), sizes)
    total = int(sum(sizes))
    got = out.cpu().numpy()
    assert_close(got[:total], ref[:total], RTOL, ATOL_FRAC, what=f"dlhs {sizes}")
    assert not got[total:].any()


@pytest.mark.parametrize("sizes", [[100, 0, 300, 128, 156, 12, 100, 100],   # partial blocks, empty
                                   [896],                                 # one group, 7 blocks
                                   [0, 5, 0, 123, 640, 0, 128, 0]])
def test_tgmm_matches_oracle(cuda, sizes):
    G, M, K, N = len(sizes), 896, 256, 384
    lhs, rhs, grad = _inputs(G, M, K, N, seed=2)
    gs = torch.tensor(sizes, dtype=torch.int32)
    lq, ls = ops.quant_col_128x1(lhs.to(cuda))
    dq, ds = ops.quant_col_128x1(grad.to(cuda))
    out = ops.tgmm_fp8(lq, ls, dq, ds, gs.to(cuda), out_dtype=torch.float32)
    assert ops.device_status() == 0
    ref = B.tgmm(_bytes(lq), ls.cpu().numpy(), _bytes(dq), ds.cpu().numpy(), sizes)
    got = out.cpu().numpy()
    for g in range(G):
        if sizes[g] == 0:
            assert not got[g].any(), f"empty group {g} must be zero"
        else:
            assert_close(got[g], ref[g], RTOL, ATOL_FRAC, what=f"tgmm group {g} of {sizes}")


def test_autograd_matches_oracle_and_reference_bound(cuda):
    G, M, K, N = 4, 768, 512, 256
    sizes = [200, 0, 312, 256]
    lhs, rhs, grad = _inputs(G, M, K, N, seed=4)
    gs = torch.tensor(sizes, dtype=torch.int32, device=cuda)
    l_d = lhs.to(cuda).requires_grad_(True)
    r_d = rhs.to(cuda).requires_grad_(True)
    out = ops.gmm_fp8_blockwise(l_d, r_d, gs, out_dtype=torch.float32)
    out.backward(grad.to(cuda).float())
    assert ops.device_status() == 0
    f = lambda t: t.float().numpy()
    dl_ref, dr_ref = B.gmm_fp8_blockwise_bwd(f(lhs), f(rhs), sizes, f(grad))
    dl = l_d.grad.float().cpu().numpy()
    dr = r_d.grad.float().cpu().numpy()
    # bf16 outputs: add half an ulp of bf16 to the tolerance
    assert_close(dl, dl_ref, RTOL + 4e-3, ATOL_FRAC, what="dlhs (autograd, bf16)")
    assert_close(dr, dr_ref, RTOL + 4e-3, ATOL_FRAC, what="drhs (autograd, bf16)")
    ul, ur = B.gmm_bwd_unquantised(f(lhs), f(rhs), sizes, f(grad))
    assert rel_fro(dl, ul) < 0.5 and rel_fro(dr, ur) < 0.5


def test_backward_full_size_sampled(cuda):
    # gmm_moe_up at full size on the GPU (dlhs and drhs); the oracle
    # recomputes sampled rows of dlhs (first / last rows of several groups)
    # and whole drhs slabs of sampled experts, each from just the rows it
    # needs.
    from glaucis_b200 import configs
    cfg = configs.GMM_CONFIGS["gmm_moe_up"]
    lhs, rhs, gs = configs.make_gmm_inputs(cfg, device=cuda, seed=0)
    gen = torch.Generator(device=cuda).manual_seed(13)
    grad = torch.randn((cfg.M, cfg.N), generator=gen, device=cuda).to(torch.bfloat16)
    b_q, b_s = ops.quant_w_128x128(rhs)
    del rhs
    dq1, ds1 = ops.quant_act_1x128(grad)
    dlhs = ops.gmm_fp8_dlhs(dq1, ds1, b_q, b_s, gs, out_dtype=torch.float32)
    lq, ls = ops.quant_col_128x1(lhs)
    dq2, ds2 = ops.quant_col_128x1(grad)
    drhs = ops.tgmm_fp8(lq, ls, dq2, ds2, gs, out_dtype=torch.float32)
    assert ops.device_status() == 0
    sizes = gs.cpu().numpy()
    off = np.concatenate([[0], np.cumsum(sizes)])
    nonempty = [g for g in range(cfg.G) if sizes[g] > 0]
    picks = [nonempty[0], nonempty[len(nonempty) // 2], nonempty[-1], int(np.argmax(sizes))]
    for g in picks:
        r0, r1 = int(off[g]), int(off[g + 1])
        rows = sorted({r0, r0 + 1, (r0 + r1) // 2, r1 - 2, r1 - 1} & set(range(r0, r1)))
        ref = B.gmm_dlhs(dq1.view(torch.uint8)[rows].cpu().numpy(), ds1[rows].cpu().numpy(),
                         _bytes(b_q[g:g + 1]),
                         b_s[g:g + 1].cpu().numpy(), [len(rows)])
        assert_close(dlhs[rows].cpu().numpy(), ref, RTOL, ATOL_FRAC, what=f"dlhs rows of group {g}")
        # drhs of group g from the 128-row blocks its rows touch
        base = (r0 // 128) * 128
        end = ((r1 + 127) // 128) * 128
        sub = slice(base, end)
        mb = slice(base // 128, end // 128)
        ref_g = B.tgmm(_bytes(lq[sub]), ls[mb].cpu().numpy(), _bytes(dq2[sub]), ds2[mb].cpu().numpy(),
                       [r0 - base, r1 - r0], groups=[1])[1]
        assert_close(drhs[g].cpu().numpy(), ref_g, RTOL, ATOL_FRAC, what=f"drhs of group {g}")
