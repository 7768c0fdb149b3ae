"""CPU checks of the grouped-FP8-matmul oracle (no GPU)."""
import os

import numpy as np
import pytest
import torch

from oracle import gmm_oracle as O
from glaucis_b200 import configs
from tests.helpers import assert_close, rel_fro

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_e4m3_cast_matches_torch_bitwise():
    # torch.float8_e4m3fn is an independent implementation of the OCP e4m3fn
    # format; the oracle's RNE cast must agree bit for bit on in-range values.
    rng = np.random.default_rng(0)
    xs = np.concatenate([rng.standard_normal(200_000).astype(np.float32) * s
                         for s in (1e-4, 3e-3, 0.1, 1, 17, 300)])
    edge = np.float32([0.0, -0.0, 448.0, -448.0, 2 ** -6, 2 ** -9, 2 ** -10, 3 * 2 ** -10,
                       1.0625, 1.1875, 15.5, 17.0, 240.0, 232.0])
    xs = np.clip(np.concatenate([xs, edge]), -448, 448)
    mine = O.f32_to_e4m3(xs)
    ref = torch.from_numpy(xs).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(mine, ref)
    back = O.e4m3_to_f32(mine)
    assert np.array_equal(back, torch.from_numpy(ref).view(torch.float8_e4m3fn).float().numpy())


def test_e4m3_saturates():
    assert O.f32_to_e4m3(np.float32([460.0]))[0] == 0x7E
    assert O.f32_to_e4m3(np.float32([-1e6]))[0] == 0xFE


def test_scale_shapes_match_reference_pins():
    # KE/tests/standalone_gmm_fp8_blockwise_test.py:287-316: activation
    # [8192, 2048] -> scale [8192, 16]; weight [32, 2048, 512] -> [32, 16, 4];
    # down weight [32, 512, 2048] -> [32, 4, 16].  Checked at reduced M / G.
    x = np.ones((64, 2048), np.float32)
    q, s = O.quant_act_1x128(x)
    assert q.shape == (64, 2048) and q.dtype == np.uint8 and s.shape == (64, 16)
    w = np.ones((2, 2048, 512), np.float32)
    q, s = O.quant_w_128x128(w)
    assert s.shape == (2, 16, 4)
    w = np.ones((2, 512, 2048), np.float32)
    q, s = O.quant_w_128x128(w)
    assert s.shape == (2, 4, 16)


def test_absmax_scale_semantics():
    x = np.zeros((2, 256), np.float32)
    x[0, :128] = np.linspace(-3, 2, 128)
    x[1, 128:] = 7.0
    q, s = O.quant_act_1x128(x)
    assert s[0, 0] == np.float32(3.0) / np.float32(448.0)
    assert s[0, 1] == 1.0 and s[1, 0] == 1.0          # all-zero blocks
    assert q[0, 0] == 0xFE                            # -3 / s == -448
    assert (q[1, 128:] == 0x7E).all()
    assert (q[1, :128] == 0).all()


def test_forward_close_to_bf16_reference():
    # The reference's own acceptance bound (standalone test :365-370):
    # relative Frobenius error of the FP8 forward vs a bf16 GMM < 0.15.
    cfg = configs.GMMConfig("t", G=4, M=512, K=512, N=256, routing="multinomial")
    lhs, rhs, gs = configs.make_gmm_inputs(cfg, device="cpu", seed=3)
    lf, rf = lhs.float().numpy(), rhs.float().numpy()
    out = O.gmm_fp8_blockwise(lf, rf, gs.numpy())
    ref = O.gmm_bf16_reference(lf, rf, gs.numpy())
    assert out.shape == (512, 256) and np.isfinite(out).all()
    assert rel_fro(out, ref) < 0.15


def test_sampled_rows_equal_full():
    rng = np.random.default_rng(5)
    G, M, K, N = 3, 300, 256, 256
    sizes = np.array([100, 0, 150], np.int32)         # 50 unassigned tail rows
    a_q, a_s = O.quant_act_1x128(rng.standard_normal((M, K)).astype(np.float32))
    b_q, b_s = O.quant_w_128x128(rng.standard_normal((G, K, N)).astype(np.float32))
    full = O.gmm_fwd(a_q, a_s, b_q, b_s, sizes)
    rows = np.array([0, 99, 100, 249, 250, 299])
    part = O.gmm_fwd(a_q, a_s, b_q, b_s, sizes, rows=rows)
    assert np.array_equal(part, full[rows])
    assert (full[250:] == 0).all()


def test_golden_fixture_reproduces():
    d = np.load(os.path.join(GOLDEN, "gmm_small_ragged.npz"))
    lf = O.bf16_bits_to_f32(d["lhs_bf16"])
    rf = O.bf16_bits_to_f32(d["rhs_bf16"])
    a_q, a_s = O.quant_act_1x128(lf)
    b_q, b_s = O.quant_w_128x128(rf)
    assert np.array_equal(a_q, d["a_q"]) and np.array_equal(a_s, d["a_s"])
    assert np.array_equal(b_q, d["b_q"]) and np.array_equal(b_s, d["b_s"])
    out = O.gmm_fwd(a_q, a_s, b_q, b_s, d["group_sizes"])
    assert_close(out, d["out"], rtol=1e-5, atol_frac=1e-6, what="golden gmm")


@pytest.mark.parametrize("routing", ["multinomial", "zipf_topk", "uniform_one_empty", "equal"])
def test_group_size_generators(routing):
    s = configs.group_sizes(routing, 128 if routing == "zipf_topk" else 8,
                            32768 if routing == "zipf_topk" else 65536, seed=0)
    assert s.dtype == np.int32 and (s >= 0).all()
    assert int(s.sum()) == (32768 if routing == "zipf_topk" else 65536)
    if routing == "uniform_one_empty":
        assert (s == 0).sum() >= 1
    if routing == "zipf_topk":
        assert s.max() <= 4096 and (s == 0).sum() >= 1


def test_torch_cpu_restatement_matches_oracle():
    # The BLAS-backed CPU baseline quantises bit-identically and agrees with
    # the per-K-block promotion oracle up to fp32 summation order.
    from oracle import cpu_fast
    cfg = configs.GMMConfig("t", G=3, M=400, K=384, N=256, routing="uniform_one_empty")
    lhs, rhs, gs = configs.make_gmm_inputs(cfg, device="cpu", seed=11)
    q, s = cpu_fast.quant_act_1x128(lhs)
    rq, rs = O.quant_act_1x128(lhs.float().numpy())
    assert np.array_equal(q.view(torch.uint8).numpy(), rq) and np.array_equal(s.numpy(), rs)
    q, s = cpu_fast.quant_w_128x128(rhs)
    rq, rs = O.quant_w_128x128(rhs.float().numpy())
    assert np.array_equal(q.view(torch.uint8).numpy(), rq) and np.array_equal(s.numpy(), rs)
    got = cpu_fast.gmm_fp8_blockwise(lhs, rhs, gs.tolist()).numpy()
    ref = O.gmm_fp8_blockwise(lhs.float().numpy(), rhs.float().numpy(), gs.numpy())
    assert_close(got, ref, rtol=1e-4, atol_frac=1e-5, what="cpu_fast gmm")


# ---------------------------------------------------------------------------
# backward oracle (oracle/gmm_bwd_oracle.py)
# ---------------------------------------------------------------------------
def test_bwd_oracle_quant_col_is_act_quant_of_transpose():
    from oracle import gmm_bwd_oracle as B
    rng = np.random.default_rng(5)
    x = rng.standard_normal((256, 384)).astype(np.float32)
    q, s = B.quant_col_128x1(x)
    qt, st = O.quant_act_1x128(np.ascontiguousarray(x.T))   # 1x128 along M of x^T
    assert np.array_equal(q, qt.T) and np.array_equal(s, st.T)


def test_bwd_oracle_close_to_exact_gradients():
    from oracle import gmm_bwd_oracle as B
    rng = np.random.default_rng(6)
    M, K, N = 512, 256, 256
    sizes = [100, 0, 200, 150, 62]
    bf = lambda a: (a.astype(np.float32).view(np.uint32) & 0xFFFF0000).view(np.float32)
    lhs = bf(rng.standard_normal((M, K)))
    rhs = bf(rng.standard_normal((len(sizes), K, N)) * 0.02)
    grad = bf(rng.standard_normal((M, N)))
    dl, dr = B.gmm_fp8_blockwise_bwd(lhs, rhs, sizes, grad)
    ul, ur = B.gmm_bwd_unquantised(lhs, rhs, sizes, grad)
    rel = lambda a, b: np.linalg.norm(a - b) / np.linalg.norm(b)
    assert rel(dl, ul) < 0.06 and rel(dr, ur) < 0.06
    assert not dr[1].any()                      # empty group
    assert not dl[sum(sizes):].any()            # rows past sum(group_sizes)
