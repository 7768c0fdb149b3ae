"""Parity of the fused sm_100a chunked-GLA forward against the CPU oracle,
through the C ABI.  The launcher reads GLAUCIS_GLA_VS at every call, so
each test runs on both kernel instances.

Tolerance (o and the final state): |gpu - ref| <= 2e-2 * |ref| + 4e-2 * rms(ref)
element-wise, plus a relative Frobenius error below 1e-2 (tests/helpers.py).
The kernel feeds the tensor cores bf16 operands (q e^G, k e^-G, the state
copy h_n, and tril(A) as a bf16 hi + lo pair or as one bf16 operand) with
fp32 accumulation and an fp32 recurrent state; the oracle is fp32
throughout.  The reference template rounds operands to bf16 as well: the
decayed v of its state update (KE/examples/kernels/chunk_gla.py:79), q e^G
and k e^-G before the intra-chunk A (:151-152), and q e^G and the state h
before its output dot (:204-205).  Where an output is a near cancellation of
its intra- and inter-chunk parts, those roundings alone move it up to 3.2 %
of rms(o) from the fp32 oracle beyond the relative term (a CPU emulation of
all of them, tests/test_oracle_gla.py::
test_reference_bf16_casts_stay_within_the_kernel_tolerance, on the inputs of
test_gla_more_sequences_than_sms among others), so the absolute term is
4e-2 * rms.  The kernel's roundings are of the same kinds; on those inputs
its largest deviation is of the same size (3.2-3.5 % of rms, one element of
5.1 M), and its relative Frobenius error is the template emulation's
(~2.5e-3).
"""
import os

import numpy as np
import pytest
import torch

from glaucis_b200 import configs, ops
from oracle import gla_oracle as O
from oracle.gmm_oracle import bf16_bits_to_f32
from tests.helpers import GLA_ATOL_FRAC, GLA_FRO, GLA_RTOL, assert_close, rel_fro

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
RTOL, ATOL_FRAC, FRO = GLA_RTOL, GLA_ATOL_FRAC, GLA_FRO


@pytest.fixture(autouse=True, params=["64", "128"])
def value_slice(request, monkeypatch):
    """Every test runs on both kernel instances: V split in two 64-wide
    slices (double-buffered state copy) and the full 128-wide V."""
    monkeypatch.setenv("GLAUCIS_GLA_VS", request.param)
    return request.param


@pytest.fixture(autouse=True, params=["exact_intra", "bf16_p"])
def intra_precision(request, monkeypatch):
    """... and in both precisions of the intra-chunk product: tril(A) as a
    bf16 hi + lo pair (exact_intra, the default) and as one bf16 operand."""
    if request.param == "bf16_p":
        import functools
        monkeypatch.setattr(ops, "chunk_gla_fwd", functools.partial(ops.chunk_gla_fwd, exact_intra=False))
    return request.param


def _run(cuda, cfg: configs.GLAConfig, seed=0):
    inp = configs.make_gla_inputs(cfg, device="cpu", seed=seed)
    dev = {k: (v.to(cuda) if v is not None else None) for k, v in inp.items()}
    res = ops.chunk_gla_fwd(dev["q"], dev["k"], dev["v"], dev["g_gamma"], cfg.K ** -0.5, cfg.C,
                            g=dev["g"], h0=dev["h0"], output_final_state=True)
    assert ops.device_status() == 0
    f = lambda t: None if t is None else t.float().numpy()
    ref_o, ref_ht = O.chunk_gla_fwd(f(inp["q"]), f(inp["k"]), f(inp["v"]), g=f(inp["g"]),
                                    g_gamma=f(inp["g_gamma"]), h0=f(inp["h0"]),
                                    scale=cfg.K ** -0.5, chunk_size=cfg.C)
    got_o = res.o.float().cpu().numpy()
    got_ht = res.ht.cpu().numpy()
    return got_o, got_ht, ref_o, ref_ht


def _check(got_o, got_ht, ref_o, ref_ht, what):
    assert_close(got_o, ref_o, RTOL, ATOL_FRAC, what=f"{what} o")
    assert_close(got_ht, ref_ht, RTOL, ATOL_FRAC, what=f"{what} ht")
    assert rel_fro(got_o, ref_o) < FRO, rel_fro(got_o, ref_o)
    assert rel_fro(got_ht, ref_ht) < FRO, rel_fro(got_ht, ref_ht)


@pytest.mark.parametrize("h0", [0.0, 0.1])
def test_gla_per_key_gate_split_v(cuda, h0):
    # B*H small -> the V dimension is split across two CTAs per sequence
    cfg = configs.GLAConfig("t", B=2, T=256, H=3, h0_std=h0)
    _check(*_run(cuda, cfg), what=f"per-key h0={h0}")


def test_gla_per_key_gate_full_v(cuda):
    # B*H > SMs/2 -> one CTA per sequence with the full V = 128 width
    cfg = configs.GLAConfig("t", B=2, T=128, H=40, h0_std=0.1)
    _check(*_run(cuda, cfg), what="per-key full-V")


def test_gla_gamma_gate_reference_mode(cuda):
    # the template's own mode: per-head constant gate g_gamma [H], no h0
    cfg = configs.GLAConfig("t", B=2, T=320, H=4, gate="gamma")
    _check(*_run(cuda, cfg, seed=5), what="g_gamma")


@pytest.mark.parametrize("nseg", [2, 3, 7])
@pytest.mark.parametrize("gate", ["per_key", "gamma"])
def test_gla_sequence_split(cuda, monkeypatch, nseg, gate):
    # Sequence split into nseg segments (state-only pass + full pass seeded
    # from the folded segment states), uneven segment lengths (20 chunks).
    monkeypatch.setenv("GLAUCIS_GLA_SEGMENTS", str(nseg))
    cfg = configs.GLAConfig("t", B=1, T=64 * 20, H=2, gate=gate,
                            h0_std=0.1 if gate == "per_key" else 0.0)
    _check(*_run(cuda, cfg, seed=7), what=f"split {nseg} {gate}")


def test_gla_sequence_split_many_segments(cuda, monkeypatch):
    # 45 segments of 48 chunks: 44 state records, more than the fold kernel
    # loads in one batch (40), so its second batch runs too.
    monkeypatch.setenv("GLAUCIS_GLA_SEGMENTS", "45")
    cfg = configs.GLAConfig("t", B=1, T=64 * 48, H=2, gate="per_key", h0_std=0.1)
    _check(*_run(cuda, cfg, seed=9), what="split 45")


@pytest.mark.parametrize("gate", ["per_key", "gamma"])
def test_gla_more_sequences_than_sms(cuda, gate):
    # 4 x 52 = 208 (batch, head) pairs, one CTA each: more CTAs than the 148
    # SMs, so a second wave of CTAs runs after the first frees its SMs.
    cfg = configs.GLAConfig("t", B=4, T=64 * 3, H=52, gate=gate,
                            h0_std=0.1 if gate == "per_key" else 0.0)
    _check(*_run(cuda, cfg, seed=12), what=f"208 sequences {gate}")


def test_gla_split_workspace_query(cuda):
    from glaucis_b200 import _lib
    lib = _lib.load()
    # few heads, long sequence: split (one CTA per SM); many heads: none
    assert lib.gl_chunk_gla_fwd_workspace_bytes(1, 32768, 32, 128, 128, 64) > 0
    assert lib.gl_chunk_gla_fwd_workspace_bytes(8, 4096, 16, 128, 128, 64) == 0


def test_gla_single_chunk(cuda):
    cfg = configs.GLAConfig("t", B=1, T=64, H=1, h0_std=0.1)
    _check(*_run(cuda, cfg, seed=2), what="T=C")


def test_gla_golden_fixture(cuda):
    d = np.load(os.path.join(GOLDEN, "gla_per_key_h0.npz"))
    to_bf = lambda a: torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).to(cuda)
    res = ops.chunk_gla_fwd(to_bf(d["q_bf16"]), to_bf(d["k_bf16"]), to_bf(d["v_bf16"]), None,
                            128 ** -0.5, 64, g=torch.from_numpy(d["g"]).to(cuda),
                            h0=torch.from_numpy(d["h0"]).to(cuda), output_final_state=True)
    _check(res.o.float().cpu().numpy(), res.ht.cpu().numpy(), d["o"], d["ht"], what="golden")


def test_gla_public_chunk_gla_op(cuda):
    cfg = configs.GLAConfig("t", B=1, T=128, H=2, gate="gamma")
    inp = configs.make_gla_inputs(cfg, device="cpu", seed=9)
    o = ops.chunk_gla(inp["q"].to(cuda), inp["k"].to(cuda), inp["v"].to(cuda),
                      inp["g_gamma"].to(cuda), 128 ** -0.5, 64)
    assert o.shape == (1, 128, 2, 128) and o.dtype == torch.bfloat16
    ref, _ = O.chunk_gla_fwd(inp["q"].float().numpy(), inp["k"].float().numpy(),
                             inp["v"].float().numpy(), g_gamma=inp["g_gamma"].numpy())
    assert_close(o.float().cpu().numpy(), ref, RTOL, ATOL_FRAC, what="chunk_gla")


@pytest.mark.parametrize("name", ["gla_b8_t4096", "gla_b1_t32768"])
def test_gla_full_size_sampled_heads(cuda, name):
    # Full benchmark shapes on the GPU; the oracle recomputes three (b, h)
    # sequences end to end (state carried through every chunk).
    cfg = configs.GLA_CONFIGS[name]
    inp = configs.make_gla_inputs(cfg, device=cuda, seed=0)
    res = ops.chunk_gla_fwd(inp["q"], inp["k"], inp["v"], inp["g_gamma"], cfg.K ** -0.5, cfg.C,
                            g=inp["g"], h0=inp["h0"], output_final_state=True)
    assert ops.device_status() == 0
    for (b, h) in [(0, 0), (cfg.B - 1, cfg.H - 1), (cfg.B // 2, cfg.H // 3)]:
        sl = lambda t: t[b:b + 1, :, h:h + 1].float().cpu().numpy()
        h0 = None if inp["h0"] is None else inp["h0"][b:b + 1, h:h + 1].cpu().numpy()
        ref_o, ref_ht = O.chunk_gla_fwd(sl(inp["q"]), sl(inp["k"]), sl(inp["v"]), g=sl(inp["g"]),
                                        h0=h0, scale=cfg.K ** -0.5)
        _check(sl(res.o), res.ht[b:b + 1, h:h + 1].cpu().numpy(), ref_o, ref_ht,
               what=f"{name} (b={b}, h={h})")


@pytest.mark.parametrize("seed", range(4))
def test_gla_random_shapes(cuda, monkeypatch, seed):
    # Seeded random problems: B x H from 1 to 24 sequences, 1 to 40 chunks,
    # either gate, with or without h0, and a random sequence split (which
    # the launcher also takes by itself when there are few heads).
    rng = np.random.default_rng(200 + seed)
    cfg = configs.GLAConfig("rand", B=int(rng.integers(1, 4)), T=64 * int(rng.integers(1, 41)),
                            H=int(rng.integers(1, 9)), h0_std=float(rng.choice([0.0, 0.1])),
                            gate=str(rng.choice(["per_key", "gamma"])))
    if rng.random() < 0.5:
        monkeypatch.setenv("GLAUCIS_GLA_SEGMENTS", str(int(rng.integers(2, 6))))
    _check(*_run(cuda, cfg, seed=seed), f"random {cfg}")


def test_exact_intra_is_closer_to_the_fp32_product(cuda, intra_precision):
    # exact_intra removes the bf16 rounding of tril(A) from the intra-chunk
    # product: against the fp32 oracle its error must not exceed the
    # default's, and both hold the forward tolerance.
    if intra_precision != "exact_intra":
        pytest.skip("compares the two precisions itself")
    cfg = configs.GLAConfig("t", B=2, T=512, H=4, h0_std=0.1)
    inp = configs.make_gla_inputs(cfg, device="cpu", seed=13)
    d = {k: (v.to(cuda) if v is not None else None) for k, v in inp.items()}
    f = lambda t: None if t is None else t.float().numpy()  # noqa: E731
    ref_o, _ = O.chunk_gla_fwd(f(inp["q"]), f(inp["k"]), f(inp["v"]), g=f(inp["g"]), h0=f(inp["h0"]))
    errs = {}
    for exact in (False, True):
        o = ops.chunk_gla_fwd(d["q"], d["k"], d["v"], None, 128 ** -0.5, 64, g=d["g"], h0=d["h0"],
                              exact_intra=exact).o.float().cpu().numpy()
        assert ops.device_status() == 0
        assert_close(o, ref_o, RTOL, ATOL_FRAC, what=f"exact_intra={exact}")
        errs[exact] = rel_fro(o, ref_o)
    assert errs[True] <= errs[False] * 1.02, errs
