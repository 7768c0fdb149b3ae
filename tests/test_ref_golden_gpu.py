"""The B200 kernels against golden fixtures produced by the reference's own
GLA code (tests/golden/make_ref_golden.py: KE/examples/kernels/chunk_gla_ref.py
and KE/upstream/fused_chunk_simple_gla/common_chunk_h.py executed unchanged on
a numpy stand-in for JAX, fp32 contractions), through the C ABI.

Outputs and tolerances:
  o, ht          |gpu - ref| <= 2e-2 |ref| + 3e-2 rms(ref), relative Frobenius
                 error < 1e-2 (the forward parity tolerance: bf16 tensor-core
                 operands, fp32 accumulation and state)
  h (per chunk)  the training forward's bf16 states: the o / ht element-wise
                 tolerance (the state is accumulated from bf16 k e^-G and v
                 tensor-core operands, as ht is)
  g_cumsum, A    the fp32 intermediates kernel: 1e-4 |ref| + 1e-4 rms(ref)
  dq, dk, dv,    the backward parity tolerance: 2e-2 |ref| + 6e-2 rms(ref),
  dh0            relative Frobenius error < 1.5e-2
The full-size fixtures hold one (b, h) of each long workload: the whole
workload runs on the GPU (so the launcher takes the path it takes at that
size) and the sampled head's o rows and final state are compared.
"""
import os

import numpy as np
import pytest
import torch

from glaucis_b200 import configs, ops
from oracle.gmm_oracle import bf16_bits_to_f32
from tests.helpers import assert_close, rel_fro
from tests.test_ref_golden import load, regenerate_head

pytestmark = pytest.mark.gpu


def _check(got, ref, rtol, atol_frac, fro, what):
    assert_close(got, ref, rtol, atol_frac, what=what)
    if fro is not None:
        assert rel_fro(got, ref) < fro, (what, rel_fro(got, ref))


def _small_inputs(cuda, d):
    to_bf16 = lambda bits: torch.from_numpy(bf16_bits_to_f32(bits)).to(torch.bfloat16).to(cuda)  # noqa: E731
    t = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    return (to_bf16(d["q_bf16"]), to_bf16(d["k_bf16"]), to_bf16(d["v_bf16"]), t(d.get("g")),
            t(d.get("g_gamma")), t(d.get("h0")), to_bf16(d["do_bf16"]), t(d.get("dht")))


@pytest.mark.parametrize("exact", [False, True])
@pytest.mark.parametrize("vs", ["64", "128"])
@pytest.mark.parametrize("name", ["ref_gla_gamma_small.npz", "ref_gla_gk_h0_small.npz"])
def test_forward_and_intermediates_match_reference_code(cuda, name, vs, exact, monkeypatch):
    monkeypatch.setenv("GLAUCIS_GLA_VS", vs)
    d = load(name)
    q, k, v, g, gg, h0, _, _ = _small_inputs(cuda, d)
    C, scale = int(d["chunk_size"]), float(d["scale"])
    res = ops.chunk_gla_fwd(q, k, v, gg, scale, C, g=g, h0=h0, output_final_state=True,
                            output_states=True, output_intermediates=True, exact_intra=exact)
    assert ops.device_status() == 0
    f = lambda x: x.float().cpu().numpy()  # noqa: E731
    _check(f(res.o), d["o"], 2e-2, 3e-2, 1e-2, f"{name} o")
    _check(f(res.ht), d["ht"], 2e-2, 3e-2, 1e-2, f"{name} ht")
    _check(f(res.h), d["h"], 2e-2, 3e-2, None, f"{name} h")
    _check(f(res.g_cumsum), d["g_cumsum"], 1e-4, 1e-4, None, f"{name} g_cumsum")
    _check(f(res.A), d["A"], 1e-4, 1e-4, None, f"{name} A")
    g_cumsum, A, h, o = res                      # the reference's tuple order
    assert g_cumsum is res.g_cumsum and A is res.A and h is res.h and o is res.o


@pytest.mark.parametrize("name", ["ref_gla_gamma_small.npz", "ref_gla_gk_h0_small.npz"])
def test_backward_matches_reference_code(cuda, name):
    d = load(name)
    q, k, v, g, gg, h0, do, dht = _small_inputs(cuda, d)
    C, scale = int(d["chunk_size"]), float(d["scale"])
    h = ops.chunk_gla_fwd(q, k, v, gg, scale, C, g=g, h0=h0, output_states=True).h
    dq, dk, dv, dh0 = ops.chunk_gla_bwd(q, k, v, do, h, gg, scale, C, g=g, dht=dht,
                                        output_dh0=h0 is not None)
    assert ops.device_status() == 0
    f = lambda x: x.float().cpu().numpy()  # noqa: E731
    for got, key in ((dq, "dq"), (dk, "dk"), (dv, "dv"), (dh0, "dh0")):
        if key in d:
            _check(f(got), d[key], 2e-2, 6e-2, 1.5e-2, f"{name} {key}")


@pytest.mark.parametrize("exact", [False, True])
@pytest.mark.parametrize("name", ["ref_gla_b8_t4096_head.npz", "ref_gla_b1_t32768_head.npz"])
def test_full_size_head_matches_reference_code(cuda, name, exact):
    d = load(name)
    cfg, inp, b, h = regenerate_head(d)
    dev = {kk: (vv.to(cuda) if vv is not None else None) for kk, vv in inp.items()}
    res = ops.chunk_gla_fwd(dev["q"], dev["k"], dev["v"], None, cfg.K ** -0.5, cfg.C, g=dev["g"],
                            h0=dev["h0"], output_final_state=True, exact_intra=exact)
    assert ops.device_status() == 0
    rows = torch.from_numpy(d["rows"]).to(cuda)
    got_o = res.o[b, :, h].index_select(0, rows).float().cpu().numpy()
    _check(got_o, d["o_rows"], 2e-2, 3e-2, 1e-2, f"{name} o")
    _check(res.ht[b, h].cpu().numpy(), d["ht"], 2e-2, 3e-2, 1e-2, f"{name} ht")
