"""The CPU oracle against golden fixtures produced by the reference's own GLA
code (tests/golden/make_ref_golden.py runs KE/examples/kernels/chunk_gla_ref.py
and KE/upstream/fused_chunk_simple_gla/common_chunk_h.py unchanged on a numpy
stand-in for JAX).  Both sides compute in fp32, so the bar is tight:
|oracle - ref| <= 1e-4 |ref| + 1e-5 rms(ref).  The full-size fixtures also
pin the seeded input generator (a digest of the sampled head's inputs)."""
import hashlib
import os

import numpy as np
import pytest
import torch

from glaucis_b200 import configs
from oracle import gla_bwd_oracle, gla_oracle
from oracle.gmm_oracle import bf16_bits_to_f32
from tests.helpers import assert_close

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
RTOL, ATOL_FRAC = 1e-4, 1e-5


def load(name):
    return dict(np.load(os.path.join(GOLDEN, name)))


def _small(name):
    d = load(name)
    q, k, v = (bf16_bits_to_f32(d[f"{x}_bf16"]) for x in "qkv")
    do = bf16_bits_to_f32(d["do_bf16"])
    return d, q, k, v, do


@pytest.mark.parametrize("name", ["ref_gla_gamma_small.npz", "ref_gla_gk_h0_small.npz"])
def test_oracle_forward_matches_reference_code(name):
    d, q, k, v, _ = _small(name)
    g, gg, h0 = d.get("g"), d.get("g_gamma"), d.get("h0")
    C, scale = int(d["chunk_size"]), float(d["scale"])
    o, ht, h = gla_oracle.chunk_gla_fwd(q, k, v, g=g, g_gamma=gg, h0=h0, scale=scale, chunk_size=C,
                                        return_states=True)
    gcs, A = gla_oracle.chunk_gla_fwd_intermediates(q, k, g=g, g_gamma=gg, scale=scale, chunk_size=C)
    for got, key in ((o, "o"), (ht, "ht"), (h, "h"), (gcs, "g_cumsum"), (A, "A")):
        assert_close(got, d[key], RTOL, ATOL_FRAC, what=f"{name}:{key}")


@pytest.mark.parametrize("name", ["ref_gla_gamma_small.npz", "ref_gla_gk_h0_small.npz"])
def test_oracle_backward_matches_reference_code(name):
    d, q, k, v, do = _small(name)
    g, gg, h0, dht = d.get("g"), d.get("g_gamma"), d.get("h0"), d.get("dht")
    C, scale = int(d["chunk_size"]), float(d["scale"])
    dq, dk, dv, dh0 = gla_bwd_oracle.chunk_gla_bwd(q, k, v, do, g=g, g_gamma=gg, h0=h0, scale=scale,
                                                   chunk_size=C, dht=dht)
    grads = [(dq, "dq"), (dk, "dk"), (dv, "dv")] + ([(dh0, "dh0")] if "dh0" in d else [])
    for got, key in grads:
        assert_close(got, d[key], RTOL, ATOL_FRAC, what=f"{name}:{key}")


def regenerate_head(d):
    """The sampled head's inputs, regenerated from the workload's seed and
    checked against the fixture's digest."""
    cfg = configs.GLA_CONFIGS[str(d["config"])]
    inp = configs.make_gla_inputs(cfg, device="cpu", seed=int(d["seed"]))
    b, h = int(d["b"]), int(d["h"])
    dig = hashlib.sha256()
    for x in ("q", "k", "v"):
        dig.update(inp[x][b, :, h].contiguous().view(torch.int16).numpy().tobytes())
    dig.update(inp["g"][b, :, h].contiguous().numpy().tobytes())
    if inp["h0"] is not None:
        dig.update(inp["h0"][b, h].contiguous().numpy().tobytes())
    assert dig.hexdigest() == str(d["input_sha256"]), "seeded inputs differ from the fixture's"
    return cfg, inp, b, h


@pytest.mark.parametrize("name", ["ref_gla_b8_t4096_head.npz", "ref_gla_b1_t32768_head.npz"])
def test_oracle_full_size_head_matches_reference_code(name):
    d = load(name)
    cfg, inp, b, h = regenerate_head(d)
    sl = lambda t: t[b:b + 1, :, h:h + 1].float().numpy()  # noqa: E731
    h0 = None if inp["h0"] is None else inp["h0"][b:b + 1, h:h + 1].numpy()
    o, ht = gla_oracle.chunk_gla_fwd(sl(inp["q"]), sl(inp["k"]), sl(inp["v"]), g=sl(inp["g"]), h0=h0,
                                     scale=cfg.K ** -0.5, chunk_size=cfg.C)
    assert_close(o[0, d["rows"], 0], d["o_rows"], RTOL, ATOL_FRAC, what=f"{name}:o")
    assert_close(ht[0, 0], d["ht"], 3e-4, ATOL_FRAC, what=f"{name}:ht")
