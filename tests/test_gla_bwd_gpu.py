"""Parity of the chunked-GLA backward (reverse state-gradient scan + the
chunk-parallel dq/dk/dv kernel) and of the training forward's per-chunk
states against the CPU oracle, through the C ABI.  Every test runs on both
instances of the sequential kernel (GLAUCIS_GLA_VS = 64 or 128).

Tolerance: a relative Frobenius error below 1.5e-2 per gradient, and
|gpu - ref| <= 2e-2 * |ref| + 6e-2 * rms(ref) element-wise: each gradient
element is a sum of 192 products of two bf16-rounded operands, scaled by
e^{+-G} afterwards, so over a million elements the largest deviations reach a
few percent of the rms where the terms cancel.  The kernels feed the tensor cores
bf16 operands (q e^G, k e^-G, tril(A), tril(dA), the states h_n and the
state gradients E_n) with fp32 accumulation and write bf16 gradients; the
oracle is fp32 throughout (the reference's Precision.HIGHEST path).
"""
import numpy as np
import pytest
import torch

from glaucis_b200 import configs, ops
from oracle import gla_oracle as O
from oracle.gla_bwd_oracle import chunk_gla_bwd as oracle_bwd
from tests.helpers import assert_close, rel_fro

pytestmark = pytest.mark.gpu
RTOL, ATOL_FRAC, FRO = 2e-2, 6e-2, 1.5e-2


@pytest.fixture(autouse=True, params=["64", "128"])
def value_slice(request, monkeypatch):
    monkeypatch.setenv("GLAUCIS_GLA_VS", request.param)
    return request.param


def _f(t):
    return None if t is None else t.float().cpu().numpy()


def _inputs(cfg, seed, with_dht):
    inp = configs.make_gla_inputs(cfg, device="cpu", seed=seed)
    gen = torch.Generator().manual_seed(seed + 100)
    do = torch.randn((cfg.B, cfg.T, cfg.H, cfg.V), generator=gen).to(torch.bfloat16)
    # dht of the order of one chunk's contribution to the state gradient: an
    # N(0,1) dht makes the last chunk's dk / dv sums of bf16-rounded terms
    # ten times larger than elsewhere, and their cancellation error exceed a
    # tolerance scaled by the whole tensor's rms (the reference rounds the
    # same operands to bf16, chunk_gla.py:350-359)
    dht = 0.25 * torch.randn((cfg.B, cfg.H, cfg.K, cfg.V), generator=gen) if with_dht else None
    return inp, do, dht


def _run_bwd(cuda, cfg, seed=0, with_dht=False):
    inp, do, dht = _inputs(cfg, seed, with_dht)
    d = {k: (v.to(cuda) if v is not None else None) for k, v in inp.items()}
    scale = cfg.K ** -0.5
    fwd = ops.chunk_gla_fwd(d["q"], d["k"], d["v"], d["g_gamma"], scale, cfg.C, g=d["g"], h0=d["h0"],
                            output_states=True)
    dq, dk, dv, dh0 = ops.chunk_gla_bwd(d["q"], d["k"], d["v"], do.to(cuda), fwd.h, d["g_gamma"],
                                        scale, cfg.C, g=d["g"],
                                        dht=None if dht is None else dht.to(cuda), output_dh0=True)
    assert ops.device_status() == 0
    ref = oracle_bwd(_f(inp["q"]), _f(inp["k"]), _f(inp["v"]), _f(do), g=_f(inp["g"]),
                     g_gamma=_f(inp["g_gamma"]), h0=_f(inp["h0"]), scale=scale, chunk_size=cfg.C,
                     dht=_f(dht))
    return (_f(dq), _f(dk), _f(dv), _f(dh0)), ref


def _check(got, ref, what):
    for name, a, b in zip(("dq", "dk", "dv", "dh0"), got, ref):
        print(f"{what} {name}: rel_fro {rel_fro(a, b):.2e} max|err|/rms "
              f"{np.abs(a - b).max() / (np.sqrt(np.mean(b.astype(np.float64) ** 2)) + 1e-30):.2e}")
        assert_close(a, b, RTOL, ATOL_FRAC, what=f"{what} {name}")
        assert rel_fro(a, b) < FRO, (what, name, rel_fro(a, b))


@pytest.mark.parametrize("gate", ["per_key", "gamma"])
def test_forward_states_match_the_oracle(cuda, gate):
    # h_states[:, n] = the state before chunk n (h_0 = h0), bf16
    cfg = configs.GLAConfig("t", B=2, T=320, H=3, h0_std=0.1, gate=gate)
    inp = configs.make_gla_inputs(cfg, device="cpu", seed=1)
    d = {k: (v.to(cuda) if v is not None else None) for k, v in inp.items()}
    res = ops.chunk_gla_fwd(d["q"], d["k"], d["v"], d["g_gamma"], cfg.K ** -0.5, cfg.C, g=d["g"],
                            h0=d["h0"], output_final_state=True, output_states=True)
    plain = ops.chunk_gla_fwd(d["q"], d["k"], d["v"], d["g_gamma"], cfg.K ** -0.5, cfg.C, g=d["g"],
                              h0=d["h0"], output_final_state=True)
    assert ops.device_status() == 0
    _, _, h_all = O.chunk_gla_fwd(_f(inp["q"]), _f(inp["k"]), _f(inp["v"]), g=_f(inp["g"]),
                                  g_gamma=_f(inp["g_gamma"]), h0=_f(inp["h0"]),
                                  scale=cfg.K ** -0.5, chunk_size=cfg.C, return_states=True)
    got = _f(res.h)
    assert got.shape == h_all.shape
    assert_close(got, h_all, RTOL, ATOL_FRAC, what="h_states")
    assert rel_fro(got, h_all) < 1e-2
    # h_0 is h0 rounded to bf16; writing the states leaves o and ht unchanged
    np.testing.assert_array_equal(got[:, 0], inp["h0"].to(torch.bfloat16).float().numpy())
    assert torch.equal(res.o, plain.o) and torch.equal(res.ht, plain.ht)


@pytest.mark.parametrize("gate", ["per_key", "gamma"])
@pytest.mark.parametrize("with_state", [False, True])
def test_backward_matches_the_oracle(cuda, gate, with_state):
    cfg = configs.GLAConfig("t", B=2, T=256, H=3, h0_std=0.1 if with_state else 0.0, gate=gate)
    got, ref = _run_bwd(cuda, cfg, seed=2, with_dht=with_state)
    _check(got, ref, f"{gate} state={with_state}")


def test_backward_full_width_many_heads(cuda):
    # B*H > SMs/2: one CTA per (batch, head) in the scan, many gradient items
    cfg = configs.GLAConfig("t", B=2, T=128, H=40, h0_std=0.1)
    got, ref = _run_bwd(cuda, cfg, seed=3, with_dht=True)
    _check(got, ref, "many heads")


@pytest.mark.parametrize("nseg", [2, 3, 7])
@pytest.mark.parametrize("gate", ["per_key", "gamma"])
def test_backward_sequence_split(cuda, monkeypatch, nseg, gate):
    # the reverse scan split into nseg segments (state-only pre-pass over the
    # later segments, reverse fold from dht, full pass), 20 chunks
    monkeypatch.setenv("GLAUCIS_GLA_SEGMENTS", str(nseg))
    cfg = configs.GLAConfig("t", B=1, T=1280, H=2, h0_std=0.1, gate=gate)
    got, ref = _run_bwd(cuda, cfg, seed=4, with_dht=True)
    _check(got, ref, f"nseg={nseg} {gate}")


def test_backward_sequence_split_many_segments(cuda, monkeypatch):
    # 45 segments: 44 records, two batches of the fold kernel's loads
    monkeypatch.setenv("GLAUCIS_GLA_SEGMENTS", "45")
    cfg = configs.GLAConfig("t", B=1, T=64 * 48, H=2, h0_std=0.1, gate="per_key")
    got, ref = _run_bwd(cuda, cfg, seed=6, with_dht=True)
    _check(got, ref, "nseg=45")


def test_autograd_function_and_template(cuda):
    from glaucis_b200.kernels import chunk_gla as tmpl
    cfg = configs.GLAConfig("t", B=1, T=192, H=2, h0_std=0.1, gate="gamma")
    inp = configs.make_gla_inputs(cfg, device=cuda, seed=6)
    q, k, v, h0 = (inp[n].clone().requires_grad_(True) for n in ("q", "k", "v", "h0"))
    o = ops.chunk_gla(q, k, v, inp["g_gamma"], cfg.K ** -0.5, cfg.C, h0=h0)
    do = torch.randn_like(o)
    o.backward(do)
    fwd = ops.chunk_gla_fwd(inp["q"], inp["k"], inp["v"], inp["g_gamma"], cfg.K ** -0.5, cfg.C,
                            h0=inp["h0"], output_states=True)
    dq, dk, dv, dh0 = ops.chunk_gla_bwd(inp["q"], inp["k"], inp["v"], do, fwd.h, inp["g_gamma"],
                                        cfg.K ** -0.5, cfg.C, output_dh0=True)
    for a, b in ((q.grad, dq), (k.grad, dk), (v.grad, dv), (h0.grad, dh0)):
        assert torch.equal(a, b)
    loss = tmpl.optimized_compute(B=1, T=256, H=2, K=128, V=128, chunk_size=64)
    assert np.isfinite(float(loss))
    assert ops.device_status() == 0


@pytest.mark.parametrize("name", ["gla_b8_t4096", "gla_b1_t32768"])
def test_backward_full_size_sampled_heads(cuda, name):
    # Full benchmark shapes on the GPU (both the plain and the sequence-split
    # scan); the oracle recomputes three (b, h) sequences end to end.
    cfg = configs.GLA_CONFIGS[name]
    inp = configs.make_gla_inputs(cfg, device=cuda, seed=0)
    gen = torch.Generator(device=cuda).manual_seed(12)
    do = torch.randn(inp["v"].shape, generator=gen, device=cuda).to(torch.bfloat16)
    scale = cfg.K ** -0.5
    h = ops.chunk_gla_fwd(inp["q"], inp["k"], inp["v"], inp["g_gamma"], scale, cfg.C, g=inp["g"],
                          h0=inp["h0"], output_states=True).h
    dq, dk, dv, dh0 = ops.chunk_gla_bwd(inp["q"], inp["k"], inp["v"], do, h, inp["g_gamma"], scale,
                                        cfg.C, g=inp["g"], output_dh0=True)
    assert ops.device_status() == 0
    for (b, hh) in [(0, 0), (cfg.B - 1, cfg.H - 1), (cfg.B // 2, cfg.H // 3)]:
        sl = lambda t: t[b:b + 1, :, hh:hh + 1].float().cpu().numpy()
        h0 = None if inp["h0"] is None else inp["h0"][b:b + 1, hh:hh + 1].cpu().numpy()
        gg = None if inp["g_gamma"] is None else inp["g_gamma"][hh:hh + 1].cpu().numpy()
        ref = oracle_bwd(sl(inp["q"]), sl(inp["k"]), sl(inp["v"]), sl(do),
                         g=None if inp["g"] is None else sl(inp["g"]), g_gamma=gg, h0=h0,
                         scale=scale, chunk_size=cfg.C)
        got = (sl(dq), sl(dk), sl(dv), dh0[b:b + 1, hh:hh + 1].cpu().numpy())
        _check(got, ref, f"{name} (b={b}, h={hh})")


@pytest.mark.parametrize("seed", range(3))
def test_backward_random_shapes(cuda, monkeypatch, seed):
    # Seeded random problems for the backward: B x H from 1 to 12 sequences,
    # 1 to 24 chunks, either gate, with or without h0 and dht, and a random
    # sequence split of the reverse scan.
    rng = np.random.default_rng(300 + seed)
    cfg = configs.GLAConfig("rand", B=int(rng.integers(1, 3)), T=64 * int(rng.integers(1, 25)),
                            H=int(rng.integers(1, 7)), h0_std=float(rng.choice([0.0, 0.1])),
                            gate=str(rng.choice(["per_key", "gamma"])))
    if rng.random() < 0.5:
        monkeypatch.setenv("GLAUCIS_GLA_SEGMENTS", str(int(rng.integers(2, 5))))
    got, ref = _run_bwd(cuda, cfg, seed=seed, with_dht=bool(rng.random() < 0.5))
    _check(got, ref, f"random {cfg}")
