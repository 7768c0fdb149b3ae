"""Reference template for the evaluator tests: same inputs as
glaucis_b200/kernels/chunk_gla.py's _make_test_data, forward computed by the
CPU oracle (oracle/gla_oracle.py).  Test infrastructure only."""
import numpy as np
import torch

from oracle import gla_oracle


def _make_test_data(B, T, H, K, V, chunk_size, seed=42):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn((B, T, H, K), generator=gen, device="cuda").to(torch.bfloat16)
    k_arr = torch.randn((B, T, H, K), generator=gen, device="cuda").to(torch.bfloat16)
    v = torch.randn((B, T, H, V), generator=gen, device="cuda").to(torch.bfloat16)
    g_gamma = -torch.randn((H,), generator=gen, device="cuda").abs() * 0.1
    return q, k_arr, v, g_gamma


def simple_compute(B=2, T=4096, H=16, K=128, V=128, chunk_size=64):
    q, k, v, g_gamma = _make_test_data(B, T, H, K, V, chunk_size)
    f = lambda t: t.float().cpu().numpy()
    o, _ = gla_oracle.chunk_gla_fwd(f(q), f(k), f(v), g_gamma=f(g_gamma), scale=K ** -0.5,
                                    chunk_size=chunk_size)
    return np.float64(o.astype(np.float64).sum())


def reference_fn(**kwargs):
    return simple_compute(**kwargs)
