"""Reference template for the evaluator tests: same inputs as
glaucis_b200/kernels/gmm_fp8_blockwise.py's _make_test_data, forward computed
by the CPU oracle (oracle/gmm_oracle.py).  Test infrastructure only."""
import numpy as np
import torch

from oracle import gmm_oracle

DEFAULT_TILE_SIZE = 128


def _make_test_data(M, K, N, G, seed=42):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    lhs = torch.randn((M, K), generator=gen, device="cuda").to(torch.bfloat16)
    rhs = torch.randn((G, K, N), generator=gen, device="cuda").to(torch.bfloat16)
    base = (M // G // DEFAULT_TILE_SIZE) * DEFAULT_TILE_SIZE
    sizes = [base] * G
    sizes[-1] = M - base * (G - 1)
    return lhs, rhs, np.array(sizes, np.int32)


def simple_compute(M=8192, K=2048, N=512, G=32):
    lhs, rhs, sizes = _make_test_data(M, K, N, G)
    out = gmm_oracle.gmm_fp8_blockwise(lhs.float().cpu().numpy(), rhs.float().cpu().numpy(), sizes)
    return np.float64(out.astype(np.float64).sum())


def reference_fn(**kwargs):
    return simple_compute(**kwargs)
