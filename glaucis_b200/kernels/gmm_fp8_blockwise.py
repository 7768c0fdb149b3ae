"""GMM block-wise FP8 for B200 (sm_100a) -- template for evolutionary optimization.

Grouped matrix multiply with DeepSeek-V3 / Transformer Engine style block-wise
FP8 quantisation (activations 1x128, weights 128x128, fp32 absmax scales),
backed by the glaucis_b200 tcgen05 kernels.  Same entry points as
KE/examples/kernels/gmm_fp8_blockwise.py: `_make_test_data`,
`gmm_fp8_blockwise(lhs, rhs, group_sizes, tiling)` and
`optimized_compute(M, K, N, G)`.

optimized_compute runs the forward and the backward (dlhs by the grouped
kernel with the weight transposed, drhs by tgmm) and returns the scalar loss
out.sum(), as the reference's jax.value_and_grad does; mode="fwd" runs the
forward only.
"""

import torch

from glaucis_b200 import ops

# ---------------------------------------------------------------------------
# Constants (fixed across optimization iterations)
# ---------------------------------------------------------------------------
FP8_DTYPE = torch.float8_e4m3fn
DEFAULT_TILE_SIZE = 128


def _make_test_data(M, K, N, G, seed=42):
    """(lhs bf16 [M,K], rhs bf16 [G,K,N], group_sizes int32 [G]) on cuda:
    N(0,1) values and equal 128-multiple group sizes with the remainder in
    the last group, as the reference's _make_test_data."""
    gen = torch.Generator(device="cuda").manual_seed(seed)
    lhs = torch.randn((M, K), generator=gen, device="cuda").to(torch.bfloat16)
    rhs = torch.randn((G, K, N), generator=gen, device="cuda").to(torch.bfloat16)
    base = (M // G // DEFAULT_TILE_SIZE) * DEFAULT_TILE_SIZE
    assert base > 0, f"M={M} / G={G} = {M // G} must be >= {DEFAULT_TILE_SIZE}"
    sizes = [base] * G
    sizes[-1] = M - base * (G - 1)
    group_sizes = torch.tensor(sizes, dtype=torch.int32, device="cuda")
    return lhs, rhs, group_sizes


# EVOLVE-BLOCK-START
def gmm_fp8_blockwise(
    lhs: torch.Tensor,
    rhs: torch.Tensor,
    group_sizes: torch.Tensor,
    tiling: tuple = (256, 512, 256, 256, 512, 128, 1024, 512, 128),
) -> torch.Tensor:
    """GMM with fp8_blockwise quantisation (fp32 output)."""
    return ops.gmm_fp8_blockwise(lhs, rhs, group_sizes, tiling, out_dtype=torch.float32)


def optimized_compute(M=8192, K=2048, N=512, G=32, mode="fwd_bwd"):
    """Forward + backward GMM with FP8 block-wise quantisation (gradients
    of lhs and rhs computed, as the reference's value_and_grad); returns the
    loss scalar."""
    lhs, rhs, group_sizes = _make_test_data(M, K, N, G)
    if mode == "fwd":
        return gmm_fp8_blockwise(lhs, rhs, group_sizes).sum().cpu()
    lhs.requires_grad_(True)
    rhs.requires_grad_(True)
    loss = gmm_fp8_blockwise(lhs, rhs, group_sizes).sum()
    loss.backward()
    return loss.detach().cpu()
# EVOLVE-BLOCK-END
