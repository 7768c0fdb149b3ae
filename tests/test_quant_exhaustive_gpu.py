"""Exhaustive check of the quantisers' division by the block scale.

The kernels divide by the block scale with a reciprocal and an FMA
correction instead of a division per element.  Inputs are bf16, so a block's
maximum and every element take one of finitely many values: this test builds,
for every finite bf16 block maximum A, 1x128 blocks holding A and every bf16
value of magnitude <= A (both signs), and compares the activation quantiser's
bytes and scales with a plain PyTorch fp32 reference (IEEE division, then the
round-to-nearest-even e4m3fn cast) on the GPU.  About 1.07e9 elements in
chunks of a few hundred MB.
"""
import pytest
import torch

from glaucis_b200 import ops

pytestmark = pytest.mark.gpu

MAX_FINITE_BF16 = 0x7F7F
ROW = 128


def _blocks_for(a_bits: torch.Tensor) -> torch.Tensor:
    """bf16 [R, 128]: for each block maximum bit pattern a (int64, on the GPU)
    rows [a, x_0 .. x_126] enumerating all magnitudes 0..a with both signs;
    the last row of each a is padded with a itself."""
    dev = a_bits.device
    n = 2 * (a_bits + 1)                              # values per block maximum
    rows = (n + ROW - 2) // (ROW - 1)                 # rows per block maximum
    row_a = torch.repeat_interleave(a_bits, rows)
    row_n = torch.repeat_interleave(n, rows)
    first = torch.cumsum(rows, 0) - rows
    local = torch.arange(int(rows.sum()), device=dev) - torch.repeat_interleave(first, rows)
    j = local[:, None] * (ROW - 1) + torch.arange(ROW - 1, device=dev)[None, :]
    mag, sign = j >> 1, j & 1
    bits = torch.where(j < row_n[:, None], (sign << 15) | mag, row_a[:, None])
    bits = torch.cat([row_a[:, None], bits], dim=1)
    return bits.to(torch.int32).to(torch.int16).view(torch.bfloat16)


def _reference(x: torch.Tensor):
    xf = x.float()
    amax = xf.abs().amax(dim=1)
    # tensor / tensor: PyTorch turns a division by a Python scalar into a
    # multiplication by its reciprocal, which is not the IEEE quotient
    s = torch.where(amax > 0, amax / torch.full_like(amax, 448.0), torch.ones_like(amax))
    q = (xf / s[:, None]).to(torch.float8_e4m3fn)
    return q.view(torch.uint8), s


def test_quant_division_exhaustive_over_bf16(cuda):
    a_all = torch.arange(0, MAX_FINITE_BF16 + 1, device=cuda, dtype=torch.int64)
    # chunks of block maxima with roughly equal element counts (~1.3e8)
    counts = 2 * (a_all + 1)
    csum = torch.cumsum(counts, 0)
    per_chunk = 130_000_000
    bounds = [0]
    while bounds[-1] < a_all.numel():
        target = (csum[bounds[-1] - 1] if bounds[-1] else 0) + per_chunk
        nxt = int(torch.searchsorted(csum, torch.tensor([target], device=cuda)).item()) + 1
        bounds.append(min(max(nxt, bounds[-1] + 1), a_all.numel()))
    checked = 0
    for lo, hi in zip(bounds[:-1], bounds[1:]):
        x = _blocks_for(a_all[lo:hi])
        q, s = ops.quant_act_1x128(x)
        assert ops.device_status() == 0
        q_ref, s_ref = _reference(x)
        assert torch.equal(s.view(-1).view(torch.int32), s_ref.view(torch.int32)), \
            f"scales differ for block maxima {lo:#x}..{hi - 1:#x}"
        bad = (q.view(torch.uint8) != q_ref).nonzero()
        assert bad.numel() == 0, (
            f"{bad.shape[0]} e4m3 bytes differ for block maxima {lo:#x}..{hi - 1:#x}; first "
            f"x={x[bad[0, 0], bad[0, 1]].item()!r} in the block of max {x[bad[0, 0], 0].item()!r}")
        checked += x.numel()
        del x, q, s, q_ref, s_ref
    assert checked > 1_000_000_000
