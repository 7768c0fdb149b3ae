"""The allocation-free grouped matmul entry point (gl_gmm_fp8_act_fwd_noalloc),
called through the C ABI, gives the same result as the allocating path
(gl_quant_act_1x128 into caller buffers + gl_gmm_fp8_fwd).

It exists for callers that cannot allocate device memory while a step runs
(runtimes that plan all device buffers up front, FFI hosts with no device
allocator), so the test also checks that repeated calls leave the device's
free memory unchanged.  Both paths run the same quantiser and the same
matmul kernel on the same bytes, so their outputs must be equal bit for bit.
Device-side errors come back only through a caller-owned error word, which
every call here passes and checks.

This file is named so that pytest collects it last.
"""
import ctypes

import pytest
import torch

from glaucis_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def _case(cuda, M, K, N, sizes, seed):
    g = torch.Generator().manual_seed(seed)
    lhs = torch.randn((M, K), generator=g).to(torch.bfloat16).to(cuda)
    rhs = (torch.randn((len(sizes), K, N), generator=g) * 0.02).to(torch.bfloat16).to(cuda)
    b_q, b_s = ops.quant_w_128x128(rhs)
    gs = torch.tensor(sizes, dtype=torch.int32, device=cuda)
    a_q, a_s = ops.quant_act_1x128(lhs)
    ref = ops.gmm_fp8_fwd(a_q, a_s, b_q, b_s, gs, out_dtype=torch.bfloat16)
    return lhs, b_q, b_s, gs, ref


def _noalloc(lhs, b_q, b_s, gs, out, err):
    lib = _lib.load()
    M, K = lhs.shape
    G, _, N = b_q.shape
    rc = lib.gl_gmm_fp8_act_fwd_noalloc(lhs.data_ptr(), b_q.data_ptr(), b_s.data_ptr(),
                                        gs.data_ptr(), G, M, K, N, out.data_ptr(),
                                        _lib.GL_OUT_BF16, err.data_ptr(),
                                        torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "gl_gmm_fp8_act_fwd_noalloc")


def _status(err):
    """Reads and clears the caller-owned device error word."""
    return _lib.device_status(torch.cuda.current_stream().cuda_stream, err.data_ptr())


def test_noalloc_matches_allocating_path_two_calls(cuda):
    # two different problems back to back through the shared scratch array
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    c1 = _case(cuda, 1000, 1024, 512, [300, 0, 129, 500, 71], seed=21)
    c2 = _case(cuda, 384, 2048, 256, [128, 256], seed=22)
    out1 = torch.empty((1000, 512), dtype=torch.bfloat16, device=cuda)
    out2 = torch.empty((384, 256), dtype=torch.bfloat16, device=cuda)
    _noalloc(*c1[:4], out1, err)
    assert _status(err) == 0
    _noalloc(*c2[:4], out2, err)
    assert _status(err) == 0
    assert torch.equal(out1, c1[4]), "first call differs from the allocating path"
    assert torch.equal(out2, c2[4]), "second call differs from the allocating path"
    # the scratch keeps the last call's contents: call the first problem again
    out1b = torch.empty_like(out1)
    _noalloc(*c1[:4], out1b, err)
    assert _status(err) == 0
    assert torch.equal(out1b, c1[4]), "repeat of the first call differs"


def test_noalloc_leaves_free_memory_unchanged(cuda):
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    lhs, b_q, b_s, gs, _ = _case(cuda, 512, 1024, 512, [200, 312], seed=23)
    out = torch.empty((512, 512), dtype=torch.bfloat16, device=cuda)
    _noalloc(lhs, b_q, b_s, gs, out, err)      # first call on the device: set-up
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(2):
        _noalloc(lhs, b_q, b_s, gs, out, err)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    assert _status(err) == 0


def test_noalloc_reports_bad_group_sizes_through_the_error_word(cuda):
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    lhs, b_q, b_s, _, _ = _case(cuda, 256, 512, 256, [128, 128], seed=24)
    bad = torch.tensor([200, 200], dtype=torch.int32, device=cuda)   # sums past M
    out = torch.empty((256, 256), dtype=torch.bfloat16, device=cuda)
    _noalloc(lhs, b_q, b_s, bad, out, err)
    assert _status(err) == 2          # GL_DEV_BAD_GROUPS
    assert _status(err) == 0          # read-and-clear


def test_noalloc_rejects_sizes_beyond_the_scratch(cuda):
    lib = _lib.load()
    limit = 16 * 1024 * 1024
    p = ctypes.c_void_p(256)  # never dereferenced: the size check fails first
    for M in (limit // 1024 + 1, 1 << 55):            # just over the limit; M*K overflowing int64
        rc = lib.gl_gmm_fp8_act_fwd_noalloc(p, p, p, p, 2, M, 1024, 256, p,
                                            _lib.GL_OUT_BF16, None, None)
        assert rc == _lib.GL_EINVAL
        assert "exceeds the static scratch limit" in lib.gl_last_error().decode()
