"""The C-ABI library loads and exports every symbol the header declares; the
argument checks that run before any device work reject bad calls (no GPU)."""
import ctypes
import os
import re

import pytest

from glaucis_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(__file__)), "include", "glaucis_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|size_t|const char\s*\*)\s*(gl_\w+)\s*\(", text, re.M)))


def test_header_declares_the_abi():
    syms = declared_symbols()
    assert set(_lib.SIGNATURES) == set(syms), syms


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_lib.lib_path()))
    for s in declared_symbols():
        assert hasattr(lib, s), s
    assert _lib.load().gl_version().startswith(b"glaucis_b200")


def _err():
    return _lib.load().gl_last_error().decode()


def test_gmm_rejects_bad_arguments_without_device():
    lib = _lib.load()
    rc = lib.gl_gmm_fp8_fwd(None, None, None, None, None, 4, 128, 256, 256, None, 0, None, None)
    assert rc == _lib.GL_EINVAL and "null pointer" in _err()
    p = ctypes.c_void_p(16)  # never dereferenced: validation fails first
    rc = lib.gl_gmm_fp8_fwd(p, p, p, p, p, 4, 128, 200, 256, p, 0, None, None)
    assert rc == _lib.GL_EINVAL and "multiples of 128" in _err()
    rc = lib.gl_gmm_fp8_fwd(p, p, p, p, p, 0, 128, 256, 256, p, 0, None, None)
    assert rc == _lib.GL_EINVAL and "G" in _err()
    rc = lib.gl_gmm_fp8_fwd(p, p, p, p, p, 4, 128, 256, 256, p, 7, None, None)
    assert rc == _lib.GL_EINVAL and "out_dtype" in _err()


def test_gla_rejects_bad_arguments_without_device():
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    f = ctypes.c_void_p(32)
    rc = lib.gl_chunk_gla_fwd(p, p, p, f, f, None, 0.1, 1, 64, 1, 128, 128, 64, p, None, None, None)
    assert rc == _lib.GL_EINVAL and "exactly one" in _err()
    rc = lib.gl_chunk_gla_fwd(p, p, p, f, None, None, 0.1, 1, 64, 1, 64, 128, 64, p, None, None, None)
    assert rc == _lib.GL_EINVAL and "128" in _err()
    rc = lib.gl_chunk_gla_fwd(p, p, p, f, None, None, 0.1, 1, 100, 1, 128, 128, 64, p, None, None, None)
    assert rc == _lib.GL_EINVAL and "multiple of 64" in _err()
    rc = lib.gl_chunk_gla_fwd(p, p, p, f, None, None, 0.1, 1, 64, 1, 128, 128, 32, p, None, None, None)
    assert rc == _lib.GL_EINVAL and "chunk_size" in _err()
    # the workspace variant: same checks, plus a 256-byte aligned workspace
    rc = lib.gl_chunk_gla_fwd_ws(p, p, p, f, f, None, 0.1, 1, 64, 1, 128, 128, 64, p, None,
                                 None, 0, None, None)
    assert rc == _lib.GL_EINVAL and "exactly one" in _err()
    rc = lib.gl_chunk_gla_fwd_ws(p, p, p, f, None, None, 0.1, 1, 64, 1, 128, 128, 64, p, None,
                                 ctypes.c_void_p(272), 4096, None, None)
    assert rc == _lib.GL_EINVAL and "256-byte" in _err()
    # workspace size query: 0 for unsupported shapes (no device needed)
    assert lib.gl_chunk_gla_fwd_workspace_bytes(1, 100, 1, 128, 128, 64) == 0
    assert lib.gl_chunk_gla_bwd_workspace_bytes(1, 100, 1, 128, 128, 64) == 0
    # training forward: the per-chunk state output is required
    rc = lib.gl_chunk_gla_fwd_states(p, p, p, f, None, None, 0.1, 1, 64, 1, 128, 128, 64, p, None,
                                     None, None, 0, None, None)
    assert rc == _lib.GL_EINVAL and "h_states" in _err()
    # backward: shape checks, then the required workspace
    rc = lib.gl_chunk_gla_bwd(p, p, p, f, f, p, p, None, 0.1, 1, 64, 1, 128, 128, 64, p, p, p,
                              None, None, 0, None, None)
    assert rc == _lib.GL_EINVAL and "exactly one" in _err()
    rc = lib.gl_chunk_gla_bwd(p, p, p, f, None, None, p, None, 0.1, 1, 64, 1, 128, 128, 64, p, p,
                              p, None, None, 0, None, None)
    assert rc == _lib.GL_EINVAL and "null pointer" in _err()
    rc = lib.gl_chunk_gla_bwd(p, p, p, f, None, p, p, None, 0.1, 1, 64, 1, 128, 128, 64, p, p, p,
                              None, None, 0, None, None)
    assert rc == _lib.GL_EINVAL and "workspace" in _err()
    rc = lib.gl_chunk_gla_bwd(p, p, p, f, None, p, p, None, 0.1, 1, 64, 1, 128, 128, 64, p, p, p,
                              None, ctypes.c_void_p(272), 1 << 20, None, None)
    assert rc == _lib.GL_EINVAL and "256-byte" in _err()


def test_quantisers_reject_bad_arguments_without_device():
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    assert lib.gl_quant_act_1x128(p, 4, 100, p, p, None, None) == _lib.GL_EINVAL
    assert lib.gl_quant_w_128x128(p, 1, 128, 96, p, p, None, None) == _lib.GL_EINVAL
    assert lib.gl_quant_act_1x128(None, 4, 128, p, p, None, None) == _lib.GL_EINVAL


def test_ops_refuse_cpu_tensors():
    import torch
    from glaucis_b200 import ops
    with pytest.raises(ValueError, match="CUDA"):
        ops.quant_act_1x128(torch.zeros(4, 128, dtype=torch.bfloat16))


def test_gla_options_and_intermediates_reject_bad_arguments_without_device():
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    f = ctypes.c_void_p(32)
    # gl_chunk_gla_fwd_ex: only GL_GLA_BF16_INTRA is a known flag
    rc = lib.gl_chunk_gla_fwd_ex(p, p, p, f, None, None, 0.1, 1, 64, 1, 128, 128, 64, p, None,
                                 None, None, 0, 2, None, None)
    assert rc == _lib.GL_EINVAL and "unknown flags" in _err()
    rc = lib.gl_chunk_gla_fwd_ex(p, p, p, f, f, None, 0.1, 1, 64, 1, 128, 128, 64, p, None,
                                 None, None, 0, _lib.GL_GLA_BF16_INTRA, None, None)
    assert rc == _lib.GL_EINVAL and "exactly one" in _err()
    # gl_chunk_gla_fwd_intermediates: at least one output, one gate, K = 128
    rc = lib.gl_chunk_gla_fwd_intermediates(p, p, f, None, 0.1, 1, 64, 1, 128, 64, None, None,
                                            None, None)
    assert rc == _lib.GL_EINVAL and "neither" in _err()
    rc = lib.gl_chunk_gla_fwd_intermediates(p, p, f, f, 0.1, 1, 64, 1, 128, 64, f, None, None, None)
    assert rc == _lib.GL_EINVAL and "exactly one" in _err()
    rc = lib.gl_chunk_gla_fwd_intermediates(p, p, f, None, 0.1, 1, 64, 1, 64, 64, f, None, None, None)
    assert rc == _lib.GL_EINVAL and "128" in _err()


def test_gla_scatter_rejects_bad_arguments_without_device():
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    f = ctypes.c_void_p(32)
    one = (ctypes.c_void_p * 1)(16)
    nine = (ctypes.c_void_p * 9)(*([16] * 9))
    odd = (ctypes.c_void_p * 2)(16, 24)  # the second output is not 16-byte aligned

    def call(outs, n, flags=0, g=f, gg=None):
        return lib.gl_chunk_gla_fwd_scatter(p, p, p, g, gg, None, 0.1, 1, 64, 1, 128, 128, 64,
                                            ctypes.cast(outs, ctypes.c_void_p) if outs is not None
                                            else None, n, None, None, 0, flags, None, None)

    assert call(None, 1) == _lib.GL_EINVAL and "null" in _err()
    assert call(one, 0) == _lib.GL_EINVAL and "n_outs" in _err()
    assert call(nine, 9) == _lib.GL_EINVAL and "n_outs" in _err()
    assert call(odd, 2) == _lib.GL_EINVAL and "aligned" in _err()
    assert call(one, 1, flags=4) == _lib.GL_EINVAL and "unknown flags" in _err()
    assert call(one, 1, gg=f) == _lib.GL_EINVAL and "exactly one" in _err()
