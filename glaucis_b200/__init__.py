"""glaucis_b200: B200-native (sm_100a) kernels for the two kernels scored by the
Glaucis kernel evaluator — the block-wise FP8 grouped matmul and the chunked
Gated Linear Attention forward — behind the reference templates' call
signatures.  See include/glaucis_b200.h for the C ABI."""
from . import _lib
from .ops import (chunk_gla, chunk_gla_fwd, device_status, gmm_fp8_blockwise, gmm_fp8_fwd,
                  quant_act_1x128, quant_w_128x128)

__all__ = ["chunk_gla", "chunk_gla_fwd", "device_status", "gmm_fp8_blockwise", "gmm_fp8_fwd",
           "quant_act_1x128", "quant_w_128x128", "_lib"]
