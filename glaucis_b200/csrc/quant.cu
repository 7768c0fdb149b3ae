// Block-wise FP8 (e4m3fn) quantisers for the grouped matmul operands.
//
// Semantics (absmax calibration, fp32 scale, RNE cast, see
// KE/examples/kernels/gmm_fp8_blockwise.py:84-107 for the qwix calls they
// replace):
//   s = absmax(block) / 448        (1.0 when the block is all zeros)
//   q = cvt.rn.satfinite.e4m3(x / s)
// The division is IEEE round-to-nearest (this file must not be compiled with
// fast-math), so the result is bit-identical to the CPU oracle.
#include "common.cuh"

namespace gl {

__device__ __forceinline__ uint16_t cvt_e4m3x2(float lo, float hi) {
  uint16_t r;
  // The first source lands in the upper byte, the second in the lower byte.
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ void bf16x8_to_f32(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

__device__ __forceinline__ uint2 quant8(const float (&f)[8], float s) {
  uint32_t p[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) p[i] = cvt_e4m3x2(f[2 * i] / s, f[2 * i + 1] / s);
  return make_uint2(p[0] | (p[1] << 16), p[2] | (p[3] << 16));
}

__device__ __forceinline__ float scale_of(float amax) { return amax > 0.f ? amax / 448.f : 1.f; }

// One 1x128 block per half-warp (16 lanes x 8 bf16).  Both half-warps of a
// warp always iterate together so the full-mask shuffles stay converged.
__global__ void __launch_bounds__(256) quant_act_1x128_kernel(const __nv_bfloat16* __restrict__ x,
                                                              int64_t M, int64_t K,
                                                              uint8_t* __restrict__ q,
                                                              float* __restrict__ s) {
  const int64_t KB = K / 128;
  const int64_t nblocks = M * KB;
  const int lane = threadIdx.x & 31;
  const int half = lane >> 4, sub = lane & 15;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t pair = warp; pair * 2 < nblocks; pair += nwarps) {
    const int64_t blk = pair * 2 + half;
    const bool valid = blk < nblocks;
    const int64_t m = valid ? blk / KB : 0, kb = valid ? blk % KB : 0;
    const int64_t off = m * K + kb * 128 + sub * 8;
    uint4 u = make_uint4(0, 0, 0, 0);
    if (valid) u = __ldg(reinterpret_cast<const uint4*>(x + off));
    float f[8];
    bf16x8_to_f32(u, f);
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(f[i]));
#pragma unroll
    for (int o = 8; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float sc = scale_of(amax);
    if (valid) {
      *reinterpret_cast<uint2*>(q + off) = quant8(f, sc);
      if (sub == 0) s[m * KB + kb] = sc;
    }
  }
}

// One 128x128 block of one group per CTA (256 threads; thread t owns the
// 16-byte column chunk t%16 of rows (t/16)*8 .. (t/16)*8+7).
__global__ void __launch_bounds__(256) quant_w_128x128_kernel(const __nv_bfloat16* __restrict__ w,
                                                              int64_t G, int64_t K, int64_t N,
                                                              uint8_t* __restrict__ q,
                                                              float* __restrict__ s) {
  const int64_t KB = K / 128, NB = N / 128;
  const int64_t nblk = G * KB * NB;
  __shared__ float red[8];
  const int t = threadIdx.x, c = t & 15, rg = t >> 4;
  for (int64_t b = blockIdx.x; b < nblk; b += gridDim.x) {
    const int64_t g = b / (KB * NB), kb = (b / NB) % KB, nb = b % NB;
    const int64_t base = (g * K + kb * 128 + rg * 8) * N + nb * 128 + c * 8;
    float f[8][8];
    float amax = 0.f;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(w + base + r * N));
      bf16x8_to_f32(u, f[r]);
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(f[r][i]));
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((t & 31) == 0) red[t >> 5] = amax;
    __syncthreads();
    amax = red[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) amax = fmaxf(amax, red[i]);
    __syncthreads();  // red[] is rewritten by the next block
    const float sc = scale_of(amax);
#pragma unroll
    for (int r = 0; r < 8; ++r) *reinterpret_cast<uint2*>(q + base + r * N) = quant8(f[r], sc);
    if (t == 0) s[(g * KB + kb) * NB + nb] = sc;
  }
}

}  // namespace gl

// Host launchers (called from capi.cu).
int gl_launch_quant_act(const void* x, int64_t M, int64_t K, void* q, float* s,
                        cudaStream_t st, int num_sms) {
  const int64_t pairs = (M * (K / 128) + 1) / 2;  // one pair per warp-iteration
  const int64_t want = (pairs + 7) / 8;           // 8 warps per CTA
  const int grid = static_cast<int>(want < static_cast<int64_t>(num_sms) * 16
                                        ? (want > 0 ? want : 1)
                                        : static_cast<int64_t>(num_sms) * 16);
  gl::quant_act_1x128_kernel<<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x), M, K,
                                                   static_cast<uint8_t*>(q), s);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int gl_launch_quant_w(const void* w, int64_t G, int64_t K, int64_t N, void* q, float* s,
                      cudaStream_t st, int num_sms) {
  const int64_t nblk = G * (K / 128) * (N / 128);
  const int64_t cap = static_cast<int64_t>(num_sms) * 8;
  const int grid = static_cast<int>(nblk < cap ? (nblk > 0 ? nblk : 1) : cap);
  gl::quant_w_128x128_kernel<<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(w), G, K, N,
                                                   static_cast<uint8_t*>(q), s);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}
