// The two intermediates of the chunked GLA forward that the fused kernel
// keeps on chip, materialised on request for callers of the template's
// chunk_gla_fwd -> (g_cumsum, A, h, o) that read them
// (KE/examples/kernels/chunk_gla.py:258-273):
//   g_cumsum fp32 [B, T, H, K]  chunk-local cumsum of the per-key gate g, or
//                               g_gamma[h] * (1..C) for the per-head gate
//                               (chunk_gla.py:265-267)
//   A        fp32 [B, T, H, C]  A[i, j] = scale * sum_k q[i,k] e^{G[i,k]}
//                               k[j,k] e^{-G[j,k]} over the full C x C square
//                               of each chunk (the causal mask is applied only
//                               when o is formed), chunk_gla.py:146-188
// A is an fp32 contraction in the reference (Precision.HIGHEST), so it is
// computed here with fp32 FMAs, not on the bf16 tensor path.  One CTA per
// (batch, chunk, head): 256 threads build q e^G and k e^-G transposed in
// shared memory (one key column per thread, the cumsum running down the
// chunk), then each thread accumulates a 4x4 block of A over the 128 keys.
#include <cuda_runtime.h>

#include <cstdint>

#include <cuda_bf16.h>

namespace gl {
namespace glai {

constexpr int C = 64, KD = 128, THREADS = 256;
constexpr int LD = C + 4;  // row pitch (floats) of the transposed tiles: 16-byte rows, 4-way stores
constexpr int SMEM_BYTES = 2 * KD * LD * 4;

__global__ void __launch_bounds__(THREADS)
gla_intermediates_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                         const float* __restrict__ g, const float* __restrict__ g_gamma,
                         float scale, int T, int H, float* __restrict__ g_cumsum,
                         float* __restrict__ A) {
  extern __shared__ __align__(16) float smem[];
  float* qgT = smem;            // [KD][LD]: q e^G, key-major
  float* kgT = smem + KD * LD;  // [KD][LD]: k e^-G
  const int NT = T / C;
  const int h = blockIdx.x % H;
  const int n = (blockIdx.x / H) % NT;
  const int b = blockIdx.x / (H * NT);
  const int64_t row0 = (static_cast<int64_t>(b) * T + static_cast<int64_t>(n) * C) * H + h;  // token row of (b, n*C, h)
  const int t = threadIdx.x;

  // one key column per thread: threads 0-127 gate q, 128-255 gate k (both run the cumsum)
  {
    const int kk = t & (KD - 1);
    const bool is_k = t >= KD;
    const __nv_bfloat16* src = is_k ? k : q;
    float* dst = is_k ? kgT : qgT;
    const float gam = g == nullptr ? g_gamma[h] : 0.f;
    float G = 0.f;
    for (int i = 0; i < C; ++i) {
      const int64_t off = (row0 + static_cast<int64_t>(i) * H) * KD + kk;
      G = g != nullptr ? G + g[off] : gam * static_cast<float>(i + 1);
      if (!is_k && g_cumsum != nullptr) g_cumsum[off] = G;
      const float x = __bfloat162float(src[off]);
      dst[kk * LD + i] = is_k ? x * expf(-G) : x * expf(G);
    }
  }
  __syncthreads();
  if (A == nullptr) return;

  const int ti = t >> 4, tj = t & 15;  // rows 4ti..4ti+3, columns 4tj..4tj+3
  float acc[4][4] = {};
#pragma unroll 4
  for (int kk = 0; kk < KD; ++kk) {
    const float4 a = *reinterpret_cast<const float4*>(qgT + kk * LD + 4 * ti);
    const float4 c = *reinterpret_cast<const float4*>(kgT + kk * LD + 4 * tj);
    const float av[4] = {a.x, a.y, a.z, a.w}, cv[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int s = 0; s < 4; ++s) acc[r][s] = fmaf(av[r], cv[s], acc[r][s]);
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int64_t off = (row0 + static_cast<int64_t>(4 * ti + r) * H) * C + 4 * tj;
    *reinterpret_cast<float4*>(A + off) =
        make_float4(acc[r][0] * scale, acc[r][1] * scale, acc[r][2] * scale, acc[r][3] * scale);
  }
}

}  // namespace glai
}  // namespace gl

bool gl_set_smem_attr(const void* func, int, int bytes, const char** why);

// Returns 0 on a launch, -1 on a bad argument (why set), -2 on a launch error.
int gl_launch_gla_intermediates(const void* q, const void* k, const float* g, const float* g_gamma,
                                float scale, int64_t B, int64_t T, int64_t H, float* g_cumsum,
                                float* A, cudaStream_t st, const char** why) {
  using namespace gl::glai;
  if (T % C != 0) {
    *why = "T must be a multiple of 64";
    return -1;
  }
  const int64_t ctas = B * (T / C) * H;
  if (ctas <= 0) return 0;
  if (ctas > 0x7fffffff) {
    *why = "B*T/64*H must fit in 31 bits";
    return -1;
  }
  if (!gl_set_smem_attr(reinterpret_cast<const void*>(&gla_intermediates_kernel), 0, SMEM_BYTES, why))
    return -2;
  gla_intermediates_kernel<<<static_cast<unsigned>(ctas), THREADS, SMEM_BYTES, st>>>(
      static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k), g, g_gamma, scale,
      static_cast<int>(T), static_cast<int>(H), g_cumsum, A);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    *why = cudaGetErrorString(e);
    return -2;
  }
  return 0;
}
