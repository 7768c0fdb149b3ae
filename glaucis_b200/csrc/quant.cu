// Block-wise FP8 (e4m3fn) quantisers for the grouped matmul operands.
//
// Semantics (absmax calibration, fp32 scale, RNE cast, see
// KE/examples/kernels/gmm_fp8_blockwise.py:84-107 for the qwix calls they
// replace):
//   s = absmax(block) / 448        (1.0 when the block is all zeros)
//   q = cvt.rn.satfinite.e4m3(x / s)
// x / s is the correctly rounded IEEE quotient (this file must not be compiled
// with fast-math), so the result is bit-identical to the CPU oracle.  It is
// computed per element from the block's correctly rounded reciprocal with
// Markstein's FMA correction instead of a full division per element, which
// made the weight quantiser issue-bound rather than HBM-bound.
//
// Data movement (both quantisers): a persistent CTA per SM takes every
// gridDim-th 128 x 128 tile, so the CTAs running together read neighbouring
// tiles (whole rows of the operand at a time).  One producer warp streams the
// bf16 tiles into a shared-memory ring with TMA (32 KB per tile; up to 96 KB
// per CTA for activations with two CTAs per SM, 128 KB for weights with
// one); 16 consumer warps quantise out of shared memory
// and store the e4m3 rows with coalesced 8-byte stores.  Stages are handed
// back through per-stage mbarriers, so consumers work on different tiles at
// the same time and no CTA-wide barrier sits on the tile path:
//   activations: every warp owns 8 rows of every tile (a 1x128 block is one
//                row of a tile, reduced within a half-warp);
//   weights:     the consumer warps form 4 groups of 4 warps, group g takes
//                the CTA's tiles g, g+4, ...; a group reduces the 128x128
//                block maximum over one named barrier, then quantises.
#include "common.cuh"
#include "tmap.h"

namespace gl {

__device__ __forceinline__ uint16_t cvt_e4m3x2(float lo, float hi) {
  uint16_t r;
  // The first source lands in the upper byte, the second in the lower byte.
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// Division by a block scale.  With y = RN(1/s) (one IEEE division per
// block), q = RN(x*y) lies within one ulp of x/s, the residual r = x - q*s is
// exact in one FMA, and RN(q + r*y) is the correctly rounded quotient
// (P. Markstein, "Computation of elementary functions on the IBM RISC
// System/6000 processor", IBM J. Res. Develop. 34(1), 1990).  The residual is
// exact only while it stays above the subnormal range: with s >= 2^-64 every
// element whose quotient can reach a non-zero e4m3 value has |x| >= 2^-74, far
// from it.  Blocks with smaller (or non-finite) scales take the plain
// division.  A quotient by s > 0 has the sign of x; the packed form
// (markstein2) works on -x and -y so that x = -0 keeps its sign without a
// copysign.  The arithmetic runs on packed f32x2 FMAs.  Tests compare this
// path with IEEE division for every finite bf16 block maximum and every bf16
// element value.
struct BlockDiv {
  float s, y;
  bool fast;
  BlockDiv() = default;
  __device__ __forceinline__ explicit BlockDiv(float scale) : s(scale) {
    fast = scale >= 0x1p-64f && scale <= 3.40282347e38f;
    y = 1.0f / scale;
  }
  // recip = 1.0f / scale computed elsewhere (the same IEEE division)
  __device__ __forceinline__ BlockDiv(float scale, float recip) : s(scale), y(recip) {
    fast = scale >= 0x1p-64f && scale <= 3.40282347e38f;
  }
};

__device__ __forceinline__ float2 bf16x2_to_f32x2(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
}

// The two bf16 values of w as negated floats (sign bit flipped in the same
// integer operation that widens them).
__device__ __forceinline__ float2 bf16x2_to_neg_f32x2(uint32_t w) {
  return make_float2(__uint_as_float((w << 16) ^ 0x80000000u), __uint_as_float((w & 0xFFFF0000u) ^ 0x80000000u));
}

// Markstein's quotient of two elements on packed FMAs, in negated form so
// that zeros keep their sign without a copysign: with nx = -x and ny = -y,
// q = nx ny = RN(x y), r' = RN(q s + nx) = q s - x (exact, = -r),
// v = RN(r' ny + q) = RN(q + r y).  For x = +0: q = +0, r' = +0,
// v = -0 + +0 = +0; for x = -0: q = -0, r' = +0, v = -0 + -0 = -0.
__device__ __forceinline__ float2 markstein2(float2 nx, float2 ny, float2 s) {
  const float2 q = __fmul2_rn(nx, ny);
  const float2 r = __ffma2_rn(q, s, nx);
  return __ffma2_rn(r, ny, q);
}

// Eight bf16 values (one 16-byte chunk) -> eight e4m3 bytes.
__device__ __forceinline__ uint2 quant8(const uint4& u, const BlockDiv& d) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
  uint32_t p[4];
  if (d.fast) {
    const float2 ny2 = make_float2(-d.y, -d.y), s2 = make_float2(d.s, d.s);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 v = markstein2(bf16x2_to_neg_f32x2(w[i]), ny2, s2);
      p[i] = cvt_e4m3x2(v.x, v.y);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 x = bf16x2_to_f32x2(w[i]);
      p[i] = cvt_e4m3x2(x.x / d.s, x.y / d.s);
    }
  }
  return make_uint2(p[0] | (p[1] << 16), p[2] | (p[3] << 16));
}

__device__ __forceinline__ float div1(float x, const BlockDiv& d) {
  if (!d.fast) return x / d.s;
  const float q = __fmul_rn(x, d.y);
  return copysignf(__fmaf_rn(__fmaf_rn(-q, d.s, x), d.y, q), x);
}

// Eight bf16 values of eight different columns (one scale each) -> e4m3.
__device__ __forceinline__ uint2 quant8_cols(const uint4& u, const BlockDiv (&d)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
  uint32_t p[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const BlockDiv& d0 = d[2 * i];
    const BlockDiv& d1 = d[2 * i + 1];
    if (d0.fast && d1.fast) {
      const float2 v = markstein2(bf16x2_to_neg_f32x2(w[i]), make_float2(-d0.y, -d1.y),
                                  make_float2(d0.s, d1.s));
      p[i] = cvt_e4m3x2(v.x, v.y);
    } else {
      const float2 x = bf16x2_to_f32x2(w[i]);
      p[i] = cvt_e4m3x2(div1(x.x, d0), div1(x.y, d1));
    }
  }
  return make_uint2(p[0] | (p[1] << 16), p[2] | (p[3] << 16));
}

// max |x| over one chunk, on packed bf16 (exact: the maximum is one of the
// values).
__device__ __forceinline__ float absmax8(const uint4& u) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
  const __nv_bfloat162 m = __hmax2(__hmax2(__habs2(h[0]), __habs2(h[1])),
                                   __hmax2(__habs2(h[2]), __habs2(h[3])));
  return fmaxf(__bfloat162float(m.x), __bfloat162float(m.y));
}

__device__ __forceinline__ float scale_of(float amax) { return amax > 0.f ? amax / 448.f : 1.f; }

namespace quant {

// Ring depth and CTAs per SM.  Activations: all consumer warps take every
// tile in order, 3 stages, two CTAs per SM.  Weights: tile i goes to group
// i % W_GROUPS and to stage i % W_STAGES; W_STAGES is a multiple of W_GROUPS,
// so every stage is only ever used by one group, which therefore waits for
// that stage's phases in order (a waiter that skipped a phase would see the
// stage as full too early).
// Modes: ACT (1x128 blocks along a row), WEIGHT (128x128 blocks), COL (128x1
// blocks: 128 rows of one column, the backward's layouts of lhs and grad).
enum Mode : int { ACT = 0, WEIGHT = 1, COL = 2 };
template <int kMode> struct Ring { static constexpr int STAGES = 4, CTAS_PER_SM = 1; };
template <> struct Ring<ACT> { static constexpr int STAGES = 3, CTAS_PER_SM = 2; };
// COL tiles are 128 rows x 64 columns (16 KB), so that each of the four warp
// groups has two stages of the ring: the next tile of a group loads while the
// group quantises the current one (with 32 KB tiles a group owns one stage
// and waits for every load).
template <> struct Ring<COL> { static constexpr int STAGES = 8, CTAS_PER_SM = 1; };
template <int kMode> struct TileShape {
  static constexpr int W = kMode == COL ? 64 : 128;         // columns of a tile
  static constexpr uint32_t BYTES = 128u * W * 2u;          // bf16
  static constexpr int CPR = W / 8;                         // 16-byte chunks per row
};
constexpr int CONSUMER_WARPS = 16;
constexpr int THREADS = 32 * (CONSUMER_WARPS + 1);  // + producer warp
constexpr int W_GROUPS = 4;                          // weight quantiser: tile groups
constexpr int W_GROUP_WARPS = CONSUMER_WARPS / W_GROUPS;
constexpr uint32_t IN_BYTES = 128 * 128 * 2;
static_assert(Ring<WEIGHT>::STAGES % W_GROUPS == 0 && Ring<COL>::STAGES % W_GROUPS == 0,
              "a grouped stage must belong to one group");
template <int kMode>
struct Layout {
  static constexpr int STAGES = Ring<kMode>::STAGES;
  // per group and parity: one float per warp (WEIGHT) or per warp and column (COL)
  static constexpr int RED_PER_WARP = kMode == COL ? TileShape<kMode>::W : 1;
  static constexpr uint32_t OFF_BAR = STAGES * TileShape<kMode>::BYTES;
  static constexpr uint32_t OFF_RED = OFF_BAR + 2 * STAGES * 8;
  // COL: per group, the tile's column scales and their reciprocals,
  // computed once per column by the thread that owns it
  static constexpr uint32_t OFF_CSC = OFF_RED + W_GROUPS * 2 * W_GROUP_WARPS * RED_PER_WARP * 4;
  static constexpr uint32_t CSC_BYTES = kMode == COL ? W_GROUPS * 2 * TileShape<kMode>::W * 4 : 0;
  static constexpr uint32_t OFF_FLAG = OFF_CSC + CSC_BYTES;
  static constexpr uint32_t SMEM_BYTES = OFF_FLAG + 16 + 1024;  // + slack for 1 KB alignment
};

struct Args {
  uint8_t* q;
  float* s;
  int* err;
  int64_t rows;  // ACT / COL: M; WEIGHT: G*K
  int64_t K;     // ACT / COL: row length; WEIGHT: K
  int64_t N;     // WEIGHT only
  int64_t tiles;
};

// Tile -> (x, y) element coordinates of its top-left corner.
//   ACT / COL: tiles are (128-row slab, column block of TileShape::W),
//              column block fastest;
//   WEIGHT:    tiles are (group, K block, N block), N block fastest.
template <int kMode>
__device__ __forceinline__ void tile_xy(const Args& a, int64_t t, int32_t& x, int32_t& y) {
  if (kMode == WEIGHT) {
    const int64_t NB = a.N / 128, KB = a.K / 128;
    const int64_t g = t / (KB * NB), kb = (t / NB) % KB, nb = t % NB;
    x = static_cast<int32_t>(nb * 128);
    y = static_cast<int32_t>(g * a.K + kb * 128);
  } else {
    constexpr int W = TileShape<kMode>::W;
    const int64_t KB = a.K / W;
    x = static_cast<int32_t>((t % KB) * W);
    y = static_cast<int32_t>((t / KB) * 128);
  }
}

// OR of `v` over the `count` threads of named barrier `id` (a barrier).
__device__ __forceinline__ bool bar_or(int id, int count, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}\n"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "r"(id), "r"(count)
      : "memory");
  return r != 0;
}

template <int kMode>
__global__ void __launch_bounds__(THREADS, Ring<kMode>::CTAS_PER_SM)
    quant_kernel(const __grid_constant__ CUtensorMap tm_in, const Args a) {
  using L = Layout<kMode>;
  constexpr int STAGES = L::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* empty = full + STAGES;
  float* red = reinterpret_cast<float*>(smem + L::OFF_RED);
  int* abort_flag = reinterpret_cast<int*>(smem + L::OFF_FLAG);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // local tile i is global tile blockIdx.x + i * gridDim.x
  const int64_t n = a.tiles > blockIdx.x ? (a.tiles - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
  if (threadIdx.x == 0) {
    prefetch_tmap(&tm_in);
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kMode == ACT ? CONSUMER_WARPS : W_GROUP_WARPS);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  const Abort ab{abort_flag, a.err};

  if (warp == CONSUMER_WARPS) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      int64_t i = 0;
      for (; i < n; ++i) {
        const int st = static_cast<int>(i % STAGES);
        if (!mbar_wait(&empty[st], (static_cast<uint32_t>(i / STAGES) & 1u) ^ 1u, ab)) break;
        int32_t x, y;
        tile_xy<kMode>(a, blockIdx.x + i * gridDim.x, x, y);
        mbar_arrive_expect_tx(&full[st], TileShape<kMode>::BYTES);
        tma_load_2d(smem + st * TileShape<kMode>::BYTES, &tm_in, &full[st], x, y);
      }
      if (i < n) {
        // Aborted: let the loads in flight land before the CTA can exit.
        for (int64_t k = i > STAGES ? i - STAGES : 0; k < i; ++k) {
          const uint64_t w0 = global_ns();
          while (!mbar_try_wait(&full[k % STAGES], static_cast<uint32_t>(k / STAGES) & 1u) &&
                 global_ns() - w0 < 100000000ull) {
          }
        }
      }
    }
    return;
  }

  if (kMode != ACT) {
    // -------------------------------- WEIGHT / COL: groups of 4 warps
    const int grp = warp / W_GROUP_WARPS, gw = warp % W_GROUP_WARPS;
    const int tg = threadIdx.x - grp * W_GROUP_WARPS * 32;  // 0..127
    const int64_t NB = a.N / 128;
    int par = 0;
    for (int64_t i = grp; i < n; i += W_GROUPS, par ^= 1) {
      const int st = static_cast<int>(i % STAGES);
      const bool ok = mbar_wait(&full[st], static_cast<uint32_t>(i / STAGES) & 1u, ab);
      const uint4* in = reinterpret_cast<const uint4*>(smem + st * TileShape<kMode>::BYTES);
      float* r = red + (grp * 2 + par) * W_GROUP_WARPS * L::RED_PER_WARP;
      // this thread's 16-byte (8-column) chunk of the tile's rows: chunk
      // tg % CPR of rows tg / CPR + (128 / CPR) j, i.e. in[tg + 128 j]
      constexpr int CPR = TileShape<kMode>::CPR, RSTEP = 128 / CPR;
      const int c16 = tg % CPR;
      if (kMode == WEIGHT) {
        float m = 0.f;
#pragma unroll 8
        for (int j = 0; j < 16; ++j) m = fmaxf(m, absmax8(in[tg + 128 * j]));
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) r[gw] = m;
      } else {
        // per-column maxima over this thread's CPR rows on packed bf16 (exact:
        // the maximum is one of the values), then over the warp's lanes that
        // share the chunk (l, l ^ CPR, l ^ 2 CPR, ...)
        __nv_bfloat162 cm2[4];
#pragma unroll
        for (int h = 0; h < 4; ++h) cm2[h] = __floats2bfloat162_rn(0.f, 0.f);
#pragma unroll 4
        for (int j = 0; j < CPR; ++j) {
          const uint4 u = in[tg + 128 * j];
          const __nv_bfloat162* hv = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
          for (int h = 0; h < 4; ++h) cm2[h] = __hmax2(cm2[h], __habs2(hv[h]));
        }
#pragma unroll
        for (int o = CPR; o < 32; o <<= 1)
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            const uint32_t v = __shfl_xor_sync(0xffffffffu, *reinterpret_cast<const uint32_t*>(&cm2[h]), o);
            cm2[h] = __hmax2(cm2[h], *reinterpret_cast<const __nv_bfloat162*>(&v));
          }
        if (lane < CPR) {
          float4* rc = reinterpret_cast<float4*>(r + gw * TileShape<kMode>::W + c16 * 8);
          rc[0] = make_float4(__low2float(cm2[0]), __high2float(cm2[0]), __low2float(cm2[1]),
                              __high2float(cm2[1]));
          rc[1] = make_float4(__low2float(cm2[2]), __high2float(cm2[2]), __low2float(cm2[3]),
                              __high2float(cm2[3]));
        }
      }
      if (bar_or(1 + grp, W_GROUP_WARPS * 32, !ok || *static_cast<volatile int*>(abort_flag))) break;
      int32_t x, y;
      tile_xy<kMode>(a, blockIdx.x + i * gridDim.x, x, y);
      const int64_t ld = kMode == WEIGHT ? a.N : a.K;  // row length of the operand
      uint8_t* qbase = a.q + static_cast<int64_t>(y) * ld + x + c16 * 8;
      if (kMode == WEIGHT) {
        float m = 0.f;
#pragma unroll
        for (int w = 0; w < W_GROUP_WARPS; ++w) m = fmaxf(m, r[w]);
        const float sc = scale_of(m);
        const BlockDiv div(sc);
#pragma unroll 4
        for (int j = 0; j < 16; ++j) {
          const int row = (tg >> 4) + 8 * j;
          *reinterpret_cast<uint2*>(qbase + static_cast<int64_t>(row) * ld) = quant8(in[tg + 128 * j], div);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
        if (tg == 0) a.s[(y / 128) * NB + x / 128] = sc;  // s[g, kb, nb]; y / 128 = g * KB + kb
      } else {
        // thread tg owns column tg of the tile: its maximum over the group's
        // warps, its scale (also stored to s[row block, column]) and the
        // scale's reciprocal, shared through shared memory
        constexpr int W = TileShape<kMode>::W;
        float* csc = reinterpret_cast<float*>(smem + L::OFF_CSC) + grp * 2 * W;
        if (tg < W) {
          float m = r[tg];
#pragma unroll
          for (int w = 1; w < W_GROUP_WARPS; ++w) m = fmaxf(m, r[w * W + tg]);
          const float sc1 = scale_of(m);
          csc[tg] = sc1;
          csc[W + tg] = 1.0f / sc1;
          a.s[static_cast<int64_t>(y / 128) * a.K + x + tg] = sc1;
        }
        asm volatile("bar.sync %0, %1;" ::"r"(1 + grp), "r"(W_GROUP_WARPS * 32) : "memory");
        BlockDiv div[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) div[e] = BlockDiv(csc[c16 * 8 + e], csc[W + c16 * 8 + e]);
#pragma unroll 4
        for (int j = 0; j < CPR; ++j) {
          const int row = tg / CPR + RSTEP * j;
          *reinterpret_cast<uint2*>(qbase + static_cast<int64_t>(row) * ld) =
              quant8_cols(in[tg + 128 * j], div);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
      }
    }
  } else {
    // ------------------------------- activations: every warp owns 8 rows
    // Pass p covers rows 8 * warp + 4 p .. + 3, eight lanes per row; lane l
    // of a row takes its 16-byte chunks l and l + 8 (conflict-free: the 8
    // lanes of a row read 128 contiguous bytes per load).
    const int64_t KB = a.K / 128;
    const int rsub = lane >> 3, l8 = lane & 7;
    for (int64_t i = 0; i < n; ++i) {
      const int st = static_cast<int>(i % STAGES);
      if (!mbar_wait(&full[st], static_cast<uint32_t>(i / STAGES) & 1u, ab)) break;
      const uint4* in = reinterpret_cast<const uint4*>(smem + st * TileShape<kMode>::BYTES);
      int32_t x, y;
      tile_xy<kMode>(a, blockIdx.x + i * gridDim.x, x, y);
      uint4 u[2][2];
#pragma unroll
      for (int pass = 0; pass < 2; ++pass)
#pragma unroll
        for (int k = 0; k < 2; ++k) u[pass][k] = in[(warp * 8 + 4 * pass + rsub) * 16 + l8 + 8 * k];
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
#pragma unroll
      for (int pass = 0; pass < 2; ++pass) {
        float m = fmaxf(absmax8(u[pass][0]), absmax8(u[pass][1]));
#pragma unroll
        for (int o = 4; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        const float sc = scale_of(m);
        const BlockDiv div(sc);
        const int64_t row = y + warp * 8 + 4 * pass + rsub;
        if (row < a.rows) {
          uint8_t* qrow = a.q + row * a.K + x;
#pragma unroll
          for (int k = 0; k < 2; ++k)
            *reinterpret_cast<uint2*>(qrow + (l8 + 8 * k) * 8) = quant8(u[pass][k], div);
          if (l8 == 0) a.s[row * KB + x / 128] = sc;
        }
      }
    }
  }
}

}  // namespace quant
}  // namespace gl

namespace {

template <int kMode>
int launch_quant(const void* in, void* q, float* s, int* err, int64_t rows, int64_t K, int64_t N,
                 cudaStream_t st, int num_sms, const char** why) {
  using namespace gl::quant;
  const int64_t inner = kMode == WEIGHT ? N : K;
  CUtensorMap tm_in;
  if (!gl_make_tmap_2d(&tm_in, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, in, inner, rows, inner,
                       gl::quant::TileShape<kMode>::W, 128, CU_TENSOR_MAP_SWIZZLE_NONE, why))
    return -1;
  Args a;
  a.q = static_cast<uint8_t*>(q);
  a.s = s;
  a.err = err;
  a.rows = rows;
  a.K = K;
  a.N = N;
  a.tiles = kMode == WEIGHT ? (rows / 128) * (N / 128)
                            : ((rows + 127) / 128) * (K / TileShape<kMode>::W);
  const void* fn = reinterpret_cast<const void*>(quant_kernel<kMode>);
  constexpr uint32_t smem_bytes = Layout<kMode>::SMEM_BYTES;
  if (!gl_set_smem_attr(fn, 0, static_cast<int>(smem_bytes), why)) return -2;
  const int64_t slots = static_cast<int64_t>(num_sms) * Ring<kMode>::CTAS_PER_SM;
  const int64_t grid = a.tiles < slots ? a.tiles : slots;
  quant_kernel<kMode><<<static_cast<unsigned>(grid > 0 ? grid : 1), THREADS, smem_bytes, st>>>(
      tm_in, a);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    *why = cudaGetErrorString(e);
    return -2;
  }
  return 0;
}

}  // namespace

// Host launchers (called from capi.cu and noalloc.cu).  0 = launched,
// -1 = operand rejected by the tensor-map encoder, -2 = launch failure.
int gl_launch_quant_act(const void* x, int64_t M, int64_t K, void* q, float* s, int* err,
                        cudaStream_t st, int num_sms, const char** why) {
  return launch_quant<gl::quant::ACT>(x, q, s, err, M, K, 0, st, num_sms, why);
}

int gl_launch_quant_w(const void* w, int64_t G, int64_t K, int64_t N, void* q, float* s, int* err,
                      cudaStream_t st, int num_sms, const char** why) {
  return launch_quant<gl::quant::WEIGHT>(w, q, s, err, G * K, K, N, st, num_sms, why);
}

// 128x1 column blocks of x [M, C] (M % 128 == 0): q [M, C], s [M/128, C].
int gl_launch_quant_col(const void* x, int64_t M, int64_t C, void* q, float* s, int* err,
                        cudaStream_t st, int num_sms, const char** why) {
  return launch_quant<gl::quant::COL>(x, q, s, err, M, C, 0, st, num_sms, why);
}
