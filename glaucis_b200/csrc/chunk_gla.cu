// Chunked Gated Linear Attention forward, fused into one sm_100a kernel.
//
// Replaces the three pallas_calls of the Glaucis template's chunk_gla_fwd
// (KE/examples/kernels/chunk_gla.py:258-273: chunk_fwd_h :94-138,
// chunk_gla_fwd_intra_gk :163-188, chunk_gla_fwd_o_gk :218-250) and adds the
// per-key gate / initial-state / final-state semantics of
// KE/upstream/fused_chunk_simple_gla/common_chunk_h.py:275-360.
//
// Per chunk n of C = 64 tokens (G = chunk-local cumsum of the log-gate):
//   Qs = scale * q * e^G,  Kg = k * e^-G                       (bf16, in place)
//   A  = Qs Kg^T                       tcgen05 M=64  N=64   K=128  (TMEM)
//   S  = Kg^T V                        tcgen05 M=128 N=VS   K=64   (TMEM)
//   O  = Qs H_n + tril(A) V            tcgen05 M=64  N=VS   K=128+64
//   h_{n+1} = e^{G_last} * (h_n + S)   fp32 in registers, H_{n+1} = bf16(h_{n+1})
// which is the reference recurrence h_{n+1} = e^{G_last} h_n
// + (k e^{G_last-G})^T v with the per-key decay factored out of the sum.
// g_cumsum, A and the per-chunk states never touch HBM: q, k, v, g are read
// once and o (+ the final state) written once.
//
// One CTA per (batch, head, V slice of width VS), 512 threads:
//   warp 0        TMA producer (q, k, v chunk; g chunk)
//   warp 1        tcgen05.mma issuer
//   warp 2        TMEM allocator
//   warps 4-7     gating (thread = key), then A -> tril -> bf16 P
//   warps 8-15    two warpgroups, each owning VS/2 state columns: state
//                 update (thread = key row), then the O epilogue
#include "common.cuh"

namespace gl {
namespace gla {

constexpr int C = 64, KD = 128, NUM_THREADS = 512;

template <int VS>
struct Cfg {
  static constexpr int V_BOXES = VS / 64;
  static constexpr uint32_t Q_BYTES = C * KD * 2;          // 16 KB (2 boxes of 64 features)
  static constexpr uint32_t V_BYTES = C * VS * 2;          // 8 / 16 KB
  static constexpr uint32_t G_BYTES = C * KD * 4;          // 32 KB
  static constexpr uint32_t P_BYTES = C * C * 2;           // 8 KB
  static constexpr uint32_t H_BYTES = KD * VS * 2;         // 16 / 32 KB
  static constexpr uint32_t OFF_Q = 0;
  static constexpr uint32_t OFF_K = OFF_Q + 2 * Q_BYTES;
  static constexpr uint32_t OFF_V = OFF_K + 2 * Q_BYTES;
  static constexpr uint32_t OFF_G = OFF_V + 2 * V_BYTES;
  static constexpr uint32_t OFF_P = OFF_G + G_BYTES;
  static constexpr uint32_t OFF_H = OFF_P + P_BYTES;
  static constexpr uint32_t OFF_DEC = OFF_H + 2 * H_BYTES;  // 2 x 128 floats
  static constexpr uint32_t OFF_BAR = OFF_DEC + 2 * KD * 4;
  static constexpr uint32_t OFF_MISC = OFF_BAR + 256;
  static constexpr uint32_t SMEM_BYTES = OFF_MISC + 64 + 1024;
  // TMEM columns: A [0,64), O [64,64+VS), S0, S1
  static constexpr uint32_t COL_A = 0, COL_O = 64, COL_S = 64 + VS;
  static constexpr uint32_t TMEM_COLS = (64 + 3 * VS) <= 256 ? 256 : 512;
  static constexpr uint32_t IDESC_A = idesc(1, 1, 1, 0, 0, 64, 64);    // bf16, K-major x K-major
  static constexpr uint32_t IDESC_S = idesc(1, 1, 1, 1, 1, 128, VS);  // MN-major x MN-major
  static constexpr uint32_t IDESC_O = idesc(1, 1, 1, 0, 1, 64, VS);   // K-major x MN-major
};

struct Params {
  const float* g_gamma;  // [H] or null
  const float* h0;       // [B,H,K,V] or null
  __nv_bfloat16* o;      // [B,T,H,V]
  float* ht;             // [B,H,K,V] or null
  int* err;
  float scale;
  int B, T, H, nsplit;
  int has_g;
};

// Barrier indices.
enum {
  B_QKV_FULL = 0,   // [2]
  B_QKV_EMPTY = 2,  // [2]
  B_G_FULL = 4,
  B_G_EMPTY = 5,
  B_PREP = 6,       // [2]
  B_DEC_FULL = 8,   // [2]
  B_DEC_EMPTY = 10, // [2]
  B_A_FULL = 12,
  B_A_EMPTY = 13,
  B_P_FULL = 14,
  B_S_FULL = 15,    // [2]
  B_S_EMPTY = 17,   // [2]
  B_H_FULL = 19,    // [2]
  B_O_FULL = 21,
  B_O_EMPTY = 22,
  B_DRAIN = 23,
  NUM_BARS = 24
};

// Offset of bf16 element (row, col) in a K-major, 128B-swizzled tile made of
// 64-column atoms stacked `atom_stride` bytes apart (rows 128 B apart).
__device__ __forceinline__ uint32_t kmaj_off(uint32_t row, uint32_t col, uint32_t atom_stride) {
  return (col >> 6) * atom_stride + row * 128u + ((((col & 63u) >> 3) ^ (row & 7u)) << 4) +
         (col & 7u) * 2u;
}

template <int VS>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    chunk_gla_fwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                         const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v,
                         const __grid_constant__ CUtensorMap tm_g, const Params p) {
  using CF = Cfg<VS>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + CF::OFF_BAR);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + CF::OFF_MISC);
  int* abort_flag = reinterpret_cast<int*>(smem + CF::OFF_MISC + 4);
  float* dec = reinterpret_cast<float*>(smem + CF::OFF_DEC);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int T = p.T, H = p.H;
  const int NT = T / C;
  const int bh = blockIdx.x / p.nsplit, vsl = blockIdx.x % p.nsplit;
  const int b = bh / H, h = bh % H;
  const int v0 = vsl * VS;
  const int tok0 = b * T;
  const Abort ab{abort_flag, p.err};

  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
    if (p.has_g) prefetch_tmap(&tm_g);
  } else if (warp == 1 && lane == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar[B_QKV_FULL + i], 1);
      mbar_init(&bar[B_QKV_EMPTY + i], 1);
      mbar_init(&bar[B_PREP + i], 4);
      mbar_init(&bar[B_DEC_FULL + i], 4);
      mbar_init(&bar[B_DEC_EMPTY + i], 8);
      mbar_init(&bar[B_S_FULL + i], 1);
      mbar_init(&bar[B_S_EMPTY + i], 8);
      mbar_init(&bar[B_H_FULL + i], 8);
    }
    mbar_init(&bar[B_G_FULL], 1);
    mbar_init(&bar[B_G_EMPTY], 4);
    mbar_init(&bar[B_A_FULL], 1);
    mbar_init(&bar[B_A_EMPTY], 4);
    mbar_init(&bar[B_P_FULL], 4);
    mbar_init(&bar[B_O_FULL], 1);
    mbar_init(&bar[B_O_EMPTY], 8);
    mbar_init(&bar[B_DRAIN], 1);
    *abort_flag = 0;
    fence_mbar_init();
  } else if (warp == 2) {
    tmem_alloc(tmem_holder, CF::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const uint32_t s_base = smem_u32(smem);

  if (warp == 0) {
    // ----------------------------------------------------------------- TMA
    if (lane == 0) {
      bool ok = true;
      for (int n = 0; n < NT && ok; ++n) {
        const int s = n & 1;
        const int tok = tok0 + n * C;
        if (!mbar_wait(&bar[B_QKV_EMPTY + s], ((n >> 1) & 1) ^ 1, ab)) { ok = false; break; }
        mbar_arrive_expect_tx(&bar[B_QKV_FULL + s], 2 * CF::Q_BYTES + CF::V_BYTES);
        uint8_t* qd = smem + CF::OFF_Q + s * CF::Q_BYTES;
        uint8_t* kd = smem + CF::OFF_K + s * CF::Q_BYTES;
        uint8_t* vd = smem + CF::OFF_V + s * CF::V_BYTES;
        tma_load_3d(qd, &tm_q, &bar[B_QKV_FULL + s], 0, h, tok);
        tma_load_3d(qd + 8192, &tm_q, &bar[B_QKV_FULL + s], 64, h, tok);
        tma_load_3d(kd, &tm_k, &bar[B_QKV_FULL + s], 0, h, tok);
        tma_load_3d(kd + 8192, &tm_k, &bar[B_QKV_FULL + s], 64, h, tok);
#pragma unroll
        for (int j = 0; j < CF::V_BOXES; ++j)
          tma_load_3d(vd + j * 8192, &tm_v, &bar[B_QKV_FULL + s], v0 + 64 * j, h, tok);
        if (p.has_g) {
          if (!mbar_wait(&bar[B_G_EMPTY], (n & 1) ^ 1, ab)) { ok = false; break; }
          mbar_arrive_expect_tx(&bar[B_G_FULL], CF::G_BYTES);
          tma_load_3d(smem + CF::OFF_G, &tm_g, &bar[B_G_FULL], 0, h, tok);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA
    if (lane == 0) {
      bool ok = true;
      const uint32_t p_addr = s_base + CF::OFF_P;
      for (int n = 0; n < NT && ok; ++n) {
        const int s = n & 1;
        const uint32_t ph2 = (n >> 1) & 1;
        const uint32_t q_addr = s_base + CF::OFF_Q + s * CF::Q_BYTES;
        const uint32_t k_addr = s_base + CF::OFF_K + s * CF::Q_BYTES;
        const uint32_t v_addr = s_base + CF::OFF_V + s * CF::V_BYTES;
        const uint32_t h_addr = s_base + CF::OFF_H + s * CF::H_BYTES;
        if (!mbar_wait(&bar[B_PREP + s], ph2, ab)) { ok = false; break; }
        if (!mbar_wait(&bar[B_A_EMPTY], (n & 1) ^ 1, ab)) { ok = false; break; }
        tc_fence_after();
        // A = Qs Kg^T: M=64 (query rows), N=64 (key rows), K=128 features.
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t koff = (kk >> 2) * 8192 + (kk & 3) * 32;
          mma_f16(tmem + CF::COL_A, sdesc(q_addr + koff, 16, 1024, kSwizzle128B),
                  sdesc(k_addr + koff, 16, 1024, kSwizzle128B), CF::IDESC_A, kk > 0);
        }
        tc_commit(&bar[B_A_FULL]);
        // S = Kg^T V: M=128 features (MN-major A), N=VS (MN-major B), K=64 tokens.
        if (!mbar_wait(&bar[B_S_EMPTY + s], ph2 ^ 1, ab)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          mma_f16(tmem + CF::COL_S + s * VS, sdesc(k_addr + kk * 2048, 8192, 1024, kSwizzle128B),
                  sdesc(v_addr + kk * 2048, 8192, 1024, kSwizzle128B), CF::IDESC_S, kk > 0);
        }
        tc_commit(&bar[B_S_FULL + s]);
        // O = Qs H_n + P V: M=64, N=VS.
        if (!mbar_wait(&bar[B_P_FULL], n & 1, ab)) { ok = false; break; }
        if (!mbar_wait(&bar[B_H_FULL + s], ph2, ab)) { ok = false; break; }
        if (!mbar_wait(&bar[B_O_EMPTY], (n & 1) ^ 1, ab)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t koff = (kk >> 2) * 8192 + (kk & 3) * 32;
          mma_f16(tmem + CF::COL_O, sdesc(q_addr + koff, 16, 1024, kSwizzle128B),
                  sdesc(h_addr + kk * 2048, 16384, 1024, kSwizzle128B), CF::IDESC_O, kk > 0);
        }
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          mma_f16(tmem + CF::COL_O, sdesc(p_addr + kk * 32, 16, 1024, kSwizzle128B),
                  sdesc(v_addr + kk * 2048, 8192, 1024, kSwizzle128B), CF::IDESC_O, 1);
        }
        tc_commit(&bar[B_O_FULL]);
        tc_commit(&bar[B_QKV_EMPTY + s]);
      }
      tc_commit(&bar[B_DRAIN]);
      const uint64_t t0 = global_ns();
      while (!mbar_try_wait(&bar[B_DRAIN], 0) && global_ns() - t0 < 100000000ull) {
      }
    }
    __syncwarp();
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------------------------ gating + P epilogue
    const int key = (warp - 4) * 32 + lane;             // gating: thread = feature
    const int quad = warp & 3;                          // TMEM lane quadrant
    const int prow = quad * 16 + lane;                  // P row (valid for lane < 16)
    const float* gsm = reinterpret_cast<const float*>(smem + CF::OFF_G);
    const float gamma = p.has_g ? 0.f : __ldg(p.g_gamma + h);
    const float scale = p.scale;
    bool ok = true;
    for (int n = 0; n < NT && ok; ++n) {
      const int s = n & 1;
      const uint32_t ph2 = (n >> 1) & 1;
      if (!mbar_wait(&bar[B_QKV_FULL + s], ph2, ab)) { ok = false; break; }
      if (p.has_g && !mbar_wait(&bar[B_G_FULL], n & 1, ab)) { ok = false; break; }
      if (!mbar_wait(&bar[B_DEC_EMPTY + s], ph2 ^ 1, ab)) { ok = false; break; }
      uint8_t* qs = smem + CF::OFF_Q + s * CF::Q_BYTES;
      uint8_t* ks = smem + CF::OFF_K + s * CF::Q_BYTES;
      float G = 0.f;
#pragma unroll 8
      for (int t = 0; t < C; ++t) {
        G = p.has_g ? G + gsm[t * KD + key] : gamma * static_cast<float>(t + 1);
        const float eg = __expf(G), en = __expf(-G);
        const uint32_t off = kmaj_off(t, key, 8192);
        __nv_bfloat16* qp = reinterpret_cast<__nv_bfloat16*>(qs + off);
        __nv_bfloat16* kp = reinterpret_cast<__nv_bfloat16*>(ks + off);
        *qp = __float2bfloat16_rn(__bfloat162float(*qp) * eg * scale);
        *kp = __float2bfloat16_rn(__bfloat162float(*kp) * en);
      }
      dec[s * KD + key] = __expf(G);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        if (p.has_g) mbar_arrive(&bar[B_G_EMPTY]);
        mbar_arrive(&bar[B_PREP + s]);
        mbar_arrive(&bar[B_DEC_FULL + s]);
      }
      // P = tril(A) in bf16, K-major (row i = query, 128 B per row).
      if (!mbar_wait(&bar[B_A_FULL], n & 1, ab)) { ok = false; break; }
      tc_fence_after();
      uint32_t a[32], a2[32];
      const uint32_t ta = tmem + (static_cast<uint32_t>(quad * 32) << 16) + CF::COL_A;
      tmem_ld32(ta, a);
      tmem_ld32(ta + 32, a2);
      tmem_ld_wait(a);
      tmem_ld_wait(a2);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[B_A_EMPTY]);
      if (lane < 16) {
        uint8_t* pp = smem + CF::OFF_P;
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {
          float f[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int j = c8 * 8 + e;
            const float x = __uint_as_float(j < 32 ? a[j] : a2[j - 32]);
            f[e] = j <= prow ? x : 0.f;
          }
          const uint4 w = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]),
                                     pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
          *reinterpret_cast<uint4*>(pp + prow * 128 + ((c8 ^ (prow & 7)) << 4)) = w;
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[B_P_FULL]);
    }
  } else if (warp >= 8) {
    // ----------------------------------------- state update + O epilogue
    constexpr int HC = VS / 2;                     // state columns per warpgroup
    const int wg = (warp - 8) >> 2;                // 0 / 1 -> columns [wg*HC, (wg+1)*HC)
    const int quad = warp & 3;
    const int key = quad * 32 + lane;              // state row == TMEM lane
    const int c0 = wg * HC;
    const int64_t bhi = static_cast<int64_t>(b) * H + h;
    float hreg[HC];
    if (p.h0) {
      const float4* src =
          reinterpret_cast<const float4*>(p.h0 + (bhi * KD + key) * 128 + v0 + c0);
#pragma unroll
      for (int j = 0; j < HC / 4; ++j) {
        const float4 x = __ldg(src + j);
        hreg[4 * j] = x.x;
        hreg[4 * j + 1] = x.y;
        hreg[4 * j + 2] = x.z;
        hreg[4 * j + 3] = x.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < HC; ++j) hreg[j] = 0.f;
    }
    // H tile: MN-major B operand [128 keys][VS], 64-column atoms 16 KB apart.
    auto store_h = [&](int buf) {
      uint8_t* hp = smem + CF::OFF_H + buf * CF::H_BYTES;
#pragma unroll
      for (int c8 = 0; c8 < HC / 8; ++c8) {
        const int col = c0 + c8 * 8;
        const uint4 w = make_uint4(pack_bf16x2(hreg[c8 * 8], hreg[c8 * 8 + 1]),
                                   pack_bf16x2(hreg[c8 * 8 + 2], hreg[c8 * 8 + 3]),
                                   pack_bf16x2(hreg[c8 * 8 + 4], hreg[c8 * 8 + 5]),
                                   pack_bf16x2(hreg[c8 * 8 + 6], hreg[c8 * 8 + 7]));
        *reinterpret_cast<uint4*>(hp + kmaj_off(key, col, 16384)) = w;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[B_H_FULL + buf]);
    };
    store_h(0);
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    bool ok = true;
    for (int n = 0; n < NT && ok; ++n) {
      const int s = n & 1;
      const uint32_t ph2 = (n >> 1) & 1;
      if (!mbar_wait(&bar[B_DEC_FULL + s], ph2, ab)) { ok = false; break; }
      const float d = dec[s * KD + key];
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[B_DEC_EMPTY + s]);
      if (!mbar_wait(&bar[B_S_FULL + s], ph2, ab)) { ok = false; break; }
      tc_fence_after();
#pragma unroll
      for (int j = 0; j < HC; j += 32) {
        uint32_t sv[32];
        tmem_ld32(lane_addr + CF::COL_S + s * VS + c0 + j, sv);
        tmem_ld_wait(sv);
#pragma unroll
        for (int i = 0; i < 32; ++i) hreg[j + i] = d * (hreg[j + i] + __uint_as_float(sv[i]));
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[B_S_EMPTY + s]);
      if (n + 1 < NT) store_h((n + 1) & 1);
      // O epilogue: rows 16*quad + lane (lane < 16) of the M=64 accumulator.
      if (!mbar_wait(&bar[B_O_FULL], n & 1, ab)) { ok = false; break; }
      tc_fence_after();
      const int64_t row = static_cast<int64_t>(tok0) + n * C + quad * 16 + (lane & 15);
      uint4* dst = reinterpret_cast<uint4*>(p.o + (row * H + h) * 128 + v0 + c0);
#pragma unroll
      for (int j = 0; j < HC; j += 32) {
        uint32_t ov[32];
        tmem_ld32(lane_addr + CF::COL_O + c0 + j, ov);
        tmem_ld_wait(ov);
        if (lane < 16) {
#pragma unroll
          for (int i = 0; i < 4; ++i)
            dst[j / 8 + i] = make_uint4(
                pack_bf16x2(__uint_as_float(ov[8 * i]), __uint_as_float(ov[8 * i + 1])),
                pack_bf16x2(__uint_as_float(ov[8 * i + 2]), __uint_as_float(ov[8 * i + 3])),
                pack_bf16x2(__uint_as_float(ov[8 * i + 4]), __uint_as_float(ov[8 * i + 5])),
                pack_bf16x2(__uint_as_float(ov[8 * i + 6]), __uint_as_float(ov[8 * i + 7])));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[B_O_EMPTY]);
    }
    if (ok && p.ht) {
      float4* dst = reinterpret_cast<float4*>(p.ht + (bhi * KD + key) * 128 + v0 + c0);
#pragma unroll
      for (int j = 0; j < HC / 4; ++j)
        dst[j] = make_float4(hreg[4 * j], hreg[4 * j + 1], hreg[4 * j + 2], hreg[4 * j + 3]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, CF::TMEM_COLS);
  }
}

}  // namespace gla
}  // namespace gl

#include "tmap.h"

template <int VS>
static int launch_vs(const void* q, const void* k, const void* v, const float* g,
                     const gl::gla::Params& p, cudaStream_t st, const char** why) {
  using CF = gl::gla::Cfg<VS>;
  const int64_t BT = static_cast<int64_t>(p.B) * p.T;
  CUtensorMap tq, tk, tv, tg;
  if (!gl_make_tmap_3d(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, q, 128, p.H, BT, 128,
                       static_cast<int64_t>(p.H) * 128, 64, 1, 64, CU_TENSOR_MAP_SWIZZLE_128B, why))
    return -1;
  if (!gl_make_tmap_3d(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, k, 128, p.H, BT, 128,
                       static_cast<int64_t>(p.H) * 128, 64, 1, 64, CU_TENSOR_MAP_SWIZZLE_128B, why))
    return -1;
  if (!gl_make_tmap_3d(&tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, v, 128, p.H, BT, 128,
                       static_cast<int64_t>(p.H) * 128, 64, 1, 64, CU_TENSOR_MAP_SWIZZLE_128B, why))
    return -1;
  if (g) {
    if (!gl_make_tmap_3d(&tg, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, g, 128, p.H, BT, 128,
                         static_cast<int64_t>(p.H) * 128, 128, 1, 64, CU_TENSOR_MAP_SWIZZLE_NONE,
                         why))
      return -1;
  } else {
    tg = tq;  // unused when the per-head gate is given
  }
  if (!gl_set_smem_attr(reinterpret_cast<const void*>(gl::gla::chunk_gla_fwd_kernel<VS>), 0,
                        static_cast<int>(CF::SMEM_BYTES), why))
    return -2;
  const int grid = p.B * p.H * p.nsplit;
  gl::gla::chunk_gla_fwd_kernel<VS><<<grid, gl::gla::NUM_THREADS, CF::SMEM_BYTES, st>>>(tq, tk, tv, tg, p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    *why = cudaGetErrorString(e);
    return -2;
  }
  return 0;
}

int gl_launch_chunk_gla(const void* q, const void* k, const void* v, const float* g,
                        const float* g_gamma, const float* h0, float scale, int64_t B, int64_t T,
                        int64_t H, int64_t K, int64_t V, void* o, float* ht, int* err,
                        cudaStream_t st, int num_sms, const char** why) {
  (void)K;
  (void)V;
  gl::gla::Params p;
  p.g_gamma = g_gamma;
  p.h0 = h0;
  p.o = static_cast<__nv_bfloat16*>(o);
  p.ht = ht;
  p.err = err;
  p.scale = scale;
  p.B = static_cast<int>(B);
  p.T = static_cast<int>(T);
  p.H = static_cast<int>(H);
  p.has_g = g != nullptr;
  // Split V in two when that is needed to give every SM a sequence.
  if (B * H * 2 <= num_sms) {
    p.nsplit = 2;
    return launch_vs<64>(q, k, v, g, p, st, why);
  }
  p.nsplit = 1;
  return launch_vs<128>(q, k, v, g, p, st, why);
}
