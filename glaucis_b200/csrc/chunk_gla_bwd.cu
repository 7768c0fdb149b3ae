// Chunk-parallel gradients of the chunked GLA forward (sm_100a): dq, dk, dv of
// every 64-token chunk from the forward's per-chunk state h_n and the reverse
// scan's E_n = e^{G_last(n)} dL/dh_{n+1} (both bf16 [B,NT,H,K,V]).
//
// Replaces the fused dq/dk/dv pallas_call of the Glaucis template's backward
// (KE/examples/kernels/chunk_gla.py:313-426, launched at :429-468 after the
// reverse dh scan :281-305; pure-jnp form chunk_gla_ref.py:146-199), with the
// per-key gate of the forward as well as the per-head g_gamma.
//
// Per chunk (G = chunk-local cumsum of the log-gate, Qs = scale q e^G,
// Kg = k e^-G, both bf16 in place):
//   A  = Qs Kg^T,  dA = do v^T                  M=64 N=64  K=128   (TMEM)
//   P  = tril(A), dP = tril(dA)                 bf16, shared memory
//   dq = scale e^G  * (do h_n^T + dP Kg)        M=64 N=128 K=128+64
//   dk = e^-G       * (dP^T Qs + v E_n^T)       M=64 N=128 K=64+128
//   dv = P^T do + Kg E_n                        M=64 N=128 K=64+128
// which is the reference's dq_intra + dq_inter, dk_intra + dk_inter and
// dv_intra + dv_inter with the decays e^{G_last - G} split into e^{G_last}
// (inside E_n) and e^-G (inside Kg or the epilogue).
//
// Persistent CTAs, one per SM, walk the (batch, chunk, head) items.  512
// threads:
//   warp 0        TMA producer: q, k (two stages), h_n, v, do, E_n of each item
//   warp 1        tcgen05.mma issuer
//   warp 2        TMEM allocator (512 columns: A, dA, dq, dk, dv)
//   warps 4-11    gating of item i (warp = 8 tokens, lane = 4 keys; the raw
//                 gate read from global memory one item ahead), then the dq
//                 epilogue of item i-1, then item i's epilogue factors
//                 scale e^G and e^-G (bf16, computed by the gating anyway) into
//                 shared memory
//   warps 12-15   dv and dk epilogues of item i-1, then P, dP of item i
// q and k have two stages, so the next item's gating and A = Qs Kg^T overlap
// the current item's MMAs; the other buffers are single and are handed to
// the next item by their last reader.
#include "common.cuh"

namespace gl {
namespace glab {

constexpr int C = 64, KD = 128, NUM_THREADS = 512;
constexpr int GATE_WARPS = 8, P_WARPS = 4;
// Register split (launch: 512 x 128): the gating warps hold the next item's
// raw gate and this item's factors across the dq epilogue.
constexpr int REG_CTRL = 104, REG_GATE = 160, REG_P = 88;
static_assert(128 * REG_CTRL + 256 * REG_GATE + 128 * REG_P <= NUM_THREADS * 128,
              "register split exceeds the launch allocation");
constexpr uint32_t T_BYTES = C * KD * 2;   // 16 KB: [64 tokens][128] bf16 (2 boxes of 64 columns)
constexpr uint32_t S_BYTES = KD * KD * 2;  // 32 KB: [128 keys][128] bf16 (2 boxes of 64 columns)
constexpr uint32_t PP_BYTES = C * C * 2;   // 8 KB: P or dP [64][64] bf16
constexpr uint32_t FAC_PITCH = KD * 2 + 16;  // padded bf16 row of an epilogue factor table
constexpr uint32_t OFF_Q = 0;                       // [2 stages]
constexpr uint32_t OFF_K = OFF_Q + 2 * T_BYTES;     // [2 stages]
constexpr uint32_t OFF_V = OFF_K + 2 * T_BYTES;
constexpr uint32_t OFF_DO = OFF_V + T_BYTES;
constexpr uint32_t OFF_H = OFF_DO + T_BYTES;
constexpr uint32_t OFF_E = OFF_H + S_BYTES;
constexpr uint32_t OFF_P = OFF_E + S_BYTES;
constexpr uint32_t OFF_DP = OFF_P + PP_BYTES;
constexpr uint32_t OFF_FQ = OFF_DP + PP_BYTES;         // [64][128] bf16 scale e^G (dq factor)
constexpr uint32_t OFF_FK = OFF_FQ + C * FAC_PITCH;    // [64][128] bf16 e^-G (dk factor)
// per-warp gate sums [2 items][8 warps][32 lanes] float4: double-buffered
// because the next item's gating may start before a slow warp has read them
constexpr uint32_t OFF_PART = OFF_FK + C * FAC_PITCH;
constexpr uint32_t OFF_BAR = OFF_PART + 2 * GATE_WARPS * 32 * 16;
constexpr uint32_t OFF_MISC = OFF_BAR + 256;
constexpr uint32_t SMEM_BYTES = OFF_MISC + 64 + 1024;
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
static_assert(OFF_H % 1024 == 0 && OFF_P % 1024 == 0 && OFF_DP % 1024 == 0, "tile alignment");

// TMEM columns.
constexpr uint32_t COL_A = 0, COL_DA = 64, COL_DQ = 128, COL_DK = 256, COL_DV = 384;
constexpr uint32_t TMEM_COLS = 512;

// Instruction descriptors (bf16 x bf16 -> f32; a_mn / b_mn = MN-major operand).
constexpr uint32_t ID_KK64 = idesc(1, 1, 1, 0, 0, 64, 64);    // A, dA
constexpr uint32_t ID_KK128 = idesc(1, 1, 1, 0, 0, 64, 128);  // do h^T, v E^T
constexpr uint32_t ID_KM128 = idesc(1, 1, 1, 0, 1, 64, 128);  // dP Kg, Kg E
constexpr uint32_t ID_MM128 = idesc(1, 1, 1, 1, 1, 64, 128);  // dP^T Qs, P^T do

struct Params {
  const float* g;        // [B,T,H,K] raw per-key gate or null
  const float* g_gamma;  // [H] or null
  __nv_bfloat16* dq;     // [B,T,H,K]
  __nv_bfloat16* dk;     // [B,T,H,K]
  __nv_bfloat16* dv;     // [B,T,H,V]
  int* err;
  float scale;
  float log2_scale;  // log2(scale) when scale > 0 (folded into the exponent), else 0
  int scale_apart;   // 1: scale <= 0 or not finite, applied as a separate multiply
  int H, items;
};

enum {
  B_QK_FULL = 0,  // [2] q, k of the stage landed
  B_QK_EMPTY = 2,  // [2] last MMA reading the stage done
  B_VD_FULL = 4,   // v, do landed
  B_VD_EMPTY,      // last MMA reading them done
  B_H_FULL,        // h_n landed
  B_H_EMPTY,       // do h^T done
  B_E_FULL,        // E_n landed
  B_E_EMPTY,       // v E^T and Kg E done
  B_PREP,          // Qs, Kg written (8 warps)
  B_GSYNC,         // per-warp gate sums written (8 warps)
  B_GC_EMPTY,      // previous item's dq and dk epilogues done with the factor tables (8 + 4 warps)
  B_GC_FULL,       // factor tables of the item written (8 warps)
  B_AD_FULL,       // A, dA committed
  B_AD_EMPTY,      // A, dA read (4 warps)
  B_P_FULL,        // P, dP written (4 warps)
  B_P_EMPTY,       // dP Kg, dP^T Qs, P^T do done
  B_DQ_FULL,
  B_DQ_EMPTY,  // 8 warps
  B_DK_FULL,
  B_DK_EMPTY,  // 4 warps
  B_DV_FULL,
  B_DV_EMPTY,  // 4 warps
  B_DRAIN,
  NUM_BARS
};
static_assert(NUM_BARS * 8 <= 256, "barrier area");

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float2 bf16x2_f32x2(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    chunk_gla_bwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                         const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v,
                         const __grid_constant__ CUtensorMap tm_do,
                         const __grid_constant__ CUtensorMap tm_h,
                         const __grid_constant__ CUtensorMap tm_e, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + OFF_MISC);
  int* abort_flag = reinterpret_cast<int*>(smem + OFF_MISC + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = p.H;
  const bool has_g = p.g != nullptr;
  const int first = blockIdx.x, stride = gridDim.x;
  const int nit = first < p.items ? (p.items - 1 - first) / stride + 1 : 0;
  // Item m of this CTA: head and global chunk (b NT + chunk).
  auto item_head = [&](int m) { return (first + m * stride) % H; };
  auto item_chunk = [&](int m) { return (first + m * stride) / H; };
  const Abort ab{abort_flag, p.err};

  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
    prefetch_tmap(&tm_do);
    prefetch_tmap(&tm_h);
    prefetch_tmap(&tm_e);
  } else if (warp == 1 && lane == 0) {
    const uint8_t counts[NUM_BARS] = {1, 1, 1, 1, 1, 1, 1, 1, 1, 1,
                                      GATE_WARPS, GATE_WARPS, GATE_WARPS + P_WARPS, GATE_WARPS,
                                      1, P_WARPS, P_WARPS, 1, 1, GATE_WARPS, 1, P_WARPS,
                                      1, P_WARPS, 1};
    for (int i = 0; i < NUM_BARS; ++i) mbar_init(&bar[i], counts[i]);
    *abort_flag = 0;
    fence_mbar_init();
  } else if (warp == 2) {
    tmem_alloc(tmem_holder, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const uint32_t s_base = smem_u32(smem);

  if (warp == 0) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_CTRL));
    // ------------------------------------------------------------- TMA
    if (lane == 0) {
      for (int i = 0; i < nit; ++i) {
        const uint32_t ph = i & 1;
        const int s = i & 1;
        const int h = item_head(i), cg = item_chunk(i);
        const int tok = cg * C;
        const int32_t srow = (cg * H + h) * KD;
        if (!mbar_wait(&bar[B_QK_EMPTY + s], ((i >> 1) & 1) ^ 1, ab)) break;
        mbar_arrive_expect_tx(&bar[B_QK_FULL + s], 2 * T_BYTES);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          tma_load_3d(smem + OFF_Q + s * T_BYTES + j * 8192, &tm_q, &bar[B_QK_FULL + s], 64 * j, h, tok);
          tma_load_3d(smem + OFF_K + s * T_BYTES + j * 8192, &tm_k, &bar[B_QK_FULL + s], 64 * j, h, tok);
        }
        if (!mbar_wait(&bar[B_H_EMPTY], ph ^ 1, ab)) break;
        mbar_arrive_expect_tx(&bar[B_H_FULL], S_BYTES);
        tma_load_2d(smem + OFF_H, &tm_h, &bar[B_H_FULL], 0, srow);
        tma_load_2d(smem + OFF_H + 16384, &tm_h, &bar[B_H_FULL], 64, srow);
        if (!mbar_wait(&bar[B_VD_EMPTY], ph ^ 1, ab)) break;
        mbar_arrive_expect_tx(&bar[B_VD_FULL], 2 * T_BYTES);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          tma_load_3d(smem + OFF_V + j * 8192, &tm_v, &bar[B_VD_FULL], 64 * j, h, tok);
          tma_load_3d(smem + OFF_DO + j * 8192, &tm_do, &bar[B_VD_FULL], 64 * j, h, tok);
        }
        if (!mbar_wait(&bar[B_E_EMPTY], ph ^ 1, ab)) break;
        mbar_arrive_expect_tx(&bar[B_E_FULL], S_BYTES);
        tma_load_2d(smem + OFF_E, &tm_e, &bar[B_E_FULL], 0, srow);
        tma_load_2d(smem + OFF_E + 16384, &tm_e, &bar[B_E_FULL], 64, srow);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_CTRL));
    // ------------------------------------------------------------- MMA
    if (lane == 0) {
      const uint32_t v_a = s_base + OFF_V, do_a = s_base + OFF_DO;
      const uint32_t h_a = s_base + OFF_H, e_a = s_base + OFF_E;
      const uint32_t p_a = s_base + OFF_P, dp_a = s_base + OFF_DP;
      // K-major [rows][128] tiles: 64-column atoms 8 KB (64 rows) or 16 KB
      // (128 rows) apart, 16 columns = 32 bytes per K step.
      auto k8 = [](int kk) { return static_cast<uint32_t>((kk >> 2) * 8192 + (kk & 3) * 32); };
      auto k16 = [](int kk) { return static_cast<uint32_t>((kk >> 2) * 16384 + (kk & 3) * 32); };
      for (int i = 0; i < nit; ++i) {
        const uint32_t ph = i & 1;
        const int s = i & 1;
        const uint32_t q_a = s_base + OFF_Q + s * T_BYTES, k_a = s_base + OFF_K + s * T_BYTES;
        if (!mbar_wait(&bar[B_PREP], ph, ab) || !mbar_wait(&bar[B_QK_FULL + s], (i >> 1) & 1, ab) ||
            !mbar_wait(&bar[B_AD_EMPTY], ph ^ 1, ab))
          break;
        tc_fence_after();
        // A = Qs Kg^T (K = 128 features)
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          mma_f16(tmem + COL_A, sdesc(q_a + k8(kk), 16, 1024, kSwizzle128B),
                  sdesc(k_a + k8(kk), 16, 1024, kSwizzle128B), ID_KK64, kk > 0);
        // dA = do v^T (K = 128 value columns)
        if (!mbar_wait(&bar[B_VD_FULL], ph, ab)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          mma_f16(tmem + COL_DA, sdesc(do_a + k8(kk), 16, 1024, kSwizzle128B),
                  sdesc(v_a + k8(kk), 16, 1024, kSwizzle128B), ID_KK64, kk > 0);
        tc_commit(&bar[B_AD_FULL]);
        // dq = do h^T (K = 128 value columns)
        if (!mbar_wait(&bar[B_H_FULL], ph, ab) || !mbar_wait(&bar[B_DQ_EMPTY], ph ^ 1, ab)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          mma_f16(tmem + COL_DQ, sdesc(do_a + k8(kk), 16, 1024, kSwizzle128B),
                  sdesc(h_a + k16(kk), 16, 1024, kSwizzle128B), ID_KK128, kk > 0);
        tc_commit(&bar[B_H_EMPTY]);
        // dq += dP Kg; dk = dP^T Qs; dv = P^T do (K = 64 tokens)
        if (!mbar_wait(&bar[B_P_FULL], ph, ab)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_f16(tmem + COL_DQ, sdesc(dp_a + kk * 32, 16, 1024, kSwizzle128B),
                  sdesc(k_a + kk * 2048, 8192, 1024, kSwizzle128B), ID_KM128, 1);
        tc_commit(&bar[B_DQ_FULL]);
        if (!mbar_wait(&bar[B_DK_EMPTY], ph ^ 1, ab)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_f16(tmem + COL_DK, sdesc(dp_a + kk * 2048, 8192, 1024, kSwizzle128B),
                  sdesc(q_a + kk * 2048, 8192, 1024, kSwizzle128B), ID_MM128, kk > 0);
        if (!mbar_wait(&bar[B_DV_EMPTY], ph ^ 1, ab)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_f16(tmem + COL_DV, sdesc(p_a + kk * 2048, 8192, 1024, kSwizzle128B),
                  sdesc(do_a + kk * 2048, 8192, 1024, kSwizzle128B), ID_MM128, kk > 0);
        tc_commit(&bar[B_P_EMPTY]);
        // dk += v E^T (K = 128 value columns); dv += Kg E (K = 128 keys)
        if (!mbar_wait(&bar[B_E_FULL], ph, ab)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          mma_f16(tmem + COL_DK, sdesc(v_a + k8(kk), 16, 1024, kSwizzle128B),
                  sdesc(e_a + k16(kk), 16, 1024, kSwizzle128B), ID_KK128, 1);
        tc_commit(&bar[B_DK_FULL]);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          mma_f16(tmem + COL_DV, sdesc(k_a + k8(kk), 16, 1024, kSwizzle128B),
                  sdesc(e_a + kk * 2048, 16384, 1024, kSwizzle128B), ID_KM128, 1);
        tc_commit(&bar[B_DV_FULL]);
        tc_commit(&bar[B_QK_EMPTY + s]);
        tc_commit(&bar[B_VD_EMPTY]);
        tc_commit(&bar[B_E_EMPTY]);
      }
      tc_commit(&bar[B_DRAIN]);
      const uint64_t td = global_ns();
      while (!mbar_try_wait(&bar[B_DRAIN], 0) && global_ns() - td < 100000000ull) {
      }
    }
    __syncwarp();
  } else if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_CTRL));
  } else if (warp < 4 + GATE_WARPS) {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REG_GATE));
    // ------------------------------------------- gating, dq epilogue
    const int gw = warp - 4;
    constexpr float kLog2e = 1.4426950408889634f;
    const float log2_scale = p.log2_scale;
    // Epilogue: TMEM lane quadrant warp%4 holds rows 16*quad .. +15 of the
    // M=64 accumulators (TMEM lanes 0-15 of the quadrant); this warp takes
    // columns 64*half .. +63.
    const int quad = warp & 3, half = gw >> 2;
    const int erow = quad * 16 + (lane & 15);
    const uint32_t e_lane = tmem + (static_cast<uint32_t>(quad * 32) << 16) + COL_DQ + half * 64;
    const uint8_t* fq_row = smem + OFF_FQ + erow * FAC_PITCH + half * 128;
    auto dq_epilogue = [&](int m) -> bool {
      const uint32_t ph = m & 1;
      const int h = item_head(m);
      const int64_t row = static_cast<int64_t>(item_chunk(m)) * C + erow;
      // per-head gate: one factor per row, scale e^{gamma (t+1)}
      const float fr = has_g ? 1.f
                             : ex2_approx(fmaf(__ldg(p.g_gamma + h) * static_cast<float>(erow + 1), kLog2e,
                                               log2_scale)) * (p.scale_apart ? p.scale : 1.f);
      if (has_g && !mbar_wait(&bar[B_GC_FULL], ph, ab)) return false;
      if (!mbar_wait(&bar[B_DQ_FULL], ph, ab)) return false;
      tc_fence_after();
      uint4* dst = reinterpret_cast<uint4*>(p.dq + (row * H + h) * KD + half * 64);
#pragma unroll
      for (int j = 0; j < 64; j += 32) {
        uint32_t x[32];
        tmem_ld32(e_lane + j, x);
        tmem_ld_wait(x);
        if (lane < 16) {
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8) {
            uint32_t w[4];
            if (has_g) {
              const uint4 f = *reinterpret_cast<const uint4*>(fq_row + (j + 8 * c8) * 2);
              const uint32_t fw[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 y = __fmul2_rn(make_float2(__uint_as_float(x[8 * c8 + 2 * e]),
                                                        __uint_as_float(x[8 * c8 + 2 * e + 1])),
                                            bf16x2_f32x2(fw[e]));
                w[e] = pack_bf16x2(y.x, y.y);
              }
            } else {
#pragma unroll
              for (int e = 0; e < 4; ++e)
                w[e] = pack_bf16x2(__uint_as_float(x[8 * c8 + 2 * e]) * fr,
                                   __uint_as_float(x[8 * c8 + 2 * e + 1]) * fr);
            }
            dst[j / 8 + c8] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&bar[B_DQ_EMPTY]);
        if (has_g) mbar_arrive(&bar[B_GC_EMPTY]);
      }
      return true;
    };
    // Gating: warp gw takes tokens 8 gw .. 8 gw + 7, lane l keys 4 l .. 4 l + 3.
    const uint32_t qk_atom = static_cast<uint32_t>(lane >> 4) * 8192u;
    const uint32_t qk_chunk = static_cast<uint32_t>(lane & 15) >> 1, qk_sub = (lane & 1) * 8u;
    float4 gnext[8];  // raw gate of the next item, loaded one item ahead
    auto load_gate = [&](int m) {
      const float4* src = reinterpret_cast<const float4*>(
          p.g + (static_cast<int64_t>(item_chunk(m)) * C + gw * 8) * H * KD +
          static_cast<int64_t>(item_head(m)) * KD) + lane;
#pragma unroll
      for (int t = 0; t < 8; ++t) gnext[t] = __ldg(src + static_cast<int64_t>(t) * H * (KD / 4));
    };
    if (has_g && nit > 0) load_gate(0);
    bool ok = true;
    for (int i = 0; i < nit && ok; ++i) {
      const int s = i & 1;
      if (!mbar_wait(&bar[B_QK_FULL + s], (i >> 1) & 1, ab)) { ok = false; break; }
      float4 gv[8];
      float4 G = make_float4(0.f, 0.f, 0.f, 0.f);
      if (has_g) {
#pragma unroll
        for (int t = 0; t < 8; ++t) gv[t] = gnext[t];
        if (i + 1 < nit) load_gate(i + 1);
        float4 tot = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          tot.x += gv[t].x;
          tot.y += gv[t].y;
          tot.z += gv[t].z;
          tot.w += gv[t].w;
        }
        float4* part = reinterpret_cast<float4*>(smem + OFF_PART) + (i & 1) * (GATE_WARPS * 32);
        part[gw * 32 + lane] = tot;
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar[B_GSYNC]);
        if (!mbar_wait(&bar[B_GSYNC], i & 1, ab)) { ok = false; break; }
        for (int w = 0; w < gw; ++w) {
          const float4 pv = part[w * 32 + lane];
          G.x += pv.x;
          G.y += pv.y;
          G.z += pv.z;
          G.w += pv.w;
        }
      }
      const float gam = has_g ? 0.f : __ldg(p.g_gamma + item_head(i));
      uint8_t* qs = smem + OFF_Q + s * T_BYTES + qk_atom + qk_sub;
      uint8_t* ks = smem + OFF_K + s * T_BYTES + qk_atom + qk_sub;
      const float2 L2 = make_float2(kLog2e, kLog2e), NL2 = make_float2(-kLog2e, -kLog2e);
      const float2 LS2 = make_float2(log2_scale, log2_scale);
      const float2 SA2 = p.scale_apart ? make_float2(p.scale, p.scale) : make_float2(1.f, 1.f);
      float2 G01 = make_float2(G.x, G.y), G23 = make_float2(G.z, G.w);
      uint2 fa[8], fb[8];  // this item's epilogue factors (bf16 pairs), written after the epilogue
#pragma unroll
      for (int t8 = 0; t8 < 8; ++t8) {
        const int t = gw * 8 + t8;
        float2 xa01, xa23, xb01, xb23;
        if (has_g) {
          G01 = __fadd2_rn(G01, make_float2(gv[t8].x, gv[t8].y));
          G23 = __fadd2_rn(G23, make_float2(gv[t8].z, gv[t8].w));
          xa01 = __ffma2_rn(G01, L2, LS2);
          xa23 = __ffma2_rn(G23, L2, LS2);
          xb01 = __fmul2_rn(G01, NL2);
          xb23 = __fmul2_rn(G23, NL2);
        } else {
          const float Gt = gam * static_cast<float>(t + 1);
          xa01 = xa23 = make_float2(fmaf(Gt, kLog2e, log2_scale), fmaf(Gt, kLog2e, log2_scale));
          xb01 = xb23 = make_float2(-Gt * kLog2e, -Gt * kLog2e);
        }
        const uint32_t off = static_cast<uint32_t>(t) * 128u + ((qk_chunk ^ (t & 7)) << 4);
        // a = scale e^G (q's and dq's factor), b = e^-G (k's and dk's factor)
        const float2 a01 = __fmul2_rn(make_float2(ex2_approx(xa01.x), ex2_approx(xa01.y)), SA2);
        const float2 a23 = __fmul2_rn(make_float2(ex2_approx(xa23.x), ex2_approx(xa23.y)), SA2);
        const float2 b01 = make_float2(ex2_approx(xb01.x), ex2_approx(xb01.y));
        const float2 b23 = make_float2(ex2_approx(xb23.x), ex2_approx(xb23.y));
        fa[t8] = make_uint2(pack_bf16x2(a01.x, a01.y), pack_bf16x2(a23.x, a23.y));
        fb[t8] = make_uint2(pack_bf16x2(b01.x, b01.y), pack_bf16x2(b23.x, b23.y));
        const uint2 q2 = *reinterpret_cast<const uint2*>(qs + off);
        const float2 q01 = __fmul2_rn(bf16x2_f32x2(q2.x), a01), q23 = __fmul2_rn(bf16x2_f32x2(q2.y), a23);
        *reinterpret_cast<uint2*>(qs + off) = make_uint2(pack_bf16x2(q01.x, q01.y), pack_bf16x2(q23.x, q23.y));
        const uint2 k2 = *reinterpret_cast<const uint2*>(ks + off);
        const float2 k01 = __fmul2_rn(bf16x2_f32x2(k2.x), b01), k23 = __fmul2_rn(bf16x2_f32x2(k2.y), b23);
        *reinterpret_cast<uint2*>(ks + off) = make_uint2(pack_bf16x2(k01.x, k01.y), pack_bf16x2(k23.x, k23.y));
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[B_PREP]);
      // the previous item's dq epilogue, then this item's factor tables once
      // both epilogues of the previous item are done with them
      if (i > 0 && !dq_epilogue(i - 1)) { ok = false; break; }
      if (has_g) {
        if (i > 0 && !mbar_wait(&bar[B_GC_EMPTY], (i - 1) & 1, ab)) { ok = false; break; }
#pragma unroll
        for (int t8 = 0; t8 < 8; ++t8) {
          const uint32_t ro = (gw * 8 + t8) * FAC_PITCH + 8 * lane;
          *reinterpret_cast<uint2*>(smem + OFF_FQ + ro) = fa[t8];
          *reinterpret_cast<uint2*>(smem + OFF_FK + ro) = fb[t8];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar[B_GC_FULL]);
      }
    }
    if (ok && nit > 0) dq_epilogue(nit - 1);
  } else {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_P));
    // --------------------------------------------- dv and dk epilogues, P and dP
    const int quad = warp & 3;
    const int prow = quad * 16 + (lane & 15);
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    auto dv_epilogue = [&](int m) -> bool {
      if (!mbar_wait(&bar[B_DV_FULL], m & 1, ab)) return false;
      tc_fence_after();
      const int h = item_head(m);
      const int64_t row = static_cast<int64_t>(item_chunk(m)) * C + prow;
      uint4* dst = reinterpret_cast<uint4*>(p.dv + (row * H + h) * KD);
#pragma unroll
      for (int j = 0; j < 128; j += 64) {
        uint32_t x0[32], x1[32];
        tmem_ld32(lane_addr + COL_DV + j, x0);
        tmem_ld32(lane_addr + COL_DV + j + 32, x1);
        tmem_ld_wait2(x0, x1);
        if (lane < 16) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            dst[j / 8 + i] = make_uint4(
                pack_bf16x2(__uint_as_float(x0[8 * i]), __uint_as_float(x0[8 * i + 1])),
                pack_bf16x2(__uint_as_float(x0[8 * i + 2]), __uint_as_float(x0[8 * i + 3])),
                pack_bf16x2(__uint_as_float(x0[8 * i + 4]), __uint_as_float(x0[8 * i + 5])),
                pack_bf16x2(__uint_as_float(x0[8 * i + 6]), __uint_as_float(x0[8 * i + 7])));
            dst[j / 8 + 4 + i] = make_uint4(
                pack_bf16x2(__uint_as_float(x1[8 * i]), __uint_as_float(x1[8 * i + 1])),
                pack_bf16x2(__uint_as_float(x1[8 * i + 2]), __uint_as_float(x1[8 * i + 3])),
                pack_bf16x2(__uint_as_float(x1[8 * i + 4]), __uint_as_float(x1[8 * i + 5])),
                pack_bf16x2(__uint_as_float(x1[8 * i + 6]), __uint_as_float(x1[8 * i + 7])));
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[B_DV_EMPTY]);
      return true;
    };
    // dk = e^-G (dP^T Qs + v E^T): this warp's 16 rows, all 128 columns.
    const uint8_t* fk_row = smem + OFF_FK + prow * FAC_PITCH;
    auto dk_epilogue = [&](int m) -> bool {
      const uint32_t ph = m & 1;
      const int h = item_head(m);
      const int64_t row = static_cast<int64_t>(item_chunk(m)) * C + prow;
      const float fr = has_g ? 1.f
                             : ex2_approx(-__ldg(p.g_gamma + h) * static_cast<float>(prow + 1) *
                                          1.4426950408889634f);
      if (has_g && !mbar_wait(&bar[B_GC_FULL], ph, ab)) return false;
      if (!mbar_wait(&bar[B_DK_FULL], ph, ab)) return false;
      tc_fence_after();
      uint4* dst = reinterpret_cast<uint4*>(p.dk + (row * H + h) * KD);
#pragma unroll
      for (int j = 0; j < 128; j += 32) {
        uint32_t x[32];
        tmem_ld32(lane_addr + COL_DK + j, x);
        tmem_ld_wait(x);
        if (lane < 16) {
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8) {
            uint32_t w[4];
            if (has_g) {
              const uint4 f = *reinterpret_cast<const uint4*>(fk_row + (j + 8 * c8) * 2);
              const uint32_t fw[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 y = __fmul2_rn(make_float2(__uint_as_float(x[8 * c8 + 2 * e]),
                                                        __uint_as_float(x[8 * c8 + 2 * e + 1])),
                                            bf16x2_f32x2(fw[e]));
                w[e] = pack_bf16x2(y.x, y.y);
              }
            } else {
#pragma unroll
              for (int e = 0; e < 4; ++e)
                w[e] = pack_bf16x2(__uint_as_float(x[8 * c8 + 2 * e]) * fr,
                                   __uint_as_float(x[8 * c8 + 2 * e + 1]) * fr);
            }
            dst[j / 8 + c8] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&bar[B_DK_EMPTY]);
        if (has_g) mbar_arrive(&bar[B_GC_EMPTY]);
      }
      return true;
    };
    // P = tril(A), dP = tril(dA), bf16 K-major rows of 128 B (row = query).
    auto p_epilogue = [&](int i) -> bool {
      const uint32_t ph = i & 1;
      if (!mbar_wait(&bar[B_AD_FULL], ph, ab) || !mbar_wait(&bar[B_P_EMPTY], ph ^ 1, ab)) return false;
      tc_fence_after();
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        uint32_t a[32], d[32];
        tmem_ld32(lane_addr + COL_A + hh * 32, a);
        tmem_ld32(lane_addr + COL_DA + hh * 32, d);
        tmem_ld_wait2(a, d);
        if (hh == 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bar[B_AD_EMPTY]);
        }
        if (lane < 16) {
          uint8_t* pp = smem + OFF_P + prow * 128;
          uint8_t* dpp = smem + OFF_DP + prow * 128;
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4) {
            float f[8], g[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const int j = hh * 32 + c4 * 8 + e;
              f[e] = j <= prow ? __uint_as_float(a[c4 * 8 + e]) : 0.f;
              g[e] = j <= prow ? __uint_as_float(d[c4 * 8 + e]) : 0.f;
            }
            const uint32_t ch = (static_cast<uint32_t>(hh * 4 + c4) ^ (prow & 7)) << 4;
            *reinterpret_cast<uint4*>(pp + ch) = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]),
                                                            pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
            *reinterpret_cast<uint4*>(dpp + ch) = make_uint4(pack_bf16x2(g[0], g[1]), pack_bf16x2(g[2], g[3]),
                                                             pack_bf16x2(g[4], g[5]), pack_bf16x2(g[6], g[7]));
          }
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[B_P_FULL]);
      return true;
    };
    bool ok = true;
    for (int i = 0; i < nit && ok; ++i) {
      if (i > 0 && !(dv_epilogue(i - 1) && dk_epilogue(i - 1))) break;
      ok = p_epilogue(i);
    }
    if (ok && nit > 0 && dv_epilogue(nit - 1)) dk_epilogue(nit - 1);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace glab
}  // namespace gl

#include <cmath>

#include "tmap.h"

// Gradient pass of the backward: dq, dk, dv (bf16) from q, k, v, do, the
// gate, the forward's per-chunk states h and the reverse scan's E.
int gl_launch_chunk_gla_grads(const void* q, const void* k, const void* v, const void* dout,
                              const float* g, const float* g_gamma, const void* h, const void* e,
                              float scale, int64_t B, int64_t T, int64_t H, void* dq, void* dk,
                              void* dv, int* err, cudaStream_t st, int num_sms, const char** why) {
  using namespace gl::glab;
  const int64_t BT = B * T;
  const int64_t srows = BT / C * H * KD;
  CUtensorMap tq, tk, tv, tdo, th, te;
  const void* tiles[4] = {q, k, v, dout};
  CUtensorMap* maps[4] = {&tq, &tk, &tv, &tdo};
  for (int i = 0; i < 4; ++i)
    if (!gl_make_tmap_3d(maps[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, tiles[i], 128, H, BT, 128, H * 128,
                         64, 1, 64, CU_TENSOR_MAP_SWIZZLE_128B, why))
      return -1;
  if (!gl_make_tmap_2d(&th, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, h, 128, srows, 128, 64, 128,
                       CU_TENSOR_MAP_SWIZZLE_128B, why) ||
      !gl_make_tmap_2d(&te, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, e, 128, srows, 128, 64, 128,
                       CU_TENSOR_MAP_SWIZZLE_128B, why))
    return -1;
  Params p;
  p.g = g;
  p.g_gamma = g_gamma;
  p.dq = static_cast<__nv_bfloat16*>(dq);
  p.dk = static_cast<__nv_bfloat16*>(dk);
  p.dv = static_cast<__nv_bfloat16*>(dv);
  p.err = err;
  p.scale = scale;
  p.scale_apart = !(scale > 0.f && std::isfinite(scale));
  p.log2_scale = p.scale_apart ? 0.f : static_cast<float>(std::log2(static_cast<double>(scale)));
  p.H = static_cast<int>(H);
  p.items = static_cast<int>(BT / C * H);
  if (!gl_set_smem_attr(reinterpret_cast<const void*>(chunk_gla_bwd_kernel), 0,
                        static_cast<int>(SMEM_BYTES), why))
    return -2;
  const int grid = p.items < num_sms ? p.items : num_sms;
  chunk_gla_bwd_kernel<<<grid, NUM_THREADS, SMEM_BYTES, st>>>(tq, tk, tv, tdo, th, te, p);
  const cudaError_t ce = cudaGetLastError();
  if (ce != cudaSuccess) {
    *why = cudaGetErrorString(ce);
    return -2;
  }
  return 0;
}
