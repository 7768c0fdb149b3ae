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
//        (tril(A) as P_hi + P_lo, two bf16 operands, in the kSplit instance:
//        A to ~2^-17 relative; one bf16 operand in the other instance)
//   h_{n+1} = e^{G_last} * (h_n + S)   fp32 in registers, H_{n+1} = bf16(h_{n+1})
// which is the reference recurrence h_{n+1} = e^{G_last} h_n
// + (k e^{G_last-G})^T v with the per-key decay factored out of the sum.
// g_cumsum, A and the per-chunk states never touch HBM: q, k, v, g are read
// once and o (+ the final state) written once.
//
// One CTA per (batch, head, V slice of width VS), 512 threads:
//   warp 0        TMA producer of q, k, v (3- or 2-stage ring)
//   warp 1        tcgen05.mma issuer (dataflow order: A/S of chunk n+1, Qs H_n
//                 as soon as H_n is stored, P V as soon as P_n is written)
//   warp 2        TMEM allocator, then TMA producer of g
//   warps 4-11    gating (warp = 8 tokens, lane = 4 keys): chunk-local cumsum
//                 of the gate (per-warp prefixes exchanged through shared
//                 memory), Qs, Kg in place, e^{G_last}; then the O epilogue
//                 of the chunk two behind (TMEM -> bf16 -> HBM; at VS = 128
//                 through per-warp shared-memory slots and TMA stores, to
//                 several buffers in the kScatter instance)
//   warps 12-15   state warpgroup: A -> tril -> bf16 P, state update
//                 (thread = key row, VS fp32 columns in registers)
// Buffers: one g buffer, q/k/v in a 3-stage ring (2 stages in the forward at
// VS = 128, whose O slots, and in the kSplit instance also the second P
// buffer, take the third stage's room); A and O double-buffered in TMEM, S
// double-buffered when VS = 64; P (P_hi, P_lo) and the bf16 state copy H
// single-buffered (rewritten only after O_n completed).
#include "common.cuh"

namespace gl {
namespace gla {

constexpr int C = 64, KD = 128, NUM_THREADS = 512;
constexpr int GATE_WARPS = 8, STATE_WARPS = 4;
// Register split (launch: 512 x 128): control warpgroup 56, the two gating
// warpgroups keep 128, the state warpgroup rises to 216.
constexpr int REG_CTRL = 40, REG_STATE = 216;
static_assert(128 * REG_CTRL + 256 * 128 + 128 * REG_STATE <= NUM_THREADS * 128,
              "register split exceeds the launch allocation");

template <int VS, bool kSplit = false, bool kFwd = false>
struct Cfg {
  // q/k/v ring depth: a stage is released only once O of its chunk has
  // completed, so the load of chunk n+3 waits for the A -> P -> O chain of
  // chunk n.  The raw gate has one buffer, reloaded for chunk n+1 as soon as
  // the gating of chunk n has read it.  The S accumulator is double-buffered
  // in TMEM when its columns fit (VS = 64).  The forward at VS = 128 (kFwd)
  // gives up the third ring stage for the O staging slots below (and kSplit,
  // P as a bf16 hi + lo pair, for its second P buffer as well): measured
  // faster than three stages with O stored from registers.
  static constexpr int QS = (kSplit || (kFwd && VS == 128)) ? 2 : 3;
  static constexpr int NS = VS == 64 ? 2 : 1;
  static constexpr int V_BOXES = VS / 64;
  static constexpr uint32_t Q_BYTES = C * KD * 2;          // 16 KB (2 boxes of 64 features)
  static constexpr uint32_t V_BYTES = C * VS * 2;          // 8 / 16 KB
  static constexpr uint32_t G_BYTES = C * KD * 4;          // 32 KB
  static constexpr uint32_t P1_BYTES = C * C * 2;          // 8 KB: one bf16 P
  static constexpr uint32_t P_BYTES = (kSplit ? 2 : 1) * P1_BYTES;  // P (+ P_lo)
  static constexpr uint32_t H_BYTES = KD * VS * 2;         // 16 / 32 KB
  static constexpr uint32_t OFF_Q = 0;
  static constexpr uint32_t OFF_K = OFF_Q + QS * Q_BYTES;
  static constexpr uint32_t OFF_V = OFF_K + QS * Q_BYTES;
  static constexpr uint32_t OFF_G = OFF_V + QS * V_BYTES;
  static constexpr uint32_t OFF_P = OFF_G + G_BYTES;
  static constexpr uint32_t OFF_H = OFF_P + P_BYTES;
  static constexpr uint32_t OFF_DEC = OFF_H + H_BYTES;      // 2 x 128 floats
  static constexpr uint32_t OFF_PART = OFF_DEC + 2 * KD * 4;  // [2][8 warps][32 lanes] float4
  static constexpr uint32_t OFF_BAR = OFF_PART + 2 * 8 * 32 * 16;
  static constexpr uint32_t OFF_MISC = OFF_BAR + 512;
  // The forward at VS = 128 sends O through shared memory and TMA stores:
  // per gating warp a 2 KB slot (its 16 rows x 64 columns, 128B-swizzled),
  // two slots deep.  At VS = 64 the gating warps store O to global memory
  // from registers.
  static constexpr bool O_STG = kFwd && VS == 128;
  static constexpr uint32_t OSTG_SLOT = 16 * 64 * 2;
  static constexpr uint32_t OFF_OSTG = (OFF_MISC + 64 + 1023) / 1024 * 1024;
  static constexpr uint32_t OSTG_BYTES = O_STG ? 2 * 8 * OSTG_SLOT : 0;
  static constexpr uint32_t SMEM_BYTES = O_STG ? OFF_OSTG + OSTG_BYTES + 1024 : OFF_MISC + 64 + 1024;
  // TMEM columns: A0, A1 [0,128), O0, O1 [128,128+2VS), S0 (, S1) from 128+2VS
  static constexpr uint32_t COL_A = 0, COL_O = 128, COL_S = 128 + 2 * VS;
  static_assert(COL_S + NS * VS <= 512, "TMEM columns");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t IDESC_A = idesc(1, 1, 1, 0, 0, 64, 64);    // bf16, K-major x K-major
  static constexpr uint32_t IDESC_S = idesc(1, 1, 1, 1, 1, 128, VS);  // MN-major x MN-major
  static constexpr uint32_t IDESC_O = idesc(1, 1, 1, 0, 1, 64, VS);   // K-major x MN-major
};

// Kernel modes.  FWD: the forward (o, ht, optionally the per-chunk states
// h_n).  FWD_STATE: state-only pre-pass of a sequence split.  DH: the reverse
// state-gradient scan of the backward, over the chunks in reverse order with
// q in the k slot and do in the v slot: D_NT = dht, and per chunk
// E_n = e^{G_last(n)} D_{n+1} (written, bf16), D_n = E_n + Qs_n^T do_n, with
// D_0 = dh0.  DH_STATE: its state-only pre-pass.
enum { MODE_FWD = 0, MODE_FWD_STATE = 1, MODE_DH_STATE = 2, MODE_DH = 3 };

// Output tensor maps of the forward at VS = 128: O is stored into each of
// Params::n_outs buffers of the layout of o (the own output and, for a
// head-sharded forward, the same block of every peer's gather buffer).
constexpr int MAX_OUTS = 8;
static_assert(MAX_OUTS == GL_MAX_SCATTER_OUTS, "output count of the C ABI");
struct OutMaps {
  CUtensorMap m[MAX_OUTS];
};

struct Params {
  const float* g_gamma;  // [H] or null
  const float* h0;       // [B,H,K,V] or null (DH: the final-state gradient dht, or null)
  __nv_bfloat16* o;      // [B,T,H,V] (the first output)
  int n_outs;            // outputs of O (1..MAX_OUTS; > 1 only at VS = 128)
  float* ht;             // [B,H,K,V] or null (DH: dh0)
  int* err;
  float scale;
  float log2_scale;  // log2(scale) when scale > 0 (folded into the exponent), else 0
  int scale_apart;   // 1: scale <= 0 or not finite, applied as a separate multiply
  // Sequence split: chunks [seg*NT/nseg, (seg+1)*NT/nseg) form segment seg.
  // The state-only pass runs segments 0..nseg-2 from a zero state and writes
  // each one's final state ws_h [nseg-1][B*H][K][V] and total decay
  // ws_d [nseg-1][B*H][K]; the fold kernel turns record j into the initial
  // state of segment j+1 (h0 folded with segments 0..j), which the full pass
  // loads like h0.  nseg == 1: no split.
  // The reverse scan (DH) uses the same records for segments 1..nseg-1 (its
  // partial state-gradient at the segment start from a zero gradient at the
  // segment end, and the total decay); the reverse fold turns record j into
  // the gradient at the end of segment j.  A state-only grid covers segments
  // seg_base .. seg_base + seg_grid - 1.
  int nseg, seg_grid, seg_base;  // segments in total / per (b, h, V slice) in this grid / first
  // Forward split with a short first segment (c_first > 0 chunks): segment 0
  // runs the full pass from h0 while the state-only pass covers segments
  // 1..nseg-2; segment 0's full pass writes its final state, as its ht, into
  // record 0 (ht = ws_h, ht_seg = 0), from which the fold starts (its decay
  // record is not written); segments 1.. share the remaining chunks.  c_first = 0:
  // equal segments as above.  Record of segment seg: seg - rec_base.
  // ht_seg: the segment whose final state is written to ht.
  int c_first, rec_base, ht_seg;
  int has_hout;  // FWD: write h_n (bf16, [B,NT,H,K,V]) through tm_h; DH: E_n (always)
  // FWD: 1 selects the kSplit instance of the kernel, which computes
  // tril(A) V as P_hi V + P_lo V (P_hi = bf16(tril(A)), P_lo =
  // bf16(tril(A) - P_hi) in a second P buffer, ~2^-17 relative: the fp32 A
  // of the template's output kernel; the buffer takes the room of the third
  // q/k/v stage); 0 feeds the tensor core bf16(tril(A)) only (the bf16
  // operands of the reference jnp einsum at TPU default precision).
  int p_split;
  float* ws_h;
  float* ws_d;
  int B, T, H, nsplit;
  int has_g;
};

// Barrier indices ([2] = one per buffer).
enum {
  B_QKV_FULL = 0,    // [QS] TMA -> gating
  B_QKV_EMPTY = 3,   // [QS] O_n committed -> TMA
  B_G_FULL = 6,      // TMA -> gating
  B_G_EMPTY = 7,     // gating -> TMA (8 warps read the gate)
  B_PREP = 10,       // [2] gating -> MMA
  B_DEC_FULL = 12,   // [2] gating -> state
  B_DEC_EMPTY = 14,  // [2] state -> gating
  B_A_FULL = 16,     // [2] MMA A_n committed -> P epilogue
  B_A_EMPTY = 18,    // [2] P epilogue -> MMA
  B_O_FULL = 20,     // [2] MMA O_n committed -> state
  B_O_EMPTY = 22,    // [2] O read (gating warps) -> MMA
  B_S_FULL = 24,     // [NS] MMA S_n committed -> state
  B_S_EMPTY = 26,    // [NS] state read S -> MMA
  B_P_FULL = 28,     // P written -> MMA
  B_H_FULL = 29,     // H_n written -> MMA
  B_DRAIN = 30,
  B_GSYNC = 31,      // [2] gating quarter sums written
  B_HST = 33,        // the TMA store of the previous state tile has read shared memory
  NUM_BARS = 34
};
static_assert(NUM_BARS * 8 <= 512, "barrier area");

// 2^x with the hardware approximation (the same unit __expf uses).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float2 bf16x2_f32x2(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
}

// Offset of bf16 element (row, col) in a K-major, 128B-swizzled tile made of
// 64-column atoms stacked `atom_stride` bytes apart (rows 128 B apart).
__device__ __forceinline__ uint32_t kmaj_off(uint32_t row, uint32_t col, uint32_t atom_stride) {
  return (col >> 6) * atom_stride + row * 128u + ((((col & 63u) >> 3) ^ (row & 7u)) << 4) +
         (col & 7u) * 2u;
}

// kScatter (forward at VS = 128 only): O goes to Params::n_outs outputs;
// a separate instance, since the extra stores cost the gating warps
// registers.
template <int VS, int kMode, bool kSplit, bool kScatter = false>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    chunk_gla_fwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                         const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v,
                         const __grid_constant__ CUtensorMap tm_g,
                         const __grid_constant__ CUtensorMap tm_h,
                         const __grid_constant__ OutMaps tm_o, const Params p) {
  using CF = Cfg<VS, kSplit, kMode == MODE_FWD>;
  // kStateOnly: S_n = (k slot)^T (v slot) only (no q, A, O).  kRev: chunks
  // in reverse order, the k slot scaled like q (Qs) instead of k (Kg).
  constexpr bool kStateOnly = kMode != MODE_FWD;
  constexpr bool kRev = kMode == MODE_DH || kMode == MODE_DH_STATE;
  extern __shared__ uint8_t smem_raw[];
  // 1 KB-aligned base derived by pointer arithmetic on the shared array so
  // that every access below stays in the shared address space.
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + CF::OFF_BAR);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + CF::OFF_MISC);
  int* abort_flag = reinterpret_cast<int*>(smem + CF::OFF_MISC + 4);
  float* dec = reinterpret_cast<float*>(smem + CF::OFF_DEC);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int T = p.T, H = p.H;
  const int seg = p.seg_base + static_cast<int>(blockIdx.x) % p.seg_grid;
  const int rest = blockIdx.x / p.seg_grid;
  const int bh = rest / p.nsplit, vsl = rest % p.nsplit;
  const int b = bh / H, h = bh % H;
  const int v0 = vsl * VS;
  auto seg_chunk = [&](int j) -> int {  // first chunk of segment j (j = nseg: the end)
    const int64_t nt = T / C;
    if (p.c_first <= 0) return static_cast<int>(j * nt / p.nseg);
    if (j == 0) return 0;
    return p.c_first + static_cast<int>((j - 1) * (nt - p.c_first) / (p.nseg - 1));
  };
  const int c0 = seg_chunk(seg);
  const int c1 = seg_chunk(seg + 1);
  const int NT = c1 - c0;  // chunks of this CTA
  const int tok0 = b * T + c0 * C;
  // Sequence position of the n-th chunk this CTA processes.
  auto chunk_of = [&](int n) { return kRev ? NT - 1 - n : n; };
  const Abort ab{abort_flag, p.err};

  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
    if (p.has_g) prefetch_tmap(&tm_g);
    if (p.has_hout) prefetch_tmap(&tm_h);
  } else if (warp == 1 && lane == 0) {
    for (int i = 0; i < CF::QS; ++i) {
      mbar_init(&bar[B_QKV_FULL + i], 1);
      mbar_init(&bar[B_QKV_EMPTY + i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar[B_PREP + i], GATE_WARPS);
      mbar_init(&bar[B_DEC_FULL + i], GATE_WARPS);
      mbar_init(&bar[B_GSYNC + i], GATE_WARPS);
      mbar_init(&bar[B_DEC_EMPTY + i], STATE_WARPS);
      mbar_init(&bar[B_A_FULL + i], 1);
      mbar_init(&bar[B_A_EMPTY + i], STATE_WARPS);
      mbar_init(&bar[B_O_FULL + i], 1);
      mbar_init(&bar[B_O_EMPTY + i], GATE_WARPS);
    }
    for (int i = 0; i < CF::NS; ++i) {
      mbar_init(&bar[B_S_FULL + i], 1);
      mbar_init(&bar[B_S_EMPTY + i], STATE_WARPS);
    }
    mbar_init(&bar[B_P_FULL], STATE_WARPS);
    mbar_init(&bar[B_H_FULL], STATE_WARPS);
    mbar_init(&bar[B_DRAIN], 1);
    mbar_init(&bar[B_HST], 1);
    mbar_init(&bar[B_G_FULL], 1);
    mbar_init(&bar[B_G_EMPTY], GATE_WARPS);
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
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_CTRL));
    // ------------------------------------------------------- TMA q, k, v
    if (lane == 0) {
      for (int n = 0; n < NT; ++n) {
        const int s = n % CF::QS;
        const int tok = tok0 + chunk_of(n) * C;
        if (!mbar_wait(&bar[B_QKV_EMPTY + s], ((n / CF::QS) & 1) ^ 1, ab)) break;
        mbar_arrive_expect_tx(&bar[B_QKV_FULL + s], (kStateOnly ? 1 : 2) * CF::Q_BYTES + CF::V_BYTES);
        uint8_t* qd = smem + CF::OFF_Q + s * CF::Q_BYTES;
        uint8_t* kd = smem + CF::OFF_K + s * CF::Q_BYTES;
        uint8_t* vd = smem + CF::OFF_V + s * CF::V_BYTES;
        if (!kStateOnly) {
          tma_load_3d(qd, &tm_q, &bar[B_QKV_FULL + s], 0, h, tok);
          tma_load_3d(qd + 8192, &tm_q, &bar[B_QKV_FULL + s], 64, h, tok);
        }
        tma_load_3d(kd, &tm_k, &bar[B_QKV_FULL + s], 0, h, tok);
        tma_load_3d(kd + 8192, &tm_k, &bar[B_QKV_FULL + s], 64, h, tok);
#pragma unroll
        for (int j = 0; j < CF::V_BOXES; ++j)
          tma_load_3d(vd + j * 8192, &tm_v, &bar[B_QKV_FULL + s], v0 + 64 * j, h, tok);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_CTRL));
    // ----------------------------------------------------------------- MMA
    if (lane == 0) {
      constexpr int QS = CF::QS, NS = CF::NS;
      const uint32_t p_addr = s_base + CF::OFF_P;
      const uint32_t h_addr = s_base + CF::OFF_H;
      // A_m = Qs Kg^T (M=64 query rows, N=64 key rows, K=128 features) into
      // TMEM buffer m%2; S_m = Kg^T V (M=128 features, N=VS, K=64 tokens).
      auto issue_a_s = [&](int m) {
        const int s = m & 1, st = m % QS;
        const uint32_t q_addr = s_base + CF::OFF_Q + st * CF::Q_BYTES;
        const uint32_t k_addr = s_base + CF::OFF_K + st * CF::Q_BYTES;
        const uint32_t v_addr = s_base + CF::OFF_V + st * CF::V_BYTES;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t koff = (kk >> 2) * 8192 + (kk & 3) * 32;
          mma_f16(tmem + CF::COL_A + s * 64, sdesc(q_addr + koff, 16, 1024, kSwizzle128B),
                  sdesc(k_addr + koff, 16, 1024, kSwizzle128B), CF::IDESC_A, kk > 0);
        }
        tc_commit(&bar[B_A_FULL + s]);
        const int sb = m % NS;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          mma_f16(tmem + CF::COL_S + sb * VS, sdesc(k_addr + kk * 2048, 8192, 1024, kSwizzle128B),
                  sdesc(v_addr + kk * 2048, 8192, 1024, kSwizzle128B), CF::IDESC_S, kk > 0);
        }
        tc_commit(&bar[B_S_FULL + sb]);
      };
      // O_n (TMEM buffer n%2) = Qs H_n (issued once H_n is stored) + P V
      // (issued once P_n is written); the second part frees the q/k/v stage.
      auto issue_o_h = [&](int n) {
        const int s = n & 1;
        const uint32_t q_addr = s_base + CF::OFF_Q + (n % QS) * CF::Q_BYTES;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t koff = (kk >> 2) * 8192 + (kk & 3) * 32;
          mma_f16(tmem + CF::COL_O + s * VS, sdesc(q_addr + koff, 16, 1024, kSwizzle128B),
                  sdesc(h_addr + kk * 2048, 16384, 1024, kSwizzle128B), CF::IDESC_O, kk > 0);
        }
      };
      // P V; with kSplit P_hi V then P_lo V (P_hi = bf16(tril(A)), P_lo =
      // bf16(tril(A) - P_hi) in the second P buffer), so that the product
      // sees A to ~2^-17 relative.
      auto issue_o_p = [&](int n) {
        const int s = n & 1;
        const uint32_t v_addr = s_base + CF::OFF_V + (n % QS) * CF::V_BYTES;
#pragma unroll
        for (int part = 0; part < (kSplit ? 2 : 1); ++part)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            mma_f16(tmem + CF::COL_O + s * VS,
                    sdesc(p_addr + part * CF::P1_BYTES + kk * 32, 16, 1024, kSwizzle128B),
                    sdesc(v_addr + kk * 2048, 8192, 1024, kSwizzle128B), CF::IDESC_O, 1);
          }
        tc_commit(&bar[B_O_FULL + s]);
        tc_commit(&bar[B_QKV_EMPTY + n % QS]);
      };
      // Dataflow issue.  na: next chunk for A/S (needs its gating, its A
      // buffer free and the previous S read); nh: next chunk for Qs H (needs
      // H_nh and its O buffer drained); no: next chunk for P V (needs P_no).
      if (kStateOnly) {
        // S_n only; the q/k/v stage is free once S_n has completed.
        for (int n = 0; n < NT; ++n) {
          const int st = n % QS, sb = n % NS;
          if (!mbar_wait(&bar[B_PREP + (n & 1)], (n >> 1) & 1, ab)) break;
          if (!mbar_wait(&bar[B_S_EMPTY + sb], ((n / NS) & 1) ^ 1, ab)) break;
          tc_fence_after();
          const uint32_t k_addr = s_base + CF::OFF_K + st * CF::Q_BYTES;
          const uint32_t v_addr = s_base + CF::OFF_V + st * CF::V_BYTES;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_f16(tmem + CF::COL_S + sb * VS, sdesc(k_addr + kk * 2048, 8192, 1024, kSwizzle128B),
                    sdesc(v_addr + kk * 2048, 8192, 1024, kSwizzle128B), CF::IDESC_S, kk > 0);
          tc_commit(&bar[B_S_FULL + sb]);
          tc_commit(&bar[B_QKV_EMPTY + st]);
        }
      } else {
        int na = 0, nh = 0, no = 0;
        uint64_t t0 = global_ns();
        uint32_t spins = 0;
        while (no < NT) {
          bool progressed = false;
          if (no < nh && mbar_test(&bar[B_P_FULL], no & 1)) {
            tc_fence_after();
            issue_o_p(no);
            ++no;
            progressed = true;
          }
          if (nh < na && nh == no && mbar_test(&bar[B_H_FULL], nh & 1) &&
              mbar_test(&bar[B_O_EMPTY + (nh & 1)], ((nh >> 1) & 1) ^ 1)) {
            tc_fence_after();
            issue_o_h(nh);
            ++nh;
            progressed = true;
          }
          if (na < NT && na <= no + QS - 1) {
            const int s = na & 1;
            const uint32_t ph2 = (na >> 1) & 1;
            if (mbar_test(&bar[B_PREP + s], ph2) && mbar_test(&bar[B_A_EMPTY + s], ph2 ^ 1) &&
                mbar_test(&bar[B_S_EMPTY + na % NS], ((na / NS) & 1) ^ 1)) {
              tc_fence_after();
              issue_a_s(na);
              ++na;
              progressed = true;
            }
          }
          if (progressed) {
            t0 = global_ns();
            spins = 0;
          } else if ((++spins & 255u) != 0) {
            __nanosleep(20);  // leave the issue slots to the gating warps
          } else {
            if (*abort_flag) break;
            if (global_ns() - t0 > kWaitNs) {
              *abort_flag = 1;
              atomicExch(p.err, GL_DEV_WAIT_TIMEOUT);
              break;
            }
          }
        }
      }
      tc_commit(&bar[B_DRAIN]);
      const uint64_t td = global_ns();
      while (!mbar_try_wait(&bar[B_DRAIN], 0) && global_ns() - td < 100000000ull) {
      }
    }
    __syncwarp();
  } else if (warp == 2) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_CTRL));
    // ----------------------------------------------------------- TMA g
    if (lane == 0 && p.has_g) {
      for (int n = 0; n < NT; ++n) {
        if (!mbar_wait(&bar[B_G_EMPTY], (n & 1) ^ 1, ab)) break;
        mbar_arrive_expect_tx(&bar[B_G_FULL], CF::G_BYTES);
        tma_load_3d(smem + CF::OFF_G, &tm_g, &bar[B_G_FULL], 0, h, tok0 + chunk_of(n) * C);
      }
    }
    __syncwarp();
  } else if (warp == 3) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_CTRL));
  } else if (warp >= 4 && warp < 4 + GATE_WARPS) {
    // ---------------------------------------------------------- gating
    // Warp gw = warp - 4 takes tokens 8 gw .. 8 gw + 7 of the chunk, lane l
    // keys 4 l .. 4 l + 3 (16-byte gate loads, 8-byte q / k accesses).  Each
    // warp sums the gate over its 8 tokens, the per-warp sums are exchanged
    // through shared memory, and the chunk-local cumsum continues from the
    // sum of the preceding warps.
    const int gw = warp - 4;
    const float gamma = p.has_g ? 0.f : __ldg(p.g_gamma + h);
    constexpr float kLog2e = 1.4426950408889634f;
    const float log2_scale = p.log2_scale;
    // q / k tiles: K-major, 128B-swizzled, 64-feature atoms 8 KB apart.
    const uint32_t qk_atom = static_cast<uint32_t>(lane >> 4) * 8192u;
    const uint32_t qk_chunk = static_cast<uint32_t>(lane & 15) >> 1, qk_sub = (lane & 1) * 8u;
    // O epilogue of chunk m (run two chunks behind the gating, when O_m is
    // long complete): this warp reads TMEM lane quadrant warp%4, i.e. rows
    // 16*quad .. 16*quad+15 of the M=64 accumulator, columns half*VS/2 ..
    constexpr int OC = VS / 2;
    const int oquad = warp & 3, ohalf = (warp - 4) >> 2;
    const int orow = oquad * 16 + (lane & 15);
    const uint32_t o_lane = tmem + (static_cast<uint32_t>(oquad * 32) << 16) + CF::COL_O + ohalf * OC;
    auto o_epilogue = [&](int m) -> bool {
      const int s = m & 1;
      if (!mbar_wait(&bar[B_O_FULL + s], (m >> 1) & 1, ab)) return false;
      tc_fence_after();
      const int64_t row = static_cast<int64_t>(tok0) + m * C + orow;
      uint4* dst = reinterpret_cast<uint4*>(p.o + (row * H + h) * 128 + v0 + ohalf * OC);
      auto store32 = [&](const uint32_t (&ov)[32], int j) {
        if (lane < 16) {
#pragma unroll
          for (int i = 0; i < 4; ++i)
            dst[j / 8 + i] = make_uint4(
                pack_bf16x2(__uint_as_float(ov[8 * i]), __uint_as_float(ov[8 * i + 1])),
                pack_bf16x2(__uint_as_float(ov[8 * i + 2]), __uint_as_float(ov[8 * i + 3])),
                pack_bf16x2(__uint_as_float(ov[8 * i + 4]), __uint_as_float(ov[8 * i + 5])),
                pack_bf16x2(__uint_as_float(ov[8 * i + 6]), __uint_as_float(ov[8 * i + 7])));
        }
      };
      if constexpr (CF::O_STG) {
        // this warp's 16 rows x 64 columns -> its slot (row = lane, 16-byte
        // chunk c at c ^ (row & 7): the 128B swizzle of the map) -> one TMA
        // store of a 64 x 1 x 16 box
        uint32_t ov0[32], ov1[32];
        tmem_ld32(o_lane + s * VS, ov0);
        tmem_ld32(o_lane + s * VS + 32, ov1);
        uint8_t* slot = smem + CF::OFF_OSTG + ((m & 1) * GATE_WARPS + (warp - 4)) * CF::OSTG_SLOT;
        if (lane == 0) bulk_wait_read<1>();  // the store of chunk m-2 has read this slot
        tmem_ld_wait2(ov0, ov1);
        __syncwarp();
        if (lane < 16) {
          const uint32_t srow = smem_u32(slot) + lane * 128u;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint32_t* w = c < 4 ? ov0 + 8 * c : ov1 + 8 * (c - 4);
            st_shared_v4(srow + ((c ^ (lane & 7)) << 4),
                         pack_bf16x2(__uint_as_float(w[0]), __uint_as_float(w[1])),
                         pack_bf16x2(__uint_as_float(w[2]), __uint_as_float(w[3])),
                         pack_bf16x2(__uint_as_float(w[4]), __uint_as_float(w[5])),
                         pack_bf16x2(__uint_as_float(w[6]), __uint_as_float(w[7])));
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          const int32_t ox = v0 + ohalf * OC, oz = tok0 + m * C + oquad * 16;
          if constexpr (kScatter) {
#pragma unroll
            for (int oo = 0; oo < MAX_OUTS; ++oo)  // constant map offsets, predicated
              if (oo < p.n_outs) tma_store_3d(&tm_o.m[oo], slot, ox, h, oz);
          } else {
            tma_store_3d(&tm_o.m[0], slot, ox, h, oz);
          }
          bulk_commit();
        }
      } else if constexpr (OC == 64) {
        // both column halves in flight before one wait
        uint32_t ov0[32], ov1[32];
        tmem_ld32(o_lane + s * VS, ov0);
        tmem_ld32(o_lane + s * VS + 32, ov1);
        tmem_ld_wait2(ov0, ov1);
        store32(ov0, 0);
        store32(ov1, 32);
      } else {
        uint32_t ov[32];
        tmem_ld32(o_lane + s * VS, ov);
        tmem_ld_wait(ov);
        store32(ov, 0);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[B_O_EMPTY + s]);
      return true;
    };
    bool gok = true;
    for (int n = 0; n < NT && gok; ++n) {
      const int s = n & 1;
      const uint32_t ph2 = (n >> 1) & 1;
      if (p.has_g && !mbar_wait(&bar[B_G_FULL], n & 1, ab)) { gok = false; break; }
      if (!mbar_wait(&bar[B_QKV_FULL + n % CF::QS], (n / CF::QS) & 1, ab)) { gok = false; break; }
      uint8_t* qs = smem + CF::OFF_Q + (n % CF::QS) * CF::Q_BYTES + qk_atom + qk_sub;
      uint8_t* ks = smem + CF::OFF_K + (n % CF::QS) * CF::Q_BYTES + qk_atom + qk_sub;
      float4 gv[8];
      float4 G = make_float4(0.f, 0.f, 0.f, 0.f);
      if (p.has_g) {
        const float4* g4 = reinterpret_cast<const float4*>(smem + CF::OFF_G) + lane;
        float4 tot = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          gv[i] = g4[(gw * 8 + i) * (KD / 4)];
          tot.x += gv[i].x;
          tot.y += gv[i].y;
          tot.z += gv[i].z;
          tot.w += gv[i].w;
        }
        // the gate buffer can take the next chunk's gate
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar[B_G_EMPTY]);
        float4* part = reinterpret_cast<float4*>(smem + CF::OFF_PART) + s * (GATE_WARPS * 32);
        part[gw * 32 + lane] = tot;
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar[B_GSYNC + s]);
        if (!mbar_wait(&bar[B_GSYNC + s], ph2, ab)) { gok = false; break; }
        for (int w = 0; w < gw; ++w) {
          const float4 pv = part[w * 32 + lane];
          G.x += pv.x;
          G.y += pv.y;
          G.z += pv.z;
          G.w += pv.w;
        }
      }
      // Qs = q * 2^(G log2e + log2 scale), Kg = k * 2^(-G log2e), packed
      // f32x2 arithmetic, four keys per lane.
      const float2 L2 = make_float2(kLog2e, kLog2e), NL2 = make_float2(-kLog2e, -kLog2e);
      const float2 LS2 = make_float2(log2_scale, log2_scale);
      float2 G01 = make_float2(G.x, G.y), G23 = make_float2(G.z, G.w);
      // The 8 tokens' q and k are read before any of them is written back,
      // so the loads do not queue behind the stores of earlier tokens.
      uint2 qv[8], kv[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int t = gw * 8 + i;
        const uint32_t off = static_cast<uint32_t>(t) * 128u + ((qk_chunk ^ (t & 7)) << 4);
        if (!kStateOnly) qv[i] = *reinterpret_cast<const uint2*>(qs + off);
        kv[i] = *reinterpret_cast<const uint2*>(ks + off);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int t = gw * 8 + i;
        float2 xa01, xa23, xb01, xb23;
        if (p.has_g) {
          G01 = __fadd2_rn(G01, make_float2(gv[i].x, gv[i].y));
          G23 = __fadd2_rn(G23, make_float2(gv[i].z, gv[i].w));
          xa01 = __ffma2_rn(G01, L2, LS2);
          xa23 = __ffma2_rn(G23, L2, LS2);
          xb01 = __fmul2_rn(G01, NL2);
          xb23 = __fmul2_rn(G23, NL2);
        } else {
          const float Gt = gamma * static_cast<float>(t + 1);
          G01 = G23 = make_float2(Gt, Gt);
          xa01 = xa23 = make_float2(fmaf(Gt, kLog2e, log2_scale), fmaf(Gt, kLog2e, log2_scale));
          xb01 = xb23 = make_float2(-Gt * kLog2e, -Gt * kLog2e);
        }
        // k slot: Kg = k e^-G, or in the reverse scan Qs = scale q e^G.
        const float2 xk01 = kRev ? xa01 : xb01, xk23 = kRev ? xa23 : xb23;
        const float2 b01 = make_float2(ex2_approx(xk01.x), ex2_approx(xk01.y));
        const float2 b23 = make_float2(ex2_approx(xk23.x), ex2_approx(xk23.y));
        const uint32_t off = static_cast<uint32_t>(t) * 128u + ((qk_chunk ^ (t & 7)) << 4);
        if (!kStateOnly) {
          const float2 a01 = make_float2(ex2_approx(xa01.x), ex2_approx(xa01.y));
          const float2 a23 = make_float2(ex2_approx(xa23.x), ex2_approx(xa23.y));
          const uint2 q2 = qv[i];
          float2 q01 = __fmul2_rn(bf16x2_f32x2(q2.x), a01), q23 = __fmul2_rn(bf16x2_f32x2(q2.y), a23);
          if (p.scale_apart) {
            q01 = __fmul2_rn(q01, make_float2(p.scale, p.scale));
            q23 = __fmul2_rn(q23, make_float2(p.scale, p.scale));
          }
          *reinterpret_cast<uint2*>(qs + off) =
              make_uint2(pack_bf16x2(q01.x, q01.y), pack_bf16x2(q23.x, q23.y));
        }
        const uint2 k2 = kv[i];
        float2 k01 = __fmul2_rn(bf16x2_f32x2(k2.x), b01), k23 = __fmul2_rn(bf16x2_f32x2(k2.y), b23);
        if (kRev && p.scale_apart) {
          k01 = __fmul2_rn(k01, make_float2(p.scale, p.scale));
          k23 = __fmul2_rn(k23, make_float2(p.scale, p.scale));
        }
        *reinterpret_cast<uint2*>(ks + off) =
            make_uint2(pack_bf16x2(k01.x, k01.y), pack_bf16x2(k23.x, k23.y));
      }
      if (gw == GATE_WARPS - 1) {
        // e^{G_last}, once the state warps have taken the decay of chunk n-2
        if (!mbar_wait(&bar[B_DEC_EMPTY + s], ph2 ^ 1, ab)) { gok = false; break; }
        const float2 d01 = __fmul2_rn(G01, L2), d23 = __fmul2_rn(G23, L2);
        *reinterpret_cast<float4*>(dec + s * KD + 4 * lane) =
            make_float4(ex2_approx(d01.x), ex2_approx(d01.y), ex2_approx(d23.x), ex2_approx(d23.y));
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&bar[B_PREP + s]);
        mbar_arrive(&bar[B_DEC_FULL + s]);
      }
      if (!kStateOnly && n >= 2 && !o_epilogue(n - 2)) gok = false;
    }
    if (!kStateOnly)
      for (int m = NT >= 2 ? NT - 2 : 0; m < NT && gok; ++m) gok = o_epilogue(m);
    if constexpr (CF::O_STG && !kStateOnly) {
      if (lane == 0) bulk_wait<0>();  // the O stores are complete before the CTA exits
      __syncwarp();
    }
  } else if (warp >= 4 + GATE_WARPS) {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REG_STATE));
    // ------------------------- P epilogue, state update, O epilogue
    const int quad = warp & 3;
    const int key = quad * 32 + lane;              // state row == TMEM lane
    const int prow = quad * 16 + (lane & 15);      // row of an M=64 accumulator
    const int64_t bhi = static_cast<int64_t>(b) * H + h;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    float hreg[VS];
    // Initial state: h0 for the first segment (DH: dht for the last); with a
    // sequence split, the other segments start from the state the fold
    // kernel left in the workspace.
    const float* init = nullptr;
    if (kMode == MODE_FWD)
      init = seg == 0 ? (p.h0 ? p.h0 + bhi * KD * 128 : nullptr)
                      : p.ws_h + (static_cast<int64_t>(seg - 1) * p.B * H + bhi) * KD * 128;
    else if (kMode == MODE_DH)
      init = seg == p.nseg - 1 ? (p.h0 ? p.h0 + bhi * KD * 128 : nullptr)
                               : p.ws_h + (static_cast<int64_t>(seg) * p.B * H + bhi) * KD * 128;
    if (init) {
      const float4* src = reinterpret_cast<const float4*>(init + static_cast<int64_t>(key) * 128 + v0);
#pragma unroll
      for (int j = 0; j < VS / 4; ++j) {
        const float4 x = __ldg(src + j);
        hreg[4 * j] = x.x;
        hreg[4 * j + 1] = x.y;
        hreg[4 * j + 2] = x.z;
        hreg[4 * j + 3] = x.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < VS; ++j) hreg[j] = 0.f;
    }
    float dacc = 1.f;  // state-only pass: product of the chunk decays
    constexpr int NS = CF::NS;
    // H: MN-major B operand [128 keys][VS], 64-column atoms 16 KB apart,
    // which is also the layout of a 128B-swizzled TMA box of 64 x 128: with
    // has_hout, thread 0 of warp 12 stores it to row ((b NT + chunk) H + h)
    // 128 of the state output once all four warps wrote it (B_H_FULL), and
    // releases the buffer (B_HST) when the store has read it.
    const bool st_issuer = warp == 4 + GATE_WARPS && lane == 0;
    int nstore = 0;
    auto store_h = [&](int chunk) -> bool {
      if (p.has_hout && nstore > 0) {
        if (st_issuer) {
          bulk_wait_read<0>();
          mbar_arrive(&bar[B_HST]);
        }
        if (!mbar_wait(&bar[B_HST], (nstore - 1) & 1, ab)) return false;
      }
      uint8_t* hp = smem + CF::OFF_H;
#pragma unroll
      for (int c8 = 0; c8 < VS / 8; ++c8) {
        const uint4 w = make_uint4(pack_bf16x2(hreg[c8 * 8], hreg[c8 * 8 + 1]),
                                   pack_bf16x2(hreg[c8 * 8 + 2], hreg[c8 * 8 + 3]),
                                   pack_bf16x2(hreg[c8 * 8 + 4], hreg[c8 * 8 + 5]),
                                   pack_bf16x2(hreg[c8 * 8 + 6], hreg[c8 * 8 + 7]));
        *reinterpret_cast<uint4*>(hp + kmaj_off(key, c8 * 8, 16384)) = w;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[B_H_FULL]);
      if (p.has_hout) {
        bool sok = true;
        if (st_issuer) {
          sok = mbar_wait(&bar[B_H_FULL], nstore & 1, ab);
          if (sok) {
            const int32_t row = ((b * (T / C) + c0 + chunk) * H + h) * KD;
#pragma unroll
            for (int j = 0; j < CF::V_BOXES; ++j) tma_store_2d(&tm_h, hp + j * 16384, v0 + 64 * j, row);
            bulk_commit();
          }
        }
        if (!__shfl_sync(0xffffffffu, sok, 0)) return false;
      }
      ++nstore;
      return true;
    };
    // P = tril(A_m) in bf16, K-major (row = query, 128 B); with kSplit also
    // P_lo = bf16(tril(A_m) - P) in the second P buffer.
    auto p_epilogue = [&](int m) -> bool {
      const int s = m & 1;
      if (!mbar_wait(&bar[B_A_FULL + s], (m >> 1) & 1, ab)) return false;
      tc_fence_after();
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t a[32];
        tmem_ld32(lane_addr + CF::COL_A + s * 64 + half * 32, a);
        tmem_ld_wait(a);
        if (half == 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bar[B_A_EMPTY + s]);
        }
        if (lane < 16) {
          uint8_t* pp = smem + CF::OFF_P + prow * 128;
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4) {
            float f[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const int j = half * 32 + c4 * 8 + e;
              f[e] = j <= prow ? __uint_as_float(a[c4 * 8 + e]) : 0.f;
            }
            const uint32_t ch = static_cast<uint32_t>(half * 4 + c4) ^ (prow & 7);
            const uint4 hi = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]),
                                        pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
            *reinterpret_cast<uint4*>(pp + (ch << 4)) = hi;
            if constexpr (kSplit) {
              const uint32_t hw[4] = {hi.x, hi.y, hi.z, hi.w};
              float r[8];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 h2 = bf16x2_f32x2(hw[e]);
                r[2 * e] = f[2 * e] - h2.x;
                r[2 * e + 1] = f[2 * e + 1] - h2.y;
              }
              *reinterpret_cast<uint4*>(pp + CF::P1_BYTES + (ch << 4)) =
                  make_uint4(pack_bf16x2(r[0], r[1]), pack_bf16x2(r[2], r[3]),
                             pack_bf16x2(r[4], r[5]), pack_bf16x2(r[6], r[7]));
            }
          }
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[B_P_FULL]);
      return true;
    };
    bool ok = true;
    if (!kStateOnly) ok = store_h(0) && p_epilogue(0);
    for (int n = 0; n < NT && ok; ++n) {
      const int s = n & 1;
      const uint32_t ph2 = (n >> 1) & 1;
      // state update: h <- e^{G_last} (h + S_n)
      if (!mbar_wait(&bar[B_DEC_FULL + s], ph2, ab)) { ok = false; break; }
      const float d = dec[s * KD + key];
      dacc *= d;
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[B_DEC_EMPTY + s]);
      if (kRev) {
        // E_n = e^{G_last} D_{n+1} (written in the DH pass), then D_n = E_n + S_n.
#pragma unroll
        for (int j = 0; j < VS; j += 2) {
          const float2 e = __fmul2_rn(make_float2(hreg[j], hreg[j + 1]), make_float2(d, d));
          hreg[j] = e.x;
          hreg[j + 1] = e.y;
        }
        if (kMode == MODE_DH && !store_h(chunk_of(n))) { ok = false; break; }
      }
      if (!mbar_wait(&bar[B_S_FULL + n % NS], (n / NS) & 1, ab)) { ok = false; break; }
      tc_fence_after();
#pragma unroll
      for (int j = 0; j < VS; j += 32) {
        uint32_t sv[32];
        tmem_ld32(lane_addr + CF::COL_S + (n % NS) * VS + j, sv);
        tmem_ld_wait(sv);
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float2 hs = __fadd2_rn(make_float2(hreg[j + i], hreg[j + i + 1]),
                                       make_float2(__uint_as_float(sv[i]), __uint_as_float(sv[i + 1])));
          if (kRev) {
            hreg[j + i] = hs.x;
            hreg[j + i + 1] = hs.y;
          } else {
            const float2 hn = __fmul2_rn(hs, make_float2(d, d));
            hreg[j + i] = hn.x;
            hreg[j + i + 1] = hn.y;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[B_S_EMPTY + n % NS]);
      if (kStateOnly) continue;
      // O_n done -> H and P may be rewritten for chunk n+1 (the next O
      // accumulates into the other TMEM buffer meanwhile)
      if (!mbar_wait(&bar[B_O_FULL + s], ph2, ab)) { ok = false; break; }
      tc_fence_after();
      if (n + 1 < NT && !(store_h(n + 1) && p_epilogue(n + 1))) { ok = false; break; }
    }
    if (st_issuer && p.has_hout) bulk_wait<0>();
    if (ok && (kMode == MODE_FWD_STATE || kMode == MODE_DH_STATE)) {
      const int64_t rec = static_cast<int64_t>(seg - p.rec_base) * p.B * H + bhi;
      float4* dst = reinterpret_cast<float4*>(p.ws_h + (rec * KD + key) * 128 + v0);
#pragma unroll
      for (int j = 0; j < VS / 4; ++j)
        dst[j] = make_float4(hreg[4 * j], hreg[4 * j + 1], hreg[4 * j + 2], hreg[4 * j + 3]);
      if (vsl == 0) p.ws_d[rec * KD + key] = dacc;
    } else if (ok && p.ht && seg == p.ht_seg) {
      float4* dst = reinterpret_cast<float4*>(p.ht + (bhi * KD + key) * 128 + v0);
#pragma unroll
      for (int j = 0; j < VS / 4; ++j)
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

// Sequence split: record j (the zero-start final state h_j and total decay
// D_j of segment j) becomes the initial state of segment j+1,
//   s_{j+1} = D_j * s_j + h_j,  s_0 = h0 (or 0),
// the recurrence h_{n+1} = d_n (h_n + S_n) being linear in h_n with a per-row
// scale.  reverse (the DH scan): record j holds segment j+1's zero-start
// gradient and decay, folded from the last segment down, starting from dht
// (passed as h0).  pass_first (forward only): record 0 already holds the
// true state after segment 0 and is the start; its decay is not read.
// One thread per 4 state entries (a float4) of one (batch, head).  The
// records do not depend on the running state, so their loads are issued NB
// at a time ahead of the dependent multiply-adds; the launcher takes NB = 4
// for few records (low registers, full occupancy) and up to 16 for many.
template <int NB>
__global__ void __launch_bounds__(256) gla_fold_kernel(const float* __restrict__ h0,
                                                       float* __restrict__ ws_h,
                                                       const float* __restrict__ ws_d, int BH,
                                                       int nseg, int reverse, int pass_first) {
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= static_cast<int64_t>(BH) * KD * 32) return;
  const int bh = static_cast<int>(t / (KD * 32));
  const int key = static_cast<int>((t / 32) % KD), c4 = static_cast<int>(t % 32);
  auto rec_of = [&](int j) -> int64_t { return static_cast<int64_t>(j) * BH + bh; };
  auto slot_of = [&](int64_t r) -> float4* {
    return reinterpret_cast<float4*>(ws_h + (r * KD + key) * 128) + c4;
  };
  const int nrec = nseg - 1;
  float4 h;
  int i = 0;
  if (pass_first && !reverse && nrec > 0) {
    h = *slot_of(rec_of(0));
    i = 1;
  } else {
    h = h0 ? reinterpret_cast<const float4*>(h0)[t] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (; i < nrec; i += NB) {
    float d[NB];
    float4 x[NB];
#pragma unroll
    for (int u = 0; u < NB; ++u) {
      if (i + u < nrec) {
        const int64_t r = rec_of(reverse ? nrec - 1 - (i + u) : i + u);
        d[u] = ws_d[r * KD + key];
        x[u] = *slot_of(r);
      }
    }
#pragma unroll
    for (int u = 0; u < NB; ++u) {
      if (i + u < nrec) {
        const int64_t r = rec_of(reverse ? nrec - 1 - (i + u) : i + u);
        h = make_float4(fmaf(d[u], h.x, x[u].x), fmaf(d[u], h.y, x[u].y), fmaf(d[u], h.z, x[u].z),
                        fmaf(d[u], h.w, x[u].w));
        *slot_of(r) = h;
      }
    }
  }
}

}  // namespace gla
}  // namespace gl

#include <cmath>
#include <cstdlib>
#include <mutex>

#include "tmap.h"

// Sequence split for few (batch, head) pairs with long sequences: how many
// segments the launcher uses (1 = none).  Each segment keeps at least 8
// chunks, and the full pass puts one CTA on each SM.
static int gla_segments(int64_t B, int64_t T, int64_t H, int num_sms) {
  const int64_t items = B * H, NT = T / 64;
  if (const char* e = std::getenv("GLAUCIS_GLA_SEGMENTS")) {
    const int64_t n = std::atoi(e);
    return static_cast<int>(n < 1 ? 1 : (n > NT ? NT : n));
  }
  if (items * 2 > num_sms) return 1;
  int64_t n = num_sms / items;
  if (n > NT / 8) n = NT / 8;
  return static_cast<int>(n < 2 ? 1 : n);
}

// Forward sequence split (short first segment, see Params): the first phase
// runs segment 0's full pass beside the state-only pass of segments
// 1..nseg-2, the second the full pass of segments 1..nseg-1, each with
// B*H*(nseg-1) CTAs, so nseg - 1 = #SMs / (B*H) puts one CTA on each SM in
// both; every segment after the first keeps at least 8 chunks.
static int gla_segments_fwd(int64_t B, int64_t T, int64_t H, int num_sms) {
  const int64_t items = B * H, NT = T / 64;
  if (const char* e = std::getenv("GLAUCIS_GLA_SEGMENTS")) {
    const int64_t n = std::atoi(e);
    return static_cast<int>(n < 1 ? 1 : (n > NT ? NT : n));
  }
  if (items * 2 > num_sms) return 1;
  int64_t n = num_sms / items + 1;
  if (n > NT / 8 + 1) n = NT / 8 + 1;
  return static_cast<int>(n < 2 ? 1 : n);
}

// Chunks of segment 0 in the forward split: its full pass should take as
// long as the state-only pass over one of the later segments, which costs
// about 0.52 of a full pass per chunk (measured on gla_b1_t32768).
static int gla_first_segment(int64_t NT, int nseg) {
  const double r = 0.52;
  int64_t c = static_cast<int64_t>(r * static_cast<double>(NT) / (nseg - 1 + r) + 0.5);
  if (c < 1) c = 1;
  if (c > NT - (nseg - 1)) c = NT - (nseg - 1);
  return static_cast<int>(c);
}

// The fold of a split's records (see gla_fold_kernel): pass_first starts
// from record 0 unchanged (forward split with a short first segment).
static int launch_fold(const float* h0, const gl::gla::Params& p, int reverse, int pass_first,
                       cudaStream_t st, const char** why) {
  const int64_t n4 = static_cast<int64_t>(p.B) * p.H * 128 * 32;
  const unsigned grid = static_cast<unsigned>((n4 + 255) / 256);
  const int nrec = p.nseg - 1 - (pass_first ? 1 : 0);
  if (nrec <= 4)
    gl::gla::gla_fold_kernel<4><<<grid, 256, 0, st>>>(h0, p.ws_h, p.ws_d, p.B * p.H, p.nseg, reverse, pass_first);
  else if (nrec <= 8)
    gl::gla::gla_fold_kernel<8><<<grid, 256, 0, st>>>(h0, p.ws_h, p.ws_d, p.B * p.H, p.nseg, reverse, pass_first);
  else
    gl::gla::gla_fold_kernel<16><<<grid, 256, 0, st>>>(h0, p.ws_h, p.ws_d, p.B * p.H, p.nseg, reverse, pass_first);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    *why = cudaGetErrorString(e);
    return -2;
  }
  return 0;
}

// A second stream per device for the first phase of the forward split, and
// the two events that fork it from and join it to the caller's stream.
struct SideStream {
  cudaStream_t s = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
};
static std::mutex g_side_mu;
static SideStream g_side[64];

static int side_stream(SideStream** out, const char** why) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    *why = "cudaGetDevice failed";
    return -2;
  }
  SideStream& d = g_side[dev];
  if (d.s == nullptr) {
    if (cudaStreamCreateWithFlags(&d.s, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&d.fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&d.join, cudaEventDisableTiming) != cudaSuccess) {
      *why = "creating the side stream of the sequence split failed";
      return -2;
    }
  }
  *out = &d;
  return 0;
}

// Workspace of a split launch: final state [B*H][nseg-1][128][128] and total
// decay [B*H][nseg-1][128], fp32, the decays 256-byte aligned after the states.
static size_t gla_ws_bytes(int64_t B, int64_t H, int nseg) {
  if (nseg <= 1) return 0;
  const size_t rec = static_cast<size_t>(B * H) * static_cast<size_t>(nseg - 1);
  const size_t hb = rec * 128 * 128 * 4;
  return ((hb + 255) / 256) * 256 + rec * 128 * 4;
}

template <int VS, int kMode, bool kSplit = false, bool kScatter = false>
static int launch_pass(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                       const CUtensorMap& tg, const CUtensorMap& th, const gl::gla::OutMaps& to,
                       const gl::gla::Params& p, int grid, cudaStream_t st, const char** why) {
  if constexpr (kMode == gl::gla::MODE_FWD && !kSplit && !kScatter) {
    if (p.p_split) return launch_pass<VS, kMode, true>(tq, tk, tv, tg, th, to, p, grid, st, why);
  }
  if constexpr (kMode == gl::gla::MODE_FWD && VS == 128 && !kScatter) {
    if (p.n_outs > 1) return launch_pass<VS, kMode, kSplit, true>(tq, tk, tv, tg, th, to, p, grid, st, why);
  }
  using CF = gl::gla::Cfg<VS, kSplit, kMode == gl::gla::MODE_FWD>;
  const void* fn = reinterpret_cast<const void*>(gl::gla::chunk_gla_fwd_kernel<VS, kMode, kSplit, kScatter>);
  if (!gl_set_smem_attr(fn, 0, static_cast<int>(CF::SMEM_BYTES), why)) return -2;
  gl::gla::chunk_gla_fwd_kernel<VS, kMode, kSplit, kScatter><<<grid, gl::gla::NUM_THREADS, CF::SMEM_BYTES, st>>>(
      tq, tk, tv, tg, th, to, p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    *why = cudaGetErrorString(e);
    return -2;
  }
  return 0;
}

// One forward (rev = false: q, k slot = k, v slot = v, state output h_n) or
// reverse state-gradient scan (rev = true: k slot = q, v slot = do, state
// output E_n), with the state-only pre-pass and the fold of a sequence split.
template <int VS>
static int launch_vs(const void* q, const void* kslot, const void* vslot, const float* g,
                     void* sout, void* const* outs, gl::gla::Params p, bool rev, cudaStream_t st,
                     const char** why) {
  const int64_t BT = static_cast<int64_t>(p.B) * p.T;
  CUtensorMap tq, tk, tv, tg, th;
  if (!gl_make_tmap_3d(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, kslot, 128, p.H, BT, 128,
                       static_cast<int64_t>(p.H) * 128, 64, 1, 64, CU_TENSOR_MAP_SWIZZLE_128B, why))
    return -1;
  if (!gl_make_tmap_3d(&tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, vslot, 128, p.H, BT, 128,
                       static_cast<int64_t>(p.H) * 128, 64, 1, 64, CU_TENSOR_MAP_SWIZZLE_128B, why))
    return -1;
  if (q) {
    if (!gl_make_tmap_3d(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, q, 128, p.H, BT, 128,
                         static_cast<int64_t>(p.H) * 128, 64, 1, 64, CU_TENSOR_MAP_SWIZZLE_128B,
                         why))
      return -1;
  } else {
    tq = tk;  // the reverse scan reads q through the k slot only
  }
  if (g) {
    if (!gl_make_tmap_3d(&tg, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, g, 128, p.H, BT, 128,
                         static_cast<int64_t>(p.H) * 128, 128, 1, 64, CU_TENSOR_MAP_SWIZZLE_NONE,
                         why))
      return -1;
  } else {
    tg = tk;  // unused when the per-head gate is given
  }
  if (sout) {
    // [B, NT, H, 128 keys, 128] bf16 as 2-D rows of 128, boxes of 64 x 128.
    if (!gl_make_tmap_2d(&th, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, sout, 128, BT / 64 * p.H * 128, 128,
                         64, 128, CU_TENSOR_MAP_SWIZZLE_128B, why))
      return -1;
  } else {
    th = tk;  // unused
  }
  gl::gla::OutMaps to;
  if (!rev && VS == 128 && p.o != nullptr) {
    // each output [B*T, H, 128] bf16, boxes of 64 columns x 1 head x 16
    // rows: one gating warp's share of a chunk's O
    for (int i = 0; i < p.n_outs; ++i)
      if (!gl_make_tmap_3d(&to.m[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, outs[i], 128, p.H, BT, 128,
                           static_cast<int64_t>(p.H) * 128, 64, 1, 16, CU_TENSOR_MAP_SWIZZLE_128B,
                           why))
        return -1;
  } else if (p.n_outs > 1) {
    *why = "several outputs need the full-width (VS = 128) forward: pass a workspace";
    return -1;
  }
  for (int i = (!rev && VS == 128 && p.o != nullptr) ? p.n_outs : 0; i < gl::gla::MAX_OUTS; ++i)
    to.m[i] = tk;  // unused
  const int items = p.B * p.H * p.nsplit;
  if (p.nseg > 1 && !rev && p.c_first > 0) {
    // Phase 1: segment 0's full pass (from h0; its final state becomes
    // record 0) on the caller's stream, beside the state-only pass of
    // segments 1..nseg-2 on the side stream.  Then the fold and the full
    // pass of segments 1..nseg-1.
    gl::gla::Params pa = p;
    pa.seg_base = 0;
    pa.seg_grid = 1;
    pa.ht = p.ws_h;  // record 0 = [B*H][K][V], the layout of ht
    pa.ht_seg = 0;
    pa.has_hout = sout != nullptr;
    {
      std::lock_guard<std::mutex> lk(g_side_mu);
      SideStream* ss = nullptr;
      if (p.nseg > 2) {
        if (int rc = side_stream(&ss, why)) return rc;
        if (cudaEventRecord(ss->fork, st) != cudaSuccess || cudaStreamWaitEvent(ss->s, ss->fork, 0) != cudaSuccess) {
          *why = "forking the side stream failed";
          return -2;
        }
        gl::gla::Params ps = p;
        ps.seg_base = 1;
        ps.seg_grid = p.nseg - 2;
        ps.rec_base = 0;
        ps.has_hout = 0;
        if (int rc = launch_pass<VS, gl::gla::MODE_FWD_STATE>(tq, tk, tv, tg, th, to, ps, items * ps.seg_grid,
                                                              ss->s, why))
          return rc;
      }
      const int rc_a = launch_pass<VS, gl::gla::MODE_FWD>(tq, tk, tv, tg, th, to, pa, items, st, why);
      // join even when that launch failed, so that nothing of this call runs
      // on the side stream after the caller's stream has moved on
      if (ss != nullptr &&
          (cudaEventRecord(ss->join, ss->s) != cudaSuccess || cudaStreamWaitEvent(st, ss->join, 0) != cudaSuccess)) {
        *why = "joining the side stream failed";
        return -2;
      }
      if (rc_a) return rc_a;
    }
    // Record 0 already holds the true state after segment 0: the fold
    // starts from it and leaves it unchanged.
    if (int rc = launch_fold(nullptr, p, 0, 1, st, why)) return rc;
    p.seg_base = 1;
    p.seg_grid = p.nseg - 1;
    p.ht_seg = p.nseg - 1;
    p.has_hout = sout != nullptr;
    return launch_pass<VS, gl::gla::MODE_FWD>(tq, tk, tv, tg, th, to, p, items * p.seg_grid, st, why);
  }
  if (p.nseg > 1) {
    // State-only pass over segments 0 .. nseg-2 (reverse: 1 .. nseg-1), the
    // fold, then the full pass.
    gl::gla::Params p1 = p;
    p1.seg_grid = p.nseg - 1;
    p1.seg_base = rev ? 1 : 0;
    p1.rec_base = p1.seg_base;
    p1.has_hout = 0;
    const int rc = rev ? launch_pass<VS, gl::gla::MODE_DH_STATE>(tq, tk, tv, tg, th, to, p1,
                                                                 items * p1.seg_grid, st, why)
                       : launch_pass<VS, gl::gla::MODE_FWD_STATE>(tq, tk, tv, tg, th, to, p1,
                                                                  items * p1.seg_grid, st, why);
    if (rc) return rc;
    if (int rc2 = launch_fold(p.h0, p, rev ? 1 : 0, 0, st, why)) return rc2;
  }
  p.seg_grid = p.nseg;
  p.seg_base = 0;
  p.ht_seg = rev ? 0 : p.nseg - 1;
  p.has_hout = sout != nullptr;
  return rev ? launch_pass<VS, gl::gla::MODE_DH>(tq, tk, tv, tg, th, to, p, items * p.nseg, st, why)
             : launch_pass<VS, gl::gla::MODE_FWD>(tq, tk, tv, tg, th, to, p, items * p.nseg, st, why);
}

size_t gl_chunk_gla_ws_bytes(int64_t B, int64_t T, int64_t H, int num_sms) {
  const size_t f = gla_ws_bytes(B, H, gla_segments_fwd(B, T, H, num_sms));
  const size_t r = gla_ws_bytes(B, H, gla_segments(B, T, H, num_sms));
  return f > r ? f : r;
}

// Shared set-up of the forward and the reverse scan: scale, segments, V split.
static int gla_dispatch(const void* q, const void* kslot, const void* vslot, const float* g,
                        const float* g_gamma, const float* init, float scale, int64_t B,
                        int64_t T, int64_t H, void* const* outs, int n_outs, float* fin, void* sout,
                        void* ws, size_t ws_bytes, int* err, bool rev, int p_split, cudaStream_t st,
                        int num_sms, const char** why) {
  gl::gla::Params p;
  p.p_split = rev ? 0 : p_split;
  p.g_gamma = g_gamma;
  p.h0 = init;
  p.o = n_outs > 0 ? static_cast<__nv_bfloat16*>(outs[0]) : nullptr;
  p.n_outs = n_outs > 0 ? n_outs : 1;
  p.ht = fin;
  p.err = err;
  p.scale = scale;
  p.scale_apart = !(scale > 0.f && std::isfinite(scale));
  p.log2_scale = p.scale_apart ? 0.f : static_cast<float>(std::log2(static_cast<double>(scale)));
  p.B = static_cast<int>(B);
  p.T = static_cast<int>(T);
  p.H = static_cast<int>(H);
  p.has_g = g != nullptr;
  p.seg_base = 0;
  p.rec_base = 0;
  p.ht_seg = 0;
  p.has_hout = 0;
  // Few (batch, head) pairs: split the sequence into segments (full V width,
  // one CTA per SM) when the workspace allows it, else split V in two.
  // GLAUCIS_GLA_VS=64|128 and GLAUCIS_GLA_SEGMENTS=n override the choice.
  int nseg = rev ? gla_segments(B, T, H, num_sms) : gla_segments_fwd(B, T, H, num_sms);
  while (nseg > 1 && (ws == nullptr || gla_ws_bytes(B, H, nseg) > ws_bytes)) --nseg;
  p.nseg = nseg;
  p.c_first = (!rev && nseg > 1) ? gla_first_segment(T / 64, nseg) : 0;
  p.seg_grid = nseg;
  if (nseg > 1) {
    const size_t rec = static_cast<size_t>(B * H) * static_cast<size_t>(nseg - 1);
    p.ws_h = static_cast<float*>(ws);
    p.ws_d = reinterpret_cast<float*>(static_cast<char*>(ws) + ((rec * 128 * 128 * 4 + 255) / 256) * 256);
  } else {
    p.ws_h = p.ws_d = nullptr;
  }
  bool split_v = nseg == 1 && B * H * 2 <= num_sms;
  if (const char* e = std::getenv("GLAUCIS_GLA_VS")) split_v = std::atoi(e) == 64;
  if (split_v) {
    p.nsplit = 2;
    return launch_vs<64>(q, kslot, vslot, g, sout, outs, p, rev, st, why);
  }
  p.nsplit = 1;
  return launch_vs<128>(q, kslot, vslot, g, sout, outs, p, rev, st, why);
}

int gl_launch_chunk_gla(const void* q, const void* k, const void* v, const float* g,
                        const float* g_gamma, const float* h0, float scale, int64_t B, int64_t T,
                        int64_t H, int64_t K, int64_t V, void* o, float* ht, void* h_out, void* ws,
                        size_t ws_bytes, int p_split, int* err, cudaStream_t st, int num_sms,
                        const char** why) {
  (void)K;
  (void)V;
  void* outs[1] = {o};
  return gla_dispatch(q, k, v, g, g_gamma, h0, scale, B, T, H, outs, 1, ht, h_out, ws, ws_bytes,
                      err, false, p_split, st, num_sms, why);
}

// The forward with O stored into n_outs buffers of o's layout (see
// gl_chunk_gla_fwd_scatter).
int gl_launch_chunk_gla_scatter(const void* q, const void* k, const void* v, const float* g,
                                const float* g_gamma, const float* h0, float scale, int64_t B,
                                int64_t T, int64_t H, void* const* outs, int n_outs, float* ht,
                                void* ws, size_t ws_bytes, int p_split, int* err, cudaStream_t st,
                                int num_sms, const char** why) {
  return gla_dispatch(q, k, v, g, g_gamma, h0, scale, B, T, H, outs, n_outs, ht, nullptr, ws,
                      ws_bytes, err, false, p_split, st, num_sms, why);
}

// Reverse state-gradient scan of the backward: E_n (bf16 [B,NT,H,K,V]) for
// every chunk and dh0 (fp32, nullable) from q, do, the gate and dht.
int gl_launch_chunk_gla_dh(const void* q, const void* dout, const float* g, const float* g_gamma,
                           const float* dht, float scale, int64_t B, int64_t T, int64_t H,
                           void* e_out, float* dh0, void* ws, size_t ws_bytes, int* err,
                           cudaStream_t st, int num_sms, const char** why) {
  return gla_dispatch(nullptr, q, dout, g, g_gamma, dht, scale, B, T, H, nullptr, 0, dh0, e_out, ws,
                      ws_bytes, err, true, 0, st, num_sms, why);
}
