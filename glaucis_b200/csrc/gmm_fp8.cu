// Grouped (ragged) FP8 matmul forward with block-wise fp32 scales, sm_100a.
//
//   out[m, n] = sum_kb a_s[m, kb] * b_s[g, kb, n/128] * (a_q[m, kb-block] . b_q[g, kb-block, n])
//
// Replaces the tokamax Pallas TPU `gmm` call made by the Glaucis template
// (KE/examples/kernels/gmm_fp8_blockwise.py:109-119).
//
// Design (one persistent CTA per SM, 384 threads, warp specialised; the tile
// is 128 rows x BN columns with BN = 128 or 256):
//   warp 0      TMA producer: per 128-deep K block loads the 128x128 e4m3
//               activation tile (K-major) and the 128xBN e4m3 weight tile
//               (N-major, 128-byte-wide boxes) into a STAGES-deep ring.
//   warp 1      MMA issuer: 4 x tcgen05.mma.kind::f8f6f4 (128xBNx32) per K
//               block into one of 512/BN TMEM accumulators; with BN = 128 the
//               MMA runs up to three K blocks ahead of the promotion.
//   warp 3      derives the ragged tile table from group_sizes.
//   warps 4-11  promotion + epilogue (two warpgroups, BN/2 columns each):
//               after every K block each thread reads its row's columns of
//               the partial sum out of TMEM (32-column loads, two in flight)
//               and accumulates partial * (a_s * b_s) in fp32 registers with
//               packed f32x2 FMAs, releasing the TMEM buffer so later K
//               blocks' MMAs overlap the promotion.  The finished row is
//               written as bf16 (or fp32).
//   Registers: the control warpgroup drops to 56 per thread and the two
//   promotion warpgroups rise to 224 (128 x 56 + 256 x 224 = 384 x 168, the
//   launch allocation).
// Ragged groups: tiles never straddle a group; M tiles start at each group's
// row offset, the last tile of a group is partial and its foreign rows are
// computed but never stored.  The tile list (group-major, N outer, M inner so
// CTAs running together share weight tiles in L2) is derived on the device
// from group_sizes; no host synchronisation.
#include "common.cuh"

namespace gl {
namespace gmm {

constexpr int BM = 128, BK = 128;
constexpr int A_BYTES = BM * BK;  // 16 KB
constexpr int NUM_THREADS = 384;
constexpr int REG_CTRL = 56, REG_EPI = 224;
static_assert(128 * REG_CTRL + 256 * REG_EPI <= NUM_THREADS * 168, "register split exceeds the launch allocation");
constexpr int MAX_G = 1024;
constexpr int TMEM_COLS = 512;

template <int BN, bool kStg = false>
struct Cfg {
  static constexpr int B_BYTES = BK * BN;                      // 16 / 32 KB
  // kStg (BN = 256): the bf16 output is staged through shared memory (one
  // 8 KB slot per promotion warp: 32 rows x 128 columns as two 128B-swizzled
  // 32x64 boxes) and TMA-stored, so the epilogue does not hold up the next
  // tile's MMAs; the slots take the room of one operand stage.  Used for
  // every bf16 output: the direct 16-byte stores of a 32-row slice go to 32
  // rows N apart, ~4k separate L2 writes per SM and tile, which held the
  // next tile's MMAs back (gmm_dense_expert 4.24 -> 3.98 ms staged; the
  // fourth operand stage it gives up is worth nothing measurable).
  static constexpr bool STG = kStg && BN == 256;
  static constexpr int STG_BYTES = STG ? 8 * 8192 : 0;
  static constexpr int STAGES = STG ? 3
                                    : ((6 * 32768) / (A_BYTES + B_BYTES) < 6
                                           ? (6 * 32768) / (A_BYTES + B_BYTES) : 6);  // 3 / 6
  static constexpr int NBUF = TMEM_COLS / BN;                  // TMEM accumulators: 2 / 4
  static constexpr int EC = BN / 2;                            // columns per promotion thread
  static constexpr int NCH = EC / 32;                          // 32-column TMEM loads per K block
  static_assert(NCH % 2 == 0, "TMEM loads go in pairs");
  static constexpr uint32_t OFF_A = 0;
  static constexpr uint32_t OFF_B = OFF_A + STAGES * A_BYTES;
  static constexpr uint32_t OFF_STG = OFF_B + STAGES * B_BYTES;  // 1 KB aligned
  static constexpr uint32_t OFF_BAR = OFF_STG + STG_BYTES;
  static constexpr uint32_t OFF_MISC = OFF_BAR + 256;
  static constexpr uint32_t OFF_ROWOFF = OFF_MISC + 128;
  static constexpr uint32_t OFF_TILEOFF = OFF_ROWOFF + (MAX_G + 1) * 4;
  static constexpr uint32_t SMEM_USED = OFF_TILEOFF + (MAX_G + 1) * 4;
  static constexpr uint32_t SMEM_BYTES = SMEM_USED + 1024;     // slack for 1 KB alignment
  static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
  // e4m3 x e4m3 -> f32, A K-major, B MN-major, M=128, N=BN.
  static constexpr uint32_t IDESC = idesc(1, 0, 0, 0, 1, BM, BN);
  // transposed weight (backward dlhs): B K-major (rows = output columns)
  static constexpr uint32_t IDESC_T = idesc(1, 0, 0, 0, 0, BM, BN);
  static_assert(2 * STAGES + 2 * NBUF + 1 <= 32, "barrier area");
};

constexpr int MAX_OUTS = 8;

struct Params {
  const float* a_s;
  const float* b_s;
  const int32_t* group_sizes;
  void* out;
  int* err;
  int G, M, K, N;
  int out_f32;
  // Output copies (single-CTA kernel): row m of this call is stored as row
  // row_off + m of every outs[0 .. n_outs-1] (device or peer-mapped buffers
  // of at least row_off + M rows of N); outs[0] = out, n_outs = 1,
  // row_off = 0 for a plain call.
  void* outs[MAX_OUTS];
  int n_outs;
  int64_t row_off;
  // 1: the outputs are bf16 and tm_o.m[o] maps outs[o] (rows row_off + M,
  // box 32 rows x 64 columns, 128B swizzle): whole 32-row slices of a tile
  // leave through shared memory and TMA stores, one pair per output (own or
  // peer-mapped memory; BN = 256 with the staged configuration only).
  int tma_out;
};

// Tensor maps of the outputs (kernel parameter).
struct OutMaps {
  CUtensorMap m[MAX_OUTS];
};

struct Tile {
  int g, m0, rows, n0;
};

__device__ __forceinline__ Tile decode_tile(int t, const int* tile_off, const int* row_off, int G,
                                            int bn, int bm = BM) {
  int lo = 0, hi = G - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (tile_off[mid] <= t) lo = mid; else hi = mid - 1;
  }
  Tile r;
  r.g = lo;
  const int local = t - tile_off[lo];
  const int size = row_off[lo + 1] - row_off[lo];
  const int mt = (size + bm - 1) / bm;
  const int i = local % mt, j = local / mt;
  r.m0 = row_off[lo] + i * bm;
  r.rows = min(bm, size - i * bm);
  r.n0 = j * bn;
  return r;
}

// Warp-scan of group_sizes into exclusive row / tile prefix sums (tiles of
// `bm` rows x `bn` columns).  Whole warp.  Returns nothing; writes the tables
// and the validated tile total into shared memory.
__device__ __forceinline__ void build_group_table(const int32_t* group_sizes, int G, int M, int bm,
                                                  int ntn, int* row_off, int* tile_off,
                                                  int* total_tiles, int* err, int lane) {
  const int per = (G + 31) / 32;
  const int g0 = min(G, lane * per), g1 = min(G, g0 + per);
  int rsum = 0, tsum = 0, bad = 0;
  for (int g = g0; g < g1; ++g) {
    const int sz = group_sizes[g];
    bad |= sz < 0;
    const int s = max(sz, 0);
    rsum += s;
    tsum += (s + bm - 1) / bm * ntn;
  }
  int rinc = rsum, tinc = tsum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int rv = __shfl_up_sync(0xffffffffu, rinc, o);
    const int tv = __shfl_up_sync(0xffffffffu, tinc, o);
    if (lane >= o) {
      rinc += rv;
      tinc += tv;
    }
  }
  int r = rinc - rsum, tt = tinc - tsum;
  for (int g = g0; g < g1; ++g) {
    const int s = max(group_sizes[g], 0);
    row_off[g] = r;
    tile_off[g] = tt;
    r += s;
    tt += (s + bm - 1) / bm * ntn;
  }
  bad = __any_sync(0xffffffffu, bad);
  if (lane == 31) {
    row_off[G] = rinc;
    tile_off[G] = tinc;
    const bool ok = !bad && rinc <= M;
    *total_tiles = ok ? tinc : 0;
    if (!ok) atomicExch(err, GL_DEV_BAD_GROUPS);
  }
}

template <int BN, bool kTransB, bool kStg>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gmm_fp8_fwd_kernel(const __grid_constant__ CUtensorMap tm_a,
                       const __grid_constant__ CUtensorMap tm_b,
                       const __grid_constant__ OutMaps tm_o, const Params p) {
  using CF = Cfg<BN, kStg>;
  constexpr int STAGES = CF::STAGES, NBUF = CF::NBUF, EC = CF::EC, NCH = CF::NCH;
  extern __shared__ uint8_t smem_raw[];
  // 1 KB-aligned base derived by pointer arithmetic on the shared array so
  // that every access below stays in the shared address space.
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + CF::OFF_BAR);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + NBUF;
  uint64_t* drain = tempty + NBUF;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + CF::OFF_MISC);
  int* abort_flag = reinterpret_cast<int*>(smem + CF::OFF_MISC + 4);
  int* total_tiles_s = reinterpret_cast<int*>(smem + CF::OFF_MISC + 8);
  int* row_off = reinterpret_cast<int*>(smem + CF::OFF_ROWOFF);
  int* tile_off = reinterpret_cast<int*>(smem + CF::OFF_TILEOFF);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.G, K = p.K, N = p.N;
  const int KB = K / BK, NB = N / 128;
  const int ntn = (N + BN - 1) / BN;
  const Abort ab{abort_flag, p.err};

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tm_a);
      prefetch_tmap(&tm_b);
    }
    tmem_alloc(tmem_holder, TMEM_COLS);
    tmem_relinquish();
  } else if (warp == 1) {
    if (lane == 0) {
      for (int i = 0; i < STAGES; ++i) {
        mbar_init(&full[i], 1);
        mbar_init(&empty[i], 1);
      }
      for (int i = 0; i < NBUF; ++i) {
        mbar_init(&tfull[i], 1);
        mbar_init(&tempty[i], 8);  // one arrival per promotion warp
      }
      mbar_init(drain, 1);
      *abort_flag = 0;
      fence_mbar_init();
    }
  } else if (warp == 3) {
    build_group_table(p.group_sizes, G, p.M, BM, ntn, row_off, tile_off, total_tiles_s, p.err, lane);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const int total = *total_tiles_s;

  if (warp == 0) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_CTRL));
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        const Tile tl = decode_tile(t, tile_off, row_off, G, BN);
        const int brow = tl.g * K;
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, ab)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[s], A_BYTES + CF::B_BYTES);
          uint8_t* sa = smem + CF::OFF_A + s * A_BYTES;
          uint8_t* sb = smem + CF::OFF_B + s * CF::B_BYTES;
          tma_load_2d(sa, &tm_a, &full[s], kb * BK, tl.m0);
#pragma unroll
          for (int j = 0; j < BN / 128; ++j) {
            if (kTransB)  // rows = output columns of weight group g, 128 reduction bytes each
              tma_load_2d(sb + j * 16384, &tm_b, &full[s], kb * BK, tl.g * N + tl.n0 + 128 * j);
            else          // rows = reduction index, 128 output columns each
              tma_load_2d(sb + j * 16384, &tm_b, &full[s], tl.n0 + 128 * j, brow + kb * BK);
          }
        }
      }
      if (!ok) {
        // Let copies already in flight land before the CTA exits.
        const int first = it > STAGES ? it - STAGES : 0;
        for (int j = first; j < it; ++j) {
          const int s = j % STAGES;
          const uint64_t t0 = global_ns();
          while (!mbar_try_wait(&full[s], (j / STAGES) & 1) && global_ns() - t0 < 100000000ull) {
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_CTRL));
    if (lane == 0) {
      // ------------------------------------------------------------ MMA
      int it = 0, acc_it = 0;
      bool ok = true;
      const uint32_t a_base = smem_u32(smem + CF::OFF_A), b_base = smem_u32(smem + CF::OFF_B);
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        for (int kb = 0; kb < KB; ++kb, ++it, ++acc_it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          const int buf = acc_it % NBUF;
          const uint32_t aph = (acc_it / NBUF) & 1;
          if (!mbar_wait(&tempty[buf], aph ^ 1, ab)) { ok = false; break; }
          if (!mbar_wait(&full[s], ph, ab)) { ok = false; break; }
          tc_fence_after();
          const uint32_t d = tmem + buf * BN;
#pragma unroll
          for (int kk = 0; kk < BK / 32; ++kk) {
            const uint64_t ad = sdesc(a_base + s * A_BYTES + kk * 32, 16, 1024, kSwizzle128B);
            const uint64_t bd =
                kTransB ? sdesc(b_base + s * CF::B_BYTES + kk * 32, 16, 1024, kSwizzle128B)
                        : sdesc(b_base + s * CF::B_BYTES + kk * 4096, 16384, 1024, kSwizzle128B);
            mma_f8f6f4(d, ad, bd, kTransB ? CF::IDESC_T : CF::IDESC, kk > 0 ? 1u : 0u);
          }
          tc_commit(&empty[s]);
          tc_commit(&tfull[buf]);
        }
      }
      // Wait for every MMA issued above before TMEM can be released.
      tc_commit(drain);
      const uint64_t t0 = global_ns();
      while (!mbar_try_wait(drain, 0) && global_ns() - t0 < 100000000ull) {
      }
    }
    __syncwarp();
  } else if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_CTRL));
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REG_EPI));
    // -------------------------------------------------------- epilogue
    const int ew = warp - 4;
    const int quad = warp & 3;
    const int chalf = ew >> 2;
    const int r = quad * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quad * 32) << 16) + chalf * EC;
    int acc_it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
      const Tile tl = decode_tile(t, tile_off, row_off, G, BN);
      const bool row_ok = r < tl.rows;
      const int64_t grow = static_cast<int64_t>(tl.m0) + r;
      const int ncol0 = tl.n0 + chalf * EC;
      const bool col_ok = ncol0 < N;
      const int nb = ncol0 >> 7;
      const float* sa_row = p.a_s + grow * KB;
      // weight scale of (K block kb, output block nb): b_s[g, kb, nb], or for
      // the transposed weight (output = weight rows) b_s[g, nb, kb]
      const int64_t sb_step = kTransB ? 1 : NB;
      const float* sb_col = p.b_s + (kTransB ? (static_cast<int64_t>(tl.g) * NB + nb) * KB
                                             : static_cast<int64_t>(tl.g) * KB * NB + nb);
      float2 acc[EC / 2];
#pragma unroll
      for (int j = 0; j < EC / 2; ++j) acc[j] = make_float2(0.f, 0.f);
      float sa_next = row_ok ? __ldg(sa_row) : 0.f;
      float sb_next = col_ok ? __ldg(sb_col) : 0.f;
      for (int kb = 0; kb < KB; ++kb, ++acc_it) {
        const float sc = sa_next * sb_next;
        if (kb + 1 < KB) {
          sa_next = row_ok ? __ldg(sa_row + kb + 1) : 0.f;
          sb_next = col_ok ? __ldg(sb_col + static_cast<int64_t>(kb + 1) * sb_step) : 0.f;
        }
        const float2 sc2 = make_float2(sc, sc);
        const int buf = acc_it % NBUF;
        if (!mbar_wait(&tfull[buf], (acc_it / NBUF) & 1, ab)) { ok = false; break; }
        tc_fence_after();
        const uint32_t ta = lane_base + buf * BN;
        uint32_t v[2][32];
        auto promote = [&](const uint32_t (&x)[32], int base) {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            acc[base + j] = __ffma2_rn(make_float2(__uint_as_float(x[2 * j]), __uint_as_float(x[2 * j + 1])),
                                       sc2, acc[base + j]);
        };
        // Chunks are loaded two at a time; the next pair's loads are issued
        // between the promotions of the current pair, and the accumulator is
        // released as soon as the last pair has landed (the last two
        // promotions run after the release).
        tmem_ld32(ta, v[0]);
        tmem_ld32(ta + 32, v[1]);
        tmem_ld_wait2(v[0], v[1]);
#pragma unroll
        for (int c = 2; c < NCH; c += 2) {
          promote(v[0], 16 * (c - 2));
          tmem_ld32(ta + 32 * c, v[0]);
          promote(v[1], 16 * (c - 1));
          tmem_ld32(ta + 32 * (c + 1), v[1]);
          tmem_ld_wait2(v[0], v[1]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[buf]);
        promote(v[0], 16 * (NCH - 2));
        promote(v[1], 16 * (NCH - 1));
      }
      if (!ok) break;
      bool staged = false;
      if constexpr (CF::STG) {
        // The tile is decoded again (from shared memory) rather than kept
        // live across the K loop, which leaves the promotion its registers.
        const Tile te = decode_tile(t, tile_off, row_off, G, BN);
        const int ecol0 = te.n0 + chalf * EC;
        if (p.tma_out && ecol0 < N && te.rows - quad * 32 >= 32) {
          // this warp's 32 rows x 128 columns -> its slot as two swizzled
          // 32x64 boxes -> two TMA stores
          uint8_t* slot = smem + CF::OFF_STG + ew * 8192;
          const uint32_t srow = smem_u32(slot) + lane * 128;
          if (lane == 0) bulk_wait_read<0>();  // the previous tile's stores have read the slot
          __syncwarp();
#pragma unroll
          for (int b = 0; b < 2; ++b)
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              const int j = b * 32 + c * 4;  // acc[j] = columns 2j, 2j+1 of this thread's range
              st_shared_v4(srow + b * 4096 + ((c ^ (lane & 7)) << 4),
                           pack_bf16x2(acc[j].x, acc[j].y), pack_bf16x2(acc[j + 1].x, acc[j + 1].y),
                           pack_bf16x2(acc[j + 2].x, acc[j + 2].y), pack_bf16x2(acc[j + 3].x, acc[j + 3].y));
            }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            const int y = static_cast<int>(p.row_off) + te.m0 + quad * 32;
            for (int o = 0; o < p.n_outs; ++o) {
              tma_store_2d(&tm_o.m[o], slot, ecol0, y);
              tma_store_2d(&tm_o.m[o], slot + 4096, ecol0 + 64, y);
            }
            bulk_commit();
          }
          staged = true;
        }
      }
      if (!staged && row_ok && col_ok) {
        const int64_t orow = p.row_off + grow;
        for (int o = 0; o < p.n_outs; ++o) {
          if (p.out_f32) {
            float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.outs[o]) + orow * N + ncol0);
#pragma unroll
            for (int i = 0; i < EC / 4; ++i)
              dst[i] = make_float4(acc[2 * i].x, acc[2 * i].y, acc[2 * i + 1].x, acc[2 * i + 1].y);
          } else {
            uint4* dst =
                reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.outs[o]) + orow * N + ncol0);
#pragma unroll
            for (int i = 0; i < EC / 8; ++i)
              dst[i] = make_uint4(pack_bf16x2(acc[4 * i].x, acc[4 * i].y),
                                  pack_bf16x2(acc[4 * i + 1].x, acc[4 * i + 1].y),
                                  pack_bf16x2(acc[4 * i + 2].x, acc[4 * i + 2].y),
                                  pack_bf16x2(acc[4 * i + 3].x, acc[4 * i + 3].y));
          }
        }
      }
    }
    if constexpr (CF::STG) {
      if (lane == 0) bulk_wait<0>();  // the TMA stores are done before the CTA exits
      __syncwarp();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ===========================================================================
// CTA-pair variant: a cluster of two CTAs (two SMs) computes a 256 x 256
// tile with tcgen05.mma.cta_group::2 (M=256 across the pair, N=256).  Each
// CTA TMA-loads its own 128 activation rows and its 128-column half of the
// weight tile (no multicast); the loads of both CTAs complete on the leader
// CTA's stage barrier, only the leader issues MMAs and its commits arrive on
// both CTAs' barriers; each CTA promotes its own 128 x 256 accumulator and
// releases it on the leader's barrier.  Per SM and K block this moves 32 KB
// instead of 48 KB into shared memory for the same MMA work.
// ===========================================================================
constexpr int PM = 256;                 // rows per pair tile
constexpr int PAIR_STAGES = 6;
constexpr int PB_BYTES = BK * 128;      // each CTA's half of the weight tile (16 KB)
constexpr uint32_t P_OFF_A = 0;
constexpr uint32_t P_OFF_B = P_OFF_A + PAIR_STAGES * A_BYTES;
constexpr uint32_t P_OFF_BAR = P_OFF_B + PAIR_STAGES * PB_BYTES;
constexpr uint32_t P_OFF_MISC = P_OFF_BAR + 256;
constexpr uint32_t P_OFF_ROWOFF = P_OFF_MISC + 128;
constexpr uint32_t P_OFF_TILEOFF = P_OFF_ROWOFF + (MAX_G + 1) * 4;
constexpr uint32_t P_SMEM_BYTES = P_OFF_TILEOFF + (MAX_G + 1) * 4 + 1024;
constexpr uint32_t P_IDESC = idesc(1, 0, 0, 0, 1, PM, 256);

__global__ void __launch_bounds__(NUM_THREADS, 1)
    gmm_fp8_fwd_pair_kernel(const __grid_constant__ CUtensorMap tm_a,
                            const __grid_constant__ CUtensorMap tm_b, const Params p) {
  constexpr int STAGES = PAIR_STAGES, NBUF = 2, BN = 256, EC = 128, NCH = 4;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + P_OFF_BAR);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + NBUF;
  uint64_t* drain = tempty + NBUF;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + P_OFF_MISC);
  int* abort_flag = reinterpret_cast<int*>(smem + P_OFF_MISC + 4);
  int* total_tiles_s = reinterpret_cast<int*>(smem + P_OFF_MISC + 8);
  int* row_off = reinterpret_cast<int*>(smem + P_OFF_ROWOFF);
  int* tile_off = reinterpret_cast<int*>(smem + P_OFF_TILEOFF);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cid = static_cast<int>(cluster_id_x()), ncl = static_cast<int>(num_clusters_x());
  const int G = p.G, K = p.K, N = p.N;
  const int KB = K / BK, NB = N / 128;
  const int ntn = (N + BN - 1) / BN;
  const Abort ab{abort_flag, p.err};

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tm_a);
      prefetch_tmap(&tm_b);
    }
    tmem_alloc_pair(tmem_holder, TMEM_COLS);
    tmem_relinquish_pair();
  } else if (warp == 1) {
    if (lane == 0) {
      for (int i = 0; i < STAGES; ++i) {
        mbar_init(&full[i], 2);    // one arrive.expect_tx per CTA of the pair
        mbar_init(&empty[i], 1);
      }
      for (int i = 0; i < NBUF; ++i) {
        mbar_init(&tfull[i], 1);
        mbar_init(&tempty[i], 16);  // promotion warps of both CTAs
      }
      mbar_init(drain, 1);
      *abort_flag = 0;
      fence_mbar_init();
    }
  } else if (warp == 3) {
    build_group_table(p.group_sizes, G, p.M, PM, ntn, row_off, tile_off, total_tiles_s, p.err, lane);
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const int total = *total_tiles_s;

  if (warp == 0) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_CTRL));
    if (lane == 0) {
      // ------------------------------------------------- producer (both CTAs)
      int it = 0;
      bool ok = true;
      for (int t = cid; t < total && ok; t += ncl) {
        const Tile tl = decode_tile(t, tile_off, row_off, G, BN, PM);
        const int brow = tl.g * K;
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, ab)) { ok = false; break; }
          const uint32_t fbar = mapa_shared(smem_u32(&full[s]), 0);
          mbar_arrive_expect_tx_cluster(fbar, A_BYTES + PB_BYTES);
          tma_load_2d_pair(smem + P_OFF_A + s * A_BYTES, &tm_a, fbar, kb * BK,
                           tl.m0 + 128 * static_cast<int>(rank));
          tma_load_2d_pair(smem + P_OFF_B + s * PB_BYTES, &tm_b, fbar,
                           tl.n0 + 128 * static_cast<int>(rank), brow + kb * BK);
        }
      }
      if (!ok) {
        // Give copies already in flight time to land before the CTA exits.
        const uint64_t t0 = global_ns();
        while (global_ns() - t0 < 2000000ull) {
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_CTRL));
    if (lane == 0 && leader) {
      // ------------------------------------------------- MMA (leader CTA)
      int it = 0, acc_it = 0;
      bool ok = true;
      const uint32_t a_base = smem_u32(smem + P_OFF_A), b_base = smem_u32(smem + P_OFF_B);
      for (int t = cid; t < total && ok; t += ncl) {
        for (int kb = 0; kb < KB; ++kb, ++it, ++acc_it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          const int buf = acc_it % NBUF;
          const uint32_t aph = (acc_it / NBUF) & 1;
          if (!mbar_wait(&tempty[buf], aph ^ 1, ab)) { ok = false; break; }
          if (!mbar_wait(&full[s], ph, ab)) { ok = false; break; }
          tc_fence_after();
          const uint32_t d = tmem + buf * BN;
#pragma unroll
          for (int kk = 0; kk < BK / 32; ++kk) {
            const uint64_t ad = sdesc(a_base + s * A_BYTES + kk * 32, 16, 1024, kSwizzle128B);
            const uint64_t bd = sdesc(b_base + s * PB_BYTES + kk * 4096, 16384, 1024, kSwizzle128B);
            mma_f8f6f4_pair(d, ad, bd, P_IDESC, kk > 0 ? 1u : 0u);
          }
          tc_commit_pair_mc(&empty[s], 0x3);
          tc_commit_pair_mc(&tfull[buf], 0x3);
        }
      }
      // Wait for every MMA issued above before TMEM can be released.
      tc_commit_pair_mc(drain, 0x1);
      const uint64_t t0 = global_ns();
      while (!mbar_try_wait(drain, 0) && global_ns() - t0 < 100000000ull) {
      }
    }
    __syncwarp();
  } else if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_CTRL));
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REG_EPI));
    // ------------------------------------------- promotion (both CTAs)
    const int ew = warp - 4;
    const int quad = warp & 3;
    const int chalf = ew >> 2;
    const int r = quad * 32 + lane;
    const int prow = static_cast<int>(rank) * 128 + r;       // row within the pair tile
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quad * 32) << 16) + chalf * EC;
    const uint32_t tempty_c0 = mapa_shared(smem_u32(&tempty[0]), 0);
    const uint32_t tempty_c1 = mapa_shared(smem_u32(&tempty[1]), 0);
    int acc_it = 0;
    bool ok = true;
    for (int t = cid; t < total && ok; t += ncl) {
      const Tile tl = decode_tile(t, tile_off, row_off, G, BN, PM);
      const bool row_ok = prow < tl.rows;
      const int64_t grow = static_cast<int64_t>(tl.m0) + prow;
      const int ncol0 = tl.n0 + chalf * EC;
      const bool col_ok = ncol0 < N;
      const int nb = ncol0 >> 7;
      const float* sa_row = p.a_s + grow * KB;
      const float* sb_col = p.b_s + static_cast<int64_t>(tl.g) * KB * NB + nb;
      float2 acc[EC / 2];
#pragma unroll
      for (int j = 0; j < EC / 2; ++j) acc[j] = make_float2(0.f, 0.f);
      float sa_next = row_ok ? __ldg(sa_row) : 0.f;
      float sb_next = col_ok ? __ldg(sb_col) : 0.f;
      for (int kb = 0; kb < KB; ++kb, ++acc_it) {
        const float sc = sa_next * sb_next;
        if (kb + 1 < KB) {
          sa_next = row_ok ? __ldg(sa_row + kb + 1) : 0.f;
          sb_next = col_ok ? __ldg(sb_col + static_cast<int64_t>(kb + 1) * NB) : 0.f;
        }
        const float2 sc2 = make_float2(sc, sc);
        const int buf = acc_it % NBUF;
        if (!mbar_wait(&tfull[buf], (acc_it / NBUF) & 1, ab)) { ok = false; break; }
        tc_fence_after();
        const uint32_t ta = lane_base + buf * BN;
        uint32_t v[2][32];
        auto promote = [&](const uint32_t (&x)[32], int base) {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            acc[base + j] = __ffma2_rn(make_float2(__uint_as_float(x[2 * j]), __uint_as_float(x[2 * j + 1])),
                                       sc2, acc[base + j]);
        };
        tmem_ld32(ta, v[0]);
        tmem_ld32(ta + 32, v[1]);
        tmem_ld_wait2(v[0], v[1]);
#pragma unroll
        for (int c = 2; c < NCH; c += 2) {
          promote(v[0], 16 * (c - 2));
          tmem_ld32(ta + 32 * c, v[0]);
          promote(v[1], 16 * (c - 1));
          tmem_ld32(ta + 32 * (c + 1), v[1]);
          tmem_ld_wait2(v[0], v[1]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(buf ? tempty_c1 : tempty_c0);
        promote(v[0], 16 * (NCH - 2));
        promote(v[1], 16 * (NCH - 1));
      }
      if (!ok) break;
      if (row_ok && col_ok) {
        if (p.out_f32) {
          float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + grow * N + ncol0);
#pragma unroll
          for (int i = 0; i < EC / 4; ++i)
            dst[i] = make_float4(acc[2 * i].x, acc[2 * i].y, acc[2 * i + 1].x, acc[2 * i + 1].y);
        } else {
          uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.out) + grow * N + ncol0);
#pragma unroll
          for (int i = 0; i < EC / 8; ++i)
            dst[i] = make_uint4(pack_bf16x2(acc[4 * i].x, acc[4 * i].y),
                                pack_bf16x2(acc[4 * i + 1].x, acc[4 * i + 1].y),
                                pack_bf16x2(acc[4 * i + 2].x, acc[4 * i + 2].y),
                                pack_bf16x2(acc[4 * i + 3].x, acc[4 * i + 3].y));
        }
      }
    }
  }

  // Both CTAs: every MMA of the pair is complete (the leader drained them) and
  // every cross-CTA arrival has been made before TMEM is released.
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, TMEM_COLS);
  }
}

// ===========================================================================
// Backward drhs = lhs^T x dout per group (tokamax tgmm):
//   drhs[g, k, n] = sum over the global 128-row blocks mb touched by group g of
//                   ls[mb, k] * ds[mb, n] * sum_{m in g and mb} lq[m, k] dq[m, n]
// with lhs and dout quantised in 128x1 column blocks (lq [M, K], ls [M/128, K],
// dq [M, N], ds [M/128, N]).  One tile = 128 rows k x 256 columns n of one
// group; the reduction runs over the group's rows one 128-row block at a
// time.  A = lq^T (k contiguous: MN-major), B = dq (n contiguous: MN-major);
// rows of a partial block that belong to other groups are zeroed in the A
// tile before its MMAs.  Empty groups get zero tiles.  Same warp roles,
// pipeline and bounded waits as the forward kernel.
// ===========================================================================
struct TParams {
  const float* ls;
  const float* ds;
  const int32_t* group_sizes;
  void* out;
  int* err;
  int G, M, K, N;
  int out_f32;
};

constexpr int T_STAGES = 3;
constexpr uint32_t T_A_BYTES = 128 * 128;  // lq block: 128 rows m x 128 bytes k
constexpr uint32_t T_B_BYTES = 128 * 256;  // dq block: 128 rows m x 256 bytes n
constexpr uint32_t T_OUT_BYTES = 128 * 256 * 2;  // bf16 output tile: 4 atoms of 64 columns
constexpr uint32_t T_OFF_A = 0;
constexpr uint32_t T_OFF_B = T_OFF_A + T_STAGES * T_A_BYTES;
constexpr uint32_t T_OFF_OUT = T_OFF_B + T_STAGES * T_B_BYTES;
// Scale ring: per row block, ls[mb, k0 .. k0+127] (512 B) then ds[mb, n0 .. n0+255] (1 KB),
// bulk-copied by the producer next to the operand tiles and released by the epilogue.
constexpr int T_SC_SLOTS = 4;
constexpr uint32_t T_SC_BYTES = 512 + 1024;
constexpr uint32_t T_OFF_SC = T_OFF_OUT + T_OUT_BYTES;
constexpr uint32_t T_OFF_BAR = T_OFF_SC + T_SC_SLOTS * T_SC_BYTES;
constexpr uint32_t T_OFF_MISC = T_OFF_BAR + 256;
constexpr uint32_t T_OFF_ROWOFF = T_OFF_MISC + 128;
constexpr uint32_t T_SMEM_BYTES = T_OFF_ROWOFF + (MAX_G + 1) * 4 + 1024;
constexpr uint32_t T_IDESC = idesc(1, 0, 0, 1, 1, 128, 256);  // A and B MN-major

// OR of `v` over the 128 threads of named barrier `id` (a barrier).
__device__ __forceinline__ bool tgmm_bar_or(int id, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, 128, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}\n"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "r"(id)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void tgmm_tile(int t, int KT, int NT, int& g, int& k0, int& n0) {
  const int per = KT * NT;
  g = t / per;
  const int r = t % per;
  n0 = (r / KT) * 256;
  k0 = (r % KT) * 128;
}

// Blocks mb0 .. mb0 + nblk - 1 of rows [r0, r1).
__device__ __forceinline__ void tgmm_blocks(const int* row_off, int g, int& r0, int& r1, int& mb0,
                                            int& nblk) {
  r0 = row_off[g];
  r1 = row_off[g + 1];
  mb0 = r0 / 128;
  nblk = r1 > r0 ? (r1 - 1) / 128 - mb0 + 1 : 0;
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    tgmm_fp8_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                    const __grid_constant__ CUtensorMap tm_o, const TParams p) {
  constexpr int STAGES = T_STAGES, NBUF = 2, BN = 256, EC = 128, NCH = 4;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + T_OFF_BAR);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + NBUF;
  uint64_t* drain = tempty + NBUF;
  uint64_t* sc_full = drain + 1;
  uint64_t* sc_empty = sc_full + T_SC_SLOTS;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + T_OFF_MISC);
  int* abort_flag = reinterpret_cast<int*>(smem + T_OFF_MISC + 4);
  int* valid_s = reinterpret_cast<int*>(smem + T_OFF_MISC + 8);
  int* row_off = reinterpret_cast<int*>(smem + T_OFF_ROWOFF);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.G, K = p.K, N = p.N;
  const int KT = K / 128, NT = (N + BN - 1) / BN;
  const Abort ab{abort_flag, p.err};

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tm_a);
      prefetch_tmap(&tm_b);
    }
    tmem_alloc(tmem_holder, TMEM_COLS);
    tmem_relinquish();
  } else if (warp == 1) {
    if (lane == 0) {
      for (int i = 0; i < STAGES; ++i) {
        mbar_init(&full[i], 1);
        mbar_init(&empty[i], 1);
      }
      for (int i = 0; i < NBUF; ++i) {
        mbar_init(&tfull[i], 1);
        mbar_init(&tempty[i], 8);
      }
      mbar_init(drain, 1);
      for (int i = 0; i < T_SC_SLOTS; ++i) {
        mbar_init(&sc_full[i], 1);
        mbar_init(&sc_empty[i], 8);
      }
      *abort_flag = 0;
      fence_mbar_init();
    }
  } else if (warp == 3) {
    // row offsets (exclusive prefix sum of group_sizes) and validation
    const int per = (G + 31) / 32;
    const int g0 = min(G, lane * per), g1 = min(G, g0 + per);
    int sum = 0, bad = 0;
    for (int g = g0; g < g1; ++g) {
      const int sz = p.group_sizes[g];
      bad |= sz < 0;
      sum += max(sz, 0);
    }
    int inc = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += v;
    }
    int r = inc - sum;
    for (int g = g0; g < g1; ++g) {
      row_off[g] = r;
      r += max(p.group_sizes[g], 0);
    }
    bad = __any_sync(0xffffffffu, bad);
    if (lane == 31) {
      row_off[G] = inc;
      const bool ok = !bad && inc <= p.M;
      *valid_s = ok;
      if (!ok) atomicExch(p.err, GL_DEV_BAD_GROUPS);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const int total = *valid_s ? G * KT * NT : 0;

  if (warp == 0) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_CTRL));
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      int it = 0, sc_it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        int g, k0, n0, r0, r1, mb0, nblk;
        tgmm_tile(t, KT, NT, g, k0, n0);
        tgmm_blocks(row_off, g, r0, r1, mb0, nblk);
        for (int b = 0; b < nblk; ++b, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(&empty[s], ((it / STAGES) & 1) ^ 1, ab)) { ok = false; break; }
          const int m0 = (mb0 + b) * 128;
          mbar_arrive_expect_tx(&full[s], T_A_BYTES + T_B_BYTES);
          uint8_t* sa = smem + T_OFF_A + s * T_A_BYTES;
          uint8_t* sb = smem + T_OFF_B + s * T_B_BYTES;
          tma_load_2d(sa, &tm_a, &full[s], k0, m0);
          tma_load_2d(sb, &tm_b, &full[s], n0, m0);
          tma_load_2d(sb + 16384, &tm_b, &full[s], n0 + 128, m0);
          // the block's scales: ls[mb, k0 ..] and ds[mb, n0 ..] (N % 128 == 0)
          const int c = it % T_SC_SLOTS;
          if (!mbar_wait(&sc_empty[c], ((it / T_SC_SLOTS) & 1) ^ 1, ab)) { ok = false; ++it; break; }
          const uint32_t dsn = static_cast<uint32_t>(min(256, N - n0)) * 4u;
          uint8_t* sc = smem + T_OFF_SC + c * T_SC_BYTES;
          mbar_arrive_expect_tx(&sc_full[c], 512u + dsn);
          bulk_load(sc, p.ls + static_cast<int64_t>(mb0 + b) * K + k0, 512u, &sc_full[c]);
          bulk_load(sc + 512, p.ds + static_cast<int64_t>(mb0 + b) * N + n0, dsn, &sc_full[c]);
          ++sc_it;
        }
      }
      if (!ok) {
        // copies in flight finish before the CTA exits (bounded waits)
        const int first = it > STAGES ? it - STAGES : 0;
        for (int j = first; j < it; ++j) {
          const uint64_t t0 = global_ns();
          while (!mbar_try_wait(&full[j % STAGES], (j / STAGES) & 1) && global_ns() - t0 < 100000000ull) {
          }
        }
        const int sfirst = sc_it > T_SC_SLOTS ? sc_it - T_SC_SLOTS : 0;
        for (int j = sfirst; j < sc_it; ++j) {
          const uint64_t t0 = global_ns();
          while (!mbar_try_wait(&sc_full[j % T_SC_SLOTS], (j / T_SC_SLOTS) & 1) &&
                 global_ns() - t0 < 100000000ull) {
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_CTRL));
    // --------------------------------------------------- masking + MMA
    int it = 0, acc_it = 0;
    bool ok = true;
    const uint32_t a_base = smem_u32(smem + T_OFF_A), b_base = smem_u32(smem + T_OFF_B);
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
      int g, k0, n0, r0, r1, mb0, nblk;
      tgmm_tile(t, KT, NT, g, k0, n0);
      tgmm_blocks(row_off, g, r0, r1, mb0, nblk);
      for (int b = 0; b < nblk; ++b, ++it, ++acc_it) {
        const int s = it % STAGES;
        const int buf = acc_it % NBUF;
        bool got = true;
        if (lane == 0)
          got = mbar_wait(&tempty[buf], ((acc_it / NBUF) & 1) ^ 1, ab) &&
                mbar_wait(&full[s], (it / STAGES) & 1, ab);
        if (!__shfl_sync(0xffffffffu, got, 0)) { ok = false; break; }  // the whole warp leaves
        // rows of this block that belong to other groups: zero them in A
        const int m0 = (mb0 + b) * 128;
        const int lo = max(r0 - m0, 0), hi = min(r1 - m0, 128);
        if (lo > 0 || hi < 128) {
          uint4* a4 = reinterpret_cast<uint4*>(smem + T_OFF_A + s * T_A_BYTES);
          const uint4 z = make_uint4(0u, 0u, 0u, 0u);
          for (int i = lane; i < 128 * 8; i += 32) {
            const int row = i >> 3;
            if (row < lo || row >= hi) a4[i] = z;
          }
          fence_proxy_async_smem();
        }
        __syncwarp();
        tc_fence_after();
        if (lane == 0) {
          const uint32_t d = tmem + buf * BN;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t ad = sdesc(a_base + s * T_A_BYTES + kk * 4096, 16384, 1024, kSwizzle128B);
            const uint64_t bd = sdesc(b_base + s * T_B_BYTES + kk * 4096, 16384, 1024, kSwizzle128B);
            mma_f8f6f4(d, ad, bd, T_IDESC, kk > 0 ? 1u : 0u);
          }
          tc_commit(&empty[s]);
          tc_commit(&tfull[buf]);
        }
        __syncwarp();
      }
    }
    if (lane == 0) {
      tc_commit(drain);
      const uint64_t t0 = global_ns();
      while (!mbar_try_wait(drain, 0) && global_ns() - t0 < 100000000ull) {
      }
    }
    __syncwarp();
  } else if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_CTRL));
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REG_EPI));
    // -------------------------------------------------------- epilogue
    const int ew = warp - 4;
    const int quad = warp & 3;
    const int chalf = ew >> 2;
    const int r = quad * 32 + lane;                     // row k0 + r of the tile
    const int ht = threadIdx.x - 128 - chalf * 128;     // 0..127 within the half
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quad * 32) << 16) + chalf * EC;
    int acc_it = 0;
    bool ok = true;     // this thread's accumulators are valid
    bool stop = false;  // set only by the half's vote: the same in all its threads
    for (int t = blockIdx.x; t < total && !stop; t += gridDim.x) {
      int g, k0, n0, r0, r1, mb0, nblk;
      tgmm_tile(t, KT, NT, g, k0, n0);
      tgmm_blocks(row_off, g, r0, r1, mb0, nblk);
      const int ncol0 = n0 + chalf * EC;
      const bool col_ok = ncol0 < N;
      float2 acc[EC / 2];
#pragma unroll
      for (int j = 0; j < EC / 2; ++j) acc[j] = make_float2(0.f, 0.f);
      for (int b = 0; b < nblk; ++b, ++acc_it) {
        const int buf = acc_it % NBUF;
        const int c = acc_it % T_SC_SLOTS;
        // the block's scales, bulk-copied by the producer (a wait that gives
        // up sets the abort flag; the tile's vote below stops the half)
        if (!mbar_wait(&sc_full[c], (acc_it / T_SC_SLOTS) & 1, ab)) { ok = false; continue; }
        const float* scl = reinterpret_cast<const float*>(smem + T_OFF_SC + c * T_SC_BYTES);
        const float lsr = scl[r];
        const float* dsb = scl + 128 + chalf * EC;
        if (!mbar_wait(&tfull[buf], (acc_it / NBUF) & 1, ab)) { ok = false; continue; }
        tc_fence_after();
        const uint32_t ta = lane_base + buf * BN;
        const float2 ls2 = make_float2(lsr, lsr);
        uint32_t v[2][32];
        auto promote = [&](const uint32_t (&x)[32], int base) {
          const float4* d4 = reinterpret_cast<const float4*>(dsb) + base / 2;
#pragma unroll
          for (int j = 0; j < 16; j += 2) {
            const float4 dd = d4[j / 2];
            const float2 s01 = __fmul2_rn(make_float2(dd.x, dd.y), ls2);
            const float2 s23 = __fmul2_rn(make_float2(dd.z, dd.w), ls2);
            acc[base + j] = __ffma2_rn(make_float2(__uint_as_float(x[2 * j]), __uint_as_float(x[2 * j + 1])),
                                       s01, acc[base + j]);
            acc[base + j + 1] = __ffma2_rn(make_float2(__uint_as_float(x[2 * j + 2]), __uint_as_float(x[2 * j + 3])),
                                           s23, acc[base + j + 1]);
          }
        };
        tmem_ld32(ta, v[0]);
        tmem_ld32(ta + 32, v[1]);
        tmem_ld_wait2(v[0], v[1]);
#pragma unroll
        for (int c = 2; c < NCH; c += 2) {
          promote(v[0], 16 * (c - 2));
          tmem_ld32(ta + 32 * c, v[0]);
          promote(v[1], 16 * (c - 1));
          tmem_ld32(ta + 32 * (c + 1), v[1]);
          tmem_ld_wait2(v[0], v[1]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[buf]);
        promote(v[0], 16 * (NCH - 2));
        promote(v[1], 16 * (NCH - 1));
        __syncwarp();
        if (lane == 0) mbar_arrive(&sc_empty[c]);
      }
      if (stop) break;
      if (p.out_f32) {
        if (ok && col_ok) {
          float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) +
                                                  (static_cast<int64_t>(g) * K + k0 + r) * N + ncol0);
#pragma unroll
          for (int i = 0; i < EC / 4; ++i)
            dst[i] = make_float4(acc[2 * i].x, acc[2 * i].y, acc[2 * i + 1].x, acc[2 * i + 1].y);
        }
      } else {
        // bf16: this half's two 64-column atoms of the shared-memory output
        // tile (128B-swizzled rows), then one TMA store per atom.  Every
        // thread of the half takes part (the condition is the half's vote).
        const bool leader = ht == 0;
        if (leader) bulk_wait_read<0>();  // the previous tile's stores have read the tile
        // a barrier of this half that also votes: once any role gave up,
        // every thread of the half leaves here together
        if (tgmm_bar_or(3 + chalf, *static_cast<volatile int*>(abort_flag) != 0)) { stop = true; break; }
        uint8_t* ot = smem + T_OFF_OUT + chalf * 2 * 16384;
#pragma unroll
        for (int i = 0; i < EC / 8; ++i) {
          const int atom = i >> 3, c = i & 7;
          *reinterpret_cast<uint4*>(ot + atom * 16384 + r * 128 + ((c ^ (r & 7)) << 4)) =
              make_uint4(pack_bf16x2(acc[4 * i].x, acc[4 * i].y),
                         pack_bf16x2(acc[4 * i + 1].x, acc[4 * i + 1].y),
                         pack_bf16x2(acc[4 * i + 2].x, acc[4 * i + 2].y),
                         pack_bf16x2(acc[4 * i + 3].x, acc[4 * i + 3].y));
        }
        fence_proxy_async_smem();
        asm volatile("bar.sync %0, 128;" ::"r"(3 + chalf) : "memory");
        if (leader && col_ok) {  // (N is a multiple of 128: both atoms are in range)
          tma_store_2d(&tm_o, ot, ncol0, g * K + k0);
          tma_store_2d(&tm_o, ot + 16384, ncol0 + 64, g * K + k0);
          bulk_commit();
        }
      }
    }
    if (ht == 0) bulk_wait<0>();  // stores complete before the CTA exits
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace gmm
}  // namespace gl

// ---------------------------------------------------------------------------
// Host launcher (called from capi.cu after argument validation).
// ---------------------------------------------------------------------------
#include <cstdlib>
#include <cstring>

#include "tmap.h"

// Sets p.tma_out and the output maps when the outputs can leave through TMA
// stores (bf16): one map per output, rows row_off + M.
static bool out_tmaps(gl::gmm::Params& p, int64_t M, int64_t N, gl::gmm::OutMaps* om,
                      const char** why) {
  p.tma_out = 0;
  if (p.out_f32) return true;
  for (int o = 0; o < p.n_outs; ++o)
    if (!gl_make_tmap_2d(&om->m[o], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, p.outs[o], N, p.row_off + M, N,
                         64, 32, CU_TENSOR_MAP_SWIZZLE_128B, why))
      return false;
  p.tma_out = 1;
  return true;
}


template <int BN, bool kTransB, bool kStg>
static int launch_cfg(const CUtensorMap& tm_a, const CUtensorMap& tm_b, const gl::gmm::OutMaps& tm_o,
                      const gl::gmm::Params& p, int64_t G, int64_t M, int64_t N, cudaStream_t st,
                      int num_sms, const char** why) {
  using namespace gl::gmm;
  using CF = Cfg<BN, kStg>;
  const void* fn = reinterpret_cast<const void*>(gmm_fp8_fwd_kernel<BN, kTransB, kStg>);
  if (!gl_set_smem_attr(fn, 0, static_cast<int>(CF::SMEM_BYTES), why)) return -2;
  const int64_t ntn = (N + BN - 1) / BN;
  const int64_t max_tiles = ((M + BM - 1) / BM + G) * ntn;
  const int grid = static_cast<int>(max_tiles < num_sms ? (max_tiles > 0 ? max_tiles : 1) : num_sms);
  gmm_fp8_fwd_kernel<BN, kTransB, kStg><<<grid, NUM_THREADS, CF::SMEM_BYTES, st>>>(tm_a, tm_b, tm_o, p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    *why = cudaGetErrorString(e);
    return -2;
  }
  return 0;
}

template <int BN, bool kTransB = false>
static int launch_bn(const CUtensorMap& tm_a, const CUtensorMap& tm_b, gl::gmm::Params p,
                     int64_t G, int64_t M, int64_t N, cudaStream_t st, int num_sms,
                     const char** why) {
  gl::gmm::OutMaps tm_o;  // unused unless p.tma_out
  for (int o = 0; o < gl::gmm::MAX_OUTS; ++o) tm_o.m[o] = tm_a;
  p.tma_out = 0;
  if constexpr (BN == 256) {
    // staged output whenever the outputs are bf16 (out_tmaps decides)
    if (!out_tmaps(p, M, N, &tm_o, why)) return -1;
    if (p.tma_out)
      return launch_cfg<BN, kTransB, true>(tm_a, tm_b, tm_o, p, G, M, N, st, num_sms, why);
  }
  return launch_cfg<BN, kTransB, false>(tm_a, tm_b, tm_o, p, G, M, N, st, num_sms, why);
}

static int launch_pair(const CUtensorMap& tm_a, const CUtensorMap& tm_b,
                       const gl::gmm::Params& p, int64_t G, int64_t M, int64_t N, cudaStream_t st,
                       int num_sms, const char** why) {
  using namespace gl::gmm;
  const void* fn = reinterpret_cast<const void*>(gmm_fp8_fwd_pair_kernel);
  if (!gl_set_smem_attr(fn, 0, static_cast<int>(P_SMEM_BYTES), why)) return -2;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = P_SMEM_BYTES;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // Persistent: as many pairs as can be resident at once, capped by the work.
  cfg.gridDim = dim3(static_cast<unsigned>(num_sms & ~1), 1, 1);
  int max_clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&max_clusters, fn, &cfg) != cudaSuccess || max_clusters < 1) {
    *why = "cudaOccupancyMaxActiveClusters failed for the CTA-pair kernel";
    return -2;
  }
  const int64_t ntn = (N + 255) / 256;
  const int64_t max_tiles = ((M + PM - 1) / PM + G) * ntn;
  const int64_t clusters = max_tiles < max_clusters ? (max_tiles > 0 ? max_tiles : 1) : max_clusters;
  cfg.gridDim = dim3(static_cast<unsigned>(2 * clusters), 1, 1);
  const cudaError_t e = cudaLaunchKernelEx(&cfg, gmm_fp8_fwd_pair_kernel, tm_a, tm_b, p);
  if (e != cudaSuccess) {
    *why = cudaGetErrorString(e);
    return -2;
  }
  return 0;
}

int gl_launch_gmm_fp8_multi(const void* a_q, const float* a_s, const void* b_q, const float* b_s,
                            const int32_t* group_sizes, int64_t G, int64_t M, int64_t K, int64_t N,
                            void* const* outs, int n_outs, int64_t row_off, int out_f32, int* err,
                            cudaStream_t st, int num_sms, const char** why) {
  using namespace gl::gmm;
  CUtensorMap tm_a, tm_b;
  if (!gl_make_tmap_2d(&tm_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, a_q, K, M, K, 128, 128,
                       CU_TENSOR_MAP_SWIZZLE_128B, why))
    return -1;
  if (!gl_make_tmap_2d(&tm_b, CU_TENSOR_MAP_DATA_TYPE_UINT8, b_q, N, G * K, N, 128, 128,
                       CU_TENSOR_MAP_SWIZZLE_128B, why))
    return -1;
  Params p;
  p.a_s = a_s;
  p.b_s = b_s;
  p.group_sizes = group_sizes;
  p.out = outs[0];
  p.err = err;
  p.G = static_cast<int>(G);
  p.M = static_cast<int>(M);
  p.K = static_cast<int>(K);
  p.N = static_cast<int>(N);
  p.out_f32 = out_f32;
  for (int o = 0; o < MAX_OUTS; ++o) p.outs[o] = o < n_outs ? outs[o] : nullptr;
  p.n_outs = n_outs;
  p.row_off = row_off;
  // several outputs or a row offset: the single-CTA kernel
  if (n_outs > 1 || row_off != 0)
    return launch_bn<256, false>(tm_a, tm_b, p, G, M, N, st, num_sms, why);
  // Variant: GLAUCIS_GMM_VARIANT=pair|256|128 overrides the default.
  int variant = 256;
  if (const char* e = std::getenv("GLAUCIS_GMM_VARIANT")) {
    if (std::strcmp(e, "pair") == 0) variant = 2;
    else if (std::atoi(e) == 128) variant = 128;
  }
  if (variant == 2) return launch_pair(tm_a, tm_b, p, G, M, N, st, num_sms, why);
  return variant == 256 ? launch_bn<256, false>(tm_a, tm_b, p, G, M, N, st, num_sms, why)
                        : launch_bn<128, false>(tm_a, tm_b, p, G, M, N, st, num_sms, why);
}

int gl_launch_gmm_fp8(const void* a_q, const float* a_s, const void* b_q, const float* b_s,
                      const int32_t* group_sizes, int64_t G, int64_t M, int64_t K, int64_t N,
                      void* out, int out_f32, int* err, cudaStream_t st, int num_sms,
                      const char** why) {
  void* outs[1] = {out};
  return gl_launch_gmm_fp8_multi(a_q, a_s, b_q, b_s, group_sizes, G, M, K, N, outs, 1, 0, out_f32,
                                 err, st, num_sms, why);
}

// Backward dlhs = dout x rhs^T per group (tokamax gmm with transpose_rhs=True):
// the same kernel with the weight read K-major.  Kernel dimensions: reduction
// K = the weight's N, output N = the weight's K; a_q / a_s = dout quantised
// 1x128 along the weight's N; b_q [G, N, K] / b_s [G, N/128, K/128] are the
// forward's weight QArray [G, K_w, N_w] / [G, K_w/128, N_w/128].
int gl_launch_gmm_fp8_dlhs(const void* a_q, const float* a_s, const void* b_q, const float* b_s,
                           const int32_t* group_sizes, int64_t G, int64_t M, int64_t K, int64_t N,
                           void* out, int out_f32, int* err, cudaStream_t st, int num_sms,
                           const char** why) {
  using namespace gl::gmm;
  CUtensorMap tm_a, tm_b;
  if (!gl_make_tmap_2d(&tm_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, a_q, K, M, K, 128, 128,
                       CU_TENSOR_MAP_SWIZZLE_128B, why))
    return -1;
  // weight as [G * N rows, K columns]: row = output column, K contiguous
  if (!gl_make_tmap_2d(&tm_b, CU_TENSOR_MAP_DATA_TYPE_UINT8, b_q, K, G * N, K, 128, 128,
                       CU_TENSOR_MAP_SWIZZLE_128B, why))
    return -1;
  Params p;
  p.a_s = a_s;
  p.b_s = b_s;
  p.group_sizes = group_sizes;
  p.out = out;
  p.err = err;
  p.G = static_cast<int>(G);
  p.M = static_cast<int>(M);
  p.K = static_cast<int>(K);
  p.N = static_cast<int>(N);
  p.out_f32 = out_f32;
  for (int o = 0; o < MAX_OUTS; ++o) p.outs[o] = o == 0 ? out : nullptr;
  p.n_outs = 1;
  p.row_off = 0;
  return launch_bn<256, true>(tm_a, tm_b, p, G, M, N, st, num_sms, why);
}

// Backward drhs (tgmm): lq [M, K] / ls [M/128, K] and dq [M, N] / ds [M/128, N]
// quantised in 128x1 column blocks; out [G, K, N].  M % 128 == 0.
int gl_launch_tgmm_fp8(const void* lq, const float* ls, const void* dq, const float* ds,
                       const int32_t* group_sizes, int64_t G, int64_t M, int64_t K, int64_t N,
                       void* out, int out_f32, int* err, cudaStream_t st, int num_sms,
                       const char** why) {
  using namespace gl::gmm;
  CUtensorMap tm_a, tm_b;
  if (!gl_make_tmap_2d(&tm_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, lq, K, M, K, 128, 128,
                       CU_TENSOR_MAP_SWIZZLE_128B, why))
    return -1;
  if (!gl_make_tmap_2d(&tm_b, CU_TENSOR_MAP_DATA_TYPE_UINT8, dq, N, M, N, 128, 128,
                       CU_TENSOR_MAP_SWIZZLE_128B, why))
    return -1;
  CUtensorMap tm_o;
  if (out_f32) {
    tm_o = tm_a;  // unused: fp32 output is stored directly
  } else if (!gl_make_tmap_2d(&tm_o, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, out, N, G * K, N, 64, 128,
                              CU_TENSOR_MAP_SWIZZLE_128B, why)) {
    return -1;
  }
  TParams p;
  p.ls = ls;
  p.ds = ds;
  p.group_sizes = group_sizes;
  p.out = out;
  p.err = err;
  p.G = static_cast<int>(G);
  p.M = static_cast<int>(M);
  p.K = static_cast<int>(K);
  p.N = static_cast<int>(N);
  p.out_f32 = out_f32;
  const void* fn = reinterpret_cast<const void*>(tgmm_fp8_kernel);
  if (!gl_set_smem_attr(fn, 0, static_cast<int>(T_SMEM_BYTES), why)) return -2;
  const int64_t tiles = G * (K / 128) * ((N + 255) / 256);
  const int grid = static_cast<int>(tiles < num_sms ? (tiles > 0 ? tiles : 1) : num_sms);
  tgmm_fp8_kernel<<<grid, NUM_THREADS, T_SMEM_BYTES, st>>>(tm_a, tm_b, tm_o, p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    *why = cudaGetErrorString(e);
    return -2;
  }
  return 0;
}
