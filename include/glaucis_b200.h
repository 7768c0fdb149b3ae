/*
 * glaucis_b200 — C ABI of the B200 (sm_100a) kernels behind the two scored
 * kernel templates of the Glaucis kernel evaluator:
 *
 *   gmm_fp8_blockwise  grouped (ragged, MoE-style) matmul with block-wise FP8
 *                      quantisation: activations 1x128 fp32 scales, weights
 *                      128x128 fp32 scales, fp32 accumulation.
 *   chunk_gla          chunked Gated Linear Attention, forward.
 *
 * Conventions shared by every entry point:
 *   - All pointers are device pointers owned by the caller.  The library
 *     borrows them for the duration of the (asynchronous) call and never
 *     frees or retains them.
 *   - `stream` is a cudaStream_t passed as void*; NULL means the legacy
 *     default stream.  Every call is stream-ordered and returns before the
 *     GPU work finishes.
 *   - `err_word` is an optional device int.  Kernels write a non-zero
 *     GL_DEV_* code there when a bounded device-side wait gives up; pass NULL
 *     to use a per-device word owned by the library.  Read it back with
 *     gl_device_status().
 *   - Return value: GL_OK (0) on a successful launch, a negative GL_E* code
 *     otherwise; gl_last_error() then holds a message (per host thread).
 *
 * Each entry point names the reference interface it replaces (paths are
 * relative to the Glaucis repository, kernel-evolve = KE).
 */
#ifndef GLAUCIS_B200_H
#define GLAUCIS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Return codes. */
#define GL_OK 0
#define GL_EINVAL (-1)   /* bad shape, alignment or argument */
#define GL_ELAUNCH (-2)  /* CUDA launch / driver failure */
#define GL_EDEVICE (-3)  /* device error word was set */

/* Device error word codes (written by kernels). */
#define GL_DEV_OK 0
#define GL_DEV_WAIT_TIMEOUT 1   /* an mbarrier wait exceeded its poll budget */
#define GL_DEV_BAD_GROUPS 2     /* group_sizes sum exceeds M or a size < 0 */

/* Output dtypes of the grouped matmul. */
#define GL_OUT_BF16 0
#define GL_OUT_F32 1

/*
 * Block-wise activation quantiser, 1x128 tiles along K.
 *   x  bf16 [M, K] row-major, K % 128 == 0
 *   q  e4m3fn [M, K] row-major (one byte per element)
 *   s  fp32 [M, K/128] row-major, s = absmax(block)/448 (1.0 for an all-zero
 *      block), q = round-to-nearest-even(x / s) saturated to +-448.
 * Replaces: qwix.pallas.quantize(lhs, float8_e4m3fn, channelwise_axes=[0],
 *   tiled_axes={1: 128}, calibration_method="absmax", scale_dtype=f32)
 *   called at KE/examples/kernels/gmm_fp8_blockwise.py:84-91.
 */
int gl_quant_act_1x128(const void* x, int64_t M, int64_t K, void* q, float* s,
                       int* err_word, void* stream);

/*
 * Block-wise weight quantiser, 128x128 tiles over (K, N) per group.
 *   w  bf16 [G, K, N] row-major, K % 128 == 0, N % 128 == 0
 *   q  e4m3fn [G, K, N] row-major
 *   s  fp32 [G, K/128, N/128]
 * Replaces: qwix.pallas.quantize(rhs, float8_e4m3fn, channelwise_axes=[0],
 *   tiled_axes={1: 128, 2: 128}, ...) at
 *   KE/examples/kernels/gmm_fp8_blockwise.py:100-107.
 */
int gl_quant_w_128x128(const void* w, int64_t G, int64_t K, int64_t N, void* q,
                       float* s, int* err_word, void* stream);

/*
 * Grouped matmul forward on pre-quantised operands:
 *   out[m, n] = sum_kb a_s[m, kb] * b_s[g, kb, n/128]
 *                      * sum_{k in block kb} a_q[m, k] * b_q[g, k, n]
 * where rows [off_g, off_g + group_sizes[g]) belong to group g and off_g is
 * the exclusive prefix sum of group_sizes.  Rows at or beyond
 * sum(group_sizes) are not written.
 *   a_q e4m3fn [M, K], a_s fp32 [M, K/128]      (layout of gl_quant_act_1x128)
 *   b_q e4m3fn [G, K, N], b_s fp32 [G, K/128, N/128] (gl_quant_w_128x128)
 *   group_sizes int32 [G] (device), out [M, N] bf16 or fp32 (out_dtype).
 *   K % 128 == 0, N % 128 == 0, 1 <= G <= 1024.
 * Replaces: tokamax pallas_mosaic_tpu_kernel.gmm(lhs=QArray, rhs=QArray,
 *   group_sizes, out_dtype=f32, transpose_rhs=False) at
 *   KE/examples/kernels/gmm_fp8_blockwise.py:109-119 (reference oracle:
 *   KE/examples/kernels/gmm_fp8_blockwise_ref.py:67-77).
 */
int gl_gmm_fp8_fwd(const void* a_q, const float* a_s, const void* b_q,
                   const float* b_s, const int32_t* group_sizes, int64_t G,
                   int64_t M, int64_t K, int64_t N, void* out, int out_dtype,
                   int* err_word, void* stream);

/* Largest n_outs of gl_gmm_fp8_fwd_scatter. */
#define GL_MAX_SCATTER_OUTS 8

/*
 * gl_gmm_fp8_fwd with its output rows stored into several buffers: row m of
 * this call is written as row row_offset + m of each of outs[0 .. n_outs-1]
 * (each at least row_offset + M rows of N elements of out_dtype, 16-byte
 * aligned).  The buffers may be other GPUs' memory mapped into this process
 * (CUDA IPC peer mappings over NVLink, e.g. gl_ipc_open): the kernel only
 * stores to them (bf16: TMA stores of each finished 32-row slice from shared
 * memory; fp32 and a group's last rows: direct stores), so a grouped matmul
 * sharded by expert group across ranks assembles the full output on every
 * rank inside its epilogue, overlapped with the MMAs, instead of an
 * all-gather after it.  The caller
 * orders the readers after the kernels of all ranks (a barrier).  Rows past
 * sum(group_sizes) are not written.  No counterpart in the reference (its
 * sharded output would be all-gathered by a collective).
 */
int gl_gmm_fp8_fwd_scatter(const void* a_q, const float* a_s, const void* b_q, const float* b_s,
                           const int32_t* group_sizes, int64_t G, int64_t M, int64_t K, int64_t N,
                           void* const* outs, int n_outs, int64_t row_offset, int out_dtype,
                           int* err_word, void* stream);

/*
 * Peer buffers for gl_gmm_fp8_fwd_scatter across processes (one per GPU):
 * gl_ipc_alloc allocates device memory on the current device and returns its
 * CUDA IPC handle (GL_IPC_HANDLE_BYTES bytes); another process opens it with
 * gl_ipc_open (a unicast peer mapping over NVLink; no multicast object) and
 * releases the mapping with gl_ipc_close; the owner frees with gl_ipc_free.
 */
#define GL_IPC_HANDLE_BYTES 64
int gl_ipc_alloc(size_t bytes, void** ptr, void* handle);
int gl_ipc_open(const void* handle, void** ptr);
int gl_ipc_close(void* ptr);
int gl_ipc_free(void* ptr);

/*
 * Chunked Gated Linear Attention forward (fixed-length sequences).
 *   q, k  bf16 [B, T, H, K];  v bf16 [B, T, H, V];  K == 128, V == 128
 *   g       fp32 [B, T, H, K] per-key log-gate (raw, not cumsummed) or NULL
 *   g_gamma fp32 [H] per-head constant log-gate or NULL (exactly one of
 *           g / g_gamma must be non-NULL)
 *   h0      fp32 [B, H, K, V] initial state or NULL (zeros)
 *   o       bf16 [B, T, H, V] output
 *   ht      fp32 [B, H, K, V] final state or NULL (not written)
 *   chunk_size == 64, T % 64 == 0.
 * Semantics: within each chunk G = cumsum(g) (chunk-local);
 *   o = scale*(q*e^G) h_n + tril(scale*(q*e^G)(k*e^-G)^T) v
 *   h_{n+1} = e^{G_last} * h_n + (k*e^{G_last-G})^T v.
 * Replaces: chunk_gla_fwd(q, k, v, g_gamma, scale, chunk_size) at
 *   KE/examples/kernels/chunk_gla.py:258-273 (three pallas_calls
 *   chunk_fwd_h :94-138, chunk_gla_fwd_intra_gk :163-188,
 *   chunk_gla_fwd_o_gk :218-250), with the per-key gate / h0 / final-state
 *   semantics of chunk_fwd_h_ref at
 *   KE/upstream/fused_chunk_simple_gla/common_chunk_h.py:363-489.
 */
int gl_chunk_gla_fwd(const void* q, const void* k, const void* v, const float* g,
                     const float* g_gamma, const float* h0, float scale,
                     int64_t B, int64_t T, int64_t H, int64_t K, int64_t V,
                     int64_t chunk_size, void* o, float* ht, int* err_word,
                     void* stream);

/* Flags of gl_chunk_gla_fwd_ex. */
#define GL_GLA_BF16_INTRA 1  /* tril(A) v with A rounded to bf16 once (see below) */

/*
 * The chunked GLA forward with every option: gl_chunk_gla_fwd_ws (h_states
 * NULL) or gl_chunk_gla_fwd_states (h_states non-NULL) plus `flags`.
 *   flags = 0 (also every other gl_chunk_gla_fwd* entry point): the
 *     intra-chunk product tril(A) v = P_hi v + P_lo v with P_hi =
 *     bf16(tril(A)) and P_lo = bf16(tril(A) - P_hi), so A enters the product
 *     to ~2^-17 relative, as the template's output kernel multiplies fp32 A
 *     by v at Precision.HIGHEST (KE/examples/kernels/chunk_gla.py:208-212).
 *   flags = GL_GLA_BF16_INTRA: A rounded to bf16 once on the tensor core
 *     (fp32 accumulation), the operand precision of the reference's jnp
 *     oracle at default matmul precision on its TPU platform
 *     (KE/examples/kernels/chunk_gla_ref.py:96-97); about 10 % faster.
 * Replaces chunk_gla_fwd (KE/examples/kernels/chunk_gla.py:258-273) as
 * gl_chunk_gla_fwd does.
 */
int gl_chunk_gla_fwd_ex(const void* q, const void* k, const void* v, const float* g,
                        const float* g_gamma, const float* h0, float scale, int64_t B, int64_t T,
                        int64_t H, int64_t K, int64_t V, int64_t chunk_size, void* o, float* ht,
                        void* h_states, void* workspace, size_t workspace_bytes, int flags,
                        int* err_word, void* stream);

/*
 * gl_chunk_gla_fwd_ex (h_states NULL) with o stored into several buffers:
 * outs[0 .. n_outs-1], each of o's layout [B, T, H, V] bf16 and 16-byte
 * aligned, receive the same output.  The buffers may be other GPUs' memory
 * mapped into this process (CUDA IPC peer mappings over NVLink, e.g.
 * gl_ipc_open): the forward stores each chunk's O from shared memory with TMA
 * stores into every buffer, so a forward sharded by head across ranks
 * assembles its output on every rank inside the kernel instead of an
 * all-gather after it.  Needs the full-width kernel, i.e. a workspace when
 * B*H*2 <= the SM count (GL_EINVAL otherwise).  The caller orders the
 * readers after the kernels of all ranks.  No counterpart in the reference
 * (chunk_gla.py:258-273 writes one o; a head-sharded caller would all-gather).
 */
int gl_chunk_gla_fwd_scatter(const void* q, const void* k, const void* v, const float* g,
                             const float* g_gamma, const float* h0, float scale, int64_t B,
                             int64_t T, int64_t H, int64_t K, int64_t V, int64_t chunk_size,
                             void* const* outs, int n_outs, float* ht, void* workspace,
                             size_t workspace_bytes, int flags, int* err_word, void* stream);

/*
 * The intermediates of the chunked GLA forward that gl_chunk_gla_fwd keeps on
 * chip, for callers that read them:
 *   g_cumsum fp32 [B, T, H, K]  chunk-local cumsum of g (or g_gamma[h]*(1..64))
 *   A        fp32 [B, T, H, 64] A[i, j] = scale * sum_k q[i,k] e^{G[i,k]}
 *                               k[j,k] e^{-G[j,k]} per chunk, full 64x64
 *                               square (not causally masked)
 * Either output may be NULL (not written); q, k, g / g_gamma, scale and the
 * shapes as gl_chunk_gla_fwd.  fp32 arithmetic (not the tensor cores), one
 * extra pass over q, k and g.  err_word is accepted for symmetry and never
 * written (the kernel has no device-side waits).
 * Replaces the g_cumsum and A outputs of chunk_gla_fwd
 * (KE/examples/kernels/chunk_gla.py:258-273; A from chunk_gla_fwd_intra_gk
 * :146-188, g_cumsum :265-267).
 */
int gl_chunk_gla_fwd_intermediates(const void* q, const void* k, const float* g,
                                   const float* g_gamma, float scale, int64_t B, int64_t T,
                                   int64_t H, int64_t K, int64_t chunk_size, float* g_cumsum,
                                   float* A, int* err_word, void* stream);

/*
 * gl_chunk_gla_fwd with a caller-owned device workspace.  When B*H is small
 * against the SM count (few heads, long sequences) the sequence is split into
 * segments.  The first, short segment runs its full pass from h0 beside a
 * state-only pass that computes each middle segment's final state from a
 * zero state, and its total decay, into the workspace; the full pass of the
 * remaining segments then starts each of them from h0 folded with the
 * preceding segments' records, so the recurrence runs on one CTA per SM
 * instead of one per (batch, head).  The first phase forks a library-owned
 * stream from `stream` and joins it back with events.
 * gl_chunk_gla_fwd_workspace_bytes gives the size the split wants on the
 * current device (0: no split for this shape); a smaller workspace gives
 * fewer segments, NULL / 0 none.  The workspace must be 256-byte aligned and
 * not be used by another call in flight.  gl_chunk_gla_fwd is this call with
 * no workspace.  No reference counterpart: the reference scans the sequence
 * once per (batch, head) (KE/examples/kernels/chunk_gla.py:94-138).
 */
size_t gl_chunk_gla_fwd_workspace_bytes(int64_t B, int64_t T, int64_t H, int64_t K,
                                        int64_t V, int64_t chunk_size);
int gl_chunk_gla_fwd_ws(const void* q, const void* k, const void* v, const float* g,
                        const float* g_gamma, const float* h0, float scale,
                        int64_t B, int64_t T, int64_t H, int64_t K, int64_t V,
                        int64_t chunk_size, void* o, float* ht, void* workspace,
                        size_t workspace_bytes, int* err_word, void* stream);

/*
 * Training forward of the chunked GLA: gl_chunk_gla_fwd_ws that also writes
 * the state before every chunk, h_states bf16 [B, T/64, H, K, V]
 * (h_states[:, n] = h_n, h_0 = h0), the residual the backward reads.
 * Replaces the h output of chunk_gla_fwd (KE/examples/kernels/chunk_gla.py
 * :258-273, kept fp32 there and cast to bf16 where the backward uses it,
 * :356-359).
 */
int gl_chunk_gla_fwd_states(const void* q, const void* k, const void* v, const float* g,
                            const float* g_gamma, const float* h0, float scale,
                            int64_t B, int64_t T, int64_t H, int64_t K, int64_t V,
                            int64_t chunk_size, void* o, float* ht, void* h_states,
                            void* workspace, size_t workspace_bytes, int* err_word,
                            void* stream);

/*
 * Backward of the chunked GLA: dq, dk, dv (bf16, shaped as q, k, v) and,
 * when dh0 is non-NULL, the gradient of the initial state (fp32 [B,H,K,V]),
 * for the loss sum(o * dout) (+ sum(ht * dht) when dht is non-NULL).
 *   h_states  the forward's bf16 [B, T/64, H, K, V] (gl_chunk_gla_fwd_states)
 *   dout      bf16 [B, T, H, V];  dht fp32 [B, H, K, V] or NULL
 *   g / g_gamma, scale, shapes as the forward.  The gate is not
 *   differentiated (the reference's custom_vjp returns dq, dk, dv).
 *   workspace device memory of gl_chunk_gla_bwd_workspace_bytes(...) bytes
 *   (required, 256-byte aligned): the reverse scan's per-chunk state
 *   gradient E_n = e^{G_last(n)} dL/dh_{n+1} (bf16) and the records of its
 *   sequence split.
 * Two launches: the reverse state-gradient scan (a mode of the forward's
 * sequential kernel, with its own sequence split) and the chunk-parallel
 * dq/dk/dv kernel.  Replaces _bwd of chunk_gla (KE/examples/kernels/
 * chunk_gla.py:446-453): _chunk_bwd_dh_scan :281-305 and
 * chunk_gla_bwd_fused :313-426.
 */
size_t gl_chunk_gla_bwd_workspace_bytes(int64_t B, int64_t T, int64_t H, int64_t K,
                                        int64_t V, int64_t chunk_size);
int gl_chunk_gla_bwd(const void* q, const void* k, const void* v, const float* g,
                     const float* g_gamma, const void* h_states, const void* dout,
                     const float* dht, float scale, int64_t B, int64_t T, int64_t H,
                     int64_t K, int64_t V, int64_t chunk_size, void* dq, void* dk, void* dv,
                     float* dh0, void* workspace, size_t workspace_bytes, int* err_word,
                     void* stream);

/*
 * Backward of the grouped matmul (KE/examples/kernels/gmm_fp8_blockwise.py:123-169).
 *
 * gl_quant_col_128x1: 128x1 column blocks of x bf16 [M, C] (M, C multiples
 *   of 128): q e4m3 [M, C], s fp32 [M/128, C], s = absmax of 128 rows of one
 *   column / 448.  Replaces qpl.quantize(grad, channelwise_axes=[1],
 *   tiled_axes={0:128}) :135-141 and, untransposed, qpl.quantize(lhs^T,
 *   channelwise_axes=[0], tiled_axes={1:128}) :92-99 (lhs_t = (q^T, s^T)).
 * gl_gmm_fp8_dlhs: dlhs [M, K] = dout x rhs^T per group: dq / ds = dout
 *   quantised 1x128 along N (gl_quant_act_1x128 of grad [M, N]); b_q / b_s the
 *   forward's weight QArray [G, K, N] / [G, K/128, N/128].  Replaces
 *   tokamax gmm(dlhs_dout, rhs, transpose_rhs=True) :143-153.  Rows at or
 *   beyond sum(group_sizes) are not written.
 * gl_tgmm_fp8: drhs [G, K, N] = per group lhs^T x dout over the group's rows:
 *   lq / ls and dq / ds quantised by gl_quant_col_128x1 (M % 128 == 0).
 *   Empty groups get zeros.  Replaces tokamax tgmm(lhs_t, drhs_dout) :155-165.
 */
int gl_quant_col_128x1(const void* x, int64_t M, int64_t C, void* q, float* s, int* err_word,
                       void* stream);
int gl_gmm_fp8_dlhs(const void* dq, const float* ds, const void* b_q, const float* b_s,
                    const int32_t* group_sizes, int64_t G, int64_t M, int64_t K, int64_t N,
                    void* out, int out_dtype, int* err_word, void* stream);
int gl_tgmm_fp8(const void* lq, const float* ls, const void* dq, const float* ds,
                const int32_t* group_sizes, int64_t G, int64_t M, int64_t K, int64_t N,
                void* out, int out_dtype, int* err_word, void* stream);

/* Largest M*K accepted by gl_gmm_fp8_act_fwd_noalloc (activation elements). */
#define GL_NOALLOC_MAX_ACT_ELEMS (16u * 1024u * 1024u)

/*
 * Grouped matmul forward from bf16 activations that allocates no device
 * memory.  No counterpart in the reference: it exists for callers that
 * cannot allocate device memory during a step (runtimes that plan every
 * buffer up front and forbid allocation while executing, FFI callers
 * without a device allocator).  It quantises lhs (1x128, as
 * gl_quant_act_1x128) into a fixed device scratch array owned by the
 * library (16 MiB of e4m3 plus 512 KiB of scales, created when the
 * library's device code loads on a GPU and held until exit) and runs
 * gl_gmm_fp8_fwd on it.
 *   lhs bf16 [M, K] with M * K <= GL_NOALLOC_MAX_ACT_ELEMS (else GL_EINVAL);
 *   b_q, b_s, group_sizes, out, out_dtype as gl_gmm_fp8_fwd.
 *   err_word: caller-owned device int for device-side error codes (invalid
 *   group_sizes, a wait that gave up).  Callers that need those errors must
 *   pass one: with NULL they go to the scratch array's own word, which every
 *   call clears first and which nothing reads back (gl_device_status(NULL)
 *   reads the library word, which this entry point never touches because
 *   that word is allocated memory).
 * All calls on a device share the scratch array and it keeps the last
 * call's contents; calls whose GPU work overlaps race on it.  The first call
 * on each device looks up the array's device address; make it before any
 * stream capture.
 */
int gl_gmm_fp8_act_fwd_noalloc(const void* lhs, const void* b_q, const float* b_s,
                               const int32_t* group_sizes, int64_t G, int64_t M,
                               int64_t K, int64_t N, void* out, int out_dtype,
                               int* err_word, void* stream);

/*
 * Synchronises `stream`, reads the device error word (the library word when
 * err_word is NULL) into *code and clears it.  Returns GL_OK or GL_ELAUNCH.
 */
int gl_device_status(int* err_word, void* stream, int* code);

/* Message of the last failing call on this host thread ("" if none). */
const char* gl_last_error(void);

/* Library version string. */
const char* gl_version(void);

#ifdef __cplusplus
}
#endif

#endif /* GLAUCIS_B200_H */
