// extern "C" surface of libglaucis_b200.so: argument validation, per-device
// state (SM count, library-owned error word), TMA descriptor encoding and the
// thread-local last-error message.  See include/glaucis_b200.h.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <mutex>
#include <set>
#include <string>
#include <utility>

#include "../../include/glaucis_b200.h"
#include "tmap.h"

// Launchers defined next to their kernels.
int gl_launch_quant_act(const void* x, int64_t M, int64_t K, void* q, float* s, int* err,
                        cudaStream_t st, int num_sms, const char** why);
int gl_launch_quant_w(const void* w, int64_t G, int64_t K, int64_t N, void* q, float* s, int* err,
                      cudaStream_t st, int num_sms, const char** why);
int gl_launch_gmm_fp8(const void* a_q, const float* a_s, const void* b_q, const float* b_s,
                      const int32_t* group_sizes, int64_t G, int64_t M, int64_t K, int64_t N,
                      void* out, int out_f32, int* err, cudaStream_t st, int num_sms,
                      const char** why);
int gl_launch_chunk_gla(const void* q, const void* k, const void* v, const float* g,
                        const float* g_gamma, const float* h0, float scale, int64_t B, int64_t T,
                        int64_t H, int64_t K, int64_t V, void* o, float* ht, void* h_out, void* ws,
                        size_t ws_bytes, int p_split, int* err, cudaStream_t st, int num_sms,
                        const char** why);
size_t gl_chunk_gla_ws_bytes(int64_t B, int64_t T, int64_t H, int num_sms);
int gl_launch_gmm_fp8_multi(const void* a_q, const float* a_s, const void* b_q, const float* b_s,
                            const int32_t* group_sizes, int64_t G, int64_t M, int64_t K, int64_t N,
                            void* const* outs, int n_outs, int64_t row_off, int out_f32, int* err,
                            cudaStream_t st, int num_sms, const char** why);
int gl_launch_chunk_gla_scatter(const void* q, const void* k, const void* v, const float* g,
                                const float* g_gamma, const float* h0, float scale, int64_t B,
                                int64_t T, int64_t H, void* const* outs, int n_outs, float* ht,
                                void* ws, size_t ws_bytes, int p_split, int* err, cudaStream_t st,
                                int num_sms, const char** why);
int gl_launch_chunk_gla_dh(const void* q, const void* dout, const float* g, const float* g_gamma,
                           const float* dht, float scale, int64_t B, int64_t T, int64_t H,
                           void* e_out, float* dh0, void* ws, size_t ws_bytes, int* err,
                           cudaStream_t st, int num_sms, const char** why);
int gl_launch_chunk_gla_grads(const void* q, const void* k, const void* v, const void* dout,
                              const float* g, const float* g_gamma, const void* h, const void* e,
                              float scale, int64_t B, int64_t T, int64_t H, void* dq, void* dk,
                              void* dv, int* err, cudaStream_t st, int num_sms, const char** why);
int gl_launch_gla_intermediates(const void* q, const void* k, const float* g, const float* g_gamma,
                                float scale, int64_t B, int64_t T, int64_t H, float* g_cumsum,
                                float* A, cudaStream_t st, const char** why);
int gl_launch_quant_col(const void* x, int64_t M, int64_t C, void* q, float* s, int* err,
                        cudaStream_t st, int num_sms, const char** why);
int gl_launch_gmm_fp8_dlhs(const void* a_q, const float* a_s, const void* b_q, const float* b_s,
                           const int32_t* group_sizes, int64_t G, int64_t M, int64_t K, int64_t N,
                           void* out, int out_f32, int* err, cudaStream_t st, int num_sms,
                           const char** why);
int gl_launch_tgmm_fp8(const void* lq, const float* ls, const void* dq, const float* ds,
                       const int32_t* group_sizes, int64_t G, int64_t M, int64_t K, int64_t N,
                       void* out, int out_f32, int* err, cudaStream_t st, int num_sms,
                       const char** why);

namespace {

thread_local std::string t_last_error;

int fail(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}

struct DeviceState {
  int num_sms = 0;
  int* err = nullptr;
};

std::mutex g_mu;
DeviceState g_dev[64];
std::set<std::pair<int, const void*>> g_smem_attr_done;

// Returns 0 and fills the current device's state, allocating the library
// error word on first use.
int device_state(DeviceState** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(GL_ELAUNCH, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(GL_ELAUNCH, "device ordinal out of range");
  // Make the device's primary context current on this thread: the tensor-map
  // encoder is a driver call, and a thread that has made no runtime call yet
  // (autograd's backward worker, for one) has no current context.
  e = cudaSetDevice(dev);
  if (e != cudaSuccess) return fail(GL_ELAUNCH, std::string("cudaSetDevice: ") + cudaGetErrorString(e));
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceState& d = g_dev[dev];
  if (d.num_sms == 0) {
    e = cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return fail(GL_ELAUNCH, std::string("cudaDeviceGetAttribute: ") + cudaGetErrorString(e));
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (major != 10 || minor != 0) {
      d.num_sms = 0;
      return fail(GL_ELAUNCH, "libglaucis_b200 is built for sm_100a (B200) only; device is sm_" +
                                  std::to_string(major) + std::to_string(minor));
    }
  }
  if (d.err == nullptr) {
    e = cudaMalloc(&d.err, sizeof(int));
    if (e != cudaSuccess) return fail(GL_ELAUNCH, std::string("cudaMalloc(error word): ") + cudaGetErrorString(e));
    e = cudaMemset(d.err, 0, sizeof(int));
    if (e != cudaSuccess) return fail(GL_ELAUNCH, std::string("cudaMemset(error word): ") + cudaGetErrorString(e));
  }
  *out = &d;
  return GL_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

PFN_cuTensorMapEncodeTiled_v12000 encode_fn(const char** why) {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  if (!fn) *why = "cuTensorMapEncodeTiled is not available from the driver";
  return fn;
}

uint32_t elem_bytes(CUtensorMapDataType dt) {
  switch (dt) {
    case CU_TENSOR_MAP_DATA_TYPE_UINT8: return 1;
    case CU_TENSOR_MAP_DATA_TYPE_BFLOAT16:
    case CU_TENSOR_MAP_DATA_TYPE_FLOAT16: return 2;
    case CU_TENSOR_MAP_DATA_TYPE_FLOAT32: return 4;
    default: return 0;
  }
}

}  // namespace

// Records `msg` as this thread's last error and returns `code` (shared with
// the other entry-point files).
int gl_set_error_message(int code, const char* msg) { return fail(code, msg); }

bool gl_make_tmap_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* ptr, int64_t inner,
                     int64_t outer, int64_t row_stride_elems, uint32_t box_inner,
                     uint32_t box_outer, CUtensorMapSwizzle sw, const char** why) {
  auto fn = encode_fn(why);
  if (!fn) return false;
  const uint32_t eb = elem_bytes(dt);
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride_elems) * eb};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    thread_local char msg[256];
    std::snprintf(msg, sizeof msg,
                  "cuTensorMapEncodeTiled (2-D) rejected the operand (alignment / stride / box): "
                  "ptr %p dims [%lld, %lld] row stride %lld B box [%u, %u] (error %d)",
                  ptr, static_cast<long long>(inner), static_cast<long long>(outer),
                  static_cast<long long>(strides[0]), box_inner, box_outer, static_cast<int>(r));
    *why = msg;
    return false;
  }
  return true;
}

bool gl_make_tmap_3d(CUtensorMap* m, CUtensorMapDataType dt, const void* ptr, int64_t d0,
                     int64_t d1, int64_t d2, int64_t s1_elems, int64_t s2_elems, uint32_t b0,
                     uint32_t b1, uint32_t b2, CUtensorMapSwizzle sw, const char** why) {
  auto fn = encode_fn(why);
  if (!fn) return false;
  const uint32_t eb = elem_bytes(dt);
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(d0), static_cast<cuuint64_t>(d1),
                        static_cast<cuuint64_t>(d2)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(s1_elems) * eb,
                           static_cast<cuuint64_t>(s2_elems) * eb};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, dt, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    thread_local char msg[256];
    std::snprintf(msg, sizeof msg,
                  "cuTensorMapEncodeTiled (3-D) rejected the operand (alignment / stride / box): "
                  "ptr %p dims [%lld, %lld, %lld] strides %lld, %lld B box [%u, %u, %u] (error %d)",
                  ptr, static_cast<long long>(d0), static_cast<long long>(d1),
                  static_cast<long long>(d2), static_cast<long long>(strides[0]),
                  static_cast<long long>(strides[1]), b0, b1, b2, static_cast<int>(r));
    *why = msg;
    return false;
  }
  return true;
}

bool gl_set_smem_attr(const void* func, int, int bytes, const char** why) {
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_smem_attr_done.count({dev, func})) return true;
  }
  if (cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) {
    *why = "cudaFuncSetAttribute(MaxDynamicSharedMemorySize) failed";
    return false;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  g_smem_attr_done.insert({dev, func});
  return true;
}

extern "C" {

const char* gl_last_error(void) { return t_last_error.c_str(); }

const char* gl_version(void) { return "glaucis_b200 0.1 (sm_100a)"; }

int gl_quant_act_1x128(const void* x, int64_t M, int64_t K, void* q, float* s, int* err_word,
                       void* stream) {
  if (!x || !q || !s) return fail(GL_EINVAL, "gl_quant_act_1x128: null pointer");
  if (M < 0 || K <= 0 || K % 128 != 0)
    return fail(GL_EINVAL, "gl_quant_act_1x128: need M >= 0 and K a positive multiple of 128");
  if (!aligned16(x) || !aligned16(q))
    return fail(GL_EINVAL, "gl_quant_act_1x128: x and q must be 16-byte aligned");
  if (M == 0) return GL_OK;
  DeviceState* d = nullptr;
  if (int rc = device_state(&d)) return rc;
  const char* why = "";
  const int rc = gl_launch_quant_act(x, M, K, q, s, err_word ? err_word : d->err,
                                     static_cast<cudaStream_t>(stream), d->num_sms, &why);
  if (rc == -1) return fail(GL_EINVAL, std::string("gl_quant_act_1x128: ") + why);
  if (rc != 0) return fail(GL_ELAUNCH, std::string("quant_act launch: ") + why);
  return GL_OK;
}

int gl_quant_w_128x128(const void* w, int64_t G, int64_t K, int64_t N, void* q, float* s,
                       int* err_word, void* stream) {
  if (!w || !q || !s) return fail(GL_EINVAL, "gl_quant_w_128x128: null pointer");
  if (G <= 0 || K <= 0 || N <= 0 || K % 128 != 0 || N % 128 != 0)
    return fail(GL_EINVAL, "gl_quant_w_128x128: need G > 0 and K, N positive multiples of 128");
  if (!aligned16(w) || !aligned16(q))
    return fail(GL_EINVAL, "gl_quant_w_128x128: w and q must be 16-byte aligned");
  DeviceState* d = nullptr;
  if (int rc = device_state(&d)) return rc;
  const char* why = "";
  const int rc = gl_launch_quant_w(w, G, K, N, q, s, err_word ? err_word : d->err,
                                   static_cast<cudaStream_t>(stream), d->num_sms, &why);
  if (rc == -1) return fail(GL_EINVAL, std::string("gl_quant_w_128x128: ") + why);
  if (rc != 0) return fail(GL_ELAUNCH, std::string("quant_w launch: ") + why);
  return GL_OK;
}

int gl_gmm_fp8_fwd(const void* a_q, const float* a_s, const void* b_q, const float* b_s,
                   const int32_t* group_sizes, int64_t G, int64_t M, int64_t K, int64_t N,
                   void* out, int out_dtype, int* err_word, void* stream) {
  if (!a_q || !a_s || !b_q || !b_s || !group_sizes || !out)
    return fail(GL_EINVAL, "gl_gmm_fp8_fwd: null pointer");
  if (G < 1 || G > 1024) return fail(GL_EINVAL, "gl_gmm_fp8_fwd: need 1 <= G <= 1024");
  if (M < 0 || K <= 0 || N <= 0 || K % 128 != 0 || N % 128 != 0)
    return fail(GL_EINVAL, "gl_gmm_fp8_fwd: need K, N positive multiples of 128");
  if (M > (int64_t(1) << 31) - 256 || G * K > (int64_t(1) << 31) - 256)
    return fail(GL_EINVAL, "gl_gmm_fp8_fwd: M and G*K must fit in 31 bits");
  if (out_dtype != GL_OUT_BF16 && out_dtype != GL_OUT_F32)
    return fail(GL_EINVAL, "gl_gmm_fp8_fwd: out_dtype must be GL_OUT_BF16 or GL_OUT_F32");
  if (!aligned16(a_q) || !aligned16(b_q) || !aligned16(out))
    return fail(GL_EINVAL, "gl_gmm_fp8_fwd: a_q, b_q and out must be 16-byte aligned");
  if (M == 0) return GL_OK;
  DeviceState* d = nullptr;
  if (int rc = device_state(&d)) return rc;
  const char* why = "";
  const int rc = gl_launch_gmm_fp8(a_q, a_s, b_q, b_s, group_sizes, G, M, K, N, out,
                                   out_dtype == GL_OUT_F32, err_word ? err_word : d->err,
                                   static_cast<cudaStream_t>(stream), d->num_sms, &why);
  if (rc == -1) return fail(GL_EINVAL, std::string("gl_gmm_fp8_fwd: ") + why);
  if (rc != 0) return fail(GL_ELAUNCH, std::string("gl_gmm_fp8_fwd: ") + why);
  return GL_OK;
}

int gl_gmm_fp8_fwd_scatter(const void* a_q, const float* a_s, const void* b_q, const float* b_s,
                           const int32_t* group_sizes, int64_t G, int64_t M, int64_t K, int64_t N,
                           void* const* outs, int n_outs, int64_t row_offset, int out_dtype,
                           int* err_word, void* stream) {
  const char* f = "gl_gmm_fp8_fwd_scatter";
  if (!a_q || !a_s || !b_q || !b_s || !group_sizes || !outs)
    return fail(GL_EINVAL, std::string(f) + ": null pointer");
  if (n_outs < 1 || n_outs > GL_MAX_SCATTER_OUTS)
    return fail(GL_EINVAL, std::string(f) + ": need 1 <= n_outs <= GL_MAX_SCATTER_OUTS");
  for (int i = 0; i < n_outs; ++i)
    if (!outs[i] || !aligned16(outs[i]))
      return fail(GL_EINVAL, std::string(f) + ": every output must be a 16-byte aligned pointer");
  if (row_offset < 0) return fail(GL_EINVAL, std::string(f) + ": row_offset must be >= 0");
  if (row_offset + M > (int64_t(1) << 31) - 256)
    return fail(GL_EINVAL, std::string(f) + ": row_offset + M must fit in 31 bits");
  if (G < 1 || G > 1024) return fail(GL_EINVAL, std::string(f) + ": need 1 <= G <= 1024");
  if (M < 0 || K <= 0 || N <= 0 || K % 128 != 0 || N % 128 != 0)
    return fail(GL_EINVAL, std::string(f) + ": need K, N positive multiples of 128");
  if (M > (int64_t(1) << 31) - 256 || G * K > (int64_t(1) << 31) - 256)
    return fail(GL_EINVAL, std::string(f) + ": M and G*K must fit in 31 bits");
  if (out_dtype != GL_OUT_BF16 && out_dtype != GL_OUT_F32)
    return fail(GL_EINVAL, std::string(f) + ": out_dtype must be GL_OUT_BF16 or GL_OUT_F32");
  if (!aligned16(a_q) || !aligned16(b_q))
    return fail(GL_EINVAL, std::string(f) + ": a_q and b_q must be 16-byte aligned");
  if (M == 0) return GL_OK;
  DeviceState* d = nullptr;
  if (int rc = device_state(&d)) return rc;
  const char* why = "";
  const int rc = gl_launch_gmm_fp8_multi(a_q, a_s, b_q, b_s, group_sizes, G, M, K, N, outs, n_outs,
                                         row_offset, out_dtype == GL_OUT_F32,
                                         err_word ? err_word : d->err,
                                         static_cast<cudaStream_t>(stream), d->num_sms, &why);
  if (rc == -1) return fail(GL_EINVAL, std::string(f) + ": " + why);
  if (rc != 0) return fail(GL_ELAUNCH, std::string(f) + ": " + why);
  return GL_OK;
}

// Cross-process peer buffers (CUDA IPC: unicast peer mappings, no multicast).
int gl_ipc_alloc(size_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes == 0) return fail(GL_EINVAL, "gl_ipc_alloc: null pointer or zero size");
  DeviceState* d = nullptr;
  if (int rc = device_state(&d)) return rc;
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) return fail(GL_ELAUNCH, std::string("gl_ipc_alloc: cudaMalloc: ") + cudaGetErrorString(e));
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, *ptr);
  if (e != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return fail(GL_ELAUNCH, std::string("gl_ipc_alloc: cudaIpcGetMemHandle: ") + cudaGetErrorString(e));
  }
  static_assert(sizeof(h) == GL_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  return GL_OK;
}

int gl_ipc_open(const void* handle, void** ptr) {
  if (!ptr || !handle) return fail(GL_EINVAL, "gl_ipc_open: null pointer");
  DeviceState* d = nullptr;
  if (int rc = device_state(&d)) return rc;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(GL_ELAUNCH, std::string("gl_ipc_open: ") + cudaGetErrorString(e));
  return GL_OK;
}

int gl_ipc_close(void* ptr) {
  if (!ptr) return GL_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return fail(GL_ELAUNCH, std::string("gl_ipc_close: ") + cudaGetErrorString(e));
  return GL_OK;
}

int gl_ipc_free(void* ptr) {
  if (!ptr) return GL_OK;
  const cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return fail(GL_ELAUNCH, std::string("gl_ipc_free: ") + cudaGetErrorString(e));
  return GL_OK;
}

static int chunk_gla_check(const char* fn, const void* q, const void* k, const void* v,
                           const float* g, const float* g_gamma, const float* h0, int64_t B,
                           int64_t T, int64_t H, int64_t K, int64_t V, int64_t chunk_size,
                           const void* o, const float* ht) {
  const std::string f(fn);
  if (!q || !k || !v || !o) return fail(GL_EINVAL, f + ": null pointer");
  if ((g == nullptr) == (g_gamma == nullptr))
    return fail(GL_EINVAL, f + ": exactly one of g / g_gamma must be given");
  if (K != 128 || V != 128) return fail(GL_EINVAL, f + ": K and V must be 128");
  if (chunk_size != 64) return fail(GL_EINVAL, f + ": chunk_size must be 64");
  if (B <= 0 || H <= 0 || T <= 0 || T % 64 != 0)
    return fail(GL_EINVAL, f + ": need B, H > 0 and T a positive multiple of 64");
  if (B * T * H > (int64_t(1) << 31) - 1) return fail(GL_EINVAL, f + ": B*T*H must fit in 31 bits");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o) || (g && !aligned16(g)) ||
      (h0 && !aligned16(h0)) || (ht && !aligned16(ht)))
    return fail(GL_EINVAL, f + ": tensors must be 16-byte aligned");
  return GL_OK;
}

int gl_chunk_gla_fwd_scatter(const void* q, const void* k, const void* v, const float* g,
                             const float* g_gamma, const float* h0, float scale, int64_t B,
                             int64_t T, int64_t H, int64_t K, int64_t V, int64_t chunk_size,
                             void* const* outs, int n_outs, float* ht, void* workspace,
                             size_t workspace_bytes, int flags, int* err_word, void* stream) {
  const char* f = "gl_chunk_gla_fwd_scatter";
  if (!outs) return fail(GL_EINVAL, std::string(f) + ": null pointer");
  if (n_outs < 1 || n_outs > GL_MAX_SCATTER_OUTS)
    return fail(GL_EINVAL, std::string(f) + ": need 1 <= n_outs <= GL_MAX_SCATTER_OUTS");
  for (int i = 0; i < n_outs; ++i)
    if (!outs[i] || !aligned16(outs[i]))
      return fail(GL_EINVAL, std::string(f) + ": every output must be a 16-byte aligned pointer");
  if (int rc = chunk_gla_check(f, q, k, v, g, g_gamma, h0, B, T, H, K, V, chunk_size, outs[0], ht))
    return rc;
  if (flags & ~GL_GLA_BF16_INTRA) return fail(GL_EINVAL, std::string(f) + ": unknown flags");
  if (workspace && (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return fail(GL_EINVAL, std::string(f) + ": workspace must be 256-byte aligned");
  DeviceState* d = nullptr;
  if (int rc = device_state(&d)) return rc;
  const char* why = "";
  const int rc = gl_launch_chunk_gla_scatter(q, k, v, g, g_gamma, h0, scale, B, T, H, outs, n_outs,
                                             ht, workspace, workspace ? workspace_bytes : 0,
                                             (flags & GL_GLA_BF16_INTRA) ? 0 : 1,
                                             err_word ? err_word : d->err,
                                             static_cast<cudaStream_t>(stream), d->num_sms, &why);
  if (rc == -1) return fail(GL_EINVAL, std::string(f) + ": " + why);
  if (rc != 0) return fail(GL_ELAUNCH, std::string(f) + ": " + why);
  return GL_OK;
}

int gl_chunk_gla_fwd_ws(const void* q, const void* k, const void* v, const float* g,
                        const float* g_gamma, const float* h0, float scale, int64_t B, int64_t T,
                        int64_t H, int64_t K, int64_t V, int64_t chunk_size, void* o, float* ht,
                        void* workspace, size_t workspace_bytes, int* err_word, void* stream) {
  return gl_chunk_gla_fwd_ex(q, k, v, g, g_gamma, h0, scale, B, T, H, K, V, chunk_size, o, ht,
                             nullptr, workspace, workspace_bytes, 0, err_word, stream);
}

int gl_chunk_gla_fwd(const void* q, const void* k, const void* v, const float* g,
                     const float* g_gamma, const float* h0, float scale, int64_t B, int64_t T,
                     int64_t H, int64_t K, int64_t V, int64_t chunk_size, void* o, float* ht,
                     int* err_word, void* stream) {
  return gl_chunk_gla_fwd_ws(q, k, v, g, g_gamma, h0, scale, B, T, H, K, V, chunk_size, o, ht,
                             nullptr, 0, err_word, stream);
}

size_t gl_chunk_gla_fwd_workspace_bytes(int64_t B, int64_t T, int64_t H, int64_t K, int64_t V,
                                        int64_t chunk_size) {
  if (B <= 0 || H <= 0 || T <= 0 || T % 64 != 0 || K != 128 || V != 128 || chunk_size != 64)
    return 0;
  DeviceState* d = nullptr;
  if (device_state(&d)) return 0;
  return gl_chunk_gla_ws_bytes(B, T, H, d->num_sms);
}

// Per-chunk state rows (B * T/64 * H * 128) are TMA row coordinates (int32).
static bool gla_states_fit(int64_t B, int64_t T, int64_t H) {
  return B * (T / 64) * H * 128 <= (int64_t(1) << 31) - 1;
}

int gl_chunk_gla_fwd_states(const void* q, const void* k, const void* v, const float* g,
                            const float* g_gamma, const float* h0, float scale, int64_t B,
                            int64_t T, int64_t H, int64_t K, int64_t V, int64_t chunk_size,
                            void* o, float* ht, void* h_states, void* workspace,
                            size_t workspace_bytes, int* err_word, void* stream) {
  if (!h_states)
    return fail(GL_EINVAL, "gl_chunk_gla_fwd_states: h_states must be a 16-byte aligned pointer");
  return gl_chunk_gla_fwd_ex(q, k, v, g, g_gamma, h0, scale, B, T, H, K, V, chunk_size, o, ht,
                             h_states, workspace, workspace_bytes, 0, err_word, stream);
}

int gl_chunk_gla_fwd_ex(const void* q, const void* k, const void* v, const float* g,
                        const float* g_gamma, const float* h0, float scale, int64_t B, int64_t T,
                        int64_t H, int64_t K, int64_t V, int64_t chunk_size, void* o, float* ht,
                        void* h_states, void* workspace, size_t workspace_bytes, int flags,
                        int* err_word, void* stream) {
  const char* f = h_states ? "gl_chunk_gla_fwd_states" : "gl_chunk_gla_fwd";
  if (int rc = chunk_gla_check(f, q, k, v, g, g_gamma, h0, B, T, H, K, V, chunk_size, o, ht))
    return rc;
  if (flags & ~GL_GLA_BF16_INTRA) return fail(GL_EINVAL, std::string(f) + ": unknown flags");
  if (h_states && !aligned16(h_states))
    return fail(GL_EINVAL, std::string(f) + ": h_states must be a 16-byte aligned pointer");
  if (h_states && !gla_states_fit(B, T, H))
    return fail(GL_EINVAL, std::string(f) + ": B*T/64*H*128 must fit in 31 bits");
  if (workspace && (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return fail(GL_EINVAL, std::string(f) + ": workspace must be 256-byte aligned");
  DeviceState* d = nullptr;
  if (int rc = device_state(&d)) return rc;
  const char* why = "";
  const int rc = gl_launch_chunk_gla(q, k, v, g, g_gamma, h0, scale, B, T, H, K, V, o, ht,
                                     h_states, workspace, workspace ? workspace_bytes : 0,
                                     (flags & GL_GLA_BF16_INTRA) ? 0 : 1,
                                     err_word ? err_word : d->err,
                                     static_cast<cudaStream_t>(stream), d->num_sms, &why);
  if (rc == -1) return fail(GL_EINVAL, std::string(f) + ": " + why);
  if (rc != 0) return fail(GL_ELAUNCH, std::string(f) + ": " + why);
  return GL_OK;
}

int gl_chunk_gla_fwd_intermediates(const void* q, const void* k, const float* g,
                                   const float* g_gamma, float scale, int64_t B, int64_t T,
                                   int64_t H, int64_t K, int64_t chunk_size, float* g_cumsum,
                                   float* A, int* err_word, void* stream) {
  const char* f = "gl_chunk_gla_fwd_intermediates";
  (void)err_word;  // no device-side waits: nothing is ever written there
  if (!q || !k) return fail(GL_EINVAL, std::string(f) + ": null pointer");
  if (!g_cumsum && !A) return fail(GL_EINVAL, std::string(f) + ": neither g_cumsum nor A requested");
  if ((g == nullptr) == (g_gamma == nullptr))
    return fail(GL_EINVAL, std::string(f) + ": exactly one of g / g_gamma must be given");
  if (K != 128) return fail(GL_EINVAL, std::string(f) + ": K must be 128");
  if (chunk_size != 64) return fail(GL_EINVAL, std::string(f) + ": chunk_size must be 64");
  if (B <= 0 || H <= 0 || T <= 0 || T % 64 != 0)
    return fail(GL_EINVAL, std::string(f) + ": need B, H > 0 and T a positive multiple of 64");
  if (B * T * H > (int64_t(1) << 31) - 1) return fail(GL_EINVAL, std::string(f) + ": B*T*H must fit in 31 bits");
  if ((A && !aligned16(A)) || (g_cumsum && !aligned16(g_cumsum)))
    return fail(GL_EINVAL, std::string(f) + ": outputs must be 16-byte aligned");
  DeviceState* d = nullptr;
  if (int rc = device_state(&d)) return rc;
  const char* why = "";
  const int rc = gl_launch_gla_intermediates(q, k, g, g_gamma, scale, B, T, H, g_cumsum, A,
                                             static_cast<cudaStream_t>(stream), &why);
  if (rc == -1) return fail(GL_EINVAL, std::string(f) + ": " + why);
  if (rc != 0) return fail(GL_ELAUNCH, std::string(f) + ": " + why);
  return GL_OK;
}

// Backward workspace: E (bf16, as h_states) then the reverse scan's split
// records, 256-byte aligned.
static size_t gla_e_bytes(int64_t B, int64_t T, int64_t H) {
  return ((static_cast<size_t>(B * (T / 64) * H) * 128 * 128 * 2 + 255) / 256) * 256;
}

size_t gl_chunk_gla_bwd_workspace_bytes(int64_t B, int64_t T, int64_t H, int64_t K, int64_t V,
                                        int64_t chunk_size) {
  if (B <= 0 || H <= 0 || T <= 0 || T % 64 != 0 || K != 128 || V != 128 || chunk_size != 64)
    return 0;
  DeviceState* d = nullptr;
  if (device_state(&d)) return 0;
  return gla_e_bytes(B, T, H) + gl_chunk_gla_ws_bytes(B, T, H, d->num_sms);
}

int gl_chunk_gla_bwd(const void* q, const void* k, const void* v, const float* g,
                     const float* g_gamma, const void* h_states, const void* dout,
                     const float* dht, float scale, int64_t B, int64_t T, int64_t H, int64_t K,
                     int64_t V, int64_t chunk_size, void* dq, void* dk, void* dv, float* dh0,
                     void* workspace, size_t workspace_bytes, int* err_word, void* stream) {
  const char* f = "gl_chunk_gla_bwd";
  if (int rc = chunk_gla_check(f, q, k, v, g, g_gamma, dht, B, T, H, K, V, chunk_size, dout, dh0))
    return rc;
  if (!h_states || !dq || !dk || !dv) return fail(GL_EINVAL, std::string(f) + ": null pointer");
  if (!aligned16(h_states) || !aligned16(dq) || !aligned16(dk) || !aligned16(dv))
    return fail(GL_EINVAL, std::string(f) + ": tensors must be 16-byte aligned");
  if (!gla_states_fit(B, T, H)) return fail(GL_EINVAL, std::string(f) + ": B*T/64*H*128 must fit in 31 bits");
  const size_t eb = gla_e_bytes(B, T, H);
  if (!workspace || workspace_bytes < eb)
    return fail(GL_EINVAL, std::string(f) + ": workspace smaller than gl_chunk_gla_bwd_workspace_bytes");
  if (reinterpret_cast<uintptr_t>(workspace) & 255u)
    return fail(GL_EINVAL, std::string(f) + ": workspace must be 256-byte aligned");
  DeviceState* d = nullptr;
  if (int rc = device_state(&d)) return rc;
  int* err = err_word ? err_word : d->err;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const char* why = "";
  int rc = gl_launch_chunk_gla_dh(q, dout, g, g_gamma, dht, scale, B, T, H, workspace, dh0,
                                  static_cast<char*>(workspace) + eb, workspace_bytes - eb, err, st,
                                  d->num_sms, &why);
  if (rc == 0)
    rc = gl_launch_chunk_gla_grads(q, k, v, dout, g, g_gamma, h_states, workspace, scale, B, T, H,
                                   dq, dk, dv, err, st, d->num_sms, &why);
  if (rc == -1) return fail(GL_EINVAL, std::string(f) + ": " + why);
  if (rc != 0) return fail(GL_ELAUNCH, std::string(f) + ": " + why);
  return GL_OK;
}

int gl_quant_col_128x1(const void* x, int64_t M, int64_t C, void* q, float* s, int* err_word,
                       void* stream) {
  if (!x || !q || !s) return fail(GL_EINVAL, "gl_quant_col_128x1: null pointer");
  if (M <= 0 || C <= 0 || M % 128 != 0 || C % 128 != 0)
    return fail(GL_EINVAL, "gl_quant_col_128x1: need M and C positive multiples of 128");
  if (!aligned16(x) || !aligned16(q) || !aligned16(s))
    return fail(GL_EINVAL, "gl_quant_col_128x1: x, q and s must be 16-byte aligned");
  DeviceState* d = nullptr;
  if (int rc = device_state(&d)) return rc;
  const char* why = "";
  const int rc = gl_launch_quant_col(x, M, C, q, s, err_word ? err_word : d->err,
                                     static_cast<cudaStream_t>(stream), d->num_sms, &why);
  if (rc == -1) return fail(GL_EINVAL, std::string("gl_quant_col_128x1: ") + why);
  if (rc != 0) return fail(GL_ELAUNCH, std::string("quant_col launch: ") + why);
  return GL_OK;
}

static int gmm_bwd_check(const char* fn, const void* a, const float* as, const void* b,
                         const float* bs, const int32_t* gs, int64_t G, int64_t M, int64_t K,
                         int64_t N, const void* out, int out_dtype) {
  const std::string f(fn);
  if (!a || !as || !b || !bs || !gs || !out) return fail(GL_EINVAL, f + ": null pointer");
  if (G <= 0 || G > 1024) return fail(GL_EINVAL, f + ": need 0 < G <= 1024");
  if (M <= 0 || K <= 0 || N <= 0 || K % 128 != 0 || N % 128 != 0)
    return fail(GL_EINVAL, f + ": need M > 0 and K, N positive multiples of 128");
  if (M > (int64_t(1) << 31) - 1 || G * K > (int64_t(1) << 31) - 1)
    return fail(GL_EINVAL, f + ": M and G*K must fit in 31 bits");
  if (out_dtype != GL_OUT_BF16 && out_dtype != GL_OUT_F32) return fail(GL_EINVAL, f + ": bad out_dtype");
  if (!aligned16(a) || !aligned16(b) || !aligned16(out) || !aligned16(as) || !aligned16(bs))
    return fail(GL_EINVAL, f + ": tensors must be 16-byte aligned");
  return GL_OK;
}

int gl_gmm_fp8_dlhs(const void* dq, const float* ds, const void* b_q, const float* b_s,
                    const int32_t* group_sizes, int64_t G, int64_t M, int64_t K, int64_t N,
                    void* out, int out_dtype, int* err_word, void* stream) {
  if (int rc = gmm_bwd_check("gl_gmm_fp8_dlhs", dq, ds, b_q, b_s, group_sizes, G, M, K, N, out,
                             out_dtype))
    return rc;
  DeviceState* d = nullptr;
  if (int rc = device_state(&d)) return rc;
  const char* why = "";
  // kernel reduction = the weight's N, kernel output = the weight's K
  const int rc = gl_launch_gmm_fp8_dlhs(dq, ds, b_q, b_s, group_sizes, G, M, N, K, out,
                                        out_dtype == GL_OUT_F32, err_word ? err_word : d->err,
                                        static_cast<cudaStream_t>(stream), d->num_sms, &why);
  if (rc == -1) return fail(GL_EINVAL, std::string("gl_gmm_fp8_dlhs: ") + why);
  if (rc != 0) return fail(GL_ELAUNCH, std::string("gl_gmm_fp8_dlhs: ") + why);
  return GL_OK;
}

int gl_tgmm_fp8(const void* lq, const float* ls, const void* dq, const float* ds,
                const int32_t* group_sizes, int64_t G, int64_t M, int64_t K, int64_t N, void* out,
                int out_dtype, int* err_word, void* stream) {
  if (int rc = gmm_bwd_check("gl_tgmm_fp8", lq, ls, dq, ds, group_sizes, G, M, K, N, out, out_dtype))
    return rc;
  if (M % 128 != 0) return fail(GL_EINVAL, "gl_tgmm_fp8: M must be a multiple of 128");
  DeviceState* d = nullptr;
  if (int rc = device_state(&d)) return rc;
  const char* why = "";
  const int rc = gl_launch_tgmm_fp8(lq, ls, dq, ds, group_sizes, G, M, K, N, out,
                                    out_dtype == GL_OUT_F32, err_word ? err_word : d->err,
                                    static_cast<cudaStream_t>(stream), d->num_sms, &why);
  if (rc == -1) return fail(GL_EINVAL, std::string("gl_tgmm_fp8: ") + why);
  if (rc != 0) return fail(GL_ELAUNCH, std::string("gl_tgmm_fp8: ") + why);
  return GL_OK;
}

int gl_device_status(int* err_word, void* stream, int* code) {
  if (!code) return fail(GL_EINVAL, "gl_device_status: null code pointer");
  DeviceState* d = nullptr;
  if (int rc = device_state(&d)) return rc;
  int* w = err_word ? err_word : d->err;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return fail(GL_ELAUNCH, std::string("stream sync: ") + cudaGetErrorString(e));
  int h = 0;
  e = cudaMemcpyAsync(&h, w, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaMemsetAsync(w, 0, sizeof(int), st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return fail(GL_ELAUNCH, std::string("reading error word: ") + cudaGetErrorString(e));
  *code = h;
  return GL_OK;
}

}  // extern "C"
