// Allocation-free grouped FP8 matmul forward from bf16 activations.
//
// Some callers cannot allocate device memory while they run a step: runtimes
// that plan every device buffer before execution and forbid allocation
// inside it (serving engines, plugin hosts), and FFI callers that have no
// device allocator of their own.  gl_gmm_fp8_act_fwd_noalloc serves them:
// the 1x128 activation quantisation writes its e4m3 values and fp32 scales
// into a fixed, file-scope device array owned by this library, and the
// grouped matmul reads them from there.  Nothing is allocated per call; the
// array itself is created when the library's device code is loaded on a GPU
// and held until the process exits.
//
// Limits and sharing:
//   * M * K <= GL_NOALLOC_MAX_ACT_ELEMS (16 Mi activation elements); larger
//     calls are rejected with GL_EINVAL.
//   * Every call on a device shares the one array and it keeps the last
//     call's contents.  Calls whose GPU work overlaps (different streams,
//     host threads or processes sharing a context) race on it; serialise
//     them on one stream.
//   * Device-side errors (invalid group_sizes, a wait that gave up) are
//     reported only through a caller-owned err_word: with NULL they land in
//     the scratch array's own word, which nothing reads back (the library
//     word that gl_device_status(NULL) reads is allocated memory, so this
//     entry point does not use it).
//   * The first call on each device looks up the array's device address
//     (cudaGetSymbolAddress, with that device current); make that first call
//     before any stream capture.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "../../include/glaucis_b200.h"

int gl_launch_quant_act(const void* x, int64_t M, int64_t K, void* q, float* s, int* err,
                        cudaStream_t st, int num_sms, const char** why);
int gl_launch_gmm_fp8(const void* a_q, const float* a_s, const void* b_q, const float* b_s,
                      const int32_t* group_sizes, int64_t G, int64_t M, int64_t K, int64_t N,
                      void* out, int out_f32, int* err, cudaStream_t st, int num_sms,
                      const char** why);
int gl_set_error_message(int code, const char* msg);

namespace {

constexpr size_t kErrBytes = 256;                          // error word, padded
constexpr size_t kQBytes = GL_NOALLOC_MAX_ACT_ELEMS;        // e4m3 activations
constexpr size_t kSBytes = GL_NOALLOC_MAX_ACT_ELEMS / 128 * sizeof(float);  // 1x128 scales
constexpr size_t kScratchBytes = kErrBytes + kQBytes + kSBytes;

// Host code must not use this name as a device address: it is a host-side
// stand-in.  Device addresses come from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

struct DevScratch {
  unsigned char* base = nullptr;  // device address of g_noalloc_scratch
  int num_sms = 0;
};

std::mutex g_mu;
DevScratch g_dev[64];

// Per-device set-up on first use: device address of the scratch array and
// the SM count.  No allocation.
int scratch_for_current_device(DevScratch* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return gl_set_error_message(GL_ELAUNCH, (std::string("cudaGetDevice: ") + cudaGetErrorString(e)).c_str());
  if (dev < 0 || dev >= 64) return gl_set_error_message(GL_ELAUNCH, "device ordinal out of range");
  std::lock_guard<std::mutex> lk(g_mu);
  DevScratch& d = g_dev[dev];
  if (d.base == nullptr) {
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (major != 10 || minor != 0)
      return gl_set_error_message(GL_ELAUNCH, "libglaucis_b200 is built for sm_100a (B200) only");
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return gl_set_error_message(
          GL_ELAUNCH, (std::string("cudaGetSymbolAddress(noalloc scratch): ") + cudaGetErrorString(e)).c_str());
    e = cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess)
      return gl_set_error_message(GL_ELAUNCH, (std::string("cudaDeviceGetAttribute: ") + cudaGetErrorString(e)).c_str());
    d.base = static_cast<unsigned char*>(p);
  }
  *out = d;
  return GL_OK;
}

}  // namespace

extern "C" int gl_gmm_fp8_act_fwd_noalloc(const void* lhs, const void* b_q, const float* b_s,
                                          const int32_t* group_sizes, int64_t G, int64_t M,
                                          int64_t K, int64_t N, void* out, int out_dtype,
                                          int* err_word, void* stream) {
  if (!lhs || !b_q || !b_s || !group_sizes || !out)
    return gl_set_error_message(GL_EINVAL, "gl_gmm_fp8_act_fwd_noalloc: null pointer");
  if (G < 1 || G > 1024)
    return gl_set_error_message(GL_EINVAL, "gl_gmm_fp8_act_fwd_noalloc: need 1 <= G <= 1024");
  if (M < 0 || K <= 0 || N <= 0 || K % 128 != 0 || N % 128 != 0)
    return gl_set_error_message(GL_EINVAL,
                                "gl_gmm_fp8_act_fwd_noalloc: need K, N positive multiples of 128");
  // division form: M * K itself may overflow for huge M
  if (M > static_cast<int64_t>(GL_NOALLOC_MAX_ACT_ELEMS) / K)
    return gl_set_error_message(
        GL_EINVAL,
        ("gl_gmm_fp8_act_fwd_noalloc: M = " + std::to_string(M) + ", K = " + std::to_string(K) +
         ": M*K exceeds the static scratch limit of " + std::to_string(GL_NOALLOC_MAX_ACT_ELEMS) +
         " activation elements; use gl_quant_act_1x128 + gl_gmm_fp8_fwd with caller buffers")
            .c_str());
  if (G * K > (int64_t(1) << 31) - 256)
    return gl_set_error_message(GL_EINVAL, "gl_gmm_fp8_act_fwd_noalloc: G*K must fit in 31 bits");
  if (out_dtype != GL_OUT_BF16 && out_dtype != GL_OUT_F32)
    return gl_set_error_message(GL_EINVAL, "gl_gmm_fp8_act_fwd_noalloc: bad out_dtype");
  if ((reinterpret_cast<uintptr_t>(lhs) & 15u) || (reinterpret_cast<uintptr_t>(b_q) & 15u) ||
      (reinterpret_cast<uintptr_t>(out) & 15u))
    return gl_set_error_message(GL_EINVAL,
                                "gl_gmm_fp8_act_fwd_noalloc: lhs, b_q and out must be 16-byte aligned");
  if (M == 0) return GL_OK;
  DevScratch d;
  if (int rc = scratch_for_current_device(&d)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int* err = err_word;
  if (err == nullptr) {
    // The scratch's own error word keeps the previous call's value: clear it.
    err = reinterpret_cast<int*>(d.base);
    if (cudaMemsetAsync(err, 0, sizeof(int), st) != cudaSuccess)
      return gl_set_error_message(GL_ELAUNCH, "gl_gmm_fp8_act_fwd_noalloc: clearing the error word failed");
  }
  unsigned char* q = d.base + kErrBytes;
  float* s = reinterpret_cast<float*>(d.base + kErrBytes + kQBytes);
  const char* why = "";
  if (gl_launch_quant_act(lhs, M, K, q, s, err, st, d.num_sms, &why) != 0)
    return gl_set_error_message(GL_ELAUNCH, (std::string("gl_gmm_fp8_act_fwd_noalloc: quantiser: ") + why).c_str());
  const int rc = gl_launch_gmm_fp8(q, s, b_q, b_s, group_sizes, G, M, K, N, out,
                                   out_dtype == GL_OUT_F32, err, st, d.num_sms, &why);
  if (rc == -1) return gl_set_error_message(GL_EINVAL, (std::string("gl_gmm_fp8_act_fwd_noalloc: ") + why).c_str());
  if (rc != 0) return gl_set_error_message(GL_ELAUNCH, (std::string("gl_gmm_fp8_act_fwd_noalloc: ") + why).c_str());
  return GL_OK;
}
