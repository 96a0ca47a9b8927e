// noalloc.cu — k-means entry point for callers that cannot allocate device
// memory.
//
// Some hosts own every byte of GPU memory through their own allocator (a
// caching allocator, a fixed arena reserved at start-up, a plugin sandbox
// with a hard memory budget) and must not have a library call cudaMalloc or
// cudaFree behind their back; others cannot afford the implicit device
// synchronisation those calls may cause. `mvr_kmeans_fit_noalloc` serves
// them: the caller passes device inputs and outputs and a stream, and all
// scratch comes from `g_noalloc_scratch`, a fixed array compiled into this
// library. Every GPU that loads the library holds that array until the
// process exits.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "../../include/mvr.h"
#include "mvr_internal.h"
#include "pq_engine.h"

namespace {

constexpr size_t kScratchBytes = (size_t)MVR_NOALLOC_SCRATCH_BYTES;

// Device scratch shared by every call of mvr_kmeans_fit_noalloc on a device.
// In host code this name is a host-side stand-in, not a device address: the
// device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;

// The array's device address belongs to the CUDA context that loaded this
// module, not to the device number: after cudaDeviceReset, or when a host
// makes another context current through the driver API, the old address is
// gone. Each device slot therefore remembers the unique id of the context
// its address was looked up in, and a call made under another context looks
// it up again.
struct ScratchSlot {
  unsigned long long ctx_id = 0;  // 0: not looked up (or no context id available)
  void* addr = nullptr;
  int arch_ok = -1;               // -1 unknown, 0 not an sm_100 device, 1 sm_100
};
ScratchSlot g_slot[kMaxDevices];

// Device address of g_noalloc_scratch in the current device's current
// context. Looked up on the first call on a device (that call should come
// before any stream capture on the device) and again whenever the current
// context is not the one of the cached address. The device must be an
// sm_100 GPU, the only architecture this library is built for.
int scratch_address(int device, unsigned char** out) {
  if (device < 0 || device >= kMaxDevices) return MVR_E_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  ScratchSlot& s = g_slot[device];
  if (s.arch_ok < 0) {
    int major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device) != cudaSuccess) {
      (void)cudaGetLastError();
      return MVR_E_NO_DEVICE;
    }
    s.arch_ok = (major == 10 && minor == 0) ? 1 : 0;
  }
  if (!s.arch_ok) return MVR_E_NO_DEVICE;
  const unsigned long long id = mvr::current_context_id();
  if (id == 0 || s.addr == nullptr || s.ctx_id != id) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      (void)cudaGetLastError();
      s.addr = nullptr;
      s.ctx_id = 0;
      return MVR_E_CUDA;
    }
    s.addr = p;
    s.ctx_id = mvr::current_context_id();  // the lookup binds the device's context if none was current
  }
  *out = static_cast<unsigned char*>(s.addr);
  return MVR_OK;
}

}  // namespace

extern "C" int mvr_kmeans_fit_noalloc(const float* d_vectors, uint64_t vectors_len, uint32_t dim,
                                      uint32_t k, uint32_t max_iters, float tol, uint64_t seed,
                                      float* d_centroids_out, uint32_t* d_assignments_out,
                                      float* wcss_out, uint32_t* iters_run_out, void* cuda_stream) {
  // kmeans.fit's own validation first, in its order.
  if (k == 0) return MVR_E_KMEANS_BUDGET_TOO_SMALL;
  if (dim == 0) return MVR_E_DIM_MISMATCH;
  if (vectors_len == 0) return MVR_E_EMPTY_VECTOR_SET;
  if (vectors_len % dim != 0) return MVR_E_DIM_MISMATCH;
  if (!d_vectors || !d_centroids_out) return MVR_E_INVALID_ARGUMENT;
  if (dim != 1 && dim != 2 && dim != 4) return MVR_E_INVALID_ARGUMENT;
  if (k > MVR_PQ_CENTROIDS) return MVR_E_INVALID_ARGUMENT;
  const uint64_t n = vectors_len / dim;
  if (n > MVR_NOALLOC_MAX_ROWS) return MVR_E_INVALID_ARGUMENT;

  mvr::PqJob job;
  job.R = d_vectors;
  job.N = n;
  job.D = (int)dim;
  job.M = 1;
  job.S = (int)dim;
  job.K = (int)k;
  job.seed = seed;
  job.max_iters = max_iters;
  job.tol = tol;
  // The grid (and with it the histogram part of the scratch) is sized for at
  // most 160 SMs, which bounds the scratch for any device.
  const int sms = std::min(mvr::sm_count_current_device(), 160);
  const mvr::PqLayout L = mvr::pq_layout(n, 1, (int)dim, (int)k, sms);
  if (L.total_bytes > kScratchBytes || L.small_bytes > 16384) return MVR_E_INVALID_ARGUMENT;

  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) {
    (void)cudaGetLastError();
    return MVR_E_NO_DEVICE;
  }
  unsigned char* ws = nullptr;
  const int st = scratch_address(device, &ws);
  if (st != MVR_OK) return st;

  alignas(16) unsigned char hsmall[16384];  // host mirror of the bookkeeping block
  float wcss = 0.f;
  uint32_t iters = 0;
  mvr::PqOut out;
  out.d_codebooks = d_centroids_out;
  out.d_assign = d_assignments_out;
  out.h_wcss = &wcss;
  out.h_iters = &iters;
  const int rc = mvr::pq_kmeans_run(nullptr, static_cast<cudaStream_t>(cuda_stream), job, out, ws, hsmall, sms);
  if (rc != MVR_OK) return rc;
  if (wcss_out) *wcss_out = wcss;
  if (iters_run_out) *iters_run_out = iters;
  return MVR_OK;
}
