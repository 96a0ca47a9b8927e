// mvr_capi.cu — the extern "C" entry points declared in include/mvr.h.
//
// Host-pointer entry points stage inputs into context-owned device buffers,
// run the device path and copy results back. There is no CPU fallback: a
// missing or unusable GPU is reported as MVR_E_NO_DEVICE / MVR_E_CUDA.
#include <cuda.h>  // driver types only: the driver calls come from cudaGetDriverEntryPointByVersion
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/mvr.h"
#include "comm.h"
#include "mvr_internal.h"
#include "pq_engine.h"
#include "tac_engine.h"

namespace mvr {

namespace {
thread_local std::string* tl_error_sink = nullptr;

using CtxGetCurrentFn = CUresult(CUDAAPI*)(CUcontext*);
using CtxGetIdFn = CUresult(CUDAAPI*)(CUcontext, unsigned long long*);
std::mutex g_ctx_id_mu;
std::mutex g_smem_mu;
std::map<std::pair<const void*, unsigned long long>, size_t> g_smem_set;
}  // namespace

unsigned long long current_context_id() {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_ctx_id_mu);
    static bool looked_up = false;
    if (!looked_up) {
      looked_up = true;
      cudaDriverEntryPointQueryResult q1 = cudaDriverEntryPointSymbolNotFound, q2 = cudaDriverEntryPointSymbolNotFound;
      if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", reinterpret_cast<void**>(&get_current), 12000,
                                           cudaEnableDefault, &q1) != cudaSuccess ||
          q1 != cudaDriverEntryPointSuccess)
        get_current = nullptr;
      if (cudaGetDriverEntryPointByVersion("cuCtxGetId", reinterpret_cast<void**>(&get_id), 12000,
                                           cudaEnableDefault, &q2) != cudaSuccess ||
          q2 != cudaDriverEntryPointSuccess)
        get_id = nullptr;
      (void)cudaGetLastError();
    }
  }
  if (!get_current || !get_id) return 0;
  CUcontext c = nullptr;
  unsigned long long id = 0;
  if (get_current(&c) != CUDA_SUCCESS || c == nullptr || get_id(c, &id) != CUDA_SUCCESS) return 0;
  return id;
}

cudaError_t raise_smem_limit(const void* func, size_t bytes) {
  const unsigned long long id = current_context_id();
  std::lock_guard<std::mutex> lock(g_smem_mu);
  if (id == 0) {  // no context id: ask the function itself
    cudaFuncAttributes a{};
    const cudaError_t q = cudaFuncGetAttributes(&a, func);
    if (q != cudaSuccess) return q;
    if ((size_t)a.maxDynamicSharedSizeBytes >= bytes) return cudaSuccess;
    return cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  }
  size_t& have = g_smem_set[{func, id}];
  if (have >= bytes) return cudaSuccess;
  const cudaError_t e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e == cudaSuccess) have = bytes;
  return e;
}

ErrorSink::ErrorSink(std::string* msg) : prev(tl_error_sink) { tl_error_sink = msg; }
ErrorSink::~ErrorSink() { tl_error_sink = prev; }

DeviceScope::DeviceScope(Ctx* c) : dev(c->device) {
  if (cudaGetDevice(&prev) != cudaSuccess) {
    (void)cudaGetLastError();
    prev = -1;
  }
  if (prev != dev) {
    const cudaError_t e = cudaSetDevice(dev);
    if (e != cudaSuccess) status = cuda_fail(c, e, "cudaSetDevice");
  }
}

DeviceScope::~DeviceScope() {
  if (prev >= 0 && prev != dev) cudaSetDevice(prev);
}

int fail(Ctx* ctx, int status, const std::string& msg) {
  if (tl_error_sink)
    *tl_error_sink = msg;
  else if (ctx)
    ctx->last_error = msg;
  return status;
}

int cuda_fail(Ctx* ctx, cudaError_t e, const char* what) {
  std::string msg = std::string(what) + ": " + cudaGetErrorString(e);
  if (e == cudaErrorMemoryAllocation) {
    (void)cudaGetLastError();
    return fail(ctx, MVR_E_OUT_OF_MEMORY, msg);
  }
  return fail(ctx, MVR_E_CUDA, msg);
}

int scratch(Ctx* ctx, int slot, size_t bytes, void** out) {
  DevBuf& b = ctx->slots[slot];
  if (bytes == 0) bytes = 256;
  if (b.bytes < bytes) {
    if (b.ptr) {
      cudaError_t e = cudaStreamSynchronize(ctx->stream);
      if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaStreamSynchronize");
      cudaFree(b.ptr);
      b.ptr = nullptr;
      b.bytes = 0;
    }
    cudaError_t e = cudaMalloc(&b.ptr, bytes);
    if (e != cudaSuccess) {
      b.ptr = nullptr;
      return cuda_fail(ctx, e, "cudaMalloc(scratch)");
    }
    b.bytes = bytes;
  }
  *out = b.ptr;
  return MVR_OK;
}

int side_stream(Ctx* ctx, cudaStream_t* out) {
  if (!ctx->side) {
    MVR_CUDA(ctx, cudaStreamCreateWithFlags(&ctx->side, cudaStreamNonBlocking));
    MVR_CUDA(ctx, cudaEventCreateWithFlags(&ctx->fork_ev, cudaEventDisableTiming));
    MVR_CUDA(ctx, cudaEventCreateWithFlags(&ctx->join_ev, cudaEventDisableTiming));
  }
  *out = ctx->side;
  return MVR_OK;
}

int tac_events(Ctx* ctx, cudaEvent_t** out) {
  for (auto& e : ctx->tev)
    if (!e) MVR_CUDA(ctx, cudaEventCreate(&e));
  *out = ctx->tev;
  return MVR_OK;
}

int pinned(Ctx* ctx, size_t bytes, void** out) {
  if (ctx->pinned_bytes < bytes) {
    if (ctx->pinned) cudaFreeHost(ctx->pinned);
    ctx->pinned = nullptr;
    ctx->pinned_bytes = 0;
    cudaError_t e = cudaMallocHost(&ctx->pinned, bytes);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaMallocHost");
    ctx->pinned_bytes = bytes;
  }
  *out = ctx->pinned;
  return MVR_OK;
}

namespace {

int h2d(Ctx* c, void* d, const void* h, size_t bytes) { return h2d_staged(c, d, h, bytes); }

int d2h(Ctx* c, void* h, const void* d, size_t bytes) { return d2h_staged(c, h, d, bytes); }

// storage.residualsAndNormsChunk (src/index/storage.zig:255-278): one
// thread per row, coordinates summed in order.
__global__ void residuals_norms_kernel(const float* __restrict__ v, const float* __restrict__ cent,
                                       const uint32_t* __restrict__ asg, uint64_t n, uint32_t dim,
                                       float* __restrict__ res, float* __restrict__ norms) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const float* vi = v + i * dim;
    const float* ci = cent + (uint64_t)asg[i] * dim;
    float* ri = res + i * dim;
    float sum = 0.f;
    for (uint32_t d = 0; d < dim; ++d) {
      const float diff = __fsub_rn(vi[d], ci[d]);
      ri[d] = diff;
      sum = __fadd_rn(sum, __fmul_rn(diff, diff));
    }
    const float norm = __fsqrt_rn(sum);
    norms[i] = norm;
    if (norm > 0.f) {
      const float inv = __fdiv_rn(1.0f, norm);
      for (uint32_t d = 0; d < dim; ++d) ri[d] = __fmul_rn(ri[d], inv);
    }
  }
}

int pq_validate(Ctx* c, uint64_t len, uint32_t dim, uint32_t pq_m) {
  // pq.train validation order (src/index/pq.zig:165-168)
  if (dim == 0) return fail(c, MVR_E_DIM_MISMATCH, "dim == 0");
  if (pq_m == 0 || dim % pq_m != 0) return fail(c, MVR_E_DIM_NOT_DIVISIBLE_BY_M, "dim % pq_m != 0");
  if (len == 0) return fail(c, MVR_E_EMPTY_CORPUS, "empty residual set");
  if (len % dim != 0) return fail(c, MVR_E_DIM_MISMATCH, "residuals_len % dim != 0");
  return MVR_OK;
}

}  // namespace
}  // namespace mvr

using mvr::Ctx;

extern "C" {

const char* mvr_status_name(int s) {
  switch (s) {
    case MVR_OK: return "Ok";
    case MVR_E_KMEANS_BUDGET_TOO_SMALL: return "KmeansBudgetTooSmall";
    case MVR_E_EMPTY_VECTOR_SET: return "EmptyVectorSet";
    case MVR_E_DIM_MISMATCH: return "DimMismatch";
    case MVR_E_DIM_NOT_DIVISIBLE_BY_M: return "DimNotDivisibleByM";
    case MVR_E_EMPTY_CORPUS: return "EmptyCorpus";
    case MVR_E_OUT_BUFFER_WRONG_SIZE: return "OutBufferWrongSize";
    case MVR_E_NQ_MISMATCH: return "NQMismatch";
    case MVR_E_EMPTY_DISTRIBUTION: return "EmptyDistribution";
    case MVR_E_NON_FINITE: return "NonFinite";
    case MVR_E_ALL_ZERO: return "AllZero";
    case MVR_E_BUDGET_TOO_SMALL: return "BudgetTooSmall";
    case MVR_E_BUDGET_TOO_LARGE: return "BudgetTooLarge";
    case MVR_E_INVALID_THRESHOLDS: return "InvalidThresholds";
    case MVR_E_EMPTY_TOKEN_DUMP: return "EmptyTokenDump";
    case MVR_E_LENGTH_MISMATCH: return "LengthMismatch";
    case MVR_E_EMPTY_INPUT: return "EmptyInput";
    case MVR_E_OUT_OF_MEMORY: return "OutOfMemory";
    case MVR_E_BUFFER_TOO_SMALL: return "BufferTooSmall";
    case MVR_E_QUERY_SHAPE_MISMATCH: return "QueryShapeMismatch";
    case MVR_E_TABLE_SIZE_MISMATCH: return "TableSizeMismatch";
    case MVR_E_DOC_OUT_OF_RANGE: return "DocOutOfRange";
    case MVR_E_DOC_LAYOUT_CORRUPT: return "DocLayoutCorrupt";
    case MVR_E_INVALID_INDEX: return "InvalidIndex";
    case MVR_E_UNSUPPORTED_VERSION: return "UnsupportedVersion";
    case MVR_E_INDEX_CORRUPT: return "IndexCorrupt";
    case MVR_E_ASSIGNMENT_OUT_OF_RANGE: return "AssignmentOutOfRange";
    case MVR_E_DOC_OFFSETS_BAD: return "DocOffsetsBad";
    case MVR_E_KAPPA_ZERO: return "KappaZero";
    case MVR_E_CUDA: return "CudaError";
    case MVR_E_NCCL: return "NcclError";
    case MVR_E_TIMEOUT: return "Timeout";
    case MVR_E_INVALID_ARGUMENT: return "InvalidArgument";
    case MVR_E_NO_DEVICE: return "NoDevice";
    case MVR_E_DEVICE_LIMIT: return "DeviceLimit";
    default: return "Unknown";
  }
}

int mvr_ctx_create(int device_ordinal, mvr_ctx** out) {
  if (!out) return MVR_E_INVALID_ARGUMENT;
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n <= device_ordinal || device_ordinal < 0) {
    (void)cudaGetLastError();
    return MVR_E_NO_DEVICE;
  }
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device_ordinal) != cudaSuccess) return MVR_E_NO_DEVICE;
  if (prop.major < 10) return MVR_E_NO_DEVICE;  // built for sm_100a only
  auto* h = new (std::nothrow) mvr_ctx;
  if (!h) return MVR_E_OUT_OF_MEMORY;
  Ctx* c = &h->impl;
  c->device = device_ordinal;
  c->sm_count = prop.multiProcessorCount;
  {
    mvr::DeviceScope dev_scope(c);  // the stream belongs to the context's device; the caller's stays current
    if (dev_scope.status != MVR_OK ||
        cudaStreamCreateWithFlags(&c->own_stream, cudaStreamNonBlocking) != cudaSuccess) {
      delete h;
      return MVR_E_CUDA;
    }
  }
  c->stream = c->own_stream;
  *out = h;
  return MVR_OK;
}

int mvr_ctx_destroy(mvr_ctx* h) {
  if (!h) return MVR_OK;
  Ctx* c = &h->impl;
  mvr::DeviceScope dev_scope(c);
  cudaStreamSynchronize(c->stream);
  for (auto& b : c->slots)
    if (b.ptr) cudaFree(b.ptr);
  if (c->pinned) cudaFreeHost(c->pinned);
  for (auto& e : c->ev)
    if (e) cudaEventDestroy(e);
  for (auto& t : c->pq_timing) {
    for (auto& e : t.phase)
      if (e) cudaEventDestroy(e);
    for (auto e : t.pool) cudaEventDestroy(e);
  }
  for (auto& e : c->pev)
    if (e) cudaEventDestroy(e);
  if (c->side) {
    cudaStreamSynchronize(c->side);
    cudaStreamDestroy(c->side);
  }
  if (c->tc_diag) cudaFree(c->tc_diag);
  mvr::destroy_comm(c);
  mvr::destroy_host_io(c);
  for (auto& e : c->tev)
    if (e) cudaEventDestroy(e);
  if (c->fork_ev) cudaEventDestroy(c->fork_ev);
  if (c->join_ev) cudaEventDestroy(c->join_ev);
  if (c->own_stream) cudaStreamDestroy(c->own_stream);
  delete h;
  return MVR_OK;
}

int mvr_ctx_set_serial_draws(mvr_ctx* h, int on) {
  if (!h) return MVR_E_INVALID_ARGUMENT;
  h->impl.serial_draws = on != 0;
  return MVR_OK;
}

int mvr_ctx_set_tensor_filter(mvr_ctx* h, int on) {
  if (!h) return MVR_E_INVALID_ARGUMENT;
  h->impl.tc_filter = on != 0;
  return MVR_OK;
}

int mvr_ctx_set_wait_limit(mvr_ctx* h, uint32_t polls) {
  if (!h) return MVR_E_INVALID_ARGUMENT;
  h->impl.wait_limit = polls;
  return MVR_OK;
}

int mvr_ctx_set_pq_tensor_filter(mvr_ctx* h, int on) {
  if (!h) return MVR_E_INVALID_ARGUMENT;
  h->impl.pq_tc_filter = on != 0;
  return MVR_OK;
}

int mvr_ctx_filter_report(mvr_ctx* h, uint64_t* violations, uint64_t* rows_rechecked) {
  if (!h) return MVR_E_INVALID_ARGUMENT;
  Ctx* c = &h->impl;
  uint32_t dg[4] = {0, 0, 0, 0};
  if (c->tc_diag) {
    mvr::DeviceScope dev_scope(c);
  MVR_TRY(dev_scope.status);
    MVR_CUDA(c, cudaMemcpyAsync(dg, c->tc_diag, sizeof(dg), cudaMemcpyDeviceToHost, c->stream));
    MVR_CUDA(c, cudaStreamSynchronize(c->stream));
  }
  if (violations) *violations = dg[0];
  if (rows_rechecked) *rows_rechecked = dg[1];
  return dg[2] ? mvr::fail(c, MVR_E_TIMEOUT, "tensor-core filter: an MMA did not complete in time") : MVR_OK;
}

int mvr_ctx_set_candidate_scan(mvr_ctx* h, int on) {
  if (!h) return MVR_E_INVALID_ARGUMENT;
  h->impl.cand_scan = on != 0;
  return MVR_OK;
}

int mvr_ctx_set_pq_groups(mvr_ctx* h, int groups) {
  if (!h || groups < 1 || groups > 2) return MVR_E_INVALID_ARGUMENT;
  h->impl.pq_groups = groups;
  return MVR_OK;
}

int mvr_ctx_set_exhaustive_assign(mvr_ctx* h, int on) {
  if (!h) return MVR_E_INVALID_ARGUMENT;
  h->impl.exhaustive_assign = on != 0;
  return MVR_OK;
}

int mvr_tac_last_stats(const mvr_ctx* h, mvr_tac_stats* out) {
  if (!h || !out) return MVR_E_INVALID_ARGUMENT;
  *out = h->impl.tac_stats;
  return MVR_OK;
}

const char* mvr_last_error(const mvr_ctx* h) { return h ? h->impl.last_error.c_str() : ""; }

int mvr_ctx_set_stream(mvr_ctx* h, void* s) {
  if (!h) return MVR_E_INVALID_ARGUMENT;
  h->impl.stream = s ? (cudaStream_t)s : h->impl.own_stream;
  return MVR_OK;
}

int mvr_ctx_trim(mvr_ctx* h) {
  if (!h) return MVR_E_INVALID_ARGUMENT;
  Ctx* c = &h->impl;
  mvr::DeviceScope dev_scope(c);
  MVR_TRY(dev_scope.status);
  MVR_CUDA(c, cudaStreamSynchronize(c->stream));
  for (auto& b : c->slots) {
    if (b.ptr) cudaFree(b.ptr);
    b.ptr = nullptr;
    b.bytes = 0;
  }
  return MVR_OK;
}

int mvr_ctx_sync(mvr_ctx* h) {
  if (!h) return MVR_E_INVALID_ARGUMENT;
  Ctx* c = &h->impl;
  MVR_CUDA(c, cudaStreamSynchronize(c->stream));
  MVR_CUDA(c, cudaGetLastError());
  return MVR_OK;
}

// ---- pq.train -------------------------------------------------------------

int mvr_pq_train_device(mvr_ctx* h, const float* d_res, uint64_t len, uint32_t dim, uint64_t seed,
                        uint32_t n_threads, uint32_t pq_m, uint32_t max_iters, float tol,
                        float* d_cb, mvr_pq_train_stats* stats) {
  (void)n_threads;
  if (!h) return MVR_E_INVALID_ARGUMENT;
  Ctx* c = &h->impl;
  MVR_TRY(mvr::pq_validate(c, len, dim, pq_m));
  if (!d_res || !d_cb) return mvr::fail(c, MVR_E_INVALID_ARGUMENT, "null pointer");
  mvr::DeviceScope dev_scope(c);
  MVR_TRY(dev_scope.status);
  mvr::PqJob job;
  job.R = d_res;
  job.N = len / dim;
  job.D = (int)dim;
  job.M = (int)pq_m;
  job.S = (int)(dim / pq_m);
  job.K = (int)MVR_PQ_CENTROIDS;
  job.seed = seed;
  job.max_iters = max_iters;
  job.tol = tol;
  mvr::PqOut out;
  out.d_codebooks = d_cb;
  out.stats = stats;
  return mvr::pq_kmeans_device(c, job, out);
}

int mvr_pq_train_sharded_device(mvr_ctx* h, const float* d_rows, uint64_t n_local, uint64_t row0,
                                uint64_t n_total, uint32_t dim, uint64_t seed, uint32_t n_threads, uint32_t pq_m,
                                uint32_t max_iters, float tol, float* d_cb, uint32_t* d_assign_out,
                                mvr_pq_train_stats* stats) {
  (void)n_threads;
  if (!h) return MVR_E_INVALID_ARGUMENT;
  Ctx* c = &h->impl;
  // pq.train's validation on the global shape (pq.zig:165-168)
  MVR_TRY(mvr::pq_validate(c, n_total * (uint64_t)dim, dim, pq_m));
  mvr::DeviceScope dev_scope(c);
  MVR_TRY(dev_scope.status);
  mvr::PqJob job;
  job.R = d_rows;
  job.N = n_local;
  job.D = (int)dim;
  job.M = (int)pq_m;
  job.S = (int)(dim / pq_m);
  job.K = (int)MVR_PQ_CENTROIDS;
  job.seed = seed;
  job.max_iters = max_iters;
  job.tol = tol;
  mvr::PqOut out;
  out.d_codebooks = d_cb;
  out.d_assign = d_assign_out;
  out.stats = stats;
  if (!mvr::comm_active(c)) {  // one rank: the whole matrix
    if (!d_rows || !d_cb) return mvr::fail(c, MVR_E_INVALID_ARGUMENT, "null pointer");
    if (row0 != 0 || n_local != n_total)
      return mvr::fail(c, MVR_E_INVALID_ARGUMENT, "without a communicator the shard is the whole matrix");
    return mvr::pq_kmeans_device(c, job, out);
  }
  // subspaces are independent problems: with at least one per rank each rank
  // trains whole subspaces (one exchange before, one gather after); with
  // fewer subspaces than ranks the rows are split and every step exchanges
  if ((int)pq_m >= mvr::comm_size(c)) return mvr::pq_kmeans_run_subspaces(c, job, row0, n_total, out, d_rows && d_cb);
  return mvr::pq_kmeans_run_dist(c, job, row0, n_total, out, d_rows && d_cb);
}

int mvr_pq_train(mvr_ctx* h, const float* res, uint64_t len, uint32_t dim, uint64_t seed,
                 uint32_t n_threads, uint32_t pq_m, uint32_t max_iters, float tol, float* cb_out,
                 mvr_pq_train_stats* stats) {
  if (!h) return MVR_E_INVALID_ARGUMENT;
  Ctx* c = &h->impl;
  MVR_TRY(mvr::pq_validate(c, len, dim, pq_m));
  if (!res || !cb_out) return mvr::fail(c, MVR_E_INVALID_ARGUMENT, "null pointer");
  mvr::DeviceScope dev_scope(c);
  MVR_TRY(dev_scope.status);
  float* d_res = nullptr;
  float* d_cb = nullptr;
  const size_t cb_floats = (size_t)MVR_PQ_CENTROIDS * dim;  // pq_m * 256 * sub_dim
  MVR_TRY(mvr::scratch(c, mvr::kSlotResiduals, len * sizeof(float), (void**)&d_res));
  MVR_TRY(mvr::scratch(c, mvr::kSlotCodebooks, cb_floats * sizeof(float), (void**)&d_cb));
  MVR_TRY(mvr::h2d(c, d_res, res, len * sizeof(float)));
  MVR_TRY(mvr_pq_train_device(h, d_res, len, dim, seed, n_threads, pq_m, max_iters, tol, d_cb, stats));
  MVR_TRY(mvr::d2h(c, cb_out, d_cb, cb_floats * sizeof(float)));
  MVR_CUDA(c, cudaStreamSynchronize(c->stream));
  return MVR_OK;
}

// ---- PQ.encode / decode ---------------------------------------------------

int mvr_pq_encode_device(mvr_ctx* h, const float* d_cb, uint32_t dim, uint32_t pq_m,
                         const float* d_res, uint64_t n, uint8_t* d_codes) {
  if (!h) return MVR_E_INVALID_ARGUMENT;
  Ctx* c = &h->impl;
  if (dim == 0) return mvr::fail(c, MVR_E_DIM_MISMATCH, "dim == 0");
  if (pq_m == 0 || dim % pq_m != 0) return mvr::fail(c, MVR_E_DIM_NOT_DIVISIBLE_BY_M, "dim % pq_m != 0");
  if (n == 0) return MVR_OK;
  if (!d_cb || !d_res || !d_codes) return mvr::fail(c, MVR_E_INVALID_ARGUMENT, "null pointer");
  mvr::DeviceScope dev_scope(c);
  MVR_TRY(dev_scope.status);
  return mvr::pq_encode_device(c, d_cb, (int)dim, (int)pq_m, d_res, n, d_codes);
}

int mvr_pq_encode(mvr_ctx* h, const float* cb, uint32_t dim, uint32_t pq_m, const float* res,
                  uint64_t n, uint8_t* codes_out) {
  if (!h) return MVR_E_INVALID_ARGUMENT;
  Ctx* c = &h->impl;
  if (dim == 0) return mvr::fail(c, MVR_E_DIM_MISMATCH, "dim == 0");
  if (pq_m == 0 || dim % pq_m != 0) return mvr::fail(c, MVR_E_DIM_NOT_DIVISIBLE_BY_M, "dim % pq_m != 0");
  if (n == 0) return MVR_OK;
  if (!cb || !res || !codes_out) return mvr::fail(c, MVR_E_INVALID_ARGUMENT, "null pointer");
  mvr::DeviceScope dev_scope(c);
  MVR_TRY(dev_scope.status);
  float* d_res = nullptr;
  float* d_cb = nullptr;
  uint8_t* d_codes = nullptr;
  const size_t cb_floats = (size_t)MVR_PQ_CENTROIDS * dim;
  MVR_TRY(mvr::scratch(c, mvr::kSlotResiduals, n * dim * sizeof(float), (void**)&d_res));
  MVR_TRY(mvr::scratch(c, mvr::kSlotCodebooks, cb_floats * sizeof(float), (void**)&d_cb));
  MVR_TRY(mvr::scratch(c, mvr::kSlotCodes, n * pq_m, (void**)&d_codes));
  MVR_TRY(mvr::h2d(c, d_cb, cb, cb_floats * sizeof(float)));
  constexpr uint64_t kPipeRows = 1ull << 18;
  if (n >= 2 * kPipeRows && mvr::host_is_pinned(res)) {
    // page-locked rows: copied in up to 8 chunks on the side stream, each
    // chunk encoded on the context stream as soon as it has landed (every
    // row's code is independent of the others)
    cudaStream_t s2 = nullptr;
    MVR_TRY(mvr::side_stream(c, &s2));
    const uint64_t nch = std::min<uint64_t>(8, (n + kPipeRows - 1) / kPipeRows);
    const uint64_t per = (n + nch - 1) / nch;
    cudaEvent_t evs[9] = {};
    struct EvFree {
      cudaEvent_t* e;
      ~EvFree() {
        for (int i = 0; i < 9; ++i)
          if (e[i]) cudaEventDestroy(e[i]);
      }
    } evfree{evs};
    for (uint64_t i = 0; i <= nch; ++i) MVR_CUDA(c, cudaEventCreateWithFlags(&evs[i], cudaEventDisableTiming));
    MVR_CUDA(c, cudaEventRecord(evs[nch], c->stream));  // the side stream follows the context stream's earlier work
    MVR_CUDA(c, cudaStreamWaitEvent(s2, evs[nch], 0));
    for (uint64_t i = 0; i < nch; ++i) {
      const uint64_t off = i * per, cnt = std::min(per, n - off);
      MVR_CUDA(c, cudaMemcpyAsync(d_res + off * dim, res + off * dim, cnt * dim * sizeof(float),
                                  cudaMemcpyHostToDevice, s2));
      MVR_CUDA(c, cudaEventRecord(evs[i], s2));
    }
    for (uint64_t i = 0; i < nch; ++i) {
      const uint64_t off = i * per, cnt = std::min(per, n - off);
      MVR_CUDA(c, cudaStreamWaitEvent(c->stream, evs[i], 0));
      MVR_TRY(mvr::pq_encode_device(c, d_cb, (int)dim, (int)pq_m, d_res + off * dim, cnt, d_codes + off * pq_m));
    }
  } else {
    MVR_TRY(mvr::h2d(c, d_res, res, n * dim * sizeof(float)));
    MVR_TRY(mvr::pq_encode_device(c, d_cb, (int)dim, (int)pq_m, d_res, n, d_codes));
  }
  if (c->tc_filter && c->pq_tc_filter && !c->exhaustive_assign && c->tc_diag) {
    uint32_t dg[4] = {0, 0, 0, 0};
    MVR_CUDA(c, cudaMemcpyAsync(dg, c->tc_diag, sizeof(dg), cudaMemcpyDeviceToHost, c->stream));
    MVR_CUDA(c, cudaStreamSynchronize(c->stream));
    if (dg[2]) return mvr::fail(c, MVR_E_TIMEOUT, "tensor-core filter: an MMA did not complete in time");
    if (dg[0] > c->tc_viol_seen) {  // a winner broke the filter's error bound: encode again exactly
      c->tc_viol_seen = dg[0];
      c->tc_filter = false;
      const int s2 = mvr::pq_encode_device(c, d_cb, (int)dim, (int)pq_m, d_res, n, d_codes);
      c->tc_filter = true;
      MVR_TRY(s2);
    }
  }
  MVR_TRY(mvr::d2h(c, codes_out, d_codes, n * pq_m));
  MVR_CUDA(c, cudaStreamSynchronize(c->stream));
  return MVR_OK;
}

int mvr_pq_decode(const float* cb, uint32_t dim, uint32_t pq_m, const uint8_t* codes, uint64_t n,
                  float* out) {
  if (dim == 0) return MVR_E_DIM_MISMATCH;
  if (pq_m == 0 || dim % pq_m != 0) return MVR_E_DIM_NOT_DIVISIBLE_BY_M;
  if (n == 0) return MVR_OK;
  if (!cb || !codes || !out) return MVR_E_INVALID_ARGUMENT;
  const uint32_t s = dim / pq_m;
  for (uint64_t i = 0; i < n; ++i)
    for (uint32_t m = 0; m < pq_m; ++m)
      std::memcpy(out + i * dim + (uint64_t)m * s,
                  cb + ((uint64_t)m * MVR_PQ_CENTROIDS + codes[i * pq_m + m]) * s, sizeof(float) * s);
  return MVR_OK;
}

// ---- kmeans.fit -----------------------------------------------------------

int mvr_kmeans_fit(mvr_ctx* h, const float* vectors, uint64_t len, uint32_t dim, uint32_t k,
                   uint32_t max_iters, float tol, uint64_t seed, uint32_t n_threads,
                   float* centroids_out, uint32_t* assignments_out, float* wcss_out,
                   uint32_t* iters_out) {
  (void)n_threads;
  if (!h) return MVR_E_INVALID_ARGUMENT;
  Ctx* c = &h->impl;
  // kmeans.fit validation order (src/tac/kmeans.zig:73-76)
  if (k == 0) return mvr::fail(c, MVR_E_KMEANS_BUDGET_TOO_SMALL, "k == 0");
  if (dim == 0) return mvr::fail(c, MVR_E_DIM_MISMATCH, "dim == 0");
  if (len == 0) return mvr::fail(c, MVR_E_EMPTY_VECTOR_SET, "no vectors");
  if (len % dim != 0) return mvr::fail(c, MVR_E_DIM_MISMATCH, "vectors_len % dim != 0");
  if (!vectors || !centroids_out) return mvr::fail(c, MVR_E_INVALID_ARGUMENT, "null pointer");
  mvr::DeviceScope dev_scope(c);
  MVR_TRY(dev_scope.status);
  const uint64_t n = len / dim;
  float* d_v = nullptr;
  float* d_cent = nullptr;
  uint32_t* d_asg = nullptr;
  MVR_TRY(mvr::scratch(c, mvr::kSlotResiduals, len * sizeof(float), (void**)&d_v));
  MVR_TRY(mvr::scratch(c, mvr::kSlotCodebooks, (size_t)k * dim * sizeof(float), (void**)&d_cent));
  MVR_TRY(mvr::scratch(c, mvr::kSlotAux0, n * sizeof(uint32_t), (void**)&d_asg));
  MVR_TRY(mvr::h2d(c, d_v, vectors, len * sizeof(float)));
  float wcss = 0.f;
  uint32_t iters = 0;
  if ((dim == 1 || dim == 2 || dim == 4) && k <= 256) {
    mvr::PqJob job;
    job.R = d_v;
    job.N = n;
    job.D = (int)dim;
    job.M = 1;
    job.S = (int)dim;
    job.K = (int)k;
    job.seed = seed;
    job.max_iters = max_iters;
    job.tol = tol;
    mvr::PqOut out;
    out.d_codebooks = d_cent;
    out.d_assign = d_asg;
    out.h_wcss = &wcss;
    out.h_iters = &iters;
    MVR_TRY(mvr::pq_kmeans_device(c, job, out));
  } else {
    MVR_TRY(mvr::kmeans_general_device(c, d_v, n, dim, k, max_iters, tol, seed, d_cent, d_asg, &wcss, &iters));
  }
  MVR_TRY(mvr::d2h(c, centroids_out, d_cent, (size_t)k * dim * sizeof(float)));
  if (assignments_out) MVR_TRY(mvr::d2h(c, assignments_out, d_asg, n * sizeof(uint32_t)));
  MVR_CUDA(c, cudaStreamSynchronize(c->stream));
  if (wcss_out) *wcss_out = wcss;
  if (iters_out) *iters_out = iters;
  return MVR_OK;
}

// ---- residuals ------------------------------------------------------------

int mvr_residuals_norms_device(mvr_ctx* h, const float* d_v, const float* d_cent, uint32_t kappa,
                               const uint32_t* d_asg, uint64_t n, uint32_t dim, float* d_res,
                               float* d_norms) {
  (void)kappa;
  if (!h) return MVR_E_INVALID_ARGUMENT;
  Ctx* c = &h->impl;
  if (n == 0) return MVR_OK;
  if (dim == 0) return mvr::fail(c, MVR_E_DIM_MISMATCH, "dim == 0");
  if (!d_v || !d_cent || !d_asg || !d_res || !d_norms)
    return mvr::fail(c, MVR_E_INVALID_ARGUMENT, "null pointer");
  mvr::DeviceScope dev_scope(c);
  MVR_TRY(dev_scope.status);
  const int grid = (int)std::min<uint64_t>((n + 255) / 256, (uint64_t)c->sm_count * 16);
  mvr::residuals_norms_kernel<<<grid, 256, 0, c->stream>>>(d_v, d_cent, d_asg, n, dim, d_res, d_norms);
  MVR_CUDA(c, cudaGetLastError());
  return MVR_OK;
}

int mvr_residuals_norms(mvr_ctx* h, const float* v, const float* cent, uint32_t kappa,
                        const uint32_t* asg, uint64_t n, uint32_t dim, float* res_out,
                        float* norms_out) {
  if (!h) return MVR_E_INVALID_ARGUMENT;
  Ctx* c = &h->impl;
  if (n == 0) return MVR_OK;
  if (dim == 0) return mvr::fail(c, MVR_E_DIM_MISMATCH, "dim == 0");
  if (!v || !cent || !asg || !res_out || !norms_out)
    return mvr::fail(c, MVR_E_INVALID_ARGUMENT, "null pointer");
  for (uint64_t i = 0; i < n; ++i)
    if (asg[i] >= kappa) return mvr::fail(c, MVR_E_INVALID_ARGUMENT, "assignment >= kappa");
  mvr::DeviceScope dev_scope(c);
  MVR_TRY(dev_scope.status);
  float *d_v, *d_cent, *d_res, *d_norms;
  uint32_t* d_asg;
  MVR_TRY(mvr::scratch(c, mvr::kSlotResiduals, n * dim * sizeof(float), (void**)&d_v));
  MVR_TRY(mvr::scratch(c, mvr::kSlotCodebooks, (size_t)kappa * dim * sizeof(float), (void**)&d_cent));
  MVR_TRY(mvr::scratch(c, mvr::kSlotAux0, n * sizeof(uint32_t), (void**)&d_asg));
  MVR_TRY(mvr::scratch(c, mvr::kSlotSorted, n * dim * sizeof(float), (void**)&d_res));
  MVR_TRY(mvr::scratch(c, mvr::kSlotAux1, n * sizeof(float), (void**)&d_norms));
  MVR_TRY(mvr::h2d(c, d_v, v, n * dim * sizeof(float)));
  MVR_TRY(mvr::h2d(c, d_cent, cent, (size_t)kappa * dim * sizeof(float)));
  MVR_TRY(mvr::h2d(c, d_asg, asg, n * sizeof(uint32_t)));
  MVR_TRY(mvr_residuals_norms_device(h, d_v, d_cent, kappa, d_asg, n, dim, d_res, d_norms));
  MVR_TRY(mvr::d2h(c, res_out, d_res, n * dim * sizeof(float)));
  MVR_TRY(mvr::d2h(c, norms_out, d_norms, n * sizeof(float)));
  MVR_CUDA(c, cudaStreamSynchronize(c->stream));
  return MVR_OK;
}

}  // extern "C"
