// mvr_internal.h — context, scratch and error plumbing shared by the C-ABI
// entry points and the kernel launchers. Not part of the public ABI.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <vector>

#include "../../include/mvr.h"

namespace mvr {

// Device buffer that only grows; freed by the context.
struct DevBuf {
  void* ptr = nullptr;
  size_t bytes = 0;
};

enum ScratchSlot {
  kSlotMinDist = 0,  // [M][N] f32: k-means++ D^2 weights, then Lloyd min_to_any
  kSlotAssign,       // [M][N] u8 / u32 assignments
  kSlotSorted,       // [M][N][S] f32 rows sorted by cluster (stable)
  kSlotHist,         // [M][K][nblk] u32 per-block histograms -> scatter bases
  kSlotChunk,        // [M][nchunk] double2 directed-rounding partial sums
  kSlotSmall,        // per-subspace bookkeeping (counts, flags, draws ...)
  kSlotResiduals,    // host-API staging of the input rows
  kSlotCodebooks,    // host-API staging of codebooks
  kSlotCodes,        // host-API staging of codes
  kSlotAux0,
  kSlotAux1,
  kSlotAux2,
  kSlotAux3,
  kSlotCount
};

class HostPool;
struct Comm;

// Timing events of one pq.train engine run: the phase marks (start, end of
// seeding, end of Lloyd) and a pool for the sampled kernel brackets.
struct PqTiming {
  cudaEvent_t phase[3] = {nullptr, nullptr, nullptr};
  std::vector<cudaEvent_t> pool;
};

struct Ctx {
  int device = 0;
  int sm_count = 0;
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;
  std::string last_error;
  DevBuf slots[kSlotCount];
  void* pinned = nullptr;  // host staging for small device->host reads
  size_t pinned_bytes = 0;
  cudaEvent_t ev[4] = {nullptr, nullptr, nullptr, nullptr};
  // pq.train timing events, one set per subspace group (created on first
  // use), and the whole call's start / end with two groups
  PqTiming pq_timing[2];
  cudaEvent_t pev[2] = {nullptr, nullptr};
  // second stream for work that overlaps the main chain (created on first
  // use), with its fork/join events
  cudaStream_t side = nullptr;
  cudaEvent_t fork_ev = nullptr, join_ev = nullptr;
  // timing events of the TAC path (created on first use) and its last report
  cudaEvent_t tev[8] = {};
  mvr_tac_stats tac_stats = {};
  // host staging of large host<->device copies (host_io.cpp)
  HostPool* io_pool = nullptr;
  void* stage[2] = {nullptr, nullptr};
  cudaEvent_t stage_ev[2] = {nullptr, nullptr};
  // NCCL communicator for row-sharded training (comm.cpp); null = one GPU
  Comm* comm = nullptr;
  // resolve every k-means++ draw with the reference's serial chain
  bool serial_draws = false;
  // compute every Lloyd distance (no bound pruning)
  bool exhaustive_assign = false;
  // tensor-core filtered assignment passes (off: the exact scans only)
  bool tc_filter = true;
  // ... also for the PQ passes (4-float sub-vectors), where the filter
  // measured no faster than the exact scans: off by default
  bool pq_tc_filter = false;
  // pruned Lloyd passes scan only the candidate centroids near the current
  // one (off: the bound check + full scans of the failing rows)
  bool cand_scan = true;
  // pq.train subspace groups run side by side on two streams (1 or 2)
  int pq_groups = 2;
  // device counters of the filtered encode passes (created on first use):
  // [0] violations, [1] rows re-scanned, [2] timeouts
  uint32_t* tc_diag = nullptr;
  uint32_t tc_viol_seen = 0;  // violations already answered by an exact re-run
  // polls of the clusterFlat spread kernel's stage waits before it gives up
  // (MVR_WAIT_LIMIT_DEFAULT; tests lower it to make the wait run out)
  uint32_t wait_limit = MVR_WAIT_LIMIT_DEFAULT;
};

// Host->device copy through the pinned stages (pageable sources: the source
// may be reused when it returns) or directly (page-locked sources: complete
// when the context stream reaches it; every host entry point synchronises
// before it returns). Ordered on the context stream.
int h2d_staged(Ctx* ctx, void* d, const void* h, size_t bytes);
// True for page-locked (pinned or registered) host memory.
bool host_is_pinned(const void* h);
// Device->host copy through the pinned stages; complete when it returns.
int d2h_staged(Ctx* ctx, void* h, const void* d, size_t bytes);
void destroy_host_io(Ctx* ctx);

// The context's TAC timing events (created on first use).
int tac_events(Ctx* ctx, cudaEvent_t** out);

// The context's side stream (created on first use on the current device).
int side_stream(Ctx* ctx, cudaStream_t* out);

// Set the context's last error and return `status`.
int fail(Ctx* ctx, int status, const std::string& msg);

// Makes the context's device current for the lifetime of the scope and then
// restores the caller's current device, so an entry point never leaves the
// calling thread on another GPU. `status` is MVR_OK or the failure to switch.
struct DeviceScope {
  explicit DeviceScope(Ctx* c);
  ~DeviceScope();
  DeviceScope(const DeviceScope&) = delete;
  DeviceScope& operator=(const DeviceScope&) = delete;
  int status = 0;
  int prev = -1;
  int dev = -1;
};

// Unique id of the calling thread's current CUDA context (cuCtxGetId), 0
// when there is none or the driver does not provide the calls.
unsigned long long current_context_id();

// Raises `func`'s dynamic shared-memory limit to at least `bytes` in the
// current CUDA context; never lowers it, and calls cudaFuncSetAttribute only
// when the limit must grow (the call costs host time at launch sites inside
// loops). Thread-safe.
cudaError_t raise_smem_limit(const void* func, size_t bytes);

// While one is alive on a thread, fail() and cuda_fail() on that thread write
// their message to *msg instead of the context (engine work that runs on
// several host threads at once; the caller reports one message afterwards).
struct ErrorSink {
  explicit ErrorSink(std::string* msg);
  ~ErrorSink();
  ErrorSink(const ErrorSink&) = delete;
  ErrorSink& operator=(const ErrorSink&) = delete;
  std::string* prev;
};

// Grow slot `slot` to at least `bytes` (contents are not preserved).
int scratch(Ctx* ctx, int slot, size_t bytes, void** out);

// Pinned host staging of at least `bytes`.
int pinned(Ctx* ctx, size_t bytes, void** out);

// Convert a CUDA error into MVR_E_CUDA with context.
int cuda_fail(Ctx* ctx, cudaError_t e, const char* what);

}  // namespace mvr

struct mvr_ctx {
  mvr::Ctx impl;
};

#define MVR_CUDA(ctx, call)                                   \
  do {                                                        \
    cudaError_t _e = (call);                                  \
    if (_e != cudaSuccess) return ::mvr::cuda_fail((ctx), _e, #call); \
  } while (0)

#define MVR_TRY(expr)              \
  do {                             \
    int _s = (expr);               \
    if (_s != MVR_OK) return _s;   \
  } while (0)
