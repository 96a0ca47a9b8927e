// pq_engine.h — batched k-means over PQ subspaces on one GPU.
//
// One "subspace problem" per m in [0, M): the rows R[i][m*S .. m*S+S) of a
// row-major N x D matrix (D = M*S, S in {1,2,4}), clustered into K <= 256
// centroids with the reference `kmeans.fit` semantics
// (src/tac/kmeans.zig:67-232) and the PQ per-subspace seed `seed +% m`
// (src/index/pq.zig:319-325). `mvr_kmeans_fit` for small dims is the M = 1
// case of the same engine.
#pragma once
#include <cstdint>

#include "mvr_internal.h"

namespace mvr {

struct PqJob {
  const float* R = nullptr;  // device, N x D row-major, 4-byte aligned
  uint64_t N = 0;
  int D = 0;
  int M = 0;
  int S = 0;
  int K = 256;
  uint64_t seed = 0;  // subspace m uses seed + m
  uint32_t max_iters = 25;
  float tol = 1e-4f;
  // the workspace's subspace-major copy XT (pq_layout o_xt) already holds the
  // rows; R is then not read
  bool xt_ready = false;
  // assignment passes through the tensor-core filter (pq_tc_assign_kernel)
  bool tc_filter = true;
  // subspace-major rows [M][N][S] held outside the workspace (the workspace
  // then has no XT region); requires xt_ready
  const float* xt = nullptr;
  // index of subspace 0 in failure messages ("subspace <sub0 + m>")
  int sub0 = 0;
};

struct PqOut {
  float* d_codebooks = nullptr;    // device [M][K][S] (required)
  uint32_t* d_assign = nullptr;    // device [M][N] final assignments (optional)
  float* h_wcss = nullptr;         // host [M] final WCSS (optional)
  uint32_t* h_iters = nullptr;     // host [M] iterations run (optional)
  mvr_pq_train_stats* stats = nullptr;
};

// Byte offsets of the engine's device workspace. The bookkeeping block
// [0, small_bytes) is mirrored on the host (RNG draws in, status out).
struct PqLayout {
  int nblk = 0, nchunk = 0;
  int nblk_s = 0;  // Lloyd histogram / scatter CTAs (one kScatTile-row tile each)
  uint64_t rows_per_cta = 0;
  size_t o_draws = 0, o_chosen = 0, o_idx0 = 0, o_thr = 0, o_counts = 0, o_starts = 0, o_wcss = 0,
         o_prev = 0, o_status = 0, o_nonf = 0, o_iters = 0, o_fb = 0, o_rs = 0, o_exact = 0, o_state = 0;
  size_t small_bytes = 0;
  size_t o_xt = 0, o_mind = 0, o_asg = 0, o_sorted = 0, o_hist = 0, o_chunk = 0, o_chunk_cnt = 0;
  size_t o_xpre = 0, o_xg = 0, o_xe = 0;  // exact chained draws (large N)
  // Lloyd bound pruning: bounds [M][N] f32 x2, per-subspace row lists
  // [M][N] u32 + counts, previous codebooks, drifts [M][K], max drift [M]
  size_t o_ub = 0, o_lb = 0, o_list = 0, o_lcnt = 0, o_cbold = 0, o_drift = 0, o_maxd = 0;
  // candidate scans: neighbour lists [M][K][32] u8 and the bound of each
  // list's last entry [M][K] f32; distances computed by
  // the pruned passes [M] u64 (in the bookkeeping block)
  size_t o_nbr = 0, o_nbr_last = 0, o_ldist = 0;
  // tensor-core filter counters (in the bookkeeping block): violations,
  // rows re-scanned, timeouts
  size_t o_diag = 0;
  size_t total_bytes = 0;
};
// Workspace layout for N rows, M subspaces of S floats, K centroids on a
// device with `sms` streaming multiprocessors (without the XT region when
// with_xt is false).
PqLayout pq_layout(uint64_t N, int M, int S, int K, int sms, bool with_xt = true);

// Subspace groups pq_kmeans_run runs side by side on separate streams: 2
// when a context is given (the second group runs on its side stream), there
// are two or more subspaces and K < N; 1 otherwise. Each group is an
// independent training of its own subspaces, so one group's latency-bound
// steps (the k-means++ draw, the per-iteration bookkeeping kernels) overlap
// the other group's bandwidth-bound passes.
int pq_groups(const Ctx* ctx, uint64_t N, int M, int K);
// Device workspace pq_kmeans_run needs for `groups` groups (256-byte
// aligned), and where the subspace-major rows XT [M][N][S] sit in it (a
// caller that sets job.xt_ready fills them there).
size_t pq_ws_bytes(uint64_t N, int M, int S, int K, int sms, int groups);
float* pq_ws_xt(unsigned char* ws, uint64_t N, int M, int S, int K, int sms, int groups);

// Multiprocessor count of the current device (148 if it cannot be read).
int sm_count_current_device();

// Runs seeding + Lloyd for all M subspaces on `stream` (and, with two
// groups, the context's side stream), with device workspace `ws`
// (pq_ws_bytes(..., pq_groups(...)), 256-byte aligned) and host buffer
// `hsmall` (pq_layout(...).small_bytes; used with one group). Allocates no
// device memory. `ctx` may be null (then one group, no timing and no error
// text). Returns the MVR status of the smallest failing subspace, or MVR_OK;
// synchronises `stream`.
int pq_kmeans_run(Ctx* ctx, cudaStream_t stream, const PqJob& job, const PqOut& out,
                  unsigned char* ws, unsigned char* hsmall, int sms);

// pq_kmeans_run with the workspace taken from the context's scratch.
int pq_kmeans_device(Ctx* ctx, const PqJob& job, const PqOut& out);

// Row-sharded pq_kmeans_device: this rank holds rows [row0, row0 + job.N) of
// an N_total-row matrix (shards contiguous in rank order, one per rank of the
// context's communicator). Every rank ends with the codebooks the one-GPU
// engine computes on the whole matrix; out.d_assign receives this rank's
// rows. Collective: every rank calls it with the same job parameters.
// local_ok = false makes every rank return MVR_E_INVALID_ARGUMENT (after the
// first exchange) instead of leaving the other ranks waiting.
int pq_kmeans_run_dist(Ctx* ctx, const PqJob& job, uint64_t row0, uint64_t N_total, const PqOut& out,
                       bool local_ok);

// Subspace-sharded training, the default for pq_m >= ranks: rank g owns a
// contiguous range of subspaces, receives those columns of every row (one
// grouped exchange), runs the one-GPU engine on them with seeds seed + m,
// and the codebooks are gathered on every rank. Same contract as
// pq_kmeans_run_dist.
int pq_kmeans_run_subspaces(Ctx* ctx, const PqJob& job, uint64_t row0, uint64_t N_total, const PqOut& out,
                            bool local_ok);

// PQ.encode of N rows (asynchronous on the context stream).
int pq_encode_device(Ctx* ctx, const float* d_codebooks, int D, int M,
                     const float* d_R, uint64_t N, uint8_t* d_codes);

}  // namespace mvr
