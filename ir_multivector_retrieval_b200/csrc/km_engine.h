// km_engine.h — ragged batch of independent k-means problems of any
// dimension on one GPU.
//
// Problem p clusters rows [off[p], off[p] + n[p]) of a row-major matrix G
// (rows x dim) into k[p] centroids stored at rows [coff[p], coff[p] + k[p])
// of C, with the reference `kmeans.fit` semantics (src/tac/kmeans.zig:67-232)
// and RNG seed seed[p]. TAC uses one problem per token id (rows gathered in
// token order, ascending original row inside a token; seed = seed ^ j,
// src/tac/tac.zig:458-514); `mvr_kmeans_fit` for general dims is P = 1.
#pragma once
#include <cstdint>
#include <vector>

#include "mvr_internal.h"

namespace mvr {

struct KmBatch {
  std::vector<uint64_t> off;   // first row of problem p in G
  std::vector<uint32_t> n;     // rows of problem p
  std::vector<uint32_t> k;     // centroids of problem p
  std::vector<uint64_t> coff;  // first centroid row of problem p in C
  std::vector<uint64_t> seed;  // RNG seed of problem p
  size_t size() const { return n.size(); }
};

struct KmResult {
  std::vector<int> status;      // MVR status per problem
  std::vector<float> wcss;      // final WCSS per problem (0 for degenerate)
  std::vector<uint32_t> iters;  // Lloyd iterations run per problem
  uint32_t seed_fallbacks = 0;  // draws settled by the exact sequential chain
  uint32_t launches = 0;
  double seed_ms = 0.0;   // device time of the seeding (degenerate copies included)
  double lloyd_ms = 0.0;  // device time of the Lloyd iterations
  uint64_t filter_rows_rechecked = 0;  // tensor-core filter: rows with several candidates
  uint32_t filter_violations = 0;      // winners outside the filter's bound (then re-run exactly)
  uint64_t filter_rows_full_scan = 0;  // rows whose candidate list overflowed (full exact scan)
};

// Group-major copy of a row set: GT holds ceil(dim / 4) groups, group g of
// row q (coordinates 4g .. 4g+3, zero past dim) as the float4 GT[g * n + q].
// Row q is V[idx[q]] (or V[q] when idx is null); when G is not null the rows
// are also written row-major to G; GT may be null when only G is wanted.
// Enqueued on the context stream.
int km_gather_groups(Ctx* ctx, const float* d_V, const uint32_t* d_idx, uint64_t n, uint32_t dim, float* d_G,
                     float* d_GT);

// Runs every problem to completion. d_G: rows x dim (device), d_GT: its
// group-major copy (km_gather_groups), d_C: sum(k) x dim (device, output),
// d_local: rows u32 (device, output: local cluster id of each row within its
// problem). Synchronises the context stream.
int km_batch_run(Ctx* ctx, const float* d_G, const float* d_GT, uint64_t rows, uint32_t dim, const KmBatch& b,
                 uint32_t max_iters, float tol, float* d_C, uint32_t* d_local, KmResult* res);

// Exclusive prefix sums of n u32 on `st`; `part` holds scan_part_words(n).
size_t scan_part_words(uint64_t n);
int exclusive_scan_u32(Ctx* ctx, cudaStream_t st, const uint32_t* in, uint64_t n, uint32_t* part, uint32_t* out);

// Stable LSD radix sort of (key, val) pairs by the low `key_bits` bits of the
// keys (8 bits per pass; vals == nullptr sorts the row indices), ping-pong
// between (k0, v0) and (k1, v1); the sorted pairs are at *keys_out /
// *vals_out. `scratch` holds radix_pairs_scratch_words(n) u32.
size_t radix_pairs_scratch_words(uint64_t n);
int radix_sort_pairs(Ctx* ctx, cudaStream_t st, const uint32_t* keys, const uint32_t* vals, uint64_t n, int key_bits,
                     uint32_t* k0, uint32_t* v0, uint32_t* k1, uint32_t* v1, uint32_t* scratch,
                     const uint32_t** keys_out, const uint32_t** vals_out);

}  // namespace mvr
