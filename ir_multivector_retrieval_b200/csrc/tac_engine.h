// tac_engine.h — general-dimension k-means and TAC per-token clustering on
// the GPU (ragged batches of independent k-means problems).
#pragma once
#include <cstdint>

#include "mvr_internal.h"

namespace mvr {

// kmeans.fit (src/tac/kmeans.zig:67-232) for any dim and k: one problem,
// rows d_v[n][dim] on the device. Outputs on the device (centroids k*dim,
// assignments n) plus host scalars. Synchronises the context stream.
int kmeans_general_device(Ctx* ctx, const float* d_v, uint64_t n, uint32_t dim, uint32_t k,
                          uint32_t max_iters, float tol, uint64_t seed, float* d_centroids,
                          uint32_t* d_assign, float* h_wcss, uint32_t* h_iters);

// Budget phases 1-4 (src/tac/tac.zig:97-402) on the host; `frac` is
// caller scratch of n floats.
int tac_allocate_budgets_host(const uint32_t* freqs, const float* spreads, uint32_t* kappa,
                              float* frac, uint64_t n, uint32_t kappa_total, uint32_t mu,
                              uint32_t tau, uint32_t eps, uint32_t theta);

// Work estimate of one token's k-means: n * (k + 1) distance evaluations
// per pass when k < n, n for the degenerate copy (k >= n), 0 without a
// problem.
uint64_t tac_token_work(uint32_t n, uint32_t k);

// Longest-processing-time split of the per-token k-means problems over
// `ranks` GPUs: owner[j] in [0, ranks) for every token (0 for tokens with
// no problem).
void tac_partition_tokens_host(const uint32_t* freqs, const uint32_t* kappa, uint64_t n, uint32_t ranks,
                               uint32_t* owner);

}  // namespace mvr
