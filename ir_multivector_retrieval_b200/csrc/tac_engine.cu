// tac_engine.cu — TAC per-token clustering and general-dimension kmeans.fit
// on the GPU.
//
// Reference: tac.clusterFlat (src/tac/tac.zig:563-838). Host side: vocabulary
// size, frequencies and the CSR grouping of rows by token id in ascending
// row order (tac.zig:576-603), budget phases 1-4 (tac_budget.cpp). Device
// side: the rows gathered in token order, the per-token Welford spreads
// (tac.zig:609-644) and one k-means per token (runOneTokenKmeans,
// tac.zig:458-514) through the ragged batch engine (km_engine.cu).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/mvr.h"
#include "km_engine.h"
#include "mvr_device.cuh"
#include "mvr_internal.h"
#include "tac_engine.h"

namespace mvr {
namespace {

// Welford spread of one token per warp (tac.zig:609-644): f32 count,
// inv = 1/count, per coordinate delta = x - mean; mean += delta*inv;
// m2 += delta*(x - mean); trace = sum of m2 in coordinate order;
// spread = trace / n. Coordinate c lives in lane c % 32, slot c / 32 (Q
// slots, d <= 32 Q). A token's rows are contiguous in G; they stream through
// a per-warp ring of kSpStages shared-memory stages filled by cp.async, so
// the dependent Welford chain, not load latency, sets the pace. The f32
// count after q rows is min(q, 2^24) exactly (x + 1 rounds back to 2^24
// there), so 32 lanes form 32 rows' 1/count at once.
constexpr int kSpWarps = 4;
constexpr int kSpStages = 3;
constexpr int kSpStageFloats = 2048;

template <int Q>
__global__ void __launch_bounds__(kSpWarps * 32)
tac_spread_kernel(const float* __restrict__ G, uint32_t d, const uint32_t* __restrict__ goff, uint64_t nd,
                  float* __restrict__ spreads) {
  extern __shared__ __align__(16) float sp_stage[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* ring = sp_stage + (size_t)warp * kSpStages * kSpStageFloats;
  const uint32_t rb = kSpStageFloats / d;  // rows per stage (>= 8)
  const uint32_t sf = rb * d;
  const bool vec = (d & 3) == 0;
  for (uint64_t j = (uint64_t)blockIdx.x * kSpWarps + warp; j < nd; j += (uint64_t)gridDim.x * kSpWarps) {
    const uint32_t start = goff[j], n = goff[j + 1] - start;
    if (n == 0) {
      if (lane == 0) spreads[j] = 0.f;
      continue;
    }
    const float* src = G + (uint64_t)start * d;
    const uint32_t nst = (n + rb - 1) / rb;
    auto issue = [&](uint32_t stg) {
      if (stg < nst) {
        const uint32_t nf = min(rb, n - stg * rb) * d;
        const float* s0 = src + (uint64_t)stg * sf;
        float* d0 = ring + (stg % kSpStages) * kSpStageFloats;
        if (vec) {
          for (uint32_t e = lane * 4; e < nf; e += 128) cp_async<16>(d0 + e, s0 + e);
        } else {
          for (uint32_t e = lane; e < nf; e += 32) cp_async<4>(d0 + e, s0 + e);
        }
      }
      cp_async_commit();
    };
    __syncwarp();  // the previous token's reads of the ring are done
#pragma unroll
    for (int q = 0; q < kSpStages - 1; ++q) issue(q);
    float mean[Q], m2[Q];
#pragma unroll
    for (int q = 0; q < Q; ++q) {
      mean[q] = 0.f;
      m2[q] = 0.f;
    }
    for (uint32_t stg = 0; stg < nst; ++stg) {
      cp_async_wait<kSpStages - 2>();
      __syncwarp();
      issue(stg + kSpStages - 1);
      const float* x = ring + (stg % kSpStages) * kSpStageFloats;
      const uint32_t rows = min(rb, n - stg * rb);
      const uint32_t row0 = stg * rb;
      float invl = 0.f;
      for (uint32_t r = 0; r < rows; ++r) {
        if ((r & 31) == 0) {
          const uint32_t q = row0 + r + lane + 1;
          invl = __fdiv_rn(1.0f, __uint2float_rn(min(q, 16777216u)));
        }
        const float inv = __shfl_sync(0xffffffffu, invl, r & 31);
        const float* xr = x + r * d;
#pragma unroll
        for (int q = 0; q < Q; ++q) {
          const uint32_t c = lane + 32 * q;
          if (c < d) {
            const float xv = xr[c];
            const float delta = __fsub_rn(xv, mean[q]);
            mean[q] = __fadd_rn(mean[q], __fmul_rn(delta, inv));
            m2[q] = __fadd_rn(m2[q], __fmul_rn(delta, __fsub_rn(xv, mean[q])));
          }
        }
      }
    }
    cp_async_wait<0>();
    float trace = 0.f;
#pragma unroll
    for (int q = 0; q < Q; ++q)
      for (uint32_t l = 0; l < 32 && 32 * q + l < d; ++l)
        trace = __fadd_rn(trace, __shfl_sync(0xffffffffu, m2[q], l));
    if (lane == 0) spreads[j] = __fdiv_rn(trace, __uint2float_rn(n));
  }
}

int launch_spreads(Ctx* c, const float* d_G, uint32_t d, const uint32_t* d_goff, uint64_t nd, float* d_sp) {
  const size_t smem = (size_t)kSpWarps * kSpStages * kSpStageFloats * sizeof(float);
  const unsigned grid = (unsigned)std::min<uint64_t>((nd + kSpWarps - 1) / kSpWarps, 1u << 20);
  auto k = d <= 32 ? tac_spread_kernel<1> : d <= 64 ? tac_spread_kernel<2> : d <= 128 ? tac_spread_kernel<4>
                                                                                     : tac_spread_kernel<8>;
  MVR_CUDA(c, cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  k<<<grid, kSpWarps * 32, smem, c->stream>>>(d_G, d, d_goff, nd, d_sp);
  MVR_CUDA(c, cudaGetLastError());
  return MVR_OK;
}

// assignments[idx[q]] = base[token of q] + local[q]
__global__ void tac_scatter_assign_kernel(const uint32_t* __restrict__ idx, const uint32_t* __restrict__ rowtok,
                                          const uint32_t* __restrict__ goffc, const uint32_t* __restrict__ local,
                                          uint64_t n, uint32_t* __restrict__ out) {
  for (uint64_t q = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; q < n; q += (uint64_t)gridDim.x * blockDim.x)
    out[idx[q]] = goffc[rowtok[q]] + local[q];
}

int set_device(Ctx* c) {
  cudaError_t e = cudaSetDevice(c->device);
  if (e != cudaSuccess) return cuda_fail(c, e, "cudaSetDevice");
  return MVR_OK;
}

}  // namespace

int kmeans_general_device(Ctx* ctx, const float* d_v, uint64_t n, uint32_t dim, uint32_t k, uint32_t max_iters,
                          float tol, uint64_t seed, float* d_centroids, uint32_t* d_assign, float* h_wcss,
                          uint32_t* h_iters) {
  KmBatch b;
  b.off = {0};
  b.n = {(uint32_t)n};
  b.k = {k};
  b.coff = {0};
  b.seed = {seed};
  if (n >= (1ull << 32)) return fail(ctx, MVR_E_INVALID_ARGUMENT, "more than 2^32-1 rows");
  if (dim > 256) return fail(ctx, MVR_E_INVALID_ARGUMENT, "dim > 256 is not supported on the GPU path");
  float* d_GT = nullptr;
  MVR_TRY(scratch(ctx, kSlotSorted, (size_t)n * ((dim + 3) / 4) * 4 * sizeof(float), (void**)&d_GT));
  MVR_TRY(km_gather_groups(ctx, d_v, nullptr, n, dim, nullptr, d_GT));
  KmResult r;
  MVR_TRY(km_batch_run(ctx, d_v, d_GT, n, dim, b, max_iters, tol, d_centroids, d_assign, &r));
  if (r.status[0] != MVR_OK) return fail(ctx, r.status[0], mvr_status_name(r.status[0]));
  if (h_wcss) *h_wcss = r.wcss[0];
  if (h_iters) *h_iters = r.iters[0];
  return MVR_OK;
}

}  // namespace mvr

using mvr::Ctx;

extern "C" int mvr_tac_cluster_flat(mvr_ctx* h, const uint32_t* token_ids, uint64_t n_tokens, const float* vectors,
                                    uint64_t vectors_len, uint32_t dim, const mvr_clustering_params* p,
                                    float* centroids_out, uint32_t* assignments_out, uint32_t* kappa_out,
                                    uint64_t kappa_cap, uint64_t* n_distinct_out, float* wcss_total_out) {
  if (!h || !p) return MVR_E_INVALID_ARGUMENT;
  Ctx* c = &h->impl;
  // clusterFlat's validation order (tac.zig:570-573)
  if (n_tokens == 0) return mvr::fail(c, MVR_E_EMPTY_TOKEN_DUMP, "no tokens");
  if (dim == 0) return mvr::fail(c, MVR_E_INVALID_THRESHOLDS, "dim == 0");
  if (vectors_len != n_tokens * (uint64_t)dim) return mvr::fail(c, MVR_E_INVALID_THRESHOLDS, "vectors_len != n*dim");
  if (p->kappa_total == 0) return mvr::fail(c, MVR_E_BUDGET_TOO_SMALL, "kappa_total == 0");
  if (!token_ids || !vectors || !centroids_out || !assignments_out || !kappa_out)
    return mvr::fail(c, MVR_E_INVALID_ARGUMENT, "null pointer");
  if (dim > 256) return mvr::fail(c, MVR_E_INVALID_ARGUMENT, "dim > 256 is not supported on the GPU path");
  if (n_tokens >= (1ull << 32)) return mvr::fail(c, MVR_E_INVALID_ARGUMENT, "more than 2^32-1 tokens");

  // ---- step 0-1: vocabulary, frequencies, CSR grouping (host) -------------
  uint32_t max_id = 0;
  for (uint64_t i = 0; i < n_tokens; ++i) max_id = std::max(max_id, token_ids[i]);
  const uint64_t nd = (uint64_t)max_id + 1;
  if (n_distinct_out) *n_distinct_out = nd;
  if (kappa_cap < nd) return mvr::fail(c, MVR_E_OUT_BUFFER_WRONG_SIZE, "kappa_per_token buffer too small");
  std::vector<uint32_t> freqs(nd, 0), goff(nd + 1, 0), gidx(n_tokens), rowtok(n_tokens);
  for (uint64_t i = 0; i < n_tokens; ++i) ++freqs[token_ids[i]];
  for (uint64_t j = 0; j < nd; ++j) goff[j + 1] = goff[j] + freqs[j];
  {
    std::vector<uint32_t> cur(goff.begin(), goff.end() - 1);
    for (uint64_t i = 0; i < n_tokens; ++i) gidx[cur[token_ids[i]]++] = (uint32_t)i;
  }
  for (uint64_t j = 0; j < nd; ++j)
    for (uint32_t q = goff[j]; q < goff[j + 1]; ++q) rowtok[q] = (uint32_t)j;

  MVR_TRY(mvr::set_device(c));
  cudaStream_t st = c->stream;
  float *d_V = nullptr, *d_G = nullptr, *d_sp = nullptr, *d_C = nullptr;
  uint32_t *d_gidx = nullptr, *d_goff = nullptr, *d_local = nullptr, *d_rowtok = nullptr, *d_goffc = nullptr,
           *d_asg = nullptr;
  const uint64_t rows = n_tokens;
  MVR_TRY(mvr::scratch(c, mvr::kSlotResiduals, rows * dim * sizeof(float), (void**)&d_V));
  MVR_TRY(mvr::scratch(c, mvr::kSlotSorted, rows * dim * sizeof(float), (void**)&d_G));
  float* d_GT = nullptr;
  MVR_TRY(mvr::scratch(c, mvr::kSlotMinDist, rows * ((dim + 3) / 4) * 4 * sizeof(float), (void**)&d_GT));
  MVR_TRY(mvr::scratch(c, mvr::kSlotAux0, rows * sizeof(uint32_t), (void**)&d_gidx));
  MVR_TRY(mvr::scratch(c, mvr::kSlotAux1, rows * sizeof(uint32_t), (void**)&d_local));
  MVR_TRY(mvr::scratch(c, mvr::kSlotAux2, rows * sizeof(uint32_t) * 2 + (nd + 1) * 4 * 2 + nd * 4 + 1024,
                       (void**)&d_rowtok));
  d_asg = d_rowtok + rows;
  d_goff = d_asg + rows;
  d_goffc = d_goff + (nd + 1);
  d_sp = reinterpret_cast<float*>(d_goffc + (nd + 1));
  MVR_CUDA(c, cudaMemcpyAsync(d_V, vectors, rows * dim * sizeof(float), cudaMemcpyHostToDevice, st));
  MVR_CUDA(c, cudaMemcpyAsync(d_gidx, gidx.data(), rows * 4, cudaMemcpyHostToDevice, st));
  MVR_CUDA(c, cudaMemcpyAsync(d_goff, goff.data(), (nd + 1) * 4, cudaMemcpyHostToDevice, st));
  MVR_CUDA(c, cudaMemcpyAsync(d_rowtok, rowtok.data(), rows * 4, cudaMemcpyHostToDevice, st));
  MVR_TRY(mvr::km_gather_groups(c, d_V, d_gidx, rows, dim, d_G, d_GT));
  MVR_TRY(mvr::launch_spreads(c, d_G, dim, d_goff, nd, d_sp));
  std::vector<float> spreads(nd);
  MVR_CUDA(c, cudaMemcpyAsync(spreads.data(), d_sp, nd * 4, cudaMemcpyDeviceToHost, st));
  MVR_CUDA(c, cudaStreamSynchronize(st));

  // ---- step 3: budget phases 1-4 (host) ------------------------------------
  std::vector<float> frac(nd);
  std::vector<uint32_t> kap(nd);
  {
    const int s = mvr::tac_allocate_budgets_host(freqs.data(), spreads.data(), kap.data(), frac.data(), nd,
                                                 p->kappa_total, p->mu, p->tau, p->epsilon, p->theta);
    std::memcpy(kappa_out, kap.data(), nd * 4);
    if (s != MVR_OK) return mvr::fail(c, s, "budget allocation");
  }
  for (uint64_t j = 0; j < nd; ++j)
    if (freqs[j] > 0 && kap[j] == 0) return mvr::fail(c, MVR_E_BUDGET_TOO_SMALL, "token with vectors got no centroid");
  std::vector<uint32_t> goffc(nd + 1, 0);
  for (uint64_t j = 0; j < nd; ++j) goffc[j + 1] = goffc[j] + kap[j];
  if (goffc[nd] != p->kappa_total) return mvr::fail(c, MVR_E_BUDGET_TOO_SMALL, "budgets do not sum to kappa_total");

  // ---- step 4: one k-means per token on the device -------------------------
  mvr::KmBatch b;
  std::vector<uint32_t> pj;  // token id of each problem
  for (uint64_t j = 0; j < nd; ++j) {
    if (kap[j] == 0 || freqs[j] == 0) continue;
    b.off.push_back(goff[j]);
    b.n.push_back(freqs[j]);
    b.k.push_back(kap[j]);
    b.coff.push_back(goffc[j]);
    b.seed.push_back(p->seed ^ (uint64_t)j);
    pj.push_back((uint32_t)j);
  }
  MVR_TRY(mvr::scratch(c, mvr::kSlotCodebooks, (size_t)p->kappa_total * dim * sizeof(float), (void**)&d_C));
  mvr::KmResult r;
  MVR_TRY(mvr::km_batch_run(c, d_G, d_GT, rows, dim, b, p->max_iters, p->tol, d_C, d_local, &r));
  for (size_t q = 0; q < r.status.size(); ++q)  // the lowest failing token, as the serial reference reports
    if (r.status[q] != MVR_OK)
      return mvr::fail(c, r.status[q], std::string("token ") + std::to_string(pj[q]) + ": " +
                                           mvr_status_name(r.status[q]));

  // ---- outputs ----------------------------------------------------------------
  MVR_CUDA(c, cudaMemcpyAsync(d_goffc, goffc.data(), (nd + 1) * 4, cudaMemcpyHostToDevice, st));
  {
    const int grid = (int)std::min<uint64_t>((rows + 255) / 256, (uint64_t)c->sm_count * 8);
    mvr::tac_scatter_assign_kernel<<<grid, 256, 0, st>>>(d_gidx, d_rowtok, d_goffc, d_local, rows, d_asg);
    MVR_CUDA(c, cudaGetLastError());
  }
  MVR_CUDA(c, cudaMemcpyAsync(assignments_out, d_asg, rows * 4, cudaMemcpyDeviceToHost, st));
  MVR_CUDA(c, cudaMemcpyAsync(centroids_out, d_C, (size_t)p->kappa_total * dim * sizeof(float),
                              cudaMemcpyDeviceToHost, st));
  MVR_CUDA(c, cudaStreamSynchronize(st));

  // wcss_total: per-token WCSS summed in token order, per static thread chunk
  // when n_threads > 1 (tac.zig:685-825).
  std::vector<float> tw(nd, 0.f);
  for (size_t q = 0; q < pj.size(); ++q) tw[pj[q]] = r.wcss[q];
  float total = 0.f;
  const uint32_t nt = p->n_threads;
  if (nt <= 1) {
    for (uint64_t j = 0; j < nd; ++j)
      if (kap[j] && freqs[j]) total += tw[j];
  } else {
    const uint64_t chunk = (nd + nt - 1) / nt;
    for (uint64_t t = 0; t < nt; ++t) {
      const uint64_t lo = t * chunk, hi = std::min<uint64_t>((t + 1) * chunk, nd);
      float w = 0.f;
      for (uint64_t j = lo; j < hi; ++j)
        if (kap[j] && freqs[j]) w += tw[j];
      total += w;
    }
  }
  if (wcss_total_out) *wcss_total_out = total;
  for (uint64_t i = 0; i < n_tokens; ++i)  // final invariant (tac.zig:827-830)
    if (assignments_out[i] >= p->kappa_total) return mvr::fail(c, MVR_E_INVALID_THRESHOLDS, "assignment out of range");
  return MVR_OK;
}
