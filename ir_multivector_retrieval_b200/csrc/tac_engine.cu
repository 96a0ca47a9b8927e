// tac_engine.cu — TAC per-token clustering and general-dimension kmeans.fit
// on the GPU.
//
// Reference: tac.clusterFlat (src/tac/tac.zig:563-838). Host side: vocabulary
// size, frequencies and the CSR grouping of rows by token id in ascending
// row order (tac.zig:576-603), budget phases 1-4 (tac_budget.cpp). Device
// side: the rows gathered in token order, the per-token Welford spreads
// (tac.zig:609-644) and one k-means per token (runOneTokenKmeans,
// tac.zig:458-514) through the ragged batch engine (km_engine.cu).
//
// Several GPUs (mvr_tac_cluster_flat_sharded): every rank groups the rows,
// computes the spreads and the budgets (identical on every rank), then runs
// only the tokens that the longest-processing-time split gives it, on a
// compact copy of their rows. The per-token results, the centroids and the
// assignments are merged with u32-sum all-reduces in which each value is
// non-zero on at most one rank, so the merge is exact.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "../../include/mvr.h"
#include "comm.h"
#include "km_engine.h"
#include "mvr_device.cuh"
#include "mvr_internal.h"
#include "tac_engine.h"

namespace mvr {
namespace {

// Welford spread of one token per CTA (tac.zig:609-644): f32 count,
// inv = 1/count, per coordinate delta = x - mean; mean += delta*inv;
// m2 += delta*(x - mean); trace = sum of m2 in coordinate order;
// spread = trace / n. Thread c owns coordinate c (blockDim = d rounded up to
// a warp); its Welford chain (sub -> mul -> add per row) is the critical
// path. A token's rows are contiguous in G and stream through a ring of
// kSpStages shared-memory stages: for d % 4 == 0 one thread issues a bulk
// async copy (TMA) per stage that completes on the stage's mbarrier, so a
// single CTA keeps several stages in flight; other d use 4-byte cp.async.
// The f32 count after q rows is min(q, 2^24) exactly (x + 1 rounds back to
// 2^24 there), so the threads form a whole stage's 1/count values at once.
// Every mbarrier wait is bounded (kSpWaitLimit polls, or the context's
// test-only limit for the stage waits); on expiry the kernel waits for its
// copies still in flight, raises *err and leaves.
constexpr int kSpStages = 6;
constexpr int kSpStageFloats = 4096;
constexpr int kSpMaxRows = 1024;  // rows per stage at most
constexpr uint32_t kSpWaitLimit = MVR_WAIT_LIMIT_DEFAULT;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t limit = kSpWaitLimit) {
  const uint32_t a = smem_u32(bar);
  for (uint32_t it = 0; it < limit; ++it) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

__global__ void __launch_bounds__(256)
tac_spread_kernel(const float* __restrict__ G, uint32_t d, const uint32_t* __restrict__ goff, uint64_t nd,
                  float* __restrict__ spreads, int* __restrict__ err, uint32_t wait_limit) {
  extern __shared__ __align__(128) float sp_ring[];
  __shared__ float sm2[256];
  __shared__ __align__(8) uint64_t bars[kSpStages];
  __shared__ float inv_s[kSpMaxRows];
  const uint32_t tid = threadIdx.x, T = blockDim.x;
  const uint32_t rb = min(kSpStageFloats / d, (uint32_t)kSpMaxRows);  // rows per stage (>= 16)
  const uint32_t sf = rb * d;
  const bool tma = (d & 3) == 0;
  const bool own = tid < d;
  if (tid == 0) {
    for (int q = 0; q < kSpStages; ++q)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(smem_u32(&bars[q])));
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  __syncthreads();
  uint32_t issued = 0;  // stages issued by this CTA, across tokens
  for (uint64_t j = blockIdx.x; j < nd; j += gridDim.x) {
    const uint32_t start = goff[j], n = goff[j + 1] - start;
    if (n == 0) {
      if (tid == 0) spreads[j] = 0.f;
      continue;
    }
    const float* src = G + (uint64_t)start * d;
    const uint32_t nst = (n + rb - 1) / rb;
    const uint32_t first = issued;  // global stage number of this token's stage 0
    auto issue = [&](uint32_t stg) {  // stg: token-local stage
      const uint32_t slot = (first + stg) % kSpStages;
      float* d0 = sp_ring + slot * kSpStageFloats;
      if (stg < nst) {
        const uint32_t nf = min(rb, n - stg * rb) * d;
        const float* s0 = src + (uint64_t)stg * sf;
        if (tma) {
          if (tid == 0) {
            const uint32_t bytes = nf * 4u;
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(&bars[slot])),
                         "r"(bytes)
                         : "memory");
            asm volatile(
                "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                    smem_u32(d0)),
                "l"(s0), "r"(bytes), "r"(smem_u32(&bars[slot]))
                : "memory");
          }
        } else {
          for (uint32_t e = tid; e < nf; e += T) cp_async<4>(d0 + e, s0 + e);
        }
      }
      if (!tma) cp_async_commit();
    };
    __syncthreads();  // the previous token's reads of the ring and sm2 are done
    const uint32_t pre = min(nst, (uint32_t)kSpStages - 1);
    for (uint32_t q = 0; q < kSpStages - 1; ++q) issue(q);
    issued = first + pre;
    float mean = 0.f, m2 = 0.f;
    bool bad = false;
    for (uint32_t stg = 0; stg < nst; ++stg) {
      const uint32_t g = first + stg, slot = g % kSpStages;
      if (tma) {
        if (!mbar_wait_bounded(&bars[slot], (g / kSpStages) & 1u, wait_limit)) bad = true;
      } else {
        cp_async_wait<kSpStages - 2>();
      }
      if (__syncthreads_or(bad)) {
        bad = true;
        break;
      }
      if (stg + kSpStages - 1 < nst) {
        issue(stg + kSpStages - 1);
        ++issued;
      } else if (!tma) {
        cp_async_commit();
      }
      const float* x = sp_ring + slot * kSpStageFloats + (own ? tid : 0);
      const uint32_t rows = min(rb, n - stg * rb);
      const uint32_t row0 = stg * rb;
      // 1/count of this stage's rows, once, by all threads
      for (uint32_t r = tid; r < rows; r += T)
        inv_s[r] = __fdiv_rn(1.0f, __uint2float_rn(min(row0 + r + 1, 16777216u)));
      __syncthreads();
      // groups of 8 rows, the next group's loads issued before this group's
      // chain (two register sets, alternating)
      const uint32_t ng = rows / 8;
      float xa[8], ia[8], xb[8], ib[8];
#define MVR_LOAD8(G8, XV, IV)                      \
  _Pragma("unroll") for (int u = 0; u < 8; ++u) { \
    XV[u] = x[((G8) * 8 + u) * d];                 \
    IV[u] = inv_s[(G8) * 8 + u];                   \
  }
#define MVR_CHAIN8(XV, IV)                                          \
  _Pragma("unroll") for (int u = 0; u < 8; ++u) {                  \
    const float e = __fsub_rn(XV[u], mean);                         \
    mean = __fadd_rn(mean, __fmul_rn(e, IV[u]));                    \
    m2 = __fadd_rn(m2, __fmul_rn(e, __fsub_rn(XV[u], mean)));       \
  }
      if (ng > 0) { MVR_LOAD8(0u, xa, ia) }
      uint32_t g8 = 0;
      for (; g8 + 2 <= ng; g8 += 2) {
        MVR_LOAD8(g8 + 1, xb, ib)
        MVR_CHAIN8(xa, ia)
        if (g8 + 2 < ng) { MVR_LOAD8(g8 + 2, xa, ia) }
        MVR_CHAIN8(xb, ib)
      }
      if (g8 < ng) { MVR_CHAIN8(xa, ia) }
#undef MVR_LOAD8
#undef MVR_CHAIN8
      for (uint32_t r = ng * 8; r < rows; ++r) {
        const float xv = x[r * d];
        const float e = __fsub_rn(xv, mean);
        mean = __fadd_rn(mean, __fmul_rn(e, inv_s[r]));
        m2 = __fadd_rn(m2, __fmul_rn(e, __fsub_rn(xv, mean)));
      }
    }
    if (!tma) cp_async_wait<0>();
    if (bad) {
      // drain: wait for every stage still in flight (with the full limit,
      // whatever the first wait's limit was), then leave: no bulk copy may
      // land in shared memory after the CTA has exited
      if (tma)
        for (uint32_t g = first; g < issued; ++g) (void)mbar_wait_bounded(&bars[g % kSpStages], (g / kSpStages) & 1u);
      if (tid == 0) atomicExch(err, 1);
      break;
    }
    if (own) sm2[tid] = m2;
    __syncthreads();
    if (tid == 0) {
      float trace = 0.f;
      for (uint32_t c = 0; c < d; ++c) trace = __fadd_rn(trace, sm2[c]);
      spreads[j] = __fdiv_rn(trace, __uint2float_rn(n));
    }
  }
}

int launch_spreads(Ctx* c, const float* d_G, uint32_t d, const uint32_t* d_goff, uint64_t nd, float* d_sp,
                   int* d_err) {
  const size_t smem = (size_t)kSpStages * kSpStageFloats * sizeof(float);
  const unsigned threads = (d + 31) / 32 * 32;
  const unsigned grid = (unsigned)std::min<uint64_t>(nd, 1u << 30);
  MVR_CUDA(c, cudaFuncSetAttribute(tac_spread_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  tac_spread_kernel<<<grid, threads, smem, c->stream>>>(d_G, d, d_goff, nd, d_sp, d_err, c->wait_limit);
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

// C[cmap[c]] = CL[c] for the local centroid rows c of one rank
__global__ void tac_place_centroids_kernel(const float* __restrict__ CL, const uint32_t* __restrict__ cmap,
                                           uint64_t nl, uint32_t d, float* __restrict__ C) {
  const uint64_t total = nl * d;
  for (uint64_t e = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (uint64_t)gridDim.x * blockDim.x)
    C[(uint64_t)cmap[e / d] * d + e % d] = CL[e];
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

namespace {

// tac.clusterFlat on one GPU (sharded = false) or split over the ranks of
// the context's communicator (sharded = true, more than one rank).
int cluster_flat(mvr_ctx* h, const uint32_t* token_ids, uint64_t n_tokens, const float* vectors,
                 uint64_t vectors_len, uint32_t dim, const mvr_clustering_params* p, float* centroids_out,
                 uint32_t* assignments_out, uint32_t* kappa_out, uint64_t kappa_cap, uint64_t* n_distinct_out,
                 float* wcss_total_out, bool sharded) {
  if (!h || !p) return MVR_E_INVALID_ARGUMENT;
  Ctx* c = &h->impl;
  const int G = sharded ? mvr::comm_size(c) : 1;
  const int me = G > 1 ? mvr::comm_rank(c) : 0;
  // clusterFlat's validation order (tac.zig:570-573)
  if (n_tokens == 0) return mvr::fail(c, MVR_E_EMPTY_TOKEN_DUMP, "no tokens");
  if (dim == 0) return mvr::fail(c, MVR_E_INVALID_THRESHOLDS, "dim == 0");
  if (vectors_len != n_tokens * (uint64_t)dim) return mvr::fail(c, MVR_E_INVALID_THRESHOLDS, "vectors_len != n*dim");
  if (p->kappa_total == 0) return mvr::fail(c, MVR_E_BUDGET_TOO_SMALL, "kappa_total == 0");
  if (!token_ids || !vectors || !centroids_out || !assignments_out || !kappa_out)
    return mvr::fail(c, MVR_E_INVALID_ARGUMENT, "null pointer");
  if (dim > 256) return mvr::fail(c, MVR_E_INVALID_ARGUMENT, "dim > 256 is not supported on the GPU path");
  if (n_tokens >= (1ull << 32)) return mvr::fail(c, MVR_E_INVALID_ARGUMENT, "more than 2^32-1 tokens");

  using clk = std::chrono::steady_clock;
  const auto t_start = clk::now();
  double host_ms = 0.0;
  auto since = [](clk::time_point a) { return std::chrono::duration<double, std::milli>(clk::now() - a).count(); };
  c->tac_stats = mvr_tac_stats{};
  // ---- step 0-1: vocabulary, frequencies, CSR grouping (host) -------------
  uint32_t max_id = 0;
  for (uint64_t i = 0; i < n_tokens; ++i) max_id = std::max(max_id, token_ids[i]);
  const uint64_t nd = (uint64_t)max_id + 1;
  if (n_distinct_out) *n_distinct_out = nd;
  if (kappa_cap < nd) return mvr::fail(c, MVR_E_OUT_BUFFER_WRONG_SIZE, "kappa_per_token buffer too small");
  std::vector<uint32_t> freqs(nd, 0), goff(nd + 1, 0), gidx(n_tokens), rowtok(n_tokens);
  auto group_rows = [&] {
    for (uint64_t i = 0; i < n_tokens; ++i) ++freqs[token_ids[i]];
    for (uint64_t j = 0; j < nd; ++j) goff[j + 1] = goff[j] + freqs[j];
    std::vector<uint32_t> cur(goff.begin(), goff.end() - 1);
    for (uint64_t i = 0; i < n_tokens; ++i) gidx[cur[token_ids[i]]++] = (uint32_t)i;
    for (uint64_t j = 0; j < nd; ++j)
      for (uint32_t q = goff[j]; q < goff[j + 1]; ++q) rowtok[q] = (uint32_t)j;
  };
  host_ms += since(t_start);
  mvr::DeviceScope dev_scope(c);
  MVR_TRY(dev_scope.status);
  cudaStream_t st = c->stream;
  cudaEvent_t* tev = nullptr;
  MVR_TRY(mvr::tac_events(c, &tev));
  float *d_V = nullptr, *d_G = nullptr, *d_sp = nullptr, *d_C = nullptr;
  uint32_t *d_gidx = nullptr, *d_goff = nullptr, *d_local = nullptr, *d_rowtok = nullptr, *d_goffc = nullptr,
           *d_asg = nullptr;
  const uint64_t rows = n_tokens;
  MVR_TRY(mvr::scratch(c, mvr::kSlotResiduals, rows * dim * sizeof(float), (void**)&d_V));
  MVR_TRY(mvr::scratch(c, mvr::kSlotSorted, rows * dim * sizeof(float), (void**)&d_G));
  float* d_GT = nullptr;
  if (G == 1) MVR_TRY(mvr::scratch(c, mvr::kSlotMinDist, rows * ((dim + 3) / 4) * 4 * sizeof(float), (void**)&d_GT));
  MVR_TRY(mvr::scratch(c, mvr::kSlotAux0, rows * sizeof(uint32_t), (void**)&d_gidx));
  MVR_TRY(mvr::scratch(c, mvr::kSlotAux1, rows * sizeof(uint32_t), (void**)&d_local));
  MVR_TRY(mvr::scratch(c, mvr::kSlotAux2, rows * sizeof(uint32_t) * 2 + (nd + 1) * 4 * 2 + nd * 4 + 1024,
                       (void**)&d_rowtok));
  d_asg = d_rowtok + rows;
  d_goff = d_asg + rows;
  d_goffc = d_goff + (nd + 1);
  d_sp = reinterpret_cast<float*>(d_goffc + (nd + 1));
  // the grouping runs on a second host thread while the rows stream in
  MVR_CUDA(c, cudaEventRecord(tev[0], st));
  {
    std::thread grouper(group_rows);
    const int s_v = mvr::h2d_staged(c, d_V, vectors, rows * dim * sizeof(float));
    grouper.join();
    MVR_TRY(s_v);
  }
  MVR_CUDA(c, cudaMemcpyAsync(d_gidx, gidx.data(), rows * 4, cudaMemcpyHostToDevice, st));
  MVR_CUDA(c, cudaMemcpyAsync(d_goff, goff.data(), (nd + 1) * 4, cudaMemcpyHostToDevice, st));
  MVR_CUDA(c, cudaMemcpyAsync(d_rowtok, rowtok.data(), rows * 4, cudaMemcpyHostToDevice, st));
  MVR_CUDA(c, cudaEventRecord(tev[1], st));
  // the sharded run gathers each rank's own tokens again below, so the
  // full group-major copy is not needed there
  MVR_TRY(mvr::km_gather_groups(c, d_V, d_gidx, rows, dim, d_G, G > 1 ? nullptr : d_GT));
  int* d_err = reinterpret_cast<int*>(d_sp + nd);
  MVR_CUDA(c, cudaMemsetAsync(d_err, 0, sizeof(int), st));
  MVR_TRY(mvr::launch_spreads(c, d_G, dim, d_goff, nd, d_sp, d_err));
  // a rank whose spread pass timed out fails with all the others
  if (G > 1) MVR_TRY(mvr::comm_allreduce_sum_u32(c, reinterpret_cast<uint32_t*>(d_err), 1));
  MVR_CUDA(c, cudaEventRecord(tev[2], st));
  std::vector<float> spreads(nd + 1);  // spreads, then the kernel's error flag
  MVR_CUDA(c, cudaMemcpyAsync(spreads.data(), d_sp, (nd + 1) * 4, cudaMemcpyDeviceToHost, st));
  MVR_CUDA(c, cudaStreamSynchronize(st));
  {
    int spread_err = 0;
    std::memcpy(&spread_err, &spreads[nd], sizeof(int));
    if (spread_err) return mvr::fail(c, MVR_E_TIMEOUT, "spread kernel: a bulk copy did not complete in time");
  }

  // ---- step 3: budget phases 1-4 (host) ------------------------------------
  const auto t_budget = clk::now();
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
  // With several ranks each one runs the problems it owns on a compact copy
  // of their rows (local row and centroid offsets).
  std::vector<uint32_t> owner(nd, 0);
  if (G > 1) mvr::tac_partition_tokens_host(freqs.data(), kap.data(), nd, (uint32_t)G, owner.data());
  mvr::KmBatch b;
  std::vector<uint32_t> pj;  // token id of each problem
  uint64_t lrows = 0, lcent = 0;
  for (uint64_t j = 0; j < nd; ++j) {
    if (kap[j] == 0 || freqs[j] == 0 || owner[j] != (uint32_t)me) continue;
    b.off.push_back(G > 1 ? lrows : goff[j]);
    b.n.push_back(freqs[j]);
    b.k.push_back(kap[j]);
    b.coff.push_back(G > 1 ? lcent : goffc[j]);
    b.seed.push_back(p->seed ^ (uint64_t)j);
    pj.push_back((uint32_t)j);
    lrows += freqs[j];
    lcent += kap[j];
  }
  std::vector<uint32_t> own_idx, own_tok, cmap;
  if (G > 1) {
    own_idx.resize(lrows);
    own_tok.resize(lrows);
    cmap.resize(lcent);
    uint64_t q = 0, cc = 0;
    for (uint32_t j : pj) {
      for (uint32_t r = goff[j]; r < goff[j + 1]; ++r, ++q) {
        own_idx[q] = gidx[r];
        own_tok[q] = j;
      }
      for (uint32_t k = 0; k < kap[j]; ++k) cmap[cc++] = goffc[j] + k;
    }
  }
  host_ms += since(t_budget);
  MVR_TRY(mvr::scratch(c, mvr::kSlotCodebooks, (size_t)p->kappa_total * dim * sizeof(float), (void**)&d_C));
  mvr::KmResult r;
  float* d_CL = d_C;       // this rank's centroids (local rows when sharded)
  uint32_t* d_oidx = nullptr;  // sharded: own rows' input positions, then their token ids
  uint32_t* d_cmap = nullptr;  // sharded: global row of each local centroid, then the per-token info
  if (G > 1) {
    float *d_G2 = nullptr, *d_GT2 = nullptr;
    MVR_TRY(mvr::scratch(c, mvr::kSlotAssign, std::max<uint64_t>(lrows * dim, 4) * sizeof(float), (void**)&d_G2));
    MVR_TRY(mvr::scratch(c, mvr::kSlotHist, std::max<uint64_t>(lrows * ((dim + 3) / 4) * 4, 4) * sizeof(float),
                         (void**)&d_GT2));
    MVR_TRY(mvr::scratch(c, mvr::kSlotChunk, std::max<uint64_t>(2 * lrows, 4) * 4, (void**)&d_oidx));
    MVR_TRY(mvr::scratch(c, mvr::kSlotCodes, std::max<uint64_t>(lcent * dim, 4) * sizeof(float), (void**)&d_CL));
    MVR_TRY(mvr::scratch(c, mvr::kSlotSmall, (lcent + 3 * nd + 4) * 4, (void**)&d_cmap));
    if (lrows) {
      MVR_CUDA(c, cudaMemcpyAsync(d_oidx, own_idx.data(), lrows * 4, cudaMemcpyHostToDevice, st));
      MVR_CUDA(c, cudaMemcpyAsync(d_oidx + lrows, own_tok.data(), lrows * 4, cudaMemcpyHostToDevice, st));
      MVR_CUDA(c, cudaMemcpyAsync(d_cmap, cmap.data(), lcent * 4, cudaMemcpyHostToDevice, st));
      MVR_TRY(mvr::km_gather_groups(c, d_V, d_oidx, lrows, dim, d_G2, d_GT2));
    }
    MVR_TRY(mvr::km_batch_run(c, d_G2, d_GT2, lrows, dim, b, p->max_iters, p->tol, d_CL, d_local, &r));
  } else {
    MVR_TRY(mvr::km_batch_run(c, d_G, d_GT, rows, dim, b, p->max_iters, p->tol, d_C, d_local, &r));
  }

  // per-token results of every rank: WCSS bits, status, iterations
  std::vector<float> tw(nd, 0.f);
  std::vector<uint32_t> tstat(nd, 0), titer(nd, 0);
  for (size_t q = 0; q < pj.size(); ++q) {
    tw[pj[q]] = r.wcss[q];
    tstat[pj[q]] = (uint32_t)r.status[q];
    titer[pj[q]] = r.iters[q];
  }
  MVR_CUDA(c, cudaMemcpyAsync(d_goffc, goffc.data(), (nd + 1) * 4, cudaMemcpyHostToDevice, st));
  const int sgrid = (int)std::min<uint64_t>((rows + 255) / 256, (uint64_t)c->sm_count * 8);
  if (G > 1) {
    // every output value is written by exactly one rank and is zero on the
    // others, so a u32 sum of the bit patterns merges them exactly
    uint32_t* d_info = d_cmap + lcent;
    std::vector<uint32_t> info(3 * nd);
    std::memcpy(info.data(), tw.data(), nd * 4);
    std::memcpy(info.data() + nd, tstat.data(), nd * 4);
    std::memcpy(info.data() + 2 * nd, titer.data(), nd * 4);
    MVR_CUDA(c, cudaMemcpyAsync(d_info, info.data(), 3 * nd * 4, cudaMemcpyHostToDevice, st));
    MVR_TRY(mvr::comm_allreduce_sum_u32(c, d_info, 3 * nd));
    MVR_CUDA(c, cudaMemcpyAsync(info.data(), d_info, 3 * nd * 4, cudaMemcpyDeviceToHost, st));
    MVR_CUDA(c, cudaStreamSynchronize(st));
    std::memcpy(tw.data(), info.data(), nd * 4);
    std::memcpy(tstat.data(), info.data() + nd, nd * 4);
    std::memcpy(titer.data(), info.data() + 2 * nd, nd * 4);
  }
  for (uint64_t j = 0; j < nd; ++j)  // the lowest failing token, as the serial reference reports
    if (tstat[j] != MVR_OK)
      return mvr::fail(c, (int)tstat[j], std::string("token ") + std::to_string(j) + ": " +
                                             mvr_status_name((int)tstat[j]));

  // ---- outputs ----------------------------------------------------------------
  if (G > 1) {
    MVR_CUDA(c, cudaMemsetAsync(d_C, 0, (size_t)p->kappa_total * dim * sizeof(float), st));
    MVR_CUDA(c, cudaMemsetAsync(d_asg, 0, rows * 4, st));
    if (lrows) {
      const int cgrid = (int)std::min<uint64_t>((lcent * dim + 255) / 256, (uint64_t)c->sm_count * 8);
      mvr::tac_place_centroids_kernel<<<cgrid, 256, 0, st>>>(d_CL, d_cmap, lcent, dim, d_C);
      mvr::tac_scatter_assign_kernel<<<sgrid, 256, 0, st>>>(d_oidx, d_oidx + lrows, d_goffc, d_local, lrows, d_asg);
      MVR_CUDA(c, cudaGetLastError());
    }
    MVR_TRY(mvr::comm_allreduce_sum_u32(c, reinterpret_cast<uint32_t*>(d_C), (size_t)p->kappa_total * dim));
    MVR_TRY(mvr::comm_allreduce_sum_u32(c, d_asg, rows));
  } else {
    mvr::tac_scatter_assign_kernel<<<sgrid, 256, 0, st>>>(d_gidx, d_rowtok, d_goffc, d_local, rows, d_asg);
    MVR_CUDA(c, cudaGetLastError());
  }
  MVR_CUDA(c, cudaEventRecord(tev[3], st));
  MVR_CUDA(c, cudaMemcpyAsync(assignments_out, d_asg, rows * 4, cudaMemcpyDeviceToHost, st));
  MVR_CUDA(c, cudaMemcpyAsync(centroids_out, d_C, (size_t)p->kappa_total * dim * sizeof(float),
                              cudaMemcpyDeviceToHost, st));
  MVR_CUDA(c, cudaEventRecord(tev[4], st));
  MVR_CUDA(c, cudaStreamSynchronize(st));
  const auto t_tail = clk::now();

  // wcss_total: per-token WCSS summed in token order, per static thread chunk
  // when n_threads > 1 (tac.zig:685-825).
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
  {
    mvr_tac_stats& ts = c->tac_stats;
    float h2d = 0.f, spr = 0.f, d2h = 0.f;
    cudaEventElapsedTime(&h2d, tev[0], tev[1]);
    cudaEventElapsedTime(&spr, tev[1], tev[2]);
    cudaEventElapsedTime(&d2h, tev[3], tev[4]);
    ts.h2d_ms = h2d;
    ts.spread_ms = spr;
    ts.d2h_ms = d2h;
    ts.seed_ms = r.seed_ms;
    ts.lloyd_ms = r.lloyd_ms;
    ts.problems = (uint32_t)pj.size();
    ts.iters_max = 0;
    for (uint64_t j = 0; j < nd; ++j) ts.iters_max = std::max(ts.iters_max, titer[j]);
    ts.seed_fallbacks = r.seed_fallbacks;
    ts.launches = r.launches + (G > 1 ? 6 : 4);
    ts.filter_rows_rechecked = r.filter_rows_rechecked;
    ts.filter_violations = r.filter_violations;
    ts.filter_rows_full_scan = r.filter_rows_full_scan;
    ts.host_ms = host_ms + since(t_tail);
    ts.total_ms = since(t_start);
  }
  for (uint64_t i = 0; i < n_tokens; ++i)  // final invariant (tac.zig:827-830)
    if (assignments_out[i] >= p->kappa_total) return mvr::fail(c, MVR_E_INVALID_THRESHOLDS, "assignment out of range");
  return MVR_OK;
}

}  // namespace

extern "C" int mvr_tac_cluster_flat(mvr_ctx* h, const uint32_t* token_ids, uint64_t n_tokens, const float* vectors,
                                    uint64_t vectors_len, uint32_t dim, const mvr_clustering_params* p,
                                    float* centroids_out, uint32_t* assignments_out, uint32_t* kappa_out,
                                    uint64_t kappa_cap, uint64_t* n_distinct_out, float* wcss_total_out) {
  return cluster_flat(h, token_ids, n_tokens, vectors, vectors_len, dim, p, centroids_out, assignments_out,
                      kappa_out, kappa_cap, n_distinct_out, wcss_total_out, false);
}

extern "C" int mvr_tac_cluster_flat_sharded(mvr_ctx* h, const uint32_t* token_ids, uint64_t n_tokens,
                                            const float* vectors, uint64_t vectors_len, uint32_t dim,
                                            const mvr_clustering_params* p, float* centroids_out,
                                            uint32_t* assignments_out, uint32_t* kappa_out, uint64_t kappa_cap,
                                            uint64_t* n_distinct_out, float* wcss_total_out) {
  return cluster_flat(h, token_ids, n_tokens, vectors, vectors_len, dim, p, centroids_out, assignments_out,
                      kappa_out, kappa_cap, n_distinct_out, wcss_total_out, true);
}
