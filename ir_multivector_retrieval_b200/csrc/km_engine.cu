// km_engine.cu — ragged batch of independent k-means problems, any dim.
//
// Reference: kmeans.fit (src/tac/kmeans.zig:67-232), rng.weightedSample
// (src/util/rng.zig:57-82), vec.l2sq (src/util/vec.zig:109-175), and the
// per-token driver runOneTokenKmeans (src/tac/tac.zig:458-514).
//
// Layout in HBM (R = rows of G, d = dim, KT = sum of k over problems):
//   G      [R][d]   rows grouped by problem (the caller gathers them)
//   C      [KT][d]  centroids, problem p at rows [coff_p, coff_p + k_p)
//   md     [R]      k-means++ D^2 weights, then Lloyd min_to_any
//   local  [R]      Lloyd assignment of each row, local to its problem
//   keys/vals [R]   global cluster id / row, radix-sorted (stable) so that
//                   each cluster's members follow in row order
//   counts/starts [KT]
//
// Schedules:
//   * seeding runs in lockstep over centroid index s; problems are ordered
//     by k descending, so the problems (and their 1024-row chunks) that
//     still draw at step s form a prefix;
//   * Lloyd runs all problems together; converged problems are skipped.
// Exactness follows pq_engine.cu: exact reference distance order, first-
// index argmin, in-order sequential centroid sums, rigorous k-means++ draws.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <numeric>
#include <vector>

#include "km_engine.h"
#include "mvr_device.cuh"
#include "mvr_rng.h"
#include "tc_filter.cuh"

namespace mvr {
namespace {

constexpr int kChunk = 1024;       // seeding chunk; one select thread per row
constexpr int kUpdT = 256;         // seed-update CTA
constexpr int kSelT = 1024;        // select CTA
constexpr int kAsgT = 128;         // assign CTA: one row per thread
constexpr int kCT = 32;            // centroids per shared-memory tile
constexpr int kRadixRows = 2048;   // rows per radix block (one warp)
constexpr int kRadixWarps = 4;
constexpr int kCrossingSlack = 300;
constexpr uint32_t kWcssSeg = 32768;  // problems at least this long take the segmented WCSS sum

enum : uint8_t { kRunning = 0, kDone = 1, kFailed = 2 };

// vec.l2sq for any length with the 4-lane layout (vec.zig:128-175 with
// lane_count 4): strided lane accumulators over whole groups of 4, the
// ordered reduction, then the scalar tail. For lengths 1-4, 64 and 128 this
// is the same arithmetic as the reference's specialisations.
__device__ __forceinline__ float l2_gen(const float* __restrict__ x, const float* __restrict__ c, int d) {
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
  int i = 0;
  for (; i + 4 <= d; i += 4) {
    const float d0 = __fsub_rn(x[i], c[i]), d1 = __fsub_rn(x[i + 1], c[i + 1]);
    const float d2 = __fsub_rn(x[i + 2], c[i + 2]), d3 = __fsub_rn(x[i + 3], c[i + 3]);
    a0 = __fadd_rn(a0, __fmul_rn(d0, d0));
    a1 = __fadd_rn(a1, __fmul_rn(d1, d1));
    a2 = __fadd_rn(a2, __fmul_rn(d2, d2));
    a3 = __fadd_rn(a3, __fmul_rn(d3, d3));
  }
  float s = __fadd_rn(__fadd_rn(__fadd_rn(a0, a1), a2), a3);
  for (; i < d; ++i) {
    const float t = __fsub_rn(x[i], c[i]);
    s = __fadd_rn(s, __fmul_rn(t, t));
  }
  return s;
}

struct Prob {
  const uint64_t* off;
  const uint32_t* n;
  const uint32_t* k;
  const uint64_t* coff;
  uint8_t* state;
  int* status;
  float* wcss;
  float* prev;
  uint32_t* iters;
  double* thr;
  uint32_t* fb;
  int* nonf;
};

__device__ __forceinline__ double gamma_bound(uint64_t n) {
  const double g = __dmul_ru(__ull2double_ru(n), 1.1102230246251565e-16);
  return __ddiv_ru(g, __dsub_rd(1.0, g));
}

// ---------------------------------------------------------------------------
// Row gather and the group-major copy. CTA = 32 rows: rows are read whole
// (V[idx[q]] or V[q]) into a shared tile whose row stride is 4 mod 32 words,
// written back row-major to G (optional) and as float4 groups to GT, where
// group g of rows q0..q0+31 is one contiguous 512-byte run. Coordinates past
// d in the last group are zero.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
km_gather_groups_kernel(const float* __restrict__ V, const uint32_t* __restrict__ idx, uint64_t n, int d,
                        int stride, float* __restrict__ G, float4* __restrict__ GT) {
  extern __shared__ __align__(16) float tile[];
  const uint64_t q0 = (uint64_t)blockIdx.x * 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ng4 = (d + 3) >> 2;
  for (int i = warp; i < 32; i += 8) {
    const uint64_t q = q0 + i;
    if (q < n) {
      const float* src = V + (idx ? (uint64_t)idx[q] : q) * d;
      for (int e = lane; e < ng4 * 4; e += 32) {
        const float v = e < d ? src[e] : 0.f;
        tile[i * stride + e] = v;
        if (G && e < d) G[q * d + e] = v;
      }
    }
  }
  if (!GT) return;
  __syncthreads();
  for (int t = threadIdx.x; t < ng4 * 32; t += 256) {
    const int g = t >> 5, i = t & 31;
    const uint64_t q = q0 + i;
    if (q < n) GT[(uint64_t)g * n + q] = *reinterpret_cast<const float4*>(tile + i * stride + 4 * g);
  }
}

// ---------------------------------------------------------------------------
// degenerate k >= n (kmeans.zig:88-104)
// ---------------------------------------------------------------------------
__global__ void km_degenerate_kernel(const float* __restrict__ G, int d, Prob P,
                                     const uint32_t* __restrict__ list, float* __restrict__ C,
                                     uint32_t* __restrict__ local, uint32_t* __restrict__ keys) {
  const uint32_t p = list[blockIdx.x];
  const uint64_t off = P.off[p];
  const uint32_t n = P.n[p], k = P.k[p];
  const uint64_t co = P.coff[p];
  for (uint64_t e = threadIdx.x; e < (uint64_t)k * d; e += blockDim.x) {
    const uint64_t c = e / d, j = e % d;
    const uint64_t row = c < n ? c : n - 1;
    C[(co + c) * d + j] = G[(off + row) * d + j];
  }
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
    local[off + i] = i;
    keys[off + i] = (uint32_t)(co + i);  // every row carries a valid sort key
  }
}

// ---------------------------------------------------------------------------
// k-means++ seeding
// ---------------------------------------------------------------------------
__global__ void km_seed_init_kernel(const float* __restrict__ G, int d, Prob P,
                                    const uint32_t* __restrict__ list, const uint64_t* __restrict__ idx0,
                                    float* __restrict__ C) {
  const uint32_t p = list[blockIdx.x];
  const uint64_t src = (P.off[p] + idx0[p]) * d, dst = P.coff[p] * d;
  for (int j = threadIdx.x; j < d; j += blockDim.x) C[dst + j] = G[src + j];
}

// l2_gen over the group-major copy GT (float4 group g of row r at
// GT[g * R + r]): the same lane layout (coordinate 4g + l feeds lane l),
// ordered reduction and scalar tail as l2_gen. NG = d / 4 when it is a
// compile-time constant (64 -> 16, 128 -> 32), 0 for any d.
template <int NG>
__device__ __forceinline__ float l2_groups(const float4* __restrict__ GT, uint64_t R, uint64_t r,
                                           const float4* __restrict__ c4, int d) {
  const int ng = NG > 0 ? NG : d >> 2;
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll(NG > 0 ? NG : 1)
  for (int g = 0; g < ng; ++g) {
    const float4 v = __ldg(GT + (uint64_t)g * R + r);
    const float4 c = c4[g];
    const float d0 = __fsub_rn(v.x, c.x), d1 = __fsub_rn(v.y, c.y);
    const float d2 = __fsub_rn(v.z, c.z), d3 = __fsub_rn(v.w, c.w);
    a0 = __fadd_rn(a0, __fmul_rn(d0, d0));
    a1 = __fadd_rn(a1, __fmul_rn(d1, d1));
    a2 = __fadd_rn(a2, __fmul_rn(d2, d2));
    a3 = __fadd_rn(a3, __fmul_rn(d3, d3));
  }
  float s = __fadd_rn(__fadd_rn(__fadd_rn(a0, a1), a2), a3);
  if (NG == 0 && (d & 3)) {
    const float4 v = __ldg(GT + (uint64_t)ng * R + r);
    const float4 c = c4[ng];
    const float t0 = __fsub_rn(v.x, c.x);
    s = __fadd_rn(s, __fmul_rn(t0, t0));
    if ((d & 3) > 1) {
      const float t1 = __fsub_rn(v.y, c.y);
      s = __fadd_rn(s, __fmul_rn(t1, t1));
    }
    if ((d & 3) > 2) {
      const float t2 = __fsub_rn(v.z, c.z);
      s = __fadd_rn(s, __fmul_rn(t2, t2));
    }
  }
  return s;
}

// min_dist update with centroid `step` for the active chunks, plus per-chunk
// directed-rounding sums and the count of non-zero weights below thr. Rows
// come from the group-major copy, so each float4 load of a warp is one
// contiguous 512-byte segment.

template <int NG>
__global__ void __launch_bounds__(kUpdT)
km_seed_update_kernel(const float4* __restrict__ GT, uint64_t R, int d, Prob P, int step,
                      const uint32_t* __restrict__ ch_p, const uint64_t* __restrict__ ch_r0,
                      const uint32_t* __restrict__ ch_len, const float* __restrict__ C,
                      float* __restrict__ md, double2* __restrict__ ch_sum,
                      uint32_t* __restrict__ ch_cnt) {
  extern __shared__ __align__(16) float4 cen4[];
  __shared__ double2 wp[kUpdT / 32];
  __shared__ uint32_t wc[kUpdT / 32];
  grid_dependency_wait();  // launched early (programmatic dependent launch): the last step completes first
  const uint32_t p = ch_p[blockIdx.x];
  if (P.state[p] != kRunning) return;
  const uint64_t co = P.coff[p] + step;
  const int ng4 = (d + 3) >> 2;
  float* cen = reinterpret_cast<float*>(cen4);
  for (int j = threadIdx.x; j < ng4 * 4; j += kUpdT) cen[j] = j < d ? C[co * d + j] : 0.f;
  __syncthreads();
  const uint64_t r0 = ch_r0[blockIdx.x];
  const uint32_t len = ch_len[blockIdx.x];
  const double T = P.thr[p];
  double lo = 0.0, hi = 0.0;
  uint32_t cnt = 0;
  bool bad = false;
  constexpr int kRowsPerThread = kChunk / kUpdT;
  float dist[kRowsPerThread];
#pragma unroll
  for (int u = 0; u < kRowsPerThread; ++u) {
    const uint32_t i = threadIdx.x + u * kUpdT;
    dist[u] = i < len ? l2_groups<NG>(GT, R, r0 + i, cen4, d) : 0.f;
  }
#pragma unroll
  for (int u = 0; u < kRowsPerThread; ++u) {
    const uint32_t i = threadIdx.x + u * kUpdT;
    if (i < len) {
      const uint64_t r = r0 + i;
      float w;
      if (step == 0) {
        w = dist[u];
      } else {
        const float old = md[r];
        w = dist[u] < old ? dist[u] : old;
      }
      md[r] = w;
      bad |= !isfinite(w) || w < 0.f;
      lo = __dadd_rd(lo, (double)w);
      hi = __dadd_ru(hi, (double)w);
      cnt += (w != 0.f && (double)w < T) ? 1u : 0u;
    }
  }
  if (bad) P.nonf[p] = 1;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  lo = warp_sum_rd(lo);
  hi = warp_sum_ru(hi);
  cnt = __reduce_add_sync(0xffffffffu, cnt);
  if (lane == 0) {
    wp[warp] = make_double2(lo, hi);
    wc[warp] = cnt;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double a = 0.0, b = 0.0;
    uint32_t c = 0;
    for (int w = 0; w < kUpdT / 32; ++w) {
      a = __dadd_rd(a, wp[w].x);
      b = __dadd_ru(b, wp[w].y);
      c += wc[w];
    }
    ch_sum[blockIdx.x] = make_double2(a, b);
    ch_cnt[blockIdx.x] = c;
  }
}

// One weightedSample draw for each active problem (see pq_seed_select_kernel
// in pq_engine.cu for the acceptance argument).
__global__ void __launch_bounds__(kSelT)
km_seed_select_kernel(const float* __restrict__ G, int d, Prob P, int step,
                      const uint32_t* __restrict__ sel_p, const uint32_t* __restrict__ cfirst,
                      const uint32_t* __restrict__ ccount, const uint64_t* __restrict__ ch_r0,
                      const uint32_t* __restrict__ ch_len, const double2* __restrict__ ch_sum,
                      const uint32_t* __restrict__ ch_cnt, const float* __restrict__ md,
                      const double* __restrict__ draws, float* __restrict__ C, int force_chain) {
  grid_dependency_wait();
  const uint32_t p = sel_p[blockIdx.x];
  if (P.state[p] != kRunning) return;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int kWarps = kSelT / 32;
  __shared__ double2 wsum[kWarps];
  __shared__ unsigned long long wcnt[kWarps];
  __shared__ double2 incl_all[kSelT];
  __shared__ double2 sh_excl;
  __shared__ int sh_chunk;
  __shared__ uint64_t sh_idx;
  __shared__ int sh_decided;

  if (P.nonf[p]) {
    if (tid == 0) { P.status[p] = MVR_E_NON_FINITE; P.state[p] = kFailed; }
    return;
  }
  const uint64_t off = P.off[p];
  const uint64_t N = P.n[p];
  const float* w = md + off;
  const double r = draws[P.coff[p] + step];
  const uint32_t cf = cfirst[p], cc = ccount[p];

  const uint32_t cpt = (cc + kSelT - 1) / kSelT;
  const uint32_t c_lo = min(cc, tid * cpt), c_hi = min(cc, c_lo + cpt);
  double tlo = 0.0, thi = 0.0;
  unsigned tcnt = 0;
  for (uint32_t j = c_lo; j < c_hi; ++j) {
    tlo = __dadd_rd(tlo, ch_sum[cf + j].x);
    thi = __dadd_ru(thi, ch_sum[cf + j].y);
    tcnt += ch_cnt[cf + j];
  }
  const double ilo = warp_scan_rd(tlo, lane), ihi = warp_scan_ru(thi, lane);
  const unsigned wc = __reduce_add_sync(0xffffffffu, tcnt);
  if (lane == 31) wsum[warp] = make_double2(ilo, ihi);
  if (lane == 0) wcnt[warp] = wc;
  __syncthreads();
  if (warp == 0) {
    const double a = warp_scan_rd(wsum[lane].x, lane);
    const double b = warp_scan_ru(wsum[lane].y, lane);
    unsigned long long cs = wcnt[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) cs += __shfl_xor_sync(0xffffffffu, cs, o);
    __syncwarp();
    wsum[lane] = make_double2(a, b);
    wcnt[lane] = cs;
  }
  __syncthreads();
  const double wlo = warp > 0 ? wsum[warp - 1].x : 0.0, whi = warp > 0 ? wsum[warp - 1].y : 0.0;
  const double incl_lo = __dadd_rd(wlo, ilo), incl_hi = __dadd_ru(whi, ihi);
  const double Lo_N = wsum[kWarps - 1].x, Hi_N = wsum[kWarps - 1].y;
  const unsigned long long C_N = wcnt[0];
  if (Hi_N <= 0.0) {
    if (tid == 0) { P.status[p] = MVR_E_ALL_ZERO; P.state[p] = kFailed; }
    return;
  }
  const double gN = gamma_bound(N);
  const double shi_classic = __dadd_ru(Hi_N, __dmul_ru(gN, Hi_N));
  int e2 = 0;
  (void)frexp(shi_classic, &e2);
  const double Gu = ldexp(1.0, e2 - 53);
  const double thr_now = ldexp(Gu, 23);
  const double B_tight = __dmul_ru(__ull2double_ru(C_N + kCrossingSlack), 0.5 * Gu);
  const double thr_prev = P.thr[p];
  const bool tight_ok = thr_now <= thr_prev;
  auto bound_at = [&](uint64_t terms, double hi_prefix) {
    const double bg = __dmul_ru(gamma_bound(terms), hi_prefix);
    return tight_ok ? fmin(bg, B_tight) : bg;
  };
  const double u_mid = r * (0.5 * (Lo_N + Hi_N));
  const bool past = !(u_mid < 0.5 * (incl_lo + incl_hi));
  incl_all[tid] = make_double2(incl_lo, incl_hi);
  const int n_before = __syncthreads_count(past);
  if (tid == 0) {
    sh_decided = 0;
    sh_chunk = -1;
    if (thr_now < thr_prev) P.thr[p] = thr_now;
  }
  __syncthreads();
  if (n_before < kSelT && tid == n_before) {
    double lo = tid > 0 ? incl_all[tid - 1].x : 0.0;
    double hi = tid > 0 ? incl_all[tid - 1].y : 0.0;
    int found = -1;
    for (uint32_t j = c_lo; j < c_hi; ++j) {
      const double nlo = __dadd_rd(lo, ch_sum[cf + j].x), nhi = __dadd_ru(hi, ch_sum[cf + j].y);
      if (u_mid < 0.5 * (nlo + nhi)) { found = (int)j; break; }
      lo = nlo;
      hi = nhi;
    }
    sh_chunk = found;
    sh_excl = make_double2(lo, hi);
  }
  __syncthreads();
  const int fchunk = sh_chunk;
  if (fchunk >= 0) {
    const uint64_t r0 = ch_r0[cf + fchunk] - off;  // row index within the problem
    const uint32_t len = ch_len[cf + fchunk];
    const uint64_t i = r0 + tid;
    const double v = (uint32_t)tid < len ? (double)w[i] : 0.0;
    const double slo = warp_scan_rd(v, lane), shi = warp_scan_ru(v, lane);
    if (lane == 31) wsum[warp] = make_double2(slo, shi);
    __syncthreads();
    if (warp == 0) {
      const double a = warp_scan_rd(wsum[lane].x, lane);
      const double b = warp_scan_ru(wsum[lane].y, lane);
      __syncwarp();
      wsum[lane] = make_double2(a, b);
    }
    __syncthreads();
    const double2 ex = sh_excl;
    const double plo = warp > 0 ? wsum[warp - 1].x : 0.0, phi = warp > 0 ? wsum[warp - 1].y : 0.0;
    const double elo = __dadd_rd(ex.x, __dadd_rd(plo, slo));
    const double ehi = __dadd_ru(ex.y, __dadd_ru(phi, shi));
    incl_all[tid] = make_double2(elo, ehi);
    const bool valid = (uint32_t)tid < len;
    const bool hit = !valid || u_mid < 0.5 * (elo + ehi);
    const int first = __syncthreads_count(!hit);
    if (first < kSelT && tid == first && valid) {
      const double2 prv = tid > 0 ? incl_all[tid - 1] : ex;
      const double BN = bound_at(N, Hi_N);
      const double ULo = __dmul_rd(r, __dsub_rd(Lo_N, BN));
      const double UHi = __dmul_ru(r, __dadd_ru(Hi_N, BN));
      bool ok = UHi < __dsub_rd(elo, bound_at(i + 1, ehi));
      if (i > 0) ok = ok && (ULo >= __dadd_ru(prv.y, bound_at(i, prv.y)));
      if (ok && !force_chain) {
        sh_idx = i;
        sh_decided = 1;
      }
    }
  }
  __syncthreads();
  if (!sh_decided && tid == 0) {  // the reference's sequential chain
    double total = 0.0;
    uint64_t last_pos = 0;
    for (uint64_t q = 0; q < N; ++q) {
      const float v = w[q];
      total = __dadd_rn(total, (double)v);
      if (v != 0.f) last_pos = q;
    }
    const double u = __dmul_rn(r, total);
    double cum = 0.0;
    uint64_t pick = last_pos;
    for (uint64_t q = 0; q < N; ++q) {
      cum = __dadd_rn(cum, (double)w[q]);
      if (u < cum) { pick = q; break; }
    }
    sh_idx = pick;
    P.fb[p] += 1;
  }
  __syncthreads();
  const uint64_t idx = sh_idx;
  const uint64_t dst = (P.coff[p] + step) * d, src = (off + idx) * d;
  for (int j = tid; j < d; j += kSelT) C[dst + j] = G[src + j];
}

// ---------------------------------------------------------------------------
// Lloyd assignment: one row per thread, centroids through shared memory in
// tiles of kCT. DIM > 0 keeps the row in registers; DIM == 0 is the generic
// path (row read through L1). Writes the local id, the min distance, the
// global sort key and the cluster count.
// ---------------------------------------------------------------------------
template <int DIM>
__global__ void __launch_bounds__(kAsgT)
km_assign_kernel(const float* __restrict__ G, int d_rt, Prob P, const uint32_t* __restrict__ t_p,
                 const uint64_t* __restrict__ t_r0, const uint32_t* __restrict__ t_len,
                 const float* __restrict__ C, uint32_t* __restrict__ local, float* __restrict__ mind,
                 uint32_t* __restrict__ keys) {
  extern __shared__ __align__(16) float ct[];
  const int d = DIM > 0 ? DIM : d_rt;
  const uint32_t p = t_p[blockIdx.x];
  if (P.state[p] != kRunning) return;
  const uint32_t k = P.k[p];
  const uint64_t co = P.coff[p];
  const uint32_t len = t_len[blockIdx.x];
  const uint64_t r = t_r0[blockIdx.x] + threadIdx.x;
  const bool ok = threadIdx.x < len;
  float xr[DIM > 0 ? DIM : 1];
  const float* xg = G + (ok ? r : t_r0[blockIdx.x]) * d;
  if constexpr (DIM > 0) {
#pragma unroll
    for (int j = 0; j < DIM; j += 4) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(xg + j));
      xr[j] = v.x; xr[j + 1] = v.y; xr[j + 2] = v.z; xr[j + 3] = v.w;
    }
  }
  float best = 0.f, d0 = 0.f;
  uint32_t bi = 0;
  for (uint32_t c0 = 0; c0 < k; c0 += kCT) {
    const uint32_t nt = min((uint32_t)kCT, k - c0);
    __syncthreads();
    for (uint32_t e = threadIdx.x; e < nt * (uint32_t)d; e += kAsgT) ct[e] = C[(co + c0) * d + e];
    __syncthreads();
    for (uint32_t j = 0; j < nt; ++j) {
      float dist;
      if constexpr (DIM > 0) dist = l2_wide<DIM>(xr, ct + j * DIM);
      else dist = l2_gen(xg, ct + j * d, d);
      const uint32_t c = c0 + j;
      if (c == 0) {
        best = dist;  // vec.argmin starts from dists[0]
        d0 = dist;
      } else if (dist < best) {
        best = dist;
        bi = c;
      }
    }
  }
  (void)d0;
  if (ok) {
    local[r] = bi;
    mind[r] = best;
    keys[r] = (uint32_t)(co + bi);
  }
}

// ---------------------------------------------------------------------------
// Tensor-core filtered Lloyd assignment for 64-dimensional rows (the TAC
// path) and problems with at least kKmTcMinK centroids.
//
// For a 128-row tile of problem p, the centroids go through in blocks of
// 256 columns; per block a chain of nine kind::tf32 MMAs (eight k-steps of
// the rows' TF32 values against -2c, plus one carrying |c|^2 and the row
// constant t) leaves a(c) = t + fl(|c|^2) - 2 x.c in a 256-column TMEM
// accumulator. With TF32 truncation of both operands (< 2^-10 relative
// each) and nine f32 accumulations,
//   |a(c) - (t + fl(|c|^2) - 2 x.c)| <= E = 2^-7 |x| max|c| + 2^-9 max|c|^2
//                                         + 2^-16 t + 2^-100,
// about twice the worst case. The reference winner (first minimum of the
// exact f32 distances, within 1 +- 2^-19 of the exact squared distances for
// 64 coordinates) then has a(w) <= T = a(c1) + 2E + 2^-17 D(c1) + 2 delta,
// delta = 2^-17 max|c|^2 bounding the f32 error of |c|^2. Each block's two
// smallest keys (f32 bits, low 8 bits = column) are merged into the row's
// running minimum; a block whose keys fall at or below the running T adds
// its columns at or below it to the row's candidate list (a re-read of the
// accumulator when there are several). T only shrinks as blocks go by, so
// the list holds every column at or below the final T, in column order; the
// exact 64-coordinate distances of the candidates decide, first minimum
// first. Lists that overflow, non-finite or huge rows, and problems whose
// centroids are non-finite or huge take the reference's full scan.
//
// One CTA per SM (two 256-column accumulators = all of TMEM): the block
// b + 1 centroid tile arrives by one bulk copy and its MMA chain runs while
// the four warps scan block b. Every wait is bounded; an expired wait sets
// *err and the CTA stops.
// ---------------------------------------------------------------------------
constexpr int kKmTcMinK = 64;
constexpr int kKmTcDim = 64;
constexpr int kKmTcSteps = kKmTcDim / 8 + 1;                     // k-steps per MMA chain
constexpr uint32_t kKmTcCols = 128;                              // centroids per block
constexpr uint32_t kKmTcStepB = kKmTcCols * 32;                  // one k-step of a block
constexpr uint32_t kKmTcBlockBytes = kKmTcSteps * kKmTcStepB;    // one 128-centroid block
constexpr uint32_t kKmTcABytes = kKmTcSteps * tc::kTileBytesA;   // one 128-row tile
constexpr int kKmTcList = 16;                                    // candidates per row
constexpr int kKmTcRows = 256;                                   // rows per unit (two warpgroups)
constexpr size_t kKmTcSmem = 2 * (size_t)kKmTcBlockBytes + 2 * (size_t)kKmTcABytes + kKmTcRows * kKmTcList * 8 + 1024;
constexpr float kKmTcPad = 0x1p64f;
constexpr float kKmTcHuge = 0x1p60f;

// Centroid block (p, b) of the filter into Bg: k-step s < 8 holds
// hi(-2 c[8s .. 8s+7]) of the 128 columns, step 8 holds (hi(fl(|c|^2)), 1);
// columns past k get the padding |c|^2 = 2^64. cmx[p] = max over the
// problem of |c|^2 rounded up (as f32 bits); bad[p] flags non-finite or
// huge centroids.
__global__ void __launch_bounds__(kKmTcCols)
km_tc_prep_kernel(Prob P, const uint2* __restrict__ blocks, const float* __restrict__ C,
                  unsigned char* __restrict__ Bg, uint32_t* __restrict__ cmx, uint32_t* __restrict__ bad) {
  const uint2 pb = blocks[blockIdx.x];
  const uint32_t p = pb.x, bk = pb.y;
  if (P.state[p] != kRunning) return;
  const uint32_t k = P.k[p], col = threadIdx.x, c = bk * kKmTcCols + col;
  const bool real = c < k;
  unsigned char* out = Bg + (size_t)blockIdx.x * kKmTcBlockBytes;
  float cn = 0.f, cn_up = 0.f;
  bool fin = true;
  const float* cv = C + (P.coff[p] + (real ? c : 0)) * kKmTcDim;
#pragma unroll
  for (int s = 0; s < kKmTcDim / 8; ++s) {
    float h[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float v = real ? cv[8 * s + q] : 0.f;
      cn = __fadd_rn(cn, __fmul_rn(v, v));
      cn_up = __fadd_ru(cn_up, __fmul_ru(v, v));
      fin = fin && isfinite(v);
      h[q] = __uint_as_float(__float_as_uint(__fmul_rn(-2.0f, v)) & 0xFFFFE000u);
    }
    unsigned char* t = out + (size_t)s * kKmTcStepB;
    *reinterpret_cast<float4*>(t + tc::operand_offset(col, 0)) = make_float4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<float4*>(t + tc::operand_offset(col, 4)) = make_float4(h[4], h[5], h[6], h[7]);
  }
  const bool ok = fin && cn_up <= kKmTcHuge;
  unsigned char* t = out + (size_t)(kKmTcSteps - 1) * kKmTcStepB;
  *reinterpret_cast<float4*>(t + tc::operand_offset(col, 0)) =
      (real && ok) ? make_float4(__uint_as_float(__float_as_uint(cn) & 0xFFFFE000u), 1.0f, 0.f, 0.f)
                   : make_float4(kKmTcPad, 0.f, 0.f, 0.f);
  *reinterpret_cast<float4*>(t + tc::operand_offset(col, 4)) = make_float4(0.f, 0.f, 0.f, 0.f);
  if (real) {
    if (!ok) atomicOr(&bad[p], 1u);
    else atomicMax(&cmx[p], __float_as_uint(cn_up));  // non-negative floats order as integers
  }
}

// Reference order for the full scan: best starts at dists[0] (kmeans.zig
// assignSlice), then the first strictly smaller distance.
__device__ __noinline__ void km_tc_full_scan(const float* __restrict__ xg, const float* __restrict__ C, uint64_t co,
                                             uint32_t k, float& best, uint32_t& bi) {
  float x[kKmTcDim];
#pragma unroll
  for (int q = 0; q < kKmTcDim; q += 4) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(xg + q));
    x[q] = v.x; x[q + 1] = v.y; x[q + 2] = v.z; x[q + 3] = v.w;
  }
  best = 0.f;
  bi = 0;
  for (uint32_t c = 0; c < k; ++c) {
    float cl[kKmTcDim];
#pragma unroll
    for (int q = 0; q < kKmTcDim; q += 4) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(C + (co + c) * kKmTcDim + q));
      cl[q] = v.x; cl[q + 1] = v.y; cl[q + 2] = v.z; cl[q + 3] = v.w;
    }
    const float f = l2_wide<kKmTcDim>(x, cl);
    if (c == 0) best = f;
    else if (f < best) { best = f; bi = c; }
  }
}

// Candidate list of one row: (column, key) pairs; a full list first drops
// the entries that the current (smaller) threshold has ruled out.
__device__ __forceinline__ void km_tc_push(uint2* l, int& nl, bool& ovf, uint32_t col, uint32_t key, uint32_t thr) {
  if (nl == kKmTcList) {
    int keep = 0;
    for (int e = 0; e < nl; ++e) {
      const uint2 en = l[e];
      if (en.y <= thr) l[keep++] = en;
    }
    nl = keep;
  }
  if (nl < kKmTcList) l[nl++] = make_uint2(col, key);
  else ovf = true;
}

// Units: up to 256 rows of one problem. Warps 0-3 and 4-7 (warpgroups 0 and
// 1) own rows 0-127 and 128-255 of the unit, one row per thread (= TMEM
// lane); warp 8 is the producer: it bulk-copies the centroid blocks (two
// buffers) and issues, per block, one MMA chain per warpgroup into that
// warpgroup's next accumulator slot (two 128-column slots each, so the chain
// of block b + 1 runs while block b is scanned).
__global__ void __launch_bounds__(288, 1)
km_tc_assign_kernel(const float* __restrict__ G, Prob P, const uint32_t* __restrict__ u_p,
                    const uint64_t* __restrict__ u_r0, const uint32_t* __restrict__ u_len, uint32_t nunits,
                    const uint32_t* __restrict__ bbase, const unsigned char* __restrict__ Bg,
                    const uint32_t* __restrict__ cmx, const uint32_t* __restrict__ bad,
                    const float* __restrict__ C, uint32_t* __restrict__ local, float* __restrict__ mind,
                    uint32_t* __restrict__ keys, uint32_t* __restrict__ diag) {
  extern __shared__ unsigned char km_raw[];
  unsigned char* base = km_raw + ((1024u - (tc::smem_addr(km_raw) & 1023u)) & 1023u);
  unsigned char* sB0 = base;                                  // [2][kKmTcBlockBytes]
  unsigned char* sA0 = base + 2 * kKmTcBlockBytes;            // [2 warpgroups][kKmTcABytes]
  uint2* lst = reinterpret_cast<uint2*>(sA0 + 2 * kKmTcABytes);  // [256][kKmTcList] (column, key)
  __shared__ __align__(8) uint64_t bfull[2], bfree[2], afull[2], accf[2][2], acce[2][2];
  __shared__ uint32_t tslot, s_abort;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (warp == 0) tc::tmem_alloc(&tslot, 2 * tc::kCols);
  if (tid == 0) {
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&bfull[b], 1);
      tc::mbar_init(&bfree[b], 1);
      tc::mbar_init(&afull[b], 128);
      for (int q = 0; q < 2; ++q) {
        tc::mbar_init(&accf[b][q], 1);
        tc::mbar_init(&acce[b][q], 128);
      }
    }
    s_abort = 0u;
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = tslot;
  auto aborted = [&]() { return *(volatile uint32_t*)&s_abort != 0u; };

  if (warp == 8) {
    // ============================ producer ===========================================
    if (lane == 0) {
      uint32_t gb = 0;          // blocks fetched by this CTA so far
      uint32_t bc[2] = {0, 0};  // blocks chained per warpgroup
      uint32_t ui = 0;          // units started
      bool ok = true;
      // fetch of the CTA's first block happens when its unit starts; the
      // next block's fetch is issued before the current block's chains
      for (uint32_t u = blockIdx.x; u < nunits && ok; u += gridDim.x) {
        const uint32_t p = u_p[u];
        if (P.state[p] != kRunning) continue;
        const uint32_t nb = (P.k[p] + kKmTcCols - 1) / kKmTcCols, b0 = bbase[p];
        for (int w = 0; w < 2 && ok; ++w) ok = tc::mbar_wait(&afull[w], ui & 1u);
        ++ui;
        if (!ok) break;
        for (uint32_t bk = 0; bk < nb && ok; ++bk, ++gb) {
          const int buf = (int)(gb & 1u);
          if (bk == 0) {  // the unit's first block (the previous unit fetched nothing ahead)
            if (gb >= 2) ok = tc::mbar_wait(&bfree[buf], ((gb >> 1) - 1u) & 1u);
            if (!ok) break;
            tc::bulk_load(sB0 + buf * kKmTcBlockBytes, Bg + (size_t)(b0 + bk) * kKmTcBlockBytes, kKmTcBlockBytes,
                          &bfull[buf]);
          }
          if (bk + 1 < nb) {  // prefetch the next block into the other buffer
            const uint32_t g1 = gb + 1;
            if (g1 >= 2) ok = tc::mbar_wait(&bfree[g1 & 1u], ((g1 >> 1) - 1u) & 1u);
            if (!ok) break;
            tc::bulk_load(sB0 + (g1 & 1u) * kKmTcBlockBytes, Bg + (size_t)(b0 + bk + 1) * kKmTcBlockBytes,
                          kKmTcBlockBytes, &bfull[g1 & 1u]);
          }
          ok = tc::mbar_wait(&bfull[buf], (gb >> 1) & 1u);
          if (!ok) break;
          for (int w = 0; w < 2 && ok; ++w) {
            const uint32_t slot = bc[w] & 1u;
            if (bc[w] >= 2) ok = tc::mbar_wait(&acce[w][slot], ((bc[w] >> 1) - 1u) & 1u);
            if (!ok) break;
            tc::fence_after_sync();
            const uint32_t d = tbase + (uint32_t)(w * 2 + (int)slot) * kKmTcCols;
            unsigned char* sa = sA0 + w * kKmTcABytes;
            unsigned char* sb = sB0 + buf * kKmTcBlockBytes;
#pragma unroll
            for (int s2 = 0; s2 < kKmTcSteps; ++s2)
              tc::mma_tf32(d, tc::operand_desc(sa + s2 * tc::kTileBytesA), tc::operand_desc(sb + s2 * kKmTcStepB),
                           s2 > 0 ? 1u : 0u, tc::kIdescTf32N128);
            tc::mma_commit(&accf[w][slot]);
            ++bc[w];
          }
          tc::mma_commit(&bfree[buf]);  // the buffer is free once both chains are done
        }
      }
      if (!ok) atomicExch(&s_abort, 1u);
    }
    __syncwarp();
  } else {
    // ============================ epilogue warpgroups ================================
    const int w = warp >> 2;                      // warpgroup
    const int r = (warp & 3) * 32 + lane;         // row within the warpgroup's tile = TMEM lane
    const int rr = w * 128 + r;                   // row within the unit
    unsigned char* sa = sA0 + w * kKmTcABytes;
    const uint32_t tlane = tbase + ((uint32_t)((warp & 3) * 32) << 16);
    uint32_t bcount = 0;  // blocks scanned by this warpgroup
    bool ok = true;
    for (uint32_t u = blockIdx.x; u < nunits && ok; u += gridDim.x) {
      const uint32_t p = u_p[u];
      if (P.state[p] != kRunning) continue;
      const uint32_t k = P.k[p];
      const uint64_t co = P.coff[p];
      const uint32_t nb = (k + kKmTcCols - 1) / kKmTcCols;
      const float cmax2 = __uint_as_float(cmx[p]);
      const bool pbad = bad[p] != 0u;
      const float cmax_up = __fsqrt_ru(cmax2), dl = __fmul_ru(0x1p-17f, cmax2);
      const uint64_t row = u_r0[u] + (uint64_t)rr;
      const bool valid = (uint32_t)rr < u_len[u];
      float x[kKmTcDim];
      {
        const float* xg = G + (valid ? row : u_r0[u]) * kKmTcDim;
#pragma unroll
        for (int q = 0; q < kKmTcDim; q += 4) {
          const float4 v = __ldg(reinterpret_cast<const float4*>(xg + q));
          x[q] = v.x; x[q + 1] = v.y; x[q + 2] = v.z; x[q + 3] = v.w;
        }
      }
      bool fin = true;
      float xn2_up = 0.f, xn2_dn = 0.f;
#pragma unroll
      for (int q = 0; q < kKmTcDim; ++q) {
        fin = fin && isfinite(x[q]);
        xn2_up = __fadd_ru(xn2_up, __fmul_ru(x[q], x[q]));
        xn2_dn = __fadd_rd(xn2_dn, __fmul_rd(x[q], x[q]));
      }
      const bool filt = valid && !pbad && fin && xn2_up <= kKmTcHuge;
      float t = 1.0f, E = 0.f;
      if (filt) {
        const float xn_up = __fsqrt_ru(xn2_up);
        const float eb = __fadd_ru(__fmul_ru(0x1p-7f, __fmul_ru(xn_up, cmax_up)), __fmul_ru(0x1p-9f, cmax2));
        const float t0 = __fadd_ru(__fmul_ru(__fadd_ru(__fadd_ru(xn2_up, dl), eb), 1.0f + 0x1p-12f), 0x1p-100f);
        t = tc::tf32_ceil_pos(t0);
        E = __fadd_ru(__fadd_ru(eb, __fmul_ru(0x1p-16f, t)), 0x1p-100f);
      }
      // operand A (the previous unit's chains, which read it, are complete:
      // this warpgroup has waited for every one of them)
#pragma unroll
      for (int s2 = 0; s2 < kKmTcDim / 8; ++s2) {
        float h[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) h[q] = filt ? __uint_as_float(__float_as_uint(x[8 * s2 + q]) & 0xFFFFE000u) : 0.f;
        unsigned char* ta = sa + s2 * tc::kTileBytesA;
        *reinterpret_cast<float4*>(ta + tc::operand_offset(r, 0)) = make_float4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<float4*>(ta + tc::operand_offset(r, 4)) = make_float4(h[4], h[5], h[6], h[7]);
      }
      {
        unsigned char* ta = sa + (kKmTcSteps - 1) * tc::kTileBytesA;
        *reinterpret_cast<float4*>(ta + tc::operand_offset(r, 0)) = make_float4(1.0f, t, 0.f, 0.f);
        *reinterpret_cast<float4*>(ta + tc::operand_offset(r, 4)) = make_float4(0.f, 0.f, 0.f, 0.f);
      }
      tc::fence_async_smem();
      tc::mbar_arrive(&afull[w]);

      uint32_t m1 = 0xFFFFFFFFu, m2 = 0xFFFFFFFFu;  // running smallest keys (value | in-block column)
      uint32_t m1b = 0;                             // block of m1
      int nl = 0;
      bool ovf = false;
      uint2* mylst = lst + rr * kKmTcList;
      for (uint32_t bk = 0; bk < nb; ++bk, ++bcount) {
        const uint32_t slot = bcount & 1u;
        const bool got = tc::mbar_wait(&accf[w][slot], (bcount >> 1) & 1u);
        if (!__all_sync(0xFFFFFFFFu, got) || __any_sync(0xFFFFFFFFu, aborted())) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
        const uint32_t taddr = tlane + (uint32_t)(w * 2 + (int)slot) * kKmTcCols;
        uint32_t q1 = 0xFFFFFFFFu, q2 = 0xFFFFFFFFu;
#pragma unroll 1
        for (int q = 0; q < 2; ++q) {
          uint32_t v[64];
          tc::tmem_ld64(taddr + (uint32_t)(q * 64), v);
          tc::tmem_wait_ld();
          float f1a = __int_as_float(0x7f800000), f2a = f1a, f1b = f1a, f2b = f1a;
#pragma unroll
          for (int jj = 0; jj < 64; jj += 4) {
            const float k0 = __uint_as_float((v[jj] & 0xFFFFFF00u) | (uint32_t)jj);
            const float k1 = __uint_as_float((v[jj + 1] & 0xFFFFFF00u) | (uint32_t)(jj + 1));
            const float k2 = __uint_as_float((v[jj + 2] & 0xFFFFFF00u) | (uint32_t)(jj + 2));
            const float k3 = __uint_as_float((v[jj + 3] & 0xFFFFFF00u) | (uint32_t)(jj + 3));
            const float loa = fminf(k0, k1), hia = fmaxf(k0, k1);
            f2a = tc::min3f(f2a, hia, fmaxf(f1a, loa));
            f1a = fminf(f1a, loa);
            const float lob = fminf(k2, k3), hib = fmaxf(k2, k3);
            f2b = tc::min3f(f2b, hib, fmaxf(f1b, lob));
            f1b = fminf(f1b, lob);
          }
          const uint32_t qb = (uint32_t)q << 6;
          const uint32_t a1 = __float_as_uint(fminf(f1a, f1b)) | qb;
          const uint32_t a2 = __float_as_uint(fminf(fmaxf(f1a, f1b), fminf(f2a, f2b))) | qb;
          const uint32_t n2 = min(max(q1, a1), min(q2, a2));
          q1 = min(q1, a1);
          q2 = n2;
        }
        if (q1 < m1) {  // a tie keeps the earlier block
          m2 = min(m1, q2);
          m1 = q1;
          m1b = bk;
        } else {
          m2 = min(m2, q1);
        }
        uint32_t thrkey = 0u;
        bool need2 = false;
        if (filt) {
          const float a1hi = __uint_as_float(m1 | 0xFFu);
          const float dup = fmaxf(__fadd_ru(__fadd_ru(__fsub_ru(__fadd_ru(a1hi, E), t), xn2_up), dl), 0.f);
          const float T = __fadd_ru(__fadd_ru(__fadd_ru(a1hi, __fmul_ru(2.0f, E)), __fmul_ru(0x1p-17f, dup)),
                                    __fmul_ru(2.0f, dl));
          thrkey = __float_as_uint(T) | 0xFFu;
          if (q1 <= thrkey) {
            if (q2 <= thrkey) need2 = true;
            else km_tc_push(mylst, nl, ovf, bk * kKmTcCols + (q1 & 0xFFu), q1, thrkey);
          }
        }
        if (__any_sync(0xFFFFFFFFu, need2)) {  // several columns of this block at or below T
#pragma unroll 1
          for (int q = 0; q < 2; ++q) {
            uint32_t v[64];
            tc::tmem_ld64(taddr + (uint32_t)(q * 64), v);
            tc::tmem_wait_ld();
            if (need2) {
              uint32_t lo = 0u, hi = 0u;
#pragma unroll
              for (int jj = 0; jj < 32; ++jj) {
                lo |= (v[jj] <= thrkey ? 1u : 0u) << jj;
                hi |= (v[jj + 32] <= thrkey ? 1u : 0u) << jj;
              }
              unsigned long long bits = ((unsigned long long)hi << 32) | lo;
              while (bits) {  // in column order
                const int jj = __ffsll((long long)bits) - 1;
                bits &= bits - 1;
                const uint32_t col = (uint32_t)(q * 64 + jj);
                km_tc_push(mylst, nl, ovf, bk * kKmTcCols + col, (v[jj] & 0xFFFFFF00u) | col, thrkey);
              }
            }
          }
        }
        tc::fence_before_sync();
        tc::mbar_arrive(&acce[w][slot]);  // the slot may take the next chain
      }
      if (!ok) break;
      // ---- the exact distances decide -------------------------------------------
      uint32_t final_thr = 0xFFFFFFFFu;
      if (filt) {
        const float a1hi = __uint_as_float(m1 | 0xFFu);
        const float dup = fmaxf(__fadd_ru(__fadd_ru(__fsub_ru(__fadd_ru(a1hi, E), t), xn2_up), dl), 0.f);
        const float T = __fadd_ru(__fadd_ru(__fadd_ru(a1hi, __fmul_ru(2.0f, E)), __fmul_ru(0x1p-17f, dup)),
                                  __fmul_ru(2.0f, dl));
        final_thr = __float_as_uint(T) | 0xFFu;
      }
      int nfin = 0;
      for (int e = 0; e < nl; ++e) nfin += mylst[e].y <= final_thr ? 1 : 0;
      if (valid) {
        uint32_t bi = 0;
        float best = 0.f;
        if (!filt || ovf || nl == 0) {
          km_tc_full_scan(G + row * kKmTcDim, C, co, k, best, bi);
        } else {
          best = __int_as_float(0x7f800000);
          for (int e = 0; e < nl; ++e) {
            const uint2 en = mylst[e];
            if (en.y > final_thr) continue;  // ruled out by the final threshold
            const uint32_t c = en.x;
            float cl[kKmTcDim];
#pragma unroll
            for (int q = 0; q < kKmTcDim; q += 4) {
              const float4 v = __ldg(reinterpret_cast<const float4*>(C + (co + c) * kKmTcDim + q));
              cl[q] = v.x; cl[q + 1] = v.y; cl[q + 2] = v.z; cl[q + 3] = v.w;
            }
            const float f = l2_wide<kKmTcDim>(x, cl);
            if (f < best) {
              best = f;
              bi = c;
            }
          }
          if (nfin == 1 && bi == m1b * kKmTcCols + (m1 & 0xFFu)) {  // canary on the single winner
            const float a1lo = __uint_as_float(m1 & 0xFFFFFF00u), a1hi = __uint_as_float(m1 | 0xFFu);
            const float phi =
                __fadd_ru(__fadd_ru(__fadd_ru(__fsub_ru(t, xn2_dn), __fmul_ru(best, 1.0f + 0x1p-18f)), dl), E);
            const float plo =
                __fsub_rd(__fsub_rd(__fadd_rd(__fsub_rd(t, xn2_up), __fmul_rd(best, 1.0f - 0x1p-18f)), dl), E);
            if (a1lo > phi || a1hi < plo) atomicAdd(&diag[0], 1u);
          }
        }
        local[row] = bi;
        mind[row] = best;
        keys[row] = (uint32_t)(co + bi);
      }
      const uint32_t mm = __ballot_sync(0xFFFFFFFFu, valid && filt && nfin > 1);
      if (mm && lane == 0) atomicAdd(&diag[1], (uint32_t)__popc(mm));
      const uint32_t mo = __ballot_sync(0xFFFFFFFFu, valid && filt && ovf);
      if (mo && lane == 0) atomicAdd(&diag[3], (uint32_t)__popc(mo));
    }
    if (!ok && lane == 0) atomicExch(&s_abort, 1u);
  }
  __syncthreads();
  if (tid == 0 && s_abort) atomicExch(&diag[2], 1u);
  tc::fence_after_sync();
  if (warp == 0) tc::tmem_free(tbase, 2 * tc::kCols);
}

// Cluster sizes from the sort keys of all rows (rows of finished problems
// keep their last keys), so counts and the radix order always agree.
__global__ void km_count_kernel(const uint32_t* __restrict__ keys, uint64_t n, uint32_t* __restrict__ counts) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    atomicAdd(&counts[keys[i]], 1u);
}

// Sequential f32 WCSS per problem (kmeans.zig:179): one warp per problem.
// The warp double-buffers 1024-value tiles of min_to_any in shared memory
// with cp.async while lane 0 adds the current tile in row order, so the
// dependent-add chain is the only serial part.
__global__ void __launch_bounds__(128)
km_wcss_kernel(Prob P, uint32_t nprob, const float* __restrict__ mind) {
  __shared__ __align__(16) float tile[4][2][1024];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t p = blockIdx.x * 4 + warp;
  if (p >= nprob || P.state[p] != kRunning || P.n[p] >= kWcssSeg) return;  // long ones: km_wcss_seg_kernel
  const float* src = mind + P.off[p];
  const uint32_t n = P.n[p];
  float acc = 0.f;
  for (uint32_t e = lane; e < min(1024u, n); e += 32) cp_async<4>(&tile[warp][0][e], src + e);
  cp_async_commit();
  int buf = 0;
  for (uint32_t t0 = 0; t0 < n; t0 += 1024) {
    const uint32_t m = min(1024u, n - t0);
    cp_async_wait<0>();
    __syncwarp();
    const uint32_t t1 = t0 + 1024;
    if (t1 < n) {
      const uint32_t m1 = min(1024u, n - t1);
      for (uint32_t e = lane; e < m1; e += 32) cp_async<4>(&tile[warp][buf ^ 1][e], src + t1 + e);
    }
    cp_async_commit();
    if (lane == 0) {
      const float4* t4 = reinterpret_cast<const float4*>(tile[warp][buf]);
      const uint32_t m4 = m >> 2;
#pragma unroll 8
      for (uint32_t e = 0; e < m4; ++e) {
        const float4 v = t4[e];
        acc = __fadd_rn(acc, v.x);
        acc = __fadd_rn(acc, v.y);
        acc = __fadd_rn(acc, v.z);
        acc = __fadd_rn(acc, v.w);
      }
      for (uint32_t e = m4 * 4; e < m; ++e) acc = __fadd_rn(acc, tile[warp][buf][e]);
    }
    __syncwarp();
    buf ^= 1;
  }
  cp_async_wait<0>();
  if (lane == 0) P.wcss[p] = acc;
}

// Sequential f32 WCSS of one long problem without the serial chain. For
// non-negative addends the running sum s stays on one grid of spacing
// u = 2^(max(e, -126) - 23) while it is inside its binade [2^e, 2^(e+1))
// (zero and subnormal sums use u = 2^-149, which also covers the first
// normal binade), and there fl(K*u + x) = (K + rne(x/u))*u with K = s/u an
// integer: the rounding of an addend is independent of K except at exact
// ties (x/u = m + 1/2), where round-half-even makes the new K even. So a tie
// rounds up exactly when the sum of the grid values since the previous tie
// (its own floor included) is odd; for the first tie of a chunk the chunk's
// starting K counts too. A CTA takes 8192 addends at a time: grid values, a
// block prefix sum, each tie's decision from the prefix at the previous tie,
// the prefix of the round-ups, and the first position where K + prefix
// reaches 2^24 (the sum enters the next binade); that one addend is added
// with an f32 add and the grid is recomputed. A problem with a non-finite
// value is added serially by one thread. The result is the reference's
// left-to-right f32 sum, bit for bit.
constexpr int kSegT = 1024, kSegV = 8, kSegChunk = kSegT * kSegV;

// Block-wide exclusive prefix sum of one int64 per thread (1024 threads);
// also returns the total. `sw` holds 33 int64 (warp totals, then their
// exclusive prefixes and the total, written by warp 0).
__device__ __forceinline__ long long seg_scan_excl(long long v, long long* sw, long long& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  long long inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const long long t = __shfl_up_sync(0xFFFFFFFFu, inc, o);
    if (lane >= o) inc += t;
  }
  __syncthreads();
  if (lane == 31) sw[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    const long long w = sw[lane];
    long long wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const long long t = __shfl_up_sync(0xFFFFFFFFu, wi, o);
      if (lane >= o) wi += t;
    }
    sw[lane] = wi - w;
    if (lane == 31) sw[32] = wi;
  }
  __syncthreads();
  total = sw[32];
  return sw[warp] + inc - v;
}

// Block-wide "latest value" carry: for each thread the value of the last
// thread before it with has = true (or `init` when none). `sw` holds 32
// int64 and `sh` 32 int.
__device__ __forceinline__ long long seg_carry_excl(bool has, long long v, long long init, long long* sw, int* sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  bool h = has;
  long long val = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const long long tv = __shfl_up_sync(0xFFFFFFFFu, val, o);
    const bool th = __shfl_up_sync(0xFFFFFFFFu, h, o);
    if (lane >= o && !h) {
      h = th;
      val = tv;
    }
  }
  long long ev = __shfl_up_sync(0xFFFFFFFFu, val, 1);  // exclusive within the warp
  bool eh = __shfl_up_sync(0xFFFFFFFFu, h, 1);
  if (lane == 0) eh = false;
  __syncthreads();
  if (lane == 31) {
    sw[warp] = val;
    sh[warp] = h ? 1 : 0;
  }
  __syncthreads();
  if (warp == 0) {  // exclusive carry over the warps
    bool wh = sh[lane] != 0;
    long long wv = sw[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const long long tv = __shfl_up_sync(0xFFFFFFFFu, wv, o);
      const bool th = __shfl_up_sync(0xFFFFFFFFu, wh, o);
      if (lane >= o && !wh) {
        wh = th;
        wv = tv;
      }
    }
    long long xv = __shfl_up_sync(0xFFFFFFFFu, wv, 1);
    bool xh = __shfl_up_sync(0xFFFFFFFFu, wh, 1);
    if (lane == 0) xh = false;
    __syncwarp();
    sw[lane] = xh ? xv : init;
  }
  __syncthreads();
  return eh ? ev : sw[warp];
}

__global__ void __launch_bounds__(kSegT)
km_wcss_seg_kernel(Prob P, const float* __restrict__ mind) {
  const uint32_t p = blockIdx.x;
  if (P.state[p] != kRunning || P.n[p] < kWcssSeg) return;
  const float* x = mind + P.off[p];
  const uint32_t n = P.n[p];
  __shared__ float s_s;
  __shared__ uint32_t s_i, s_cross;
  __shared__ long long sw[kSegT / 32 + 1];
  __shared__ int sh[kSegT / 32];
  const int tid = threadIdx.x;
  bool bad = false;
  for (uint32_t j = tid; j < n; j += kSegT) bad = bad || !isfinite(x[j]);
  if (__syncthreads_or(bad)) {
    if (tid == 0) {
      float a = 0.f;
      for (uint32_t j = 0; j < n; ++j) a = __fadd_rn(a, x[j]);
      P.wcss[p] = a;
    }
    return;
  }
  if (tid == 0) {  // the first addends serially: the sum changes binade often early on
    float a = 0.f;
    const uint32_t h = min(n, 2048u);
    for (uint32_t j = 0; j < h; ++j) a = __fadd_rn(a, x[j]);
    s_s = a;
    s_i = h;
  }
  __syncthreads();
  for (;;) {
    const uint32_t i = s_i;
    const float s = s_s;
    __syncthreads();  // everyone has read the state
    if (i >= n || !isfinite(s)) break;
    const uint32_t eb = (__float_as_uint(s) >> 23) & 0xFFu;
    const int ue = (eb == 0u ? -126 : (int)eb - 127) - 23;  // grid spacing 2^ue
    const long long K = (long long)ldexp((double)s, -ue);   // exact, < 2^24
    const uint32_t C = min((uint32_t)kSegChunk, n - i);
    long long val[kSegV];
    bool tie[kSegV];
    long long mine = 0;
#pragma unroll
    for (int v = 0; v < kSegV; ++v) {
      const uint32_t j = (uint32_t)(kSegV * tid + v);
      val[v] = 0;
      tie[v] = false;
      if (j < C) {
        const double y = ldexp((double)x[i + j], -ue);  // exact
        if (y >= 0x1p40) {
          val[v] = 1ll << 40;  // crosses the binade by itself
        } else {
          const double fl = floor(y), f = y - fl;
          tie[v] = f == 0.5;
          val[v] = (long long)fl + (f > 0.5 ? 1 : 0);
        }
        mine += val[v];
      }
    }
    long long total0 = 0;
    const long long base0 = seg_scan_excl(mine, sw, total0);
    // prefix P0 at each addend; the last tie's P0 inside this thread
    long long p0[kSegV];
    bool has = false;
    long long lastp = 0;
    {
      long long run = base0;
#pragma unroll
      for (int v = 0; v < kSegV; ++v) {
        run += val[v];
        p0[v] = run;
        if (tie[v]) {
          has = true;
          lastp = run;
        }
      }
    }
    const long long prev_in = seg_carry_excl(has, lastp, -K, sw, sh);
    // round-ups at ties: the sum since the previous tie is odd
    int ups = 0;
    bool up[kSegV];
    {
      long long prev = prev_in;
#pragma unroll
      for (int v = 0; v < kSegV; ++v) {
        up[v] = tie[v] && (((p0[v] - prev) & 1ll) != 0);
        if (tie[v]) prev = p0[v];
        ups += up[v] ? 1 : 0;
      }
    }
    long long tot_up = 0;
    const long long ubase = seg_scan_excl((long long)ups, sw, tot_up);
    if (tid == 0) s_cross = 0xFFFFFFFFu;
    __syncthreads();
    // first addend at which the sum reaches the next binade
    int cv = -1;
    long long before_c = 0;
    {
      long long u = ubase;
#pragma unroll
      for (int v = 0; v < kSegV; ++v) {
        const uint32_t j = (uint32_t)(kSegV * tid + v);
        u += up[v] ? 1 : 0;
        if (cv < 0 && j < C && K + p0[v] + u >= (1ll << 24)) {
          cv = v;
          before_c = K + (p0[v] - val[v]) + (u - (up[v] ? 1 : 0));
        }
      }
    }
    if (cv >= 0) atomicMin(&s_cross, (uint32_t)(kSegV * tid + cv));
    __syncthreads();
    const uint32_t cj = s_cross;
    if (cj == 0xFFFFFFFFu) {
      if (tid == 0) {
        s_s = (float)ldexp((double)(K + total0 + tot_up), ue);
        s_i = i + C;
      }
    } else if (cv >= 0 && (uint32_t)(kSegV * tid + cv) == cj) {
      // the sum leaves its binade at addend cj: that one add in f32
      s_s = __fadd_rn((float)ldexp((double)before_c, ue), x[i + cj]);
      s_i = i + cj + 1;
    }
    __syncthreads();
  }
  if (tid == 0) P.wcss[p] = s_s;
}

// Exclusive scan of n u32 in three launches: per-tile sums (tiles of
// kScanTile), one CTA scanning the tile sums, per-tile scans plus offsets.
constexpr int kScanT = 512;
constexpr int kScanV = 8;
constexpr int kScanTile = kScanT * kScanV;

__device__ __forceinline__ uint32_t warp_incl_scan_u32(uint32_t x, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  return x;
}

__global__ void __launch_bounds__(kScanT)
km_scan_reduce_kernel(const uint32_t* __restrict__ in, uint64_t n, uint32_t* __restrict__ part) {
  __shared__ uint32_t ws[kScanT / 32];
  const uint64_t base = (uint64_t)blockIdx.x * kScanTile;
  uint32_t s = 0;
#pragma unroll
  for (int u = 0; u < kScanV; ++u) {
    const uint64_t e = base + (uint64_t)u * kScanT + threadIdx.x;
    if (e < n) s += in[e];
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  s = __reduce_add_sync(0xffffffffu, s);
  if (lane == 0) ws[warp] = s;
  __syncthreads();
  if (warp == 0) {
    uint32_t v = lane < kScanT / 32 ? ws[lane] : 0u;
    v = __reduce_add_sync(0xffffffffu, v);
    if (lane == 0) part[blockIdx.x] = v;
  }
}

__global__ void __launch_bounds__(1024)
km_scan_partials_kernel(uint32_t* __restrict__ part, uint32_t np) {
  __shared__ uint32_t ws[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t carry = 0;
  for (uint32_t t0 = 0; t0 < np; t0 += 1024) {
    const uint32_t e = t0 + threadIdx.x;
    const uint32_t v = e < np ? part[e] : 0u;
    const uint32_t x = warp_incl_scan_u32(v, lane);
    if (lane == 31) ws[warp] = x;
    __syncthreads();
    if (warp == 0) ws[lane] = warp_incl_scan_u32(ws[lane], lane);
    __syncthreads();
    const uint32_t incl = x + (warp > 0 ? ws[warp - 1] : 0u);
    if (e < np) part[e] = carry + incl - v;
    carry += ws[31];
    __syncthreads();
  }
}

__global__ void __launch_bounds__(kScanT)
km_scan_apply_kernel(const uint32_t* __restrict__ in, uint64_t n, const uint32_t* __restrict__ part,
                     uint32_t* __restrict__ out) {
  __shared__ uint32_t ws[kScanT / 32];
  const uint64_t base = (uint64_t)blockIdx.x * kScanTile + (uint64_t)threadIdx.x * kScanV;
  uint32_t v[kScanV];
  uint32_t s = 0;
#pragma unroll
  for (int u = 0; u < kScanV; ++u) {
    v[u] = base + u < n ? in[base + u] : 0u;
    s += v[u];
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t x = warp_incl_scan_u32(s, lane);
  if (lane == 31) ws[warp] = x;
  __syncthreads();
  if (warp == 0) {
    const uint32_t w = lane < kScanT / 32 ? ws[lane] : 0u;
    const uint32_t wi = warp_incl_scan_u32(w, lane);
    __syncwarp();
    if (lane < kScanT / 32) ws[lane] = wi;
  }
  __syncthreads();
  uint32_t run = part[blockIdx.x] + (x - s) + (warp > 0 ? ws[warp - 1] : 0u);
#pragma unroll
  for (int u = 0; u < kScanV; ++u) {
    if (base + u < n) out[base + u] = run;
    run += v[u];
  }
}

// Stable LSD radix pass (8-bit digit at `shift`) over (key, val) pairs.
// Block b (one warp) owns rows [b*kRadixRows, ...). vals == nullptr means
// val = row index (the first pass).
__global__ void __launch_bounds__(kRadixWarps * 32)
km_radix_hist_kernel(const uint32_t* __restrict__ keys, uint64_t n, int shift, int nblk,
                     uint32_t* __restrict__ hist) {
  __shared__ uint32_t h[kRadixWarps][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x * kRadixWarps + warp;
  for (int e = lane; e < 256; e += 32) h[warp][e] = 0;
  __syncwarp();
  if (b < nblk) {
    const uint64_t lo = (uint64_t)b * kRadixRows, hi = min(n, lo + kRadixRows);
    for (uint64_t i = lo + lane; i < hi; i += 32) atomicAdd(&h[warp][(keys[i] >> shift) & 255u], 1u);
    __syncwarp();
    for (int e = lane; e < 256; e += 32) hist[(size_t)e * nblk + b] = h[warp][e];
  }
}

__global__ void __launch_bounds__(kRadixWarps * 32)
km_radix_scatter_kernel(const uint32_t* __restrict__ keys, const uint32_t* __restrict__ vals,
                        uint64_t n, int shift, int nblk, const uint32_t* __restrict__ base,
                        uint32_t* __restrict__ keys_out, uint32_t* __restrict__ vals_out) {
  __shared__ uint32_t run_all[kRadixWarps][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x * kRadixWarps + warp;
  if (b >= nblk) return;
  uint32_t* run = run_all[warp];
  for (int e = lane; e < 256; e += 32) run[e] = base[(size_t)e * nblk + b];
  __syncwarp();
  const uint64_t lo = (uint64_t)b * kRadixRows, hi = min(n, lo + kRadixRows);
  for (uint64_t i0 = lo; i0 < hi; i0 += 32) {
    const uint64_t i = i0 + lane;
    const bool ok = i < hi;
    const uint32_t key = ok ? keys[i] : 0u, val = ok ? (vals ? vals[i] : (uint32_t)i) : 0u;
    const int dig = ok ? (int)((key >> shift) & 255u) : 256 + lane;
    const uint32_t peers = __match_any_sync(0xffffffffu, dig);
    const uint32_t rank = __popc(peers & lanemask_lt());
    uint32_t dst = 0;
    if (ok) dst = run[dig] + rank;
    __syncwarp();
    if (ok && rank == 0) run[dig] += __popc(peers);
    __syncwarp();
    if (ok) {
      keys_out[dst] = key;
      vals_out[dst] = val;
    }
  }
}

// In-order centroid sums: one warp per global cluster, lane = coordinates
// lane, lane+32, ...; members are the cluster's rows in row order.
template <int DIM>
__global__ void __launch_bounds__(256)
km_chain_kernel(const float* __restrict__ G, int d_rt, Prob P, const uint32_t* __restrict__ cprob,
                uint64_t KT, const uint32_t* __restrict__ counts, const uint32_t* __restrict__ starts,
                const uint32_t* __restrict__ vals, float* __restrict__ C) {
  constexpr int Q = DIM > 0 ? (DIM + 31) / 32 : 8;  // coordinates per lane (generic: d <= 256)
  const int d = DIM > 0 ? DIM : d_rt;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint64_t g = (uint64_t)blockIdx.x * 8 + warp;
  if (g >= KT) return;
  if (P.state[cprob[g]] != kRunning) return;
  const uint32_t cnt = counts[g];
  if (cnt == 0) return;  // left for the reseed
  const uint32_t st = starts[g];
  float acc[Q];
#pragma unroll
  for (int q = 0; q < Q; ++q) acc[q] = 0.f;
  for (uint32_t b0 = 0; b0 < cnt; b0 += 32) {
    const uint32_t m = min(32u, cnt - b0);
    const uint32_t myrow = lane < (int)m ? vals[st + b0 + lane] : 0u;
    for (uint32_t e = 0; e < m; ++e) {
      const uint64_t row = __shfl_sync(0xffffffffu, myrow, e);
      const float* x = G + row * d;
#pragma unroll
      for (int q = 0; q < Q; ++q) {
        const int j = lane + 32 * q;
        if (j < d) acc[q] = __fadd_rn(acc[q], __ldg(x + j));
      }
    }
  }
  const float inv = __fdiv_rn(1.0f, __uint2float_rn(cnt));
#pragma unroll
  for (int q = 0; q < Q; ++q) {
    const int j = lane + 32 * q;
    if (j < d) C[g * d + j] = __fmul_rn(acc[q], inv);
  }
}

// First maximum of v[0..n) with vec.argmax semantics.
__device__ uint64_t block_argmax_first(const float* v, uint64_t n) {
  __shared__ float bv[32];
  __shared__ uint64_t bi[32];
  float best = -__int_as_float(0x7f800000);
  uint64_t idx = n;
  for (uint64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const float x = v[i];
    if (x > best || (x == best && i < idx)) { best = x; idx = i; }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const uint64_t oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ob > best || (ob == best && oi < idx)) { best = ob; idx = oi; }
  }
  if (lane == 0) { bv[warp] = best; bi[warp] = idx; }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? bv[lane] : -__int_as_float(0x7f800000);
    idx = lane < nw ? bi[lane] : n;
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const uint64_t oi = __shfl_xor_sync(0xffffffffu, idx, o);
      if (ob > best || (ob == best && oi < idx)) { best = ob; idx = oi; }
    }
    if (lane == 0) bi[0] = (isnan(v[0]) || idx >= n) ? 0 : idx;
  }
  __syncthreads();
  const uint64_t r = bi[0];
  __syncthreads();
  return r;
}

// Empty-cluster reseed in cluster order, then the convergence test.
__global__ void __launch_bounds__(256)
km_reseed_converge_kernel(const float* __restrict__ G, int d, Prob P, uint32_t nprob,
                          const uint32_t* __restrict__ counts, float* __restrict__ mind,
                          float* __restrict__ C, uint32_t* __restrict__ reseeds, int iter, int check,
                          float tol) {
  const uint32_t p = blockIdx.x;
  if (p >= nprob || P.state[p] != kRunning) return;
  const uint32_t k = P.k[p];
  const uint64_t co = P.coff[p], off = P.off[p];
  const uint32_t n = P.n[p];
  __shared__ int any_empty;
  if (threadIdx.x == 0) any_empty = 0;
  __syncthreads();
  for (uint32_t c = threadIdx.x; c < k; c += blockDim.x)
    if (counts[co + c] == 0) any_empty = 1;
  __syncthreads();
  if (any_empty) {
    float* mm = mind + off;
    for (uint32_t c = 0; c < k; ++c) {
      if (counts[co + c] != 0) continue;
      const uint64_t far = block_argmax_first(mm, n);
      for (int j = threadIdx.x; j < d; j += blockDim.x) C[(co + c) * d + j] = G[(off + far) * d + j];
      __syncthreads();
      if (threadIdx.x == 0) {
        mm[far] = -__int_as_float(0x7f800000);
        reseeds[p] += 1;
      }
      __syncthreads();
    }
  }
  if (threadIdx.x == 0) {
    P.iters[p] = (uint32_t)iter + 1;
    if (check) {
      const float w = P.wcss[p];
      if (iter > 0) {
        const float prev = P.prev[p];
        const float denom = prev > 0.f ? prev : 1.0f;
        if (__fdiv_rn(__fsub_rn(prev, w), denom) < tol) P.state[p] = kDone;
      }
      P.prev[p] = w;
    }
  }
}

struct Carver {
  size_t off = 0;
  size_t take(size_t bytes) {
    const size_t o = off;
    off = (off + bytes + 255) & ~(size_t)255;
    return o;
  }
};

template <typename T>
T* at(unsigned char* base, size_t o) { return reinterpret_cast<T*>(base + o); }

}  // namespace

int km_gather_groups(Ctx* ctx, const float* d_V, const uint32_t* d_idx, uint64_t n, uint32_t dim, float* d_G,
                     float* d_GT) {
  if (n == 0) return MVR_OK;
  const int ng4 = (int)((dim + 3) / 4);
  const int stride = 4 * ng4 + ((4 - 4 * ng4) % 32 + 32) % 32;  // 4 mod 32 words
  const size_t smem = (size_t)32 * stride * sizeof(float);
  km_gather_groups_kernel<<<(unsigned)((n + 31) / 32), 256, smem, ctx->stream>>>(
      d_V, d_idx, n, (int)dim, stride, d_G, reinterpret_cast<float4*>(d_GT));
  MVR_CUDA(ctx, cudaGetLastError());
  return MVR_OK;
}

namespace {
// Exclusive scan of n u32 (n >= 1); `part` holds ceil(n / kScanTile) u32.
int scan_u32(Ctx* ctx, cudaStream_t st, const uint32_t* in, uint64_t n, uint32_t* part, uint32_t* out) {
  const unsigned nt = (unsigned)((n + kScanTile - 1) / kScanTile);
  km_scan_reduce_kernel<<<nt, kScanT, 0, st>>>(in, n, part);
  km_scan_partials_kernel<<<1, 1024, 0, st>>>(part, nt);
  km_scan_apply_kernel<<<nt, kScanT, 0, st>>>(in, n, part, out);
  MVR_CUDA(ctx, cudaGetLastError());
  return MVR_OK;
}
}  // namespace

size_t scan_part_words(uint64_t n) { return (size_t)(n / kScanTile + 2); }

int exclusive_scan_u32(Ctx* ctx, cudaStream_t st, const uint32_t* in, uint64_t n, uint32_t* part, uint32_t* out) {
  if (n == 0) return MVR_OK;
  return scan_u32(ctx, st, in, n, part, out);
}

size_t radix_pairs_scratch_words(uint64_t n) {
  const uint64_t nblk = (n + kRadixRows - 1) / kRadixRows;
  return (size_t)(2 * 256 * nblk) + scan_part_words(256 * nblk);
}

int radix_sort_pairs(Ctx* ctx, cudaStream_t st, const uint32_t* keys, const uint32_t* vals, uint64_t n, int key_bits,
                     uint32_t* k0, uint32_t* v0, uint32_t* k1, uint32_t* v1, uint32_t* scratch,
                     const uint32_t** keys_out, const uint32_t** vals_out) {
  *keys_out = keys;
  *vals_out = vals;
  if (n == 0) return MVR_OK;
  const int nblk = (int)((n + kRadixRows - 1) / kRadixRows);
  uint32_t* hist = scratch;
  uint32_t* base = scratch + (size_t)256 * nblk;
  uint32_t* part = base + (size_t)256 * nblk;
  const uint32_t* ki = keys;
  const uint32_t* vi = vals;
  uint32_t *ko = k0, *vo = v0;
  const int passes = std::max(1, (key_bits + 7) / 8);
  for (int pass = 0; pass < passes; ++pass) {
    const int shift = 8 * pass;
    const unsigned g = (unsigned)((nblk + kRadixWarps - 1) / kRadixWarps);
    km_radix_hist_kernel<<<g, kRadixWarps * 32, 0, st>>>(ki, n, shift, nblk, hist);
    MVR_TRY(scan_u32(ctx, st, hist, (uint64_t)256 * nblk, part, base));
    km_radix_scatter_kernel<<<g, kRadixWarps * 32, 0, st>>>(ki, vi, n, shift, nblk, base, ko, vo);
    MVR_CUDA(ctx, cudaGetLastError());
    ki = ko;
    vi = vo;
    ko = ko == k0 ? k1 : k0;
    vo = vo == v0 ? v1 : v0;
  }
  *keys_out = ki;
  *vals_out = vi;
  return MVR_OK;
}

int km_batch_run(Ctx* ctx, const float* d_G, const float* d_GT, uint64_t rows, uint32_t dim, const KmBatch& b,
                 uint32_t max_iters, float tol, float* d_C, uint32_t* d_local, KmResult* res) {
  const size_t NP = b.size();
  res->status.assign(NP, MVR_OK);
  res->wcss.assign(NP, 0.f);
  res->iters.assign(NP, 0);
  if (NP == 0) return MVR_OK;
  if (dim == 0) return fail(ctx, MVR_E_DIM_MISMATCH, "dim == 0");
  if (dim > 256) return fail(ctx, MVR_E_INVALID_ARGUMENT, "dim > 256 is not supported on the GPU path");
  if (rows >= (1ull << 32)) return fail(ctx, MVR_E_INVALID_ARGUMENT, "more than 2^32-1 rows");
  cudaStream_t st = ctx->stream;
  const uint64_t KT = b.coff.back() + b.k.back();
  if (KT >= (1ull << 32)) return fail(ctx, MVR_E_INVALID_ARGUMENT, "more than 2^32-1 centroids");

  // ---- problem classes ---------------------------------------------------
  std::vector<uint32_t> degen, live, seeders;
  for (uint32_t p = 0; p < NP; ++p) {
    if (b.k[p] == 0 || b.n[p] == 0) return fail(ctx, MVR_E_INVALID_ARGUMENT, "empty problem");
    if (b.k[p] >= b.n[p]) {
      degen.push_back(p);
    } else {
      live.push_back(p);
      if (b.k[p] >= 2) seeders.push_back(p);
    }
  }
  std::stable_sort(seeders.begin(), seeders.end(), [&](uint32_t a, uint32_t c) { return b.k[a] > b.k[c]; });
  uint32_t kmax = 0;
  for (uint32_t p : seeders) kmax = std::max(kmax, b.k[p]);

  // seeding chunks, in seeder order
  std::vector<uint32_t> ch_p, ch_len, cfirst(NP, 0), ccount(NP, 0);
  std::vector<uint64_t> ch_r0;
  std::vector<uint32_t> chunks_upto;  // chunks of seeders[0..i]
  for (uint32_t p : seeders) {
    cfirst[p] = (uint32_t)ch_p.size();
    for (uint64_t r = 0; r < b.n[p]; r += kChunk) {
      ch_p.push_back(p);
      ch_r0.push_back(b.off[p] + r);
      ch_len.push_back((uint32_t)std::min<uint64_t>(kChunk, b.n[p] - r));
    }
    ccount[p] = (uint32_t)ch_p.size() - cfirst[p];
    chunks_upto.push_back((uint32_t)ch_p.size());
  }
  // assignment tiles of the live problems: problems with many centroids (and
  // 64-dim rows) go through the tensor-core filter, the rest through the
  // exact scan
  const bool tc_on = ctx->tc_filter && !ctx->exhaustive_assign && dim == (uint32_t)kKmTcDim;
  std::vector<uint32_t> t_p, t_len, u_p, u_len, bbase(NP, 0);
  std::vector<uint64_t> t_r0, u_r0;
  std::vector<uint2> tcblocks;
  for (uint32_t p : live) {
    const bool filt = tc_on && b.k[p] >= (uint32_t)kKmTcMinK;
    if (filt) {
      bbase[p] = (uint32_t)tcblocks.size();
      for (uint32_t bk = 0; bk < (b.k[p] + kKmTcCols - 1) / kKmTcCols; ++bk) tcblocks.push_back(make_uint2(p, bk));
      for (uint64_t r = 0; r < b.n[p]; r += kKmTcRows) {
        u_p.push_back(p);
        u_r0.push_back(b.off[p] + r);
        u_len.push_back((uint32_t)std::min<uint64_t>(kKmTcRows, b.n[p] - r));
      }
      continue;
    }
    for (uint64_t r = 0; r < b.n[p]; r += kAsgT) {
      t_p.push_back(p);
      t_r0.push_back(b.off[p] + r);
      t_len.push_back((uint32_t)std::min<uint64_t>(kAsgT, b.n[p] - r));
    }
  }
  std::vector<uint32_t> cprob(KT);
  for (uint32_t p = 0; p < NP; ++p)
    for (uint32_t c = 0; c < b.k[p]; ++c) cprob[b.coff[p] + c] = p;

  // ---- host RNG draws: draw s of problem p at draws[coff_p + s] -----------
  std::vector<double> draws(KT, 0.0);
  std::vector<uint64_t> idx0(NP, 0);
  for (uint32_t p : live) {
    Xoshiro256pp rng(b.seed[p]);
    idx0[p] = rng.below(b.n[p]);
    for (uint32_t s = 1; s < b.k[p]; ++s) draws[b.coff[p] + s] = rng.unit_f64();
  }

  // ---- workspace -------------------------------------------------------------
  const int radix_nblk = (int)((rows + kRadixRows - 1) / kRadixRows);
  int passes = 1;
  while (passes < 4 && (KT >> (8 * passes)) > 0) ++passes;
  Carver cv;
  const size_t o_off = cv.take(NP * 8), o_n = cv.take(NP * 4), o_k = cv.take(NP * 4), o_coff = cv.take(NP * 8),
               o_state = cv.take(NP), o_status = cv.take(NP * 4), o_wcss = cv.take(NP * 4),
               o_prev = cv.take(NP * 4), o_iters = cv.take(NP * 4), o_thr = cv.take(NP * 8),
               o_fb = cv.take(NP * 4), o_nonf = cv.take(NP * 4), o_rs = cv.take(NP * 4),
               o_idx0 = cv.take(NP * 8), o_cfirst = cv.take(NP * 4), o_ccount = cv.take(NP * 4),
               o_seeders = cv.take(std::max<size_t>(1, seeders.size()) * 4),
               o_degen = cv.take(std::max<size_t>(1, degen.size()) * 4),
               o_live = cv.take(std::max<size_t>(1, live.size()) * 4),
               o_chp = cv.take(std::max<size_t>(1, ch_p.size()) * 4),
               o_chr0 = cv.take(std::max<size_t>(1, ch_r0.size()) * 8),
               o_chlen = cv.take(std::max<size_t>(1, ch_len.size()) * 4),
               o_tp = cv.take(std::max<size_t>(1, t_p.size()) * 4),
               o_tr0 = cv.take(std::max<size_t>(1, t_r0.size()) * 8),
               o_tlen = cv.take(std::max<size_t>(1, t_len.size()) * 4), o_cprob = cv.take(KT * 4),
               o_draws = cv.take(KT * 8), o_up = cv.take(std::max<size_t>(1, u_p.size()) * 4),
               o_ur0 = cv.take(std::max<size_t>(1, u_r0.size()) * 8),
               o_ulen = cv.take(std::max<size_t>(1, u_len.size()) * 4), o_bbase = cv.take(NP * 4),
               o_tcblk = cv.take(std::max<size_t>(1, tcblocks.size()) * 8);
  const size_t host_bytes = cv.off;  // everything above is copied from the host
  const size_t o_chsum = cv.take(std::max<size_t>(1, ch_p.size()) * sizeof(double2)),
               o_chcnt = cv.take(std::max<size_t>(1, ch_p.size()) * 4), o_md = cv.take(rows * 4),
               o_keys = cv.take(rows * 4), o_keys2 = cv.take(rows * 4), o_vals2 = cv.take(rows * 4),
               o_keys3 = cv.take(rows * 4), o_vals3 = cv.take(rows * 4), o_counts = cv.take(KT * 4), o_starts = cv.take(KT * 4),
               o_hist = cv.take((size_t)256 * radix_nblk * 4), o_base = cv.take((size_t)256 * radix_nblk * 4),
               o_part = cv.take((std::max<uint64_t>(KT, (uint64_t)256 * radix_nblk) / kScanTile + 2) * 4),
               o_cmx = cv.take(NP * 4 * 2), o_diag = cv.take(16),
               o_bg = cv.take(std::max<size_t>(1, tcblocks.size()) * (size_t)kKmTcBlockBytes);
  unsigned char* ws = nullptr;
  MVR_TRY(scratch(ctx, kSlotAux3, cv.off, (void**)&ws));
  std::vector<unsigned char> hb(host_bytes, 0);
  auto put = [&](size_t o, const void* src, size_t bytes) {
    if (bytes) std::memcpy(hb.data() + o, src, bytes);
  };
  put(o_off, b.off.data(), NP * 8);
  put(o_n, b.n.data(), NP * 4);
  put(o_k, b.k.data(), NP * 4);
  put(o_coff, b.coff.data(), NP * 8);
  {
    std::vector<uint8_t> st0(NP, kRunning);
    for (uint32_t p : degen) st0[p] = kDone;
    put(o_state, st0.data(), NP);
    std::vector<double> thr0(NP, HUGE_VAL);
    put(o_thr, thr0.data(), NP * 8);
  }
  put(o_idx0, idx0.data(), NP * 8);
  put(o_cfirst, cfirst.data(), NP * 4);
  put(o_ccount, ccount.data(), NP * 4);
  put(o_seeders, seeders.data(), seeders.size() * 4);
  put(o_degen, degen.data(), degen.size() * 4);
  put(o_live, live.data(), live.size() * 4);
  put(o_chp, ch_p.data(), ch_p.size() * 4);
  put(o_chr0, ch_r0.data(), ch_r0.size() * 8);
  put(o_chlen, ch_len.data(), ch_len.size() * 4);
  put(o_tp, t_p.data(), t_p.size() * 4);
  put(o_tr0, t_r0.data(), t_r0.size() * 8);
  put(o_tlen, t_len.data(), t_len.size() * 4);
  put(o_cprob, cprob.data(), KT * 4);
  put(o_draws, draws.data(), KT * 8);
  put(o_up, u_p.data(), u_p.size() * 4);
  put(o_ur0, u_r0.data(), u_r0.size() * 8);
  put(o_ulen, u_len.data(), u_len.size() * 4);
  put(o_bbase, bbase.data(), NP * 4);
  put(o_tcblk, tcblocks.data(), tcblocks.size() * 8);
  MVR_CUDA(ctx, cudaMemcpyAsync(ws, hb.data(), host_bytes, cudaMemcpyHostToDevice, st));

  Prob P;
  P.off = at<uint64_t>(ws, o_off);
  P.n = at<uint32_t>(ws, o_n);
  P.k = at<uint32_t>(ws, o_k);
  P.coff = at<uint64_t>(ws, o_coff);
  P.state = at<uint8_t>(ws, o_state);
  P.status = at<int>(ws, o_status);
  P.wcss = at<float>(ws, o_wcss);
  P.prev = at<float>(ws, o_prev);
  P.iters = at<uint32_t>(ws, o_iters);
  P.thr = at<double>(ws, o_thr);
  P.fb = at<uint32_t>(ws, o_fb);
  P.nonf = at<int>(ws, o_nonf);
  uint32_t* d_rs = at<uint32_t>(ws, o_rs);
  const int d = (int)dim;
  uint32_t launches = 0;

  cudaEvent_t* tev = nullptr;
  MVR_TRY(tac_events(ctx, &tev));
  MVR_CUDA(ctx, cudaEventRecord(tev[5], st));
  // every row carries a sort key below KT from the start (rows of problems
  // that fail while seeding are never assigned)
  MVR_CUDA(ctx, cudaMemsetAsync(at<uint32_t>(ws, o_keys), 0, rows * 4, st));

  // ---- degenerate problems ------------------------------------------------
  if (!degen.empty()) {
    km_degenerate_kernel<<<(unsigned)degen.size(), 128, 0, st>>>(d_G, d, P, at<uint32_t>(ws, o_degen), d_C, d_local,
                                                                 at<uint32_t>(ws, o_keys));
    MVR_CUDA(ctx, cudaGetLastError());
    ++launches;
  }

  // ---- seeding -----------------------------------------------------------------
  if (!live.empty()) {
    km_seed_init_kernel<<<(unsigned)live.size(), 64, 0, st>>>(d_G, d, P, at<uint32_t>(ws, o_live),
                                                              at<uint64_t>(ws, o_idx0), d_C);
    MVR_CUDA(ctx, cudaGetLastError());
    ++launches;
  }
  for (uint32_t s = 1; s < kmax; ++s) {
    // seeders with k > s form the prefix seeders[0 .. na)
    const uint32_t na = (uint32_t)(std::partition_point(seeders.begin(), seeders.end(),
                                                        [&](uint32_t p) { return b.k[p] > s; }) -
                                   seeders.begin());
    if (na == 0) break;
    const uint32_t nch = chunks_upto[na - 1];
    {
      const float4* gt4 = reinterpret_cast<const float4*>(d_GT);
      const size_t sm = (size_t)((d + 3) / 4) * sizeof(float4);
      auto upd = d == 64 ? km_seed_update_kernel<16> : d == 128 ? km_seed_update_kernel<32> : km_seed_update_kernel<0>;
      MVR_CUDA(ctx, launch_pdl(upd, dim3(nch), dim3(kUpdT), sm, st, gt4, rows, d, P, (int)s - 1,
                               (const uint32_t*)at<uint32_t>(ws, o_chp), (const uint64_t*)at<uint64_t>(ws, o_chr0),
                               (const uint32_t*)at<uint32_t>(ws, o_chlen), (const float*)d_C, at<float>(ws, o_md),
                               at<double2>(ws, o_chsum), at<uint32_t>(ws, o_chcnt)));
    }
    MVR_CUDA(ctx, launch_pdl(km_seed_select_kernel, dim3(na), dim3(kSelT), 0, st, (const float*)d_G, d, P, (int)s,
                             (const uint32_t*)at<uint32_t>(ws, o_seeders), (const uint32_t*)at<uint32_t>(ws, o_cfirst),
                             (const uint32_t*)at<uint32_t>(ws, o_ccount), (const uint64_t*)at<uint64_t>(ws, o_chr0),
                             (const uint32_t*)at<uint32_t>(ws, o_chlen), (const double2*)at<double2>(ws, o_chsum),
                             (const uint32_t*)at<uint32_t>(ws, o_chcnt), (const float*)at<float>(ws, o_md),
                             (const double*)at<double>(ws, o_draws), d_C, ctx->serial_draws ? 1 : 0));
    launches += 2;
  }

  MVR_CUDA(ctx, cudaEventRecord(tev[6], st));
  // ---- Lloyd iterations ---------------------------------------------------------
  const bool check = !(tol == -INFINITY) && !std::isnan(tol);
  float* mind = at<float>(ws, o_md);
  uint32_t* keys = at<uint32_t>(ws, o_keys);
  uint32_t* keys2 = at<uint32_t>(ws, o_keys2);
  uint32_t* vals2 = at<uint32_t>(ws, o_vals2);
  uint32_t* keys3 = at<uint32_t>(ws, o_keys3);
  uint32_t* vals3 = at<uint32_t>(ws, o_vals3);
  uint32_t* counts = at<uint32_t>(ws, o_counts);
  uint32_t* starts = at<uint32_t>(ws, o_starts);
  uint32_t* hist = at<uint32_t>(ws, o_hist);
  uint32_t* base = at<uint32_t>(ws, o_base);
  uint32_t* part = at<uint32_t>(ws, o_part);
  cudaStream_t side = nullptr;
  MVR_TRY(side_stream(ctx, &side));
  const unsigned ntiles = (unsigned)t_p.size();
  const size_t asg_smem = (size_t)kCT * d * sizeof(float);
  bool long_problems = false;
  for (uint32_t p : live) long_problems = long_problems || b.n[p] >= kWcssSeg;
  uint32_t* cmx = at<uint32_t>(ws, o_cmx);
  uint32_t* d_diag = at<uint32_t>(ws, o_diag);
  MVR_CUDA(ctx, cudaMemsetAsync(d_diag, 0, 16, st));
  if (!u_p.empty())
    MVR_CUDA(ctx, cudaFuncSetAttribute(km_tc_assign_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)kKmTcSmem));
  for (uint32_t it = 0; it < max_iters && !live.empty(); ++it) {
    MVR_CUDA(ctx, cudaMemsetAsync(counts, 0, KT * 4, st));
    if (!u_p.empty()) {  // filtered problems: operand tiles of the current centroids, then the filter
      MVR_CUDA(ctx, cudaMemsetAsync(cmx, 0, NP * 4 * 2, st));
      km_tc_prep_kernel<<<(unsigned)tcblocks.size(), kKmTcCols, 0, st>>>(P, at<uint2>(ws, o_tcblk), d_C,
                                                                   at<unsigned char>(ws, o_bg), cmx, cmx + NP);
      const unsigned g = (unsigned)std::min<size_t>(u_p.size(), (size_t)std::max(1, ctx->sm_count));
      km_tc_assign_kernel<<<g, 288, kKmTcSmem, st>>>(d_G, P, at<uint32_t>(ws, o_up), at<uint64_t>(ws, o_ur0),
                                                     at<uint32_t>(ws, o_ulen), (uint32_t)u_p.size(),
                                                     at<uint32_t>(ws, o_bbase), at<unsigned char>(ws, o_bg), cmx,
                                                     cmx + NP, d_C, d_local, mind, keys, d_diag);
      MVR_CUDA(ctx, cudaGetLastError());
      launches += 2;
    }
    if (ntiles == 0) {
    } else if (d == 64) {
      km_assign_kernel<64><<<ntiles, kAsgT, asg_smem, st>>>(d_G, d, P, at<uint32_t>(ws, o_tp), at<uint64_t>(ws, o_tr0),
                                                             at<uint32_t>(ws, o_tlen), d_C, d_local, mind, keys);
    } else if (d == 128) {
      km_assign_kernel<128><<<ntiles, kAsgT, asg_smem, st>>>(d_G, d, P, at<uint32_t>(ws, o_tp), at<uint64_t>(ws, o_tr0),
                                                              at<uint32_t>(ws, o_tlen), d_C, d_local, mind, keys);
    } else {
      km_assign_kernel<0><<<ntiles, kAsgT, asg_smem, st>>>(d_G, d, P, at<uint32_t>(ws, o_tp), at<uint64_t>(ws, o_tr0),
                                                            at<uint32_t>(ws, o_tlen), d_C, d_local, mind, keys);
    }
    MVR_CUDA(ctx, cudaGetLastError());
    km_count_kernel<<<1024, 256, 0, st>>>(keys, rows, counts);
    MVR_CUDA(ctx, cudaGetLastError());
    launches += 2;
    const bool last = it + 1 == max_iters;
    const bool want_wcss = check || last;
    if (want_wcss) {  // the serial WCSS overlaps the sort and the centroid sums
      MVR_CUDA(ctx, cudaEventRecord(ctx->fork_ev, st));
      MVR_CUDA(ctx, cudaStreamWaitEvent(side, ctx->fork_ev, 0));
      km_wcss_kernel<<<(unsigned)((NP + 3) / 4), 128, 0, side>>>(P, (uint32_t)NP, mind);
      MVR_CUDA(ctx, cudaGetLastError());
      if (long_problems) {
        km_wcss_seg_kernel<<<(unsigned)NP, kSegT, 0, side>>>(P, mind);
        MVR_CUDA(ctx, cudaGetLastError());
        ++launches;
      }
      MVR_CUDA(ctx, cudaEventRecord(ctx->join_ev, side));
      ++launches;
    }
    MVR_TRY(scan_u32(ctx, st, counts, KT, part, starts));
    // stable radix sort of (global cluster, row); `keys` stays in row order
    // (rows of finished problems keep their keys), the passes ping-pong
    // between the 2 and 3 buffers
    const uint32_t* ki = keys;
    const uint32_t* vi = nullptr;
    uint32_t *ko = keys2, *vo = vals2;
    for (int pass = 0; pass < passes; ++pass) {
      const int shift = 8 * pass;
      const unsigned g = (unsigned)((radix_nblk + kRadixWarps - 1) / kRadixWarps);
      km_radix_hist_kernel<<<g, kRadixWarps * 32, 0, st>>>(ki, rows, shift, radix_nblk, hist);
      MVR_TRY(scan_u32(ctx, st, hist, (uint64_t)256 * radix_nblk, part, base));
      km_radix_scatter_kernel<<<g, kRadixWarps * 32, 0, st>>>(ki, vi, rows, shift, radix_nblk, base, ko, vo);
      MVR_CUDA(ctx, cudaGetLastError());
      ki = ko;
      vi = vo;
      ko = ko == keys2 ? keys3 : keys2;
      vo = vo == vals2 ? vals3 : vals2;
      launches += 5;
    }
    const unsigned cgrid = (unsigned)((KT + 7) / 8);
    if (d == 64)
      km_chain_kernel<64><<<cgrid, 256, 0, st>>>(d_G, d, P, at<uint32_t>(ws, o_cprob), KT, counts, starts, vi, d_C);
    else if (d == 128)
      km_chain_kernel<128><<<cgrid, 256, 0, st>>>(d_G, d, P, at<uint32_t>(ws, o_cprob), KT, counts, starts, vi, d_C);
    else
      km_chain_kernel<0><<<cgrid, 256, 0, st>>>(d_G, d, P, at<uint32_t>(ws, o_cprob), KT, counts, starts, vi, d_C);
    MVR_CUDA(ctx, cudaGetLastError());
    if (want_wcss) MVR_CUDA(ctx, cudaStreamWaitEvent(st, ctx->join_ev, 0));
    km_reseed_converge_kernel<<<(unsigned)NP, 256, 0, st>>>(d_G, d, P, (uint32_t)NP, counts, mind, d_C, d_rs,
                                                            (int)it, check ? 1 : 0, tol);
    MVR_CUDA(ctx, cudaGetLastError());
    launches += 5;
  }

  MVR_CUDA(ctx, cudaEventRecord(tev[7], st));
  // ---- results ------------------------------------------------------------------
  uint32_t hdiag[4] = {0, 0, 0, 0};
  MVR_CUDA(ctx, cudaMemcpyAsync(hdiag, d_diag, 16, cudaMemcpyDeviceToHost, st));
  MVR_CUDA(ctx, cudaStreamSynchronize(st));
  if (hdiag[2]) return fail(ctx, MVR_E_TIMEOUT, "tensor-core filter: a bulk copy or an MMA did not complete in time");
  if (hdiag[0]) {
    // a winner's approximation broke its error bound: the whole batch again
    // with the exact scans
    ctx->tc_filter = false;
    const int s2 = km_batch_run(ctx, d_G, d_GT, rows, dim, b, max_iters, tol, d_C, d_local, res);
    ctx->tc_filter = true;
    res->filter_violations = hdiag[0];
    return s2;
  }
  res->filter_rows_rechecked = hdiag[1];
  res->filter_rows_full_scan = hdiag[3];
  std::vector<int> hstatus(NP);
  std::vector<uint32_t> hfb(NP);
  MVR_CUDA(ctx, cudaMemcpyAsync(hstatus.data(), P.status, NP * 4, cudaMemcpyDeviceToHost, st));
  MVR_CUDA(ctx, cudaMemcpyAsync(res->wcss.data(), P.wcss, NP * 4, cudaMemcpyDeviceToHost, st));
  MVR_CUDA(ctx, cudaMemcpyAsync(res->iters.data(), P.iters, NP * 4, cudaMemcpyDeviceToHost, st));
  MVR_CUDA(ctx, cudaMemcpyAsync(hfb.data(), P.fb, NP * 4, cudaMemcpyDeviceToHost, st));
  MVR_CUDA(ctx, cudaStreamSynchronize(st));
  res->status = hstatus;
  {
    float a = 0.f, b2 = 0.f;
    cudaEventElapsedTime(&a, tev[5], tev[6]);
    cudaEventElapsedTime(&b2, tev[6], tev[7]);
    res->seed_ms = a;
    res->lloyd_ms = b2;
  }
  res->seed_fallbacks = std::accumulate(hfb.begin(), hfb.end(), 0u);
  res->launches = launches;
  for (uint32_t p : degen) {
    res->wcss[p] = 0.f;
    res->iters[p] = 0;
  }
  if (max_iters == 0)
    for (size_t p = 0; p < NP; ++p) {
      res->wcss[p] = 0.f;
      res->iters[p] = 0;
    }
  return MVR_OK;
}

}  // namespace mvr
