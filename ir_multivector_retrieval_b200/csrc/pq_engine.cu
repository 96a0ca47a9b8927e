// pq_engine.cu — PQ subspace k-means and PQ encoding on sm_100a.
//
// Reference path (BleedingDev/ir-multivector-retrieval):
//   pq.train            src/index/pq.zig:158-336
//   kmeans.fit          src/tac/kmeans.zig:67-232
//   kmeans.assignSlice  src/tac/kmeans.zig:344-365
//   rng.weightedSample  src/util/rng.zig:57-82
//   PQ.encode           src/index/pq.zig:59-76
//
// Data layout in HBM (N rows, M subspaces of S floats, K centroids):
//   R        [N][D]      caller's rows, read in place (no transpose)
//   codebook [M][K][S]   the reference layout codebook[m][c][k]
//   minDist  [M][N] f32  k-means++ D^2 weights, then Lloyd min_to_any
//   assign   [M][N] u8   Lloyd assignments (K <= 256)
//   hist     [M][nblk][K] u32 per-CTA cluster histograms -> scatter bases
//   sorted   [M][N][S]   rows of each subspace stably sorted by cluster
//
// Bit-exactness with the reference:
//   * distances: mvr_device.cuh (exact order, no FMA);
//   * argmin: first minimum (strict <), kmeans.fit starts from dists[0],
//     PQ.encode from +inf;
//   * centroid sums: the reference adds members in row order into one f32
//     accumulator per (cluster, coordinate). A stable counting sort by
//     cluster followed by one sequential f32 chain per (cluster,
//     coordinate) reproduces that order exactly;
//   * mean: sum * (1 / (float)count), both correctly rounded;
//   * k-means++ draws: the reference's sequential f64 prefix sum is bounded
//     rigorously with directed-rounding partial sums plus the recursive
//     summation error bound; a draw whose outcome the bound cannot decide
//     is recomputed with the exact sequential chain on the device.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "mvr_device.cuh"
#include "mvr_rng.h"
#include "pq_engine.h"

namespace mvr {
namespace {

constexpr int kThreads = 256;          // assign / scatter / seed-update CTA size
constexpr int kPtsPerThread = 2;       // rows per thread in assign / scatter
constexpr int kTile = kThreads * kPtsPerThread;  // rows per assign CTA
constexpr int kSeedChunk = kThreads;   // rows per seed-update CTA
constexpr int kSelectThreads = 1024;
constexpr int kChainCh = 32;           // elements per cluster per pipeline stage
constexpr int kChainStages = 6;

enum : uint8_t { kRunning = 0, kDone = 1, kFailed = 2 };
enum { kModeEncode = 0, kModeLloyd = 1 };

template <int S>
__device__ __forceinline__ void load_sub(const float* __restrict__ p, float (&x)[S]) {
#pragma unroll
  for (int k = 0; k < S; ++k) x[k] = __ldg(p + k);
}

// ---------------------------------------------------------------------------
// Assignment / encode: one thread handles kPtsPerThread rows across all M
// subspaces; the M codebooks sit in shared memory as negated centroid pairs
// so that two distances come out of each packed f32x2 instruction.
// ---------------------------------------------------------------------------
template <int S, int MODE>
__global__ void __launch_bounds__(kThreads)
pq_assign_kernel(const float* __restrict__ R, uint64_t N, int D, int M, int K,
                 const float* __restrict__ cb, uint8_t* __restrict__ codes,
                 uint8_t* __restrict__ asg, float* __restrict__ mind,
                 uint32_t* __restrict__ hist, const uint8_t* __restrict__ state, float one) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int KP = (K + 1) >> 1;
  float2* cbp = reinterpret_cast<float2*>(smem_raw);  // [M][KP][S]
  uint32_t* h = reinterpret_cast<uint32_t*>(cbp + (size_t)M * KP * S);  // [M][K]

  for (int e = threadIdx.x; e < M * KP * S; e += kThreads) {
    const int k = e % S;
    const int p = (e / S) % KP;
    const int m = e / (S * KP);
    const int ca = 2 * p, cbi = 2 * p + 1;
    const float a = cb[((size_t)m * K + ca) * S + k];
    const float b = cbi < K ? cb[((size_t)m * K + cbi) * S + k] : f32_nan();
    cbp[e] = make_float2(-a, -b);  // a NaN pad never wins a strict '<'
  }
  if (MODE == kModeLloyd)
    for (int e = threadIdx.x; e < M * K; e += kThreads) h[e] = 0;
  __syncthreads();

  const uint64_t base = (uint64_t)blockIdx.x * kTile;
  uint64_t row[kPtsPerThread];
  bool ok[kPtsPerThread];
#pragma unroll
  for (int j = 0; j < kPtsPerThread; ++j) {
    row[j] = base + (uint64_t)j * kThreads + threadIdx.x;
    ok[j] = row[j] < N;
  }
  uint32_t packed[kPtsPerThread] = {0u};
  const float2 one2 = make_float2(one, one);  // 1.0f, opaque to the compiler

  for (int m = 0; m < M; ++m) {
    if (MODE == kModeLloyd && state[m] != kRunning) continue;
    float2 xx[kPtsPerThread][S];
#pragma unroll
    for (int j = 0; j < kPtsPerThread; ++j) {
      float x[S];
      if (ok[j]) {
        load_sub<S>(R + row[j] * (uint64_t)D + (uint64_t)m * S, x);
      } else {
#pragma unroll
        for (int k = 0; k < S; ++k) x[k] = 0.f;
      }
#pragma unroll
      for (int k = 0; k < S; ++k) xx[j][k] = make_float2(x[k], x[k]);
    }
    float best[kPtsPerThread], d0[kPtsPerThread];
    int bi[kPtsPerThread];
#pragma unroll
    for (int j = 0; j < kPtsPerThread; ++j) {
      best[j] = __int_as_float(0x7f800000);
      bi[j] = 0;
      d0[j] = 0.f;
    }
    const float2* cm = cbp + (size_t)m * KP * S;
    for (int p = 0; p < KP; ++p) {
      float2 nc[S];
#pragma unroll
      for (int k = 0; k < S; ++k) nc[k] = cm[p * S + k];
#pragma unroll
      for (int j = 0; j < kPtsPerThread; ++j) {
        const float2 dd = l2_small_pair<S>(xx[j], nc, one2);
        if (p == 0) d0[j] = dd.x;
        if (dd.x < best[j]) { best[j] = dd.x; bi[j] = 2 * p; }
        if (dd.y < best[j]) { best[j] = dd.y; bi[j] = 2 * p + 1; }
      }
    }
#pragma unroll
    for (int j = 0; j < kPtsPerThread; ++j) {
      if (MODE == kModeLloyd) {
        // vec.argmin starts from dists[0]: a NaN there wins by default.
        if (isnan(d0[j])) { bi[j] = 0; best[j] = d0[j]; }
        if (ok[j]) {
          asg[(size_t)m * N + row[j]] = (uint8_t)bi[j];
          mind[(size_t)m * N + row[j]] = best[j];
          atomicAdd(&h[m * K + bi[j]], 1u);
        }
      } else {
        if (ok[j]) {
          packed[j] |= (uint32_t)bi[j] << (8 * (m & 3));
          if ((m & 3) == 3 || m == M - 1) {
            uint8_t* dst = codes + row[j] * (uint64_t)M + (m & ~3);
            const int nb = (m & 3) + 1;
            if (nb == 4 && (reinterpret_cast<uintptr_t>(dst) & 3) == 0) {
              *reinterpret_cast<uint32_t*>(dst) = packed[j];
            } else {
              for (int b = 0; b < nb; ++b) dst[b] = (uint8_t)(packed[j] >> (8 * b));
            }
            packed[j] = 0u;
          }
        }
      }
    }
  }
  if (MODE == kModeLloyd) {
    __syncthreads();
    const int nblk = gridDim.x;
    for (int e = threadIdx.x; e < M * K; e += kThreads) {
      const int m = e / K, c = e % K;
      hist[((size_t)m * nblk + blockIdx.x) * K + c] = h[e];
    }
  }
}

// ---------------------------------------------------------------------------
// Per-cluster counts and stable scatter bases: for each (m, c), base of CTA
// b = start[c] + sum_{b' < b} hist[b'][c].
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
pq_scan_kernel(uint32_t* __restrict__ hist, int nblk, int K,
               uint32_t* __restrict__ counts, uint32_t* __restrict__ starts,
               const uint8_t* __restrict__ state) {
  const int m = blockIdx.x;
  if (state[m] != kRunning) return;
  __shared__ uint32_t tot[256];
  const int c = threadIdx.x;
  uint32_t* hm = hist + (size_t)m * nblk * K;
  uint32_t total = 0;
  if (c < K)
    for (int b = 0; b < nblk; ++b) total += hm[(size_t)b * K + c];
  tot[c] = c < K ? total : 0u;
  __syncthreads();
  // exclusive scan over clusters (256 entries, Hillis-Steele)
  for (int o = 1; o < 256; o <<= 1) {
    const uint32_t v = c >= o ? tot[c - o] : 0u;
    __syncthreads();
    tot[c] += v;
    __syncthreads();
  }
  const uint32_t start = tot[c] - (c < K ? total : 0u);
  if (c < K) {
    counts[(size_t)m * K + c] = total;
    starts[(size_t)m * K + c] = start;
    uint32_t run = start;
    for (int b = 0; b < nblk; ++b) {
      const uint32_t v = hm[(size_t)b * K + c];
      hm[(size_t)b * K + c] = run;
      run += v;
    }
  }
}

// ---------------------------------------------------------------------------
// Stable scatter of every subspace's rows into cluster order. Rows of a CTA
// are ranked in row order: 16 groups of 32 consecutive rows, ranks within a
// group from __match_any_sync, group prefixes per cluster in shared memory.
// ---------------------------------------------------------------------------
template <int S>
__global__ void __launch_bounds__(kThreads)
pq_scatter_kernel(const float* __restrict__ R, uint64_t N, int D, int M, int K,
                  const uint8_t* __restrict__ asg, const uint32_t* __restrict__ bases,
                  float* __restrict__ sorted, const uint8_t* __restrict__ state) {
  constexpr int kGroups = kTile / 32;
  __shared__ uint32_t gcnt[kGroups][256];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint64_t base = (uint64_t)blockIdx.x * kTile;
  const int nblk = gridDim.x;
  for (int m = 0; m < M; ++m) {
    if (state[m] != kRunning) continue;
    for (int e = threadIdx.x; e < kGroups * 256; e += kThreads) (&gcnt[0][0])[e] = 0u;
    __syncthreads();
    int cl[kPtsPerThread], rank[kPtsPerThread];
#pragma unroll
    for (int j = 0; j < kPtsPerThread; ++j) {
      const uint64_t r = base + (uint64_t)j * kThreads + threadIdx.x;
      const bool ok = r < N;
      cl[j] = ok ? (int)asg[(size_t)m * N + r] : 256 + lane;  // unique dummy keys
      const uint32_t peers = __match_any_sync(0xffffffffu, cl[j]);
      rank[j] = __popc(peers & lanemask_lt());
      const int g = j * (kThreads / 32) + warp;
      if (ok && rank[j] == 0) gcnt[g][cl[j]] = __popc(peers);
    }
    __syncthreads();
    {  // exclusive prefix over groups, per cluster
      const int c = threadIdx.x;
      uint32_t run = 0;
      for (int g = 0; g < kGroups; ++g) {
        const uint32_t v = gcnt[g][c];
        gcnt[g][c] = run;
        run += v;
      }
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kPtsPerThread; ++j) {
      const uint64_t r = base + (uint64_t)j * kThreads + threadIdx.x;
      if (r < N) {
        const int g = j * (kThreads / 32) + warp;
        const uint32_t dst = bases[((size_t)m * nblk + blockIdx.x) * K + cl[j]] +
                             gcnt[g][cl[j]] + (uint32_t)rank[j];
        const float* src = R + r * (uint64_t)D + (uint64_t)m * S;
        float* o = sorted + ((size_t)m * N + dst) * S;
        if constexpr (S == 4) {
          *reinterpret_cast<float4*>(o) = make_float4(__ldg(src), __ldg(src + 1), __ldg(src + 2), __ldg(src + 3));
        } else if constexpr (S == 2) {
          *reinterpret_cast<float2*>(o) = make_float2(__ldg(src), __ldg(src + 1));
        } else {
          o[0] = __ldg(src);
        }
      }
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Centroid sums in the reference order: one warp per 32 clusters of a
// subspace, lane = cluster, S sequential f32 chains per lane. Cluster
// members stream through a multi-stage cp.async ring in shared memory.
// Empty clusters are left for the reseed kernel.
// ---------------------------------------------------------------------------
template <int S>
__global__ void __launch_bounds__(32)
pq_chain_kernel(const float* __restrict__ sorted, uint64_t N, int K,
                const uint32_t* __restrict__ counts, const uint32_t* __restrict__ starts,
                float* __restrict__ cb, const uint8_t* __restrict__ state) {
  extern __shared__ __align__(16) float ring[];  // [stages][32][(CH+1)*S]
  constexpr int kRow = (kChainCh + 1) * S;      // padded: conflict-free reads
  constexpr int kStage = 32 * kRow;
  const int wpm = (K + 31) / 32;
  const int m = blockIdx.x / wpm;
  const int c0 = (blockIdx.x % wpm) * 32;
  if (state[m] != kRunning) return;
  const int lane = threadIdx.x;
  const int c = c0 + lane;
  const uint32_t cnt = c < K ? counts[(size_t)m * K + c] : 0u;
  const uint32_t st = c < K ? starts[(size_t)m * K + c] : 0u;
  uint32_t maxcnt = cnt;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) maxcnt = max(maxcnt, __shfl_xor_sync(0xffffffffu, maxcnt, o));
  const int nst = (int)((maxcnt + kChainCh - 1) / kChainCh);
  const float* sm = sorted + (size_t)m * N * S;

  auto issue = [&](int t) {
    if (t < nst) {
      float* dstage = ring + (t % kChainStages) * kStage;
      for (int j = 0; j < 32; ++j) {
        const uint32_t cj = __shfl_sync(0xffffffffu, cnt, j);
        const uint32_t sj = __shfl_sync(0xffffffffu, st, j);
        const uint32_t e = (uint32_t)t * kChainCh + lane;
        if (e < cj) cp_async<4 * S>(dstage + j * kRow + lane * S, sm + (size_t)(sj + e) * S);
      }
    }
    cp_async_commit();
  };

  float acc[S];
#pragma unroll
  for (int k = 0; k < S; ++k) acc[k] = 0.f;
  for (int t = 0; t < kChainStages - 1; ++t) issue(t);
  for (int t = 0; t < nst; ++t) {
    cp_async_wait<kChainStages - 2>();
    __syncwarp();
    const float* src = ring + (t % kChainStages) * kStage + lane * kRow;
    const uint32_t done = (uint32_t)t * kChainCh;
    const int n = cnt > done ? (int)min((uint32_t)kChainCh, cnt - done) : 0;
    for (int e = 0; e < n; ++e) {
      if constexpr (S == 4) {
        const float4 v = *reinterpret_cast<const float4*>(src + e * 4);
        acc[0] = __fadd_rn(acc[0], v.x);
        acc[1] = __fadd_rn(acc[1], v.y);
        acc[2] = __fadd_rn(acc[2], v.z);
        acc[3] = __fadd_rn(acc[3], v.w);
      } else if constexpr (S == 2) {
        const float2 v = *reinterpret_cast<const float2*>(src + e * 2);
        acc[0] = __fadd_rn(acc[0], v.x);
        acc[1] = __fadd_rn(acc[1], v.y);
      } else {
        acc[0] = __fadd_rn(acc[0], src[e]);
      }
    }
    __syncwarp();
    issue(t + kChainStages - 1);
  }
  cp_async_wait<0>();
  if (c < K && cnt > 0) {
    const float inv = __fdiv_rn(1.0f, __uint2float_rn(cnt));
#pragma unroll
    for (int k = 0; k < S; ++k) cb[((size_t)m * K + c) * S + k] = __fmul_rn(acc[k], inv);
  }
}

// ---------------------------------------------------------------------------
// Sequential f32 WCSS of one subspace (kmeans.zig:179), row order.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
pq_wcss_kernel(const float* __restrict__ mind, uint64_t N, float* __restrict__ wcss,
               const uint8_t* __restrict__ state) {
  const int m = blockIdx.x;
  if (state[m] != kRunning) return;
  __shared__ __align__(16) float tile[4096];
  const float* src = mind + (size_t)m * N;
  float acc = 0.f;
  for (uint64_t t0 = 0; t0 < N; t0 += 4096) {
    const uint64_t n = min((uint64_t)4096, N - t0);
    for (uint32_t e = threadIdx.x; e < n; e += 256) tile[e] = src[t0 + e];
    __syncthreads();
    if (threadIdx.x == 0)
      for (uint32_t e = 0; e < n; ++e) acc = __fadd_rn(acc, tile[e]);
    __syncthreads();
  }
  if (threadIdx.x == 0) wcss[m] = acc;
}

// First maximum of v[0..n) with vec.argmax semantics (vec.zig:287-299):
// strict '>' scan from v[0]; a NaN at index 0 wins, later NaNs never do.
__device__ uint64_t block_argmax_first(const float* v, uint64_t n) {
  __shared__ float bv[32];
  __shared__ uint64_t bi[32];
  float best = -__int_as_float(0x7f800000);
  uint64_t idx = n;  // sentinel: larger than any index
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
    if (lane == 0) { bi[0] = (isnan(v[0]) || idx >= n) ? 0 : idx; }
  }
  __syncthreads();
  const uint64_t r = bi[0];
  __syncthreads();
  return r;
}

// ---------------------------------------------------------------------------
// Empty-cluster reseed in cluster order (kmeans.zig:199-211), then the
// relative-WCSS convergence test (kmeans.zig:214-223).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024)
pq_reseed_converge_kernel(const float* __restrict__ R, uint64_t N, int D, int S, int K,
                          const uint32_t* __restrict__ counts, float* __restrict__ mind,
                          float* __restrict__ cb, uint8_t* __restrict__ state,
                          const float* __restrict__ wcss, float* __restrict__ prev_wcss,
                          uint32_t* __restrict__ iters_run, uint32_t* __restrict__ reseeds,
                          int iter, int check, float tol) {
  const int m = blockIdx.x;
  if (state[m] != kRunning) return;
  __shared__ int any_empty;
  if (threadIdx.x == 0) any_empty = 0;
  __syncthreads();
  for (int c = threadIdx.x; c < K; c += blockDim.x)
    if (counts[(size_t)m * K + c] == 0) atomicOr(&any_empty, 1);
  __syncthreads();
  if (any_empty) {
    float* mm = mind + (size_t)m * N;
    for (int c = 0; c < K; ++c) {
      if (counts[(size_t)m * K + c] != 0) continue;
      const uint64_t far = block_argmax_first(mm, N);
      if (threadIdx.x < (unsigned)S)
        cb[((size_t)m * K + c) * S + threadIdx.x] = R[far * (uint64_t)D + (uint64_t)m * S + threadIdx.x];
      __syncthreads();
      if (threadIdx.x == 0) {
        mm[far] = -__int_as_float(0x7f800000);
        reseeds[m] += 1;
      }
      __syncthreads();
    }
  }
  if (threadIdx.x == 0) {
    iters_run[m] = (uint32_t)iter + 1;
    if (check) {
      const float w = wcss[m];
      if (iter > 0) {
        const float prev = prev_wcss[m];
        const float denom = prev > 0.f ? prev : 1.0f;
        const float rel = __fdiv_rn(__fsub_rn(prev, w), denom);
        if (rel < tol) state[m] = kDone;
      }
      prev_wcss[m] = w;
    }
  }
}

// ---------------------------------------------------------------------------
// k-means++ seeding
// ---------------------------------------------------------------------------
__global__ void pq_seed_init_kernel(const float* __restrict__ R, int D, int S, int K,
                                    const uint64_t* __restrict__ idx0, float* __restrict__ cb,
                                    uint64_t* __restrict__ chosen) {
  const int m = blockIdx.x;
  if (threadIdx.x < (unsigned)S)
    cb[(size_t)m * K * S + threadIdx.x] = R[idx0[m] * (uint64_t)D + (uint64_t)m * S + threadIdx.x];
  if (threadIdx.x == 0) chosen[(size_t)m * K] = idx0[m];
}

// min_dist update with centroid `step` (kmeans.zig:117-135) fused with the
// per-CTA directed-rounding partial sums of the new weights.
template <int S>
__global__ void __launch_bounds__(kThreads)
pq_seed_update_kernel(const float* __restrict__ R, uint64_t N, int D, int M, int K, int step,
                      const float* __restrict__ cb, float* __restrict__ md,
                      double2* __restrict__ chunk, int* __restrict__ nonfinite,
                      const uint8_t* __restrict__ state) {
  __shared__ double2 red[kThreads / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint64_t i = (uint64_t)blockIdx.x * kSeedChunk + threadIdx.x;
  const int nchunk = gridDim.x;
  for (int m = 0; m < M; ++m) {
    if (state[m] != kRunning) continue;
    const float* c = cb + ((size_t)m * K + step) * S;
    float w = 0.f;
    if (i < N) {
      float x[S], cc[S];
      load_sub<S>(R + i * (uint64_t)D + (uint64_t)m * S, x);
#pragma unroll
      for (int k = 0; k < S; ++k) cc[k] = c[k];
      const float d = l2_small<S>(x, cc);
      float* slot = md + (size_t)m * N + i;
      if (step == 0) {
        w = d;
      } else {
        const float old = *slot;
        w = d < old ? d : old;
      }
      *slot = w;
      if (!isfinite(w) || w < 0.f) nonfinite[m] = 1;
    }
    const double lo = warp_sum_rd((double)w);
    const double hi = warp_sum_ru((double)w);
    if (lane == 0) red[warp] = make_double2(lo, hi);
    __syncthreads();
    if (warp == 0) {
      double2 v = lane < kThreads / 32 ? red[lane] : make_double2(0.0, 0.0);
      const double l2 = warp_sum_rd(v.x), h2 = warp_sum_ru(v.y);
      if (lane == 0) chunk[(size_t)m * nchunk + blockIdx.x] = make_double2(l2, h2);
    }
    __syncthreads();
  }
}

// Upper bound of gamma_n = n u / (1 - n u), u = 2^-53: the recursive
// summation error bound |S_n - E_n| <= gamma_{n-1} * sum |w_i| (Higham,
// "Accuracy and Stability of Numerical Algorithms", 2nd ed., eq. 4.4).
__device__ __forceinline__ double gamma_bound(uint64_t n) {
  const double g = __dmul_ru(__ull2double_ru(n), 1.1102230246251565e-16);
  return __ddiv_ru(g, __dsub_rd(1.0, g));
}

// Draw for centroid `step` (weightedSample, rng.zig:57-82): candidate from
// the directed-rounding prefix bounds, accepted when the reference's
// sequential f64 prefix provably selects the same row; otherwise the exact
// sequential chain decides.
__global__ void __launch_bounds__(kSelectThreads)
pq_seed_select_kernel(const float* __restrict__ R, uint64_t N, int D, int S, int K, int step,
                      float* __restrict__ cb, const float* __restrict__ md,
                      const double2* __restrict__ chunk, int nchunk,
                      const double* __restrict__ draws, int* __restrict__ nonfinite,
                      int* __restrict__ status, uint8_t* __restrict__ state,
                      uint32_t* __restrict__ fallbacks, uint64_t* __restrict__ chosen) {
  const int m = blockIdx.x;
  if (state[m] != kRunning) return;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int kWarps = kSelectThreads / 32;
  __shared__ double2 wsum[kWarps];
  __shared__ double2 incl_all[kSelectThreads];
  __shared__ double2 sh_excl;      // exclusive prefix of the found chunk
  __shared__ int sh_chunk;
  __shared__ double2 pre[kSeedChunk];  // element inclusive prefixes in the chunk
  __shared__ uint64_t sh_idx;
  __shared__ int sh_decided;
  __shared__ float tile[4096];
  __shared__ double sh_u;

  if (nonfinite[m]) {  // weightedSample validates every weight first
    if (tid == 0) { status[m] = MVR_E_NON_FINITE; state[m] = kFailed; }
    return;
  }
  const double2* ch = chunk + (size_t)m * nchunk;
  const float* w = md + (size_t)m * N;
  const double r = draws[(size_t)m * K + step];

  // 1. per-thread contiguous chunk ranges, then a block scan of the totals
  const int cpt = (nchunk + kSelectThreads - 1) / kSelectThreads;
  const int c_lo = min(nchunk, tid * cpt), c_hi = min(nchunk, c_lo + cpt);
  double tlo = 0.0, thi = 0.0;
  for (int j = c_lo; j < c_hi; ++j) { tlo = __dadd_rd(tlo, ch[j].x); thi = __dadd_ru(thi, ch[j].y); }
  double ilo = warp_scan_rd(tlo, lane), ihi = warp_scan_ru(thi, lane);
  if (lane == 31) wsum[warp] = make_double2(ilo, ihi);
  __syncthreads();
  if (warp == 0) {
    double a = wsum[lane].x, b = wsum[lane].y;
    a = warp_scan_rd(a, lane);
    b = warp_scan_ru(b, lane);
    wsum[lane] = make_double2(a, b);
  }
  __syncthreads();
  const double wlo = warp > 0 ? wsum[warp - 1].x : 0.0, whi = warp > 0 ? wsum[warp - 1].y : 0.0;
  const double incl_lo = __dadd_rd(wlo, ilo), incl_hi = __dadd_ru(whi, ihi);
  const double Lo_N = wsum[kWarps - 1].x, Hi_N = wsum[kWarps - 1].y;
  if (Hi_N <= 0.0) {  // every weight is exactly zero
    if (tid == 0) { status[m] = MVR_E_ALL_ZERO; state[m] = kFailed; }
    return;
  }
  const double u_mid = r * (0.5 * (Lo_N + Hi_N));
  const bool past = !(u_mid < 0.5 * (incl_lo + incl_hi));
  incl_all[tid] = make_double2(incl_lo, incl_hi);
  const int n_before = __syncthreads_count(past);  // prefixes are monotone
  if (tid == 0) { sh_decided = 0; sh_chunk = -1; }
  __syncthreads();

  // 2. the first thread whose inclusive mid-prefix exceeds u_mid walks its
  //    chunks, starting from its predecessor's inclusive bounds.
  if (n_before < kSelectThreads && tid == n_before) {
    double lo = tid > 0 ? incl_all[tid - 1].x : 0.0;
    double hi = tid > 0 ? incl_all[tid - 1].y : 0.0;
    int found = -1;
    for (int j = c_lo; j < c_hi; ++j) {
      const double nlo = __dadd_rd(lo, ch[j].x), nhi = __dadd_ru(hi, ch[j].y);
      if (u_mid < 0.5 * (nlo + nhi)) { found = j; break; }
      lo = nlo; hi = nhi;
    }
    sh_chunk = found;
    sh_excl = make_double2(lo, hi);
  }
  __syncthreads();

  // 3. fine search inside the chunk (warp 0, 8 rows per lane)
  if (sh_chunk >= 0 && warp == 0) {
    const uint64_t cbase = (uint64_t)sh_chunk * kSeedChunk;
    constexpr int kPer = kSeedChunk / 32;
    double llo[kPer], lhi[kPer];
    double slo = 0.0, shi = 0.0;
#pragma unroll
    for (int e = 0; e < kPer; ++e) {
      const uint64_t i = cbase + (uint64_t)lane * kPer + e;
      const double v = i < N ? (double)w[i] : 0.0;
      slo = __dadd_rd(slo, v); shi = __dadd_ru(shi, v);
      llo[e] = slo; lhi[e] = shi;
    }
    const double plo = warp_scan_rd(slo, lane), phi = warp_scan_ru(shi, lane);
    double xlo = __shfl_up_sync(0xffffffffu, plo, 1), xhi = __shfl_up_sync(0xffffffffu, phi, 1);
    if (lane == 0) { xlo = 0.0; xhi = 0.0; }
    const double2 ex = sh_excl;
    const double blo = __dadd_rd(ex.x, xlo), bhi = __dadd_ru(ex.y, xhi);
    int first = -1;
#pragma unroll
    for (int e = 0; e < kPer; ++e) {
      const double elo = __dadd_rd(blo, llo[e]), ehi = __dadd_ru(bhi, lhi[e]);
      pre[lane * kPer + e] = make_double2(elo, ehi);
      const uint64_t i = cbase + (uint64_t)lane * kPer + e;
      if (first < 0 && i < N && u_mid < 0.5 * (elo + ehi)) first = e;
    }
    __syncwarp();
    const uint32_t bal = __ballot_sync(0xffffffffu, first >= 0);
    if (bal) {
      const int fl = __ffs(bal) - 1;
      const int fe = __shfl_sync(0xffffffffu, first, fl);
      if (lane == 0) {
        const int e = fl * kPer + fe;
        const uint64_t istar = cbase + (uint64_t)e;
        const double2 cur = pre[e];
        const double2 prv = e > 0 ? pre[e - 1] : ex;
        const double gN = gamma_bound(N);
        const double SLoN = __dsub_rd(Lo_N, __dmul_ru(gN, Hi_N));
        const double SHiN = __dadd_ru(Hi_N, __dmul_ru(gN, Hi_N));
        // u = fl(r * S_N) lies between the directed roundings of r * S_N.
        const double ULo = __dmul_rd(r, SLoN);
        const double UHi = __dmul_ru(r, SHiN);
        const double gi = gamma_bound(istar + 1);
        const double SLoI = __dsub_rd(cur.x, __dmul_ru(gi, cur.y));
        bool ok = UHi < SLoI;
        if (istar > 0) {
          const double gp = gamma_bound(istar);
          const double SHiP = __dadd_ru(prv.y, __dmul_ru(gp, prv.y));
          ok = ok && (ULo >= SHiP);
        }
        if (ok) { sh_idx = istar; sh_decided = 1; }
      }
    }
  }
  __syncthreads();

  // 4. undecided: the reference's sequential chain, verbatim.
  if (!sh_decided) {
    double total = 0.0;
    uint64_t last_pos = 0;
    for (uint64_t t0 = 0; t0 < N; t0 += 4096) {
      const uint32_t n = (uint32_t)min((uint64_t)4096, N - t0);
      for (uint32_t e = tid; e < n; e += kSelectThreads) tile[e] = w[t0 + e];
      __syncthreads();
      if (tid == 0)
        for (uint32_t e = 0; e < n; ++e) {
          total = __dadd_rn(total, (double)tile[e]);
          if (tile[e] != 0.f) last_pos = t0 + e;
        }
      __syncthreads();
    }
    if (tid == 0) { sh_u = __dmul_rn(r, total); sh_idx = last_pos; }
    __syncthreads();
    const double u = sh_u;
    double cum = 0.0;
    for (uint64_t t0 = 0; t0 < N; t0 += 4096) {
      const uint32_t n = (uint32_t)min((uint64_t)4096, N - t0);
      for (uint32_t e = tid; e < n; e += kSelectThreads) tile[e] = w[t0 + e];
      __syncthreads();
      if (tid == 0 && !sh_decided)
        for (uint32_t e = 0; e < n; ++e) {
          cum = __dadd_rn(cum, (double)tile[e]);
          if (u < cum) { sh_idx = t0 + e; sh_decided = 1; break; }
        }
      __syncthreads();
      if (sh_decided) break;
    }
    if (tid == 0) fallbacks[m] += 1;
  }
  __syncthreads();
  const uint64_t idx = sh_idx;
  if (tid < S) cb[((size_t)m * K + step) * S + tid] = R[idx * (uint64_t)D + (uint64_t)m * S + tid];
  if (tid == 0) chosen[(size_t)m * K + step] = idx;
}

// Degenerate k >= n (kmeans.zig:88-104): every row is its own centroid,
// the remaining slots copy the last row.
__global__ void pq_degenerate_kernel(const float* __restrict__ R, uint64_t N, int D, int S, int K,
                                     float* __restrict__ cb) {
  const int m = blockIdx.x;
  for (int e = threadIdx.x; e < K * S; e += blockDim.x) {
    const int c = e / S, k = e % S;
    const uint64_t row = (uint64_t)c < N ? (uint64_t)c : N - 1;
    cb[((size_t)m * K + c) * S + k] = R[row * (uint64_t)D + (uint64_t)m * S + k];
  }
}

__global__ void u8_to_u32_kernel(const uint8_t* __restrict__ a, uint32_t* __restrict__ b, uint64_t n) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    b[i] = a[i];
}

__global__ void iota_u32_kernel(uint32_t* __restrict__ b, uint64_t N, int M) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < N * (uint64_t)M;
       i += (uint64_t)gridDim.x * blockDim.x)
    b[i] = (uint32_t)(i % N);
}

template <int S>
size_t assign_smem(int M, int K, int mode) {
  const size_t kp = (size_t)(K + 1) / 2;
  size_t b = (size_t)M * kp * S * sizeof(float2);
  if (mode == kModeLloyd) b += (size_t)M * K * sizeof(uint32_t);
  return b;
}

template <int S>
int launch_assign(Ctx* ctx, cudaStream_t st, int mode, const float* R, uint64_t N, int D, int M, int K,
                  const float* cb, uint8_t* codes, uint8_t* asg, float* mind,
                  uint32_t* hist, const uint8_t* state, int nblk) {
  const size_t sm = assign_smem<S>(M, K, mode);
  if (mode == kModeLloyd) {
    auto kern = pq_assign_kernel<S, kModeLloyd>;
    MVR_CUDA(ctx, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
    kern<<<nblk, kThreads, sm, st>>>(R, N, D, M, K, cb, codes, asg, mind, hist, state, 1.0f);
  } else {
    auto kern = pq_assign_kernel<S, kModeEncode>;
    MVR_CUDA(ctx, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
    kern<<<nblk, kThreads, sm, st>>>(R, N, D, M, K, cb, codes, asg, mind, hist, state, 1.0f);
  }
  MVR_CUDA(ctx, cudaGetLastError());
  return MVR_OK;
}

template <int S>
int launch_chain(Ctx* ctx, cudaStream_t st, const float* sorted, uint64_t N, int M, int K,
                 const uint32_t* counts, const uint32_t* starts, float* cb, const uint8_t* state) {
  const size_t sm = (size_t)kChainStages * 32 * (kChainCh + 1) * S * sizeof(float);
  auto kern = pq_chain_kernel<S>;
  MVR_CUDA(ctx, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
  const int grid = M * ((K + 31) / 32);
  kern<<<grid, 32, sm, st>>>(sorted, N, K, counts, starts, cb, state);
  MVR_CUDA(ctx, cudaGetLastError());
  return MVR_OK;
}

int check_shape(Ctx* ctx, int D, int M, int S, int K) {
  if (M <= 0 || S <= 0 || D != M * S) return fail(ctx, MVR_E_INVALID_ARGUMENT, "D must equal M*S");
  if (S != 1 && S != 2 && S != 4)
    return fail(ctx, MVR_E_INVALID_ARGUMENT, "sub-vector length must be 1, 2 or 4");
  if (K <= 0 || K > 256) return fail(ctx, MVR_E_INVALID_ARGUMENT, "K must be in [1, 256]");
  const size_t sm = (size_t)M * ((K + 1) / 2) * S * sizeof(float2) + (size_t)M * K * 4;
  if (sm > 200 * 1024) return fail(ctx, MVR_E_INVALID_ARGUMENT, "codebooks exceed shared memory");
  return MVR_OK;
}

}  // namespace

int pq_encode_device(Ctx* ctx, const float* d_cb, int D, int M, const float* d_R, uint64_t N,
                     uint8_t* d_codes) {
  if (N == 0) return MVR_OK;
  const int S = D / M;
  MVR_TRY(check_shape(ctx, D, M, S, 256));
  const int nblk = (int)((N + kTile - 1) / kTile);
  switch (S) {
    case 1: return launch_assign<1>(ctx, ctx->stream, kModeEncode, d_R, N, D, M, 256, d_cb, d_codes, nullptr, nullptr, nullptr, nullptr, nblk);
    case 2: return launch_assign<2>(ctx, ctx->stream, kModeEncode, d_R, N, D, M, 256, d_cb, d_codes, nullptr, nullptr, nullptr, nullptr, nblk);
    default: return launch_assign<4>(ctx, ctx->stream, kModeEncode, d_R, N, D, M, 256, d_cb, d_codes, nullptr, nullptr, nullptr, nullptr, nblk);
  }
}

PqLayout pq_layout(uint64_t N, int M, int S, int K) {
  PqLayout L;
  L.nblk = (int)((N + kTile - 1) / kTile);
  L.nchunk = (int)((N + kSeedChunk - 1) / kSeedChunk);
  size_t off = 0;
  auto carve = [&](size_t bytes) {
    const size_t o = off;
    off = (off + bytes + 255) & ~(size_t)255;
    return o;
  };
  // host-mirrored bookkeeping first, so one copy moves it both ways
  L.o_draws = carve((size_t)M * K * 8);
  L.o_chosen = carve((size_t)M * K * 8);
  L.o_idx0 = carve((size_t)M * 8);
  L.o_counts = carve((size_t)M * K * 4);
  L.o_starts = carve((size_t)M * K * 4);
  L.o_wcss = carve((size_t)M * 4);
  L.o_prev = carve((size_t)M * 4);
  L.o_status = carve((size_t)M * 4);
  L.o_nonf = carve((size_t)M * 4);
  L.o_iters = carve((size_t)M * 4);
  L.o_fb = carve((size_t)M * 4);
  L.o_rs = carve((size_t)M * 4);
  L.o_state = carve((size_t)M);
  L.small_bytes = off;
  L.o_mind = carve((size_t)M * N * sizeof(float));
  L.o_asg = carve((size_t)M * N);
  L.o_sorted = carve((size_t)M * N * S * sizeof(float));
  L.o_hist = carve((size_t)M * L.nblk * K * sizeof(uint32_t));
  L.o_chunk = carve((size_t)M * L.nchunk * sizeof(double2));
  L.total_bytes = off;
  return L;
}

int pq_kmeans_run(Ctx* ctx, cudaStream_t st, const PqJob& job, const PqOut& out, unsigned char* ws,
                  unsigned char* hsmall) {
  const uint64_t N = job.N;
  const int D = job.D, M = job.M, S = job.S, K = job.K;
  MVR_TRY(check_shape(ctx, D, M, S, K));
  if (N == 0) return fail(ctx, MVR_E_EMPTY_VECTOR_SET, "no rows");
  if (N >= (1ull << 32)) return fail(ctx, MVR_E_INVALID_ARGUMENT, "more than 2^32-1 rows per subspace");
  const bool timing = out.stats != nullptr && ctx != nullptr;
  if (timing) {
    for (int e = 0; e < 4; ++e)
      if (!ctx->ev[e]) MVR_CUDA(ctx, cudaEventCreate(&ctx->ev[e]));
    MVR_CUDA(ctx, cudaEventRecord(ctx->ev[0], st));
  }

  // ---- degenerate k >= n -------------------------------------------------
  if ((uint64_t)K >= N) {
    pq_degenerate_kernel<<<M, 256, 0, st>>>(job.R, N, D, S, K, out.d_codebooks);
    MVR_CUDA(ctx, cudaGetLastError());
    if (out.d_assign) {
      iota_u32_kernel<<<256, 256, 0, st>>>(out.d_assign, N, M);
      MVR_CUDA(ctx, cudaGetLastError());
    }
    MVR_CUDA(ctx, cudaStreamSynchronize(st));
    for (int m = 0; m < M; ++m) {
      if (out.h_wcss) out.h_wcss[m] = 0.f;
      if (out.h_iters) out.h_iters[m] = 0;
    }
    if (out.stats) std::memset(out.stats, 0, sizeof(*out.stats));
    return MVR_OK;
  }

  const PqLayout L = pq_layout(N, M, S, K);
  const int nblk = L.nblk, nchunk = L.nchunk;
  float* mind = (float*)(ws + L.o_mind);
  uint8_t* asg = (uint8_t*)(ws + L.o_asg);
  float* sorted = (float*)(ws + L.o_sorted);
  uint32_t* hist = (uint32_t*)(ws + L.o_hist);
  double2* chunk = (double2*)(ws + L.o_chunk);
  unsigned char* small = ws;  // bookkeeping lives at the start of the workspace
  const size_t small_bytes = L.small_bytes;
  double* d_draws = (double*)(small + L.o_draws);
  uint64_t* d_chosen = (uint64_t*)(small + L.o_chosen);
  uint64_t* d_idx0 = (uint64_t*)(small + L.o_idx0);
  uint32_t* d_counts = (uint32_t*)(small + L.o_counts);
  uint32_t* d_starts = (uint32_t*)(small + L.o_starts);
  float* d_wcss = (float*)(small + L.o_wcss);
  float* d_prev = (float*)(small + L.o_prev);
  int* d_status = (int*)(small + L.o_status);
  int* d_nonf = (int*)(small + L.o_nonf);
  uint32_t* d_iters = (uint32_t*)(small + L.o_iters);
  uint32_t* d_fb = (uint32_t*)(small + L.o_fb);
  uint32_t* d_rs = (uint32_t*)(small + L.o_rs);
  uint8_t* d_state = (uint8_t*)(small + L.o_state);

  // ---- host RNG draws (data independent); the rest of the bookkeeping
  // starts at zero (state = running, counters = 0) -------------------------
  std::memset(hsmall, 0, small_bytes);
  {
    double* hd = (double*)(hsmall + L.o_draws);
    uint64_t* hi0 = (uint64_t*)(hsmall + L.o_idx0);
    for (int m = 0; m < M; ++m) {
      Xoshiro256pp rng(job.seed + (uint64_t)m);
      hi0[m] = rng.below(N);
      hd[(size_t)m * K] = 0.0;
      for (int c = 1; c < K; ++c) hd[(size_t)m * K + c] = rng.unit_f64();
    }
  }
  MVR_CUDA(ctx, cudaMemcpyAsync(small, hsmall, small_bytes, cudaMemcpyHostToDevice, st));

  float* cb = out.d_codebooks;
  pq_seed_init_kernel<<<M, 32, 0, st>>>(job.R, D, S, K, d_idx0, cb, d_chosen);
  MVR_CUDA(ctx, cudaGetLastError());
  for (int step = 0; step + 1 < K; ++step) {
    switch (S) {
      case 1: pq_seed_update_kernel<1><<<nchunk, kThreads, 0, st>>>(job.R, N, D, M, K, step, cb, mind, chunk, d_nonf, d_state); break;
      case 2: pq_seed_update_kernel<2><<<nchunk, kThreads, 0, st>>>(job.R, N, D, M, K, step, cb, mind, chunk, d_nonf, d_state); break;
      default: pq_seed_update_kernel<4><<<nchunk, kThreads, 0, st>>>(job.R, N, D, M, K, step, cb, mind, chunk, d_nonf, d_state); break;
    }
    MVR_CUDA(ctx, cudaGetLastError());
    pq_seed_select_kernel<<<M, kSelectThreads, 0, st>>>(job.R, N, D, S, K, step + 1, cb, mind, chunk, nchunk,
                                                        d_draws, d_nonf, d_status, d_state, d_fb, d_chosen);
    MVR_CUDA(ctx, cudaGetLastError());
  }
  if (timing) MVR_CUDA(ctx, cudaEventRecord(ctx->ev[1], st));

  // ---- Lloyd iterations ---------------------------------------------------
  const bool check = !(job.tol == -INFINITY) && !std::isnan(job.tol);
  uint32_t launches = 1 + 2 * (uint32_t)(K - 1);
  std::vector<cudaEvent_t> aev;  // assignment-kernel brackets (stats only)
  if (timing) {
    aev.resize(2 * (size_t)job.max_iters, nullptr);
    for (auto& e : aev) MVR_CUDA(ctx, cudaEventCreate(&e));
  }
  struct EvGuard {
    std::vector<cudaEvent_t>& v;
    ~EvGuard() {
      for (auto e : v)
        if (e) cudaEventDestroy(e);
    }
  } ev_guard{aev};
  for (uint32_t it = 0; it < job.max_iters; ++it) {
    if (timing) MVR_CUDA(ctx, cudaEventRecord(aev[2 * it], st));
    switch (S) {
      case 1: MVR_TRY(launch_assign<1>(ctx, st, kModeLloyd, job.R, N, D, M, K, cb, nullptr, asg, mind, hist, d_state, nblk)); break;
      case 2: MVR_TRY(launch_assign<2>(ctx, st, kModeLloyd, job.R, N, D, M, K, cb, nullptr, asg, mind, hist, d_state, nblk)); break;
      default: MVR_TRY(launch_assign<4>(ctx, st, kModeLloyd, job.R, N, D, M, K, cb, nullptr, asg, mind, hist, d_state, nblk)); break;
    }
    if (timing) MVR_CUDA(ctx, cudaEventRecord(aev[2 * it + 1], st));
    launches += 5;
    const bool last = it + 1 == job.max_iters;
    if (check || (last && out.h_wcss)) {
      pq_wcss_kernel<<<M, 256, 0, st>>>(mind, N, d_wcss, d_state);
      MVR_CUDA(ctx, cudaGetLastError());
      ++launches;
    }
    pq_scan_kernel<<<M, 256, 0, st>>>(hist, nblk, K, d_counts, d_starts, d_state);
    MVR_CUDA(ctx, cudaGetLastError());
    switch (S) {
      case 1: pq_scatter_kernel<1><<<nblk, kThreads, 0, st>>>(job.R, N, D, M, K, asg, hist, sorted, d_state); break;
      case 2: pq_scatter_kernel<2><<<nblk, kThreads, 0, st>>>(job.R, N, D, M, K, asg, hist, sorted, d_state); break;
      default: pq_scatter_kernel<4><<<nblk, kThreads, 0, st>>>(job.R, N, D, M, K, asg, hist, sorted, d_state); break;
    }
    MVR_CUDA(ctx, cudaGetLastError());
    switch (S) {
      case 1: MVR_TRY(launch_chain<1>(ctx, st, sorted, N, M, K, d_counts, d_starts, cb, d_state)); break;
      case 2: MVR_TRY(launch_chain<2>(ctx, st, sorted, N, M, K, d_counts, d_starts, cb, d_state)); break;
      default: MVR_TRY(launch_chain<4>(ctx, st, sorted, N, M, K, d_counts, d_starts, cb, d_state)); break;
    }
    pq_reseed_converge_kernel<<<M, 1024, 0, st>>>(job.R, N, D, S, K, d_counts, mind, cb, d_state, d_wcss,
                                                  d_prev, d_iters, d_rs, (int)it, check ? 1 : 0, job.tol);
    MVR_CUDA(ctx, cudaGetLastError());
  }
  if (timing) MVR_CUDA(ctx, cudaEventRecord(ctx->ev[2], st));
  if (out.d_assign && job.max_iters > 0) {
    // Converged subspaces keep the assignments of their last iteration,
    // which later iterations did not touch.
    u8_to_u32_kernel<<<1024, 256, 0, st>>>(asg, out.d_assign, (uint64_t)M * N);
    MVR_CUDA(ctx, cudaGetLastError());
    ++launches;
  }
  MVR_CUDA(ctx, cudaMemcpyAsync(hsmall, small, small_bytes, cudaMemcpyDeviceToHost, st));
  MVR_CUDA(ctx, cudaStreamSynchronize(st));

  const int* hstatus = (const int*)(hsmall + L.o_status);
  for (int m = 0; m < M; ++m)
    if (hstatus[m] != MVR_OK)
      return fail(ctx, hstatus[m], std::string("subspace ") + std::to_string(m) + ": " + mvr_status_name(hstatus[m]));
  const uint32_t* hiters = (const uint32_t*)(hsmall + L.o_iters);
  const float* hw = (const float*)(hsmall + L.o_wcss);
  if (out.h_iters)
    for (int m = 0; m < M; ++m) out.h_iters[m] = job.max_iters ? hiters[m] : 0;
  if (out.h_wcss)
    for (int m = 0; m < M; ++m) out.h_wcss[m] = job.max_iters ? hw[m] : 0.f;
  if (out.stats) {
    std::memset(out.stats, 0, sizeof(*out.stats));
    if (timing) {
      float t01 = 0, t12 = 0, t02 = 0;
      cudaEventElapsedTime(&t01, ctx->ev[0], ctx->ev[1]);
      cudaEventElapsedTime(&t12, ctx->ev[1], ctx->ev[2]);
      cudaEventElapsedTime(&t02, ctx->ev[0], ctx->ev[2]);
      out.stats->seed_ms = t01;
      out.stats->lloyd_ms = t12;
      out.stats->total_ms = t02;
      double am = 0.0;
      for (uint32_t it = 0; it < job.max_iters; ++it) {
        float t = 0.f;
        cudaEventElapsedTime(&t, aev[2 * it], aev[2 * it + 1]);
        am += t;
      }
      out.stats->assign_ms = am;
      out.stats->assign_launches = job.max_iters;
    }
    uint32_t mx = 0, mn = UINT32_MAX, fb = 0, rs = 0;
    const uint32_t* hfb = (const uint32_t*)(hsmall + L.o_fb);
    const uint32_t* hrs = (const uint32_t*)(hsmall + L.o_rs);
    for (int m = 0; m < M; ++m) {
      const uint32_t v = job.max_iters ? hiters[m] : 0;
      mx = std::max(mx, v);
      mn = std::min(mn, v);
      fb += hfb[m];
      rs += hrs[m];
    }
    out.stats->iters_max = mx;
    out.stats->iters_min = mn;
    out.stats->seed_fallbacks = fb;
    out.stats->reseeds = rs;
    out.stats->launches = launches;
  }
  return MVR_OK;
}

int pq_kmeans_device(Ctx* ctx, const PqJob& job, const PqOut& out) {
  MVR_TRY(check_shape(ctx, job.D, job.M, job.S, job.K));
  const PqLayout L = pq_layout(job.N, job.M, job.S, job.K);
  unsigned char* ws = nullptr;
  MVR_TRY(scratch(ctx, kSlotMinDist, L.total_bytes, (void**)&ws));
  std::vector<unsigned char> hsmall(L.small_bytes);
  return pq_kmeans_run(ctx, ctx->stream, job, out, ws, hsmall.data());
}

}  // namespace mvr
