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
//   R        [N][D]      caller's rows (read by the transpose and by encode)
//   XT       [M][N][S]   subspace-major copy of R: every per-subspace pass
//                        reads 32 consecutive rows as one contiguous segment
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
//     rigorously (directed-rounding partial sums plus an error bound on the
//     sequential chain); a draw whose outcome the bound cannot decide is
//     recomputed with the exact sequential chain on the device.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "mvr_device.cuh"
#include "mvr_rng.h"
#include "tc_filter.cuh"
#include "pq_engine.h"
#include "comm.h"

namespace mvr {
namespace {

// Sequential 256-byte-aligned carving of a workspace.
struct Carve {
  size_t off = 0;
  size_t take(size_t bytes) {
    const size_t o = off;
    off = (off + bytes + 255) & ~(size_t)255;
    return o;
  }
};

constexpr int kAsgThreads = 512;            // assign / encode CTA size
constexpr int kPtsPerThread = 2;            // rows per thread per assign pass
constexpr int kAsgTile = kAsgThreads * kPtsPerThread;
constexpr int kSeedThreads = 256;
constexpr int kSeedRowsPerThread = 4;
constexpr int kSeedChunk = kSeedThreads * kSeedRowsPerThread;  // rows per chunk
constexpr int kSelectThreads = 1024;
static_assert(kSelectThreads == kSeedChunk, "the fine search maps one thread to one row");
constexpr int kChainWarps = 4;              // warps per chain CTA
constexpr int kChainE = 128;                // elements per cluster per ring stage
constexpr int kChainStages = 3;
constexpr int kMaxM = 32;                   // subspaces per call (scatter: one warp each)
constexpr int kCrossingSlack = 300;         // binade crossings of a monotone f64 sum

enum : uint8_t { kRunning = 0, kDone = 1, kFailed = 2 };
enum { kModeEncode = 0, kModeLloyd = 1 };

template <int S>
__device__ __forceinline__ void load_sub(const float* __restrict__ p, float (&x)[S]) {
  if constexpr (S == 4) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(p));
    x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
  } else if constexpr (S == 2) {
    const float2 v = __ldg(reinterpret_cast<const float2*>(p));
    x[0] = v.x; x[1] = v.y;
  } else {
    x[0] = __ldg(p);
  }
}

template <int S>
__device__ __forceinline__ void load_sub_unaligned(const float* __restrict__ p, float (&x)[S]) {
#pragma unroll
  for (int k = 0; k < S; ++k) x[k] = __ldg(p + k);
}

// ---------------------------------------------------------------------------
// XT[m][r][:] = R[r][m*S : m*S+S]
// ---------------------------------------------------------------------------
template <int S>
__global__ void __launch_bounds__(256)
pq_transpose_kernel(const float* __restrict__ R, uint64_t N, int D, int M, float* __restrict__ XT) {
  for (uint64_t r = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; r < N;
       r += (uint64_t)gridDim.x * blockDim.x) {
    const float* row = R + r * (uint64_t)D;
    for (int m = 0; m < M; ++m) {
      float x[S];
      load_sub_unaligned<S>(row + m * S, x);
      float* o = XT + ((size_t)m * N + r) * S;
      if constexpr (S == 4) {
        *reinterpret_cast<float4*>(o) = make_float4(x[0], x[1], x[2], x[3]);
      } else if constexpr (S == 2) {
        *reinterpret_cast<float2*>(o) = make_float2(x[0], x[1]);
      } else {
        o[0] = x[0];
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Exact Hamerly bounds for the Lloyd assignment. An f32 distance of an
// S <= 4 sub-vector is within (1 +- g) of the exact squared distance,
// g = 2^-21 (at most six roundings of 2^-24 each touch any term). From the
// winner's distance `best` and the runner-up's `sec`:
//   ub = sqrt(best) / sqrt(1 - g)  >= the exact distance to the winner,
//   lb = sqrt(sec)  / sqrt(1 + g)  <= the exact distance to every other,
// rounded outwards. After a centroid update with drifts d_c (rounded up),
// ub += d_a and lb -= max_c d_c keep both true (triangle inequality). When
// ub * (1 + 2^-18) < lb and lb >= 2^-60, the winner's f32 distance is
// strictly below every other f32 distance (the factor covers
// sqrt((1+g)/(1-g)) and leaves an absolute margin far above subnormal
// rounding), so the reference's first-index argmin is still the winner and
// the row's distances need not be computed.
// ---------------------------------------------------------------------------
constexpr float kUbScale = 1.0f + 0x1p-21f;      // >= 1 / sqrt(1 - 2^-21)
constexpr float kLbScale = 1.0f - 0x1p-21f;      // <= 1 / sqrt(1 + 2^-21)
constexpr float kPruneMargin = 1.0f + 0x1p-18f;
constexpr float kLbMin = 0x1p-60f;

__device__ __forceinline__ float bound_upper(float best) { return __fmul_ru(__fsqrt_ru(best), kUbScale); }
__device__ __forceinline__ float bound_lower(float sec) { return __fmul_rd(__fsqrt_rd(sec), kLbScale); }

// ---------------------------------------------------------------------------
// Assignment / encode. Persistent CTAs: CTA b owns rows
// [b*rows_per_cta, (b+1)*rows_per_cta), processed kAsgTile at a time, one
// thread per kPtsPerThread rows across all M subspaces. The M codebooks sit
// in shared memory as negated centroid pairs so that two distances come out
// of each packed f32x2 instruction. Lloyd mode reads XT and writes
// assignments, min distances and the CTA's cluster histogram; encode mode
// reads R and writes codes.
// ---------------------------------------------------------------------------
template <int S, int MODE, bool BOUNDS>
__global__ void __launch_bounds__(kAsgThreads, 2)
pq_assign_kernel(const float* __restrict__ R, const float* __restrict__ XT, uint64_t N, int D,
                 int M, int K, const float* __restrict__ cb, uint8_t* __restrict__ codes,
                 uint8_t* __restrict__ asg, float* __restrict__ mind, uint32_t* __restrict__ hist,
                 const uint8_t* __restrict__ state, float one, uint64_t rows_per_cta,
                 float* __restrict__ ubnd, float* __restrict__ lbnd) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int KP = (K + 1) >> 1;
  float2* cbp = reinterpret_cast<float2*>(smem_raw);  // [M][KP][S]
  uint32_t* h = reinterpret_cast<uint32_t*>(cbp + (size_t)M * KP * S);  // [M][K]

  for (int e = threadIdx.x; e < M * KP * S; e += kAsgThreads) {
    const int k = e % S;
    const int p = (e / S) % KP;
    const int m = e / (S * KP);
    const int ca = 2 * p, cbi = 2 * p + 1;
    const float a = cb[((size_t)m * K + ca) * S + k];
    const float b = cbi < K ? cb[((size_t)m * K + cbi) * S + k] : f32_nan();
    cbp[e] = make_float2(-a, -b);  // a NaN pad never wins a strict '<'
  }
  if (MODE == kModeLloyd && hist)
    for (int e = threadIdx.x; e < M * K; e += kAsgThreads) h[e] = 0;
  __syncthreads();

  const float2 one2 = make_float2(one, one);  // 1.0f, opaque to the compiler
  const uint64_t lo = (uint64_t)blockIdx.x * rows_per_cta;
  const uint64_t hi = min(N, lo + rows_per_cta);
  for (uint64_t base = lo; base < hi; base += kAsgTile) {
    uint64_t row[kPtsPerThread];
    bool ok[kPtsPerThread];
#pragma unroll
    for (int j = 0; j < kPtsPerThread; ++j) {
      row[j] = base + (uint64_t)j * kAsgThreads + threadIdx.x;
      ok[j] = row[j] < hi;
    }
    // Tail of the CTA's range: whole warps without rows skip the tile.
    if (!__any_sync(0xffffffffu, ok[0] || ok[kPtsPerThread - 1])) continue;
    uint32_t packed[kPtsPerThread] = {0u};
    for (int m = 0; m < M; ++m) {
      if (MODE == kModeLloyd && state[m] != kRunning) continue;
      float2 xx[kPtsPerThread][S];
#pragma unroll
      for (int j = 0; j < kPtsPerThread; ++j) {
        float x[S];
        if (ok[j]) {
          if (MODE == kModeLloyd)
            load_sub<S>(XT + ((size_t)m * N + row[j]) * S, x);
          else
            load_sub_unaligned<S>(R + row[j] * (uint64_t)D + (uint64_t)m * S, x);
        } else {
#pragma unroll
          for (int k = 0; k < S; ++k) x[k] = 0.f;
        }
#pragma unroll
        for (int k = 0; k < S; ++k) xx[j][k] = make_float2(x[k], x[k]);
      }
      float best[kPtsPerThread], d0[kPtsPerThread], sec[kPtsPerThread];
      int bi[kPtsPerThread];
#pragma unroll
      for (int j = 0; j < kPtsPerThread; ++j) {
        best[j] = __int_as_float(0x7f800000);
        sec[j] = __int_as_float(0x7f800000);
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
          if (BOUNDS) {  // also the second smallest distance (a tie makes it equal the best)
            if (dd.x < best[j]) { sec[j] = best[j]; best[j] = dd.x; bi[j] = 2 * p; } else { sec[j] = fminf(sec[j], dd.x); }
            if (dd.y < best[j]) { sec[j] = best[j]; best[j] = dd.y; bi[j] = 2 * p + 1; } else { sec[j] = fminf(sec[j], dd.y); }
          } else {
            if (dd.x < best[j]) { best[j] = dd.x; bi[j] = 2 * p; }
            if (dd.y < best[j]) { best[j] = dd.y; bi[j] = 2 * p + 1; }
          }
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
            if (hist) atomicAdd(&h[m * K + bi[j]], 1u);
            if (BOUNDS) {
              ubnd[(size_t)m * N + row[j]] = bound_upper(best[j]);
              lbnd[(size_t)m * N + row[j]] = isnan(d0[j]) ? -__int_as_float(0x7f800000) : bound_lower(sec[j]);
            }
          }
        } else if (ok[j]) {
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
  if (MODE == kModeLloyd && hist) {  // per-CTA histograms (the row-sharded path's scatter)
    __syncthreads();
    const int nblk = gridDim.x;
    for (int e = threadIdx.x; e < M * K; e += kAsgThreads) {
      const int m = e / K, c = e % K;
      hist[((size_t)m * nblk + blockIdx.x) * K + c] = h[e];
    }
  }
}

// ---------------------------------------------------------------------------
// Pruned Lloyd iterations (after the first): drift of every centroid, a check
// pass that keeps rows whose bounds prove the winner unchanged and lists the
// others per subspace, a dense pass over the lists, and the per-CTA cluster
// histograms of all rows for the stable sort.
// ---------------------------------------------------------------------------
// drift[m][c] >= |c_new - c_old| (exact Euclidean, rounded up). maxd[m] =
// (largest drift, its centroid, second largest) as floats: a row's lower
// bound drops by the largest drift among the centroids other than its own.
__global__ void __launch_bounds__(256)
pq_drift_kernel(const float* __restrict__ cb_old, const float* __restrict__ cb, int M, int K, int S,
                const uint8_t* __restrict__ state, float* __restrict__ drift, float* __restrict__ maxd) {
  const int m = blockIdx.x;
  if (state[m] != kRunning) return;
  __shared__ float sd[256];
  for (int c = threadIdx.x; c < 256; c += blockDim.x) sd[c] = 0.f;
  __syncthreads();
  for (int c = threadIdx.x; c < K; c += blockDim.x) {
    double d2 = 0.0;
    for (int k = 0; k < S; ++k) {
      const double a = cb[((size_t)m * K + c) * S + k], b = cb_old[((size_t)m * K + c) * S + k];
      const double hi = __dsub_ru(a, b), lo = __dsub_rd(a, b);
      const double t = fmax(fabs(hi), fabs(lo));  // >= |a - b|
      d2 = __dadd_ru(d2, __dmul_ru(t, t));
    }
    const float d = __double2float_ru(__dsqrt_ru(d2));
    drift[(size_t)m * K + c] = d;
    sd[c] = d;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float m1 = 0.f, m2 = 0.f;
    int i1 = -1;
    for (int c = 0; c < K; ++c) {
      const float d = sd[c];
      if (d > m1) { m2 = m1; m1 = d; i1 = c; } else if (d > m2) { m2 = d; }
    }
    maxd[3 * m] = m1;
    maxd[3 * m + 1] = (float)i1;
    maxd[3 * m + 2] = m2;
  }
}

// Row r of subspace m (blockIdx.y): bounds moved by the drifts; a row whose
// bounds still prove its winner keeps it (and, if need_mind, gets its f32
// distance to it); every other row is appended to list[m]. One atomic per
// CTA pass reserves the pass's list segment (warp offsets from a block scan).
template <int S>
__global__ void __launch_bounds__(256)
pq_prune_check_kernel(const float* __restrict__ XT, uint64_t N, int K, const float* __restrict__ cb,
                      const uint8_t* __restrict__ asg, float* __restrict__ ubnd, float* __restrict__ lbnd,
                      const float* __restrict__ drift, const float* __restrict__ maxd,
                      const uint8_t* __restrict__ state, uint32_t* __restrict__ list,
                      uint32_t* __restrict__ list_cnt, float* __restrict__ mind, int need_mind) {
  __shared__ uint32_t wcnt[8], wbase[8], bbase;
  const int m = blockIdx.y;
  if (state[m] != kRunning) return;
  const float md1 = maxd[3 * m], md2 = maxd[3 * m + 2];
  const uint32_t mi1 = (uint32_t)(int)maxd[3 * m + 1];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t base = (uint64_t)blockIdx.x * blockDim.x; base < N; base += stride) {
    const uint64_t r = base + threadIdx.x;
    const bool ok = r < N;
    bool keep = false;
    if (ok) {
      const size_t e = (size_t)m * N + r;
      const uint32_t a = asg[e];
      const float u = __fadd_ru(ubnd[e], drift[(size_t)m * K + a]);
      const float l = __fsub_rd(lbnd[e], a == mi1 ? md2 : md1);
      keep = l >= kLbMin && __fmul_ru(u, kPruneMargin) < l;
      if (keep) {
        ubnd[e] = u;
        lbnd[e] = l;
        if (need_mind) {
          float x[S], c[S];
          load_sub<S>(XT + e * S, x);
#pragma unroll
          for (int k = 0; k < S; ++k) c[k] = cb[((size_t)m * K + a) * S + k];
          mind[e] = l2_small<S>(x, c);
        }
      } else if (l >= kLbMin) {
        // the drifts loosened ub: one exact distance to the winner tightens it
        float x[S], c[S];
        load_sub<S>(XT + e * S, x);
#pragma unroll
        for (int k = 0; k < S; ++k) c[k] = cb[((size_t)m * K + a) * S + k];
        const float da = l2_small<S>(x, c);
        const float ut = bound_upper(da);
        if (__fmul_ru(ut, kPruneMargin) < l) {
          keep = true;
          ubnd[e] = ut;
          lbnd[e] = l;
          mind[e] = da;
        }
      }
    }
    const uint32_t need = __ballot_sync(0xffffffffu, ok && !keep);
    if (lane == 0) wcnt[warp] = (uint32_t)__popc(need);
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t t = 0;
      for (int w = 0; w < 8; ++w) {
        wbase[w] = t;
        t += wcnt[w];
      }
      bbase = t ? atomicAdd(&list_cnt[m], t) : 0u;
    }
    __syncthreads();
    if (ok && !keep) list[(size_t)m * N + bbase + wbase[warp] + __popc(need & lanemask_lt())] = (uint32_t)r;
    __syncthreads();  // wcnt / wbase / bbase are reused by the next pass
  }
}

// Dense assignment of the listed rows: work units of kAsgTile rows of one
// subspace (all M codebooks in shared memory, as in pq_assign_kernel).
template <int S>
__global__ void __launch_bounds__(kAsgThreads, 2)
pq_assign_list_kernel(const float* __restrict__ XT, uint64_t N, int M, int K, const float* __restrict__ cb,
                      const uint32_t* __restrict__ list, const uint32_t* __restrict__ list_cnt,
                      uint8_t* __restrict__ asg, float* __restrict__ mind, float* __restrict__ ubnd,
                      float* __restrict__ lbnd, const uint8_t* __restrict__ state, float one) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ uint32_t upre[kMaxM + 1];
  const int KP = (K + 1) >> 1;
  float2* cbp = reinterpret_cast<float2*>(smem_raw);  // [M][KP][S]
  for (int e = threadIdx.x; e < M * KP * S; e += kAsgThreads) {
    const int k = e % S;
    const int p = (e / S) % KP;
    const int m = e / (S * KP);
    const int ca = 2 * p, cbi = 2 * p + 1;
    const float a = cb[((size_t)m * K + ca) * S + k];
    const float b = cbi < K ? cb[((size_t)m * K + cbi) * S + k] : f32_nan();
    cbp[e] = make_float2(-a, -b);
  }
  if (threadIdx.x == 0) {
    uint32_t acc = 0;
    for (int m = 0; m < M; ++m) {
      upre[m] = acc;
      acc += state[m] == kRunning ? (list_cnt[m] + kAsgTile - 1) / kAsgTile : 0u;
    }
    upre[M] = acc;
  }
  __syncthreads();
  const float2 one2 = make_float2(one, one);
  const uint32_t units = upre[M];
  for (uint32_t u = blockIdx.x; u < units; u += gridDim.x) {
    int m = 0;
    while (upre[m + 1] <= u) ++m;
    const uint32_t i0 = (u - upre[m]) * kAsgTile, cnt = list_cnt[m];
    uint64_t row[kPtsPerThread];
    bool ok[kPtsPerThread];
    float2 xx[kPtsPerThread][S];
#pragma unroll
    for (int j = 0; j < kPtsPerThread; ++j) {
      const uint32_t i = i0 + (uint32_t)j * kAsgThreads + threadIdx.x;
      ok[j] = i < cnt;
      row[j] = ok[j] ? list[(size_t)m * N + i] : 0;
      float x[S];
      if (ok[j]) {
        load_sub<S>(XT + ((size_t)m * N + row[j]) * S, x);
      } else {
#pragma unroll
        for (int k = 0; k < S; ++k) x[k] = 0.f;
      }
#pragma unroll
      for (int k = 0; k < S; ++k) xx[j][k] = make_float2(x[k], x[k]);
    }
    if (!__any_sync(0xffffffffu, ok[0] || ok[kPtsPerThread - 1])) continue;
    float best[kPtsPerThread], sec[kPtsPerThread], d0[kPtsPerThread];
    int bi[kPtsPerThread];
#pragma unroll
    for (int j = 0; j < kPtsPerThread; ++j) {
      best[j] = __int_as_float(0x7f800000);
      sec[j] = __int_as_float(0x7f800000);
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
        if (dd.x < best[j]) { sec[j] = best[j]; best[j] = dd.x; bi[j] = 2 * p; } else { sec[j] = fminf(sec[j], dd.x); }
        if (dd.y < best[j]) { sec[j] = best[j]; best[j] = dd.y; bi[j] = 2 * p + 1; } else { sec[j] = fminf(sec[j], dd.y); }
      }
    }
#pragma unroll
    for (int j = 0; j < kPtsPerThread; ++j) {
      if (isnan(d0[j])) { bi[j] = 0; best[j] = d0[j]; }
      if (ok[j]) {
        const size_t e = (size_t)m * N + row[j];
        asg[e] = (uint8_t)bi[j];
        mind[e] = best[j];
        ubnd[e] = bound_upper(best[j]);
        lbnd[e] = isnan(d0[j]) ? -__int_as_float(0x7f800000) : bound_lower(sec[j]);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Candidate-pruned Lloyd pass (iterations >= 1): the bound check above fused
// with a scan of only the centroids near the row's current one.
//
// pq_nbr_kernel lists, for every centroid a, its kCandL nearest other
// centroids in increasing v_j, v_j <= |c_a - c_j| a lower bound (f64 with
// directed rounding), and v_last, the bound of the last one listed. A row x
// whose bounds fail, with current cluster a and ut = bound_upper(f_a) >=
// |x - c_a| (f_a its exact f32 distance to c_a), gets the exact f32
// distances to all listed neighbours. Every centroid c_j off the list has
// v_j >= v_last and |x - c_j| >= |c_a - c_j| - |x - c_a| >= v_last - ut.
// When v_last > T = RU(RU(ut (2 + 2^-18)) + 2^-50), that is
// |x - c_j| > ut (1 + 2^-18) + 2^-50: the exact squared distance D_j exceeds
// D_a (1 + 2^-17) and 2^-100, and since the f32 distances are within
// (1 +- g) of D (g = 2^-21, plus underflow terms below 2^-145), f_j > f_a >=
// f_w for the winner w among the scanned centroids. No centroid off the
// list can be the minimum or tie with it, so the first minimum among a and
// the listed neighbours (smallest index on equal values) is the reference's
// first-index argmin over all K. Otherwise (v_last <= T), or when x, f_a or
// a codeword is not finite, the row gets the full scan of all K in index
// order (a NaN distance to centroid 0 wins, as vec.argmin starts from
// dists[0]). Lower bound for the next iteration: the smaller of
// bound_lower(second smallest scanned distance) and RD(v_last - ut).
//
// Work layout: each warp checks the bounds of 32 rows at a time (one lane
// per row) and appends the rows that need a scan to a warp-private queue in
// shared memory; whenever 32 rows are queued, each lane scans one of them
// through its fixed window of kCandL neighbours (no divergence). Rows that
// need the full scan are then done one at a time by the whole warp (8
// centroids per lane, then a shuffle reduction that keeps the smallest index
// among equal distances). No block barrier
// after the codebook and neighbour table are staged.
// ---------------------------------------------------------------------------
constexpr int kCandThreads = 256;
constexpr int kCandWarps = kCandThreads / 32;
constexpr int kCandL = 32;                       // listed neighbours per centroid
constexpr int kCandH = 16;                       // neighbours scanned before the second-stage test
constexpr int kCandQ = 64;                       // warp queue capacity (< 32 left + 32 new)
constexpr float kCandCut = 2.0f + 0x1p-18f;      // 1 + kPruneMargin
constexpr float kCandFloor = 0x1p-50f;

// Lower bound of |a - b| (f64, a and b floats): 0 when the sign is unsure.
__device__ __forceinline__ double abs_diff_rd(double a, double b) {
  const double lo = __dsub_rd(a, b), hi = __dsub_ru(a, b);
  return lo > 0.0 ? lo : (hi < 0.0 ? -hi : 0.0);
}

// Sort key of neighbour j at lower-bound distance v >= 0: a float no larger
// than v whose low 8 bits hold j (keys order like the values, ties by j).
__device__ __forceinline__ uint32_t nbr_key(float v, int j) {
  const uint32_t b = __float_as_uint(v);
  return (b >= 0x200u ? ((b & ~0xFFu) - 0x100u) : 0u) | (uint32_t)j;
}

// nbr_idx[m][a][0..kCandL): the min(kCandL, K - 1) nearest centroids other
// than a, by increasing key; nbr_last[m][a][0]: the value of the last key
// when kCandL are listed, nbr_last[m][a][1]: the value of key kCandH (the
// first of the list's second half; every later entry's bound is at least
// that). One warp per (m, a); each lane holds 8 candidates
// sorted in registers, rounds of a warp minimum pop them in order.
template <int S>
__global__ void __launch_bounds__(256)
pq_nbr_kernel(const float* __restrict__ cb, int K, const uint8_t* __restrict__ state, uint8_t* __restrict__ nbr_idx,
              float* __restrict__ nbr_last) {
  const int m = blockIdx.y;
  if (state[m] != kRunning) return;
  const int lane = threadIdx.x & 31, a = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (a >= K) return;
  const float* cm = cb + (size_t)m * K * S;
  double ca[S];
#pragma unroll
  for (int k = 0; k < S; ++k) ca[k] = cm[(size_t)a * S + k];
  uint32_t key[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const int j = lane * 8 + q;
    key[q] = 0xFFFFFFFFu;
    if (j < K && j != a) {
      double d2 = 0.0;
#pragma unroll
      for (int k = 0; k < S; ++k) {
        const double t = abs_diff_rd(ca[k], (double)cm[(size_t)j * S + k]);
        d2 = __dadd_rd(d2, __dmul_rd(t, t));
      }
      float v = __double2float_rd(__dsqrt_rd(d2));
      if (!(v >= 0.f)) v = 0.f;  // non-finite codewords: the scan kernel takes full scans
      key[q] = nbr_key(v, j);
    }
  }
#pragma unroll
  for (int i = 1; i < 8; ++i)
#pragma unroll
    for (int k = i; k > 0; --k) {
      const uint32_t lo = min(key[k - 1], key[k]), hi = max(key[k - 1], key[k]);
      key[k - 1] = lo;
      key[k] = hi;
    }
  uint32_t mine = 0xFFFFFFFFu;
  const int L = min(kCandL, K - 1);
  for (int i = 0; i < L; ++i) {
    const uint32_t mn = __reduce_min_sync(0xffffffffu, key[0]);
    if (key[0] == mn) {  // keys are unique (the index is in the low bits): one lane pops
#pragma unroll
      for (int q = 0; q < 7; ++q) key[q] = key[q + 1];
      key[7] = 0xFFFFFFFFu;
    }
    if (lane == i) mine = mn;
  }
  nbr_idx[((size_t)m * K + a) * kCandL + lane] = (uint8_t)(mine & 0xFFu);
  if (lane == L - 1) nbr_last[((size_t)m * K + a) * 2] = __uint_as_float(mine);
  // the bound of the entry that opens the second half of the list (read only
  // when the list is full)
  if (lane == kCandH) nbr_last[((size_t)m * K + a) * 2 + 1] = __uint_as_float(mine);
}

template <int S>
__device__ __forceinline__ void load_centroid(const float* sC, int j, float (&c)[S]) {
  if constexpr (S == 4) {
    const float4 v = reinterpret_cast<const float4*>(sC)[j];
    c[0] = v.x; c[1] = v.y; c[2] = v.z; c[3] = v.w;
  } else {
#pragma unroll
    for (int k = 0; k < S; ++k) c[k] = sC[j * S + k];
  }
}

size_t cand_smem(int K, int S) {
  const size_t cbytes = ((size_t)K * S * 4 + 15) & ~(size_t)15;
  const size_t ibytes = (size_t)K * kCandL;                   // multiple of 16
  const size_t fbytes = ((size_t)K * 4 + 15) & ~(size_t)15;   // per-centroid floats
  return cbytes + ibytes + 3 * fbytes + (size_t)kCandWarps * kCandQ * (32 + 40);
}

template <int S>
__global__ void __launch_bounds__(kCandThreads, 4)
pq_cand_kernel(const float* __restrict__ XT, uint64_t N, int K, const float* __restrict__ cb,
               const uint8_t* __restrict__ nbr_idx, const float* __restrict__ nbr_last, uint8_t* __restrict__ asg,
               float* __restrict__ ubnd, float* __restrict__ lbnd, const float* __restrict__ drift,
               const float* __restrict__ maxd, const uint8_t* __restrict__ state, float* __restrict__ mind,
               int need_mind, uint32_t* __restrict__ list_cnt, unsigned long long* __restrict__ dist_cnt) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ int s_bad;
  const int m = blockIdx.y;
  if (state[m] != kRunning) return;
  const size_t cbytes = ((size_t)K * S * 4 + 15) & ~(size_t)15;
  const size_t ibytes = (size_t)K * kCandL;
  const size_t fbytes = ((size_t)K * 4 + 15) & ~(size_t)15;
  float* sC = reinterpret_cast<float*>(smem_raw);                                   // [K][S]
  uint8_t* sI = smem_raw + cbytes;                                                   // [K][kCandL] neighbours
  float* sV = reinterpret_cast<float*>(smem_raw + cbytes + ibytes);                 // [K] v_last
  float* sD = reinterpret_cast<float*>(smem_raw + cbytes + ibytes + fbytes);        // [K] drifts
  float* sH = reinterpret_cast<float*>(smem_raw + cbytes + ibytes + 2 * fbytes);    // [K] mid-list bound
  unsigned char* qbase = smem_raw + cbytes + ibytes + 3 * fbytes;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float4* qx = reinterpret_cast<float4*>(qbase) + warp * kCandQ;                    // rows
  float* qd = reinterpret_cast<float*>(qbase + (size_t)kCandWarps * kCandQ * 16) + warp * kCandQ;  // f_a
  float* qu = reinterpret_cast<float*>(qbase + (size_t)kCandWarps * kCandQ * 20) + warp * kCandQ;  // ut
  uint32_t* qr = reinterpret_cast<uint32_t*>(qbase + (size_t)kCandWarps * kCandQ * 24) + warp * kCandQ;
  uint32_t* qa = reinterpret_cast<uint32_t*>(qbase + (size_t)kCandWarps * kCandQ * 28) + warp * kCandQ;
  // second-stage queue: rows that go on to the second half of their list,
  // with their first-stage minimum, its index and the second smallest
  unsigned char* q2base = qbase + (size_t)kCandWarps * kCandQ * 32;
  float4* q2x = reinterpret_cast<float4*>(q2base) + warp * kCandQ;
  float* q2u = reinterpret_cast<float*>(q2base + (size_t)kCandWarps * kCandQ * 16) + warp * kCandQ;
  float* q2b = reinterpret_cast<float*>(q2base + (size_t)kCandWarps * kCandQ * 20) + warp * kCandQ;
  float* q2s = reinterpret_cast<float*>(q2base + (size_t)kCandWarps * kCandQ * 24) + warp * kCandQ;
  uint32_t* q2i = reinterpret_cast<uint32_t*>(q2base + (size_t)kCandWarps * kCandQ * 28) + warp * kCandQ;
  uint32_t* q2r = reinterpret_cast<uint32_t*>(q2base + (size_t)kCandWarps * kCandQ * 32) + warp * kCandQ;
  uint32_t* q2a = reinterpret_cast<uint32_t*>(q2base + (size_t)kCandWarps * kCandQ * 36) + warp * kCandQ;
  if (tid == 0) s_bad = 0;
  __syncthreads();
  {
    int bad = 0;
    for (int e = tid; e < K * S; e += kCandThreads) {
      const float v = cb[(size_t)m * K * S + e];
      sC[e] = v;
      bad |= !isfinite(v);
    }
    const uint4* gi = reinterpret_cast<const uint4*>(nbr_idx + (size_t)m * K * kCandL);
    for (int e = tid; e < K * kCandL / 16; e += kCandThreads) reinterpret_cast<uint4*>(sI)[e] = gi[e];
    for (int c = tid; c < K; c += kCandThreads) {
      sV[c] = nbr_last[((size_t)m * K + c) * 2];
      sH[c] = nbr_last[((size_t)m * K + c) * 2 + 1];
      sD[c] = drift[(size_t)m * K + c];
    }
    if (bad) atomicOr(&s_bad, 1);
  }
  __syncthreads();
  const bool bad_cb = s_bad != 0;
  const int L = min(kCandL, K - 1);  // listed neighbours; L < kCandL: every centroid is listed
  const float md1 = maxd[3 * m], md2 = maxd[3 * m + 2];
  const uint32_t mi1 = (uint32_t)(int)maxd[3 * m + 1];
  uint32_t qn = 0, q2n = 0, listed = 0;
  unsigned long long dists = 0;

  // Exact distances of x to listed neighbours [h * 16, h * 16 + 16) of a
  // (those below L), folded into the running first minimum (b, bi; smallest
  // index on equal values) and second smallest sc.
  auto scan_half = [&](int h, const float (&x)[S], uint32_t a, float& b, int& bi, float& sc) {
    const uint4 w = reinterpret_cast<const uint4*>(sI + (size_t)a * kCandL)[h];
    const uint32_t wd[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int q = 0; q < 16; ++q) {
      if (h * 16 + q < L) {
        const int j = (int)((wd[q >> 2] >> (8 * (q & 3))) & 0xFFu);
        float c[S];
        load_centroid<S>(sC, j, c);
        const float f = l2_small<S>(x, c);
        if (f < b || (f == b && j < bi)) {
          sc = fminf(sc, b);
          b = f;
          bi = j;
        } else {
          sc = fminf(sc, f);
        }
      }
    }
  };

  // Scan the last `cnt` (1..32) queued rows, one per lane.
  auto scan_rows = [&](uint32_t cnt) {
    const bool act = (uint32_t)lane < cnt;
    const uint32_t e = qn - cnt + (act ? (uint32_t)lane : 0u);
    const float4 v = qx[e];
    float x[S];
    x[0] = v.x;
    if constexpr (S > 1) x[1] = v.y;
    if constexpr (S > 2) { x[2] = v.z; x[3] = v.w; }
    const uint32_t a = qa[e];
    const float ut = qu[e];
    float b = qd[e], sc = __int_as_float(0x7f800000);
    int bi = (int)a;
    // first stage: the first half of a full list (all of a shorter one)
    scan_half(0, x, a, b, bi, sc);
    if (L < kCandL) scan_half(1, x, a, b, bi, sc);
    const float vlast = sV[a];
    const float T = __fadd_ru(__fmul_ru(ut, kCandCut), kCandFloor);
    const bool full = act && (bad_cb || !(ut <= 3.0e38f) || (L == kCandL && !(vlast > T)));
    // A full list whose second half may hold a centroid inside the cutoff
    // (its first entry's bound at or below T) goes on to the second stage;
    // otherwise every unscanned centroid has a bound above T (the second
    // half's entries and the unlisted ones alike), as the argument above
    // requires, and the next lower bound uses the second half's first bound.
    const float vmid = sH[a];
    const bool cont = act && !full && L == kCandL && !(vmid > T);
    float lb = fminf(bound_lower(sc), L == kCandL ? __fsub_rd(vmid, ut) : __int_as_float(0x7f800000));
    unsigned long long cnt_d = (unsigned long long)(L == kCandL ? kCandH : L) + 1;
    // rows whose cutoff reaches past the list: the warp scans all K, one row at a time
    unsigned fm = __ballot_sync(0xffffffffu, full);
    while (fm) {
      const int src = __ffs(fm) - 1;
      fm &= fm - 1;
      float xs[S];
#pragma unroll
      for (int k = 0; k < S; ++k) xs[k] = __shfl_sync(0xffffffffu, x[k], src);
      float fb = __int_as_float(0x7f800000), fs = __int_as_float(0x7f800000), d0 = 0.f;
      int fi = 0x7fffffff;
      // lane l takes centroids l, l + 32, ... (consecutive lanes read
      // consecutive codewords: no bank conflicts); equal distances across
      // lanes are settled by index in the reduction
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int j = lane + 32 * q;
        if (j < K) {
          float c[S];
          load_centroid<S>(sC, j, c);
          const float f = l2_small<S>(xs, c);
          if (j == 0) d0 = f;
          const float fk = isnan(f) ? __int_as_float(0x7f800000) : f;
          if (fk < fb || fi == 0x7fffffff) {
            fs = fminf(fs, fb);
            fb = fk;
            fi = j;
          } else {
            fs = fminf(fs, fk);
          }
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, fb, o);
        const int oi = __shfl_xor_sync(0xffffffffu, fi, o);
        const float os = __shfl_xor_sync(0xffffffffu, fs, o);
        if (ob < fb || (ob == fb && oi < fi)) {
          fs = fminf(fminf(fs, fb), os);
          fb = ob;
          fi = oi;
        } else {
          fs = fminf(fminf(fs, ob), os);
        }
      }
      d0 = __shfl_sync(0xffffffffu, d0, 0);
      if (lane == src) {
        if (isnan(d0)) {  // vec.argmin starts from dists[0]: a NaN there wins
          b = d0;
          bi = 0;
          lb = -__int_as_float(0x7f800000);
        } else {
          b = fb;
          bi = fi;
          lb = bound_lower(fs);
        }
        cnt_d = (unsigned long long)K;
      }
    }
    const uint32_t cb2 = __ballot_sync(0xffffffffu, cont);
    if (cont) {
      const uint32_t q = q2n + __popc(cb2 & lanemask_lt());
      q2x[q] = v;
      q2u[q] = ut;
      q2b[q] = b;
      q2s[q] = sc;
      q2i[q] = (uint32_t)bi;
      q2r[q] = qr[e];
      q2a[q] = a;
    } else if (act) {
      const size_t eo = (size_t)m * N + qr[e];
      asg[eo] = (uint8_t)bi;
      mind[eo] = b;
      ubnd[eo] = bound_upper(b);
      lbnd[eo] = lb;
      dists += cnt_d;
    }
    q2n += __popc(cb2);
    qn -= cnt;
    __syncwarp();
  };

  // Second stage for the last `cnt` (1..32) rows of the second-stage queue:
  // the second half of the list, then the bounds as for a full first stage.
  auto scan2_rows = [&](uint32_t cnt) {
    const bool act = (uint32_t)lane < cnt;
    const uint32_t e = q2n - cnt + (act ? (uint32_t)lane : 0u);
    const float4 v = q2x[e];
    float x[S];
    x[0] = v.x;
    if constexpr (S > 1) x[1] = v.y;
    if constexpr (S > 2) { x[2] = v.z; x[3] = v.w; }
    const uint32_t a = q2a[e];
    const float ut = q2u[e];
    float b = q2b[e], sc = q2s[e];
    int bi = (int)q2i[e];
    scan_half(1, x, a, b, bi, sc);
    if (act) {
      const float lb = fminf(bound_lower(sc), __fsub_rd(sV[a], ut));
      const size_t eo = (size_t)m * N + q2r[e];
      asg[eo] = (uint8_t)bi;
      mind[eo] = b;
      ubnd[eo] = bound_upper(b);
      lbnd[eo] = lb;
      dists += (unsigned long long)L + 1;
    }
    q2n -= cnt;
    __syncwarp();
  };

  const uint64_t wstride = (uint64_t)gridDim.x * kCandWarps * 32;
  for (uint64_t base = ((uint64_t)blockIdx.x * kCandWarps + warp) * 32; base < N; base += wstride) {
    // ---- bounds of 32 rows; one exact distance when they fail; queue the rest
    const uint64_t r = base + lane;
    bool queue = false;
    float x[S];
    float da = 0.f, ut = 0.f;
    uint32_t a = 0;
    if (r < N) {
      const size_t e = (size_t)m * N + r;
      a = asg[e];
      const float u = __fadd_ru(ubnd[e], sD[a]);
      const float l = __fsub_rd(lbnd[e], a == mi1 ? md2 : md1);
      if (l >= kLbMin && __fmul_ru(u, kPruneMargin) < l) {
        ubnd[e] = u;
        lbnd[e] = l;
        if (need_mind) {
          float c[S];
          load_sub<S>(XT + e * S, x);
          load_centroid<S>(sC, (int)a, c);
          mind[e] = l2_small<S>(x, c);
        }
      } else {
        float c[S];
        load_sub<S>(XT + e * S, x);
        load_centroid<S>(sC, (int)a, c);
        da = l2_small<S>(x, c);
        ut = bound_upper(da);
        if (l >= kLbMin && __fmul_ru(ut, kPruneMargin) < l) {
          ubnd[e] = ut;
          lbnd[e] = l;
          mind[e] = da;
        } else {
          queue = true;
        }
      }
    }
    const uint32_t qb = __ballot_sync(0xffffffffu, queue);
    if (queue) {
      const uint32_t q = qn + __popc(qb & lanemask_lt());
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      v.x = x[0];
      if constexpr (S > 1) v.y = x[1];
      if constexpr (S > 2) { v.z = x[2]; v.w = x[3]; }
      qx[q] = v;
      qd[q] = da;
      qu[q] = ut;
      qr[q] = (uint32_t)r;
      qa[q] = a;
    }
    qn += __popc(qb);
    listed += __popc(qb);
    __syncwarp();
    if (qn >= 32) scan_rows(32);
    if (q2n >= 32) scan2_rows(32);
  }
  if (qn > 0) scan_rows(qn);
  while (q2n > 0) scan2_rows(q2n < 32u ? q2n : 32u);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) dists += __shfl_xor_sync(0xffffffffu, dists, o);
  if (lane == 0) {
    if (dists) atomicAdd(&dist_cnt[m], dists);
    if (listed) atomicAdd(&list_cnt[m], listed);
  }
}

// ---------------------------------------------------------------------------
// Tensor-core filtered assignment (Lloyd passes with bounds, and encode).
//
// Per 128-row tile of one subspace m, a kind::tf32 MMA chain (tc_filter.cuh)
// yields a(c) = t + fl(|c|^2) - 2 x.c for all 256 columns, within E of its
// exact value, where (all bounds rounded outwards)
//   E = 2^-17 (2 |x| max|c| + max|c|^2 + t) + 2^-100.
// The dropped lo*lo terms and the TF32 truncation of the lo parts add at
// most 3 * 2^-20 * sum|x_k y_k| (y = -2c) + 2^-20 |c|^2. The accumulation
// is bounded as an f32 accumulator that rounds (or truncates) once per
// addition: the three MMAs add at most 27 terms, each addition off by at
// most 2^-23 of the running magnitude, so at most 27 * 2^-23 < 2^-18.2 of
// the summed magnitudes (NVIDIA does not document the order or width of the
// tensor core's internal sums; the measured error is about one ulp per
// MMA). Both stay below 2^-17.3 of (2 |x| max|c| + max|c|^2 + t), so E
// holds. The row
// constant t (TF32-exact, >= |x|^2 + E + ...) keeps every a(c) positive, so
// the f32 bit patterns order like the values; the low 8 bits are replaced
// by the column index, and integer min/max per column track the smallest
// and the second smallest key with its index.
//
// One persistent CTA per SM, warp-specialised: a producer warp stages the
// next 128-row tile (operand A, the rows' constants) into one of two
// buffers and issues its MMA chain into that buffer's 256 TMEM columns,
// while two epilogue warpgroups (one per buffer, one thread per row) scan
// the previous tiles' accumulators. mbarriers hand the buffers over
// (acc_full: MMA done; acc_empty: epilogue done); every wait is bounded and
// an expired wait stops the CTA and raises diag[2].
//
// The reference winner w (first minimum of the exact f32 distances f, which
// are within (1 +- g) of the exact squared distances D, g = 2^-21) satisfies
//   a(w) <= a(c1) + 2E + ((1+g)/(1-g) - 1) D(c1) + 2 delta
// (c1 the smallest key, delta >= |fl(|c|^2) - |c|^2|), so every column whose
// key is above that threshold T is out. When only c1 is at or below T, w =
// c1; otherwise the columns at or below T (about 0.5 % of rows) are
// re-scanned and their exact distances decide in index order. The exact
// distance of the winner is always computed, so min_to_any and the WCSS are
// the reference's. A row whose winner's approximation disagrees with its
// exact distance beyond E counts as a violation (diag[0]); the host then
// repeats the pass with the exact kernels. Lower bounds for the Lloyd
// pruning come from the second key (or T) minus E, or from the exact
// distances of the other re-scanned columns.
//
// Rows or codebooks with non-finite values or magnitudes above 2^60 take
// the exact scan over all K centroids (the reference's own loop).
// ---------------------------------------------------------------------------
constexpr float kTcErr = 0x1p-17f;
constexpr float kTcDelta = 0x1p-20f;  // |fl(|c|^2) - |c|^2| <= 2^-20 max|c|^2 (S <= 4)
constexpr float kTcRho = 0x1p-19f;    // >= (1 + g) / (1 - g) - 1
constexpr float kTcTiny = 0x1p-100f;
constexpr float kTcHuge = 0x1p60f;
constexpr float kTcPad = 0x1p64f;     // a(c) of the padding columns c >= K

// Exact distances of the columns whose bit is set in `mask` (columns
// base .. base + 31), in index order: first strict minimum, runner-up.
template <int S>
__device__ __noinline__ void tc_exact_columns(const float* x, const float* sC, uint32_t mask, int base, float& best,
                                              int& bi, float& sec) {
  while (mask) {
    const int c = base + __ffs(mask) - 1;
    mask &= mask - 1;
    float xv[S];
#pragma unroll
    for (int k = 0; k < S; ++k) xv[k] = x[k];
    const float f = l2_small<S>(xv, sC + c * S);
    if (f < best) {
      sec = best;
      best = f;
      bi = c;
    } else {
      sec = fminf(sec, f);
    }
  }
}

// One row of a staged tile, written by the producer warp for the epilogue.
struct TcRow {
  float x[4];
  float t, E, xn2_up, xn2_dn;
  uint64_t row;
  uint32_t flags;  // bit 0: valid, bit 1: filtered (else the exact scan when valid)
  uint32_t pad;
};
static_assert(sizeof(TcRow) == 48, "TcRow layout");

// Per accumulator buffer: operand tiles, the exact codebook, the staged rows
// and the codebook's scalars.
struct TcBuf {
  static constexpr uint32_t kBhi = 0, kBlo = tc::kTileBytesB, kAhi = 2 * tc::kTileBytesB,
                            kAlo = kAhi + tc::kTileBytesA, kC = kAlo + tc::kTileBytesA, kRows = kC + 256 * 4 * 4,
                            kBytes = kRows + 128 * sizeof(TcRow);
};
constexpr int kTcEpiWarps = 8;                       // two epilogue warpgroups, one per buffer
constexpr int kTcBlock = (kTcEpiWarps + 1) * 32;     // + the producer / MMA warp
// more than half of an SM's shared memory: one CTA (and its 512 TMEM
// columns) per SM
constexpr size_t kTcSmemBytes = 120 * 1024;
static_assert(2 * TcBuf::kBytes + 1024 <= kTcSmemBytes, "filter buffers exceed the shared-memory request");

template <int S, int MODE, bool LIST>
__global__ void __launch_bounds__(kTcBlock, 1)
pq_tc_assign_kernel(const float* __restrict__ R, const float* __restrict__ XT, uint64_t N, int D, int M, int K,
                    const float* __restrict__ cb, const uint32_t* __restrict__ list,
                    const uint32_t* __restrict__ list_cnt, uint8_t* __restrict__ codes, uint8_t* __restrict__ asg,
                    float* __restrict__ mind, float* __restrict__ ubnd, float* __restrict__ lbnd,
                    const uint8_t* __restrict__ state, uint32_t* __restrict__ diag) {
  extern __shared__ unsigned char tc_raw[];
  unsigned char* base = tc_raw + ((1024u - (tc::smem_addr(tc_raw) & 1023u)) & 1023u);
  __shared__ __align__(8) uint64_t acc_full[2], acc_empty[2];
  __shared__ uint32_t tslot, upre[kMaxM + 1], s_abort, s_lcnt[kMaxM];
  __shared__ uint8_t s_run[kMaxM];  // subspace still running (Lloyd) / always (encode)
  __shared__ int buf_m[2];
  __shared__ float buf_cmax2[2], buf_cmax[2], buf_dl[2];
  __shared__ uint32_t buf_bad[2];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (warp == 0) tc::tmem_alloc(&tslot, 2 * tc::kCols);
  if (tid == 0) {
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&acc_full[b], 2);  // the producer's rows + the MMA commit
      tc::mbar_init(&acc_empty[b], 128);
      buf_m[b] = -1;
    }
    s_abort = 0u;
    for (int m = 0; m < M; ++m) {
      s_run[m] = (MODE == kModeEncode || state[m] == kRunning) ? 1 : 0;
      s_lcnt[m] = LIST ? list_cnt[m] : 0u;
    }
    if (LIST) {
      uint32_t acc = 0;
      for (int m = 0; m < M; ++m) {
        upre[m] = acc;
        acc += s_run[m] ? (s_lcnt[m] + 127u) / 128u : 0u;
      }
      upre[M] = acc;
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = tslot;
  const uint32_t ntiles = (uint32_t)((N + 127) / 128);
  const uint32_t units = LIST ? upre[M] : (uint32_t)M * ntiles;
  auto unit_of = [&](uint32_t u, int& m, uint32_t& i0) {
    if (LIST) {
      m = 0;
      while (upre[m + 1] <= u) ++m;
      i0 = (u - upre[m]) * 128u;
    } else {
      m = (int)(u / ntiles);
      i0 = (u % ntiles) * 128u;
    }
  };
  // this CTA's next unit at or after u whose subspace is still running
  auto next_unit = [&](uint32_t u) -> uint32_t {
    for (; u < units; u += gridDim.x) {
      int m;
      uint32_t i0;
      unit_of(u, m, i0);
      if (s_run[m]) return u;
    }
    return units;
  };

  if (warp == kTcEpiWarps) {
    // ======================= producer / MMA warp ===============================
    // rows of unit u for this lane (rows lane, lane + 32, ...), loaded one
    // tile ahead so that their latency overlaps the wait for a free buffer
    int pm = 0;
    uint64_t prow[4];
    bool pvalid[4];
    float pxs[4][S];
    auto prefetch = [&](uint32_t u) {
      uint32_t i0;
      unit_of(u, pm, i0);
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const uint32_t r = (uint32_t)(lane + 32 * h);
        if (LIST) {
          const uint32_t li = i0 + r;
          pvalid[h] = li < s_lcnt[pm];
          prow[h] = pvalid[h] ? list[(size_t)pm * N + li] : 0;
        } else {
          prow[h] = (uint64_t)i0 + r;
          pvalid[h] = prow[h] < N;
        }
      }
#pragma unroll
      for (int h = 0; h < 4; ++h) {
#pragma unroll
        for (int k = 0; k < S; ++k) pxs[h][k] = 0.f;
        if (pvalid[h]) {
          if (MODE == kModeLloyd) load_sub<S>(XT + ((size_t)pm * N + prow[h]) * S, pxs[h]);
          else load_sub_unaligned<S>(R + prow[h] * (uint64_t)D + (uint64_t)pm * S, pxs[h]);
        }
      }
    };
    uint32_t u = next_unit(blockIdx.x);
    if (u < units) prefetch(u);
    for (uint32_t i = 0; u < units; ++i) {
      const int b = (int)(i & 1u);
      unsigned char* bb = base + b * TcBuf::kBytes;
      const bool ok_wait = i < 2 || tc::mbar_wait(&acc_empty[b], ((i >> 1) - 1u) & 1u);
      if (!__all_sync(0xFFFFFFFFu, ok_wait) || __any_sync(0xFFFFFFFFu, *(volatile uint32_t*)&s_abort != 0u)) {
        if (lane == 0) atomicExch(&s_abort, 1u);
        break;
      }
      const int m = pm;
      const uint32_t u_next = next_unit(u + gridDim.x);
      if (m != buf_m[b]) {  // operand B (hi, lo) and the exact codebook of subspace m
        float* sC = reinterpret_cast<float*>(bb + TcBuf::kC);
        uint32_t cmax2 = 0u;
        bool badc = false;
        for (int c = lane; c < (int)tc::kCols; c += 32) {
          const bool real = c < K;
          float cv[4] = {0.f, 0.f, 0.f, 0.f};
          if (real) {
#pragma unroll
            for (int k = 0; k < S; ++k) {
              cv[k] = cb[((size_t)m * K + c) * S + k];
              sC[c * S + k] = cv[k];
            }
          }
          float cn = 0.f, cn_up = 0.f;
          bool fin = true;
#pragma unroll
          for (int k = 0; k < S; ++k) {
            cn = __fadd_rn(cn, __fmul_rn(cv[k], cv[k]));
            cn_up = __fadd_ru(cn_up, __fmul_ru(cv[k], cv[k]));
            fin = fin && isfinite(cv[k]);
          }
          float yh[4], yl[4], cnh, cnl;
#pragma unroll
          for (int k = 0; k < 4; ++k) tc::split_tf32(__fmul_rn(-2.0f, cv[k]), yh[k], yl[k]);
          tc::split_tf32(cn, cnh, cnl);
          const bool ok = fin && cn_up <= kTcHuge;
          if (!real || !ok) {
#pragma unroll
            for (int k = 0; k < 4; ++k) yh[k] = yl[k] = 0.f;
          }
          *reinterpret_cast<float4*>(bb + TcBuf::kBhi + tc::operand_offset(c, 0)) = make_float4(yh[0], yh[1], yh[2], yh[3]);
          *reinterpret_cast<float4*>(bb + TcBuf::kBlo + tc::operand_offset(c, 0)) = make_float4(yl[0], yl[1], yl[2], yl[3]);
          *reinterpret_cast<float4*>(bb + TcBuf::kBhi + tc::operand_offset(c, 4)) =
              (real && ok) ? make_float4(cnh, 1.0f, 0.f, 0.f) : make_float4(kTcPad, 0.f, 0.f, 0.f);
          *reinterpret_cast<float4*>(bb + TcBuf::kBlo + tc::operand_offset(c, 4)) =
              make_float4((real && ok) ? cnl : 0.f, 0.f, 0.f, 0.f);
          if (real) {
            if (!ok) badc = true;
            else cmax2 = max(cmax2, __float_as_uint(cn_up));  // non-negative floats order as integers
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) cmax2 = max(cmax2, __shfl_xor_sync(0xFFFFFFFFu, cmax2, o));
        badc = __any_sync(0xFFFFFFFFu, badc);
        if (lane == 0) {
          const float c2 = __uint_as_float(cmax2);
          buf_cmax2[b] = c2;
          buf_cmax[b] = __fsqrt_ru(c2);
          buf_dl[b] = __fmul_ru(kTcDelta, c2);
          buf_bad[b] = badc ? 1u : 0u;
          buf_m[b] = m;
        }
        __syncwarp();
      }
      const float cmax2 = buf_cmax2[b], cmax_up = buf_cmax[b], dl = buf_dl[b];
      const bool bad = buf_bad[b] != 0u;
      // operand A and the staged rows
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const uint32_t r = (uint32_t)(lane + 32 * h);
        bool fin = true;
        float xn2_up = 0.f, xn2_dn = 0.f;
#pragma unroll
        for (int k = 0; k < S; ++k) {
          fin = fin && isfinite(pxs[h][k]);
          xn2_up = __fadd_ru(xn2_up, __fmul_ru(pxs[h][k], pxs[h][k]));
          xn2_dn = __fadd_rd(xn2_dn, __fmul_rd(pxs[h][k], pxs[h][k]));
        }
        const bool filt = pvalid[h] && !bad && fin && xn2_up <= kTcHuge;
        float t = 1.0f, E = 0.f;
        if (filt) {
          const float xn_up = __fsqrt_ru(xn2_up);
          const float eb = __fmul_ru(kTcErr, __fadd_ru(__fmul_ru(2.0f, __fmul_ru(xn_up, cmax_up)), cmax2));
          const float t0 = __fadd_ru(__fmul_ru(__fadd_ru(__fadd_ru(xn2_up, dl), eb), 1.0f + 0x1p-12f), kTcTiny);
          t = tc::tf32_ceil_pos(t0);
          E = __fadd_ru(__fadd_ru(eb, __fmul_ru(kTcErr, t)), kTcTiny);
        }
        float xh[4] = {0.f, 0.f, 0.f, 0.f}, xl[4] = {0.f, 0.f, 0.f, 0.f};
        if (filt) {
#pragma unroll
          for (int k = 0; k < S; ++k) tc::split_tf32(pxs[h][k], xh[k], xl[k]);
        }
        *reinterpret_cast<float4*>(bb + TcBuf::kAhi + tc::operand_offset(r, 0)) = make_float4(xh[0], xh[1], xh[2], xh[3]);
        *reinterpret_cast<float4*>(bb + TcBuf::kAlo + tc::operand_offset(r, 0)) = make_float4(xl[0], xl[1], xl[2], xl[3]);
        *reinterpret_cast<float4*>(bb + TcBuf::kAhi + tc::operand_offset(r, 4)) = make_float4(1.0f, t, 0.f, 0.f);
        *reinterpret_cast<float4*>(bb + TcBuf::kAlo + tc::operand_offset(r, 4)) = make_float4(0.f, 0.f, 0.f, 0.f);
        TcRow* tr = reinterpret_cast<TcRow*>(bb + TcBuf::kRows) + r;
#pragma unroll
        for (int k = 0; k < 4; ++k) tr->x[k] = k < S ? pxs[h][k] : 0.f;
        tr->t = t;
        tr->E = E;
        tr->xn2_up = xn2_up;
        tr->xn2_dn = xn2_dn;
        tr->row = prow[h];
        tr->flags = (pvalid[h] ? 1u : 0u) | (filt ? 2u : 0u);
      }
      tc::fence_async_smem();  // operand tiles -> the tensor core's proxy
      __syncwarp();
      if (lane == 0) {
        tc::mbar_arrive(&acc_full[b]);  // releases the staged rows and scalars to the epilogue
        tc::fence_after_sync();
        const uint32_t d = tbase + (uint32_t)b * tc::kCols;
        const uint64_t dah = tc::operand_desc(bb + TcBuf::kAhi), dal = tc::operand_desc(bb + TcBuf::kAlo);
        const uint64_t dbh = tc::operand_desc(bb + TcBuf::kBhi), dbl = tc::operand_desc(bb + TcBuf::kBlo);
        tc::mma_tf32(d, dah, dbh, 0u);
        tc::mma_tf32(d, dah, dbl, 1u);
        tc::mma_tf32(d, dal, dbh, 1u);
        tc::mma_commit(&acc_full[b]);  // second arrival: the accumulator is complete
      }
      __syncwarp();
      if (u_next < units) prefetch(u_next);
      u = u_next;
    }
  } else {
    // ======================= epilogue warpgroups ===============================
    // warpgroup g works on buffer g, one thread per row (= TMEM lane)
    const int g = warp >> 2;
    const int r = (warp & 3) * 32 + lane;
    unsigned char* bb = base + g * TcBuf::kBytes;
    const float* sC = reinterpret_cast<const float*>(bb + TcBuf::kC);
    const uint32_t taddr = tbase + (uint32_t)g * tc::kCols + ((uint32_t)((warp & 3) * 32) << 16);
    uint32_t u = next_unit(blockIdx.x);
    if (g == 1 && u < units) u = next_unit(u + gridDim.x);
    for (uint32_t j = 0; u < units; ++j) {
      const bool got = tc::mbar_wait(&acc_full[g], j & 1u);
      if (!__all_sync(0xFFFFFFFFu, got)) {
        if (lane == 0) atomicExch(&s_abort, 1u);
        break;
      }
      tc::fence_after_sync();

      // ---- pass 1: the two smallest keys, a quarter of the columns per wait ---
      // key = (bits of a(c), low 8 bits cleared) | c, compared as positive
      // floats (same order as the integers); two independent chains.
      uint32_t m1 = 0xFFFFFFFFu, m2 = 0xFFFFFFFFu;
#pragma unroll 1
      for (int q = 0; q < 4; ++q) {
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
        const uint32_t qb = (uint32_t)q << 6;  // jj < 64 leaves bits 6-7 free
        const uint32_t q1 = __float_as_uint(fminf(f1a, f1b)) | qb;
        const uint32_t q2 = __float_as_uint(fminf(fmaxf(f1a, f1b), fminf(f2a, f2b))) | qb;
        const uint32_t n2 = min(max(m1, q1), min(m2, q2));
        m1 = min(m1, q1);
        m2 = n2;
      }
      const int m = buf_m[g];
      const float dl = buf_dl[g];
      const TcRow tr = reinterpret_cast<const TcRow*>(bb + TcBuf::kRows)[r];
      const bool valid = (tr.flags & 1u) != 0u, filt = (tr.flags & 2u) != 0u;
      float x[S];
#pragma unroll
      for (int k = 0; k < S; ++k) x[k] = tr.x[k];
      const float t = tr.t, E = tr.E;
      uint32_t thrkey = 0u;
      float T = 0.f;
      if (filt) {
        const float a1hi = __uint_as_float(m1 | 0xFFu);
        const float dup = fmaxf(__fadd_ru(__fadd_ru(__fsub_ru(__fadd_ru(a1hi, E), t), tr.xn2_up), dl), 0.f);
        T = __fadd_ru(__fadd_ru(__fadd_ru(a1hi, __fmul_ru(2.0f, E)), __fmul_ru(kTcRho, dup)), __fmul_ru(2.0f, dl));
        thrkey = __float_as_uint(T) | 0xFFu;  // column c is in when bits(a(c)) <= thrkey
      }
      const bool need2 = filt && m2 <= thrkey;
      int bi = 0;
      float best = 0.f, lbv = 0.f;
      bool viol = false;
      if (filt && !need2) {
        bi = (int)(m1 & 0xFFu);
        best = l2_small<S>(x, sC + bi * S);
        const float a2lo = __uint_as_float(m2 & 0xFFFFFF00u);
        const float lsq = __fsub_rd(__fadd_rd(__fsub_rd(__fsub_rd(a2lo, E), t), tr.xn2_dn), dl);
        lbv = __fsqrt_rd(fmaxf(lsq, 0.f));
        const float a1lo = __uint_as_float(m1 & 0xFFFFFF00u), a1hi = __uint_as_float(m1 | 0xFFu);
        const float phi =
            __fadd_ru(__fadd_ru(__fadd_ru(__fsub_ru(t, tr.xn2_dn), __fmul_ru(best, 1.0f + 0x1p-20f)), dl), E);
        const float plo =
            __fsub_rd(__fsub_rd(__fadd_rd(__fsub_rd(t, tr.xn2_up), __fmul_rd(best, 1.0f - 0x1p-20f)), dl), E);
        viol = a1lo > phi || a1hi < plo;
      }
      {
        const uint32_t vm = __ballot_sync(0xFFFFFFFFu, viol);
        if (vm && lane == 0) atomicAdd(&diag[0], (uint32_t)__popc(vm));
      }
      // ---- pass 2 (rare): exact distances of every column at or below T -------
      const uint32_t need_mask = __ballot_sync(0xFFFFFFFFu, need2);
      if (need_mask) {
        float sec = __int_as_float(0x7f800000);
        if (need2) best = __int_as_float(0x7f800000);
#pragma unroll 1
        for (int q = 0; q < 4; ++q) {
          uint32_t v[64];
          tc::tmem_ld64(taddr + (uint32_t)(q * 64), v);
          tc::tmem_wait_ld();
          if (need2) {
#pragma unroll
            for (int w32 = 0; w32 < 2; ++w32) {
              uint32_t bits = 0u;
#pragma unroll
              for (int jj = 0; jj < 32; ++jj) bits |= (v[w32 * 32 + jj] <= thrkey ? 1u : 0u) << jj;
              tc_exact_columns<S>(x, sC, bits, q * 64 + w32 * 32, best, bi, sec);
            }
          }
        }
        if (need2) {
          const float lsq = __fsub_rd(__fadd_rd(__fsub_rd(__fsub_rd(T, E), t), tr.xn2_dn), dl);
          lbv = __fsqrt_rd(fmaxf(lsq, 0.f));
          if (sec < __int_as_float(0x7f800000)) lbv = fminf(lbv, bound_lower(sec));
        }
        if (lane == 0) atomicAdd(&diag[1], (uint32_t)__popc(need_mask));
      }
      // ---- rows outside the filter's range: the reference's own scan ----------
      if (valid && !filt) {
        float sec = __int_as_float(0x7f800000), d0 = 0.f;
        best = __int_as_float(0x7f800000);
        bi = 0;
#pragma unroll 1
        for (int c = 0; c < K; ++c) {
          const float f = l2_small<S>(x, sC + c * S);
          if (c == 0) d0 = f;
          if (f < best) {
            sec = best;
            best = f;
            bi = c;
          } else {
            sec = fminf(sec, f);
          }
        }
        if (MODE == kModeLloyd) {
          if (isnan(d0)) {  // vec.argmin starts from dists[0]
            bi = 0;
            best = d0;
          }
          lbv = isnan(d0) ? -__int_as_float(0x7f800000) : bound_lower(sec);
        }
      }
      if (valid) {
        if (MODE == kModeLloyd) {
          const size_t e = (size_t)m * N + tr.row;
          asg[e] = (uint8_t)bi;
          mind[e] = best;
          ubnd[e] = bound_upper(best);
          lbnd[e] = lbv;
        } else {
          codes[tr.row * (uint64_t)M + m] = (uint8_t)bi;
        }
      }
      tc::fence_before_sync();
      tc::mbar_arrive(&acc_empty[g]);  // buffer g (TMEM and staged rows) is free again
      u = next_unit(u + gridDim.x);
      if (u < units) u = next_unit(u + gridDim.x);
      if (__any_sync(0xFFFFFFFFu, *(volatile uint32_t*)&s_abort != 0u)) break;
    }
  }
  __syncthreads();
  if (tid == 0 && s_abort) atomicExch(&diag[2], 1u);
  tc::fence_after_sync();
  if (warp == 0) tc::tmem_free(tbase, 2 * tc::kCols);
}

// Per-CTA cluster histograms of all rows (the row ranges of pq_assign_kernel).
__global__ void __launch_bounds__(512)
pq_hist_kernel(const uint8_t* __restrict__ asg, uint64_t N, int M, int K, const uint8_t* __restrict__ state,
               uint64_t rows_per_cta, uint32_t* __restrict__ hist) {
  extern __shared__ uint32_t hh[];  // [M][K]
  for (int e = threadIdx.x; e < M * K; e += blockDim.x) hh[e] = 0;
  __syncthreads();
  const uint64_t lo = (uint64_t)blockIdx.x * rows_per_cta, hi = min(N, lo + rows_per_cta);
  for (int m = 0; m < M; ++m) {
    if (state[m] != kRunning) continue;
    const uint8_t* a = asg + (size_t)m * N;
    for (uint64_t r = lo + threadIdx.x; r < hi; r += blockDim.x) atomicAdd(&hh[m * K + a[r]], 1u);
  }
  __syncthreads();
  const int nblk = gridDim.x;
  for (int e = threadIdx.x; e < M * K; e += blockDim.x) {
    const int m = e / K, c = e % K;
    hist[((size_t)m * nblk + blockIdx.x) * K + c] = hh[e];
  }
}

// Before an empty-cluster reseed: f32 distances of every row to its winner
// (rows kept by their bounds have no fresh value). Subspaces without an
// empty cluster leave at once.
template <int S>
__global__ void __launch_bounds__(256)
pq_mind_refresh_kernel(const float* __restrict__ XT, uint64_t N, int K, const float* __restrict__ cb,
                       const uint8_t* __restrict__ asg, const uint32_t* __restrict__ counts,
                       const uint8_t* __restrict__ state, float* __restrict__ mind) {
  const int m = blockIdx.y;
  if (state[m] != kRunning) return;
  const bool empty = threadIdx.x < (unsigned)K && counts[(size_t)m * K + threadIdx.x] == 0;
  if (!__syncthreads_or(empty)) return;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t r = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; r < N; r += stride) {
    const size_t e = (size_t)m * N + r;
    const uint32_t a = asg[e];
    float x[S], c[S];
    load_sub<S>(XT + e * S, x);
#pragma unroll
    for (int k = 0; k < S; ++k) c[k] = cb[((size_t)m * K + a) * S + k];
    mind[e] = l2_small<S>(x, c);
  }
}

// ---------------------------------------------------------------------------
// Per-cluster counts and stable scatter bases: for each (m, c), base of CTA
// b = start[c] + sum_{b' < b} hist[b'][c].
// ---------------------------------------------------------------------------
constexpr int kScanThreads = 1024;
constexpr int kScanWarps = kScanThreads / 32;

// One CTA per subspace: warp w sums the histogram rows of its range of CTAs
// (nblk split in kScanWarps contiguous ranges, lane = cluster within a group
// of 32), the per-cluster totals and the ranges' exclusive offsets come from
// the shared partial sums, one scan over the clusters gives the starts, and
// each warp rewrites its rows as running bases. Every histogram element is
// read twice by independent loads (no serial walk over nblk per thread).
__global__ void __launch_bounds__(kScanThreads)
pq_scan_kernel(uint32_t* __restrict__ hist, int nblk, int K, uint32_t* __restrict__ counts,
               uint32_t* __restrict__ starts, const uint8_t* __restrict__ state) {
  const int m = blockIdx.x;
  if (state[m] != kRunning) return;
  __shared__ uint32_t part[kScanWarps][256];  // range sums, then the ranges' exclusive offsets
  __shared__ uint32_t cstart[256];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t* hm = hist + (size_t)m * nblk * K;
  const int b0 = (int)((int64_t)nblk * warp / kScanWarps), b1 = (int)((int64_t)nblk * (warp + 1) / kScanWarps);
  uint32_t sum[8] = {0, 0, 0, 0, 0, 0, 0, 0};  // clusters lane, lane + 32, ...
#pragma unroll 4
  for (int b = b0; b < b1; ++b) {
#pragma unroll
    for (int q = 0; q < 8; ++q)
      if (q * 32 + lane < K) sum[q] += hm[(size_t)b * K + q * 32 + lane];
  }
#pragma unroll
  for (int q = 0; q < 8; ++q) part[warp][q * 32 + lane] = sum[q];
  __syncthreads();
  if (tid < 256) {
    uint32_t tot = 0;
    for (int w = 0; w < kScanWarps; ++w) {
      const uint32_t v = part[w][tid];
      part[w][tid] = tot;
      tot += v;
    }
    cstart[tid] = tid < K ? tot : 0u;
  }
  __syncthreads();
  if (warp == 0) {  // exclusive scan of the 256 totals, 8 per lane
    uint32_t v[8], sum = 0;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      v[q] = cstart[lane * 8 + q];
      sum += v[q];
    }
    uint32_t incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    uint32_t acc = incl - sum;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int c = lane * 8 + q;
      if (c < K) {
        counts[(size_t)m * K + c] = v[q];
        starts[(size_t)m * K + c] = acc;
      }
      cstart[c] = acc;
      acc += v[q];
    }
  }
  __syncthreads();
  uint32_t run[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) run[q] = cstart[q * 32 + lane] + part[warp][q * 32 + lane];
  for (int b = b0; b < b1; b += 4) {  // four rows' loads go out before their stores
    uint32_t v[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int q = 0; q < 8; ++q)
        v[i][q] = (b + i < b1 && q * 32 + lane < K) ? hm[(size_t)(b + i) * K + q * 32 + lane] : 0u;
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        if (b + i < b1 && q * 32 + lane < K) hm[(size_t)(b + i) * K + q * 32 + lane] = run[q];
        run[q] += v[i][q];
      }
  }
}

// ---------------------------------------------------------------------------
// Stable scatter into cluster order. One warp per subspace walks the CTA's
// row range 32 rows at a time: ranks inside the 32 from __match_any_sync,
// per-cluster running offsets in shared memory owned by the warp. No block
// barrier in the loop.
//
// For S = 4 (16-byte elements) the two elements that share a 32-byte
// sector are written back to back by the same thread, so L2 always sees
// whole sectors (a lone half sector evicted before its partner arrives
// costs a DRAM read-modify-write). The even element of a pair comes from
// the previous lane of the same cluster in the group (shuffle) or, when it
// arrived in an earlier group, from the warp's pending slot for that
// cluster. Only the two ends of each (CTA, cluster) segment are written as
// half sectors.
// ---------------------------------------------------------------------------
template <int S>
__global__ void __launch_bounds__(kMaxM * 32)
pq_scatter_kernel(const float* __restrict__ XT, uint64_t N, int M, int K,
                                  const uint8_t* __restrict__ asg, const uint32_t* __restrict__ bases,
                                  float* __restrict__ sorted, const uint8_t* __restrict__ state,
                                  uint64_t rows_per_cta) {
  extern __shared__ __align__(16) unsigned char scat_smem[];
  const int lane = threadIdx.x & 31, m = threadIdx.x >> 5;
  // per warp: run[256] u32, seg0[256] u32, pend[256] float4
  unsigned char* wbase = scat_smem + (size_t)m * (256 * 8 + (S == 4 ? 256 * 16 : 0));
  uint32_t* run = reinterpret_cast<uint32_t*>(wbase);
  uint32_t* seg0 = run + 256;
  float4* pend = reinterpret_cast<float4*>(seg0 + 256);
  if (m >= M || state[m] != kRunning) return;
  const int nblk = gridDim.x;
  for (int c = lane; c < K; c += 32) {
    const uint32_t b0 = bases[((size_t)m * nblk + blockIdx.x) * K + c];
    run[c] = b0;
    seg0[c] = b0;
  }
  __syncwarp();
  const uint64_t lo = (uint64_t)blockIdx.x * rows_per_cta;
  const uint64_t hi = min(N, lo + rows_per_cta);
  const uint8_t* am = asg + (size_t)m * N;
  const float* xm = XT + (size_t)m * N * S;
  float* sm = sorted + (size_t)m * N * S;
  constexpr int kU = 8;  // 32-row groups loaded ahead
  for (uint64_t base = lo; base < hi; base += 32 * kU) {
    int cl[kU];
    float x[kU][S];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const uint64_t r = base + (uint64_t)u * 32 + lane;
      if (r < hi) {
        cl[u] = __ldcs(am + r);
        if constexpr (S == 4) {
          const float4 v = __ldcs(reinterpret_cast<const float4*>(xm + r * 4));
          x[u][0] = v.x; x[u][1] = v.y; x[u][2] = v.z; x[u][3] = v.w;
        } else {
#pragma unroll
          for (int k = 0; k < S; ++k) x[u][k] = __ldcs(xm + r * S + k);
        }
      } else {
        cl[u] = 256 + lane;  // unique keys never match a real cluster
#pragma unroll
        for (int k = 0; k < S; ++k) x[u][k] = 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const uint32_t peers = __match_any_sync(0xffffffffu, cl[u]);
      const uint32_t below = peers & lanemask_lt();
      const uint32_t rank = __popc(below);
      const uint32_t cnt = __popc(peers);
      const bool ok = cl[u] < 256;
      const int c = ok ? cl[u] : 0;
      const uint32_t p = ok ? run[c] + rank : 0u;
      if constexpr (S == 4) {
        const int prev_lane = below ? 31 - __clz(below) : lane;
        float4 xv = make_float4(x[u][0], x[u][1], x[u][2], x[u][3]);
        float4 xp;
        xp.x = __shfl_sync(0xffffffffu, xv.x, prev_lane);
        xp.y = __shfl_sync(0xffffffffu, xv.y, prev_lane);
        xp.z = __shfl_sync(0xffffffffu, xv.z, prev_lane);
        xp.w = __shfl_sync(0xffffffffu, xv.w, prev_lane);
        // read phase: the pending even element, if this odd element's
        // partner arrived in an earlier group of this segment
        bool have_prev = false;
        if (ok && (p & 1u)) {
          if (rank > 0) {
            have_prev = true;
          } else if (p > seg0[c]) {
            xp = pend[c];
            have_prev = true;
          }
        }
        __syncwarp();
        if (ok) {
          float4* o = reinterpret_cast<float4*>(sm) + p;
          if (p & 1u) {
            if (have_prev) o[-1] = xp;  // same 32-byte sector, back to back
            o[0] = xv;
          } else if (rank + 1 == cnt) {
            pend[c] = xv;  // partner comes later (or never: segment end)
          }
          if (rank == 0) run[c] += cnt;
        }
        __syncwarp();
      } else {
        if (ok) {
          float* o = sm + (size_t)p * S;
#pragma unroll
          for (int k = 0; k < S; ++k) o[k] = x[u][k];
        }
        __syncwarp();
        if (ok && rank == 0) run[c] += cnt;
        __syncwarp();
      }
    }
  }
  if constexpr (S == 4) {
    // segment ends: a last element at an even position has no partner here
    for (int c = lane; c < K; c += 32) {
      const uint32_t r = run[c];
      if (r > seg0[c] && ((r - 1) & 1u) == 0) reinterpret_cast<float4*>(sm)[r - 1] = pend[c];
    }
  }
}

size_t scatter_smem(int M, int S) { return (size_t)M * (256 * 8 + (S == 4 ? 256 * 16 : 0)); }

// ---------------------------------------------------------------------------
// Stable scatter into cluster order, tiled: block (b, m) walks row range b
// (the pq_hist_kernel ranges) of subspace m in tiles of kScatTile rows. Each
// warp ranks its kScatTile / kScatWarps consecutive rows within their
// clusters (__match_any_sync per 32 rows plus a warp-private running count),
// one scan across the warps gives every row its slot in the tile's cluster
// order, the rows are staged there in shared memory and written out by
// consecutive threads, so each cluster's part of the tile leaves as one
// contiguous run of its segment. Row order inside a cluster is kept (warps
// hold consecutive rows, lanes and groups are in row order).
// ---------------------------------------------------------------------------
constexpr int kScatT = 256;
constexpr int kScatWarps = kScatT / 32;
constexpr int kScatTile = 2048;
constexpr int kScatPerWarp = kScatTile / kScatWarps;  // 512 rows: 16 groups of 32

template <int S> struct RowT;
template <> struct RowT<1> { using T = float; };
template <> struct RowT<2> { using T = float2; };
template <> struct RowT<4> { using T = float4; };

size_t scatter_tile_smem(int S) {
  return (size_t)kScatTile * (S * 4 + 1) + (size_t)kScatWarps * 256 * 4 + 3 * 256 * 4;
}

template <int S>
__global__ void __launch_bounds__(kScatT, 3)
pq_scatter_tile_kernel(const float* __restrict__ XT, uint64_t N, int K, const uint8_t* __restrict__ asg,
                       const uint32_t* __restrict__ bases, float* __restrict__ sorted,
                       const uint8_t* __restrict__ state, uint64_t rows_per_cta) {
  using T = typename RowT<S>::T;
  extern __shared__ __align__(16) unsigned char scat_smem[];
  T* srow = reinterpret_cast<T*>(scat_smem);                                   // [kScatTile] rows, tile order
  uint32_t* wcnt = reinterpret_cast<uint32_t*>(srow + kScatTile);              // [kScatWarps][256]
  uint32_t* run = wcnt + kScatWarps * 256;                                     // [256] next global slot
  uint32_t* tstart = run + 256;                                                // [256] tile-local start
  uint32_t* ttot = tstart + 256;                                               // [256] tile count
  uint8_t* scl = reinterpret_cast<uint8_t*>(ttot + 256);                       // [kScatTile] cluster per slot
  const int m = blockIdx.y, b = blockIdx.x, nblk = gridDim.x;
  if (state[m] != kRunning) return;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int c = tid; c < 256; c += kScatT) run[c] = c < K ? bases[((size_t)m * nblk + b) * K + c] : 0u;
  const uint64_t lo = (uint64_t)b * rows_per_cta, hi = min(N, lo + rows_per_cta);
  const uint8_t* am = asg + (size_t)m * N;
  const T* xm = reinterpret_cast<const T*>(XT + (size_t)m * N * S);
  T* sm = reinterpret_cast<T*>(sorted + (size_t)m * N * S);
  uint32_t* myc = wcnt + warp * 256;
  for (uint64_t t0 = lo; t0 < hi; t0 += kScatTile) {
    for (int e = tid; e < kScatWarps * 256; e += kScatT) wcnt[e] = 0;
    __syncthreads();
    // ranks inside the warp's rows, in row order
    constexpr int kG = kScatPerWarp / 32;
    int cl[kG];
    uint32_t rk[kG];
    T xr[kG];  // the rows themselves, loaded with the assignments: their latency overlaps the ranking
    const uint64_t w0 = t0 + (uint64_t)warp * kScatPerWarp;
#pragma unroll
    for (int g = 0; g < kG; ++g) {
      const uint64_t r = w0 + (uint64_t)g * 32 + lane;
      cl[g] = r < hi ? (int)__ldcs(am + r) : 256 + lane;  // 256 + lane: unique, never a cluster
      if (r < hi) xr[g] = __ldcs(xm + r);
    }
#pragma unroll
    for (int g = 0; g < kG; ++g) {
      const uint32_t peers = __match_any_sync(0xffffffffu, cl[g]);
      const uint32_t below = __popc(peers & lanemask_lt());
      const bool ok = cl[g] < 256;
      rk[g] = ok ? myc[cl[g]] + below : 0u;
      __syncwarp();
      if (ok && below == 0) myc[cl[g]] += __popc(peers);
      __syncwarp();
    }
    __syncthreads();
    // per cluster: exclusive offsets of the warps, tile totals, tile starts
    uint32_t tot = 0;
    if (tid < 256) {
      for (int w = 0; w < kScatWarps; ++w) {
        const uint32_t v = wcnt[w * 256 + tid];
        wcnt[w * 256 + tid] = tot;
        tot += v;
      }
      ttot[tid] = tot;
    }
    __syncthreads();
    if (tid < 32) {  // exclusive scan of the 256 tile totals, 8 per lane
      uint32_t v[8], sum = 0;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        v[q] = ttot[tid * 8 + q];
        sum += v[q];
      }
      uint32_t incl = sum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      uint32_t acc = incl - sum;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        tstart[tid * 8 + q] = acc;
        acc += v[q];
      }
    }
    __syncthreads();
    // stage every row at its slot of the tile's cluster order
#pragma unroll
    for (int g = 0; g < kG; ++g) {
      if (cl[g] < 256) {
        const uint32_t slot = tstart[cl[g]] + wcnt[warp * 256 + cl[g]] + rk[g];
        srow[slot] = xr[g];
        scl[slot] = (uint8_t)cl[g];
      }
    }
    __syncthreads();
    // write out: consecutive threads, consecutive slots of a cluster's run
    const uint32_t nt = (uint32_t)min((uint64_t)kScatTile, hi - t0);
#pragma unroll 4
    for (uint32_t i = tid; i < nt; i += kScatT) {
      const int c = scl[i];
      sm[run[c] + (i - tstart[c])] = srow[i];
    }
    __syncthreads();
    if (tid < 256) run[tid] += tot;
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Centroid sums in the reference order. A warp covers 32/S clusters of one
// subspace; lane = (cluster j, coordinate k) runs one sequential f32 chain.
// Cluster members stream through a cp.async ring in shared memory
// (kChainE elements per cluster per stage). Empty clusters are left for the
// reseed kernel.
// ---------------------------------------------------------------------------
template <int S>
__global__ void __launch_bounds__(kChainWarps * 32)
pq_chain_kernel(const float* __restrict__ sorted, uint64_t N, int M, int K,
                const uint32_t* __restrict__ counts, const uint32_t* __restrict__ starts,
                float* __restrict__ cb, const uint8_t* __restrict__ state,
                const float* __restrict__ start_sums, int raw) {
  constexpr int CPW = 32 / S;              // clusters per warp
  constexpr int kRow = kChainE * S + S;    // padded: conflict-free reads
  constexpr int kStage = CPW * kRow;
  extern __shared__ __align__(16) float ring_all[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* ring = ring_all + (size_t)warp * kChainStages * kStage;
  const int wpm = (K + CPW - 1) / CPW;
  const int gw = blockIdx.x * kChainWarps + warp;
  if (gw >= M * wpm) return;
  const int m = gw / wpm;
  if (state[m] != kRunning) return;
  const int j = lane / S, k = lane % S;
  const int c = (gw % wpm) * CPW + j;
  const uint32_t cnt = c < K ? counts[(size_t)m * K + c] : 0u;
  const uint32_t st = c < K ? starts[(size_t)m * K + c] : 0u;
  uint32_t maxcnt = cnt;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) maxcnt = max(maxcnt, __shfl_xor_sync(0xffffffffu, maxcnt, o));
  const int nst = (int)((maxcnt + kChainE - 1) / kChainE);
  const float* sm = sorted + (size_t)m * N * S;

  auto issue = [&](int t) {
    if (t < nst) {
      float* dstage = ring + (t % kChainStages) * kStage;
      for (int jj = 0; jj < CPW; ++jj) {
        const uint32_t cj = __shfl_sync(0xffffffffu, cnt, jj * S);
        const uint32_t sj = __shfl_sync(0xffffffffu, st, jj * S);
        for (int e = lane; e < kChainE; e += 32) {
          const uint32_t g = (uint32_t)t * kChainE + e;
          if (g < cj) cp_async<4 * S>(dstage + jj * kRow + e * S, sm + (size_t)(sj + g) * S);
        }
      }
    }
    cp_async_commit();
  };

  // a row-sharded run continues the previous rank's running sums
  float acc = (start_sums && c < K) ? start_sums[((size_t)m * K + c) * S + k] : 0.f;
  for (int t = 0; t < kChainStages - 1; ++t) issue(t);
  for (int t = 0; t < nst; ++t) {
    cp_async_wait<kChainStages - 2>();
    __syncwarp();
    const float* src = ring + (t % kChainStages) * kStage + j * kRow + k;
    const uint32_t done = (uint32_t)t * kChainE;
    const int n = cnt > done ? (int)min((uint32_t)kChainE, cnt - done) : 0;
    int e = 0;
    for (; e + 8 <= n; e += 8) {  // loads first, then the dependent adds
      float v[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) v[q] = src[(e + q) * S];
#pragma unroll
      for (int q = 0; q < 8; ++q) acc = __fadd_rn(acc, v[q]);
    }
    for (; e < n; ++e) acc = __fadd_rn(acc, src[e * S]);
    __syncwarp();
    issue(t + kChainStages - 1);
  }
  cp_async_wait<0>();
  if (c < K && raw) {
    cb[((size_t)m * K + c) * S + k] = acc;  // running sums for the next rank
  } else if (c < K && cnt > 0) {
    const float inv = __fdiv_rn(1.0f, __uint2float_rn(cnt));
    cb[((size_t)m * K + c) * S + k] = __fmul_rn(acc, inv);
  }
}

// The same chains for 16-byte sub-vectors (S = 4), fed by bulk copies from a
// producer warp. A CTA is one consumer warp (8 clusters of one subspace, lane
// = (cluster j, coordinate k), one sequential f32 chain per lane, members
// added in the order of the sorted copy, as pq_chain_kernel adds them) and
// one producer warp. A cluster's members are one contiguous run of 16-byte
// rows in the sorted copy, so a ring stage of a cluster (kChainE members) is
// one cp.async.bulk; the producer's lane 0 announces each stage's bytes on
// the stage's `full` mbarrier and issues the stage's copies, and waits on the
// stage's `empty` mbarrier (released by the consumer) before it refills a
// slot. The copies thus never hold up the sequential adds, which read full
// stages through a fully unrolled loop. Every wait is bounded: a wait that
// expires sets diag[3], the consumer leaves without writing its clusters,
// and the producer waits (bounded) for the copies it issued before it leaves.
constexpr int kChainBulkMaxStages = 13;
constexpr int kChainBulkRow = kChainE * 4 + 4;                  // floats per cluster per stage (+16 B: banks)
constexpr int kChainBulkStage = 8 * kChainBulkRow;              // floats per stage (8 clusters)
constexpr int kChainBulkBarBytes = 2 * kChainBulkMaxStages * 8 + 16;  // full, empty, abort flag (16 B aligned)

__device__ __forceinline__ void mbar_expect_arrive(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(tc::smem_addr(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_g2s(void* smem, const void* gmem, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
          tc::smem_addr(smem)),
      "l"(gmem), "r"(bytes), "r"(tc::smem_addr(bar))
      : "memory");
}

__global__ void __launch_bounds__(64)
pq_chain_bulk_kernel(const float* __restrict__ sorted, uint64_t N, int M, int K,
                     const uint32_t* __restrict__ counts, const uint32_t* __restrict__ starts,
                     float* __restrict__ cb, const uint8_t* __restrict__ state,
                     const float* __restrict__ start_sums, int raw, int stages, uint32_t* __restrict__ diag) {
  constexpr int S = 4, CPW = 8;
  extern __shared__ __align__(128) unsigned char chain_smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(chain_smem);
  uint64_t* empty = full + kChainBulkMaxStages;
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(empty + kChainBulkMaxStages);
  float* ring = reinterpret_cast<float*>(chain_smem + kChainBulkBarBytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wpm = (K + CPW - 1) / CPW;
  const int gw = blockIdx.x;
  if (gw >= M * wpm) return;  // whole CTA
  const int m = gw / wpm;
  if (state[m] != kRunning) return;  // whole CTA
  if (threadIdx.x == 0) {
    for (int q = 0; q < stages; ++q) {
      tc::mbar_init(&full[q], 1);
      tc::mbar_init(&empty[q], 1);
    }
    *abort_flag = 0u;
  }
  __syncthreads();
  const int c0 = (gw % wpm) * CPW;

  if (warp == 1) {  // producer: lane 0 issues every copy
    if (lane != 0) return;
    uint32_t cj[CPW], sj[CPW], maxcnt = 0;
#pragma unroll
    for (int q = 0; q < CPW; ++q) {
      cj[q] = c0 + q < K ? counts[(size_t)m * K + c0 + q] : 0u;
      sj[q] = c0 + q < K ? starts[(size_t)m * K + c0 + q] : 0u;
      maxcnt = max(maxcnt, cj[q]);
    }
    const int nst = (int)((maxcnt + kChainE - 1) / kChainE);
    const float* sm = sorted + (size_t)m * N * S;
    int slot = 0, issued = 0;
    uint32_t phase = 0;
    for (int t = 0; t < nst; ++t) {
      if (*abort_flag) break;
      if (t >= stages && !tc::mbar_wait(&empty[slot], phase ^ 1u)) {
        atomicExch(&diag[3], 1u);
        break;
      }
      const uint32_t g0 = (uint32_t)t * kChainE;
      uint32_t total = 0;
#pragma unroll
      for (int q = 0; q < CPW; ++q) total += cj[q] > g0 ? min((uint32_t)kChainE, cj[q] - g0) * 16u : 0u;
      mbar_expect_arrive(&full[slot], total);
      float* dst = ring + (size_t)slot * kChainBulkStage;
#pragma unroll
      for (int q = 0; q < CPW; ++q)
        if (cj[q] > g0)
          bulk_g2s(dst + q * kChainBulkRow, sm + (size_t)(sj[q] + g0) * S, min((uint32_t)kChainE, cj[q] - g0) * 16u,
                   &full[slot]);
      ++issued;
      if (++slot == stages) {
        slot = 0;
        phase ^= 1u;
      }
    }
    // the last copies of each slot have landed before the CTA may leave
    for (int u = max(0, issued - stages); u < issued; ++u)
      if (!tc::mbar_wait(&full[u % stages], (uint32_t)(u / stages) & 1u)) atomicExch(&diag[3], 1u);
    return;
  }

  // consumer
  const int j = lane >> 2, k = lane & 3;
  const int c = c0 + j;
  const uint32_t cnt = c < K ? counts[(size_t)m * K + c] : 0u;
  const uint32_t maxcnt = __reduce_max_sync(0xffffffffu, cnt);
  const int nst = (int)((maxcnt + kChainE - 1) / kChainE);
  // a row-sharded run continues the previous rank's running sums
  float acc = (start_sums && c < K) ? start_sums[((size_t)m * K + c) * S + k] : 0.f;
  int slot = 0;
  uint32_t phase = 0;
  for (int t = 0; t < nst; ++t) {
    if (!__all_sync(0xffffffffu, tc::mbar_wait(&full[slot], phase))) {
      if (lane == 0) {
        atomicExch(&diag[3], 1u);
        *abort_flag = 1u;
      }
      return;
    }
    const float* src = ring + (size_t)slot * kChainBulkStage + j * kChainBulkRow + k;
    const uint32_t done = (uint32_t)t * kChainE;
    const int n = cnt > done ? (int)min((uint32_t)kChainE, cnt - done) : 0;
    if (n == kChainE) {
#pragma unroll
      for (int e = 0; e < kChainE; ++e) acc = __fadd_rn(acc, src[e * S]);
    } else {
      int e = 0;
      for (; e + 8 <= n; e += 8) {
        float v[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) v[q] = src[(e + q) * S];
#pragma unroll
        for (int q = 0; q < 8; ++q) acc = __fadd_rn(acc, v[q]);
      }
      for (; e < n; ++e) acc = __fadd_rn(acc, src[e * S]);
    }
    __syncwarp();
    if (lane == 0) tc::mbar_arrive(&empty[slot]);
    if (++slot == stages) {
      slot = 0;
      phase ^= 1u;
    }
  }
  if (c < K && raw) {
    cb[((size_t)m * K + c) * S + k] = acc;  // running sums for the next rank
  } else if (c < K && cnt > 0) {
    const float inv = __fdiv_rn(1.0f, __uint2float_rn(cnt));
    cb[((size_t)m * K + c) * S + k] = __fmul_rn(acc, inv);
  }
}

// ---------------------------------------------------------------------------
// Sequential f32 WCSS of one subspace (kmeans.zig:179), row order.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
pq_wcss_kernel(const float* __restrict__ mind, uint64_t N, float* __restrict__ wcss,
               const uint8_t* __restrict__ state, const float* __restrict__ start) {
  const int m = blockIdx.x;
  if (state[m] != kRunning) return;
  __shared__ __align__(16) float tile[4096];
  const float* src = mind + (size_t)m * N;
  float acc = start ? start[m] : 0.f;  // a row-sharded run continues the previous rank's sum
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
pq_reseed_converge_kernel(const float* __restrict__ XT, uint64_t N, int S, int K,
                          const uint32_t* __restrict__ counts, float* __restrict__ mind,
                          float* __restrict__ cb, uint8_t* __restrict__ state,
                          const float* __restrict__ wcss, float* __restrict__ prev_wcss,
                          uint32_t* __restrict__ iters_run, uint32_t* __restrict__ reseeds,
                          int iter, int check, float tol, int do_reseed,
                          const uint32_t* __restrict__ list_cnt, unsigned long long* __restrict__ exact) {
  const int m = blockIdx.x;
  if (state[m] != kRunning) return;
  __shared__ int any_empty;
  if (threadIdx.x == 0) any_empty = 0;
  __syncthreads();
  if (do_reseed)
    for (int c = threadIdx.x; c < K; c += blockDim.x)
      if (counts[(size_t)m * K + c] == 0) atomicOr(&any_empty, 1);
  __syncthreads();
  if (any_empty) {
    float* mm = mind + (size_t)m * N;
    for (int c = 0; c < K; ++c) {
      if (counts[(size_t)m * K + c] != 0) continue;
      const uint64_t far = block_argmax_first(mm, N);
      if (threadIdx.x < (unsigned)S)
        cb[((size_t)m * K + c) * S + threadIdx.x] = XT[((size_t)m * N + far) * S + threadIdx.x];
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
    // rows of this iteration whose distances were all computed (stats)
    if (exact) exact[m] += list_cnt ? list_cnt[m] : N;
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
__global__ void pq_seed_init_kernel(const float* __restrict__ XT, uint64_t N, int S, int K,
                                    const uint64_t* __restrict__ idx0, float* __restrict__ cb,
                                    uint64_t* __restrict__ chosen) {
  const int m = blockIdx.x;
  if (threadIdx.x < (unsigned)S)
    cb[(size_t)m * K * S + threadIdx.x] = XT[((size_t)m * N + idx0[m]) * S + threadIdx.x];
  if (threadIdx.x == 0) chosen[(size_t)m * K] = idx0[m];
}

// min_dist update with centroid `step` (kmeans.zig:117-135), fused with the
// per-chunk directed-rounding sums of the new weights and the count of
// non-zero weights below thr[m] (the weights whose f64 addition may round,
// see pq_seed_select_kernel).
template <int S>
__global__ void __launch_bounds__(kSeedThreads)
pq_seed_update_kernel(const float* __restrict__ XT, uint64_t N, int M, int K, int step,
                      const float* __restrict__ cb, float* __restrict__ md,
                      double2* __restrict__ chunk, uint32_t* __restrict__ chunk_cnt,
                      int* __restrict__ nonfinite, const uint8_t* __restrict__ state,
                      const double* __restrict__ thr, int chunk_stride) {
  __shared__ double2 wp[kSeedThreads / 32][kMaxM];
  __shared__ uint32_t wc[kSeedThreads / 32][kMaxM];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nchunk = chunk_stride;  // chunk b of subspace m at m * chunk_stride + b
  for (int m = 0; m < M; ++m) {
    if (state[m] != kRunning) continue;
    float c[S];
#pragma unroll
    for (int k = 0; k < S; ++k) c[k] = cb[((size_t)m * K + step) * S + k];
    const double T = thr[m];
    double lo = 0.0, hi = 0.0;
    uint32_t cnt = 0;
    bool bad = false;
#pragma unroll
    for (int u = 0; u < kSeedRowsPerThread; ++u) {
      const uint64_t r = (uint64_t)blockIdx.x * kSeedChunk + (uint64_t)u * kSeedThreads + threadIdx.x;
      if (r < N) {
        float x[S];
        load_sub<S>(XT + ((size_t)m * N + r) * S, x);
        const float d = l2_small<S>(x, c);
        float* slot = md + (size_t)m * N + r;
        float w;
        if (step == 0) {
          w = d;
          *slot = w;
        } else {
          const float old = *slot;
          w = d < old ? d : old;
          if (__float_as_uint(w) != __float_as_uint(old)) *slot = w;  // stored only when it changes
        }
        bad |= !isfinite(w) || w < 0.f;
        lo = __dadd_rd(lo, (double)w);
        hi = __dadd_ru(hi, (double)w);
        cnt += (w != 0.f && (double)w < T) ? 1u : 0u;
      }
    }
    if (bad) nonfinite[m] = 1;
    lo = warp_sum_rd(lo);
    hi = warp_sum_ru(hi);
    cnt = __reduce_add_sync(0xffffffffu, cnt);
    if (lane == 0) {
      wp[warp][m] = make_double2(lo, hi);
      wc[warp][m] = cnt;
    }
  }
  __syncthreads();
  for (int m = threadIdx.x; m < M; m += kSeedThreads) {
    if (state[m] != kRunning) continue;
    double lo = 0.0, hi = 0.0;
    uint32_t cnt = 0;
    for (int w = 0; w < kSeedThreads / 32; ++w) {
      lo = __dadd_rd(lo, wp[w][m].x);
      hi = __dadd_ru(hi, wp[w][m].y);
      cnt += wc[w][m];
    }
    chunk[(size_t)m * nchunk + blockIdx.x] = make_double2(lo, hi);
    chunk_cnt[(size_t)m * nchunk + blockIdx.x] = cnt;
  }
}

// The same update with one warp per subspace (block = 32 x M threads, one
// 1024-row chunk per CTA): lane l takes rows l, l + 32, ... of the chunk in
// batches of 8 (every load of a batch goes out before the first store), so
// each subspace's chunk sums need one warp reduction instead of one per warp
// and per subspace. A weight is stored only when it changes: after the first
// steps few rows move to the new centroid, so most of the pass only reads.
// A non-finite weight shows up as a non-finite chunk bound (weights are sums
// of squares, never negative). Odd steps walk the chunks in reverse order, so
// each pass starts on the rows and weights the previous pass left in L2
// (every chunk still writes its own sums: the results do not depend on it).
// Measured on B200 at 1.52M rows: 6.4 TB/s of row and weight reads for 16
// subspaces and 2, ahead of splitting a chunk over several warps per
// subspace (fewer rows in flight per warp, a block reduction, a partial
// last wave).
template <int S>
__global__ void __launch_bounds__(kMaxM * 32)
pq_seed_update_w_kernel(const float* __restrict__ XT, uint64_t N, int M, int K, int step,
                        const float* __restrict__ cb, float* __restrict__ md, double2* __restrict__ chunk,
                        uint32_t* __restrict__ chunk_cnt, int* __restrict__ nonfinite,
                        const uint8_t* __restrict__ state, const double* __restrict__ thr, int chunk_stride) {
  constexpr int kB = 8;
  grid_dependency_wait();  // launched early (programmatic dependent launch): the last step completes first
  const int lane = threadIdx.x & 31, m = threadIdx.x >> 5;
  if (m >= M || state[m] != kRunning) return;
  float c[S];
#pragma unroll
  for (int k = 0; k < S; ++k) c[k] = cb[((size_t)m * K + step) * S + k];
  const double T = thr[m];
  const uint32_t ch = (step & 1) ? gridDim.x - 1 - blockIdx.x : blockIdx.x;
  const uint64_t r0 = (uint64_t)ch * kSeedChunk;
  const float* xm = XT + (size_t)m * N * S;
  float* mm = md + (size_t)m * N;
  double lo = 0.0, hi = 0.0;
  uint32_t cnt = 0;
  for (int q0 = 0; q0 < kSeedChunk / 32; q0 += kB) {
    float x[kB][S], old[kB];
#pragma unroll
    for (int b = 0; b < kB; ++b) {
      const uint64_t r = r0 + (uint64_t)((q0 + b) * 32 + lane);
      if (r < N) {
        load_sub<S>(xm + r * S, x[b]);
        old[b] = step == 0 ? 0.f : mm[r];
      }
    }
#pragma unroll
    for (int b = 0; b < kB; ++b) {
      const uint64_t r = r0 + (uint64_t)((q0 + b) * 32 + lane);
      if (r < N) {
        const float d = l2_small<S>(x[b], c);
        const float w = step == 0 ? d : fminf(d, old[b]);  // the old weight when d is NaN
        if (step == 0 || __float_as_uint(w) != __float_as_uint(old[b])) mm[r] = w;
        lo = __dadd_rd(lo, (double)w);
        hi = __dadd_ru(hi, (double)w);
        cnt += (w != 0.f && (double)w < T) ? 1u : 0u;
      }
    }
  }
  lo = warp_sum_rd(lo);
  hi = warp_sum_ru(hi);
  cnt = __reduce_add_sync(0xffffffffu, cnt);
  if (lane == 0) {
    chunk[(size_t)m * chunk_stride + ch] = make_double2(lo, hi);
    chunk_cnt[(size_t)m * chunk_stride + ch] = cnt;
    if (!isfinite(lo) || !isfinite(hi)) nonfinite[m] = 1;
  }
}

// Upper bound of gamma_n = n u / (1 - n u), u = 2^-53: the recursive
// summation error bound |S_n - E_n| <= gamma_{n-1} * sum |w_i| (Higham,
// "Accuracy and Stability of Numerical Algorithms", 2nd ed., eq. 4.4).
__device__ __forceinline__ double gamma_bound(uint64_t n) {
  const double g = __dmul_ru(__ull2double_ru(n), 1.1102230246251565e-16);
  return __ddiv_ru(g, __dsub_rd(1.0, g));
}

// ---------------------------------------------------------------------------
// The reference's sequential f64 sum of the weights, exactly, by one CTA
// (weightedSample, rng.zig:57-82), for draws the interval bounds cannot
// decide when N is large (the bounds widen with N; one thread running the
// chain over tens of millions of weights takes a large fraction of a
// second).
//
// A running f64 sum S in the binade [2^e, 2^(e+1)) is K u with u = 2^(e-52)
// and K an integer. While S + w stays in that binade, fl(S + w) = (K + g) u,
// g = w / u rounded to nearest: a function of w and e alone unless w's part
// below u is exactly u / 2 (a tie), where round-half-even adds the parity
// of K + floor(w / u); after a tie K is even. So each row maps the parity
// of K to (new parity, g): flip or keep for a row without a tie, reset to
// even for a tie, and a chunk's rows compose into one such map (two
// (parity, G) pairs, for an even and an odd incoming K), built by a warp
// scan. A chunk is clean when its sums provably stay in one binade (the
// directed-rounding prefix bounds widened by the classic recursive-sum
// error bound gamma_N sum w); one thread then walks the chunks applying
// each clean chunk's map to the exact running S (an exact add of G u) and
// adding the weights of the few other chunks (binade crossings) one by one
// in the reference's order. The exact chunk-end sums locate the first row
// with u_draw < S_i.
// ---------------------------------------------------------------------------
constexpr uint64_t kExactChunkedMinRows = 1u << 18;  // smaller N: the one-thread chain

// A row's (or chunk's) map on the parity of K: for an incoming parity p,
// K grows by add[p] and leaves with parity out[p].
struct ParMap {
  unsigned long long add0, add1;
  uint32_t out0, out1;
};

__device__ __forceinline__ ParMap parmap_identity() { return ParMap{0ull, 0ull, 0u, 1u}; }

// first then second
__device__ __forceinline__ ParMap parmap_then(const ParMap& f, const ParMap& s) {
  ParMap r;
  r.add0 = f.add0 + (f.out0 ? s.add1 : s.add0);
  r.out0 = f.out0 ? s.out1 : s.out0;
  r.add1 = f.add1 + (f.out1 ? s.add1 : s.add0);
  r.out1 = f.out1 ? s.out1 : s.out0;
  return r;
}

// The map of adding w >= 0 to a sum in binade e.
__device__ __forceinline__ ParMap parmap_row(float w, int e) {
  const uint32_t b = __float_as_uint(w);
  const int be = (int)(b >> 23);
  const uint64_t mant = be ? (uint64_t)((b & 0x7FFFFFu) | 0x800000u) : (uint64_t)(b & 0x7FFFFFu);
  const int E = be ? be - 127 : -126;  // w = mant * 2^(E - 23)
  const int sh = E - 23 + 52 - e;      // w / u = mant * 2^sh
  uint64_t g = 0;
  if (mant != 0) {
    if (sh >= 0) {
      g = mant << sh;  // the chunk stays below 2^(e+1): g < 2^53
    } else if (-sh <= 25) {  // below: w / u < 1/4, rounds to 0
      const int rs = -sh;
      const uint64_t q = mant >> rs;
      const uint64_t frac = mant & ((1ull << rs) - 1);
      const uint64_t half = 1ull << (rs - 1);
      if (frac == half) {  // tie: even K + q stays, odd rounds up; K leaves even
        const uint64_t q1 = q & 1ull;
        return ParMap{q + q1, q + (q1 ^ 1ull), 0u, 0u};
      }
      g = frac > half ? q + 1 : q;
    }
  }
  const uint32_t gb = (uint32_t)(g & 1ull);
  return ParMap{g, g, gb, 1u ^ gb};
}

// Called by all kSelectThreads threads of the CTA of subspace m. ex_lo /
// ex_hi: this thread's exclusive prefix bounds at chunk c_lo. Returns the
// reference's pick (valid in every thread).
__device__ __noinline__ uint64_t exact_chain_draw(const float* __restrict__ w, uint64_t N, const double2* __restrict__ ch,
                                                  int nchunk, int c_lo, int c_hi, double ex_lo, double ex_hi,
                                                  double B, double r, double2* __restrict__ xpre,
                                                  ulonglong2* __restrict__ xg, int* __restrict__ xe) {
  __shared__ unsigned long long s_last;
  __shared__ int s_first;
  __shared__ double s_total;
  __shared__ uint64_t s_pick;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    s_last = 0;
    s_first = nchunk;
  }
  // 1a. exclusive prefix bounds of every chunk
  {
    double lo = ex_lo, hi = ex_hi;
    for (int c = c_lo; c < c_hi; ++c) {
      xpre[c] = make_double2(lo, hi);
      lo = __dadd_rd(lo, ch[c].x);
      hi = __dadd_ru(hi, ch[c].y);
    }
  }
  __syncthreads();
  // 1b. per chunk (one warp each): its binade if it provably stays in one,
  // and the chunk's parity map (xe = e | out0 << 16 | out1 << 17, or
  // INT_MIN to chain it); the last non-zero weight
  unsigned long long last = 0;
  for (int c = warp; c < nchunk; c += kSelectThreads / 32) {
    const double2 pre = xpre[c];
    const double lo_s = __dsub_rd(pre.x, B);
    const double hi_e = __dadd_ru(__dadd_ru(pre.y, ch[c].y), B);
    int e = INT_MIN;
    if (lo_s >= 0x1p-1022) {
      const int e0 = ilogb(lo_s);
      if (hi_e < ldexp(1.0, e0 + 1)) e = e0;
    }
    const uint64_t r0 = (uint64_t)c * kSeedChunk, r1 = min(N, r0 + kSeedChunk);
    ParMap acc = parmap_identity();
    for (uint64_t i0 = r0; i0 < r1; i0 += 32) {
      const uint64_t i = i0 + lane;
      const float v = i < r1 ? w[i] : 0.f;
      if (v != 0.f) last = max(last, (unsigned long long)i);
      if (e == INT_MIN) continue;  // warp-uniform
      ParMap f = parmap_row(v, e);
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {  // inclusive scan of the maps in row order
        ParMap p;
        p.add0 = __shfl_up_sync(0xffffffffu, f.add0, o);
        p.add1 = __shfl_up_sync(0xffffffffu, f.add1, o);
        p.out0 = __shfl_up_sync(0xffffffffu, f.out0, o);
        p.out1 = __shfl_up_sync(0xffffffffu, f.out1, o);
        if (lane >= o) f = parmap_then(p, f);
      }
      ParMap t;
      t.add0 = __shfl_sync(0xffffffffu, f.add0, 31);
      t.add1 = __shfl_sync(0xffffffffu, f.add1, 31);
      t.out0 = __shfl_sync(0xffffffffu, f.out0, 31);
      t.out1 = __shfl_sync(0xffffffffu, f.out1, 31);
      acc = parmap_then(acc, t);
    }
    if (lane == 0) {
      xg[c] = make_ulonglong2(acc.add0, acc.add1);
      xe[c] = e == INT_MIN ? INT_MIN : (int)((uint32_t)(e & 0xFFFF) | (acc.out0 << 16) | (acc.out1 << 17));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) last = max(last, __shfl_xor_sync(0xffffffffu, last, o));
  if (lane == 0) atomicMax(&s_last, last);
  __syncthreads();
  // 2. one thread: exact chunk-end sums (xpre[c].x), in the reference's
  //    order; the per-chunk maps are staged in shared memory a tile at a time
  constexpr int kTile = 1024;
  __shared__ ulonglong2 s_add[kTile];
  __shared__ int s_e[kTile];
  double S = 0.0;
  for (int t0 = 0; t0 < nchunk; t0 += kTile) {
    const int tn = min(kTile, nchunk - t0);
    for (int q = tid; q < tn; q += kSelectThreads) {
      s_add[q] = xg[t0 + q];
      s_e[q] = xe[t0 + q];
    }
    __syncthreads();
    if (tid == 0) {
      for (int q = 0; q < tn; ++q) {
        const int x = s_e[q];
        if (x != INT_MIN) {
          const int e = (int)(int16_t)(x & 0xFFFF);
          const uint64_t K0 = (uint64_t)ldexp(S, 52 - e);  // S = K0 * 2^(e-52) exactly
          const ulonglong2 a = s_add[q];
          S = __dadd_rn(S, ldexp((double)((K0 & 1ull) ? a.y : a.x), e - 52));  // exact: same binade
        } else {
          const uint64_t r0 = (uint64_t)(t0 + q) * kSeedChunk, r1 = min(N, r0 + kSeedChunk);
          uint64_t i = r0;
          for (; i + 8 <= r1; i += 8) {
            float v[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) v[k] = w[i + k];
#pragma unroll
            for (int k = 0; k < 8; ++k) S = __dadd_rn(S, (double)v[k]);
          }
          for (; i < r1; ++i) S = __dadd_rn(S, (double)w[i]);
        }
        xpre[t0 + q].x = S;
      }
    }
    __syncthreads();
  }
  if (tid == 0) s_total = S;
  __syncthreads();
  // 3. the first chunk whose end sum exceeds u, then its rows in order
  const double u = __dmul_rn(r, s_total);
  int first = nchunk;
  for (int c = c_lo; c < c_hi; ++c)
    if (u < xpre[c].x) { first = c; break; }
  if (first < nchunk) atomicMin(&s_first, first);
  __syncthreads();
  if (tid == 0) {
    uint64_t pick = s_last;  // the reference's fallback: last positive weight
    const int c = s_first;
    if (c < nchunk) {
      double Sc = c > 0 ? xpre[c - 1].x : 0.0;
      const uint64_t r0 = (uint64_t)c * kSeedChunk, r1 = min(N, r0 + kSeedChunk);
      for (uint64_t i = r0; i < r1; ++i) {
        Sc = __dadd_rn(Sc, (double)w[i]);
        if (u < Sc) { pick = i; break; }
      }
    }
    s_pick = pick;
  }
  __syncthreads();
  return s_pick;
}

// Draw for centroid `step` (weightedSample, rng.zig:57-82).
//
// The reference returns the first i with u < S_i, where S_i is the
// sequential f64 sum of the first i+1 weights and u = fl(r * S_N). Here:
//   * Lo_i <= E_i <= Hi_i bound the exact prefix E_i (directed rounding);
//   * |S_i - E_i| <= B, with B the smaller of the classic gamma bound and a
//     tighter one: an f64 add of a non-negative f32 weight w to a sum whose
//     binade does not change is exact unless w has bits below the sum's
//     ulp, which needs w < 2^23 * G with G = 2^(E-52) the largest ulp any
//     prefix can have (E = exponent of an upper bound of S_N). So at most
//     (#weights below 2^23 G) + (#binade crossings) adds round, each by at
//     most G/2. The weights are counted below the previous draw's threshold
//     (weights never grow between draws), and the tight bound is used only
//     when that threshold covers the current one;
//   * the candidate row is accepted when u's interval lies strictly between
//     the intervals of S_{i-1} and S_i. Otherwise one thread runs the
//     reference's sequential chain.
__global__ void __launch_bounds__(kSelectThreads)
pq_seed_select_kernel(const float* __restrict__ XT, uint64_t N, int S, int K, int step,
                      float* __restrict__ cb, const float* __restrict__ md,
                      const double2* __restrict__ chunk, const uint32_t* __restrict__ chunk_cnt,
                      int nchunk, const double* __restrict__ draws, int* __restrict__ nonfinite,
                      int* __restrict__ status, uint8_t* __restrict__ state,
                      uint32_t* __restrict__ fallbacks, uint64_t* __restrict__ chosen,
                      double* __restrict__ thr, int force_chain, double2* __restrict__ xpre,
                      ulonglong2* __restrict__ xg, int* __restrict__ xe) {
  grid_dependency_wait();
  const int m = blockIdx.x;
  if (state[m] != kRunning) return;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int kWarps = kSelectThreads / 32;
  __shared__ double2 wsum[kWarps];
  __shared__ unsigned long long wcnt[kWarps];
  __shared__ double2 incl_all[kSelectThreads];
  __shared__ double2 sh_excl;
  __shared__ int sh_chunk;
  __shared__ uint64_t sh_idx;
  __shared__ int sh_decided;

  if (nonfinite[m]) {  // weightedSample validates every weight first
    if (tid == 0) { status[m] = MVR_E_NON_FINITE; state[m] = kFailed; }
    return;
  }
  const double2* ch = chunk + (size_t)m * nchunk;
  const uint32_t* cc = chunk_cnt + (size_t)m * nchunk;
  const float* w = md + (size_t)m * N;
  const double r = draws[(size_t)m * K + step];

  // 1. contiguous chunk ranges per thread, block scan of the totals
  const int cpt = (nchunk + kSelectThreads - 1) / kSelectThreads;
  const int c_lo = min(nchunk, tid * cpt), c_hi = min(nchunk, c_lo + cpt);
  double tlo = 0.0, thi = 0.0;
  unsigned tcnt = 0;
  for (int j = c_lo; j < c_hi; ++j) {
    tlo = __dadd_rd(tlo, ch[j].x);
    thi = __dadd_ru(thi, ch[j].y);
    tcnt += cc[j];
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
  if (Hi_N <= 0.0) {  // every weight is exactly zero
    if (tid == 0) { status[m] = MVR_E_ALL_ZERO; state[m] = kFailed; }
    return;
  }

  // 2. error bound of the sequential chain
  const double gN = gamma_bound(N);
  const double shi_classic = __dadd_ru(Hi_N, __dmul_ru(gN, Hi_N));
  int e2 = 0;
  (void)frexp(shi_classic, &e2);          // shi_classic < 2^e2
  const double G = ldexp(1.0, e2 - 53);   // >= ulp of every prefix
  const double thr_now = ldexp(G, 23);
  const double B_tight = __dmul_ru(__ull2double_ru(C_N + kCrossingSlack), 0.5 * G);
  const double thr_prev = thr[m];
  const bool tight_ok = thr_now <= thr_prev;
  auto bound_at = [&](uint64_t terms, double hi_prefix) {
    const double bg = __dmul_ru(gamma_bound(terms), hi_prefix);
    return tight_ok ? fmin(bg, B_tight) : bg;
  };

  const double u_mid = r * (0.5 * (Lo_N + Hi_N));
  const bool past = !(u_mid < 0.5 * (incl_lo + incl_hi));
  incl_all[tid] = make_double2(incl_lo, incl_hi);
  const int n_before = __syncthreads_count(past);  // prefixes are monotone
  // this thread's exclusive prefix bounds (incl_all is reused below)
  const double ex_lo = tid > 0 ? incl_all[tid - 1].x : 0.0, ex_hi = tid > 0 ? incl_all[tid - 1].y : 0.0;
  if (tid == 0) {
    sh_decided = 0;
    sh_chunk = -1;
    if (thr_now < thr_prev) thr[m] = thr_now;  // threshold for the next draw
  }
  __syncthreads();

  // 3. the first thread whose inclusive mid-prefix exceeds u_mid walks its
  //    chunks, starting from its predecessor's inclusive bounds.
  if (n_before < kSelectThreads && tid == n_before) {
    double lo = tid > 0 ? incl_all[tid - 1].x : 0.0;
    double hi = tid > 0 ? incl_all[tid - 1].y : 0.0;
    int found = -1;
    for (int j = c_lo; j < c_hi; ++j) {
      const double nlo = __dadd_rd(lo, ch[j].x), nhi = __dadd_ru(hi, ch[j].y);
      if (u_mid < 0.5 * (nlo + nhi)) { found = j; break; }
      lo = nlo;
      hi = nhi;
    }
    sh_chunk = found;
    sh_excl = make_double2(lo, hi);
  }
  __syncthreads();

  // 4. fine search inside the chunk: one thread per row, block scan
  const int fchunk = sh_chunk;
  if (fchunk >= 0) {
    const uint64_t i = (uint64_t)fchunk * kSeedChunk + tid;
    const double v = i < N ? (double)w[i] : 0.0;
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
    // Rows past N sort after every real row: counting them as hits keeps the
    // hits a suffix, and a first hit past N means no candidate.
    const bool hit = i >= N || u_mid < 0.5 * (elo + ehi);
    const int first = __syncthreads_count(!hit);
    if (first < kSelectThreads && tid == first && i < N) {
      const uint64_t istar = i;
      const double2 prv = tid > 0 ? incl_all[tid - 1] : ex;
      const double BN = bound_at(N, Hi_N);
      const double SLoN = __dsub_rd(Lo_N, BN);
      const double SHiN = __dadd_ru(Hi_N, BN);
      // u = fl(r * S_N) lies between the directed roundings of r * S_N.
      const double ULo = __dmul_rd(r, SLoN);
      const double UHi = __dmul_ru(r, SHiN);
      const double SLoI = __dsub_rd(elo, bound_at(istar + 1, ehi));
      bool ok = UHi < SLoI;
      if (istar > 0) {
        const double SHiP = __dadd_ru(prv.y, bound_at(istar, prv.y));
        ok = ok && (ULo >= SHiP);
      }
      if (ok && !force_chain) {
        sh_idx = istar;
        sh_decided = 1;
      }
    }
  }
  __syncthreads();

  // 5. undecided: the reference's sequential chain, exactly: chunked by the
  //    whole CTA for large N, by one thread otherwise.
  if (!sh_decided && N >= kExactChunkedMinRows) {
    const uint64_t pick = exact_chain_draw(w, N, ch, nchunk, c_lo, c_hi, ex_lo, ex_hi,
                                           __dmul_ru(gamma_bound(N), Hi_N), r, xpre + (size_t)m * nchunk,
                                           xg + (size_t)m * nchunk, xe + (size_t)m * nchunk);
    if (tid == 0) {
      sh_idx = pick;
      fallbacks[m] += 1;
    }
  } else if (!sh_decided && tid == 0) {
    double total = 0.0;
    uint64_t last_pos = 0;
    uint64_t i = 0;
    for (; i + 8 <= N; i += 8) {
      float v[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) v[q] = w[i + q];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        total = __dadd_rn(total, (double)v[q]);
        if (v[q] != 0.f) last_pos = i + q;
      }
    }
    for (; i < N; ++i) {
      total = __dadd_rn(total, (double)w[i]);
      if (w[i] != 0.f) last_pos = i;
    }
    const double u = __dmul_rn(r, total);
    double cum = 0.0;
    uint64_t pick = last_pos;  // the reference's fallback: last positive weight
    bool got = false;
    for (i = 0; i + 8 <= N && !got; i += 8) {
      float v[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) v[q] = w[i + q];
      for (int q = 0; q < 8; ++q) {
        cum = __dadd_rn(cum, (double)v[q]);
        if (u < cum) { pick = i + q; got = true; break; }
      }
    }
    for (; i < N && !got; ++i) {
      cum = __dadd_rn(cum, (double)w[i]);
      if (u < cum) { pick = i; got = true; }
    }
    sh_idx = pick;
    fallbacks[m] += 1;
  }
  __syncthreads();
  const uint64_t idx = sh_idx;
  if (tid < S) cb[((size_t)m * K + step) * S + tid] = XT[((size_t)m * N + idx) * S + tid];
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

// ---------------------------------------------------------------------------
// host-side launch helpers
// ---------------------------------------------------------------------------
size_t assign_smem(int M, int K, int S, int mode) {
  size_t b = (size_t)M * ((K + 1) / 2) * S * sizeof(float2);
  if (mode == kModeLloyd) b += (size_t)M * K * sizeof(uint32_t);
  return b;
}

template <int S>
int launch_assign(Ctx* ctx, cudaStream_t st, int mode, const float* R, const float* XT, uint64_t N,
                  int D, int M, int K, const float* cb, uint8_t* codes, uint8_t* asg, float* mind,
                  uint32_t* hist, const uint8_t* state, int nblk, uint64_t rows_per_cta,
                  float* ubnd = nullptr, float* lbnd = nullptr) {
  const size_t sm = assign_smem(M, K, S, mode);
  if (mode == kModeLloyd && ubnd) {
    auto kern = pq_assign_kernel<S, kModeLloyd, true>;
    MVR_CUDA(ctx, raise_smem_limit((const void*)kern, (size_t)(sm)));
    kern<<<nblk, kAsgThreads, sm, st>>>(R, XT, N, D, M, K, cb, codes, asg, mind, hist, state, 1.0f, rows_per_cta,
                                        ubnd, lbnd);
  } else if (mode == kModeLloyd) {
    auto kern = pq_assign_kernel<S, kModeLloyd, false>;
    MVR_CUDA(ctx, raise_smem_limit((const void*)kern, (size_t)(sm)));
    kern<<<nblk, kAsgThreads, sm, st>>>(R, XT, N, D, M, K, cb, codes, asg, mind, hist, state, 1.0f, rows_per_cta,
                                        nullptr, nullptr);
  } else {
    auto kern = pq_assign_kernel<S, kModeEncode, false>;
    MVR_CUDA(ctx, raise_smem_limit((const void*)kern, (size_t)(sm)));
    kern<<<nblk, kAsgThreads, sm, st>>>(R, XT, N, D, M, K, cb, codes, asg, mind, hist, state, 1.0f, rows_per_cta,
                                        nullptr, nullptr);
  }
  MVR_CUDA(ctx, cudaGetLastError());
  return MVR_OK;
}

// Tensor-core filtered pass (persistent: one CTA per SM, two accumulators).
template <int S>
int launch_tc_assign(Ctx* ctx, cudaStream_t st, int mode, bool use_list, const float* R, const float* XT,
                     uint64_t N, int D, int M, int K, const float* cb, const uint32_t* list, const uint32_t* lcnt,
                     uint8_t* codes, uint8_t* asg, float* mind, float* ubnd, float* lbnd, const uint8_t* state,
                     uint32_t* diag, int sms) {
  const int grid = std::max(1, sms);
#define MVR_TC_LAUNCH(MODE_, LIST_)                                                                            \
  {                                                                                                            \
    auto k = pq_tc_assign_kernel<S, MODE_, LIST_>;                                                             \
    MVR_CUDA(ctx, raise_smem_limit((const void*)k, (size_t)(kTcSmemBytes)));    \
    k<<<grid, kTcBlock, kTcSmemBytes, st>>>(R, XT, N, D, M, K, cb, list, lcnt, codes, asg, mind, ubnd, lbnd, state, \
                                            diag);                                                             \
  }
  if (mode == kModeEncode) MVR_TC_LAUNCH(kModeEncode, false)
  else if (use_list) MVR_TC_LAUNCH(kModeLloyd, true)
  else MVR_TC_LAUNCH(kModeLloyd, false)
#undef MVR_TC_LAUNCH
  MVR_CUDA(ctx, cudaGetLastError());
  return MVR_OK;
}

template <int S>
int launch_chain(Ctx* ctx, cudaStream_t st, const float* sorted, uint64_t N, int M, int K,
                 const uint32_t* counts, const uint32_t* starts, float* cb, const uint8_t* state,
                 uint32_t* diag, int sm_count, const float* start_sums = nullptr, int raw = 0) {
  constexpr int CPW = 32 / S;
  if constexpr (S == 4) {
    // one consumer warp (+ its producer warp) per CTA; the ring is as deep as
    // the shared memory of the CTAs an SM must hold at once allows
    const int ctas = M * ((K + CPW - 1) / CPW);
    const int per_sm = std::max(1, (ctas + std::max(1, sm_count) - 1) / std::max(1, sm_count));
    const size_t stage_bytes = (size_t)kChainBulkStage * sizeof(float);
    const size_t fit = (227 * 1024 / (size_t)per_sm - kChainBulkBarBytes) / stage_bytes;
    const int stages = (int)std::max<size_t>(2, std::min<size_t>(kChainBulkMaxStages, fit));
    const size_t sm = kChainBulkBarBytes + (size_t)stages * stage_bytes;
    MVR_CUDA(ctx, raise_smem_limit((const void*)pq_chain_bulk_kernel, (size_t)(sm)));
    pq_chain_bulk_kernel<<<ctas, 64, sm, st>>>(sorted, N, M, K, counts, starts, cb, state, start_sums, raw, stages,
                                               diag);
    MVR_CUDA(ctx, cudaGetLastError());
    return MVR_OK;
  }
  const size_t sm = (size_t)kChainWarps * kChainStages * CPW * (kChainE * S + S) * sizeof(float);
  auto kern = pq_chain_kernel<S>;
  MVR_CUDA(ctx, raise_smem_limit((const void*)kern, (size_t)(sm)));
  const int warps = M * ((K + CPW - 1) / CPW);
  const int grid = (warps + kChainWarps - 1) / kChainWarps;
  kern<<<grid, kChainWarps * 32, sm, st>>>(sorted, N, M, K, counts, starts, cb, state, start_sums, raw);
  MVR_CUDA(ctx, cudaGetLastError());
  return MVR_OK;
}

int check_shape(Ctx* ctx, int D, int M, int S, int K) {
  if (M <= 0 || S <= 0 || D != M * S) return fail(ctx, MVR_E_INVALID_ARGUMENT, "D must equal M*S");
  if (M > kMaxM) return fail(ctx, MVR_E_INVALID_ARGUMENT, "at most 32 subspaces per call");
  if (S != 1 && S != 2 && S != 4)
    return fail(ctx, MVR_E_INVALID_ARGUMENT, "sub-vector length must be 1, 2 or 4");
  if (K <= 0 || K > 256) return fail(ctx, MVR_E_INVALID_ARGUMENT, "K must be in [1, 256]");
  // Up to ~100 KB two CTAs share an SM; larger codebook sets (e.g. D = 128)
  // run one CTA per SM.
  if (assign_smem(M, K, S, kModeLloyd) > 220 * 1024)
    return fail(ctx, MVR_E_INVALID_ARGUMENT, "codebooks exceed shared memory");
  return MVR_OK;
}

// Persistent grid: two CTAs per SM, rows split evenly at warp granularity
// (every CTA gets the same number of 32-row groups, +-1).
void grid_for(uint64_t N, int sms, int* nblk, uint64_t* rows_per_cta) {
  const uint64_t groups = (N + 31) / 32;
  const uint64_t ctas = std::max<uint64_t>(1, std::min<uint64_t>(groups, (uint64_t)std::max(1, sms) * 2));
  *rows_per_cta = ((groups + ctas - 1) / ctas) * 32;
  *nblk = (int)((N + *rows_per_cta - 1) / *rows_per_cta);
}

// ---------------------------------------------------------------------------
// Row-sharded training: rank g holds global rows [row0_g, row0_g + N_g) in
// rank order. Every rank ends with the same codebooks as the one-GPU run:
//   * k-means++: per-chunk bounds of every rank are gathered, all ranks run
//     the same coarse search, the rank owning the chosen chunk resolves the
//     row and offers it (RowContrib) to the others;
//   * Lloyd: counts are summed; the in-order centroid sums run rank after
//     rank, each continuing the previous rank's running sums (the reference's
//     serial loop split at shard borders), and the last rank scales and
//     broadcasts; WCSS is continued the same way;
//   * the rare paths (the exact draw chain, empty-cluster reseeds) gather the
//     whole subspace and run the one-GPU logic on every rank.
// ---------------------------------------------------------------------------
struct RowContrib {
  uint32_t flag;  // 0: nothing; 1: row below; 2: the owner could not settle the draw
  uint32_t pad;
  uint64_t gidx;  // global row index
  float row[4];
};

// Offer row gidx[m] of subspace m when this rank holds it (want[m] != 0).
__global__ void pq_dist_offer_kernel(const float* __restrict__ XT, uint64_t N, int S, int M, uint64_t row0,
                                     const uint64_t* __restrict__ gidx, const uint32_t* __restrict__ want,
                                     RowContrib* __restrict__ contrib) {
  for (int m = threadIdx.x; m < M; m += blockDim.x) {
    RowContrib rc;
    rc.flag = 0;
    rc.pad = 0;
    rc.gidx = 0;
    for (int k = 0; k < 4; ++k) rc.row[k] = 0.f;
    const uint64_t g = gidx[m];
    if ((!want || want[m]) && g >= row0 && g < row0 + N) {
      rc.flag = 1;
      rc.gidx = g;
      for (int k = 0; k < S; ++k) rc.row[k] = XT[((size_t)m * N + (g - row0)) * S + k];
    }
    contrib[m] = rc;
  }
}

// Take the offered rows as centroid `step`; flag 2 asks the host for the
// exact chain.
__global__ void pq_dist_take_kernel(const RowContrib* __restrict__ all, int G, int M, int S, int K, int step,
                                    float* __restrict__ cb, uint64_t* __restrict__ chosen,
                                    const uint8_t* __restrict__ state, uint32_t* __restrict__ need_chain) {
  for (int m = threadIdx.x; m < M; m += blockDim.x) {
    need_chain[m] = 0;
    if (state[m] != kRunning) continue;
    for (int r = 0; r < G; ++r) {
      const RowContrib& rc = all[(size_t)r * M + m];
      if (rc.flag == 1) {
        for (int k = 0; k < S; ++k) cb[((size_t)m * K + step) * S + k] = rc.row[k];
        chosen[(size_t)m * K + step] = rc.gidx;
        break;
      }
      if (rc.flag == 2) {
        need_chain[m] = 1;
        break;
      }
    }
  }
}

// Byte layout of one rank's seeding exchange block.
struct SeedBlock {
  size_t o_cnt, o_nonf, bytes;
};
__host__ __device__ inline SeedBlock seed_block(int M, int ncmax) {
  SeedBlock b;
  b.o_cnt = (size_t)M * ncmax * sizeof(double2);
  b.o_nonf = b.o_cnt + (size_t)M * ncmax * sizeof(uint32_t);
  b.bytes = (b.o_nonf + (size_t)M * sizeof(int) + 255) & ~(size_t)255;
  return b;
}

// pq_seed_select_kernel over the gathered chunk bounds of all ranks (global
// chunk j = rank j / ncmax, local chunk j % ncmax; padding chunks are empty).
__global__ void __launch_bounds__(kSelectThreads)
pq_seed_select_dist_kernel(const unsigned char* __restrict__ gath, int G, int ncmax,
                           const uint64_t* __restrict__ rank_row0, int me, uint64_t N_total,
                           const float* __restrict__ XT, uint64_t N, int S, int M, int K, int step,
                           const float* __restrict__ md, const double* __restrict__ draws,
                           int* __restrict__ status, uint8_t* __restrict__ state, double* __restrict__ thr,
                           RowContrib* __restrict__ contrib, int force_chain) {
  const int m = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    RowContrib z;
    z.flag = 0;
    z.pad = 0;
    z.gidx = 0;
    for (int k = 0; k < 4; ++k) z.row[k] = 0.f;
    contrib[m] = z;
  }
  if (state[m] != kRunning) return;
  constexpr int kWarps = kSelectThreads / 32;
  __shared__ double2 wsum[kWarps];
  __shared__ unsigned long long wcnt[kWarps];
  __shared__ double2 incl_all[kSelectThreads];
  __shared__ double2 sh_excl;
  __shared__ int sh_chunk;
  __shared__ uint64_t sh_idx;
  __shared__ int sh_decided;
  const SeedBlock sb = seed_block(M, ncmax);
  const size_t bpr = sb.bytes;

  bool nonf = false;
  for (int r = 0; r < G; ++r) nonf |= reinterpret_cast<const int*>(gath + (size_t)r * bpr + sb.o_nonf)[m] != 0;
  if (nonf) {
    if (tid == 0) { status[m] = MVR_E_NON_FINITE; state[m] = kFailed; }
    return;
  }
  auto CH = [&](int j) -> double2 {
    const int r = j / ncmax, lc = j - r * ncmax;
    return reinterpret_cast<const double2*>(gath + (size_t)r * bpr)[(size_t)m * ncmax + lc];
  };
  auto CC = [&](int j) -> uint32_t {
    const int r = j / ncmax, lc = j - r * ncmax;
    return reinterpret_cast<const uint32_t*>(gath + (size_t)r * bpr + sb.o_cnt)[(size_t)m * ncmax + lc];
  };
  const int nchunk = G * ncmax;
  const float* w = md + (size_t)m * N;
  const double r = draws[(size_t)m * K + step];

  const int cpt = (nchunk + kSelectThreads - 1) / kSelectThreads;
  const int c_lo = min(nchunk, tid * cpt), c_hi = min(nchunk, c_lo + cpt);
  double tlo = 0.0, thi = 0.0;
  unsigned tcnt = 0;
  for (int j = c_lo; j < c_hi; ++j) {
    const double2 v = CH(j);
    tlo = __dadd_rd(tlo, v.x);
    thi = __dadd_ru(thi, v.y);
    tcnt += CC(j);
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
    if (tid == 0) { status[m] = MVR_E_ALL_ZERO; state[m] = kFailed; }
    return;
  }
  const double gN = gamma_bound(N_total);
  const double shi_classic = __dadd_ru(Hi_N, __dmul_ru(gN, Hi_N));
  int e2 = 0;
  (void)frexp(shi_classic, &e2);
  const double Gu = ldexp(1.0, e2 - 53);
  const double thr_now = ldexp(Gu, 23);
  const double B_tight = __dmul_ru(__ull2double_ru(C_N + kCrossingSlack), 0.5 * Gu);
  const double thr_prev = thr[m];
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
    if (thr_now < thr_prev) thr[m] = thr_now;
  }
  __syncthreads();
  if (n_before < kSelectThreads && tid == n_before) {
    double lo = tid > 0 ? incl_all[tid - 1].x : 0.0;
    double hi = tid > 0 ? incl_all[tid - 1].y : 0.0;
    int found = -1;
    for (int j = c_lo; j < c_hi; ++j) {
      const double2 v = CH(j);
      const double nlo = __dadd_rd(lo, v.x), nhi = __dadd_ru(hi, v.y);
      if (u_mid < 0.5 * (nlo + nhi)) { found = j; break; }
      lo = nlo;
      hi = nhi;
    }
    sh_chunk = found;
    sh_excl = make_double2(lo, hi);
  }
  __syncthreads();
  const int fchunk = sh_chunk;
  if (fchunk < 0) {  // no candidate: the exact chain decides
    if (me == 0 && tid == 0) contrib[m].flag = 2;
    return;
  }
  const int owner = fchunk / ncmax, lc = fchunk - owner * ncmax;
  if (owner != me) return;
  const uint64_t li = (uint64_t)lc * kSeedChunk + tid;
  const bool valid = li < N;
  const double v = valid ? (double)w[li] : 0.0;
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
  const bool hit = !valid || u_mid < 0.5 * (elo + ehi);
  const int first = __syncthreads_count(!hit);
  if (first < kSelectThreads && tid == first && valid) {
    const uint64_t gi = rank_row0[me] + li;
    const double2 prv = tid > 0 ? incl_all[tid - 1] : ex;
    const double BN = bound_at(N_total, Hi_N);
    const double ULo = __dmul_rd(r, __dsub_rd(Lo_N, BN));
    const double UHi = __dmul_ru(r, __dadd_ru(Hi_N, BN));
    bool ok = UHi < __dsub_rd(elo, bound_at(gi + 1, ehi));
    if (gi > 0) ok = ok && (ULo >= __dadd_ru(prv.y, bound_at(gi, prv.y)));
    if (ok && !force_chain) {
      sh_idx = gi;
      sh_decided = 1;
    }
  }
  __syncthreads();
  if (tid == 0) {
    RowContrib rc;
    rc.pad = 0;
    for (int k = 0; k < 4; ++k) rc.row[k] = 0.f;
    if (sh_decided) {
      rc.flag = 1;
      rc.gidx = sh_idx;
      const uint64_t l = sh_idx - rank_row0[me];
      for (int k = 0; k < S; ++k) rc.row[k] = XT[((size_t)m * N + l) * S + k];
    } else {
      rc.flag = 2;
      rc.gidx = 0;
    }
    contrib[m] = rc;
  }
}

// Subspace m's rows of this rank, padded to Nmax with `pad`, for a gather:
// out[m][i] (weights / min distances) and, when xt_out is set, the rows.
__global__ void pq_dist_pack_kernel(const float* __restrict__ src, const float* __restrict__ XT, uint64_t N,
                                    uint64_t Nmax, int S, int m, float pad, float* __restrict__ out,
                                    float* __restrict__ xt_out) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < Nmax;
       i += (uint64_t)gridDim.x * blockDim.x) {
    out[i] = i < N ? src[(size_t)m * N + i] : pad;
    if (xt_out)
      for (int k = 0; k < S; ++k) xt_out[i * S + k] = i < N ? XT[((size_t)m * N + i) * S + k] : 0.f;
  }
}

// The reference's sequential weightedSample chain over the gathered weights
// of subspace m (rank-major, zero padding changes neither sum nor search).
__global__ void pq_dist_chain_draw_kernel(const float* __restrict__ gw, int G, uint64_t Nmax,
                                          const uint64_t* __restrict__ rank_row0, const double* __restrict__ draws,
                                          int m, int K, int step, uint64_t* __restrict__ pick,
                                          uint32_t* __restrict__ fallbacks) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const uint64_t total_n = (uint64_t)G * Nmax;
  double total = 0.0;
  uint64_t last_pos = 0;
  for (uint64_t p = 0; p < total_n; ++p) {
    const float v = gw[p];
    total = __dadd_rn(total, (double)v);
    if (v != 0.f) last_pos = p;
  }
  const double u = __dmul_rn(draws[(size_t)m * K + step], total);
  double cum = 0.0;
  uint64_t hitp = last_pos;
  for (uint64_t p = 0; p < total_n; ++p) {
    cum = __dadd_rn(cum, (double)gw[p]);
    if (u < cum) {
      hitp = p;
      break;
    }
  }
  const uint64_t r = hitp / Nmax;
  pick[m] = rank_row0[r] + (hitp - r * Nmax);
  fallbacks[m] += 1;
}

// Centroids from the last rank's running sums and the summed counts.
__global__ void pq_dist_scale_kernel(const float* __restrict__ sums, const uint32_t* __restrict__ gcounts,
                                     float* __restrict__ cb, const uint8_t* __restrict__ state, int M, int K,
                                     int S) {
  const int n = M * K * S;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < n; e += gridDim.x * blockDim.x) {
    const int m = e / (K * S), c = (e / S) % K;
    if (state[m] != kRunning) continue;
    const uint32_t cnt = gcounts[(size_t)m * K + c];
    if (cnt > 0) cb[e] = __fmul_rn(sums[e], __fdiv_rn(1.0f, __uint2float_rn(cnt)));
  }
}

// empty[m] = 1 when running subspace m has an empty cluster (summed counts)
__global__ void pq_dist_empty_kernel(const uint32_t* __restrict__ gcounts, const uint8_t* __restrict__ state,
                                     int M, int K, uint32_t* __restrict__ empty) {
  const int m = blockIdx.x;
  __shared__ int any;
  if (threadIdx.x == 0) any = 0;
  __syncthreads();
  if (state[m] == kRunning)
    for (int c = threadIdx.x; c < K; c += blockDim.x)
      if (gcounts[(size_t)m * K + c] == 0) atomicOr(&any, 1);
  __syncthreads();
  if (threadIdx.x == 0) empty[m] = (uint32_t)any;
}

// Empty-cluster reseed of subspace m over the gathered min distances and
// rows (-inf padding never wins), identically on every rank; this rank also
// marks its own copy of each chosen row.
__global__ void __launch_bounds__(1024)
pq_dist_reseed_kernel(float* __restrict__ gmind, const float* __restrict__ gxt, int G, uint64_t Nmax, int S, int K,
                      int m, const uint32_t* __restrict__ gcounts, float* __restrict__ cb, float* __restrict__ mind,
                      uint64_t N, int me, uint32_t* __restrict__ reseeds) {
  const uint64_t total_n = (uint64_t)G * Nmax;
  for (int c = 0; c < K; ++c) {
    if (gcounts[(size_t)m * K + c] != 0) continue;
    const uint64_t far = block_argmax_first(gmind, total_n);
    if (threadIdx.x < (unsigned)S) cb[((size_t)m * K + c) * S + threadIdx.x] = gxt[far * S + threadIdx.x];
    __syncthreads();
    if (threadIdx.x == 0) {
      gmind[far] = -__int_as_float(0x7f800000);
      const uint64_t r = far / Nmax, l = far - r * Nmax;
      if ((int)r == me && l < N) mind[(size_t)m * N + l] = -__int_as_float(0x7f800000);
      reseeds[m] += 1;
    }
    __syncthreads();
  }
}

}  // namespace

int sm_count_current_device() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
    (void)cudaGetLastError();
    return 148;
  }
  return n;
}

int pq_encode_device(Ctx* ctx, const float* d_cb, int D, int M, const float* d_R, uint64_t N,
                     uint8_t* d_codes) {
  if (N == 0) return MVR_OK;
  const int S = D / M;
  MVR_TRY(check_shape(ctx, D, M, S, 256));
  int nblk = 0;
  uint64_t rpc = 0;
  grid_for(N, ctx->sm_count, &nblk, &rpc);
  cudaStream_t st = ctx->stream;
  if (ctx->tc_filter && ctx->pq_tc_filter && !ctx->exhaustive_assign) {
    if (!ctx->tc_diag) {
      MVR_CUDA(ctx, cudaMalloc(&ctx->tc_diag, 4 * sizeof(uint32_t)));
      MVR_CUDA(ctx, cudaMemsetAsync(ctx->tc_diag, 0, 4 * sizeof(uint32_t), st));
    }
    switch (S) {
      case 1: return launch_tc_assign<1>(ctx, st, kModeEncode, false, d_R, nullptr, N, D, M, 256, d_cb, nullptr, nullptr, d_codes, nullptr, nullptr, nullptr, nullptr, nullptr, ctx->tc_diag, ctx->sm_count);
      case 2: return launch_tc_assign<2>(ctx, st, kModeEncode, false, d_R, nullptr, N, D, M, 256, d_cb, nullptr, nullptr, d_codes, nullptr, nullptr, nullptr, nullptr, nullptr, ctx->tc_diag, ctx->sm_count);
      default: return launch_tc_assign<4>(ctx, st, kModeEncode, false, d_R, nullptr, N, D, M, 256, d_cb, nullptr, nullptr, d_codes, nullptr, nullptr, nullptr, nullptr, nullptr, ctx->tc_diag, ctx->sm_count);
    }
  }
  switch (S) {
    case 1: return launch_assign<1>(ctx, st, kModeEncode, d_R, nullptr, N, D, M, 256, d_cb, d_codes, nullptr, nullptr, nullptr, nullptr, nblk, rpc);
    case 2: return launch_assign<2>(ctx, st, kModeEncode, d_R, nullptr, N, D, M, 256, d_cb, d_codes, nullptr, nullptr, nullptr, nullptr, nblk, rpc);
    default: return launch_assign<4>(ctx, st, kModeEncode, d_R, nullptr, N, D, M, 256, d_cb, d_codes, nullptr, nullptr, nullptr, nullptr, nblk, rpc);
  }
}

PqLayout pq_layout(uint64_t N, int M, int S, int K, int sms, bool with_xt) {
  PqLayout L;
  uint64_t rpc = 0;
  grid_for(N, sms, &L.nblk, &rpc);
  L.rows_per_cta = rpc;
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
  L.o_thr = carve((size_t)M * 8);
  L.o_counts = carve((size_t)M * K * 4);
  L.o_starts = carve((size_t)M * K * 4);
  L.o_wcss = carve((size_t)M * 4);
  L.o_prev = carve((size_t)M * 4);
  L.o_status = carve((size_t)M * 4);
  L.o_nonf = carve((size_t)M * 4);
  L.o_iters = carve((size_t)M * 4);
  L.o_fb = carve((size_t)M * 4);
  L.o_rs = carve((size_t)M * 4);
  L.o_exact = carve((size_t)M * 8);
  L.o_state = carve((size_t)M);
  L.o_diag = carve(4 * sizeof(uint32_t));
  L.o_ldist = carve((size_t)M * 8);
  L.small_bytes = off;
  L.o_xt = carve(with_xt ? (size_t)M * N * S * sizeof(float) : 0);
  L.o_mind = carve((size_t)M * N * sizeof(float));
  L.o_asg = carve((size_t)M * N);
  L.o_sorted = carve((size_t)M * N * S * sizeof(float));
  // the histograms, scan and scatter of the Lloyd passes work on CTAs of one
  // full scatter tile each (the row-sharded path keeps the persistent grid)
  L.nblk_s = (int)std::max<uint64_t>(1, (N + kScatTile - 1) / kScatTile);
  L.o_hist = carve((size_t)M * std::max(L.nblk, L.nblk_s) * K * sizeof(uint32_t));
  L.o_chunk = carve((size_t)M * L.nchunk * sizeof(double2));
  L.o_chunk_cnt = carve((size_t)M * L.nchunk * sizeof(uint32_t));
  // exact chained draws (large N): chunk prefix bounds / end sums, G, binade
  L.o_xpre = carve((size_t)M * L.nchunk * sizeof(double2));
  L.o_xg = carve((size_t)M * L.nchunk * sizeof(ulonglong2));
  L.o_xe = carve((size_t)M * L.nchunk * sizeof(int));
  L.o_ub = carve((size_t)M * N * sizeof(float));
  L.o_lb = carve((size_t)M * N * sizeof(float));
  L.o_list = carve((size_t)M * N * sizeof(uint32_t));
  L.o_lcnt = carve((size_t)M * sizeof(uint32_t));
  L.o_cbold = carve((size_t)M * K * S * sizeof(float));
  L.o_drift = carve((size_t)M * K * sizeof(float));
  L.o_maxd = carve((size_t)M * 3 * sizeof(float));
  L.o_nbr = carve((size_t)M * K * kCandL);
  L.o_nbr_last = carve((size_t)M * K * 2 * sizeof(float));
  L.total_bytes = off;
  return L;
}

// Timing events of one engine run, from the context's pool (created on
// first use, kept for the context's lifetime): v[i] = pool[offset + i].
static int pool_events(Ctx* ctx, PqTiming* tm, size_t offset, std::vector<cudaEvent_t>& v) {
  while (tm->pool.size() < offset + v.size()) {
    cudaEvent_t e = nullptr;
    MVR_CUDA(ctx, cudaEventCreate(&e));
    tm->pool.push_back(e);
  }
  for (size_t i = 0; i < v.size(); ++i) v[i] = tm->pool[offset + i];
  return MVR_OK;
}

// One group of subspaces (all of them when the engine runs one group):
// seeding + Lloyd on `st`, then the bookkeeping read back and checked.
// `ev` holds three timing events (created here when null) when the call
// reports statistics.
static int pq_kmeans_run_one(Ctx* ctx, cudaStream_t st, const PqJob& job, const PqOut& out, unsigned char* ws,
                             unsigned char* hsmall, int sms, PqTiming* tm) {
  cudaEvent_t* ev = tm ? tm->phase : nullptr;
  const uint64_t N = job.N;
  const int D = job.D, M = job.M, S = job.S, K = job.K;
  MVR_TRY(check_shape(ctx, D, M, S, K));
  if (N == 0) return fail(ctx, MVR_E_EMPTY_VECTOR_SET, "no rows");
  if (N >= (1ull << 32)) return fail(ctx, MVR_E_INVALID_ARGUMENT, "more than 2^32-1 rows per subspace");
  if (job.xt && !job.xt_ready) return fail(ctx, MVR_E_INVALID_ARGUMENT, "external subspace-major rows not filled");
  const bool timing = out.stats != nullptr && ctx != nullptr && ev != nullptr;
  const auto host_t0 = std::chrono::steady_clock::now();
  if (timing) {
    for (int e = 0; e < 3; ++e)
      if (!ev[e]) MVR_CUDA(ctx, cudaEventCreate(&ev[e]));
    MVR_CUDA(ctx, cudaEventRecord(ev[0], st));
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
    if (out.stats) {
      std::memset(out.stats, 0, sizeof(*out.stats));
      out.stats->groups = 1;
    }
    return MVR_OK;
  }

  const PqLayout L = pq_layout(N, M, S, K, sms, job.xt == nullptr);
  const int nblk = L.nblk, nchunk = L.nchunk;
  const uint64_t rpc = L.rows_per_cta;
  const int sblk = L.nblk_s;  // histogram / scatter CTAs: one kScatTile-row tile each
  const uint64_t srpc = kScatTile;
  float* XT = job.xt ? const_cast<float*>(job.xt) : (float*)(ws + L.o_xt);
  float* mind = (float*)(ws + L.o_mind);
  uint8_t* asg = (uint8_t*)(ws + L.o_asg);
  float* sorted = (float*)(ws + L.o_sorted);
  uint32_t* hist = (uint32_t*)(ws + L.o_hist);
  double2* chunk = (double2*)(ws + L.o_chunk);
  uint32_t* chunk_cnt = (uint32_t*)(ws + L.o_chunk_cnt);
  unsigned char* small = ws;  // bookkeeping lives at the start of the workspace
  const size_t small_bytes = L.small_bytes;
  double* d_draws = (double*)(small + L.o_draws);
  uint64_t* d_chosen = (uint64_t*)(small + L.o_chosen);
  uint64_t* d_idx0 = (uint64_t*)(small + L.o_idx0);
  double* d_thr = (double*)(small + L.o_thr);
  uint32_t* d_counts = (uint32_t*)(small + L.o_counts);
  uint32_t* d_starts = (uint32_t*)(small + L.o_starts);
  float* d_wcss = (float*)(small + L.o_wcss);
  float* d_prev = (float*)(small + L.o_prev);
  int* d_status = (int*)(small + L.o_status);
  int* d_nonf = (int*)(small + L.o_nonf);
  uint32_t* d_iters = (uint32_t*)(small + L.o_iters);
  uint32_t* d_fb = (uint32_t*)(small + L.o_fb);
  uint32_t* d_rs = (uint32_t*)(small + L.o_rs);
  unsigned long long* d_exact = (unsigned long long*)(small + L.o_exact);
  uint8_t* d_state = (uint8_t*)(small + L.o_state);
  uint32_t* d_diag = (uint32_t*)(small + L.o_diag);

  // ---- host RNG draws (data independent); thresholds start at +inf; the
  // rest of the bookkeeping starts at zero (state = running) ---------------
  std::memset(hsmall, 0, small_bytes);
  {
    double* hd = (double*)(hsmall + L.o_draws);
    uint64_t* hi0 = (uint64_t*)(hsmall + L.o_idx0);
    double* ht = (double*)(hsmall + L.o_thr);
    for (int m = 0; m < M; ++m) {
      Xoshiro256pp rng(job.seed + (uint64_t)m);
      hi0[m] = rng.below(N);
      hd[(size_t)m * K] = 0.0;
      for (int c = 1; c < K; ++c) hd[(size_t)m * K + c] = rng.unit_f64();
      ht[m] = HUGE_VAL;
    }
  }
  MVR_CUDA(ctx, cudaMemcpyAsync(small, hsmall, small_bytes, cudaMemcpyHostToDevice, st));

  uint32_t launches = 0;
  if (!job.xt_ready) {
    const int grid = (int)std::min<uint64_t>((N + 255) / 256, (uint64_t)std::max(1, sms) * 8);
    switch (S) {
      case 1: pq_transpose_kernel<1><<<grid, 256, 0, st>>>(job.R, N, D, M, XT); break;
      case 2: pq_transpose_kernel<2><<<grid, 256, 0, st>>>(job.R, N, D, M, XT); break;
      default: pq_transpose_kernel<4><<<grid, 256, 0, st>>>(job.R, N, D, M, XT); break;
    }
    MVR_CUDA(ctx, cudaGetLastError());
    ++launches;
  }

  float* cb = out.d_codebooks;
  pq_seed_init_kernel<<<M, 32, 0, st>>>(XT, N, S, K, d_idx0, cb, d_chosen);
  MVR_CUDA(ctx, cudaGetLastError());
  ++launches;
  // every 8th update launch (step >= 1) bracketed by events: the sampled
  // duration of the HBM-bound update kernel (stats only)
  std::vector<cudaEvent_t> sev;
  if (timing) {
    sev.resize(2 * (size_t)((K - 2 + 7) / 8), nullptr);
    MVR_TRY(pool_events(ctx, tm, 0, sev));
  }
  for (int step = 0; step + 1 < K; ++step) {
    const bool sample = timing && step >= 1 && (step - 1) % 8 == 0 && (size_t)(2 * ((step - 1) / 8) + 1) < sev.size();
    if (sample) MVR_CUDA(ctx, cudaEventRecord(sev[2 * ((step - 1) / 8)], st));
    {
      auto upd = S == 1 ? pq_seed_update_w_kernel<1> : S == 2 ? pq_seed_update_w_kernel<2> : pq_seed_update_w_kernel<4>;
      MVR_CUDA(ctx, launch_pdl(upd, dim3(nchunk), dim3(32 * M), 0, st, (const float*)XT, N, M, K, step,
                               (const float*)cb, mind, chunk, chunk_cnt, d_nonf, (const uint8_t*)d_state,
                               (const double*)d_thr, nchunk));
    }
    if (sample) MVR_CUDA(ctx, cudaEventRecord(sev[2 * ((step - 1) / 8) + 1], st));
    MVR_CUDA(ctx, launch_pdl(pq_seed_select_kernel, dim3(M), dim3(kSelectThreads), 0, st, (const float*)XT, N, S, K,
                             step + 1, cb, (const float*)mind, (const double2*)chunk, (const uint32_t*)chunk_cnt,
                             nchunk, (const double*)d_draws, d_nonf, d_status, d_state, d_fb, d_chosen, d_thr,
                             ctx && ctx->serial_draws ? 1 : 0, (double2*)(ws + L.o_xpre),
                             (ulonglong2*)(ws + L.o_xg), (int*)(ws + L.o_xe)));
    launches += 2;
  }
  if (timing) MVR_CUDA(ctx, cudaEventRecord(ev[1], st));

  // ---- Lloyd iterations ---------------------------------------------------
  const bool check = !(job.tol == -INFINITY) && !std::isnan(job.tol);
  std::vector<cudaEvent_t> aev;  // assignment-kernel brackets (stats only)
  if (timing) {
    aev.resize(2 * (size_t)job.max_iters, nullptr);
    MVR_TRY(pool_events(ctx, tm, sev.size(), aev));
  }
  std::vector<cudaEvent_t> lev;  // pruned-pass brackets (stats only)
  if (timing) {
    lev.resize(2 * (size_t)job.max_iters, nullptr);
    MVR_TRY(pool_events(ctx, tm, sev.size() + aev.size(), lev));
  }
  uint32_t list_passes = 0;
  // Bound pruning (Hamerly) from the second iteration on; exact, see
  // bound_upper / bound_lower.
  const bool prune = !(ctx && ctx->exhaustive_assign);
  // The tensor-core filter for the first pass only when the context asks for
  // it on PQ (the exact scan measured as fast for 4-float sub-vectors).
  const bool use_tc = prune && job.tc_filter && ctx && ctx->tc_filter && ctx->pq_tc_filter;
  // The pruned passes (row lists) stay on the exact kernel: for 4-float
  // sub-vectors the filter's accumulator read-out per (row, centroid) costs
  // about as much as the exact distance, and the exact list pass measured
  // faster (1.87 vs 2.07 ms per iteration at 1.52M x 16 subspaces).
  const bool tc_lists = false;
  // Candidate scans (pq_cand_kernel) replace the check + full-scan list
  // passes unless the context asks for the latter (verification).
  const bool cand = prune && !(ctx && !ctx->cand_scan);
  uint8_t* nbr_idx = (uint8_t*)(ws + L.o_nbr);
  float* nbr_last = (float*)(ws + L.o_nbr_last);
  unsigned long long* d_ldist = (unsigned long long*)(small + L.o_ldist);
  const size_t csmem = cand_smem(K, S);
  const unsigned cgx = (unsigned)std::max<uint64_t>(
      1, std::min<uint64_t>((N + kCandThreads - 1) / kCandThreads, (uint64_t)(std::max(1, sms) * 4 + M - 1) / M));
  float* ubnd = (float*)(ws + L.o_ub);
  float* lbnd = (float*)(ws + L.o_lb);
  uint32_t* plist = (uint32_t*)(ws + L.o_list);
  uint32_t* lcnt = (uint32_t*)(ws + L.o_lcnt);
  float* cb_old = (float*)(ws + L.o_cbold);
  float* drift = (float*)(ws + L.o_drift);
  float* maxd = (float*)(ws + L.o_maxd);
  const unsigned pgx = (unsigned)std::min<uint64_t>((N + 255) / 256, (uint64_t)std::max(1, sms) * 4);
  const size_t list_smem = assign_smem(M, K, S, kModeEncode);  // the codebooks only
  for (uint32_t it = 0; it < job.max_iters; ++it) {
    const bool last = it + 1 == job.max_iters;
    const bool need_mind = check || (last && out.h_wcss);
    if (timing) MVR_CUDA(ctx, cudaEventRecord(aev[2 * it], st));
    if (use_tc && it == 0) {  // every row through the tensor-core filter, then the histograms
      switch (S) {
        case 1: MVR_TRY(launch_tc_assign<1>(ctx, st, kModeLloyd, false, job.R, XT, N, D, M, K, cb, nullptr, nullptr, nullptr, asg, mind, ubnd, lbnd, d_state, d_diag, sms)); break;
        case 2: MVR_TRY(launch_tc_assign<2>(ctx, st, kModeLloyd, false, job.R, XT, N, D, M, K, cb, nullptr, nullptr, nullptr, asg, mind, ubnd, lbnd, d_state, d_diag, sms)); break;
        default: MVR_TRY(launch_tc_assign<4>(ctx, st, kModeLloyd, false, job.R, XT, N, D, M, K, cb, nullptr, nullptr, nullptr, asg, mind, ubnd, lbnd, d_state, d_diag, sms)); break;
      }
      pq_hist_kernel<<<sblk, 512, (size_t)M * K * sizeof(uint32_t), st>>>(asg, N, M, K, d_state, srpc, hist);
      MVR_CUDA(ctx, cudaGetLastError());
      ++launches;
    } else if (!prune || it == 0) {
      float* ub_o = prune ? ubnd : nullptr;
      float* lb_o = prune ? lbnd : nullptr;
      switch (S) {
        case 1: MVR_TRY(launch_assign<1>(ctx, st, kModeLloyd, job.R, XT, N, D, M, K, cb, nullptr, asg, mind, nullptr, d_state, nblk, rpc, ub_o, lb_o)); break;
        case 2: MVR_TRY(launch_assign<2>(ctx, st, kModeLloyd, job.R, XT, N, D, M, K, cb, nullptr, asg, mind, nullptr, d_state, nblk, rpc, ub_o, lb_o)); break;
        default: MVR_TRY(launch_assign<4>(ctx, st, kModeLloyd, job.R, XT, N, D, M, K, cb, nullptr, asg, mind, nullptr, d_state, nblk, rpc, ub_o, lb_o)); break;
      }
      pq_hist_kernel<<<sblk, 512, (size_t)M * K * sizeof(uint32_t), st>>>(asg, N, M, K, d_state, srpc, hist);
      MVR_CUDA(ctx, cudaGetLastError());
      ++launches;
    } else {
      pq_drift_kernel<<<M, 256, 0, st>>>(cb_old, cb, M, K, S, d_state, drift, maxd);
      MVR_CUDA(ctx, cudaMemsetAsync(lcnt, 0, (size_t)M * sizeof(uint32_t), st));
      if (timing) MVR_CUDA(ctx, cudaEventRecord(lev[2 * list_passes], st));
      const dim3 cg(pgx, (unsigned)M);
      if (cand) {
        const dim3 ng((unsigned)((K + 7) / 8), (unsigned)M), cgrid(cgx, (unsigned)M);
        const int nm = need_mind ? 1 : 0;
        switch (S) {
          case 1: pq_nbr_kernel<1><<<ng, 256, 0, st>>>(cb, K, d_state, nbr_idx, nbr_last); break;
          case 2: pq_nbr_kernel<2><<<ng, 256, 0, st>>>(cb, K, d_state, nbr_idx, nbr_last); break;
          default: pq_nbr_kernel<4><<<ng, 256, 0, st>>>(cb, K, d_state, nbr_idx, nbr_last); break;
        }
        MVR_CUDA(ctx, cudaGetLastError());
        switch (S) {
          case 1: { auto k = pq_cand_kernel<1>; MVR_CUDA(ctx, raise_smem_limit((const void*)k, (size_t)(csmem))); k<<<cgrid, kCandThreads, csmem, st>>>(XT, N, K, cb, nbr_idx, nbr_last, asg, ubnd, lbnd, drift, maxd, d_state, mind, nm, lcnt, d_ldist); } break;
          case 2: { auto k = pq_cand_kernel<2>; MVR_CUDA(ctx, raise_smem_limit((const void*)k, (size_t)(csmem))); k<<<cgrid, kCandThreads, csmem, st>>>(XT, N, K, cb, nbr_idx, nbr_last, asg, ubnd, lbnd, drift, maxd, d_state, mind, nm, lcnt, d_ldist); } break;
          default: { auto k = pq_cand_kernel<4>; MVR_CUDA(ctx, raise_smem_limit((const void*)k, (size_t)(csmem))); k<<<cgrid, kCandThreads, csmem, st>>>(XT, N, K, cb, nbr_idx, nbr_last, asg, ubnd, lbnd, drift, maxd, d_state, mind, nm, lcnt, d_ldist); } break;
        }
        MVR_CUDA(ctx, cudaGetLastError());
      } else {
      switch (S) {
        case 1: pq_prune_check_kernel<1><<<cg, 256, 0, st>>>(XT, N, K, cb, asg, ubnd, lbnd, drift, maxd, d_state, plist, lcnt, mind, need_mind ? 1 : 0); break;
        case 2: pq_prune_check_kernel<2><<<cg, 256, 0, st>>>(XT, N, K, cb, asg, ubnd, lbnd, drift, maxd, d_state, plist, lcnt, mind, need_mind ? 1 : 0); break;
        default: pq_prune_check_kernel<4><<<cg, 256, 0, st>>>(XT, N, K, cb, asg, ubnd, lbnd, drift, maxd, d_state, plist, lcnt, mind, need_mind ? 1 : 0); break;
      }
      MVR_CUDA(ctx, cudaGetLastError());
      if (use_tc && tc_lists) {
        switch (S) {
          case 1: MVR_TRY(launch_tc_assign<1>(ctx, st, kModeLloyd, true, job.R, XT, N, D, M, K, cb, plist, lcnt, nullptr, asg, mind, ubnd, lbnd, d_state, d_diag, sms)); break;
          case 2: MVR_TRY(launch_tc_assign<2>(ctx, st, kModeLloyd, true, job.R, XT, N, D, M, K, cb, plist, lcnt, nullptr, asg, mind, ubnd, lbnd, d_state, d_diag, sms)); break;
          default: MVR_TRY(launch_tc_assign<4>(ctx, st, kModeLloyd, true, job.R, XT, N, D, M, K, cb, plist, lcnt, nullptr, asg, mind, ubnd, lbnd, d_state, d_diag, sms)); break;
        }
      } else {
        switch (S) {
          case 1: { auto k = pq_assign_list_kernel<1>; MVR_CUDA(ctx, raise_smem_limit((const void*)k, (size_t)(list_smem))); k<<<nblk, kAsgThreads, list_smem, st>>>(XT, N, M, K, cb, plist, lcnt, asg, mind, ubnd, lbnd, d_state, 1.0f); } break;
          case 2: { auto k = pq_assign_list_kernel<2>; MVR_CUDA(ctx, raise_smem_limit((const void*)k, (size_t)(list_smem))); k<<<nblk, kAsgThreads, list_smem, st>>>(XT, N, M, K, cb, plist, lcnt, asg, mind, ubnd, lbnd, d_state, 1.0f); } break;
          default: { auto k = pq_assign_list_kernel<4>; MVR_CUDA(ctx, raise_smem_limit((const void*)k, (size_t)(list_smem))); k<<<nblk, kAsgThreads, list_smem, st>>>(XT, N, M, K, cb, plist, lcnt, asg, mind, ubnd, lbnd, d_state, 1.0f); } break;
        }
      }
      }
      MVR_CUDA(ctx, cudaGetLastError());
      if (timing) MVR_CUDA(ctx, cudaEventRecord(lev[2 * list_passes + 1], st));
      ++list_passes;
      pq_hist_kernel<<<sblk, 512, (size_t)M * K * sizeof(uint32_t), st>>>(asg, N, M, K, d_state, srpc, hist);
      MVR_CUDA(ctx, cudaGetLastError());
      launches += 5;
    }
    if (timing) MVR_CUDA(ctx, cudaEventRecord(aev[2 * it + 1], st));
    launches += 5;
    if (check || (last && out.h_wcss)) {
      pq_wcss_kernel<<<M, 256, 0, st>>>(mind, N, d_wcss, d_state, nullptr);
      MVR_CUDA(ctx, cudaGetLastError());
      ++launches;
    }
    pq_scan_kernel<<<M, kScanThreads, 0, st>>>(hist, sblk, K, d_counts, d_starts, d_state);
    MVR_CUDA(ctx, cudaGetLastError());
    if (prune && it > 0 && !need_mind) {  // kept rows have no fresh distance: refresh where a reseed follows
      const dim3 cg(pgx, (unsigned)M);
      switch (S) {
        case 1: pq_mind_refresh_kernel<1><<<cg, 256, 0, st>>>(XT, N, K, cb, asg, d_counts, d_state, mind); break;
        case 2: pq_mind_refresh_kernel<2><<<cg, 256, 0, st>>>(XT, N, K, cb, asg, d_counts, d_state, mind); break;
        default: pq_mind_refresh_kernel<4><<<cg, 256, 0, st>>>(XT, N, K, cb, asg, d_counts, d_state, mind); break;
      }
      MVR_CUDA(ctx, cudaGetLastError());
      ++launches;
    }
    if (prune) MVR_CUDA(ctx, cudaMemcpyAsync(cb_old, cb, (size_t)M * K * S * sizeof(float), cudaMemcpyDeviceToDevice, st));
    {
      const size_t sm = scatter_tile_smem(S);
      const dim3 sg((unsigned)sblk, (unsigned)M);
      switch (S) {
        case 1: { auto k = pq_scatter_tile_kernel<1>; MVR_CUDA(ctx, raise_smem_limit((const void*)k, (size_t)(sm))); k<<<sg, kScatT, sm, st>>>(XT, N, K, asg, hist, sorted, d_state, srpc); } break;
        case 2: { auto k = pq_scatter_tile_kernel<2>; MVR_CUDA(ctx, raise_smem_limit((const void*)k, (size_t)(sm))); k<<<sg, kScatT, sm, st>>>(XT, N, K, asg, hist, sorted, d_state, srpc); } break;
        default: { auto k = pq_scatter_tile_kernel<4>; MVR_CUDA(ctx, raise_smem_limit((const void*)k, (size_t)(sm))); k<<<sg, kScatT, sm, st>>>(XT, N, K, asg, hist, sorted, d_state, srpc); } break;
      }
    }
    MVR_CUDA(ctx, cudaGetLastError());
    switch (S) {
      case 1: MVR_TRY(launch_chain<1>(ctx, st, sorted, N, M, K, d_counts, d_starts, cb, d_state, d_diag, sms)); break;
      case 2: MVR_TRY(launch_chain<2>(ctx, st, sorted, N, M, K, d_counts, d_starts, cb, d_state, d_diag, sms)); break;
      default: MVR_TRY(launch_chain<4>(ctx, st, sorted, N, M, K, d_counts, d_starts, cb, d_state, d_diag, sms)); break;
    }
    pq_reseed_converge_kernel<<<M, 1024, 0, st>>>(XT, N, S, K, d_counts, mind, cb, d_state, d_wcss, d_prev,
                                                  d_iters, d_rs, (int)it, check ? 1 : 0, job.tol, 1,
                                                  (prune && it > 0) ? lcnt : nullptr, d_exact);
    MVR_CUDA(ctx, cudaGetLastError());
  }
  if (timing) MVR_CUDA(ctx, cudaEventRecord(ev[2], st));
  if (out.d_assign && job.max_iters > 0) {
    // Converged subspaces keep the assignments of their last iteration,
    // which later iterations did not touch.
    u8_to_u32_kernel<<<1024, 256, 0, st>>>(asg, out.d_assign, (uint64_t)M * N);
    MVR_CUDA(ctx, cudaGetLastError());
    ++launches;
  }
  // (measured before the read-back: a copy into pageable memory waits for the stream)
  const double host_enqueue_ms =
      std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - host_t0).count();
  MVR_CUDA(ctx, cudaMemcpyAsync(hsmall, small, small_bytes, cudaMemcpyDeviceToHost, st));
  MVR_CUDA(ctx, cudaStreamSynchronize(st));

  const int* hstatus = (const int*)(hsmall + L.o_status);
  for (int m = 0; m < M; ++m)
    if (hstatus[m] != MVR_OK)
      return fail(ctx, hstatus[m], std::string("subspace ") + std::to_string(job.sub0 + m) + ": " +
                                        mvr_status_name(hstatus[m]));
  if (((const uint32_t*)(hsmall + L.o_diag))[3])
    return fail(ctx, MVR_E_TIMEOUT, "centroid sums: a bulk copy of cluster members did not complete in time");
  const uint32_t* hdiag = (const uint32_t*)(hsmall + L.o_diag);
  if (hdiag[2]) return fail(ctx, MVR_E_TIMEOUT, "tensor-core filter: an MMA did not complete in time");
  if (use_tc && hdiag[0] > 0) {
    // a winner's approximation broke its error bound: the whole training
    // again with the exact scans (the transposed rows are still in place)
    const uint32_t viol = hdiag[0];
    PqJob exact = job;
    exact.tc_filter = false;
    exact.xt_ready = true;
    MVR_TRY(pq_kmeans_run_one(ctx, st, exact, out, ws, hsmall, sms, tm));
    if (out.stats) out.stats->filter_violations = viol;
    return MVR_OK;
  }
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
      cudaEventElapsedTime(&t01, ev[0], ev[1]);
      cudaEventElapsedTime(&t12, ev[1], ev[2]);
      cudaEventElapsedTime(&t02, ev[0], ev[2]);
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
      double su = 0.0;
      uint32_t ns = 0;
      for (size_t q = 0; q + 1 < sev.size(); q += 2) {
        float t = 0.f;
        if (cudaEventElapsedTime(&t, sev[q], sev[q + 1]) == cudaSuccess) {
          su += t;
          ++ns;
        }
      }
      (void)cudaGetLastError();
      out.stats->seed_update_ms_sampled = su;
      out.stats->seed_update_samples = ns;
      out.stats->assign_launches = job.max_iters;
      double lm = 0.0;
      for (uint32_t q = 0; q < list_passes; ++q) {
        float t = 0.f;
        cudaEventElapsedTime(&t, lev[2 * q], lev[2 * q + 1]);
        lm += t;
      }
      out.stats->list_ms = lm;
      out.stats->list_launches = list_passes;
      if (job.max_iters > 0) {
        float t0 = 0.f;
        cudaEventElapsedTime(&t0, aev[0], aev[1]);
        out.stats->assign_first_ms = t0;
      }
    }
    uint32_t mx = 0, mn = UINT32_MAX, fb = 0, rs = 0;
    const uint32_t* hfb = (const uint32_t*)(hsmall + L.o_fb);
    const uint32_t* hrs = (const uint32_t*)(hsmall + L.o_rs);
    const unsigned long long* hex = (const unsigned long long*)(hsmall + L.o_exact);
    for (int m = 0; m < M; ++m) {
      out.stats->lloyd_rows_exact += hex[m];
      out.stats->lloyd_rows_total += (uint64_t)(job.max_iters ? hiters[m] : 0) * N;
    }
    // distances computed by the pruned passes: counted on the device by the
    // candidate scans; the full-scan lists compute K per listed row (the
    // first pass scans every row of every subspace, the rest were listed)
    if (cand) {
      const unsigned long long* hld = (const unsigned long long*)(hsmall + L.o_ldist);
      for (int m = 0; m < M; ++m) out.stats->list_distances += hld[m];
    } else if (prune && job.max_iters > 1 && out.stats->lloyd_rows_exact >= (uint64_t)M * N) {
      out.stats->list_distances = (out.stats->lloyd_rows_exact - (uint64_t)M * N) * (uint64_t)K;
    }
    for (int m = 0; m < M; ++m) {
      const uint32_t v = job.max_iters ? hiters[m] : 0;
      mx = std::max(mx, v);
      mn = std::min(mn, v);
      fb += hfb[m];
      rs += hrs[m];
    }
    out.stats->iters_max = mx;
    out.stats->iters_min = mn;
    out.stats->filter_rows_rechecked = hdiag[1];
    out.stats->seed_fallbacks = fb;
    out.stats->reseeds = rs;
    out.stats->launches = launches;
    out.stats->groups = 1;
    out.stats->host_enqueue_ms = host_enqueue_ms;
  }
  return MVR_OK;
}

// ---------------------------------------------------------------------------
// Subspace groups side by side: the subspaces split in two contiguous
// groups, each an independent training (its own bookkeeping, seeds seed + m,
// draws, bounds) on its own stream and host thread, over one subspace-major
// copy of the rows. The k-means++ chain of a group is a sequence of short
// dependent launches (update, draw) and a Lloyd iteration has latency-bound
// steps (the sequential centroid sums, the scans, the bound bookkeeping):
// with two groups in flight the GPU fills one group's gaps with the other's
// work. Results are those of one group over all subspaces (subspaces do not
// interact).
// ---------------------------------------------------------------------------
constexpr int kPqGroups = 2;

int pq_groups(const Ctx* ctx, uint64_t N, int M, int K) {
  return (ctx != nullptr && ctx->pq_groups >= 2 && M >= 2 && (uint64_t)K < N) ? kPqGroups : 1;
}

static size_t align256(size_t b) { return (b + 255) & ~(size_t)255; }
static int group_lo(int M, int G, int g) { return (int)((int64_t)M * g / G); }

size_t pq_ws_bytes(uint64_t N, int M, int S, int K, int sms, int groups) {
  if (groups <= 1) return pq_layout(N, M, S, K, sms).total_bytes;
  size_t b = align256((size_t)M * N * S * sizeof(float));
  for (int g = 0; g < groups; ++g) {
    const int mg = group_lo(M, groups, g + 1) - group_lo(M, groups, g);
    b += align256(pq_layout(N, mg, S, K, sms, false).total_bytes);
  }
  return b;
}

float* pq_ws_xt(unsigned char* ws, uint64_t N, int M, int S, int K, int sms, int groups) {
  if (groups <= 1) return (float*)(ws + pq_layout(N, M, S, K, sms).o_xt);
  return (float*)ws;
}

int pq_kmeans_run(Ctx* ctx, cudaStream_t st, const PqJob& job, const PqOut& out, unsigned char* ws,
                  unsigned char* hsmall, int sms) {
  const uint64_t N = job.N;
  const int D = job.D, M = job.M, S = job.S, K = job.K;
  const int G = pq_groups(ctx, N, M, K);
  if (G <= 1) return pq_kmeans_run_one(ctx, st, job, out, ws, hsmall, sms, ctx ? &ctx->pq_timing[0] : nullptr);
  MVR_TRY(check_shape(ctx, D, M, S, K));
  if (N >= (1ull << 32)) return fail(ctx, MVR_E_INVALID_ARGUMENT, "more than 2^32-1 rows per subspace");
  if (!job.xt_ready && !job.R) return fail(ctx, MVR_E_INVALID_ARGUMENT, "no rows given");
  cudaStream_t side = nullptr;
  MVR_TRY(side_stream(ctx, &side));
  if (!ctx->fork_ev) MVR_CUDA(ctx, cudaEventCreateWithFlags(&ctx->fork_ev, cudaEventDisableTiming));
  if (!ctx->join_ev) MVR_CUDA(ctx, cudaEventCreateWithFlags(&ctx->join_ev, cudaEventDisableTiming));
  const bool timing = out.stats != nullptr;
  if (timing) {
    for (auto& e : ctx->pev)
      if (!e) MVR_CUDA(ctx, cudaEventCreate(&e));
    MVR_CUDA(ctx, cudaEventRecord(ctx->pev[0], st));
  }
  // one subspace-major copy of the rows for both groups
  float* XT = job.xt ? const_cast<float*>(job.xt) : (float*)ws;
  uint32_t launches = 0;
  if (!job.xt_ready) {
    const int grid = (int)std::min<uint64_t>((N + 255) / 256, (uint64_t)std::max(1, sms) * 8);
    switch (S) {
      case 1: pq_transpose_kernel<1><<<grid, 256, 0, st>>>(job.R, N, D, M, XT); break;
      case 2: pq_transpose_kernel<2><<<grid, 256, 0, st>>>(job.R, N, D, M, XT); break;
      default: pq_transpose_kernel<4><<<grid, 256, 0, st>>>(job.R, N, D, M, XT); break;
    }
    MVR_CUDA(ctx, cudaGetLastError());
    ++launches;
  }
  MVR_CUDA(ctx, cudaEventRecord(ctx->fork_ev, st));
  MVR_CUDA(ctx, cudaStreamWaitEvent(side, ctx->fork_ev, 0));

  PqJob jg[kPqGroups];
  PqOut og[kPqGroups];
  mvr_pq_train_stats sg[kPqGroups] = {};
  unsigned char* wsg[kPqGroups];
  std::vector<unsigned char> hs[kPqGroups];
  size_t off = align256((size_t)M * N * S * sizeof(float));
  for (int g = 0; g < G; ++g) {
    const int m0 = group_lo(M, G, g), mg = group_lo(M, G, g + 1) - m0;
    jg[g] = job;
    jg[g].M = mg;
    jg[g].D = mg * S;
    jg[g].R = nullptr;  // the group reads XT only
    jg[g].seed = job.seed + (uint64_t)m0;  // subspace m0 + i uses seed +% (m0 + i)
    jg[g].xt = XT + (size_t)m0 * N * S;
    jg[g].xt_ready = true;
    jg[g].sub0 = job.sub0 + m0;
    og[g].d_codebooks = out.d_codebooks + (size_t)m0 * K * S;
    og[g].d_assign = out.d_assign ? out.d_assign + (size_t)m0 * N : nullptr;
    og[g].h_wcss = out.h_wcss ? out.h_wcss + m0 : nullptr;
    og[g].h_iters = out.h_iters ? out.h_iters + m0 : nullptr;
    og[g].stats = timing ? &sg[g] : nullptr;
    const PqLayout Lg = pq_layout(N, mg, S, K, sms, false);
    wsg[g] = ws + off;
    off += align256(Lg.total_bytes);
    hs[g].resize(Lg.small_bytes);
  }
  // group 1 on a second host thread and the side stream, group 0 here
  std::string err1;
  int rc1 = MVR_OK;
  std::thread worker([&] {
    ErrorSink sink(&err1);
    // a new host thread starts on device 0: bind it to the context's device
    // before it creates events or launches onto the side stream
    const cudaError_t e = cudaSetDevice(ctx->device);
    rc1 = e != cudaSuccess ? cuda_fail(ctx, e, "cudaSetDevice(ctx->device)")
                           : pq_kmeans_run_one(ctx, side, jg[1], og[1], wsg[1], hs[1].data(), sms, &ctx->pq_timing[1]);
  });
  std::string err0;
  int rc0 = MVR_OK;
  {
    ErrorSink sink(&err0);
    rc0 = pq_kmeans_run_one(ctx, st, jg[0], og[0], wsg[0], hs[0].data(), sms, &ctx->pq_timing[0]);
  }
  worker.join();
  // both groups' work is complete (each run synchronises its stream); the
  // join keeps the caller's stream ordered after the side stream's work
  const cudaError_t es = cudaStreamSynchronize(side);
  if (rc0 != MVR_OK) return fail(ctx, rc0, err0);
  if (rc1 != MVR_OK) return fail(ctx, rc1, err1);
  MVR_CUDA(ctx, es);
  MVR_CUDA(ctx, cudaEventRecord(ctx->join_ev, side));
  MVR_CUDA(ctx, cudaStreamWaitEvent(st, ctx->join_ev, 0));
  if (timing) {
    MVR_CUDA(ctx, cudaEventRecord(ctx->pev[1], st));
    MVR_CUDA(ctx, cudaEventSynchronize(ctx->pev[1]));
    mvr_pq_train_stats& o = *out.stats;
    o = sg[0];
    const mvr_pq_train_stats& b = sg[1];
    float t = 0.f;
    MVR_CUDA(ctx, cudaEventElapsedTime(&t, ctx->pev[0], ctx->pev[1]));
    o.total_ms = t;  // the whole call, both groups
    o.seed_ms = std::max(o.seed_ms, b.seed_ms);
    o.lloyd_ms = std::max(o.lloyd_ms, b.lloyd_ms);
    o.iters_max = std::max(o.iters_max, b.iters_max);
    o.iters_min = std::min(o.iters_min, b.iters_min);
    o.seed_fallbacks += b.seed_fallbacks;
    o.reseeds += b.reseeds;
    o.assign_ms += b.assign_ms;
    o.assign_launches += b.assign_launches;
    o.launches += b.launches + launches;
    o.assign_first_ms = std::max(o.assign_first_ms, b.assign_first_ms);
    o.lloyd_rows_total += b.lloyd_rows_total;
    o.lloyd_rows_exact += b.lloyd_rows_exact;
    o.filter_rows_rechecked += b.filter_rows_rechecked;
    o.filter_violations += b.filter_violations;
    o.seed_update_ms_sampled += b.seed_update_ms_sampled;
    o.seed_update_samples += b.seed_update_samples;
    o.list_ms += b.list_ms;
    o.list_launches += b.list_launches;
    o.list_distances += b.list_distances;
    o.groups = (uint32_t)G;
    o.host_enqueue_ms = std::max(o.host_enqueue_ms, b.host_enqueue_ms);
  } else {
    MVR_CUDA(ctx, cudaStreamSynchronize(st));
  }
  return MVR_OK;
}

int pq_kmeans_device(Ctx* ctx, const PqJob& job, const PqOut& out) {
  MVR_TRY(check_shape(ctx, job.D, job.M, job.S, job.K));
  const PqLayout L = pq_layout(job.N, job.M, job.S, job.K, ctx->sm_count);
  const int groups = pq_groups(ctx, job.N, job.M, job.K);
  unsigned char* ws = nullptr;
  MVR_TRY(scratch(ctx, kSlotMinDist, pq_ws_bytes(job.N, job.M, job.S, job.K, ctx->sm_count, groups), (void**)&ws));
  std::vector<unsigned char> hsmall(L.small_bytes);
  return pq_kmeans_run(ctx, ctx->stream, job, out, ws, hsmall.data(), ctx->sm_count);
}

int pq_kmeans_run_dist(Ctx* ctx, const PqJob& job, uint64_t row0, uint64_t N_total, const PqOut& out,
                       bool local_ok) {
  cudaStream_t st = ctx->stream;
  const int G = comm_size(ctx), me = comm_rank(ctx);
  const uint64_t N = job.N;
  const int D = job.D, M = job.M, S = job.S, K = job.K;
  MVR_TRY(check_shape(ctx, D, M, S, K));  // same parameters on every rank
  // rank-dependent checks travel with the rank table, so every rank fails
  // together instead of leaving the others in a collective
  local_ok = local_ok && N > 0 && N < (1ull << 32) && job.R && out.d_codebooks;
  const int sms = ctx->sm_count;

  // ---- dist bookkeeping (kSlotAux2) -----------------------------------------
  // rank table first: every rank's (row0, N) -> contiguous shards in rank order
  const size_t cb_floats = (size_t)M * K * S;
  Carve dc;
  const size_t o_tab_send = dc.take(16), o_tab = dc.take((size_t)G * 16), o_row0 = dc.take((size_t)G * 8);
  unsigned char* dws = nullptr;
  MVR_TRY(scratch(ctx, kSlotAux2, dc.off + 64, (void**)&dws));
  uint64_t* hp = nullptr;
  MVR_TRY(pinned(ctx, std::max<size_t>((size_t)G * 16 + (size_t)M * 8, 4096), (void**)&hp));
  hp[0] = row0;
  hp[1] = local_ok ? N : 0;  // a zero row count marks a rank that cannot run
  MVR_CUDA(ctx, cudaMemcpyAsync(dws + o_tab_send, hp, 16, cudaMemcpyHostToDevice, st));
  MVR_TRY(comm_allgather(ctx, dws + o_tab_send, dws + o_tab, 16));
  MVR_CUDA(ctx, cudaMemcpyAsync(hp, dws + o_tab, (size_t)G * 16, cudaMemcpyDeviceToHost, st));
  MVR_CUDA(ctx, cudaStreamSynchronize(st));
  std::vector<uint64_t> r0(G), rn(G);
  uint64_t expect = 0, Nmax = 0;
  for (int r = 0; r < G; ++r) {
    r0[r] = hp[2 * r];
    rn[r] = hp[2 * r + 1];
    if (rn[r] == 0)
      return fail(ctx, MVR_E_INVALID_ARGUMENT,
                  "rank " + std::to_string(r) + " cannot run (empty shard, null pointer or > 2^32-1 rows)");
    if (r0[r] != expect) return fail(ctx, MVR_E_INVALID_ARGUMENT, "shards must be contiguous in rank order");
    expect += rn[r];
    Nmax = std::max(Nmax, rn[r]);
  }
  if (expect != N_total) return fail(ctx, MVR_E_INVALID_ARGUMENT, "the shards do not add up to n_total");
  if ((uint64_t)K >= N_total) return fail(ctx, MVR_E_INVALID_ARGUMENT, "row-sharded training needs n_total > 256");
  const int ncmax = (int)((Nmax + kSeedChunk - 1) / kSeedChunk);
  const SeedBlock sb = seed_block(M, ncmax);
  const size_t o_seed = dc.take(sb.bytes), o_seed_all = dc.take(sb.bytes * G),
               o_con = dc.take((size_t)M * sizeof(RowContrib)), o_con_all = dc.take((size_t)G * M * sizeof(RowContrib)),
               o_need = dc.take((size_t)M * 4), o_empty = dc.take((size_t)M * 4), o_pick = dc.take((size_t)M * 8),
               o_sin = dc.take(cb_floats * 4), o_sout = dc.take(cb_floats * 4), o_gcnt = dc.take((size_t)M * K * 4),
               o_wst = dc.take((size_t)M * 4);
  MVR_TRY(scratch(ctx, kSlotAux2, dc.off, (void**)&dws));  // may move: re-derive everything below
  {
    for (int r = 0; r < G; ++r) hp[r] = r0[r];
    MVR_CUDA(ctx, cudaMemcpyAsync(dws + o_row0, hp, (size_t)G * 8, cudaMemcpyHostToDevice, st));
  }
  const uint64_t* d_row0 = (const uint64_t*)(dws + o_row0);
  unsigned char* seed_send = dws + o_seed;
  unsigned char* seed_all = dws + o_seed_all;
  RowContrib* con = (RowContrib*)(dws + o_con);
  RowContrib* con_all = (RowContrib*)(dws + o_con_all);
  uint32_t* d_need = (uint32_t*)(dws + o_need);
  uint32_t* d_empty = (uint32_t*)(dws + o_empty);
  uint64_t* d_pick = (uint64_t*)(dws + o_pick);
  float* sums_in = (float*)(dws + o_sin);
  float* sums_out = (float*)(dws + o_sout);
  uint32_t* gcounts = (uint32_t*)(dws + o_gcnt);
  float* wstart = (float*)(dws + o_wst);
  MVR_CUDA(ctx, cudaMemsetAsync(seed_send, 0, sb.bytes, st));  // padding chunks stay empty

  // ---- local engine workspace (kSlotMinDist) ---------------------------------
  const PqLayout L = pq_layout(N, M, S, K, sms);
  unsigned char* ws = nullptr;
  MVR_TRY(scratch(ctx, kSlotMinDist, L.total_bytes, (void**)&ws));
  std::vector<unsigned char> hsmall_v(L.small_bytes);
  unsigned char* hsmall = hsmall_v.data();
  const int nblk = L.nblk, nchunk = L.nchunk;
  const uint64_t rpc = L.rows_per_cta;
  float* XT = (float*)(ws + L.o_xt);
  float* mind = (float*)(ws + L.o_mind);
  uint8_t* asg = (uint8_t*)(ws + L.o_asg);
  float* sorted = (float*)(ws + L.o_sorted);
  uint32_t* hist = (uint32_t*)(ws + L.o_hist);
  unsigned char* small = ws;
  double* d_draws = (double*)(small + L.o_draws);
  uint64_t* d_chosen = (uint64_t*)(small + L.o_chosen);
  uint64_t* d_idx0 = (uint64_t*)(small + L.o_idx0);
  double* d_thr = (double*)(small + L.o_thr);
  uint32_t* d_counts = (uint32_t*)(small + L.o_counts);
  uint32_t* d_starts = (uint32_t*)(small + L.o_starts);
  float* d_wcss = (float*)(small + L.o_wcss);
  float* d_prev = (float*)(small + L.o_prev);
  int* d_status = (int*)(small + L.o_status);
  uint32_t* d_iters = (uint32_t*)(small + L.o_iters);
  uint32_t* d_fb = (uint32_t*)(small + L.o_fb);
  uint32_t* d_rs = (uint32_t*)(small + L.o_rs);
  uint8_t* d_state = (uint8_t*)(small + L.o_state);
  uint32_t* d_diag = (uint32_t*)(small + L.o_diag);
  double2* chunk = (double2*)seed_send;
  uint32_t* chunk_cnt = (uint32_t*)(seed_send + sb.o_cnt);
  int* d_nonf = (int*)(seed_send + sb.o_nonf);

  const bool timing = out.stats != nullptr;
  if (timing) {
    for (int e = 0; e < 4; ++e)
      if (!ctx->ev[e]) MVR_CUDA(ctx, cudaEventCreate(&ctx->ev[e]));
    MVR_CUDA(ctx, cudaEventRecord(ctx->ev[0], st));
  }
  // host RNG draws over the global row count, as the one-GPU engine
  std::memset(hsmall, 0, L.small_bytes);
  {
    double* hd = (double*)(hsmall + L.o_draws);
    uint64_t* hi0 = (uint64_t*)(hsmall + L.o_idx0);
    double* ht = (double*)(hsmall + L.o_thr);
    for (int m = 0; m < M; ++m) {
      Xoshiro256pp rng(job.seed + (uint64_t)m);
      hi0[m] = rng.below(N_total);
      hd[(size_t)m * K] = 0.0;
      for (int c = 1; c < K; ++c) hd[(size_t)m * K + c] = rng.unit_f64();
      ht[m] = HUGE_VAL;
    }
  }
  MVR_CUDA(ctx, cudaMemcpyAsync(small, hsmall, L.small_bytes, cudaMemcpyHostToDevice, st));
  uint32_t launches = 0;
  {
    const int grid = (int)std::min<uint64_t>((N + 255) / 256, (uint64_t)std::max(1, sms) * 8);
    switch (S) {
      case 1: pq_transpose_kernel<1><<<grid, 256, 0, st>>>(job.R, N, D, M, XT); break;
      case 2: pq_transpose_kernel<2><<<grid, 256, 0, st>>>(job.R, N, D, M, XT); break;
      default: pq_transpose_kernel<4><<<grid, 256, 0, st>>>(job.R, N, D, M, XT); break;
    }
    MVR_CUDA(ctx, cudaGetLastError());
    ++launches;
  }
  float* cb = out.d_codebooks;
  const size_t con_bytes = (size_t)M * sizeof(RowContrib);
  auto exchange_rows = [&](int step) -> int {  // contrib -> every rank's centroid `step`
    MVR_TRY(comm_allgather(ctx, con, con_all, con_bytes));
    pq_dist_take_kernel<<<1, 32, 0, st>>>(con_all, G, M, S, K, step, cb, d_chosen, d_state, d_need);
    MVR_CUDA(ctx, cudaGetLastError());
    launches += 1;
    return MVR_OK;
  };
  // rare paths: gathered copies of one subspace (kSlotAux3)
  auto gather_subspace = [&](int m, const float* src, float pad, bool with_rows, float** gv, float** gx) -> int {
    const size_t vb = (size_t)Nmax * 4, xb = with_rows ? (size_t)Nmax * S * 4 : 0;
    Carve rc;
    const size_t o_pv = rc.take(vb), o_px = rc.take(xb), o_gv = rc.take(vb * G), o_gx = rc.take(xb * G);
    unsigned char* rws = nullptr;
    MVR_TRY(scratch(ctx, kSlotAux3, rc.off, (void**)&rws));
    float* pv = (float*)(rws + o_pv);
    float* px = with_rows ? (float*)(rws + o_px) : nullptr;
    const int grid = (int)std::min<uint64_t>((Nmax + 255) / 256, 4096);
    pq_dist_pack_kernel<<<grid, 256, 0, st>>>(src, XT, N, Nmax, S, m, pad, pv, px);
    MVR_CUDA(ctx, cudaGetLastError());
    MVR_TRY(comm_allgather(ctx, pv, rws + o_gv, vb));
    if (with_rows) MVR_TRY(comm_allgather(ctx, px, rws + o_gx, xb));
    *gv = (float*)(rws + o_gv);
    *gx = with_rows ? (float*)(rws + o_gx) : nullptr;
    launches += 1;
    return MVR_OK;
  };
  uint32_t* hneed = (uint32_t*)hp;

  // ---- k-means++ ----------------------------------------------------------------
  pq_dist_offer_kernel<<<1, 32, 0, st>>>(XT, N, S, M, row0, d_idx0, nullptr, con);
  MVR_CUDA(ctx, cudaGetLastError());
  MVR_TRY(exchange_rows(0));
  for (int step = 0; step + 1 < K; ++step) {
    switch (S) {
      case 1: pq_seed_update_kernel<1><<<nchunk, kSeedThreads, 0, st>>>(XT, N, M, K, step, cb, mind, chunk, chunk_cnt, d_nonf, d_state, d_thr, ncmax); break;
      case 2: pq_seed_update_kernel<2><<<nchunk, kSeedThreads, 0, st>>>(XT, N, M, K, step, cb, mind, chunk, chunk_cnt, d_nonf, d_state, d_thr, ncmax); break;
      default: pq_seed_update_kernel<4><<<nchunk, kSeedThreads, 0, st>>>(XT, N, M, K, step, cb, mind, chunk, chunk_cnt, d_nonf, d_state, d_thr, ncmax); break;
    }
    MVR_CUDA(ctx, cudaGetLastError());
    MVR_TRY(comm_allgather(ctx, seed_send, seed_all, sb.bytes));
    pq_seed_select_dist_kernel<<<M, kSelectThreads, 0, st>>>(seed_all, G, ncmax, d_row0, me, N_total, XT, N, S, M,
                                                             K, step + 1, mind, d_draws, d_status, d_state, d_thr,
                                                             con, ctx->serial_draws ? 1 : 0);
    MVR_CUDA(ctx, cudaGetLastError());
    launches += 2;
    MVR_TRY(exchange_rows(step + 1));
    MVR_CUDA(ctx, cudaMemcpyAsync(hneed, d_need, (size_t)M * 4, cudaMemcpyDeviceToHost, st));
    MVR_CUDA(ctx, cudaStreamSynchronize(st));
    bool any = false;
    std::vector<uint32_t> need(hneed, hneed + M);
    for (int m = 0; m < M; ++m) {
      if (!need[m]) continue;
      any = true;
      float *gw = nullptr, *gx = nullptr;
      MVR_TRY(gather_subspace(m, mind, 0.f, false, &gw, &gx));
      pq_dist_chain_draw_kernel<<<1, 1, 0, st>>>(gw, G, Nmax, d_row0, d_draws, m, K, step + 1, d_pick, d_fb);
      MVR_CUDA(ctx, cudaGetLastError());
      ++launches;
    }
    if (any) {
      MVR_CUDA(ctx, cudaMemcpyAsync(d_need, need.data(), (size_t)M * 4, cudaMemcpyHostToDevice, st));
      pq_dist_offer_kernel<<<1, 32, 0, st>>>(XT, N, S, M, row0, d_pick, d_need, con);
      MVR_CUDA(ctx, cudaGetLastError());
      MVR_TRY(exchange_rows(step + 1));
    }
  }
  if (timing) MVR_CUDA(ctx, cudaEventRecord(ctx->ev[1], st));

  // ---- Lloyd ------------------------------------------------------------------------
  const bool check = !(job.tol == -INFINITY) && !std::isnan(job.tol);
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
      case 1: MVR_TRY(launch_assign<1>(ctx, st, kModeLloyd, job.R, XT, N, D, M, K, cb, nullptr, asg, mind, hist, d_state, nblk, rpc)); break;
      case 2: MVR_TRY(launch_assign<2>(ctx, st, kModeLloyd, job.R, XT, N, D, M, K, cb, nullptr, asg, mind, hist, d_state, nblk, rpc)); break;
      default: MVR_TRY(launch_assign<4>(ctx, st, kModeLloyd, job.R, XT, N, D, M, K, cb, nullptr, asg, mind, hist, d_state, nblk, rpc)); break;
    }
    if (timing) MVR_CUDA(ctx, cudaEventRecord(aev[2 * it + 1], st));
    pq_scan_kernel<<<M, kScanThreads, 0, st>>>(hist, nblk, K, d_counts, d_starts, d_state);
    MVR_CUDA(ctx, cudaGetLastError());
    MVR_CUDA(ctx, cudaMemcpyAsync(gcounts, d_counts, (size_t)M * K * 4, cudaMemcpyDeviceToDevice, st));
    MVR_TRY(comm_allreduce_sum_u32(ctx, gcounts, (size_t)M * K));
    launches += 6;
    const bool last = it + 1 == job.max_iters;
    if (check || (last && out.h_wcss)) {  // WCSS continued rank after rank
      if (me > 0) MVR_TRY(comm_recv(ctx, wstart, (size_t)M * 4, me - 1));
      pq_wcss_kernel<<<M, 256, 0, st>>>(mind, N, d_wcss, d_state, me > 0 ? wstart : nullptr);
      MVR_CUDA(ctx, cudaGetLastError());
      if (me + 1 < G) MVR_TRY(comm_send(ctx, d_wcss, (size_t)M * 4, me + 1));
      MVR_TRY(comm_broadcast(ctx, d_wcss, (size_t)M * 4, G - 1));
      ++launches;
    }
    switch (S) {
      case 1: { auto k = pq_scatter_kernel<1>; const size_t sm = scatter_smem(M, 1); MVR_CUDA(ctx, raise_smem_limit((const void*)k, (size_t)(sm))); k<<<nblk, 32 * M, sm, st>>>(XT, N, M, K, asg, hist, sorted, d_state, rpc); } break;
      case 2: { auto k = pq_scatter_kernel<2>; const size_t sm = scatter_smem(M, 2); MVR_CUDA(ctx, raise_smem_limit((const void*)k, (size_t)(sm))); k<<<nblk, 32 * M, sm, st>>>(XT, N, M, K, asg, hist, sorted, d_state, rpc); } break;
      default: { auto k = pq_scatter_kernel<4>; const size_t sm = scatter_smem(M, 4); MVR_CUDA(ctx, raise_smem_limit((const void*)k, (size_t)(sm))); k<<<nblk, 32 * M, sm, st>>>(XT, N, M, K, asg, hist, sorted, d_state, rpc); } break;
    }
    MVR_CUDA(ctx, cudaGetLastError());
    // centroid sums continued rank after rank; the last rank scales
    if (me > 0) MVR_TRY(comm_recv(ctx, sums_in, cb_floats * 4, me - 1));
    const float* sstart = me > 0 ? sums_in : nullptr;
    switch (S) {
      case 1: MVR_TRY(launch_chain<1>(ctx, st, sorted, N, M, K, d_counts, d_starts, sums_out, d_state, d_diag, sms, sstart, 1)); break;
      case 2: MVR_TRY(launch_chain<2>(ctx, st, sorted, N, M, K, d_counts, d_starts, sums_out, d_state, d_diag, sms, sstart, 1)); break;
      default: MVR_TRY(launch_chain<4>(ctx, st, sorted, N, M, K, d_counts, d_starts, sums_out, d_state, d_diag, sms, sstart, 1)); break;
    }
    if (me + 1 < G) {
      MVR_TRY(comm_send(ctx, sums_out, cb_floats * 4, me + 1));
    } else {
      pq_dist_scale_kernel<<<(int)((cb_floats + 255) / 256), 256, 0, st>>>(sums_out, gcounts, cb, d_state, M, K, S);
      MVR_CUDA(ctx, cudaGetLastError());
    }
    MVR_TRY(comm_broadcast(ctx, cb, cb_floats * 4, G - 1));
    // empty clusters (same decision on every rank)
    pq_dist_empty_kernel<<<M, 256, 0, st>>>(gcounts, d_state, M, K, d_empty);
    MVR_CUDA(ctx, cudaGetLastError());
    MVR_CUDA(ctx, cudaMemcpyAsync(hneed, d_empty, (size_t)M * 4, cudaMemcpyDeviceToHost, st));
    MVR_CUDA(ctx, cudaStreamSynchronize(st));
    std::vector<uint32_t> empty(hneed, hneed + M);
    for (int m = 0; m < M; ++m) {
      if (!empty[m]) continue;
      float *gv = nullptr, *gx = nullptr;
      MVR_TRY(gather_subspace(m, mind, -__builtin_inff(), true, &gv, &gx));
      pq_dist_reseed_kernel<<<1, 1024, 0, st>>>(gv, gx, G, Nmax, S, K, m, gcounts, cb, mind, N, me, d_rs);
      MVR_CUDA(ctx, cudaGetLastError());
      ++launches;
    }
    pq_reseed_converge_kernel<<<M, 1024, 0, st>>>(XT, N, S, K, gcounts, mind, cb, d_state, d_wcss, d_prev, d_iters,
                                                  d_rs, (int)it, check ? 1 : 0, job.tol, 0, nullptr, nullptr);
    MVR_CUDA(ctx, cudaGetLastError());
    launches += 5;
  }
  if (timing) MVR_CUDA(ctx, cudaEventRecord(ctx->ev[2], st));
  if (out.d_assign && job.max_iters > 0) {
    u8_to_u32_kernel<<<1024, 256, 0, st>>>(asg, out.d_assign, (uint64_t)M * N);
    MVR_CUDA(ctx, cudaGetLastError());
    ++launches;
  }
  MVR_CUDA(ctx, cudaMemcpyAsync(hsmall, small, L.small_bytes, cudaMemcpyDeviceToHost, st));
  MVR_CUDA(ctx, cudaStreamSynchronize(st));
  const int* hstatus = (const int*)(hsmall + L.o_status);
  for (int m = 0; m < M; ++m)
    if (hstatus[m] != MVR_OK)
      return fail(ctx, hstatus[m], std::string("subspace ") + std::to_string(m) + ": " + mvr_status_name(hstatus[m]));
  if (((const uint32_t*)(hsmall + L.o_diag))[3])
    return fail(ctx, MVR_E_TIMEOUT, "centroid sums: a bulk copy of cluster members did not complete in time");
  const uint32_t* hiters = (const uint32_t*)(hsmall + L.o_iters);
  const float* hw = (const float*)(hsmall + L.o_wcss);
  if (out.h_iters)
    for (int m = 0; m < M; ++m) out.h_iters[m] = job.max_iters ? hiters[m] : 0;
  if (out.h_wcss)
    for (int m = 0; m < M; ++m) out.h_wcss[m] = job.max_iters ? hw[m] : 0.f;
  if (out.stats) {
    std::memset(out.stats, 0, sizeof(*out.stats));
    out.stats->groups = 1;
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

int pq_kmeans_run_subspaces(Ctx* ctx, const PqJob& job, uint64_t row0, uint64_t N_total, const PqOut& out,
                            bool local_ok) {
  cudaStream_t st = ctx->stream;
  const int G = comm_size(ctx), me = comm_rank(ctx);
  const uint64_t N = job.N;
  const int D = job.D, M = job.M, S = job.S, K = job.K;
  MVR_TRY(check_shape(ctx, D, M, S, K));  // same parameters on every rank
  local_ok = local_ok && N > 0 && N < (1ull << 32) && job.R && out.d_codebooks;
  const int sms = ctx->sm_count;

  // ---- rank table: contiguous non-empty shards in rank order -------------
  Carve dc;
  const size_t o_tab_send = dc.take(16), o_tab = dc.take((size_t)G * 16), o_stat = dc.take((size_t)G * 8);
  unsigned char* dws = nullptr;
  MVR_TRY(scratch(ctx, kSlotAux2, dc.off, (void**)&dws));
  uint64_t* hp = nullptr;
  MVR_TRY(pinned(ctx, std::max<size_t>((size_t)G * 16, 4096), (void**)&hp));
  hp[0] = row0;
  hp[1] = local_ok ? N : 0;
  MVR_CUDA(ctx, cudaMemcpyAsync(dws + o_tab_send, hp, 16, cudaMemcpyHostToDevice, st));
  MVR_TRY(comm_allgather(ctx, dws + o_tab_send, dws + o_tab, 16));
  MVR_CUDA(ctx, cudaMemcpyAsync(hp, dws + o_tab, (size_t)G * 16, cudaMemcpyDeviceToHost, st));
  MVR_CUDA(ctx, cudaStreamSynchronize(st));
  std::vector<uint64_t> r0(G), rn(G);
  uint64_t expect = 0;
  for (int r = 0; r < G; ++r) {
    r0[r] = hp[2 * r];
    rn[r] = hp[2 * r + 1];
    if (rn[r] == 0)
      return fail(ctx, MVR_E_INVALID_ARGUMENT,
                  "rank " + std::to_string(r) + " cannot run (empty shard, null pointer or > 2^32-1 rows)");
    if (r0[r] != expect) return fail(ctx, MVR_E_INVALID_ARGUMENT, "shards must be contiguous in rank order");
    expect += rn[r];
  }
  if (expect != N_total) return fail(ctx, MVR_E_INVALID_ARGUMENT, "the shards do not add up to n_total");
  if ((uint64_t)K >= N_total) return fail(ctx, MVR_E_INVALID_ARGUMENT, "sharded training needs n_total > 256");
  if (N_total >= (1ull << 32)) return fail(ctx, MVR_E_INVALID_ARGUMENT, "more than 2^32-1 rows");
  auto m_lo = [&](int g) { return (int)((int64_t)M * g / G); };
  const int m0 = m_lo(me), m1 = m_lo(me + 1), Ml = m1 - m0;

  const bool timing = out.stats != nullptr;
  if (timing) {
    for (int e = 0; e < 4; ++e)
      if (!ctx->ev[e]) MVR_CUDA(ctx, cudaEventCreate(&ctx->ev[e]));
    MVR_CUDA(ctx, cudaEventRecord(ctx->ev[3], st));
  }

  // ---- this rank's rows, subspace-major (kSlotAux1) ---------------------------
  float* XT_loc = nullptr;
  MVR_TRY(scratch(ctx, kSlotAux1, (size_t)M * N * S * sizeof(float), (void**)&XT_loc));
  {
    const int grid = (int)std::min<uint64_t>((N + 255) / 256, (uint64_t)std::max(1, sms) * 8);
    switch (S) {
      case 1: pq_transpose_kernel<1><<<grid, 256, 0, st>>>(job.R, N, D, M, XT_loc); break;
      case 2: pq_transpose_kernel<2><<<grid, 256, 0, st>>>(job.R, N, D, M, XT_loc); break;
      default: pq_transpose_kernel<4><<<grid, 256, 0, st>>>(job.R, N, D, M, XT_loc); break;
    }
    MVR_CUDA(ctx, cudaGetLastError());
  }
  // ---- engine workspace for the owned subspaces over all rows ----------------
  const PqLayout L = pq_layout(N_total, std::max(Ml, 1), S, K, sms);
  const int groups = pq_groups(ctx, N_total, std::max(Ml, 1), K);
  unsigned char* ws = nullptr;
  MVR_TRY(scratch(ctx, kSlotMinDist, pq_ws_bytes(N_total, std::max(Ml, 1), S, K, sms, groups), (void**)&ws));
  float* XT_own = pq_ws_xt(ws, N_total, std::max(Ml, 1), S, K, sms, groups);
  uint32_t* asg_own = nullptr;
  if (out.d_assign) MVR_TRY(scratch(ctx, kSlotAux0, (size_t)std::max(Ml, 1) * N_total * 4, (void**)&asg_own));
  // exchange: subspace m of rank g's rows goes to the owner of m
  const size_t col = (size_t)S * sizeof(float);
  MVR_TRY(comm_group_start(ctx));
  for (int h = 0; h < G; ++h) {
    if (h == me) continue;
    for (int m = m_lo(h); m < m_lo(h + 1); ++m) MVR_TRY(comm_send(ctx, XT_loc + (size_t)m * N * S, N * col, h));
  }
  for (int g = 0; g < G; ++g) {
    if (g == me) continue;
    for (int m = m0; m < m1; ++m)
      MVR_TRY(comm_recv(ctx, XT_own + ((size_t)(m - m0) * N_total + r0[g]) * S, rn[g] * col, g));
  }
  MVR_TRY(comm_group_end(ctx));
  for (int m = m0; m < m1; ++m)
    MVR_CUDA(ctx, cudaMemcpyAsync(XT_own + ((size_t)(m - m0) * N_total + row0) * S, XT_loc + (size_t)m * N * S,
                                  N * col, cudaMemcpyDeviceToDevice, st));

  // ---- the one-GPU engine on the owned subspaces ----------------------------------
  int status = MVR_OK;
  int fail_m = M;
  mvr_pq_train_stats local_stats{};
  if (Ml > 0) {
    PqJob j2 = job;
    j2.R = nullptr;
    j2.N = N_total;
    j2.M = Ml;
    j2.D = Ml * S;  // the rows are read from XT only
    j2.seed = job.seed + (uint64_t)m0;  // subspace m0 + i uses seed +% (m0 + i)
    j2.xt_ready = true;
    PqOut o2;
    o2.d_codebooks = out.d_codebooks + (size_t)m0 * K * S;
    o2.d_assign = asg_own;
    o2.stats = timing ? &local_stats : nullptr;
    std::vector<unsigned char> hsmall(L.small_bytes);
    status = pq_kmeans_run(ctx, st, j2, o2, ws, hsmall.data(), sms);
    if (status != MVR_OK) {
      // the engine names the first failing local subspace in the message
      const std::string& e = ctx->last_error;
      const size_t p = e.find("subspace ");
      fail_m = m0 + (p == std::string::npos ? 0 : std::atoi(e.c_str() + p + 9));
      if (status == MVR_E_CUDA || status == MVR_E_OUT_OF_MEMORY) return status;  // no collective can follow safely
    }
  }
  // ---- statuses: every rank returns the first failing subspace's status -----
  {
    int64_t* hs = (int64_t*)hp;
    hs[0] = ((int64_t)fail_m << 32) | (uint32_t)status;
    MVR_CUDA(ctx, cudaMemcpyAsync(dws + o_tab_send, hs, 8, cudaMemcpyHostToDevice, st));
    MVR_TRY(comm_allgather(ctx, dws + o_tab_send, dws + o_stat, 8));
    MVR_CUDA(ctx, cudaMemcpyAsync(hs, dws + o_stat, (size_t)G * 8, cudaMemcpyDeviceToHost, st));
    MVR_CUDA(ctx, cudaStreamSynchronize(st));
    int best_m = M, best_s = MVR_OK;
    for (int r = 0; r < G; ++r) {
      const int s_r = (int)(uint32_t)(hs[r] & 0xffffffff), m_r = (int)(hs[r] >> 32);
      if (s_r != MVR_OK && m_r < best_m) {
        best_m = m_r;
        best_s = s_r;
      }
    }
    if (best_s != MVR_OK)
      return fail(ctx, best_s, std::string("subspace ") + std::to_string(best_m) + ": " + mvr_status_name(best_s));
  }
  // ---- codebooks to every rank; assignments back to the row owners -------------
  const size_t cb_sub = (size_t)K * S * sizeof(float);
  MVR_TRY(comm_group_start(ctx));
  for (int g = 0; g < G; ++g) {
    const int lo = m_lo(g), hi = m_lo(g + 1);
    if (hi > lo) MVR_TRY(comm_broadcast(ctx, out.d_codebooks + (size_t)lo * K * S, (size_t)(hi - lo) * cb_sub, g));
  }
  MVR_TRY(comm_group_end(ctx));
  if (out.d_assign) {
    MVR_TRY(comm_group_start(ctx));
    for (int h = 0; h < G; ++h) {
      if (h == me) continue;
      for (int m = m0; m < m1; ++m)
        MVR_TRY(comm_send(ctx, asg_own + (size_t)(m - m0) * N_total + r0[h], rn[h] * 4, h));
    }
    for (int g = 0; g < G; ++g) {
      if (g == me) continue;
      for (int m = m_lo(g); m < m_lo(g + 1); ++m) MVR_TRY(comm_recv(ctx, out.d_assign + (size_t)m * N, N * 4, g));
    }
    MVR_TRY(comm_group_end(ctx));
    for (int m = m0; m < m1; ++m)
      MVR_CUDA(ctx, cudaMemcpyAsync(out.d_assign + (size_t)m * N, asg_own + (size_t)(m - m0) * N_total + row0, N * 4,
                                    cudaMemcpyDeviceToDevice, st));
  }
  if (timing) MVR_CUDA(ctx, cudaEventRecord(ctx->ev[2], st));
  MVR_CUDA(ctx, cudaStreamSynchronize(st));
  if (out.stats) {
    *out.stats = local_stats;  // seeding / Lloyd / assign: this rank's engine
    float t = 0.f;
    cudaEventElapsedTime(&t, ctx->ev[3], ctx->ev[2]);
    out.stats->total_ms = t;  // exchange, engine and gather
  }
  return MVR_OK;
}

}  // namespace mvr
