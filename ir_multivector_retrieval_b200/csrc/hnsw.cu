// hnsw.cu — HNSW over the TAC centroids on the GPU: hnsw.build
// (src/index/hnsw.zig:314-946) and vec.normalizeRowsInPlace (vec.zig:185-253).
//
// The reference inserts nodes 1..n-1 in chunks (buildParallel, :639-946): for
// a chunk of min(256, q_base) nodes it plans every node against the graph as
// it stood at the chunk's start — greedy descent through the layers above
// the node's level, then per layer a beam search of width efConstruction and
// the heuristic neighbour selection — and then commits the plans in node
// order: the node's own lists, and the node appended to each chosen
// neighbour's list, which is shrunk by the heuristic when it exceeds its cap
// (2M on layer 0, M above). The serial path (n_threads <= 1, :477-625) is the
// same loop with chunks of one node.
//
// On the GPU, per chunk:
//   hnsw_plan_kernel     one CTA per node of the chunk: the whole plan, with
//                        the beam in shared memory
//   hnsw_commit_own      the chunk's own lists, and one bit per (layer,
//                        neighbour, node) marking every reverse edge
//   hnsw_commit_reverse  one warp per (layer, neighbour) that received edges:
//                        appends them in node order, shrinking as it goes.
//                        The chosen neighbours of a chunk are all older nodes
//                        (a chunk's nodes have no edges in the snapshot), and a
//                        shrink reads only its own node's list, so the
//                        neighbours are independent of one another and each
//                        replays exactly the reference's sequence.
// Levels come from the reference's RNG on the host (pickLevel draws one
// nextFloat per node, in node order, and nothing else draws), so the host
// knows every chunk's snapshot entry point and top level without waiting for
// the device; a build is one asynchronous stream of launches.
//
// The beam search (searchLayer, :995-1043) as a sorted array. The reference
// keeps a frontier max-heap C and a beam min-heap W of at most ef entries; a
// neighbour e of the expanded node is pushed to both when |W| < ef or
// sim(e) > min(W), and the worst of W is dropped when |W| > ef. Here:
//   * W is kept sorted (higher similarity first, equal similarities by the
//     smaller node id) with an "expanded" bit per entry.
//   * Candidate j of an expansion (the unvisited neighbours in list order) is
//     accepted iff fewer than ef of W ∪ {candidates before j} have similarity
//     >= sim(j). That is the reference's sequential test: W's similarities
//     are always the ef largest of everything offered so far, and a rejected
//     candidate is never above the minimum it was tested against.
//   * The new W is the first ef of the merge of W and the accepted set.
//   * The frontier entries that can still be expanded are the unexpanded
//     entries of W and those dropped from W with a similarity equal to W's
//     minimum (the reference stops only at a candidate strictly below the
//     minimum); anything lower never expands. Those ties are kept in a small
//     list; all of W ranks above them, so the next expansion is the first
//     unexpanded entry of W, else the tie with the smallest id.
// Latency: each expansion is a chain of dependent steps (pick, neighbour list,
// rows, similarities, acceptance, merge), so the kernel overlaps the global
// reads of the likely next expansion (the next unexpanded entry of W) with
// the current one: its neighbours' rows are copied into shared memory with
// cp.async while the current expansion proceeds, and the list of the one
// after it is prefetched into L1. A wrong guess costs only the copies.
// Equal similarities: the reference's heaps order them by similarity alone,
// so among exactly equal similarities its pop order follows the heap layout
// of Zig's std.PriorityQueue; here they go by node id (the smaller id first
// from the frontier and in the beam's output, the larger id first out of the
// beam). Everything else — the comparisons (similarity alone), list orders,
// the stable sorts of selectHeuristic, vec.dot's order — is the reference's.
//
// Arithmetic: vec.dot in the reference's order (len 64/128: four lane
// accumulators from +0 over the 4-wide chunks, then ((a0+a1)+a2)+a3; other
// lengths the same 4-lane loop plus the scalar tail; len 2 a0*b0 + a1*b1),
// every operation __fmul_rn/__fadd_rn.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <new>
#include <vector>

#include "../../include/mvr.h"
#include "mvr_internal.h"
#include "mvr_rng.h"

namespace mvr {
namespace {

constexpr uint32_t kChunk = 256;                // CHUNK_SIZE (hnsw.zig:272)
constexpr uint32_t kMaxLayers = 32;             // pickLevel caps levels at 31
constexpr uint32_t kMaxM = 32;                  // M; lists hold <= 2M at rest
constexpr uint32_t kMaxList = 2 * kMaxM + 1;    // cap + 1 during a commit
constexpr uint32_t kListPad = kMaxList + 1;     // even: keeps 8-byte entries aligned
constexpr uint32_t kPlanThreads = 256;
constexpr uint32_t kTieCap = 512;
constexpr uint32_t kExpanded = 0x80000000u;
constexpr uint32_t kMaskWords = kChunk / 32;    // one bit per node of a chunk
constexpr uint32_t kMaxEf = 2048;  // beam entries per CTA (8 per thread in a merge)
constexpr uint32_t kMaxDim = 256;
constexpr size_t kSmemLimit = 226 * 1024;  // 227 KB per CTA less the static control block

// device status bits
constexpr uint32_t kErrTies = 1u, kErrLoop = 2u;

struct DevGraph {
  uint32_t n, dim, m;
  uint32_t cap[kMaxLayers];
  uint32_t* ids[kMaxLayers];  // n x (cap + 1) per layer
  uint32_t* len[kMaxLayers];  // n per layer
};

struct Ent {
  float sim;
  uint32_t node;  // bit 31: expanded
};

__device__ __forceinline__ bool better(Ent a, Ent b) {
  const uint32_t na = a.node & ~kExpanded, nb = b.node & ~kExpanded;
  return a.sim > b.sim || (a.sim == b.sim && na < nb);
}

__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// vec.dot(a, b) in the reference's order; a and b 16-byte aligned when dim
// is a multiple of 4.
__device__ __forceinline__ float dot_ref(const float* __restrict__ a, const float* __restrict__ b, uint32_t dim) {
  if (dim == 2) return __fadd_rn(__fmul_rn(a[0], b[0]), __fmul_rn(a[1], b[1]));
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
  uint32_t i = 0;
  if ((dim & 3u) == 0) {
    const float4* a4 = reinterpret_cast<const float4*>(a);
    const float4* b4 = reinterpret_cast<const float4*>(b);
    for (uint32_t c = 0; c < dim / 4; ++c) {
      const float4 x = a4[c], y = b4[c];
      a0 = __fadd_rn(a0, __fmul_rn(x.x, y.x));
      a1 = __fadd_rn(a1, __fmul_rn(x.y, y.y));
      a2 = __fadd_rn(a2, __fmul_rn(x.z, y.z));
      a3 = __fadd_rn(a3, __fmul_rn(x.w, y.w));
    }
    return __fadd_rn(__fadd_rn(__fadd_rn(a0, a1), a2), a3);
  }
  for (; i + 4 <= dim; i += 4) {
    a0 = __fadd_rn(a0, __fmul_rn(a[i], b[i]));
    a1 = __fadd_rn(a1, __fmul_rn(a[i + 1], b[i + 1]));
    a2 = __fadd_rn(a2, __fmul_rn(a[i + 2], b[i + 2]));
    a3 = __fadd_rn(a3, __fmul_rn(a[i + 3], b[i + 3]));
  }
  float s = __fadd_rn(__fadd_rn(__fadd_rn(a0, a1), a2), a3);
  for (; i < dim; ++i) s = __fadd_rn(s, __fmul_rn(a[i], b[i]));
  return s;
}

// The same with b at a padded shared-memory row (scalar loads; the rows of
// consecutive lanes sit in consecutive banks).
__device__ __forceinline__ float dot_ref_scalar(const float* a, const float* b, uint32_t dim) {
  if (dim == 2) return __fadd_rn(__fmul_rn(a[0], b[0]), __fmul_rn(a[1], b[1]));
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
  uint32_t i = 0;
  for (; i + 4 <= dim; i += 4) {
    a0 = __fadd_rn(a0, __fmul_rn(a[i], b[i]));
    a1 = __fadd_rn(a1, __fmul_rn(a[i + 1], b[i + 1]));
    a2 = __fadd_rn(a2, __fmul_rn(a[i + 2], b[i + 2]));
    a3 = __fadd_rn(a3, __fmul_rn(a[i + 3], b[i + 3]));
  }
  float s = __fadd_rn(__fadd_rn(__fadd_rn(a0, a1), a2), a3);
  for (; i < dim; ++i) s = __fadd_rn(s, __fmul_rn(a[i], b[i]));
  return s;
}

// ---------------------------------------------------------------------------
// plan
// ---------------------------------------------------------------------------

struct PlanLayout {  // byte offsets into dynamic shared memory
  uint32_t qv, w, vis, cn, cs, cacc, as, apos, ev, ties, rv, rid, cv, stg;
  uint32_t nwords, rstride, stage_slots, bytes;
};

struct PlanArgs {
  DevGraph g;
  PlanLayout lay;
  const float* x;
  const uint8_t* levels;
  uint32_t q_base, snap_entry, snap_max, ef;
  uint32_t* chosen;    // [kChunk][kMaxLayers][kMaxM]
  uint32_t* n_chosen;  // [kChunk][kMaxLayers]
  uint32_t* status;
};

struct PlanCtl {
  uint32_t wn, hint, newhint, pop, nt, nev, p0, full, cur;
  uint32_t scan[kPlanThreads / 32];
  float tsim, newmin;
  uint32_t bal[2];
  uint32_t stg_node[2], stg_mask[2][2];
  uint32_t hk[kPlanThreads / 32], hp[kPlanThreads / 32], hslot[kPlanThreads / 32], hkept, nr;
};

// greedySearchLayer (hnsw.zig:969-991), warp 0: the first strict maximum of
// each list, while it improves.
__device__ uint32_t greedy_layer(const PlanArgs& a, const float* qv, uint32_t L, uint32_t cur) {
  const uint32_t lane = threadIdx.x & 31, dim = a.g.dim, cap = a.g.cap[L];
  float cur_sim = dot_ref(qv, a.x + (size_t)cur * dim, dim);
  for (uint32_t step = 0; step <= a.g.n; ++step) {
    const uint32_t cnt = a.g.len[L][cur];
    const uint32_t* list = a.g.ids[L] + (size_t)cur * (cap + 1);
    float bs = -INFINITY;
    uint32_t bi = 0xFFFFFFFFu;
    for (uint32_t i = lane; i < cnt; i += 32) {
      const float s = dot_ref(qv, a.x + (size_t)list[i] * dim, dim);
      if (bi == 0xFFFFFFFFu || s > bs) {  // first maximum of this lane's entries
        bs = s;
        bi = i;
      }
    }
    for (int o = 16; o; o >>= 1) {
      const float os = __shfl_xor_sync(~0u, bs, o);
      const uint32_t oi = __shfl_xor_sync(~0u, bi, o);
      if (oi != 0xFFFFFFFFu && (bi == 0xFFFFFFFFu || os > bs || (os == bs && oi < bi))) {
        bs = os;
        bi = oi;
      }
    }
    if (bi == 0xFFFFFFFFu || !(bs > cur_sim)) return cur;
    cur_sim = bs;
    cur = list[bi];
  }
  return cur;
}

// vec.dot(q, x) for dim 64 / 128 with every load of the row issued before
// the first add (the reference's order: lane accumulators over the 4-wide
// chunks in order, then ((a0 + a1) + a2) + a3).
template <int D>
__device__ __forceinline__ float dot_fixed(const float* qv, const float* __restrict__ xr) {
  const float4* q4 = reinterpret_cast<const float4*>(qv);
  const float4* x4 = reinterpret_cast<const float4*>(xr);
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
  for (int h = 0; h < D / 64; ++h) {
    float4 v[16];
#pragma unroll
    for (int c = 0; c < 16; ++c) v[c] = x4[h * 16 + c];
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      const float4 y = q4[h * 16 + c];
      a0 = __fadd_rn(a0, __fmul_rn(y.x, v[c].x));
      a1 = __fadd_rn(a1, __fmul_rn(y.y, v[c].y));
      a2 = __fadd_rn(a2, __fmul_rn(y.z, v[c].z));
      a3 = __fadd_rn(a3, __fmul_rn(y.w, v[c].w));
    }
  }
  return __fadd_rn(__fadd_rn(__fadd_rn(a0, a1), a2), a3);
}

__device__ __forceinline__ float dot_row(const float* qv, const float* __restrict__ xr, uint32_t dim) {
  if (dim == 64) return dot_fixed<64>(qv, xr);
  if (dim == 128) return dot_fixed<128>(qv, xr);
  return dot_ref(qv, xr, dim);
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(smem))),
               "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ void prefetch_l1(const void* p) { asm volatile("prefetch.global.L1 [%0];" ::"l"(p)); }

// Number of leading entries of W[lo, hi) for which pred holds (pred is true
// on a prefix: W is sorted). Whole warp, 32-way steps.
template <class Pred>
__device__ __forceinline__ uint32_t warp_boundary(const Ent* W, uint32_t lo, uint32_t hi, Pred pred) {
  const uint32_t lane = threadIdx.x & 31;
  while (lo < hi) {
    const uint32_t stride = (hi - lo + 31) / 32, idx = lo + lane * stride;
    const uint32_t c = __popc(__ballot_sync(~0u, idx < hi && pred(W[idx])));
    if (c == 0) break;
    const uint32_t nhi = lo + c * stride;
    lo = lo + (c - 1) * stride + 1;
    hi = nhi < hi ? nhi : hi;
  }
  return lo;
}

constexpr uint32_t kTail = kMaxEf / kPlanThreads;  // beam entries per thread in a merge

__global__ void __launch_bounds__(kPlanThreads, 2) hnsw_plan_kernel(PlanArgs a) {
  extern __shared__ __align__(16) unsigned char sm[];
  __shared__ PlanCtl ctl;
  const PlanLayout& lay = a.lay;
  float* qv = reinterpret_cast<float*>(sm + lay.qv);
  Ent* W = reinterpret_cast<Ent*>(sm + lay.w);
  uint32_t* vis = reinterpret_cast<uint32_t*>(sm + lay.vis);
  uint32_t* cn = reinterpret_cast<uint32_t*>(sm + lay.cn);
  float* cs = reinterpret_cast<float*>(sm + lay.cs);
  uint32_t* cacc = reinterpret_cast<uint32_t*>(sm + lay.cacc);
  Ent* as = reinterpret_cast<Ent*>(sm + lay.as);
  uint32_t* apos = reinterpret_cast<uint32_t*>(sm + lay.apos);
  Ent* ev = reinterpret_cast<Ent*>(sm + lay.ev);
  uint32_t* ties = reinterpret_cast<uint32_t*>(sm + lay.ties);
  float* rv = reinterpret_cast<float*>(sm + lay.rv);
  uint32_t* rid = reinterpret_cast<uint32_t*>(sm + lay.rid);
  float* cv = reinterpret_cast<float*>(sm + lay.cv);
  float* stg = reinterpret_cast<float*>(sm + lay.stg);

  const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t qi = blockIdx.x, q = a.q_base + qi, dim = a.g.dim, ef = a.ef, m = a.g.m;
  for (uint32_t i = tid; i < dim; i += blockDim.x) qv[i] = a.x[(size_t)q * dim + i];
  const uint32_t l_new = a.levels[q];
  __syncthreads();

  // Phase A: greedy descent through the layers above l_new
  if (warp == 0) {
    uint32_t cur = a.snap_entry;
    if (a.snap_max > l_new)
      for (uint32_t L = a.snap_max; L > l_new; --L) cur = greedy_layer(a, qv, L, cur);
    if (lane == 0) ctl.cur = cur;
  }
  __syncthreads();
  const uint32_t top = a.snap_max < l_new ? a.snap_max : l_new;

  for (int Ls = (int)top; Ls >= 0; --Ls) {
    const uint32_t L = (uint32_t)Ls, cap = a.g.cap[L];
    const uint32_t* ids = a.g.ids[L];
    const uint32_t* lens = a.g.len[L];
    // ---- searchLayer from ctl.cur
    for (uint32_t i = tid; i < lay.nwords; i += blockDim.x) vis[i] = 0;
    __syncthreads();
    if (tid == 0) {
      const uint32_t e0 = ctl.cur;
      W[0] = Ent{dot_ref(qv, a.x + (size_t)e0 * dim, dim), e0};
      vis[e0 >> 5] |= 1u << (e0 & 31);
      ctl.wn = 1;
      ctl.hint = 0;
      ctl.nt = 0;
      ctl.tsim = 0.f;
      ctl.full = 0;
      ctl.nev = 0;
      ctl.stg_node[0] = ctl.stg_node[1] = 0xFFFFFFFFu;
    }
    __syncthreads();
    for (uint32_t it = 0;; ++it) {
      if (it > a.g.n) {  // every node expands at most once
        if (tid == 0) atomicOr(a.status, kErrLoop);
        break;
      }
      // ---- P1: the next expansion. All warps scan 256 entries of W from
      // the hint (one ballot each); the first unexpanded entry is the next
      // expansion and the two after it are guesses that only steer the
      // copies below. Meanwhile the last warp keeps the ties the last merge
      // evicted: entries dropped with similarity equal to the new minimum
      // stay expandable (the reference stops only strictly below it).
      const uint32_t wn = ctl.wn, hint0 = ctl.hint;
      if (warp == kPlanThreads / 32 - 1 && ctl.full) {
        uint32_t nt = ctl.nt;
        const float mn = ctl.newmin;
        if (nt && ctl.tsim != mn) nt = 0;
        const uint32_t nev = ctl.nev;
        for (uint32_t base = 0; base < nev; base += 32) {
          const uint32_t i = base + lane;
          const bool tt = i < nev && ev[i].sim == mn;
          const uint32_t bt = __ballot_sync(~0u, tt);
          if (tt) {
            const uint32_t slot = nt + __popc(bt & lanemask_lt());
            if (slot < kTieCap) ties[slot] = ev[i].node & ~kExpanded;
          }
          nt += __popc(bt);
        }
        if (nt > kTieCap) {
          nt = kTieCap;
          if (lane == 0) atomicOr(a.status, kErrTies);
        }
        __syncwarp();
        if (lane == 0) {
          ctl.nt = nt;
          ctl.tsim = mn;
          ctl.full = 0;
        }
      }
      uint32_t p = wn, p2 = wn, p3 = wn;
      for (uint32_t base = hint0;;) {  // uniform: every thread reads the same words
        const uint32_t i = base + 32 * warp + lane;
        const uint32_t bw = __ballot_sync(~0u, i < wn && !(W[i].node & kExpanded));
        if (lane == 0) ctl.scan[warp] = bw;
        __syncthreads();
        uint32_t nf = 0;
        for (uint32_t w = 0; w < kPlanThreads / 32 && nf < 3; ++w) {
          uint32_t bb = ctl.scan[w];
          while (bb && nf < 3) {
            const uint32_t idx = base + 32 * w + __ffs(bb) - 1;
            if (nf == 0)
              p = idx;
            else if (nf == 1)
              p2 = idx;
            else
              p3 = idx;
            ++nf;
            bb &= bb - 1;
          }
        }
        if (nf || base + kPlanThreads >= wn) break;
        base += kPlanThreads;
        __syncthreads();  // the words are rewritten by the next window
      }
      uint32_t c, spec = 0xFFFFFFFFu, spec2 = 0xFFFFFFFFu;
      if (p < wn) {
        c = W[p].node & ~kExpanded;
        if (p2 < wn) spec = W[p2].node & ~kExpanded;
        if (p3 < wn) spec2 = W[p3].node & ~kExpanded;
        if (tid == 0) {
          W[p].node = c | kExpanded;
          ctl.hint = p;
        }
      } else {  // W is exhausted: the tie with the smallest id, if any
        const uint32_t nt = ctl.nt;
        if (nt == 0) break;
        if (warp == 0) {
          uint32_t best = 0xFFFFFFFFu, bi = 0;
          for (uint32_t i = lane; i < nt; i += 32)
            if (ties[i] < best) {
              best = ties[i];
              bi = i;
            }
          for (int o = 16; o; o >>= 1) {
            const uint32_t ob = __shfl_xor_sync(~0u, best, o), oi = __shfl_xor_sync(~0u, bi, o);
            if (ob < best) {
              best = ob;
              bi = oi;
            }
          }
          __syncwarp();
          if (lane == 0) {
            ctl.pop = best;
            ties[bi] = ties[nt - 1];
            ctl.nt = nt - 1;
          }
        }
        __syncthreads();
        c = ctl.pop;
      }
      // ---- P2: the unvisited neighbours of c in list order (threads < 64;
      // the count and the ids are read together). Warps 2-3 stage the rows of
      // the guessed next expansion's unvisited neighbours into shared memory
      // with asynchronous copies that complete during the next iteration (a
      // wrong guess costs only the copies); warp 4 prefetches the list of the
      // guess after it into L1.
      const uint32_t sbuf = it & 1u;  // staged now; the previous iteration's is sbuf ^ 1
      uint32_t e = 0;
      bool fresh = false;
      if (tid < 64) {
        const uint32_t cnt = lens[c];
        if (tid <= cap) e = ids[(size_t)c * (cap + 1) + tid];
        if (tid < cnt) {
          const uint32_t bit = 1u << (e & 31);
          fresh = !(atomicOr(&vis[e >> 5], bit) & bit);
        }
        const uint32_t b = __ballot_sync(~0u, fresh);
        if (lane == 0) ctl.bal[warp] = b;
      } else if (warp < 4) {
        cp_async_wait_all();  // this thread's copies of the previous iteration
        const uint32_t u = tid - 64;
        bool staged = false;
        if (spec != 0xFFFFFFFFu && u < lay.stage_slots) {
          const uint32_t cnt2 = lens[spec];
          const uint32_t v = u <= cap ? ids[(size_t)spec * (cap + 1) + u] : 0u;
          if (u < cnt2 && !((vis[v >> 5] >> (v & 31)) & 1u)) {
            const char* src = reinterpret_cast<const char*>(a.x + (size_t)v * dim);
            char* dst = reinterpret_cast<char*>(stg + ((size_t)sbuf * lay.stage_slots + u) * dim);
            for (uint32_t o = 0; o < dim * 4; o += 16) cp_async16(dst + o, src + o);
            staged = true;
          }
        }
        cp_async_commit();
        const uint32_t b = __ballot_sync(~0u, staged);
        if (lane == 0) ctl.stg_mask[sbuf][warp - 2] = b;
        if (u == 0) ctl.stg_node[sbuf] = spec;
      } else if (warp == 4) {
        if (spec2 != 0xFFFFFFFFu) {
          const uint32_t lines = ((cap + 1) * 4 + 127) / 128;
          if (lane < lines) prefetch_l1(reinterpret_cast<const char*>(ids + (size_t)spec2 * (cap + 1)) + lane * 128);
          if (lane == lines) prefetch_l1(lens + spec2);
        }
      }
      __syncthreads();
      const uint32_t b0 = ctl.bal[0], b1 = ctl.bal[1];
      const uint32_t k = __popc(b0) + __popc(b1);
      // ---- P3: similarity of each fresh neighbour, by the thread that read
      // it: from the staged row when the previous iteration guessed c
      if (fresh) {
        const uint32_t j = (warp == 0 ? 0u : (uint32_t)__popc(b0)) + __popc((warp == 0 ? b0 : b1) & lanemask_lt());
        const uint32_t pb = sbuf ^ 1u;
        const bool hit = ctl.stg_node[pb] == c && tid < lay.stage_slots && ((ctl.stg_mask[pb][tid >> 5] >> (tid & 31)) & 1u);
        cn[j] = e;
        cs[j] = dot_row(qv, hit ? stg + ((size_t)pb * lay.stage_slots + tid) * dim : a.x + (size_t)e * dim, dim);
      }
      if (tid == 0) {
        ctl.p0 = 0xFFFFFFFFu;
        ctl.newhint = 0xFFFFFFFFu;
        ctl.nev = 0;
      }
      __syncthreads();
      if (k == 0) continue;
      // ---- P4: acceptance of candidate j: fewer than ef of W and the
      // candidates before j are at least as similar. One warp per candidate;
      // the count in W by 32-way steps (W's similarities never increase).
      for (uint32_t j = warp; j < k; j += kPlanThreads / 32) {
        const float sj = cs[j];
        const uint32_t inw = warp_boundary(W, 0, wn, [sj](Ent w) { return w.sim >= sj; });
        const uint32_t cp = __popc(__ballot_sync(~0u, lane < j && cs[lane] >= sj)) +
                            __popc(__ballot_sync(~0u, lane + 32 < j && cs[lane + 32] >= sj));
        if (lane == 0) cacc[j] = (inw + cp < ef) ? 1u : 0u;
      }
      __syncthreads();
      const uint32_t a0 = __ballot_sync(~0u, lane < k && cacc[lane]);
      const uint32_t a1 = __ballot_sync(~0u, lane + 32 < k && cacc[lane + 32]);
      const uint32_t na = __popc(a0) + __popc(a1);
      if (na == 0) continue;
      // ---- P5: rank among the accepted (beam order) and the place in W,
      // one warp per accepted candidate
      for (uint32_t j = warp; j < k; j += kPlanThreads / 32) {
        if (!((j < 32 ? (a0 >> j) : (a1 >> (j - 32))) & 1u)) continue;
        const Ent me{cs[j], cn[j]};
        const uint32_t r =
            __popc(__ballot_sync(~0u, ((a0 >> lane) & 1u) && better(Ent{cs[lane], cn[lane]}, me))) +
            __popc(__ballot_sync(~0u, ((a1 >> lane) & 1u) && better(Ent{cs[lane + 32], cn[lane + 32]}, me)));
        const uint32_t pw = warp_boundary(W, 0, wn, [me](Ent w) { return better(w, me); });
        if (lane == 0) {
          as[r] = me;
          apos[r] = r + pw;
          atomicMin(&ctl.p0, pw);
          if (r == 0) atomicMin(&ctl.newhint, pw);
        }
      }
      __syncthreads();
      // ---- P6/P7: merge in place: entries of W from p0 on move down by the
      // number of accepted entries ahead of them; the first ef are kept.
      // Every move is read before any is written.
      const uint32_t p0 = ctl.p0, hint = ctl.hint, total = wn + na;
      Ent te[kTail];
      uint32_t tp[kTail];
#pragma unroll
      for (uint32_t t = 0; t < kTail; ++t) {
        const uint32_t i = p0 + tid + t * kPlanThreads;
        tp[t] = 0xFFFFFFFFu;
        if (i < wn) {
          te[t] = W[i];
          uint32_t lo = 0, hi = na;
          while (lo < hi) {
            const uint32_t mid = (lo + hi) >> 1;
            if (better(as[mid], te[t]))
              lo = mid + 1;
            else
              hi = mid;
          }
          tp[t] = i + lo;
          if (i == hint) atomicMin(&ctl.newhint, tp[t]);
        }
      }
      __syncthreads();
#pragma unroll
      for (uint32_t t = 0; t < kTail; ++t) {
        if (tp[t] == 0xFFFFFFFFu) continue;
        if (tp[t] < ef) {
          W[tp[t]] = te[t];
          if (tp[t] == ef - 1) ctl.newmin = te[t].sim;
        } else if (!(te[t].node & kExpanded)) {  // at most na <= 64 leave
          ev[atomicAdd(&ctl.nev, 1u)] = te[t];
        }
      }
      if (tid < na) {
        const uint32_t np = apos[tid];
        if (np < ef) {
          W[np] = as[tid];
          if (np == ef - 1) ctl.newmin = as[tid].sim;
        } else {
          ev[atomicAdd(&ctl.nev, 1u)] = as[tid];
        }
      }
      if (tid == 0) {
        const uint32_t nw = total < ef ? total : ef;
        ctl.wn = nw;
        ctl.hint = hint < p0 ? hint : (ctl.newhint < nw ? ctl.newhint : nw);
        ctl.full = total > ef ? 1u : 0u;  // the next P1 keeps the live ties
      }
      __syncthreads();
    }
    cp_async_wait_all();
    __syncthreads();
    // ---- the beam, best first, is W[0 .. wn); next layer starts at its best
    const uint32_t wn = ctl.wn;
    // ---- selectHeuristic: keep a candidate unless a chosen neighbour is
    // strictly more similar to it than the query is. Eight candidates per
    // round, one per warp: each is tested against the neighbours chosen
    // before the round and against the earlier candidates of the round, then
    // one thread keeps them in order — the reference's sequential rule.
    constexpr uint32_t kHB = kPlanThreads / 32;
    if (tid == 0) ctl.nr = 0;
    __syncthreads();
    for (uint32_t b = 0; b < wn; b += kHB) {
      const uint32_t nr = ctl.nr;
      if (nr >= m) break;
      const uint32_t i = b + warp;
      float* cvw = cv + (size_t)warp * lay.rstride;
      Ent ce{0.f, 0u};
      if (i < wn) {
        ce = W[i];
        const uint32_t cnode = ce.node & ~kExpanded;
        for (uint32_t d = lane; d < dim; d += 32) cvw[d] = a.x[(size_t)cnode * dim + d];
      }
      __syncthreads();
      if (i < wn) {
        bool pk = false, pp = false;
        if (lane < nr) pk = dot_ref_scalar(cvw, rv + (size_t)lane * lay.rstride, dim) > ce.sim;
        if (lane < warp) pp = dot_ref_scalar(cvw, cv + (size_t)lane * lay.rstride, dim) > ce.sim;
        const uint32_t bk = __ballot_sync(~0u, pk), bp = __ballot_sync(~0u, pp);
        if (lane == 0) {
          ctl.hk[warp] = bk;
          ctl.hp[warp] = bp;
        }
      }
      __syncthreads();
      if (tid == 0) {
        uint32_t n = nr, kept = 0;
        for (uint32_t w = 0; w < kHB && b + w < wn && n < m; ++w)
          if (ctl.hk[w] == 0 && (ctl.hp[w] & kept) == 0) {
            kept |= 1u << w;
            rid[n] = W[b + w].node & ~kExpanded;
            ctl.hslot[w] = n++;
          }
        ctl.hkept = kept;
        ctl.nr = n;
      }
      __syncthreads();
      if ((ctl.hkept >> warp) & 1u) {
        float* dst = rv + (size_t)ctl.hslot[warp] * lay.rstride;
        for (uint32_t d = lane; d < dim; d += 32) dst[d] = cvw[d];
      }
      __syncthreads();
    }
    if (warp == 0) {
      const uint32_t nr = ctl.nr;
      uint32_t* out = a.chosen + ((size_t)qi * kMaxLayers + L) * kMaxM;
      if (lane < nr) out[lane] = rid[lane];
      if (lane == 0) {
        a.n_chosen[(size_t)qi * kMaxLayers + L] = nr;
        ctl.cur = wn ? (W[0].node & ~kExpanded) : ctl.cur;
      }
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// commit
// ---------------------------------------------------------------------------

struct CommitArgs {
  DevGraph g;
  const float* x;
  const uint8_t* levels;
  uint32_t q_base, chunk_len, snap_max;
  const uint32_t* chosen;
  const uint32_t* n_chosen;
  uint32_t* mask;     // [layers][n][kMaskWords]
  uint32_t* touched;  // [layers][n]
  uint32_t* tlist;    // layer * n + node
  uint32_t* tcount;
  uint32_t warp_smem_floats;
  uint32_t rstride;
};

// The chunk's own lists (each empty before: nothing links to a node of its
// own chunk) and the reverse-edge marks. One warp per node of the chunk.
__global__ void hnsw_commit_own(CommitArgs a) {
  const uint32_t qi = blockIdx.x, lane = threadIdx.x, q = a.q_base + qi, n = a.g.n;
  const uint32_t l_new = a.levels[q];
  const uint32_t top = a.snap_max < l_new ? a.snap_max : l_new;
  for (uint32_t L = 0; L <= top; ++L) {
    const uint32_t nc = a.n_chosen[(size_t)qi * kMaxLayers + L], cap = a.g.cap[L];
    if (lane < nc) {
      const uint32_t r = a.chosen[((size_t)qi * kMaxLayers + L) * kMaxM + lane];
      a.g.ids[L][(size_t)q * (cap + 1) + lane] = r;
      const size_t key = (size_t)L * n + r;
      atomicOr(&a.mask[key * kMaskWords + (qi >> 5)], 1u << (qi & 31));
      if (atomicExch(&a.touched[key], 1u) == 0u) a.tlist[atomicAdd(a.tcount, 1u)] = (uint32_t)key;
    }
    if (lane == 0) a.g.len[L][q] = nc;
  }
}

// shrinkNeighbours (hnsw.zig:1090-1107) of node r's list (len = cap + 1),
// whole warp; returns the kept count. Shared scratch per warp: xr[dimp],
// cv[dimp], rv[2M][rstride], ss[kListPad], sid[kListPad], so[kMaxList].
__device__ uint32_t shrink_list(const CommitArgs& a, uint32_t* list, uint32_t len, uint32_t cap, float* xr,
                                float* cv, float* rv, float* ss, uint32_t* sid, Ent* so) {
  const uint32_t lane = threadIdx.x & 31, dim = a.g.dim;
  for (uint32_t i = lane; i < len; i += 32) {
    const uint32_t id = list[i];
    sid[i] = id;
    ss[i] = dot_ref(xr, a.x + (size_t)id * dim, dim);
  }
  __syncwarp();
  // std.mem.sort by similarity, descending, stable
  for (uint32_t i = lane; i < len; i += 32) {
    const float s = ss[i];
    uint32_t r = 0;
    for (uint32_t j = 0; j < len; ++j) r += (ss[j] > s || (ss[j] == s && j < i)) ? 1u : 0u;
    so[r] = Ent{s, sid[i]};
  }
  __syncwarp();
  uint32_t nr = 0;
  for (uint32_t i = 0; i < len && nr < cap; ++i) {
    const Ent ce = so[i];
    for (uint32_t d = lane; d < dim; d += 32) cv[d] = a.x[(size_t)ce.node * dim + d];
    __syncwarp();
    bool pr = false;
    for (uint32_t j = lane; j < nr; j += 32) pr |= dot_ref_scalar(cv, rv + (size_t)j * a.rstride, dim) > ce.sim;
    if (__ballot_sync(~0u, pr) == 0) {
      for (uint32_t d = lane; d < dim; d += 32) rv[(size_t)nr * a.rstride + d] = cv[d];
      if (lane == 0) sid[nr] = ce.node;  // sid[0 .. nr) is no longer read
      ++nr;
    }
    __syncwarp();
  }
  for (uint32_t i = lane; i < nr; i += 32) list[i] = sid[i];
  __syncwarp();
  return nr;
}

// The reverse edges of the chunk: for each (layer, neighbour) that received
// any, append the chunk's nodes in order, shrinking whenever the list
// exceeds its cap (hnsw.zig:908-923). One warp per (layer, neighbour).
__global__ void hnsw_commit_reverse(CommitArgs a) {
  extern __shared__ __align__(16) unsigned char sm[];
  const uint32_t lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const uint32_t dim = a.g.dim, dimp = (dim + 3u) & ~3u, n = a.g.n;
  float* base = reinterpret_cast<float*>(sm) + (size_t)wib * a.warp_smem_floats;
  float* xr = base;
  float* cv = xr + dimp;
  float* rv = cv + dimp;
  float* ss = rv + (size_t)2 * kMaxM * a.rstride;
  uint32_t* sid = reinterpret_cast<uint32_t*>(ss + kListPad);
  Ent* so = reinterpret_cast<Ent*>(sid + kListPad);  // 8-byte aligned: every piece before is even
  const uint32_t nent = *a.tcount;
  const uint32_t warps = gridDim.x * (blockDim.x >> 5);
  for (uint32_t t = blockIdx.x * (blockDim.x >> 5) + wib; t < nent; t += warps) {
    const uint32_t key = a.tlist[t];
    const uint32_t L = key / n, r = key - L * n, cap = a.g.cap[L];
    uint32_t* list = a.g.ids[L] + (size_t)r * (cap + 1);
    uint32_t len = a.g.len[L][r];
    for (uint32_t d = lane; d < dim; d += 32) xr[d] = a.x[(size_t)r * dim + d];
    const uint32_t mw = lane < kMaskWords ? a.mask[(size_t)key * kMaskWords + lane] : 0u;
    __syncwarp();
    for (uint32_t w = 0; w < kMaskWords; ++w) {
      uint32_t bits = __shfl_sync(~0u, mw, w);
      while (bits) {
        const uint32_t b = __ffs(bits) - 1;
        bits &= bits - 1;
        if (lane == 0) list[len] = a.q_base + w * 32 + b;
        ++len;
        __syncwarp();
        if (len > cap) len = shrink_list(a, list, len, cap, xr, cv, rv, ss, sid, so);
      }
    }
    if (lane < kMaskWords) a.mask[(size_t)key * kMaskWords + lane] = 0u;
    if (lane == 0) {
      a.touched[key] = 0u;
      a.g.len[L][r] = len;
    }
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// freeze to CSR (hnsw.zig:427-462)
// ---------------------------------------------------------------------------

// offsets[i + 1] = offsets[i] + len[i]: one CTA, 1024 threads, sequential
// blocks of 1024 nodes.
__global__ void __launch_bounds__(1024) hnsw_offsets_kernel(const uint32_t* len, uint32_t n, uint32_t* offsets) {
  __shared__ uint32_t wsum[32];
  __shared__ uint32_t carry;
  const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    carry = 0;
    offsets[0] = 0;
  }
  __syncthreads();
  for (uint32_t base = 0; base < n; base += 1024) {
    const uint32_t i = base + tid;
    const uint32_t v = i < n ? len[i] : 0u;
    uint32_t s = v;
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(~0u, s, o);
      if (lane >= (uint32_t)o) s += y;
    }
    if (lane == 31) wsum[warp] = s;
    __syncthreads();
    if (warp == 0) {
      uint32_t w = wsum[lane];
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(~0u, w, o);
        if (lane >= (uint32_t)o) w += y;
      }
      wsum[lane] = w;
    }
    __syncthreads();
    const uint32_t incl = carry + (warp ? wsum[warp - 1] : 0u) + s;
    if (i < n) offsets[i + 1] = incl;
    __syncthreads();
    if (tid == 1023) carry = incl;
    __syncthreads();
  }
}

__global__ void hnsw_gather_kernel(const uint32_t* ids, const uint32_t* len, uint32_t n, uint32_t stride,
                                   const uint32_t* offsets, uint32_t* out) {
  const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const uint32_t node = (uint32_t)(t / stride), j = (uint32_t)(t % stride);
  if (node < n && j < len[node]) out[offsets[node] + j] = ids[(size_t)node * stride + j];
}

// vec.normalizeRowsInPlace: one warp per row
__global__ void normalize_rows_kernel(float* x, uint64_t n_rows, uint32_t dim) {
  const uint64_t row = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const uint32_t lane = threadIdx.x & 31;
  if (row >= n_rows) return;
  float* v = x + row * dim;
  float ns = 0.f;
  if (lane == 0) ns = dot_ref_scalar(v, v, dim);
  ns = __shfl_sync(~0u, ns, 0);
  if (ns == 0.0f) return;
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(ns));
  for (uint32_t d = lane; d < dim; d += 32) v[d] = __fmul_rn(v[d], inv);
}

// pickLevel (hnsw.zig:949-956)
uint8_t pick_level(Xoshiro256pp& r, float m_l) {
  const float u = 1.0f - r.unit_f32();
  const float lvl = std::floor(-std::log(u) * m_l);
  if (lvl < 0.0f) return 0;
  if (lvl > 31.0f) return 31;
  return (uint8_t)lvl;
}


}  // namespace

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

struct HnswGraphHost {
  uint32_t n = 0, dim = 0, entry_point = 0, max_level = 0;
  float device_ms = 0.f;
  uint64_t launches = 0;
  std::vector<uint8_t> levels;
  std::vector<std::vector<uint32_t>> offsets, nbrs;
};

int hnsw_build_device(Ctx* c, const float* d_x, uint64_t n_floats, uint32_t dim, uint64_t seed, uint32_t ef,
                      uint32_t m, uint32_t n_threads, HnswGraphHost* out) {
  if (dim == 0 || n_floats % dim) return fail(c, MVR_E_DIM_MISMATCH, "hnsw.build: centroids.len % dim != 0");
  const uint64_t n64 = n_floats / dim;
  if (n64 == 0) return fail(c, MVR_E_EMPTY_CORPUS, "hnsw.build: no centroids");
  if (n64 > (1ull << 27) || m == 0 || m > kMaxM || ef == 0 || ef > kMaxEf || dim > kMaxDim)
    return fail(c, MVR_E_INVALID_ARGUMENT, "hnsw.build: unsupported n, m, ef_construction or dim");
  if ((dim & 3u) == 0 && (reinterpret_cast<uintptr_t>(d_x) & 15u))
    return fail(c, MVR_E_INVALID_ARGUMENT, "hnsw.build: centroids must be 16-byte aligned");
  const uint32_t n = (uint32_t)n64;
  const uint32_t dimp = (dim + 3u) & ~3u;
  cudaStream_t st = c->stream;

  // the plan kernel's shared memory
  PlanLayout lay{};
  {
    uint32_t off = 0;
    auto take = [&](uint32_t bytes) {
      const uint32_t o = off;
      off = (off + bytes + 15u) & ~15u;
      return o;
    };
    lay.nwords = (n + 31) / 32;
    lay.rstride = dim + 1;
    lay.qv = take(dimp * 4);
    lay.w = take(ef * 8);
    lay.vis = take(lay.nwords * 4);
    lay.cn = take(64 * 4);
    lay.cs = take(64 * 4);
    lay.cacc = take(64 * 4);
    lay.as = take(64 * 8);
    lay.apos = take(64 * 4);
    lay.ev = take(64 * 8);
    lay.ties = take(kTieCap * 4);
    lay.rv = take(kMaxM * lay.rstride * 4);
    lay.rid = take(kMaxM * 4);
    lay.cv = take((kPlanThreads / 32) * lay.rstride * 4);  // one candidate row per warp
    // staged rows of the guessed next expansion: 16 KB per buffer, whole rows
    lay.stage_slots = (dim & 3u) == 0 ? std::min<uint32_t>(64, 16384 / (dim * 4)) : 0u;
    lay.stg = take(2 * lay.stage_slots * dim * 4);
    lay.bytes = off;
  }
  if (lay.bytes > kSmemLimit)
    return fail(c, MVR_E_INVALID_ARGUMENT, "hnsw.build: search state exceeds one CTA's shared memory");
  // the reverse-commit kernel's shared memory per warp
  const uint32_t rstride = dim + 1;
  const uint32_t warp_floats = 2 * dimp + 2 * kMaxM * rstride + 2 * kListPad + 2 * kMaxList;
  const uint32_t warp_bytes = ((warp_floats * 4 + 15u) & ~15u);
  uint32_t commit_warps = 4;
  while (commit_warps > 1 && (size_t)commit_warps * warp_bytes > kSmemLimit) --commit_warps;
  if ((size_t)warp_bytes > kSmemLimit) return fail(c, MVR_E_INVALID_ARGUMENT, "hnsw.build: dim too large");

  // levels, in the reference's draw order (levels[0] first, then node order)
  std::vector<uint8_t> levels(n);
  Xoshiro256pp rng(seed);
  const float m_l = 1.0f / std::log((float)m);
  uint32_t top_level = 0;
  for (uint32_t i = 0; i < n; ++i) {
    levels[i] = pick_level(rng, m_l);
    top_level = std::max<uint32_t>(top_level, levels[i]);
  }
  const uint32_t layers = top_level + 1;

  // one workspace for the whole build, carved from the context's grow-only
  // scratch (a repeated build allocates nothing)
  DevGraph g{};
  g.n = n;
  g.dim = dim;
  g.m = m;
  const size_t tl_cap = (size_t)kChunk * kMaxM * layers;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = (off + bytes + 255) & ~(size_t)255;
    return o;
  };
  size_t o_ids[kMaxLayers], o_len[kMaxLayers], o_off[kMaxLayers], o_nb[kMaxLayers];
  for (uint32_t L = 0; L < layers; ++L) {
    g.cap[L] = L == 0 ? 2 * m : m;
    o_ids[L] = take((size_t)n * (g.cap[L] + 1) * 4);
    o_len[L] = take((size_t)n * 4);
    o_off[L] = take(((size_t)n + 1) * 4);
    o_nb[L] = take((size_t)n * g.cap[L] * 4);  // lists hold at most cap entries at rest
  }
  const size_t o_levels = take(n), o_chosen = take((size_t)kChunk * kMaxLayers * kMaxM * 4),
               o_nchosen = take((size_t)kChunk * kMaxLayers * 4), o_mask = take((size_t)layers * n * kMaskWords * 4),
               o_touched = take((size_t)layers * n * 4), o_tlist = take(tl_cap * 4), o_small = take(64);
  unsigned char* ws = nullptr;
  MVR_TRY(scratch(c, kSlotAux3, off, (void**)&ws));
  std::vector<uint32_t*> d_off(layers), d_nb(layers);
  for (uint32_t L = 0; L < layers; ++L) {
    g.ids[L] = reinterpret_cast<uint32_t*>(ws + o_ids[L]);
    g.len[L] = reinterpret_cast<uint32_t*>(ws + o_len[L]);
    d_off[L] = reinterpret_cast<uint32_t*>(ws + o_off[L]);
    d_nb[L] = reinterpret_cast<uint32_t*>(ws + o_nb[L]);
    MVR_CUDA(c, cudaMemsetAsync(g.len[L], 0, (size_t)n * 4, st));
  }
  uint8_t* d_levels = ws + o_levels;
  uint32_t* d_chosen = reinterpret_cast<uint32_t*>(ws + o_chosen);
  uint32_t* d_nchosen = reinterpret_cast<uint32_t*>(ws + o_nchosen);
  uint32_t* d_mask = reinterpret_cast<uint32_t*>(ws + o_mask);
  uint32_t* d_touched = reinterpret_cast<uint32_t*>(ws + o_touched);
  uint32_t* d_tlist = reinterpret_cast<uint32_t*>(ws + o_tlist);
  uint32_t* d_small = reinterpret_cast<uint32_t*>(ws + o_small);  // [0] tcount, [1] status
  MVR_CUDA(c, cudaMemsetAsync(d_mask, 0, (size_t)layers * n * kMaskWords * 4, st));
  MVR_CUDA(c, cudaMemsetAsync(d_touched, 0, (size_t)layers * n * 4, st));
  MVR_CUDA(c, cudaMemsetAsync(d_small, 0, 64, st));
  MVR_CUDA(c, cudaMemcpyAsync(d_levels, levels.data(), n, cudaMemcpyHostToDevice, st));
  MVR_CUDA(c, cudaFuncSetAttribute(hnsw_plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)lay.bytes));
  {  // shared memory for two CTAs per SM; the rest of the unified L1 stays cache
    const int pct = (int)std::min<size_t>(100, (2 * (lay.bytes + 1024) * 100 + 228 * 1024 - 1) / (228 * 1024));
    MVR_CUDA(c, cudaFuncSetAttribute(hnsw_plan_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, pct));
  }
  MVR_CUDA(c, cudaFuncSetAttribute(hnsw_commit_reverse, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)(commit_warps * warp_bytes)));

  cudaEvent_t e0 = nullptr, e1 = nullptr;
  MVR_CUDA(c, cudaEventCreate(&e0));
  MVR_CUDA(c, cudaEventCreate(&e1));
  struct EvGuard {
    cudaEvent_t a, b;
    ~EvGuard() {
      cudaEventDestroy(a);
      cudaEventDestroy(b);
    }
  } evg{e0, e1};
  MVR_CUDA(c, cudaEventRecord(e0, st));

  uint64_t launches = 0;
  uint32_t entry = 0, max_level = levels[0];
  const uint32_t commit_grid = (uint32_t)std::max(1, c->sm_count) * 4;
  for (uint32_t q_base = 1; q_base < n;) {
    const uint32_t csz = n_threads <= 1 ? 1u : std::min(kChunk, q_base);
    const uint32_t q_end = (uint32_t)std::min<uint64_t>((uint64_t)q_base + csz, n);
    const uint32_t len = q_end - q_base;
    PlanArgs pa{};
    pa.g = g;
    pa.lay = lay;
    pa.x = d_x;
    pa.levels = d_levels;
    pa.q_base = q_base;
    pa.snap_entry = entry;
    pa.snap_max = max_level;
    pa.ef = ef;
    pa.chosen = d_chosen;
    pa.n_chosen = d_nchosen;
    pa.status = d_small + 1;
    hnsw_plan_kernel<<<len, kPlanThreads, lay.bytes, st>>>(pa);
    CommitArgs ca{};
    ca.g = g;
    ca.x = d_x;
    ca.levels = d_levels;
    ca.q_base = q_base;
    ca.chunk_len = len;
    ca.snap_max = max_level;
    ca.chosen = d_chosen;
    ca.n_chosen = d_nchosen;
    ca.mask = d_mask;
    ca.touched = d_touched;
    ca.tlist = d_tlist;
    ca.tcount = d_small;
    ca.warp_smem_floats = warp_bytes / 4;
    ca.rstride = rstride;
    MVR_CUDA(c, cudaMemsetAsync(d_small, 0, 4, st));
    hnsw_commit_own<<<len, 32, 0, st>>>(ca);
    hnsw_commit_reverse<<<commit_grid, commit_warps * 32, commit_warps * warp_bytes, st>>>(ca);
    launches += 3;
    MVR_CUDA(c, cudaGetLastError());
    for (uint32_t i = q_base; i < q_end; ++i)
      if (levels[i] > max_level) {
        max_level = levels[i];
        entry = i;
      }
    q_base = q_end;
  }

  // freeze
  for (uint32_t L = 0; L < layers && L <= max_level; ++L) {
    hnsw_offsets_kernel<<<1, 1024, 0, st>>>(g.len[L], n, d_off[L]);
    ++launches;
  }
  MVR_CUDA(c, cudaGetLastError());
  std::vector<uint32_t> totals(layers, 0);
  for (uint32_t L = 0; L <= max_level; ++L)
    MVR_CUDA(c, cudaMemcpyAsync(&totals[L], d_off[L] + n, 4, cudaMemcpyDeviceToHost, st));
  uint32_t hstatus = 0;
  MVR_CUDA(c, cudaMemcpyAsync(&hstatus, d_small + 1, 4, cudaMemcpyDeviceToHost, st));
  MVR_CUDA(c, cudaStreamSynchronize(st));
  for (uint32_t L = 0; L <= max_level; ++L) {
    const uint32_t stride = g.cap[L] + 1;
    const uint64_t threads = (uint64_t)n * stride;
    hnsw_gather_kernel<<<(uint32_t)((threads + 255) / 256), 256, 0, st>>>(g.ids[L], g.len[L], n, stride, d_off[L],
                                                                         d_nb[L]);
    ++launches;
  }
  MVR_CUDA(c, cudaGetLastError());
  MVR_CUDA(c, cudaEventRecord(e1, st));
  if (hstatus & kErrTies) return fail(c, MVR_E_DEVICE_LIMIT, "hnsw.build: more than 512 exact ties at the beam minimum");
  if (hstatus & kErrLoop) return fail(c, MVR_E_DEVICE_LIMIT, "hnsw.build: search did not terminate");

  out->n = n;
  out->dim = dim;
  out->entry_point = entry;
  out->max_level = max_level;
  out->levels = std::move(levels);
  out->offsets.assign(max_level + 1, {});
  out->nbrs.assign(max_level + 1, {});
  for (uint32_t L = 0; L <= max_level; ++L) {
    out->offsets[L].resize((size_t)n + 1);
    out->nbrs[L].resize(std::max<uint32_t>(totals[L], 1));
    MVR_TRY(d2h_staged(c, out->offsets[L].data(), d_off[L], ((size_t)n + 1) * 4));
    MVR_TRY(d2h_staged(c, out->nbrs[L].data(), d_nb[L], (size_t)totals[L] * 4));
    out->nbrs[L].resize(totals[L]);
  }
  MVR_CUDA(c, cudaEventSynchronize(e1));
  MVR_CUDA(c, cudaEventElapsedTime(&out->device_ms, e0, e1));
  out->launches = launches;
  return MVR_OK;
}

int normalize_rows_device(Ctx* c, float* d, uint64_t n_floats, uint32_t dim) {
  if (dim == 0) return fail(c, MVR_E_EMPTY_INPUT, "normalizeRowsInPlace: dim 0");
  if (n_floats % dim) return fail(c, MVR_E_LENGTH_MISMATCH, "normalizeRowsInPlace: len % dim != 0");
  const uint64_t rows = n_floats / dim;
  if (rows == 0) return MVR_OK;
  const uint64_t threads = rows * 32;
  normalize_rows_kernel<<<(uint32_t)((threads + 255) / 256), 256, 0, c->stream>>>(d, rows, dim);
  MVR_CUDA(c, cudaGetLastError());
  return MVR_OK;
}

}  // namespace mvr

struct mvr_hnsw {
  mvr::HnswGraphHost g;
};

extern "C" {

int mvr_hnsw_build_device(mvr_ctx* ctx, const float* d_centroids, uint64_t n_floats, uint32_t dim, uint64_t seed,
                          uint32_t ef_construction, uint32_t m, uint32_t n_threads, mvr_hnsw** out) {
  if (!ctx || !out || (!d_centroids && n_floats)) return MVR_E_INVALID_ARGUMENT;
  *out = nullptr;
  mvr::Ctx* c = &ctx->impl;
  mvr::DeviceScope dev_scope(c);
  MVR_TRY(dev_scope.status);
  mvr_hnsw* h = new (std::nothrow) mvr_hnsw;
  if (!h) return mvr::fail(c, MVR_E_OUT_OF_MEMORY, "hnsw.build: host allocation");
  const int s = mvr::hnsw_build_device(c, d_centroids, n_floats, dim, seed, ef_construction, m, n_threads, &h->g);
  if (s != MVR_OK) {
    delete h;
    return s;
  }
  *out = h;
  return MVR_OK;
}

int mvr_hnsw_build(mvr_ctx* ctx, const float* centroids, uint64_t n_floats, uint32_t dim, uint64_t seed,
                   uint32_t ef_construction, uint32_t m, uint32_t n_threads, mvr_hnsw** out) {
  if (!ctx || !out || (!centroids && n_floats)) return MVR_E_INVALID_ARGUMENT;
  *out = nullptr;
  mvr::Ctx* c = &ctx->impl;
  mvr::DeviceScope dev_scope(c);
  MVR_TRY(dev_scope.status);
  if (dim == 0 || n_floats % dim) return mvr::fail(c, MVR_E_DIM_MISMATCH, "hnsw.build: centroids.len % dim != 0");
  if (n_floats == 0) return mvr::fail(c, MVR_E_EMPTY_CORPUS, "hnsw.build: no centroids");
  float* d = nullptr;  // staged in the context's scratch (the build's workspace uses another slot)
  MVR_TRY(mvr::scratch(c, mvr::kSlotAux2, n_floats * 4, (void**)&d));
  MVR_TRY(mvr::h2d_staged(c, d, centroids, n_floats * 4));
  return mvr_hnsw_build_device(ctx, d, n_floats, dim, seed, ef_construction, m, n_threads, out);
}

void mvr_hnsw_info(const mvr_hnsw* h, uint32_t* n, uint32_t* entry_point, uint32_t* max_level, float* device_ms,
                   uint64_t* kernel_launches) {
  if (!h) return;
  if (n) *n = h->g.n;
  if (entry_point) *entry_point = h->g.entry_point;
  if (max_level) *max_level = h->g.max_level;
  if (device_ms) *device_ms = h->g.device_ms;
  if (kernel_launches) *kernel_launches = h->g.launches;
}

const uint8_t* mvr_hnsw_node_levels(const mvr_hnsw* h) { return h ? h->g.levels.data() : nullptr; }

const uint32_t* mvr_hnsw_layer_offsets(const mvr_hnsw* h, uint32_t layer) {
  if (!h || layer > h->g.max_level) return nullptr;
  return h->g.offsets[layer].data();
}

const uint32_t* mvr_hnsw_layer_neighbours(const mvr_hnsw* h, uint32_t layer, uint64_t* count) {
  if (!h || layer > h->g.max_level) {
    if (count) *count = 0;
    return nullptr;
  }
  if (count) *count = h->g.nbrs[layer].size();
  return h->g.nbrs[layer].data();
}

void mvr_hnsw_free(mvr_hnsw* h) { delete h; }

int mvr_normalize_rows_device(mvr_ctx* ctx, float* d_rows, uint64_t n_floats, uint32_t dim) {
  if (!ctx || (!d_rows && n_floats)) return MVR_E_INVALID_ARGUMENT;
  mvr::DeviceScope dev_scope(&ctx->impl);
  MVR_TRY(dev_scope.status);
  return mvr::normalize_rows_device(&ctx->impl, d_rows, n_floats, dim);
}

int mvr_normalize_rows(mvr_ctx* ctx, float* rows, uint64_t n_floats, uint32_t dim) {
  if (!ctx || (!rows && n_floats)) return MVR_E_INVALID_ARGUMENT;
  mvr::Ctx* c = &ctx->impl;
  mvr::DeviceScope dev_scope(c);
  MVR_TRY(dev_scope.status);
  if (dim == 0) return mvr::fail(c, MVR_E_EMPTY_INPUT, "normalizeRowsInPlace: dim 0");
  if (n_floats % dim) return mvr::fail(c, MVR_E_LENGTH_MISMATCH, "normalizeRowsInPlace: len % dim != 0");
  if (n_floats == 0) return MVR_OK;
  float* d = nullptr;
  MVR_TRY(mvr::scratch(c, mvr::kSlotAux2, n_floats * 4, (void**)&d));
  MVR_TRY(mvr::h2d_staged(c, d, rows, n_floats * 4));
  MVR_TRY(mvr::normalize_rows_device(c, d, n_floats, dim));
  MVR_TRY(mvr::d2h_staged(c, rows, d, n_floats * 4));
  MVR_CUDA(c, cudaStreamSynchronize(c->stream));
  return MVR_OK;
}

}  // extern "C"
