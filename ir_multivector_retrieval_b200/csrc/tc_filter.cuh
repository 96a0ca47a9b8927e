// tc_filter.cuh — 5th-generation tensor-core (tcgen05) building blocks for
// the distance filters of the assignment kernels.
//
// The filters compute, per (row, centroid), an approximation of
//     a(c) = t + |c|^2 - 2 x.c          (t >= |x|^2: a(c) ~ |x - c|^2 + t - |x|^2)
// with one kind::tf32 MMA chain per 128-row tile (M = 128, N = 256, the
// accumulator in tensor memory, one TMEM lane per row). Each f32 operand is
// split into hi = its 13 low mantissa bits cleared (exact in TF32) and
// lo = v - hi (exact in f32); the chain hi*hi + hi*lo + lo*hi misses only
// lo*lo and the TF32 truncation of the lo parts (each below 2^-20 of the
// product), so the accumulator is within a small, bounded distance of the
// exact value. The kernels then compute the reference's exact f32 distance
// only for the centroids whose approximation is within that bound of the
// smallest one, so the selected centroid is the reference's.
//
// Shared-memory operand layout (K-major, no swizzle, the canonical UMMA
// "interleave" form): one MMA covers K = 8 TF32 values = two 16-byte core
// columns. Row r, core column j (j = 0: values 0..3, j = 1: values 4..7)
// sits at byte (r / 8) * 256 + j * 128 + (r % 8) * 16, i.e. leading-byte
// offset 128 (between the two core columns) and stride-byte offset 256
// (between groups of 8 rows).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

namespace mvr {
namespace tc {

constexpr uint32_t kRowsPerTile = 128;   // MMA M: one TMEM lane per row
constexpr uint32_t kCols = 256;          // MMA N: one TMEM column per centroid
constexpr uint32_t kTileBytesA = kRowsPerTile * 32;  // 128 rows x 8 TF32
constexpr uint32_t kTileBytesB = kCols * 32;         // 256 centroids x 8 TF32
constexpr uint32_t kWaitLimit = 1u << 26;            // bounded mbarrier polls

// kind::tf32 instruction descriptor: D f32 (bits 4-5 = 1), A and B TF32
// (bits 7-9 and 10-12 = 2), both K-major (bits 15, 16 = 0), N >> 3 at bits
// 17-22, M >> 4 at bits 24-28.
constexpr uint32_t kIdescTf32 =
    (1u << 4) | (2u << 7) | (2u << 10) | ((kCols >> 3) << 17) | ((kRowsPerTile >> 4) << 24);

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Byte offset of (row r, TF32 value k in [0, 8)) in a K-major tile.
__host__ __device__ __forceinline__ uint32_t operand_offset(uint32_t r, uint32_t k) {
  return (r >> 3) * 256u + (k >> 2) * 128u + (r & 7u) * 16u + (k & 3u) * 4u;
}

// Shared-memory matrix descriptor: start address >> 4 (bits 0-13),
// leading-byte offset >> 4 (16-29), stride-byte offset >> 4 (32-45),
// descriptor version 1 (bits 46-47), base offset 0, no swizzle.
__device__ __forceinline__ uint64_t operand_desc(const void* tile) {
  const uint32_t a = smem_addr(tile);
  return (uint64_t)((a & 0x3FFFFu) >> 4) | ((uint64_t)(128u >> 4) << 16) | ((uint64_t)(256u >> 4) << 32) |
         ((uint64_t)1 << 46);
}

// f32 -> (hi, lo): hi has the 13 low mantissa bits cleared (exact in TF32),
// lo = v - hi exactly.
__device__ __forceinline__ void split_tf32(float v, float& hi, float& lo) {
  hi = __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
  lo = __fsub_rn(v, hi);
}

// Smallest TF32-representable value >= v, for v > 0 finite.
__device__ __forceinline__ float tf32_ceil_pos(float v) {
  uint32_t b = __float_as_uint(v);
  if (b & 0x1FFFu) b = (b + 0x2000u) & 0xFFFFE000u;
  return __uint_as_float(b);
}

// Three-input f32 minimum (sm_100).
__device__ __forceinline__ float min3f(float a, float b, float c) {
  float d;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// generic-proxy shared-memory writes become visible to the tensor core
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Whole warp: allocate `cols` TMEM columns, base address to *slot.
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)), "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_free(uint32_t base, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(cols) : "memory");
}

// The same with N = 128.
constexpr uint32_t kIdescTf32N128 =
    (1u << 4) | (2u << 7) | (2u << 10) | ((128u >> 3) << 17) | ((kRowsPerTile >> 4) << 24);

// One thread: D[tmem] (+)= A * B^T, M = 128, K = 8, N = 256 (or 128 with
// idesc = kIdescTf32N128).
__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate,
                                         uint32_t idesc = kIdescTf32) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned)
// from global memory into shared memory, completing on *bar (which expects
// the bytes through this same call's arrive).
__device__ __forceinline__ void bulk_load(void* smem, const void* gmem, uint32_t bytes, uint64_t* bar) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
          smem_addr(smem)),
      "l"(gmem), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}
// One thread: arrive on *bar once every MMA issued so far has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
// Bounded wait for the phase with the given parity; false on expiry (about
// two seconds of SM clock, or kWaitLimit polls, whichever comes first).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_addr(bar);
  const long long t0 = clock64();
  for (uint32_t it = 0; it < kWaitLimit; ++it) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
    if (clock64() - t0 > (1ll << 32)) return false;
  }
  return false;
}

// One arrival on *bar (count-based phase completion).
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Whole warp: 64 consecutive 32-bit TMEM columns of the warp's 32 lanes
// (lane = row), into v[0..63]; tmem_wait_ld() before reading v.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, uint32_t (&v)[64]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,"
      "%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];\n"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31]), "=r"(v[32]),
        "=r"(v[33]), "=r"(v[34]), "=r"(v[35]), "=r"(v[36]), "=r"(v[37]), "=r"(v[38]), "=r"(v[39]), "=r"(v[40]),
        "=r"(v[41]), "=r"(v[42]), "=r"(v[43]), "=r"(v[44]), "=r"(v[45]), "=r"(v[46]), "=r"(v[47]), "=r"(v[48]),
        "=r"(v[49]), "=r"(v[50]), "=r"(v[51]), "=r"(v[52]), "=r"(v[53]), "=r"(v[54]), "=r"(v[55]), "=r"(v[56]),
        "=r"(v[57]), "=r"(v[58]), "=r"(v[59]), "=r"(v[60]), "=r"(v[61]), "=r"(v[62]), "=r"(v[63])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

}  // namespace tc
}  // namespace mvr
