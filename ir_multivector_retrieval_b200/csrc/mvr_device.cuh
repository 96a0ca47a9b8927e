// mvr_device.cuh — device helpers: the reference's exact f32 arithmetic and
// directed-rounding reductions.
//
// Exactness contract. The reference computes squared L2 distances in Zig's
// strict float mode (no FMA contraction, IEEE round-to-nearest, denormals
// kept). Every distance here uses __fadd_rn/__fmul_rn (or their sm_100
// packed-pair forms, arranged so that no product feeds an add; see
// l2_small_pair) in the reference's summation order, so results are
// bit-identical. The library is built with -fmad=false and without
// --use_fast_math as a second guard.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

namespace mvr {

__device__ __forceinline__ float f32_nan() { return __int_as_float(0x7fc00000); }

// vec.l2sq order for sub-vector lengths 1, 2, 4 (src/util/vec.zig:109-139):
// s = d0^2; s += d1^2; ... (the length-1 generic path reduces a zero vector
// and adds the single tail term, which is d0^2 as well).
template <int S>
__device__ __forceinline__ float l2_small(const float* x, const float* c) {
  float d = __fsub_rn(x[0], c[0]);
  float acc = __fmul_rn(d, d);
#pragma unroll
  for (int k = 1; k < S; ++k) {
    d = __fsub_rn(x[k], c[k]);
    acc = __fadd_rn(acc, __fmul_rn(d, d));
  }
  return acc;
}

// Two distances at once: xx[k] = (x_k, x_k), nc[k] = (-ca_k, -cb_k).
// x + (-c) is IEEE-identical to x - c, so lane 0 is l2_small(x, ca) and
// lane 1 is l2_small(x, cb), bit for bit.
//
// The accumulation is written as fma(q, one, acc) with q = d*d already
// rounded and `one` == 1.0f supplied at run time (a kernel argument):
// fma(q, 1, acc) = round(acc + q), exactly the reference's add. Written as
// a packed add of a packed product instead, the assembler contracts the
// pair into one fused multiply-add (measured on sm_100a, even with
// -fmad=false and explicit .rn), which rounds d*d away and breaks parity.
// With `one` opaque there is no multiply feeding an add left to contract.
template <int S>
__device__ __forceinline__ float2 l2_small_pair(const float2 (&xx)[S],
                                                const float2* nc, float2 one) {
  float2 d = __fadd2_rn(xx[0], nc[0]);
  float2 acc = __fmul2_rn(d, d);
#pragma unroll
  for (int k = 1; k < S; ++k) {
    d = __fadd2_rn(xx[k], nc[k]);
    const float2 q = __fmul2_rn(d, d);
    acc = __ffma2_rn(q, one, acc);
  }
  return acc;
}

// vec.l2sq for len 64/128 (vec.zig:142-155): four strided lane
// accumulators acc[l] += d[4q+l]^2, then @reduce(.Add) as the ordered
// reduction ((a0+a1)+a2)+a3.
template <int D>
__device__ __forceinline__ float l2_wide(const float* x, const float* c) {
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
  for (int q = 0; q < D; q += 4) {
    float d0 = __fsub_rn(x[q + 0], c[q + 0]);
    float d1 = __fsub_rn(x[q + 1], c[q + 1]);
    float d2 = __fsub_rn(x[q + 2], c[q + 2]);
    float d3 = __fsub_rn(x[q + 3], c[q + 3]);
    a0 = __fadd_rn(a0, __fmul_rn(d0, d0));
    a1 = __fadd_rn(a1, __fmul_rn(d1, d1));
    a2 = __fadd_rn(a2, __fmul_rn(d2, d2));
    a3 = __fadd_rn(a3, __fmul_rn(d3, d3));
  }
  return __fadd_rn(__fadd_rn(__fadd_rn(a0, a1), a2), a3);
}

// Warp sums of non-negative doubles rounded down / up: rigorous lower and
// upper bounds of the exact sum whatever the association order.
__device__ __forceinline__ double warp_sum_rd(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __dadd_rd(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ double warp_sum_ru(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __dadd_ru(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Inclusive warp scans with directed rounding.
__device__ __forceinline__ double warp_scan_rd(double v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v = __dadd_rd(v, t);
  }
  return v;
}
__device__ __forceinline__ double warp_scan_ru(double v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v = __dadd_ru(v, t);
  }
  return v;
}

__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// 16-, 8- or 4-byte asynchronous global->shared copy (LDGSTS).
template <int BYTES>
__device__ __forceinline__ void cp_async(void* smem, const void* gmem) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  if constexpr (BYTES == 16) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
  } else {
    asm volatile("cp.async.ca.shared.global [%0], [%1], %2;\n" ::"r"(s), "l"(gmem), "n"(BYTES));
  }
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }


// Programmatic dependent launch: a kernel launched with the
// programmatic-stream-serialization attribute may be scheduled before the
// previous kernel in the stream finishes; this waits (in hardware) until that
// kernel has completed and its writes are visible. The previous kernels never
// trigger early, so nothing overlaps but the launch itself. A no-op for a
// normal launch.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Launch with programmatic stream serialization (the kernel must start with
// grid_dependency_wait()).
template <class... KArgs, class... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

}  // namespace mvr
