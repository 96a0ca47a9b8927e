// probe.cu — measured FP32 issue rate of this GPU, the denominator of the
// FP32 rooflines the benchmark reports (the driver's peak file carries HBM
// and tensor figures only). No reference counterpart.
//
// Independent chains of packed f32x2 adds and multiplies (the instructions
// the exact distance kernels issue), 8 per thread, enough warps to fill
// every sub-partition: lane operations per second.
#include <cuda_runtime.h>

#include <cstdint>

#include "mvr_internal.h"

namespace {

__global__ void __launch_bounds__(256) f32x2_rate_kernel(float* __restrict__ out, int iters, float a) {
  float2 x[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) x[q] = make_float2((float)threadIdx.x + q, (float)threadIdx.x - q);
  const float2 aa = make_float2(a, a);
  for (int i = 0; i < iters; ++i) {
#pragma unroll
    for (int u = 0; u < 8; ++u) {
#pragma unroll
      for (int q = 0; q < 8; ++q) x[q] = __fadd2_rn(x[q], aa);
#pragma unroll
      for (int q = 0; q < 8; ++q) x[q] = __fmul2_rn(x[q], aa);
    }
  }
  float s = 0.f;
#pragma unroll
  for (int q = 0; q < 8; ++q) s += x[q].x + x[q].y;
  out[(size_t)blockIdx.x * blockDim.x + threadIdx.x] = s;  // keeps the chains alive
}

}  // namespace

extern "C" int mvr_measure_f32x2_rate(mvr_ctx* h, double* lane_ops_per_s) {
  if (!h || !lane_ops_per_s) return MVR_E_INVALID_ARGUMENT;
  mvr::Ctx* c = &h->impl;
  mvr::DeviceScope dev_scope(c);
  MVR_TRY(dev_scope.status);
  MVR_CUDA(c, cudaSetDevice(c->device));
  const int blocks = c->sm_count * 8, threads = 256, iters = 4000;
  float* out = nullptr;
  MVR_TRY(mvr::scratch(c, mvr::kSlotAux3, (size_t)blocks * threads * sizeof(float), (void**)&out));
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  MVR_CUDA(c, cudaEventCreate(&e0));
  const cudaError_t ce = cudaEventCreate(&e1);
  if (ce != cudaSuccess) {
    cudaEventDestroy(e0);
    return mvr::cuda_fail(c, ce, "cudaEventCreate");
  }
  float best = 0.f;
  cudaError_t err = cudaSuccess;
  for (int rep = 0; rep < 3 && err == cudaSuccess; ++rep) {  // the first launch warms up
    cudaEventRecord(e0, c->stream);
    f32x2_rate_kernel<<<blocks, threads, 0, c->stream>>>(out, iters, 0.999f);
    cudaEventRecord(e1, c->stream);
    err = cudaEventSynchronize(e1);
    float ms = 0.f;
    if (err == cudaSuccess) err = cudaEventElapsedTime(&ms, e0, e1);
    if (err == cudaSuccess && rep > 0 && (best == 0.f || ms < best)) best = ms;
  }
  if (err == cudaSuccess) err = cudaGetLastError();
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (err != cudaSuccess) return mvr::cuda_fail(c, err, "f32x2 rate probe");
  // lane operations: blocks x threads x iters x 8 x 16 instructions x 2 lanes
  const double ops = (double)blocks * threads * iters * 8.0 * 16.0 * 2.0;
  *lane_ops_per_s = ops / (best * 1e-3);
  return MVR_OK;
}
