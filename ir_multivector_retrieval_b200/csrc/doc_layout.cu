// doc_layout.cu — the .tac per-doc section (storage.writeDocLayouts,
// src/index/storage.zig:705-749) built on the GPU, and the footer CRC-32.
//
// Section = doc index ((n_docs + 1) u64 offsets into the payload, relative
// to the byte after the index) + per doc d:
//   [n_d u32 | assignments[tok_lo .. tok_lo + n_d) u32 |
//    codes[tok_lo * M .. (tok_lo + n_d) * M) bytes | zero pad to 8 bytes].
// Every doc starts 8-byte aligned, so the count, the assignment block and
// (for M % 4 == 0) the code block are written as whole u32 words; one warp
// per doc streams its words. The doc offsets are host data (they come with
// the token dump), so the payload offsets are an O(n_docs) host prefix sum.
#include <cuda_runtime.h>

#include <cstring>
#include <vector>

#include "../../include/mvr.h"
#include "mvr_internal.h"

namespace mvr {
namespace {

__host__ __device__ inline uint64_t align8(uint64_t v) { return (v + 7) & ~(uint64_t)7; }

int payload_offsets(const uint64_t* doc_offsets, uint64_t n_docs, uint32_t M, std::vector<uint64_t>* pay) {
  pay->resize(n_docs + 1);
  uint64_t at = 0;
  for (uint64_t d = 0; d < n_docs; ++d) {
    if (doc_offsets[d + 1] < doc_offsets[d]) return MVR_E_INVALID_ARGUMENT;
    (*pay)[d] = at;
    const uint64_t n_d = doc_offsets[d + 1] - doc_offsets[d];
    at += align8(4 + n_d * 4 + n_d * (uint64_t)M);
  }
  (*pay)[n_docs] = at;
  return MVR_OK;
}

// One warp per doc. `pay` = payload offsets (n_docs + 1, device), `out` =
// section start (index first).
__global__ void __launch_bounds__(256)
doc_layout_kernel(const uint64_t* __restrict__ doc_off, const uint64_t* __restrict__ pay, uint64_t n_docs,
                  const uint32_t* __restrict__ asg, const uint8_t* __restrict__ codes, uint32_t M,
                  int words, uint8_t* __restrict__ out) {
  const uint64_t w = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const uint64_t stride = ((uint64_t)gridDim.x * blockDim.x) >> 5;
  const uint64_t idx_bytes = (n_docs + 1) * 8;
  for (uint64_t d = w; d <= n_docs; d += stride) {
    if (lane == 0) reinterpret_cast<uint64_t*>(out)[d] = pay[d];  // doc index
    if (d == n_docs) continue;
    const uint64_t tok_lo = doc_off[d], n_d = doc_off[d + 1] - tok_lo;
    uint8_t* doc = out + idx_bytes + pay[d];  // 8-byte aligned
    uint32_t* w32 = reinterpret_cast<uint32_t*>(doc);
    if (lane == 0) w32[0] = (uint32_t)n_d;
    for (uint64_t i = lane; i < n_d; i += 32) w32[1 + i] = asg[tok_lo + i];
    uint8_t* cdst = doc + 4 + 4 * n_d;
    const uint8_t* csrc = codes + tok_lo * (uint64_t)M;
    const uint64_t nc = n_d * (uint64_t)M;
    if (words) {  // M % 4 == 0 and a 4-byte aligned source: both ends aligned
      const uint32_t* s32 = reinterpret_cast<const uint32_t*>(csrc);
      uint32_t* d32 = reinterpret_cast<uint32_t*>(cdst);
      for (uint64_t i = lane; i < nc / 4; i += 32) d32[i] = s32[i];
    } else {
      for (uint64_t i = lane; i < nc; i += 32) cdst[i] = csrc[i];
    }
    const uint64_t used = 4 + 4 * n_d + nc, total = align8(used);
    if ((uint64_t)lane < total - used) doc[used + lane] = 0;
  }
}

int check_args(Ctx* c, const uint64_t* doc_offsets, uint64_t n_docs, uint64_t n_tokens, uint32_t pq_m,
               std::vector<uint64_t>* pay, uint64_t out_len) {
  if (!doc_offsets || pq_m == 0) return fail(c, MVR_E_INVALID_ARGUMENT, "null doc offsets or pq_m == 0");
  if (doc_offsets[0] != 0 || doc_offsets[n_docs] != n_tokens)
    return fail(c, MVR_E_INVALID_ARGUMENT, "doc offsets must run from 0 to n_tokens");
  if (payload_offsets(doc_offsets, n_docs, pq_m, pay) != MVR_OK)
    return fail(c, MVR_E_INVALID_ARGUMENT, "doc offsets must be non-decreasing");
  const uint64_t need = (n_docs + 1) * 8 + (*pay)[n_docs];
  if (out_len < need) return fail(c, MVR_E_BUFFER_TOO_SMALL, "output shorter than the doc section");
  return MVR_OK;
}

int launch(Ctx* c, const uint64_t* doc_offsets, uint64_t n_docs, const std::vector<uint64_t>& pay,
           const uint32_t* d_asg, const uint8_t* d_codes, uint32_t pq_m, uint8_t* d_out) {
  uint64_t* d_meta = nullptr;
  MVR_TRY(scratch(c, kSlotAux2, (n_docs + 1) * 16, (void**)&d_meta));
  MVR_CUDA(c, cudaMemcpyAsync(d_meta, doc_offsets, (n_docs + 1) * 8, cudaMemcpyHostToDevice, c->stream));
  MVR_CUDA(c, cudaMemcpyAsync(d_meta + n_docs + 1, pay.data(), (n_docs + 1) * 8, cudaMemcpyHostToDevice,
                              c->stream));
  const uint64_t warps = n_docs + 1;
  const unsigned grid = (unsigned)std::min<uint64_t>((warps * 32 + 255) / 256, (uint64_t)c->sm_count * 16);
  const int words = (pq_m % 4 == 0) && (reinterpret_cast<uintptr_t>(d_codes) % 4 == 0);
  doc_layout_kernel<<<grid, 256, 0, c->stream>>>(d_meta, d_meta + n_docs + 1, n_docs, d_asg, d_codes, pq_m, words,
                                                 d_out);
  MVR_CUDA(c, cudaGetLastError());
  return MVR_OK;
}

// CRC-32 (reflected 0xEDB88320), slicing by 8.
struct Crc32Tables {
  uint32_t t[8][256];
  Crc32Tables() {
    for (uint32_t i = 0; i < 256; ++i) {
      uint32_t c = i;
      for (int k = 0; k < 8; ++k) c = (c & 1) ? 0xEDB88320u ^ (c >> 1) : c >> 1;
      t[0][i] = c;
    }
    for (uint32_t i = 0; i < 256; ++i)
      for (int s = 1; s < 8; ++s) t[s][i] = (t[s - 1][i] >> 8) ^ t[0][t[s - 1][i] & 0xff];
  }
};
const Crc32Tables& crc_tables() {
  static const Crc32Tables T;
  return T;
}

}  // namespace
}  // namespace mvr

using mvr::Ctx;

extern "C" {

int mvr_doc_layouts_bytes(const uint64_t* doc_offsets, uint64_t n_docs, uint32_t pq_m, uint64_t* bytes_out) {
  if (!doc_offsets || !bytes_out || pq_m == 0) return MVR_E_INVALID_ARGUMENT;
  std::vector<uint64_t> pay;
  if (mvr::payload_offsets(doc_offsets, n_docs, pq_m, &pay) != MVR_OK) return MVR_E_INVALID_ARGUMENT;
  *bytes_out = (n_docs + 1) * 8 + pay[n_docs];
  return MVR_OK;
}

int mvr_write_doc_layouts_device(mvr_ctx* h, const uint64_t* doc_offsets, uint64_t n_docs,
                                 const uint32_t* d_assignments, const uint8_t* d_codes, uint64_t n_tokens,
                                 uint32_t pq_m, uint8_t* d_out, uint64_t out_len) {
  if (!h) return MVR_E_INVALID_ARGUMENT;
  Ctx* c = &h->impl;
  mvr::DeviceScope dev_scope(c);
  MVR_TRY(dev_scope.status);
  std::vector<uint64_t> pay;
  MVR_TRY(mvr::check_args(c, doc_offsets, n_docs, n_tokens, pq_m, &pay, out_len));
  if (!d_out || (n_tokens && (!d_assignments || !d_codes))) return mvr::fail(c, MVR_E_INVALID_ARGUMENT, "null pointer");
  if (reinterpret_cast<uintptr_t>(d_out) % 8 || reinterpret_cast<uintptr_t>(d_assignments) % 4)
    return mvr::fail(c, MVR_E_INVALID_ARGUMENT, "out must be 8-byte and assignments 4-byte aligned");
  MVR_CUDA(c, cudaSetDevice(c->device));
  return mvr::launch(c, doc_offsets, n_docs, pay, d_assignments, d_codes, pq_m, d_out);
}

int mvr_write_doc_layouts(mvr_ctx* h, const uint64_t* doc_offsets, uint64_t n_docs, const uint32_t* assignments,
                          const uint8_t* codes, uint64_t n_tokens, uint32_t pq_m, uint8_t* out, uint64_t out_len) {
  if (!h) return MVR_E_INVALID_ARGUMENT;
  Ctx* c = &h->impl;
  mvr::DeviceScope dev_scope(c);
  MVR_TRY(dev_scope.status);
  std::vector<uint64_t> pay;
  MVR_TRY(mvr::check_args(c, doc_offsets, n_docs, n_tokens, pq_m, &pay, out_len));
  if (!out || (n_tokens && (!assignments || !codes))) return mvr::fail(c, MVR_E_INVALID_ARGUMENT, "null pointer");
  MVR_CUDA(c, cudaSetDevice(c->device));
  const uint64_t bytes = (n_docs + 1) * 8 + pay[n_docs];
  uint32_t* d_asg = nullptr;
  uint8_t *d_codes = nullptr, *d_out = nullptr;
  MVR_TRY(mvr::scratch(c, mvr::kSlotAux0, n_tokens * 4 + 16, (void**)&d_asg));
  MVR_TRY(mvr::scratch(c, mvr::kSlotCodes, n_tokens * pq_m + 16, (void**)&d_codes));
  MVR_TRY(mvr::scratch(c, mvr::kSlotAux1, bytes + 16, (void**)&d_out));
  MVR_TRY(mvr::h2d_staged(c, d_asg, assignments, n_tokens * 4));
  MVR_TRY(mvr::h2d_staged(c, d_codes, codes, n_tokens * (uint64_t)pq_m));
  MVR_TRY(mvr::launch(c, doc_offsets, n_docs, pay, d_asg, d_codes, pq_m, d_out));
  MVR_TRY(mvr::d2h_staged(c, out, d_out, bytes));
  return MVR_OK;
}

uint32_t mvr_crc32(uint32_t crc, const void* data, uint64_t len) {
  const auto& T = mvr::crc_tables().t;
  const uint8_t* p = static_cast<const uint8_t*>(data);
  uint32_t c = ~crc;
  while (len >= 8) {
    uint32_t lo, hi;
    std::memcpy(&lo, p, 4);
    std::memcpy(&hi, p + 4, 4);
    lo ^= c;
    c = T[7][lo & 0xff] ^ T[6][(lo >> 8) & 0xff] ^ T[5][(lo >> 16) & 0xff] ^ T[4][lo >> 24] ^ T[3][hi & 0xff] ^
        T[2][(hi >> 8) & 0xff] ^ T[1][(hi >> 16) & 0xff] ^ T[0][hi >> 24];
    p += 8;
    len -= 8;
  }
  while (len--) c = T[0][(c ^ *p++) & 0xff] ^ (c >> 8);
  return ~c;
}

}  // extern "C"
