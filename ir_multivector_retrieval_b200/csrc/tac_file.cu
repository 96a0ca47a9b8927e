// tac_file.cu — inverted lists on the GPU and the .tac index image.
//
// Reference (BleedingDev/ir-multivector-retrieval):
//   inverted_list.build   src/index/inverted_list.zig:64-150
//   storage.computeSize   src/index/storage.zig:490-551
//   storage.serialise     src/index/storage.zig:560-665 (writeHnsw :667-703,
//                         writeDocLayouts :705-749)
//
// Inverted lists: the reference walks the documents in order with a stamp
// set per centroid. Here every token carries (centroid, doc); a stable radix
// sort by centroid keeps the docs ascending inside each centroid (tokens are
// in doc order), adjacent equal pairs collapse to one entry (a flag, an
// exclusive scan, a scatter), and each centroid's first position gives the
// CSR offsets. The result is the reference's byte for byte: offsets[j] is
// the number of distinct (doc, centroid' < j) pairs, the payload of j is its
// distinct docs in increasing order.
//
// The image is assembled in the caller's host buffer: fixed-layout sections
// are copied, the per-doc section is interleaved on the GPU
// (mvr_write_doc_layouts), and the footer CRC-32 runs over host threads
// (chunk CRCs joined with the GF(2) combination of zlib's crc32_combine).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <thread>
#include <vector>

#include "../../include/mvr.h"
#include "km_engine.h"
#include "mvr_internal.h"

namespace mvr {
namespace {

// Doc id of every token (one warp per doc) and a flag for assignments
// outside [0, kappa).
__global__ void __launch_bounds__(256)
ilist_doc_ids_kernel(const uint64_t* __restrict__ doc_off, uint64_t n_docs, const uint32_t* __restrict__ asg,
                     uint32_t kappa, uint32_t* __restrict__ doc_of, int* __restrict__ err) {
  const uint64_t d = (uint64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (d >= n_docs) return;
  const int lane = threadIdx.x & 31;
  bool bad = false;
  for (uint64_t t = doc_off[d] + lane; t < doc_off[d + 1]; t += 32) {
    doc_of[t] = (uint32_t)d;
    bad |= asg[t] >= kappa;
  }
  if (__any_sync(0xffffffffu, bad) && lane == 0) atomicExch(err, 1);
}

// flag[i] = 1 when (key, val)[i] starts a new (centroid, doc) pair.
__global__ void __launch_bounds__(256)
ilist_flags_kernel(const uint32_t* __restrict__ k, const uint32_t* __restrict__ v, uint64_t n,
                   uint32_t* __restrict__ flag) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    flag[i] = (i == 0 || k[i] != k[i - 1] || v[i] != v[i - 1]) ? 1u : 0u;
}

// Payload (first occurrence of each pair at its scanned position) and the
// CSR offsets: centroids c in (previous key, key[i]] start at pos[i]; the
// thread past the end fills (last key, kappa] with the total.
__global__ void __launch_bounds__(256)
ilist_scatter_kernel(const uint32_t* __restrict__ k, const uint32_t* __restrict__ v, const uint32_t* __restrict__ flag,
                     const uint32_t* __restrict__ pos, uint64_t n, uint32_t kappa, uint32_t* __restrict__ payload,
                     unsigned long long* __restrict__ offsets) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i <= n; i += (uint64_t)gridDim.x * blockDim.x) {
    if (i == n) {
      const uint64_t total = n ? (uint64_t)pos[n - 1] + flag[n - 1] : 0;
      for (uint64_t c = n ? (uint64_t)k[n - 1] + 1 : 0; c <= kappa; ++c) offsets[c] = total;
      continue;
    }
    if (flag[i]) payload[pos[i]] = v[i];
    if (i == 0 || k[i] != k[i - 1])
      for (uint64_t c = i == 0 ? 0 : (uint64_t)k[i - 1] + 1; c <= k[i]; ++c) offsets[c] = pos[i];
  }
}

uint64_t up8(uint64_t v) { return (v + 7u) & ~(uint64_t)7u; }

int check_parts(const mvr_tac_parts* p) {
  if (!p || !p->centroids || !p->codebooks || !p->doc_offsets || !p->ilist_offsets || !p->hnsw_node_levels ||
      !p->hnsw_layer_offsets || !p->hnsw_layer_neighbours)
    return MVR_E_INVALID_ARGUMENT;
  if (p->n_tokens && (!p->assignments || !p->pq_codes || !p->residual_norms)) return MVR_E_INVALID_ARGUMENT;
  if (p->hnsw_max_level > 255) return MVR_E_INVALID_ARGUMENT;
  for (uint32_t L = 0; L <= p->hnsw_max_level; ++L)
    if (!p->hnsw_layer_offsets[L] || (p->hnsw_layer_offsets[L][p->hnsw_n] && !p->hnsw_layer_neighbours[L]))
      return MVR_E_INVALID_ARGUMENT;
  if (p->ilist_offsets[p->kappa] && !p->ilist_payload) return MVR_E_INVALID_ARGUMENT;
  if (p->doc_offsets[p->n_docs] != p->n_tokens) return MVR_E_INVALID_ARGUMENT;
  return MVR_OK;
}

uint64_t file_size(const mvr_tac_parts* p) {
  uint64_t off = MVR_TAC_HEADER_REGION;
  off = up8(off + (uint64_t)p->kappa * p->dim * 4);
  uint64_t h = up8(24 + (uint64_t)p->hnsw_n);  // hnswSize (storage.zig:521-537)
  for (uint32_t L = 0; L <= p->hnsw_max_level; ++L) {
    h = up8(h + ((uint64_t)p->hnsw_n + 1) * 4);
    h = up8(h + (uint64_t)p->hnsw_layer_offsets[L][p->hnsw_n] * 4);
  }
  off = up8(off + h);
  off = up8(off + (uint64_t)p->pq_m * MVR_PQ_CENTROIDS * p->sub_dim * 4);
  off += ((uint64_t)p->kappa + 1) * 8;
  off = up8(off + p->ilist_offsets[p->kappa] * 4);
  off += (p->n_docs + 1) * 8;
  uint64_t docs = 0;  // docPayloadSize (storage.zig:539-551)
  for (uint64_t d = 0; d < p->n_docs; ++d) {
    const uint64_t n_d = p->doc_offsets[d + 1] - p->doc_offsets[d];
    docs += up8(4 + n_d * 4 + n_d * (uint64_t)p->pq_m);
  }
  off = up8(off + docs);
  off = up8(off + (p->n_docs + 1) * 8);
  off = up8(off + p->n_tokens * 4);
  return off + 8;
}

// Copy n bytes at cur, zero-pad to 8, return the next offset.
uint64_t put(uint8_t* buf, uint64_t cur, const void* src, uint64_t n) {
  if (n) std::memcpy(buf + cur, src, n);
  const uint64_t end = up8(cur + n);
  std::memset(buf + cur + n, 0, end - cur - n);
  return end;
}

void put32(uint8_t* b, uint64_t off, uint32_t v) { std::memcpy(b + off, &v, 4); }
void put64(uint8_t* b, uint64_t off, uint64_t v) { std::memcpy(b + off, &v, 8); }

// CRC-32 combination (zlib's crc32_combine, Mark Adler): the CRC of A||B
// from crc(A), crc(B) and |B|, by applying |B| zero bytes to crc(A) as
// repeated squarings of the GF(2) operator of one zero bit.
uint32_t gf2_times(const uint32_t* mat, uint32_t vec) {
  uint32_t sum = 0;
  for (int i = 0; vec; ++i, vec >>= 1)
    if (vec & 1u) sum ^= mat[i];
  return sum;
}
void gf2_square(uint32_t* sq, const uint32_t* mat) {
  for (int n = 0; n < 32; ++n) sq[n] = gf2_times(mat, mat[n]);
}
uint32_t crc32_combine_impl(uint32_t crc1, uint32_t crc2, uint64_t len2) {
  if (len2 == 0) return crc1;
  uint32_t even[32], odd[32];
  odd[0] = 0xEDB88320u;  // the operator of one zero bit
  uint32_t row = 1;
  for (int n = 1; n < 32; ++n) {
    odd[n] = row;
    row <<= 1;
  }
  gf2_square(even, odd);  // two zero bits
  gf2_square(odd, even);  // four zero bits
  do {
    gf2_square(even, odd);
    if (len2 & 1) crc1 = gf2_times(even, crc1);
    len2 >>= 1;
    if (len2 == 0) break;
    gf2_square(odd, even);
    if (len2 & 1) crc1 = gf2_times(odd, crc1);
    len2 >>= 1;
  } while (len2 != 0);
  return crc1 ^ crc2;
}

// The footer checksum over host threads (same value as one pass).
uint32_t crc32_parallel(const uint8_t* p, uint64_t len) {
  const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
  const uint64_t min_chunk = 4ull << 20;
  const unsigned T = (unsigned)std::min<uint64_t>(std::min(hw, 32u), std::max<uint64_t>(1, len / min_chunk));
  if (T <= 1) return mvr_crc32(0, p, len);
  std::vector<uint32_t> part(T);
  std::vector<uint64_t> lo(T + 1);
  for (unsigned t = 0; t <= T; ++t) lo[t] = len * t / T;
  std::vector<std::thread> th;
  for (unsigned t = 0; t < T; ++t)
    th.emplace_back([&, t] { part[t] = mvr_crc32(0, p + lo[t], lo[t + 1] - lo[t]); });
  for (auto& x : th) x.join();
  uint32_t crc = part[0];
  for (unsigned t = 1; t < T; ++t) crc = crc32_combine_impl(crc, part[t], lo[t + 1] - lo[t]);
  return crc;
}

}  // namespace
}  // namespace mvr

using mvr::Ctx;

extern "C" {

uint32_t mvr_crc32_combine(uint32_t crc1, uint32_t crc2, uint64_t len2) {
  return mvr::crc32_combine_impl(crc1, crc2, len2);
}

int mvr_inverted_lists_build(mvr_ctx* h, const uint32_t* assignments, uint64_t n_tokens, const uint64_t* doc_offsets,
                             uint64_t doc_offsets_len, uint32_t kappa, uint64_t* offsets_out, uint32_t* payload_out,
                             uint64_t payload_cap, uint64_t* payload_len_out) {
  if (!h || !offsets_out || !payload_len_out) return MVR_E_INVALID_ARGUMENT;
  Ctx* c = &h->impl;
  mvr::DeviceScope dev_scope(c);
  MVR_TRY(dev_scope.status);
  // inverted_list.zig:70-87, in order
  if (kappa == 0) return mvr::fail(c, MVR_E_KAPPA_ZERO, "kappa == 0");
  if (doc_offsets_len < 1 || !doc_offsets) return mvr::fail(c, MVR_E_DOC_OFFSETS_BAD, "no doc offsets");
  const uint64_t n_docs = doc_offsets_len - 1;
  if (n_docs > 0xFFFFFFFFull) return mvr::fail(c, MVR_E_DOC_OFFSETS_BAD, "more than 2^32 - 1 docs");
  if (doc_offsets[n_docs] != n_tokens) return mvr::fail(c, MVR_E_DOC_OFFSETS_BAD, "last offset != n_tokens");
  if (doc_offsets[0] != 0) return mvr::fail(c, MVR_E_DOC_OFFSETS_BAD, "first offset != 0");
  for (uint64_t d = 1; d <= n_docs; ++d)
    if (doc_offsets[d] < doc_offsets[d - 1]) return mvr::fail(c, MVR_E_DOC_OFFSETS_BAD, "decreasing offsets");
  if (n_tokens && !assignments) return MVR_E_INVALID_ARGUMENT;
  if (n_tokens >= (1ull << 32)) return mvr::fail(c, MVR_E_INVALID_ARGUMENT, "more than 2^32 - 1 tokens");
  MVR_CUDA(c, cudaSetDevice(c->device));
  cudaStream_t st = c->stream;
  // workspace: asg | doc ids | 2 x (keys, vals) | flags | positions | scratch | offsets | payload | doc offsets | err
  const uint64_t n = n_tokens;
  const size_t rs = mvr::radix_pairs_scratch_words(n), sp = mvr::scan_part_words(n);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = (off + bytes + 255) & ~(size_t)255;
    return o;
  };
  const size_t o_asg = take(n * 4), o_doc = take(n * 4), o_k0 = take(n * 4), o_v0 = take(n * 4),
               o_k1 = take(n * 4), o_v1 = take(n * 4), o_flag = take(n * 4), o_pos = take(n * 4),
               o_rs = take(rs * 4), o_sp = take(sp * 4), o_off = take(((size_t)kappa + 1) * 8),
               o_pay = take(n * 4), o_doff = take((n_docs + 1) * 8), o_err = take(16);
  unsigned char* ws = nullptr;
  MVR_TRY(mvr::scratch(c, mvr::kSlotAux3, off, (void**)&ws));
  auto at = [&](size_t o) { return reinterpret_cast<uint32_t*>(ws + o); };
  int* d_err = reinterpret_cast<int*>(ws + o_err);
  MVR_CUDA(c, cudaMemsetAsync(d_err, 0, sizeof(int), st));
  if (n) MVR_TRY(mvr::h2d_staged(c, at(o_asg), assignments, n * 4));
  MVR_TRY(mvr::h2d_staged(c, ws + o_doff, doc_offsets, (n_docs + 1) * 8));
  if (n_docs) {
    mvr::ilist_doc_ids_kernel<<<(unsigned)((n_docs + 7) / 8), 256, 0, st>>>(
        reinterpret_cast<const uint64_t*>(ws + o_doff), n_docs, at(o_asg), kappa, at(o_doc), d_err);
    MVR_CUDA(c, cudaGetLastError());
  }
  int herr = 0;
  MVR_CUDA(c, cudaMemcpyAsync(&herr, d_err, sizeof(int), cudaMemcpyDeviceToHost, st));
  MVR_CUDA(c, cudaStreamSynchronize(st));
  if (herr) return mvr::fail(c, MVR_E_ASSIGNMENT_OUT_OF_RANGE, "assignment >= kappa");
  int bits = 1;
  while (bits < 32 && ((uint64_t)kappa - 1) >> bits) ++bits;
  const uint32_t *sk = nullptr, *sv = nullptr;
  MVR_TRY(mvr::radix_sort_pairs(c, st, at(o_asg), at(o_doc), n, bits, at(o_k0), at(o_v0), at(o_k1), at(o_v1),
                                at(o_rs), &sk, &sv));
  const unsigned grid = (unsigned)std::min<uint64_t>((n + 256) / 256 + 1, (uint64_t)c->sm_count * 8);
  if (n) {
    mvr::ilist_flags_kernel<<<grid, 256, 0, st>>>(sk, sv, n, at(o_flag));
    MVR_CUDA(c, cudaGetLastError());
    MVR_TRY(mvr::exclusive_scan_u32(c, st, at(o_flag), n, at(o_sp), at(o_pos)));
  }
  unsigned long long* d_off = reinterpret_cast<unsigned long long*>(ws + o_off);
  mvr::ilist_scatter_kernel<<<grid, 256, 0, st>>>(sk, sv, at(o_flag), at(o_pos), n, kappa, at(o_pay), d_off);
  MVR_CUDA(c, cudaGetLastError());
  MVR_TRY(mvr::d2h_staged(c, offsets_out, d_off, ((size_t)kappa + 1) * 8));
  const uint64_t total = offsets_out[kappa];
  *payload_len_out = total;
  if (total > payload_cap || (total && !payload_out))
    return mvr::fail(c, MVR_E_BUFFER_TOO_SMALL, "inverted-list payload does not fit");
  if (total) MVR_TRY(mvr::d2h_staged(c, payload_out, at(o_pay), total * 4));
  return MVR_OK;
}

int mvr_tac_file_size(const mvr_tac_parts* p, uint64_t* bytes_out) {
  if (!bytes_out) return MVR_E_INVALID_ARGUMENT;
  MVR_TRY(mvr::check_parts(p));
  *bytes_out = mvr::file_size(p);
  return MVR_OK;
}

int mvr_tac_serialise(mvr_ctx* h, const mvr_tac_parts* p, void* out, uint64_t buf_len, uint64_t* written_out) {
  if (!h || !out) return MVR_E_INVALID_ARGUMENT;
  Ctx* c = &h->impl;
  mvr::DeviceScope dev_scope(c);
  MVR_TRY(dev_scope.status);
  MVR_TRY(mvr::check_parts(p));
  const uint64_t total = mvr::file_size(p);
  if (buf_len < total) return mvr::fail(c, MVR_E_BUFFER_TOO_SMALL, "serialise: buffer smaller than the image");
  uint8_t* buf = static_cast<uint8_t*>(out);
  std::memset(buf, 0, MVR_TAC_HEADER_REGION);
  uint64_t cur = MVR_TAC_HEADER_REGION;
  const uint64_t centroids_off = cur;
  cur = mvr::put(buf, cur, p->centroids, (uint64_t)p->kappa * p->dim * 4);
  const uint64_t hnsw_off = cur;
  {  // writeHnsw (storage.zig:667-703)
    std::memset(buf + cur, 0, 24);
    buf[cur] = (uint8_t)p->hnsw_max_level;
    mvr::put32(buf, cur + 8, p->hnsw_entry_point);
    mvr::put32(buf, cur + 16, p->hnsw_n);
    cur = mvr::put(buf, cur + 24, p->hnsw_node_levels, p->hnsw_n);
    for (uint32_t L = 0; L <= p->hnsw_max_level; ++L) {
      cur = mvr::put(buf, cur, p->hnsw_layer_offsets[L], ((uint64_t)p->hnsw_n + 1) * 4);
      cur = mvr::put(buf, cur, p->hnsw_layer_neighbours[L], (uint64_t)p->hnsw_layer_offsets[L][p->hnsw_n] * 4);
    }
  }
  const uint64_t pq_off = cur;
  cur = mvr::put(buf, cur, p->codebooks, (uint64_t)p->pq_m * MVR_PQ_CENTROIDS * p->sub_dim * 4);
  const uint64_t ilist_off = cur;
  std::memcpy(buf + cur, p->ilist_offsets, ((uint64_t)p->kappa + 1) * 8);
  cur += ((uint64_t)p->kappa + 1) * 8;
  cur = mvr::put(buf, cur, p->ilist_payload, p->ilist_offsets[p->kappa] * 4);
  const uint64_t doc_off = cur;
  {
    uint64_t doc_bytes = 0;
    MVR_TRY(mvr_doc_layouts_bytes(p->doc_offsets, p->n_docs, p->pq_m, &doc_bytes));
    MVR_TRY(mvr_write_doc_layouts(h, p->doc_offsets, p->n_docs, p->assignments, p->pq_codes, p->n_tokens, p->pq_m,
                                  buf + cur, doc_bytes));
    const uint64_t end = mvr::up8(cur + doc_bytes);
    std::memset(buf + cur + doc_bytes, 0, end - cur - doc_bytes);
    cur = end;
  }
  const uint64_t doc_tok_off = cur;
  cur = mvr::put(buf, cur, p->doc_offsets, (p->n_docs + 1) * 8);
  const uint64_t norms_off = cur;
  cur = mvr::put(buf, cur, p->residual_norms, p->n_tokens * 4);
  const uint64_t footer_off = cur;
  // Header (storage.zig:52-73, 112 bytes, little-endian) in the zeroed region
  std::memcpy(buf, "TAC_IDX1", 8);
  mvr::put32(buf, 8, MVR_TAC_VERSION);
  mvr::put32(buf, 12, p->dim);
  mvr::put32(buf, 16, p->kappa);
  mvr::put32(buf, 20, p->pq_m);
  buf[24] = 8;  // pq_bits
  mvr::put32(buf, 28, p->sub_dim);
  mvr::put64(buf, 32, p->n_docs);
  mvr::put64(buf, 40, p->n_tokens);
  const uint64_t offs[8] = {centroids_off, hnsw_off, pq_off, ilist_off, doc_off, doc_tok_off, norms_off, footer_off};
  for (int i = 0; i < 8; ++i) mvr::put64(buf, 48 + 8 * (uint64_t)i, offs[i]);
  // footer: CRC-32 of everything before it, then 4 zero bytes
  mvr::put32(buf, footer_off, mvr::crc32_parallel(buf, footer_off));
  mvr::put32(buf, footer_off + 4, 0);
  if (footer_off + 8 != total) return mvr::fail(c, MVR_E_INVALID_INDEX, "serialise: image size mismatch");
  if (written_out) *written_out = total;
  return MVR_OK;
}

}  // extern "C"
