// refine.cu — query side of the index on the GPU: PQ.buildDistanceTable
// (src/index/pq.zig:92-123) and refine.refine (src/retrieval/refine.zig:
// 83-155) for a batch of candidate documents.
//
// Arithmetic follows the reference exactly (no FMA):
//   vec.dot (vec.zig:37-103): len 2 `a0*b0 + a1*b1`; len 4 left fold from
//   +0; len 64/128 four lane accumulators from +0 then ((a0+a1)+a2)+a3;
//   other lengths the 4-lane loop plus the scalar tail;
//   score(k, i) = dot(q_i, c_{id_k}) + norm_k * sum_m table[m][code_km][i]
//   (the sum from +0 in m order); per query token the first strict maximum
//   over the doc's tokens from -inf; S = sum_i max_i from +0 in i order, and
//   0 for an empty doc.
// Layout: one warp per candidate; lane owns query tokens lane, lane+32, ...
// (the distance table [M][256][n_q] makes each m/code lookup one coalesced
// row); the query sits in shared memory with a padded row stride.
#include <cuda_runtime.h>

#include <algorithm>
#include <vector>

#include "../../include/mvr.h"
#include "mvr_internal.h"

namespace mvr {
namespace {

constexpr int kRefineWarps = 8;

struct Carve {
  size_t off = 0;
  size_t take(size_t bytes) {
    const size_t o = off;
    off = (off + bytes + 255) & ~(size_t)255;
    return o;
  }
};
constexpr uint32_t kMaxQ = 128;  // query tokens per call (4 per lane)

__device__ __forceinline__ float dot_ref(const float* __restrict__ a, const float* __restrict__ b, uint32_t len) {
  if (len == 2) return __fadd_rn(__fmul_rn(a[0], b[0]), __fmul_rn(a[1], b[1]));
  if (len == 4) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) s = __fadd_rn(s, __fmul_rn(a[i], b[i]));
    return s;
  }
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
  uint32_t i = 0;
  for (; i + 4 <= len; i += 4) {
    a0 = __fadd_rn(a0, __fmul_rn(a[i], b[i]));
    a1 = __fadd_rn(a1, __fmul_rn(a[i + 1], b[i + 1]));
    a2 = __fadd_rn(a2, __fmul_rn(a[i + 2], b[i + 2]));
    a3 = __fadd_rn(a3, __fmul_rn(a[i + 3], b[i + 3]));
  }
  float s = __fadd_rn(__fadd_rn(__fadd_rn(a0, a1), a2), a3);
  if (len != 64 && len != 128)  // the generic loop's scalar tail
    for (; i < len; ++i) s = __fadd_rn(s, __fmul_rn(a[i], b[i]));
  return s;
}

// out[(m*256 + c)*n_q + i] = dot(q_i[m*s .. m*s+s], codebook[m][c])
__global__ void pq_table_kernel(const float* __restrict__ cb, uint32_t dim, uint32_t M,
                                const float* __restrict__ q, uint32_t n_q, float* __restrict__ out) {
  const uint32_t s = dim / M;
  const uint64_t total = (uint64_t)M * 256 * n_q;
  for (uint64_t e = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t i = (uint32_t)(e % n_q);
    const uint64_t mc = e / n_q;  // m * 256 + c
    const uint32_t m = (uint32_t)(mc / 256);
    out[e] = dot_ref(q + (uint64_t)i * dim + (uint64_t)m * s, cb + mc * s, s);
  }
}

template <int QS>  // query tokens per lane
__global__ void __launch_bounds__(kRefineWarps * 32)
refine_kernel(const float* __restrict__ cent, uint32_t kappa, uint32_t dim, uint32_t M,
              const uint8_t* __restrict__ sec, uint64_t sec_len, uint64_t n_docs, uint64_t n_tokens,
              const uint64_t* __restrict__ dto,
              const float* __restrict__ norms, const float* __restrict__ table, const float* __restrict__ q,
              uint32_t n_q, const uint32_t* __restrict__ cand, uint64_t n_cand, float* __restrict__ scores,
              int* __restrict__ status) {
  extern __shared__ float qs[];  // n_q rows of dim floats, stride dim + 1
  const uint32_t stride = dim + 1;
  for (uint32_t e = threadIdx.x; e < n_q * dim; e += blockDim.x) qs[(e / dim) * stride + e % dim] = q[e];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const uint64_t* idx = reinterpret_cast<const uint64_t*>(sec);
  const uint8_t* payload = sec + (n_docs + 1) * 8;
  const uint64_t w0 = (uint64_t)blockIdx.x * kRefineWarps + (threadIdx.x >> 5);
  const uint64_t wstride = (uint64_t)gridDim.x * kRefineWarps;
  for (uint64_t c = w0; c < n_cand; c += wstride) {
    const uint32_t doc = cand[c];
    int st = MVR_OK;
    uint32_t n_d = 0;
    uint64_t lo = 0, t_lo = 0;
    if (doc >= n_docs) {
      st = MVR_E_DOC_OUT_OF_RANGE;
    } else {
      lo = idx[doc];
      const uint64_t hi = idx[doc + 1];
      const uint64_t pay_len = sec_len - (n_docs + 1) * 8;
      // every doc block starts 8-byte aligned inside the section
      if (hi < lo || hi - lo < 4 || hi > pay_len || (lo & 7)) {
        st = MVR_E_DOC_LAYOUT_CORRUPT;
      } else {
        n_d = *reinterpret_cast<const uint32_t*>(payload + lo);
        t_lo = dto[doc];
        if (hi - lo < 4 + (uint64_t)n_d * (4 + M) || dto[doc + 1] - t_lo != n_d || t_lo + n_d > n_tokens)
          st = MVR_E_DOC_LAYOUT_CORRUPT;
      }
    }
    if (st == MVR_OK) {
      const uint32_t* ids = reinterpret_cast<const uint32_t*>(payload + lo + 4);
      const uint8_t* codes = payload + lo + 4 + 4 * (uint64_t)n_d;
      float best[QS];
#pragma unroll
      for (int j = 0; j < QS; ++j) best[j] = -__int_as_float(0x7f800000);
      bool bad_id = false;
      for (uint32_t k = 0; k < n_d; ++k) {
        const uint32_t cid = ids[k];
        if (cid >= kappa) {  // the reference would read past the centroids
          bad_id = true;
          break;
        }
        const float* cv = cent + (uint64_t)cid * dim;
        const float norm_k = norms[t_lo + k];
        const uint8_t* ck = codes + (uint64_t)k * M;
#pragma unroll
        for (int j = 0; j < QS; ++j) {
          const uint32_t i = lane + 32 * j;
          if (i < n_q) {
            const float ct = dot_ref(qs + (uint64_t)i * stride, cv, dim);
            float res = 0.f;
            for (uint32_t m = 0; m < M; ++m) res = __fadd_rn(res, table[((uint64_t)m * 256 + ck[m]) * n_q + i]);
            const float sc = __fadd_rn(ct, __fmul_rn(norm_k, res));
            if (sc > best[j]) best[j] = sc;
          }
        }
      }
      if (bad_id) {
        st = MVR_E_DOC_LAYOUT_CORRUPT;
      } else {
        float sum = 0.f;
        if (n_d > 0) {
#pragma unroll
          for (int j = 0; j < QS; ++j)
            for (int l = 0; l < 32; ++l) {
              const float v = __shfl_sync(0xffffffffu, best[j], l);
              if ((uint32_t)(32 * j + l) < n_q) sum = __fadd_rn(sum, v);
            }
        }
        if (lane == 0) scores[c] = sum;
      }
    }
    if (lane == 0) status[c] = st;
  }
}

int set_dev(Ctx* c) {
  MVR_CUDA(c, cudaSetDevice(c->device));
  return MVR_OK;
}

int table_checks(Ctx* c, uint32_t dim, uint32_t pq_m, uint64_t query_len, uint32_t n_q, uint64_t out_len) {
  if (pq_m == 0 || dim == 0 || dim % pq_m) return fail(c, MVR_E_INVALID_ARGUMENT, "dim must be a multiple of pq_m");
  if (n_q == 0 || query_len != (uint64_t)n_q * dim) return fail(c, MVR_E_NQ_MISMATCH, "query length != n_q * dim");
  if (out_len != (uint64_t)pq_m * 256 * n_q) return fail(c, MVR_E_OUT_BUFFER_WRONG_SIZE, "table length");
  return MVR_OK;
}

int launch_table(Ctx* c, const float* d_cb, uint32_t dim, uint32_t pq_m, const float* d_q, uint32_t n_q,
                 float* d_out) {
  const uint64_t total = (uint64_t)pq_m * 256 * n_q;
  const unsigned grid = (unsigned)std::min<uint64_t>((total + 255) / 256, (uint64_t)c->sm_count * 8);
  pq_table_kernel<<<grid, 256, 0, c->stream>>>(d_cb, dim, pq_m, d_q, n_q, d_out);
  MVR_CUDA(c, cudaGetLastError());
  return MVR_OK;
}

struct RefineArgs {
  const float* cent;
  uint32_t kappa, dim, pq_m;
  const uint8_t* sec;
  uint64_t sec_len, n_docs, n_tokens;
  const uint64_t* dto;
  const float* norms;
  const float* table;
  const float* q;
  uint32_t n_q;
  const uint32_t* cand;
  uint64_t n_cand;
  float* scores;
  int* status;
};

int refine_checks(Ctx* c, uint32_t dim, uint32_t pq_m, uint64_t query_len, uint32_t n_q, uint64_t table_len) {
  if (pq_m == 0 || dim == 0) return fail(c, MVR_E_INVALID_ARGUMENT, "dim and pq_m must be positive");
  if (n_q == 0 || query_len != (uint64_t)n_q * dim) return fail(c, MVR_E_QUERY_SHAPE_MISMATCH, "query shape");
  if (table_len != (uint64_t)pq_m * 256 * n_q) return fail(c, MVR_E_TABLE_SIZE_MISMATCH, "table length");
  if (n_q > kMaxQ) return fail(c, MVR_E_INVALID_ARGUMENT, "more than 128 query tokens per call");
  if ((size_t)n_q * (dim + 1) * sizeof(float) > 200 * 1024)
    return fail(c, MVR_E_INVALID_ARGUMENT, "query too large for shared memory");
  return MVR_OK;
}

int launch_refine(Ctx* c, const RefineArgs& a) {
  if (a.n_cand == 0) return MVR_OK;
  const size_t smem = (size_t)a.n_q * (a.dim + 1) * sizeof(float);
  const unsigned grid = (unsigned)std::min<uint64_t>((a.n_cand + kRefineWarps - 1) / kRefineWarps,
                                                     (uint64_t)c->sm_count * 16);
  auto kern = a.n_q <= 32 ? refine_kernel<1> : a.n_q <= 64 ? refine_kernel<2> : refine_kernel<4>;
  MVR_CUDA(c, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  kern<<<grid, kRefineWarps * 32, smem, c->stream>>>(a.cent, a.kappa, a.dim, a.pq_m, a.sec, a.sec_len, a.n_docs,
                                                    a.n_tokens, a.dto,
                                                    a.norms, a.table, a.q, a.n_q, a.cand, a.n_cand, a.scores,
                                                    a.status);
  MVR_CUDA(c, cudaGetLastError());
  return MVR_OK;
}

// First failing candidate (candidate order), as a serial caller would see.
int first_status(Ctx* c, const std::vector<int>& st) {
  for (size_t i = 0; i < st.size(); ++i)
    if (st[i] != MVR_OK)
      return fail(c, st[i], "candidate " + std::to_string(i) + ": " + mvr_status_name(st[i]));
  return MVR_OK;
}

}  // namespace
}  // namespace mvr

using mvr::Ctx;

extern "C" {

int mvr_pq_distance_table_device(mvr_ctx* h, const float* d_codebooks, uint32_t dim, uint32_t pq_m,
                                 const float* d_query, uint64_t query_len, uint32_t n_q, float* d_out,
                                 uint64_t out_len) {
  if (!h) return MVR_E_INVALID_ARGUMENT;
  Ctx* c = &h->impl;
  mvr::DeviceScope dev_scope(c);
  MVR_TRY(dev_scope.status);
  MVR_TRY(mvr::table_checks(c, dim, pq_m, query_len, n_q, out_len));
  if (!d_codebooks || !d_query || !d_out) return mvr::fail(c, MVR_E_INVALID_ARGUMENT, "null pointer");
  MVR_TRY(mvr::set_dev(c));
  return mvr::launch_table(c, d_codebooks, dim, pq_m, d_query, n_q, d_out);
}

int mvr_pq_distance_table(mvr_ctx* h, const float* codebooks, uint32_t dim, uint32_t pq_m, const float* query,
                          uint64_t query_len, uint32_t n_q, float* out, uint64_t out_len) {
  if (!h) return MVR_E_INVALID_ARGUMENT;
  Ctx* c = &h->impl;
  mvr::DeviceScope dev_scope(c);
  MVR_TRY(dev_scope.status);
  MVR_TRY(mvr::table_checks(c, dim, pq_m, query_len, n_q, out_len));
  if (!codebooks || !query || !out) return mvr::fail(c, MVR_E_INVALID_ARGUMENT, "null pointer");
  MVR_TRY(mvr::set_dev(c));
  const size_t cb_bytes = (size_t)pq_m * 256 * (dim / pq_m) * sizeof(float);
  float *d_cb = nullptr, *d_q = nullptr, *d_out = nullptr;
  MVR_TRY(mvr::scratch(c, mvr::kSlotCodebooks, cb_bytes, (void**)&d_cb));
  MVR_TRY(mvr::scratch(c, mvr::kSlotAux0, query_len * 4, (void**)&d_q));
  MVR_TRY(mvr::scratch(c, mvr::kSlotAux1, out_len * 4, (void**)&d_out));
  MVR_TRY(mvr::h2d_staged(c, d_cb, codebooks, cb_bytes));
  MVR_TRY(mvr::h2d_staged(c, d_q, query, query_len * 4));
  MVR_TRY(mvr::launch_table(c, d_cb, dim, pq_m, d_q, n_q, d_out));
  return mvr::d2h_staged(c, out, d_out, out_len * 4);
}

int mvr_refine_batch_device(mvr_ctx* h, const float* d_centroids, uint32_t kappa, uint32_t dim, uint32_t pq_m,
                            const uint8_t* d_doc_section, uint64_t doc_section_len, uint64_t n_docs,
                            const uint64_t* d_doc_token_offsets, const float* d_residual_norms, uint64_t n_tokens,
                            const float* d_table, uint64_t table_len,
                            const float* d_query, uint64_t query_len, uint32_t n_q, const uint32_t* d_doc_ids,
                            uint64_t n_cand, float* d_scores, int* d_status) {
  if (!h) return MVR_E_INVALID_ARGUMENT;
  Ctx* c = &h->impl;
  mvr::DeviceScope dev_scope(c);
  MVR_TRY(dev_scope.status);
  MVR_TRY(mvr::refine_checks(c, dim, pq_m, query_len, n_q, table_len));
  if (n_cand && (!d_centroids || !d_doc_section || !d_doc_token_offsets || !d_residual_norms || !d_table ||
                 !d_query || !d_doc_ids || !d_scores || !d_status))
    return mvr::fail(c, MVR_E_INVALID_ARGUMENT, "null pointer");
  if (reinterpret_cast<uintptr_t>(d_doc_section) % 8)
    return mvr::fail(c, MVR_E_INVALID_ARGUMENT, "doc section must be 8-byte aligned");
  if (doc_section_len < (n_docs + 1) * 8) return mvr::fail(c, MVR_E_DOC_LAYOUT_CORRUPT, "doc section too short");
  MVR_TRY(mvr::set_dev(c));
  mvr::RefineArgs a{d_centroids, kappa, dim, pq_m, d_doc_section, doc_section_len, n_docs, n_tokens,
                    d_doc_token_offsets, d_residual_norms, d_table, d_query, n_q, d_doc_ids, n_cand, d_scores,
                    d_status};
  return mvr::launch_refine(c, a);
}

int mvr_refine_batch(mvr_ctx* h, const float* centroids, uint32_t kappa, uint32_t dim, uint32_t pq_m,
                     const uint8_t* doc_section, uint64_t doc_section_len, uint64_t n_docs,
                     const uint64_t* doc_token_offsets, const float* residual_norms, uint64_t n_tokens,
                     const float* table, uint64_t table_len, const float* query, uint64_t query_len, uint32_t n_q,
                     const uint32_t* doc_ids, uint64_t n_cand, float* scores_out) {
  if (!h) return MVR_E_INVALID_ARGUMENT;
  Ctx* c = &h->impl;
  mvr::DeviceScope dev_scope(c);
  MVR_TRY(dev_scope.status);
  MVR_TRY(mvr::refine_checks(c, dim, pq_m, query_len, n_q, table_len));
  if (n_cand == 0) return MVR_OK;
  if (!centroids || !doc_section || !doc_token_offsets || !residual_norms || !table || !query || !doc_ids ||
      !scores_out)
    return mvr::fail(c, MVR_E_INVALID_ARGUMENT, "null pointer");
  if (doc_section_len < (n_docs + 1) * 8) return mvr::fail(c, MVR_E_DOC_LAYOUT_CORRUPT, "doc section too short");
  // the doc index must stay inside the section
  const uint64_t* idx = reinterpret_cast<const uint64_t*>(doc_section);
  for (uint64_t d = 0; d <= n_docs; ++d)
    if (idx[d] > doc_section_len - (n_docs + 1) * 8)
      return mvr::fail(c, MVR_E_DOC_LAYOUT_CORRUPT, "doc index points past the section");
  if (doc_token_offsets[n_docs] > n_tokens)
    return mvr::fail(c, MVR_E_DOC_LAYOUT_CORRUPT, "token offsets past the norms");
  MVR_TRY(mvr::set_dev(c));
  const size_t cent_b = (size_t)kappa * dim * 4, tab_b = table_len * 4, q_b = query_len * 4;
  mvr::Carve cv;  // one workspace for the index sections and the query
  const size_t o_cent = cv.take(cent_b), o_sec = cv.take(doc_section_len), o_dto = cv.take((n_docs + 1) * 8),
               o_norm = cv.take(n_tokens * 4), o_tab = cv.take(tab_b), o_q = cv.take(q_b),
               o_cand = cv.take(n_cand * 4), o_sc = cv.take(n_cand * 4), o_st = cv.take(n_cand * 4);
  unsigned char* ws = nullptr;
  MVR_TRY(mvr::scratch(c, mvr::kSlotAux3, cv.off, (void**)&ws));
  MVR_TRY(mvr::h2d_staged(c, ws + o_cent, centroids, cent_b));
  MVR_TRY(mvr::h2d_staged(c, ws + o_sec, doc_section, doc_section_len));
  MVR_TRY(mvr::h2d_staged(c, ws + o_dto, doc_token_offsets, (n_docs + 1) * 8));
  MVR_TRY(mvr::h2d_staged(c, ws + o_norm, residual_norms, n_tokens * 4));
  MVR_TRY(mvr::h2d_staged(c, ws + o_tab, table, tab_b));
  MVR_TRY(mvr::h2d_staged(c, ws + o_q, query, q_b));
  MVR_TRY(mvr::h2d_staged(c, ws + o_cand, doc_ids, n_cand * 4));
  mvr::RefineArgs a{(const float*)(ws + o_cent), kappa, dim, pq_m, ws + o_sec, doc_section_len, n_docs, n_tokens,
                    (const uint64_t*)(ws + o_dto),
                    (const float*)(ws + o_norm), (const float*)(ws + o_tab), (const float*)(ws + o_q), n_q,
                    (const uint32_t*)(ws + o_cand), n_cand, (float*)(ws + o_sc), (int*)(ws + o_st)};
  MVR_TRY(mvr::launch_refine(c, a));
  std::vector<int> st(n_cand);
  MVR_TRY(mvr::d2h_staged(c, st.data(), ws + o_st, n_cand * 4));
  MVR_TRY(mvr::d2h_staged(c, scores_out, ws + o_sc, n_cand * 4));
  return mvr::first_status(c, st);
}

}  // extern "C"
