/* tac_file_oracle.c — CPU restatement of the reference's inverted lists and
 * .tac index image, for tests only (the parity checker of the GPU builder
 * and serialiser; never part of the product path).
 *
 *   inverted_list.build   src/index/inverted_list.zig:64-150
 *   storage.computeSize   src/index/storage.zig:490-519 (+ hnswSize :521-537,
 *                         docPayloadSize :539-551)
 *   storage.serialise     src/index/storage.zig:560-665
 *   storage.writeHnsw     src/index/storage.zig:667-703
 *   storage.parse         src/index/storage.zig:765-860 (+ parseHnsw
 *                         :862-930, parsePq :932-951, parseInvertedLists
 *                         :953-978)
 *   std.hash.Crc32        the IEEE CRC-32 (reflected 0xEDB88320, initial and
 *                         final xor 0xFFFFFFFF), one table, byte at a time.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "mvr_oracle.h"

static uint64_t up8(uint64_t v) { return (v + 7u) & ~(uint64_t)7u; }

static uint32_t g_crc_table[256];
static int g_crc_ready = 0;

uint32_t orc_crc32(const uint8_t* p, uint64_t len) {
  if (!g_crc_ready) {
    for (uint32_t i = 0; i < 256; ++i) {
      uint32_t c = i;
      for (int k = 0; k < 8; ++k) c = (c & 1u) ? (0xEDB88320u ^ (c >> 1)) : (c >> 1);
      g_crc_table[i] = c;
    }
    g_crc_ready = 1;
  }
  uint32_t c = 0xFFFFFFFFu;
  for (uint64_t i = 0; i < len; ++i) c = g_crc_table[(c ^ p[i]) & 0xFFu] ^ (c >> 8);
  return c ^ 0xFFFFFFFFu;
}

/* inverted_list.build: validation in the reference's order, then the
 * two-pass stamp-set CSR (counts, exclusive scan, cursors). */
int orc_inverted_lists_build(const uint32_t* assignments, uint64_t n_assign, const uint64_t* doc_offsets,
                             uint64_t doc_offsets_len, uint32_t kappa, uint64_t* offsets, uint32_t* payload,
                             uint64_t payload_cap, uint64_t* total_out) {
  if (kappa == 0) return MVR_E_KAPPA_ZERO;
  if (doc_offsets_len < 1) return MVR_E_DOC_OFFSETS_BAD;
  const uint64_t n_docs = doc_offsets_len - 1;
  if (n_docs > 0xFFFFFFFFull) return MVR_E_DOC_OFFSETS_BAD;
  const uint64_t n_tokens = doc_offsets[doc_offsets_len - 1];
  if (n_assign != n_tokens) return MVR_E_DOC_OFFSETS_BAD;
  if (doc_offsets[0] != 0) return MVR_E_DOC_OFFSETS_BAD;
  for (uint64_t d = 1; d < doc_offsets_len; ++d)
    if (doc_offsets[d] < doc_offsets[d - 1]) return MVR_E_DOC_OFFSETS_BAD;
  for (uint64_t i = 0; i < n_assign; ++i)
    if (assignments[i] >= kappa) return MVR_E_ASSIGNMENT_OUT_OF_RANGE;
  uint64_t* stamps = (uint64_t*)malloc(sizeof(uint64_t) * kappa);
  if (!stamps) return MVR_E_OUT_OF_MEMORY;
  memset(stamps, 0xFF, sizeof(uint64_t) * kappa);
  memset(offsets, 0, sizeof(uint64_t) * ((uint64_t)kappa + 1));
  for (uint64_t d = 0; d < n_docs; ++d)
    for (uint64_t t = doc_offsets[d]; t < doc_offsets[d + 1]; ++t) {
      const uint32_t j = assignments[t];
      if (stamps[j] != d) {
        stamps[j] = d;
        offsets[(uint64_t)j + 1] += 1;
      }
    }
  uint64_t total = 0;
  for (uint64_t j = 0; j < kappa; ++j) {
    total += offsets[j + 1];
    offsets[j + 1] = total;
  }
  if (total > payload_cap) {
    free(stamps);
    return MVR_E_BUFFER_TOO_SMALL;
  }
  uint64_t* cursor = (uint64_t*)malloc(sizeof(uint64_t) * kappa);
  if (!cursor) {
    free(stamps);
    return MVR_E_OUT_OF_MEMORY;
  }
  memcpy(cursor, offsets, sizeof(uint64_t) * kappa);
  memset(stamps, 0xFF, sizeof(uint64_t) * kappa);
  for (uint64_t d = 0; d < n_docs; ++d)
    for (uint64_t t = doc_offsets[d]; t < doc_offsets[d + 1]; ++t) {
      const uint32_t j = assignments[t];
      if (stamps[j] != d) {
        stamps[j] = d;
        payload[cursor[j]++] = (uint32_t)d;
      }
    }
  free(stamps);
  free(cursor);
  *total_out = total;
  return MVR_OK;
}

static uint64_t hnsw_size(const mvr_tac_parts* p) {
  uint64_t b = 24;
  b = up8(b + p->hnsw_n);
  for (uint32_t L = 0; L <= p->hnsw_max_level; ++L) {
    b = up8(b + ((uint64_t)p->hnsw_n + 1) * 4);
    b = up8(b + (uint64_t)p->hnsw_layer_offsets[L][p->hnsw_n] * 4);
  }
  return b;
}

static uint64_t doc_payload_size(const mvr_tac_parts* p) {
  uint64_t total = 0;
  for (uint64_t d = 0; d < p->n_docs; ++d) {
    const uint64_t n_d = p->doc_offsets[d + 1] - p->doc_offsets[d];
    total += up8(4 + n_d * 4 + n_d * (uint64_t)p->pq_m);
  }
  return total;
}

uint64_t orc_tac_file_size(const mvr_tac_parts* p) {
  uint64_t off = MVR_TAC_HEADER_REGION;
  off = up8(off + (uint64_t)p->kappa * p->dim * 4);
  off = up8(off + hnsw_size(p));
  off = up8(off + (uint64_t)p->pq_m * 256u * p->sub_dim * 4);
  off += ((uint64_t)p->kappa + 1) * 8;
  off = up8(off + p->ilist_offsets[p->kappa] * 4);
  off += (p->n_docs + 1) * 8;
  off = up8(off + doc_payload_size(p));
  off = up8(off + (p->n_docs + 1) * 8);
  off = up8(off + p->n_tokens * 4);
  return off + 8;
}

static void put32(uint8_t* b, uint64_t off, uint32_t v) { memcpy(b + off, &v, 4); }
static void put64(uint8_t* b, uint64_t off, uint64_t v) { memcpy(b + off, &v, 8); }
static uint32_t get32(const uint8_t* b, uint64_t off) {
  uint32_t v;
  memcpy(&v, b + off, 4);
  return v;
}
static uint64_t get64(const uint8_t* b, uint64_t off) {
  uint64_t v;
  memcpy(&v, b + off, 8);
  return v;
}

/* Copy `n` bytes at `cur`, advance, pad the section with zeros to 8. */
static uint64_t put_section(uint8_t* buf, uint64_t cur, const void* src, uint64_t n) {
  if (n) memcpy(buf + cur, src, n);
  const uint64_t end = up8(cur + n);
  memset(buf + cur + n, 0, end - cur - n);
  return end;
}

int orc_tac_serialise(const mvr_tac_parts* p, uint8_t* buf, uint64_t len, uint64_t* written) {
  const uint64_t total = orc_tac_file_size(p);
  if (len < total) return MVR_E_BUFFER_TOO_SMALL;
  memset(buf, 0, MVR_TAC_HEADER_REGION);
  uint64_t cur = MVR_TAC_HEADER_REGION;
  const uint64_t centroids_off = cur;
  cur = put_section(buf, cur, p->centroids, (uint64_t)p->kappa * p->dim * 4);
  const uint64_t hnsw_off = cur;
  { /* writeHnsw */
    buf[cur] = (uint8_t)p->hnsw_max_level;
    memset(buf + cur + 1, 0, 7);
    put32(buf, cur + 8, p->hnsw_entry_point);
    put32(buf, cur + 12, 0);
    put32(buf, cur + 16, p->hnsw_n);
    put32(buf, cur + 20, 0);
    cur = put_section(buf, cur + 24, p->hnsw_node_levels, p->hnsw_n);
    for (uint32_t L = 0; L <= p->hnsw_max_level; ++L) {
      cur = put_section(buf, cur, p->hnsw_layer_offsets[L], ((uint64_t)p->hnsw_n + 1) * 4);
      cur = put_section(buf, cur, p->hnsw_layer_neighbours[L], (uint64_t)p->hnsw_layer_offsets[L][p->hnsw_n] * 4);
    }
  }
  const uint64_t pq_off = cur;
  cur = put_section(buf, cur, p->codebooks, (uint64_t)p->pq_m * 256u * p->sub_dim * 4);
  const uint64_t ilist_off = cur;
  memcpy(buf + cur, p->ilist_offsets, ((uint64_t)p->kappa + 1) * 8);
  cur += ((uint64_t)p->kappa + 1) * 8;
  cur = put_section(buf, cur, p->ilist_payload, p->ilist_offsets[p->kappa] * 4);
  const uint64_t doc_off = cur;
  {
    const uint64_t n = orc_write_doc_layouts(p->doc_offsets, p->n_docs, p->assignments, p->pq_codes, p->pq_m,
                                             buf + cur, len - cur);
    if (n == 0) return MVR_E_BUFFER_TOO_SMALL;
    cur = up8(cur + n);
  }
  const uint64_t doc_tok_off = cur;
  cur = put_section(buf, cur, p->doc_offsets, (p->n_docs + 1) * 8);
  const uint64_t norms_off = cur;
  cur = put_section(buf, cur, p->residual_norms, p->n_tokens * 4);
  const uint64_t footer_off = cur;
  /* Header (storage.zig:52-73), little-endian, then the CRC footer */
  memcpy(buf, "TAC_IDX1", 8);
  put32(buf, 8, MVR_TAC_VERSION);
  put32(buf, 12, p->dim);
  put32(buf, 16, p->kappa);
  put32(buf, 20, p->pq_m);
  buf[24] = 8; /* pq_bits */
  buf[25] = buf[26] = buf[27] = 0;
  put32(buf, 28, p->sub_dim);
  put64(buf, 32, p->n_docs);
  put64(buf, 40, p->n_tokens);
  put64(buf, 48, centroids_off);
  put64(buf, 56, hnsw_off);
  put64(buf, 64, pq_off);
  put64(buf, 72, ilist_off);
  put64(buf, 80, doc_off);
  put64(buf, 88, doc_tok_off);
  put64(buf, 96, norms_off);
  put64(buf, 104, footer_off);
  put32(buf, footer_off, orc_crc32(buf, footer_off));
  put32(buf, footer_off + 4, 0);
  *written = footer_off + 8;
  return *written == total ? MVR_OK : MVR_E_INVALID_INDEX;
}

/* storage.parse with the reader's PQ_M = `reader_pq_m`: header checks,
 * monotone in-bounds offsets, CRC, then each section's size checks in the
 * reference's order. On success `v` holds the header fields and the byte
 * offsets of every array. */
int orc_tac_parse(const uint8_t* b, uint64_t len, uint32_t reader_pq_m, orc_tac_view* v) {
  memset(v, 0, sizeof(*v));
  if (len < MVR_TAC_HEADER_REGION + 8) return MVR_E_INVALID_INDEX;
  if (memcmp(b, "TAC_IDX1", 8) != 0) return MVR_E_INVALID_INDEX;
  v->version = get32(b, 8);
  v->dim = get32(b, 12);
  v->kappa = get32(b, 16);
  v->pq_m = get32(b, 20);
  v->pq_bits = b[24];
  v->sub_dim = get32(b, 28);
  v->n_docs = get64(b, 32);
  v->n_tokens = get64(b, 40);
  uint64_t offs[8];
  for (int i = 0; i < 8; ++i) offs[i] = get64(b, 48 + 8 * (uint64_t)i);
  if (v->version != MVR_TAC_VERSION) return MVR_E_UNSUPPORTED_VERSION;
  if (v->pq_m != reader_pq_m) return MVR_E_INVALID_INDEX;
  if (v->pq_bits != 8) return MVR_E_INVALID_INDEX;
  if ((uint64_t)v->sub_dim * v->pq_m != v->dim) return MVR_E_INVALID_INDEX;
  if (v->dim == 0 || v->kappa == 0) return MVR_E_INVALID_INDEX;
  if (offs[0] != MVR_TAC_HEADER_REGION) return MVR_E_INVALID_INDEX;
  for (int i = 1; i < 8; ++i) {
    if (offs[i] < offs[i - 1]) return MVR_E_INVALID_INDEX;
    if (offs[i] > len) return MVR_E_INVALID_INDEX;
  }
  const uint64_t footer = offs[7];
  if (footer + 8 > len) return MVR_E_INVALID_INDEX;
  if (get32(b, footer) != orc_crc32(b, footer)) return MVR_E_INDEX_CORRUPT;
  v->centroids_off = offs[0];
  if (offs[1] - offs[0] < (uint64_t)v->kappa * v->dim * 4) return MVR_E_INVALID_INDEX;
  { /* parseHnsw */
    const uint64_t s0 = offs[1], s1 = offs[2], slen = s1 - s0;
    if (slen < 24) return MVR_E_INVALID_INDEX;
    v->hnsw_max_level = b[s0];
    v->hnsw_entry_point = get32(b, s0 + 8);
    v->hnsw_n = get32(b, s0 + 16);
    uint64_t cur = 24;
    if (v->hnsw_n == 0) return MVR_E_INVALID_INDEX;
    if (slen < cur + v->hnsw_n) return MVR_E_INVALID_INDEX;
    v->hnsw_levels_off = s0 + cur;
    cur = up8(cur + v->hnsw_n);
    for (uint32_t L = 0; L <= v->hnsw_max_level; ++L) {
      const uint64_t ob = ((uint64_t)v->hnsw_n + 1) * 4;
      if (slen < cur + ob) return MVR_E_INVALID_INDEX;
      v->hnsw_layer_offsets_off[L] = s0 + cur;
      const uint32_t last = get32(b, s0 + cur + (uint64_t)v->hnsw_n * 4);
      cur = up8(cur + ob);
      const uint64_t pb = (uint64_t)last * 4;
      if (slen < cur + pb) return MVR_E_INVALID_INDEX;
      v->hnsw_layer_neighbours_off[L] = s0 + cur;
      v->hnsw_layer_edges[L] = last;
      cur = up8(cur + pb);
    }
  }
  /* parsePq */
  if (offs[3] - offs[2] < (uint64_t)v->pq_m * 256u * v->sub_dim * 4) return MVR_E_INVALID_INDEX;
  v->pq_off = offs[2];
  { /* parseInvertedLists */
    const uint64_t ob = ((uint64_t)v->kappa + 1) * 8;
    if (offs[4] - offs[3] < ob) return MVR_E_INVALID_INDEX;
    v->ilist_offsets_off = offs[3];
    v->ilist_total = get64(b, offs[3] + (uint64_t)v->kappa * 8);
    if (offs[4] - offs[3] < ob + v->ilist_total * 4) return MVR_E_INVALID_INDEX;
    v->ilist_payload_off = offs[3] + ob;
  }
  {
    const uint64_t ib = (v->n_docs + 1) * 8;
    if (offs[5] - offs[4] < ib) return MVR_E_INVALID_INDEX;
    v->doc_index_off = offs[4];
    v->doc_payload_off = offs[4] + ib;
    v->doc_payload_len = offs[5] - offs[4] - ib;
  }
  if (offs[6] - offs[5] < (v->n_docs + 1) * 8) return MVR_E_INVALID_INDEX;
  v->doc_tok_off = offs[5];
  if (offs[7] - offs[6] < v->n_tokens * 4) return MVR_E_INVALID_INDEX;
  v->norms_off = offs[6];
  v->footer_off = footer;
  return MVR_OK;
}
