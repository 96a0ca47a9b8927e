/*
 * mvr_oracle.h — CPU restatement of the reference build path, used ONLY as
 * the parity checker in tests/, in __graft_entry__.smoke() and as the timed
 * CPU baseline in bench.py. Nothing in the product links or calls it.
 *
 * Every function follows a reference function (BleedingDev/
 * ir-multivector-retrieval, Zig), cited as path:line beside its body in
 * mvr_oracle.c. Status codes are the MVR_* values of include/mvr.h.
 */
#ifndef MVR_ORACLE_H
#define MVR_ORACLE_H

#include <stdint.h>

/* status codes and the shared parts struct of the .tac image (types only:
 * the oracle links nothing of the product) */
#include "../include/mvr.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Order of the final 4-lane `@reduce(.Add)` in vec.l2sq for len 64/128.
 * 0: ((a0+a1)+a2)+a3 (LLVM ordered reduction, the strict-mode lowering);
 * 1: (a0+a1)+(a2+a3) (tree). Default 0. */
void orc_set_reduce_tree(int tree);
/* Lane count of vec.l2sqGeneric (`std.simd.suggestVectorLength(f32)`,
 * 4 on the reference's Apple NEON hosts). Default 4. */
void orc_set_lane_count(int lanes);
/* Worker threads of orc_tac_cluster_flat (tokens in parallel; results are
 * the same bytes for any count; 1 = the serial loop). Test speed only. */
void orc_set_workers(int n);

float orc_l2sq(const float* a, const float* b, uint32_t len);
int64_t orc_argmin(const float* v, uint64_t n);
int64_t orc_argmax(const float* v, uint64_t n);

typedef struct orc_rng {
  uint64_t s[4];
} orc_rng;
void orc_rng_init(orc_rng* r, uint64_t seed);
uint64_t orc_rng_next(orc_rng* r);
uint64_t orc_rng_index(orc_rng* r, uint64_t n);
double orc_rng_f64(orc_rng* r);
float orc_rng_f32(orc_rng* r);
int orc_weighted_sample(orc_rng* r, const float* w, uint64_t n, uint64_t* out);

int orc_kmeans_fit(const float* vectors, uint64_t vectors_len, uint32_t dim,
                   uint32_t k, uint32_t max_iters, float tol, uint64_t seed,
                   uint32_t n_threads, float* centroids, uint32_t* assignments,
                   float* wcss, uint32_t* iters_run, uint32_t* trace);

int orc_pq_train(const float* residuals, uint64_t residuals_len, uint32_t dim,
                 uint64_t seed, uint32_t n_threads, uint32_t pq_m,
                 uint32_t max_iters, float tol, float* codebooks);
int orc_pq_encode(const float* codebooks, uint32_t dim, uint32_t pq_m,
                  const float* residuals, uint64_t n, uint8_t* codes,
                  uint32_t n_threads);
/* Timing helper for the CPU baseline: `iters` Lloyd iterations of every
 * subspace starting from the given codebooks (no seeding), subspaces spread
 * over n_threads like pq.train's work-stealing loop. */
int orc_pq_lloyd_iters(const float* residuals, uint64_t n, uint32_t dim,
                       uint32_t pq_m, uint32_t iters, uint32_t n_threads,
                       float* codebooks_inout);

int orc_residuals_norms(const float* vectors, const float* centroids,
                        const uint32_t* assignments, uint64_t n, uint32_t dim,
                        float* residuals, float* norms);

int orc_tac_allocate_tail(const uint32_t* freqs, uint32_t* kappa, uint64_t n,
                          uint32_t mu, uint32_t tau, uint32_t kappa_total,
                          uint32_t* budget_out);
int orc_tac_damped_phase2(const uint32_t* freqs, const float* spreads,
                          uint32_t* kappa, float* frac, uint64_t n,
                          uint32_t budget_active, uint32_t mu, uint32_t tau);
int orc_tac_bound_phase3(const uint32_t* freqs, uint32_t* kappa, uint64_t n,
                         uint32_t mu, uint32_t tau, uint32_t epsilon,
                         uint32_t theta);
int orc_tac_reconcile_phase4(const uint32_t* freqs, uint32_t* kappa,
                             const float* frac, uint64_t n,
                             uint32_t kappa_total, uint32_t mu, uint32_t tau,
                             uint32_t epsilon, uint32_t theta);
int orc_tac_allocate_budgets(const uint32_t* freqs, const float* spreads,
                             uint32_t* kappa, float* frac, uint64_t n,
                             uint32_t kappa_total, uint32_t mu, uint32_t tau,
                             uint32_t epsilon, uint32_t theta);
int orc_tac_spreads(const uint32_t* token_ids, uint64_t n_tokens,
                    const float* vectors, uint32_t dim, uint64_t n_distinct,
                    uint32_t* freqs_out, float* spreads_out);
int orc_tac_cluster_flat(const uint32_t* token_ids, uint64_t n_tokens,
                         const float* vectors, uint64_t vectors_len,
                         uint32_t dim, uint32_t kappa_total, uint32_t mu,
                         uint32_t tau, uint32_t epsilon, uint32_t theta,
                         uint32_t max_iters, float tol, uint64_t seed,
                         uint32_t n_threads, float* centroids,
                         uint32_t* assignments, uint32_t* kappa_per_token,
                         uint64_t kappa_cap, uint64_t* n_distinct_out,
                         float* wcss_total);

/* storage.writeDocLayouts (src/index/storage.zig:705-749): doc index
 * (n_docs + 1 u64 payload offsets) + per doc [n_d u32 | assignments u32 |
 * codes u8 * n_d * pq_m | zero pad to 8]. Returns the bytes written, or 0
 * when `out_len` is too small (BufferTooSmall). */
uint64_t orc_write_doc_layouts(const uint64_t* doc_offsets, uint64_t n_docs,
                               const uint32_t* assignments, const uint8_t* codes,
                               uint32_t pq_m, uint8_t* out, uint64_t out_len);
/* vec.dot (src/util/vec.zig:37-103): len 2 `a0*b0 + a1*b1`; len 4 left
 * fold from +0; len 64/128 four lane accumulators from +0, then the
 * ordered reduce; other lengths the lane-count loop plus the tail. */
float orc_dot(const float* a, const float* b, uint32_t len);

/* PQ.buildDistanceTable (src/index/pq.zig:92-123): out[(m*256+c)*n_q+i] =
 * dot(q_i[m*s .. m*s+s], codebook[m][c]). Returns MVR status. */
int orc_pq_distance_table(const float* codebooks, uint32_t dim, uint32_t pq_m,
                          const float* query, uint64_t query_len, uint32_t n_q,
                          float* out, uint64_t out_len);

/* refine.refine (src/retrieval/refine.zig:83-155) for one candidate doc:
 * `doc_section` is the writeDocLayouts section (index + payload). */
int orc_refine(const float* centroids, uint32_t dim, uint32_t pq_m,
               const uint8_t* doc_section, uint64_t n_docs,
               const uint64_t* doc_token_offsets, const float* residual_norms,
               const float* table, uint64_t table_len, const float* query,
               uint64_t query_len, uint32_t n_q, uint32_t doc_id, float* score);


/* ---- HNSW over the centroids (src/index/hnsw.zig), hnsw_oracle.c ---- */
typedef struct orc_hnsw orc_hnsw;
typedef struct orc_hnsw_stats {
  uint64_t searches, expansions, sims, accepted, heur_examined, heur_dots;
} orc_hnsw_stats;
/* hnsw.build: n_threads <= 1 the serial path, >= 2 the chunked
 * deferred-commit path (identical for every count >= 2); `workers` host
 * threads plan each chunk (any count gives the same graph). */
int orc_hnsw_build(const float* centroids, uint64_t n_floats, uint32_t dim, uint64_t seed, uint32_t ef_c,
                   uint32_t m, uint32_t n_threads, uint32_t workers, orc_hnsw** out);
void orc_hnsw_free(orc_hnsw* h);
void orc_hnsw_info(const orc_hnsw* h, uint32_t* n, uint32_t* entry_point, uint32_t* max_level);
void orc_hnsw_levels(const orc_hnsw* h, uint8_t* out);
uint64_t orc_hnsw_layer_size(const orc_hnsw* h, uint32_t L);
void orc_hnsw_layer(const orc_hnsw* h, uint32_t L, uint32_t* offsets, uint32_t* nbrs);
void orc_hnsw_last_stats(orc_hnsw_stats* out);
/* hnsw.search over a frozen per-layer CSR graph */
int orc_hnsw_search_csr(const float* centroids, uint32_t n, uint32_t dim, uint32_t entry_point, uint32_t max_level,
                        const uint32_t* const* offsets, const uint32_t* const* nbrs, const float* query,
                        uint32_t k, uint32_t ef, uint32_t* out, uint32_t* written);
int orc_hnsw_search(const orc_hnsw* h, const float* query, uint32_t k, uint32_t ef, uint32_t* out,
                    uint32_t* written);
/* vec.normalizeRowsInPlace */
void orc_normalize_rows(float* v, uint64_t n_rows, uint32_t dim);


/* ---- .tac image and inverted lists (tac_file_oracle.c) ---- */
uint32_t orc_crc32(const uint8_t* p, uint64_t len);
int orc_inverted_lists_build(const uint32_t* assignments, uint64_t n_assign, const uint64_t* doc_offsets,
                             uint64_t doc_offsets_len, uint32_t kappa, uint64_t* offsets, uint32_t* payload,
                             uint64_t payload_cap, uint64_t* total_out);
uint64_t orc_tac_file_size(const mvr_tac_parts* p);
int orc_tac_serialise(const mvr_tac_parts* p, uint8_t* buf, uint64_t len, uint64_t* written);

/* What orc_tac_parse finds: header fields and the byte offset of every
 * array in the image (HNSW: up to max_level + 1 <= 256 layers). */
typedef struct orc_tac_view {
  uint32_t version, dim, kappa, pq_m, pq_bits, sub_dim;
  uint64_t n_docs, n_tokens;
  uint64_t centroids_off;
  uint32_t hnsw_n, hnsw_entry_point, hnsw_max_level;
  uint64_t hnsw_levels_off;
  uint64_t hnsw_layer_offsets_off[256], hnsw_layer_neighbours_off[256], hnsw_layer_edges[256];
  uint64_t pq_off;
  uint64_t ilist_offsets_off, ilist_payload_off, ilist_total;
  uint64_t doc_index_off, doc_payload_off, doc_payload_len;
  uint64_t doc_tok_off, norms_off, footer_off;
} orc_tac_view;
int orc_tac_parse(const uint8_t* b, uint64_t len, uint32_t reader_pq_m, orc_tac_view* v);

#ifdef __cplusplus
}
#endif
#endif
