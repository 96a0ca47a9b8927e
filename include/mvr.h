/*
 * mvr.h — C ABI of the B200 build path for the TAC multivector index:
 * PQ codebook training, PQ encoding, the shared k-means primitive and
 * TAC per-token clustering.
 *
 * Every entry point replaces one function of the reference Zig build path
 * (BleedingDev/ir-multivector-retrieval). The citation beside each
 * declaration names the reference function it stands in for, as
 * `path:line` inside that project. A Zig host binds these symbols with
 * `@cImport(@cInclude("mvr.h"))` and keeps its own signatures.
 *
 * Conventions
 *   - Plain pointers and sizes only. Host-pointer entry points copy inputs
 *     to the GPU and results back; `*_device` entry points take device
 *     pointers and run on the context's stream.
 *   - Caller-allocated outputs. The library owns only its device scratch,
 *     which lives in the opaque `mvr_ctx`.
 *   - Every entry point returns an `int` status. `MVR_OK` is 0; the other
 *     codes map one-to-one onto the reference's Zig error names (listed
 *     beside each code). `mvr_last_error(ctx)` gives the message of the last
 *     failing call on that context.
 *   - Validation order follows the reference, so the same bad input yields
 *     the same error name.
 *   - Calls on one context are serialised by the caller (the reference's
 *     callers are single-threaded at these call sites).
 *   - `n_threads` arguments are accepted for signature parity. They change
 *     nothing on the GPU except the WCSS summation order that
 *     `tac.clusterFlat` reports, which the reference defines per thread count.
 *   - Lloyd stopping rule: the reference's `rel_delta < tol` test. Pass
 *     `tol = -INFINITY` to run exactly `max_iters` iterations.
 */
#ifndef MVR_H
#define MVR_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
enum {
  MVR_OK = 0,
  MVR_E_KMEANS_BUDGET_TOO_SMALL = 1, /* kmeans.KMeansError.KmeansBudgetTooSmall */
  MVR_E_EMPTY_VECTOR_SET = 2,        /* kmeans.KMeansError.EmptyVectorSet */
  MVR_E_DIM_MISMATCH = 3,            /* kmeans/pq DimMismatch */
  MVR_E_DIM_NOT_DIVISIBLE_BY_M = 4,  /* pq.PqError.DimNotDivisibleByM */
  MVR_E_EMPTY_CORPUS = 5,            /* pq.PqError.EmptyCorpus */
  MVR_E_OUT_BUFFER_WRONG_SIZE = 6,   /* pq.PqError.OutBufferWrongSize */
  MVR_E_NQ_MISMATCH = 7,             /* pq.PqError.NQMismatch */
  MVR_E_EMPTY_DISTRIBUTION = 8,      /* rng.RngError.EmptyDistribution */
  MVR_E_NON_FINITE = 9,              /* rng.RngError.NonFinite */
  MVR_E_ALL_ZERO = 10,               /* rng.RngError.AllZero */
  MVR_E_BUDGET_TOO_SMALL = 11,       /* tac.ClusteringError.BudgetTooSmall */
  MVR_E_BUDGET_TOO_LARGE = 12,       /* tac.ClusteringError.BudgetTooLarge */
  MVR_E_INVALID_THRESHOLDS = 13,     /* tac.ClusteringError.InvalidThresholds */
  MVR_E_EMPTY_TOKEN_DUMP = 14,       /* tac.ClusteringError.EmptyTokenDump */
  MVR_E_LENGTH_MISMATCH = 15,        /* vec.VecError.LengthMismatch */
  MVR_E_EMPTY_INPUT = 16,            /* vec.VecError.EmptyInput */
  MVR_E_OUT_OF_MEMORY = 17,          /* Allocator.Error.OutOfMemory (host or device) */
  MVR_E_BUFFER_TOO_SMALL = 18,       /* storage.StorageError.BufferTooSmall */
  MVR_E_QUERY_SHAPE_MISMATCH = 19,   /* refine.RefineError.QueryShapeMismatch */
  MVR_E_TABLE_SIZE_MISMATCH = 20,    /* refine.RefineError.TableSizeMismatch */
  MVR_E_DOC_OUT_OF_RANGE = 21,       /* refine.RefineError.DocOutOfRange */
  MVR_E_DOC_LAYOUT_CORRUPT = 22,     /* refine.RefineError.DocLayoutCorrupt */
  MVR_E_INVALID_INDEX = 23,          /* storage.StorageError.InvalidIndex */
  MVR_E_UNSUPPORTED_VERSION = 24,    /* storage.StorageError.UnsupportedVersion */
  MVR_E_INDEX_CORRUPT = 25,          /* storage.StorageError.IndexCorrupt */
  MVR_E_ASSIGNMENT_OUT_OF_RANGE = 26, /* inverted_list.InvertedListError.AssignmentOutOfRange */
  MVR_E_DOC_OFFSETS_BAD = 27,        /* inverted_list.InvertedListError.DocOffsetsBad */
  MVR_E_KAPPA_ZERO = 28,             /* inverted_list.InvertedListError.KappaZero */
  /* B200-side failures with no reference counterpart */
  MVR_E_CUDA = 100,             /* a CUDA runtime call failed */
  MVR_E_NCCL = 101,             /* an NCCL call failed */
  MVR_E_TIMEOUT = 102,          /* a bounded device wait ran out */
  MVR_E_INVALID_ARGUMENT = 103, /* null pointer, unsupported shape */
  MVR_E_NO_DEVICE = 104,        /* no CUDA device with sm_100 */
  MVR_E_DEVICE_LIMIT = 105      /* a device-side capacity was exceeded; nothing returned */
};

/* Number of centroids per PQ subspace (reference constants.PQ_CENTROIDS). */
#define MVR_PQ_CENTROIDS 256u

typedef struct mvr_ctx mvr_ctx;

/* ---- context ----------------------------------------------------------- */

/* Create a context bound to CUDA device `device_ordinal`. The context owns a
 * stream and grows device scratch on demand. No reference counterpart: the
 * Zig build keeps all state in `gpa`-allocated slices. */
int mvr_ctx_create(int device_ordinal, mvr_ctx** out);

/* Free the context and all its device scratch. */
int mvr_ctx_destroy(mvr_ctx* ctx);

/* Message of the last failing call on `ctx` ("" if none). */
const char* mvr_last_error(const mvr_ctx* ctx);

/* Zig error name of a status code, e.g. "DimNotDivisibleByM". */
const char* mvr_status_name(int status);

/* Use an existing CUDA stream (a `cudaStream_t`) for the `*_device` entry
 * points. NULL restores the context's own stream. */
int mvr_ctx_set_stream(mvr_ctx* ctx, void* cuda_stream);

/* Release device scratch held by the context (it is regrown on demand). */
int mvr_ctx_trim(mvr_ctx* ctx);

/* ---- kmeans.fit -------------------------------------------------------- */

/* Replaces `kmeans.fit(vectors, dim, KMeansParams{k, max_iters, tol, seed,
 * n_threads}, gpa)` (src/tac/kmeans.zig:67-72; params :28-41; result
 * :43-54). `vectors` holds `vectors_len` floats, row-major, n =
 * vectors_len / dim rows. Outputs: centroids k*dim floats, assignments n
 * u32, wcss and iters_run scalars (any output pointer may be NULL except
 * `centroids_out`). k-means++ seeding, Lloyd iterations with the reference's
 * serial in-order centroid sums, empty-cluster reseed and relative-WCSS
 * stopping, bit-exact with the reference arithmetic. */
int mvr_kmeans_fit(mvr_ctx* ctx, const float* vectors, uint64_t vectors_len,
                   uint32_t dim, uint32_t k, uint32_t max_iters, float tol,
                   uint64_t seed, uint32_t n_threads, float* centroids_out,
                   uint32_t* assignments_out, float* wcss_out,
                   uint32_t* iters_run_out);

/* ---- kmeans.fit without device allocation ------------------------------- */

/* Largest row count and the size of the fixed device scratch of
 * `mvr_kmeans_fit_noalloc`. */
#define MVR_NOALLOC_MAX_ROWS 65536u
#define MVR_NOALLOC_SCRATCH_BYTES (4096u * 1024u)

/* No counterpart in the reference: an extra entry point for hosts that
 * cannot let a library allocate GPU memory (their own allocator owns the
 * device, their memory budget is fixed up front, or cudaMalloc's implicit
 * synchronisation is not acceptable on their path). Same result as
 * `mvr_kmeans_fit` (bit for bit), but
 *   - inputs and outputs are device pointers: `d_vectors` (vectors_len
 *     floats), `d_centroids_out` (k*dim floats), `d_assignments_out`
 *     (n u32, may be NULL); `wcss_out` / `iters_run_out` are host pointers
 *     and may be NULL;
 *   - work runs on `cuda_stream` (NULL = the legacy default stream) of the
 *     current device, and the call returns when the result is ready;
 *   - no context: it calls no cudaMalloc, cudaFree or other allocating
 *     routine. All scratch lives in one fixed device array of
 *     MVR_NOALLOC_SCRATCH_BYTES compiled into the library, which every GPU
 *     that loads the library keeps until the process exits;
 *   - limits: dim in {1, 2, 4}, k <= 256, n <= MVR_NOALLOC_MAX_ROWS rows;
 *     larger inputs return MVR_E_INVALID_ARGUMENT before any GPU work.
 * The first call on a device looks up the array's device address (with that
 * device current); make that first call before any stream capture on the
 * device. The address belongs to the device's CUDA context: a call made
 * under another context (after cudaDeviceReset, or with a context made
 * current through the driver API) looks it up again. Devices other than
 * sm_100 return MVR_E_NO_DEVICE. All calls share the one array, so calls that
 * overlap on the GPU (other streams, other threads) race: serialise them.
 * The array keeps the last call's contents; the call initialises everything
 * it reads. */
int mvr_kmeans_fit_noalloc(const float* d_vectors, uint64_t vectors_len,
                           uint32_t dim, uint32_t k, uint32_t max_iters,
                           float tol, uint64_t seed, float* d_centroids_out,
                           uint32_t* d_assignments_out, float* wcss_out,
                           uint32_t* iters_run_out, void* cuda_stream);

/* ---- pq.train / PQ.encode ---------------------------------------------- */

/* Per-call timing and iteration report of `mvr_pq_train*` (no reference
 * counterpart; the reference prints `[stage]` lines instead,
 * src/index/storage.zig:382). Times are device times in milliseconds. */
typedef struct mvr_pq_train_stats {
  double seed_ms;        /* k-means++ seeding, all subspaces */
  double lloyd_ms;       /* Lloyd iterations, all subspaces */
  double total_ms;       /* whole call on the device */
  uint32_t iters_max;    /* largest iters_run over subspaces */
  uint32_t iters_min;    /* smallest iters_run over subspaces */
  uint32_t seed_fallbacks; /* k-means++ draws resolved by the exact serial chain */
  uint32_t reseeds;      /* empty-cluster reseeds, summed over iterations */
  double assign_ms;      /* summed device time of the Lloyd assignment kernel */
  uint32_t assign_launches; /* launches of that kernel */
  uint32_t launches;     /* all kernel launches of the call */
  double assign_first_ms;   /* the first Lloyd assignment (every distance computed) */
  uint64_t lloyd_rows_total; /* (row, subspace) assignments over all Lloyd iterations */
  uint64_t lloyd_rows_exact; /* of those, the ones whose K distances were all computed
                                (the rest kept their cluster by exact bounds) */
  uint64_t filter_rows_rechecked; /* tensor-core filter: rows whose near-ties were
                                     settled by exact distances */
  uint32_t filter_violations;     /* winners outside the filter's error bound (then the
                                     training ran again with exact scans); 0 expected */
  double seed_update_ms_sampled;  /* summed device time of every 8th k-means++ update
                                     launch (steps >= 1) */
  uint32_t seed_update_samples;   /* launches in that sum */
  double list_ms;                 /* summed device time of the pruned Lloyd passes
                                     (iterations >= 1: bound checks and the distance
                                     scans of the rows the bounds did not settle) */
  uint32_t list_launches;         /* pruned passes timed in list_ms */
  uint64_t list_distances;        /* exact (row, centroid) distances those passes
                                     computed */
  uint32_t groups;                /* subspace groups trained side by side on two
                                     streams (1 or 2): each k-means++ update and
                                     each pruned-pass launch covers pq_m / groups
                                     subspaces */
  double host_enqueue_ms;         /* host time spent issuing the work (the longest
                                     group), against total_ms on the device */
} mvr_pq_train_stats;

/* Replaces `pq.train(residuals, dim, seed, n_threads, gpa)`
 * (src/index/pq.zig:158-164, per subspace `trainOneSubspace` :301-336).
 * `pq_m` is the number of subspaces (the reference's comptime PQ_M; 32 in the
 * stock build, 16 in the M=16x4 configuration). Each subspace runs
 * kmeans.fit(k=256, max_iters, tol, seed +% m). The reference hard-codes
 * max_iters=25, tol=1e-4 (pq.zig:319-325). Output: pq_m*256*(dim/pq_m)
 * floats laid out codebook[m][c][k] (pq.zig:14-15). `stats` may be NULL. */
int mvr_pq_train(mvr_ctx* ctx, const float* residuals, uint64_t residuals_len,
                 uint32_t dim, uint64_t seed, uint32_t n_threads, uint32_t pq_m,
                 uint32_t max_iters, float tol, float* codebooks_out,
                 mvr_pq_train_stats* stats);

/* As `mvr_pq_train`, with `d_residuals` and `d_codebooks_out` in device
 * memory. Runs on the context's stream and returns when the result is
 * ready. */
int mvr_pq_train_device(mvr_ctx* ctx, const float* d_residuals,
                        uint64_t residuals_len, uint32_t dim, uint64_t seed,
                        uint32_t n_threads, uint32_t pq_m, uint32_t max_iters,
                        float tol, float* d_codebooks_out,
                        mvr_pq_train_stats* stats);

/* Replaces the encode loop `storage.parallelTokenLoop(pqEncodeChunk)`
 * (src/index/storage.zig:287-295, :389-400), i.e. `PQ.encode` per row
 * (src/index/pq.zig:59-76): for each of the n rows and each subspace m, the
 * first codeword of minimum exact squared L2 distance. `codebooks` is
 * pq_m*256*(dim/pq_m) floats, `residuals` n*dim floats, `codes_out` n*pq_m
 * bytes. Page-locked `residuals` of 524,288 rows or more are copied in chunks
 * that overlap the encoding of the chunks already on the device. */
int mvr_pq_encode(mvr_ctx* ctx, const float* codebooks, uint32_t dim,
                  uint32_t pq_m, const float* residuals, uint64_t n,
                  uint8_t* codes_out);

/* As `mvr_pq_encode`, all pointers in device memory; asynchronous on the
 * context's stream (call `mvr_ctx_sync` before reading the codes). */
int mvr_pq_encode_device(mvr_ctx* ctx, const float* d_codebooks, uint32_t dim,
                         uint32_t pq_m, const float* d_residuals, uint64_t n,
                         uint8_t* d_codes_out);

/* ---- several GPUs (one process per GPU) ------------------------------- */

/* No counterpart in the reference (its pq.train runs on one host). An NCCL
 * unique id (`mvr_comm_unique_id_bytes()` bytes) made by one process and
 * handed to every rank by the caller (e.g. over torch.distributed), then
 * `mvr_ctx_init_comm` on every rank joins its context to the communicator.
 * NCCL is loaded at run time; MVR_E_NCCL when it is missing. */
size_t mvr_comm_unique_id_bytes(void);
int mvr_comm_unique_id(void* id_out, size_t id_bytes);
int mvr_ctx_init_comm(mvr_ctx* ctx, int nranks, int rank, const void* id,
                      size_t id_bytes);
int mvr_ctx_comm_size(const mvr_ctx* ctx);
int mvr_ctx_comm_rank(const mvr_ctx* ctx);

/* Row-sharded `pq.train` (src/index/pq.zig:158-291) over the context's
 * communicator: this rank holds rows [row0, row0 + n_local) of an n_total x
 * dim matrix in device memory; the shards are non-empty and contiguous in
 * rank order. Collective: every rank calls it with the same dim, seed,
 * pq_m, max_iters and tol. Every rank receives the codebooks that
 * `mvr_pq_train` computes on the whole matrix (identical bytes for any
 * number of ranks); `d_assign_out` (optional, pq_m*n_local u32, [m][row])
 * receives this rank's final assignments. Without a communicator the shard
 * must be the whole matrix. With pq_m >= ranks each rank trains a range of
 * whole subspaces over all rows (their columns are exchanged once before and
 * the codebooks gathered after); with fewer subspaces than ranks the rows
 * stay split and every k-means++ draw and Lloyd iteration exchanges bounds,
 * counts and running sums. Returns when the result is ready. */
int mvr_pq_train_sharded_device(mvr_ctx* ctx, const float* d_rows,
                                uint64_t n_local, uint64_t row0,
                                uint64_t n_total, uint32_t dim, uint64_t seed,
                                uint32_t n_threads, uint32_t pq_m,
                                uint32_t max_iters, float tol,
                                float* d_codebooks_out, uint32_t* d_assign_out,
                                mvr_pq_train_stats* stats);

/* ---- .tac per-doc payload (storage.zig:705-749) -------------------------- */

/* Bytes of the per-doc section of a .tac file: the doc index
 * ((n_docs + 1) u64 payload offsets) followed by, per doc d with
 * n_d = doc_offsets[d+1] - doc_offsets[d] tokens,
 * [n_d u32 | n_d assignment u32 | n_d * pq_m code bytes | zero pad to 8]
 * (storage.zig:506-508, docPayloadSize). `doc_offsets` is host memory. */
int mvr_doc_layouts_bytes(const uint64_t* doc_offsets, uint64_t n_docs,
                          uint32_t pq_m, uint64_t* bytes_out);

/* Replaces storage.writeDocLayouts (src/index/storage.zig:705-749): writes
 * the section above into `out` (out_len bytes; BufferTooSmall when short).
 * `doc_offsets` (n_docs + 1 u64, non-decreasing, last = n_tokens) is host
 * memory; `assignments` (n_tokens u32, TAC centroid ids), `codes`
 * (n_tokens * pq_m bytes, token-major) and `out` are host memory here and
 * device memory in the _device variant (asynchronous on the context
 * stream; `d_out` 8-byte and `d_assignments` 4-byte aligned). The bytes
 * are identical to the reference's. */
int mvr_write_doc_layouts(mvr_ctx* ctx, const uint64_t* doc_offsets,
                          uint64_t n_docs, const uint32_t* assignments,
                          const uint8_t* codes, uint64_t n_tokens,
                          uint32_t pq_m, uint8_t* out, uint64_t out_len);
int mvr_write_doc_layouts_device(mvr_ctx* ctx, const uint64_t* doc_offsets,
                                 uint64_t n_docs, const uint32_t* d_assignments,
                                 const uint8_t* d_codes, uint64_t n_tokens,
                                 uint32_t pq_m, uint8_t* d_out,
                                 uint64_t out_len);

/* CRC-32 of the .tac footer (std.hash.Crc32: reflected polynomial
 * 0xEDB88320, initial and final xor 0xFFFFFFFF, as zlib's crc32), over
 * host memory; `crc` continues a previous value (0 to start). */
uint32_t mvr_crc32(uint32_t crc, const void* data, uint64_t len);

/* CRC-32 of A || B from crc(A), crc(B) and the length of B (the GF(2)
 * combination zlib calls crc32_combine); the footer checksum of
 * mvr_tac_serialise is computed in chunks on host threads and joined this
 * way. No reference counterpart. */
uint32_t mvr_crc32_combine(uint32_t crc1, uint32_t crc2, uint64_t len2);

/* ---- query side: PQ distance table and refine ------------------------- */

/* Replaces PQ.buildDistanceTable (src/index/pq.zig:92-123): out[(m*256 + c)
 * * n_q + i] = vec.dot(q_i[m*s .. m*s + s], codebook[m][c]) for the n_q
 * query tokens (query: n_q * dim floats), out: pq_m * 256 * n_q floats.
 * NQMismatch / OutBufferWrongSize as the reference. Host pointers here,
 * device pointers (asynchronous) in the _device variant. */
int mvr_pq_distance_table(mvr_ctx* ctx, const float* codebooks, uint32_t dim,
                          uint32_t pq_m, const float* query, uint64_t query_len,
                          uint32_t n_q, float* out, uint64_t out_len);
int mvr_pq_distance_table_device(mvr_ctx* ctx, const float* d_codebooks,
                                 uint32_t dim, uint32_t pq_m,
                                 const float* d_query, uint64_t query_len,
                                 uint32_t n_q, float* d_out, uint64_t out_len);

/* Replaces refine.refine (src/retrieval/refine.zig:83-155) for n_cand
 * candidate docs of one query: scores_out[c] = the exact MaxSim estimate
 * S(q, doc_ids[c]) from the TAC centroids (kappa x dim), the per-doc
 * section of mvr_write_doc_layouts (doc_section_len bytes, n_docs docs),
 * the doc token offsets (n_docs + 1), the residual norms (n_tokens), the
 * distance table and the query (n_q <= 128 tokens). The first failing
 * candidate's status is returned (QueryShapeMismatch, TableSizeMismatch,
 * DocOutOfRange, DocLayoutCorrupt; a centroid id >= kappa counts as a
 * corrupt layout instead of reading past the centroids). Host pointers. */
int mvr_refine_batch(mvr_ctx* ctx, const float* centroids, uint32_t kappa,
                     uint32_t dim, uint32_t pq_m, const uint8_t* doc_section,
                     uint64_t doc_section_len, uint64_t n_docs,
                     const uint64_t* doc_token_offsets,
                     const float* residual_norms, uint64_t n_tokens,
                     const float* table, uint64_t table_len, const float* query,
                     uint64_t query_len, uint32_t n_q, const uint32_t* doc_ids,
                     uint64_t n_cand, float* scores_out);
/* As mvr_refine_batch with every array in device memory (the index stays
 * resident across queries; `d_doc_section` 8-byte aligned) and a per-
 * candidate status array instead of a returned first failure;
 * asynchronous on the context stream. */
int mvr_refine_batch_device(mvr_ctx* ctx, const float* d_centroids,
                            uint32_t kappa, uint32_t dim, uint32_t pq_m,
                            const uint8_t* d_doc_section, uint64_t doc_section_len,
                            uint64_t n_docs, const uint64_t* d_doc_token_offsets,
                            const float* d_residual_norms, uint64_t n_tokens,
                            const float* d_table, uint64_t table_len,
                            const float* d_query, uint64_t query_len,
                            uint32_t n_q, const uint32_t* d_doc_ids,
                            uint64_t n_cand, float* d_scores, int* d_status);

/* Timing report of the most recent `mvr_tac_cluster_flat` call on the
 * context (no reference counterpart; the reference prints `[stage]` lines,
 * src/tac/tac.zig:660-680). Device times come from CUDA events on the
 * context's stream, wall times from the host clock; milliseconds. */
typedef struct mvr_tac_stats {
  double total_ms;   /* wall time of the whole call */
  double host_ms;    /* wall time of the host-side grouping and budgets */
  double h2d_ms;     /* device: host->device copies of the inputs */
  double spread_ms;  /* device: row gather, group-major copy, spreads */
  double seed_ms;    /* device: k-means++ seeding of every token */
  double lloyd_ms;   /* device: Lloyd iterations of every token */
  double d2h_ms;     /* device: assignments and centroids back to the host */
  uint32_t problems; /* tokens clustered (k_j > 0) */
  uint32_t iters_max; /* largest iters_run over tokens */
  uint32_t seed_fallbacks; /* k-means++ draws resolved by the exact serial chain */
  uint32_t launches; /* kernel launches of the call */
  uint64_t filter_rows_rechecked; /* tensor-core filter: row assignments with several
                                     candidates settled by exact distances */
  uint32_t filter_violations;     /* winners outside the filter's bound (then the per-token
                                     k-means ran again with exact scans); 0 expected */
  uint64_t filter_rows_full_scan; /* row assignments whose candidate list overflowed and
                                     took the exact scan over all centroids */
} mvr_tac_stats;

/* Copies the report of the context's most recent `mvr_tac_cluster_flat`
 * call (all zero before the first call). */
int mvr_tac_last_stats(const mvr_ctx* ctx, mvr_tac_stats* out);

/* Verification mode (no reference counterpart): with `on` != 0 every
 * k-means++ draw of the context is resolved by the reference's serial f64
 * chain (rng.zig:57-82) instead of the interval-bounded parallel search.
 * Results are identical either way; only the speed differs. */
int mvr_ctx_set_serial_draws(mvr_ctx* ctx, int on);

/* Verification mode (no reference counterpart): with `on` != 0 every Lloyd
 * assignment of pq.train computes all K distances of every row instead of
 * skipping rows whose exact distance bounds prove their cluster unchanged.
 * Results are identical either way; only the speed differs. */
int mvr_ctx_set_exhaustive_assign(mvr_ctx* ctx, int on);

/* Verification mode (no reference counterpart): with `on` == 0 the pruned
 * Lloyd passes of pq.train scan all K centroids of every row whose bounds
 * fail; by default (`on` != 0) such a row scans only the centroids whose
 * distance from its current centroid is within twice its distance bound
 * (the rest provably cannot win). Results are identical either way. */
int mvr_ctx_set_candidate_scan(mvr_ctx* ctx, int on);

/* Tuning switch (no reference counterpart): pq.train runs its subspaces in
 * `groups` groups side by side, each on its own stream (1 or 2; default 2,
 * used when there are two or more subspaces). Results are identical either
 * way. */
int mvr_ctx_set_pq_groups(mvr_ctx* ctx, int groups);

/* Verification mode (no reference counterpart): with `on` == 0 the Lloyd
 * and encode assignments skip the tensor-core filter (a TF32 MMA chain that
 * approximates every distance within an error bound, after which only the
 * near-ties get exact distances) and scan every centroid with the exact
 * f32 arithmetic. Results are identical either way; on is the default, and
 * it applies to the 64-dim k-means of tac.clusterFlat. */
int mvr_ctx_set_tensor_filter(mvr_ctx* ctx, int on);

/* The tensor-core filter for pq.train's first Lloyd pass and PQ.encode
 * too (`on` != 0; needs mvr_ctx_set_tensor_filter on as well). Off by
 * default: for 4-float sub-vectors the exact f32 scans measured as fast as
 * the filter (whose accumulator read-out costs about as much as the exact
 * distance). No reference counterpart; results are identical either way. */
int mvr_ctx_set_pq_tensor_filter(mvr_ctx* ctx, int on);

/* Counters of the filtered encode passes on this context since it was
 * created: winners whose approximation fell outside the filter's error
 * bound (0 expected; the host-pointer encode then re-runs exactly) and rows
 * whose near-ties were settled by exact distances. Synchronises the
 * context's stream; MVR_E_TIMEOUT if an MMA did not complete. */
int mvr_ctx_filter_report(mvr_ctx* ctx, uint64_t* violations, uint64_t* rows_rechecked);

/* Polls of a bounded device wait before it gives up: the stage waits of the
 * clusterFlat spread kernel's bulk-copy ring. No reference counterpart; for
 * tests of the expiry path. `polls` = 0 gives up at the first wait (the call
 * then returns MVR_E_TIMEOUT after the kernel has waited, with the default
 * limit, for its copies still in flight); MVR_WAIT_LIMIT_DEFAULT restores
 * the normal limit. */
#define MVR_WAIT_LIMIT_DEFAULT 4194304u
int mvr_ctx_set_wait_limit(mvr_ctx* ctx, uint32_t polls);

/* Measured FP32 issue rate of the context's GPU, in lane operations per
 * second: independent chains of packed f32x2 adds and multiplies (the
 * instructions of the exact distance kernels) on every SM, best of two runs
 * after a warm-up. No reference counterpart; the benchmark's FP32 rooflines
 * divide by it. Synchronises the context's stream. */
int mvr_measure_f32x2_rate(mvr_ctx* ctx, double* lane_ops_per_s);

/* Wait for all work on the context's stream; reports device-side errors. */
int mvr_ctx_sync(mvr_ctx* ctx);

/* Replaces `PQ.decode` (src/index/pq.zig:79-88) over a batch: rows of
 * concatenated codewords. Host pointers; runs on the host (it is a copy). */
int mvr_pq_decode(const float* codebooks, uint32_t dim, uint32_t pq_m,
                  const uint8_t* codes, uint64_t n, float* out);

/* ---- storage residuals ------------------------------------------------- */

/* Replaces `residualsAndNormsChunk` over all rows
 * (src/index/storage.zig:255-278): r = v - centroids[assign[i]];
 * norm = sqrt(sum r^2) summed in coordinate order; r *= 1/norm if norm > 0.
 * vectors n*dim, centroids kappa*dim, assignments n, residuals_out n*dim,
 * norms_out n. Host pointers. */
int mvr_residuals_norms(mvr_ctx* ctx, const float* vectors,
                        const float* centroids, uint32_t kappa,
                        const uint32_t* assignments, uint64_t n, uint32_t dim,
                        float* residuals_out, float* norms_out);

/* Device-pointer variant of `mvr_residuals_norms` (asynchronous). */
int mvr_residuals_norms_device(mvr_ctx* ctx, const float* d_vectors,
                               const float* d_centroids, uint32_t kappa,
                               const uint32_t* d_assignments, uint64_t n,
                               uint32_t dim, float* d_residuals_out,
                               float* d_norms_out);

/* ---- tac.clusterFlat --------------------------------------------------- */

/* Mirrors `tac.ClusteringParams` (src/tac/tac.zig:35-57). Reference
 * defaults: mu=128 tau=256 epsilon=4 theta=39 max_iters=25 tol=1e-4
 * n_threads=1 (src/constants.zig:10-13). */
typedef struct mvr_clustering_params {
  uint32_t kappa_total;
  uint32_t mu;
  uint32_t tau;
  uint32_t epsilon;
  uint32_t theta;
  uint32_t max_iters;
  float tol;
  uint64_t seed;
  uint32_t n_threads;
} mvr_clustering_params;

/* Fill `p` with the reference defaults and the given budget and seed. */
void mvr_clustering_params_default(mvr_clustering_params* p,
                                   uint32_t kappa_total, uint64_t seed);

/* Replaces `tac.clusterFlat(token_ids, vectors, dim, p, gpa)`
 * (src/tac/tac.zig:563-838): per-token frequencies and CSR grouping,
 * Welford spreads, budget phases 1-4 (tac.zig:97-402), then one
 * kmeans.fit(k=kappa_j, seed ^ j) per token (runOneTokenKmeans,
 * tac.zig:458-514), all per-token k-means on the GPU.
 * Inputs: n_tokens ids, vectors_len = n_tokens*dim floats.
 * Outputs: centroids_out kappa_total*dim floats (token-id order),
 * assignments_out n_tokens global centroid ids, kappa_per_token_out with
 * room for `kappa_per_token_cap` entries (the vocabulary size
 * max(token_ids)+1 is written to *n_distinct_out; a smaller cap returns
 * MVR_E_OUT_BUFFER_WRONG_SIZE), wcss_total_out summed in the reference's
 * per-thread-chunk order for `p->n_threads`. */
int mvr_tac_cluster_flat(mvr_ctx* ctx, const uint32_t* token_ids,
                         uint64_t n_tokens, const float* vectors,
                         uint64_t vectors_len, uint32_t dim,
                         const mvr_clustering_params* p, float* centroids_out,
                         uint32_t* assignments_out,
                         uint32_t* kappa_per_token_out,
                         uint64_t kappa_per_token_cap, uint64_t* n_distinct_out,
                         float* wcss_total_out);

/* Several GPUs (no reference counterpart; the reference runs the per-token
 * k-means of tac.clusterFlat on host threads, src/tac/tac.zig:685-825):
 * collective over the context's communicator (`mvr_ctx_init_comm`). Every
 * rank passes the same inputs and receives the full outputs of
 * `mvr_tac_cluster_flat`, bit for bit. Grouping, spreads and budgets run on
 * every rank; the per-token k-means problems are split over the ranks by
 * `mvr_tac_partition_tokens`, and the results are merged with one exact
 * all-reduce (each value comes from exactly one rank). Without a
 * communicator it is `mvr_tac_cluster_flat`. */
int mvr_tac_cluster_flat_sharded(mvr_ctx* ctx, const uint32_t* token_ids,
                                 uint64_t n_tokens, const float* vectors,
                                 uint64_t vectors_len, uint32_t dim,
                                 const mvr_clustering_params* p,
                                 float* centroids_out,
                                 uint32_t* assignments_out,
                                 uint32_t* kappa_per_token_out,
                                 uint64_t kappa_per_token_cap,
                                 uint64_t* n_distinct_out,
                                 float* wcss_total_out);

/* The token split of `mvr_tac_cluster_flat_sharded` (host-only):
 * longest-processing-time first over the work estimate n_j * (k_j + 1)
 * (n_j when k_j >= n_j), heaviest token first (ties in token order), each to
 * the least-loaded rank (ties: the lowest rank). owner_out[j] in
 * [0, n_ranks); 0 for tokens without a problem (n_j = 0 or k_j = 0). */
int mvr_tac_partition_tokens(const uint32_t* freqs, const uint32_t* kappa,
                             uint64_t n, uint32_t n_ranks,
                             uint32_t* owner_out);

/* Replaces `tac.allocateBudgets` (src/tac/tac.zig:390-402): phases 1-4 on
 * per-token (freq, spread) arrays of length n. Host-only integer/float
 * logic; `frac` is caller scratch of n floats. */
int mvr_tac_allocate_budgets(const uint32_t* freqs, const float* spreads,
                             uint32_t* kappa, float* frac, uint64_t n,
                             uint32_t kappa_total,
                             const mvr_clustering_params* p);

/* ------------------------------------------------------------------------
 * Inverted lists and the .tac index image (src/index/inverted_list.zig,
 * src/index/storage.zig)
 * ------------------------------------------------------------------------ */

/* Replaces `inverted_list.build(assignments, doc_offsets, kappa, gpa)`
 * (src/index/inverted_list.zig:54-150) on the GPU: for each centroid j the
 * ascending ids of the documents with at least one token assigned to j
 * (one entry per document). `doc_offsets` has `doc_offsets_len` = n_docs + 1
 * entries (CSR token ranges). Outputs: `offsets_out` kappa + 1 u64 (from 0),
 * `payload_out` the doc ids, `payload_cap` entries available (n_tokens
 * always suffices); `payload_len_out` = offsets_out[kappa]. Errors in the
 * reference's order: MVR_E_KAPPA_ZERO, MVR_E_DOC_OFFSETS_BAD (empty
 * offsets, more than 2^32 - 1 docs, last offset != n_tokens, first != 0,
 * decreasing), MVR_E_ASSIGNMENT_OUT_OF_RANGE; MVR_E_BUFFER_TOO_SMALL when
 * the payload does not fit. All pointers are host memory. */
int mvr_inverted_lists_build(mvr_ctx* ctx, const uint32_t* assignments, uint64_t n_tokens,
                             const uint64_t* doc_offsets, uint64_t doc_offsets_len, uint32_t kappa,
                             uint64_t* offsets_out, uint32_t* payload_out, uint64_t payload_cap,
                             uint64_t* payload_len_out);

/* The parts of a built index, the reference's `BuildOutput`
 * (storage.zig:127-148), as plain host arrays. `pq_m` is the subspace count
 * (the reference's comptime PQ_M; the header records it and a reader checks
 * it). The HNSW graph is given as the reference's `Hnsw` fields
 * (hnsw.zig:136-170): `hnsw_layer_offsets[L]` (n + 1 u32) and
 * `hnsw_layer_neighbours[L]` (offsets[L][n] u32) for L = 0 .. max_level. */
typedef struct mvr_tac_parts {
  uint32_t dim, kappa, sub_dim, pq_m;
  uint64_t n_docs, n_tokens;
  const float* centroids;          /* kappa * dim (normalised, as storage.build stores them) */
  const uint32_t* assignments;     /* n_tokens */
  const uint8_t* pq_codes;         /* n_tokens * pq_m */
  const uint64_t* doc_offsets;     /* n_docs + 1 */
  const float* codebooks;          /* pq_m * 256 * sub_dim */
  uint32_t hnsw_n, hnsw_entry_point, hnsw_max_level;
  const uint8_t* hnsw_node_levels; /* hnsw_n */
  const uint32_t* const* hnsw_layer_offsets;
  const uint32_t* const* hnsw_layer_neighbours;
  const uint64_t* ilist_offsets;   /* kappa + 1 */
  const uint32_t* ilist_payload;   /* ilist_offsets[kappa] */
  const float* residual_norms;     /* n_tokens */
} mvr_tac_parts;

/* On-disk header region (storage.zig:75-77): the 112-byte Header padded to
 * 128 bytes. Magic "TAC_IDX1", version 2 (constants.zig:43-45). */
#define MVR_TAC_HEADER_REGION 128u
#define MVR_TAC_VERSION 2u

/* Replaces `storage.computeSize` (storage.zig:495-528): bytes of the image. */
int mvr_tac_file_size(const mvr_tac_parts* parts, uint64_t* bytes_out);

/* Replaces `storage.serialise` (storage.zig:560-665) with `writeHnsw`
 * (:667-703) and `writeDocLayouts` (:705-749): header, centroids, HNSW, PQ
 * codebooks, inverted lists, per-doc layouts (interleaved on the GPU),
 * doc token offsets, residual norms, each section padded to 8 bytes, then
 * the footer CRC-32 of everything before it (std.hash.Crc32) and 4 zero
 * bytes. `buf` (host, `buf_len` >= mvr_tac_file_size) receives the image;
 * MVR_E_BUFFER_TOO_SMALL otherwise. */
int mvr_tac_serialise(mvr_ctx* ctx, const mvr_tac_parts* parts, void* buf, uint64_t buf_len,
                      uint64_t* written_out);

/* ------------------------------------------------------------------------
 * HNSW over the TAC centroids (src/index/hnsw.zig)
 * ------------------------------------------------------------------------ */

/* A built graph: the reference's `Hnsw` (hnsw.zig:136-170) in host memory,
 * owned by the library. */
typedef struct mvr_hnsw mvr_hnsw;

/* hnsw.build (hnsw.zig:314-475) on the GPU over `n_floats / dim` centroids,
 * which the caller has L2-normalised (storage.zig:408-411 does that with
 * vec.normalizeRowsInPlace; mvr_normalize_rows is its GPU form).
 * n_threads <= 1 builds the reference's serial path (buildSerial,
 * hnsw.zig:477-625); n_threads >= 2 its chunked deferred-commit path
 * (buildParallel, hnsw.zig:639-946), whose graph is the same for every
 * thread count >= 2, so the value only selects the path. Supported:
 * 1 <= m <= 32, 1 <= ef_construction <= 2048, dim <= 256, at most 2^27
 * centroids (MVR_E_INVALID_ARGUMENT otherwise). Equal similarities are
 * ordered by node id where the reference's heaps leave the order to their
 * layout. Errors: MVR_E_DIM_MISMATCH, MVR_E_EMPTY_CORPUS (the reference's
 * HnswError), MVR_E_DEVICE_LIMIT when more than 512 beam entries tie
 * exactly at the beam's minimum. */
int mvr_hnsw_build(mvr_ctx* ctx, const float* centroids, uint64_t n_floats, uint32_t dim,
                   uint64_t seed, uint32_t ef_construction, uint32_t m, uint32_t n_threads,
                   mvr_hnsw** out);
/* The same with the centroids in device memory (read only). */
int mvr_hnsw_build_device(mvr_ctx* ctx, const float* d_centroids, uint64_t n_floats,
                          uint32_t dim, uint64_t seed, uint32_t ef_construction, uint32_t m,
                          uint32_t n_threads, mvr_hnsw** out);
/* n, entry_point, max_level of a built graph; device time of the build in
 * milliseconds and the number of kernels it launched. */
void mvr_hnsw_info(const mvr_hnsw* g, uint32_t* n, uint32_t* entry_point, uint32_t* max_level,
                   float* device_ms, uint64_t* kernel_launches);
/* Top level of every node (n bytes). */
const uint8_t* mvr_hnsw_node_levels(const mvr_hnsw* g);
/* Layer `layer` as CSR: offsets (n + 1 entries, from 0) and the neighbour
 * ids (offsets[n] entries); null when layer > max_level. */
const uint32_t* mvr_hnsw_layer_offsets(const mvr_hnsw* g, uint32_t layer);
const uint32_t* mvr_hnsw_layer_neighbours(const mvr_hnsw* g, uint32_t layer, uint64_t* count);
void mvr_hnsw_free(mvr_hnsw* g);

/* vec.normalizeRowsInPlace (src/util/vec.zig:185-253) on the GPU, in place
 * on a host buffer: each row times 1 / sqrt(dot(row, row)), zero rows kept. */
int mvr_normalize_rows(mvr_ctx* ctx, float* rows, uint64_t n_floats, uint32_t dim);
/* The same on a device buffer, ordered on the context's stream. */
int mvr_normalize_rows_device(mvr_ctx* ctx, float* d_rows, uint64_t n_floats, uint32_t dim);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* MVR_H */
