/*
 * mvr_oracle.c — TEST INFRASTRUCTURE, NOT PRODUCT CODE.
 *
 * A plain-C restatement of the reference's PQ / k-means / TAC build path
 * (BleedingDev/ir-multivector-retrieval, Zig 0.16, CPU only). It is the
 * parity checker for the CUDA path: tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg load it; the product never does.
 *
 * Parity status: the arithmetic (vec.l2sq order, argmin/argmax, k-means,
 * PQ, TAC budget phases, residuals) is pinned by the reference's own
 * hand-checked tests, which tests/test_oracle.py replays. The RNG stream
 * restates Zig std's DefaultPrng (Xoshiro256++ seeded through SplitMix64),
 * `uintLessThan` and `float(f64)` from their published algorithms; the
 * SplitMix64 expansion is pinned to its published seed-0 outputs, the
 * Xoshiro/float conventions are not pinned against a Zig binary (there is
 * no Zig toolchain here) — "parity unpinned" for RNG-dependent outputs.
 *
 * Build: -O2 -ffp-contract=off (no FMA contraction, IEEE binary32/64, no
 * flush-to-zero), matching Zig's strict float mode.
 */
#include "mvr_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>

#include "../include/mvr.h"

/* ------------------------------------------------------------------------
 * vec.zig
 * ------------------------------------------------------------------------ */

static int g_reduce_tree = 0;
static int g_lane_count = 4;

void orc_set_reduce_tree(int tree) { g_reduce_tree = tree ? 1 : 0; }
void orc_set_lane_count(int lanes) {
  if (lanes >= 1 && lanes <= 64) g_lane_count = lanes;
}

/* @reduce(.Add, acc) over `lanes` f32 lanes. */
static float reduce_lanes(const float* acc, int lanes) {
  if (g_reduce_tree && lanes == 4) return (acc[0] + acc[1]) + (acc[2] + acc[3]);
  float s = acc[0];
  for (int l = 1; l < lanes; ++l) s = s + acc[l];
  return s;
}

/* vec.l2sq (src/util/vec.zig:109-124) with its specialisations:
 *   len 2   : d0*d0 + d1*d1                         (:114-118)
 *   len 4   : s = 0; s += d_i*d_i in order          (l2sqComptime :133-139)
 *   len 64/128: 4 strided lane accumulators, @reduce (:142-155)
 *   other   : l2sqGeneric with lane_count lanes + scalar tail (:159-175) */
float orc_l2sq(const float* a, const float* b, uint32_t len) {
  if (len == 2) {
    const float d0 = a[0] - b[0];
    const float d1 = a[1] - b[1];
    return d0 * d0 + d1 * d1;
  }
  if (len == 4) {
    float s = 0.0f;
    for (int i = 0; i < 4; ++i) {
      const float d = a[i] - b[i];
      s += d * d;
    }
    return s;
  }
  if (len == 64 || len == 128) {
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (uint32_t off = 0; off < len; off += 4) {
      for (int l = 0; l < 4; ++l) {
        const float d = a[off + l] - b[off + l];
        acc[l] += d * d;
      }
    }
    return reduce_lanes(acc, 4);
  }
  /* generic */
  const int L = g_lane_count;
  float acc[64] = {0.0f};
  uint32_t i = 0;
  while (i + (uint32_t)L <= len) {
    for (int l = 0; l < L; ++l) {
      const float d = a[i + l] - b[i + l];
      acc[l] += d * d;
    }
    i += (uint32_t)L;
  }
  float sum = reduce_lanes(acc, L);
  while (i < len) {
    const float d = a[i] - b[i];
    sum += d * d;
    ++i;
  }
  return sum;
}

/* vec.argmin (src/util/vec.zig:271-283): first index of the minimum. */
int64_t orc_argmin(const float* v, uint64_t n) {
  if (n == 0) return -1;
  uint64_t best = 0;
  float bv = v[0];
  for (uint64_t i = 1; i < n; ++i)
    if (v[i] < bv) {
      bv = v[i];
      best = i;
    }
  return (int64_t)best;
}

/* vec.argmax (src/util/vec.zig:287-299): first index of the maximum. */
int64_t orc_argmax(const float* v, uint64_t n) {
  if (n == 0) return -1;
  uint64_t best = 0;
  float bv = v[0];
  for (uint64_t i = 1; i < n; ++i)
    if (v[i] > bv) {
      bv = v[i];
      best = i;
    }
  return (int64_t)best;
}

/* ------------------------------------------------------------------------
 * rng.zig over Zig std.Random.DefaultPrng (Xoshiro256++)
 * ------------------------------------------------------------------------ */

static uint64_t splitmix64_next(uint64_t* s) {
  *s += 0x9e3779b97f4a7c15ULL;
  uint64_t z = *s;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
  return z ^ (z >> 31);
}

static inline uint64_t rotl64(uint64_t x, int k) {
  return (x << k) | (x >> (64 - k));
}

/* Rng.init(seed) (src/util/rng.zig:25-27): four SplitMix64 outputs. */
void orc_rng_init(orc_rng* r, uint64_t seed) {
  uint64_t sm = seed;
  for (int i = 0; i < 4; ++i) r->s[i] = splitmix64_next(&sm);
}

/* Xoshiro256++ step (Blackman & Vigna). */
uint64_t orc_rng_next(orc_rng* r) {
  uint64_t* s = r->s;
  const uint64_t out = rotl64(s[0] + s[3], 23) + s[0];
  const uint64_t t = s[1] << 17;
  s[2] ^= s[0];
  s[3] ^= s[1];
  s[1] ^= s[2];
  s[0] ^= s[3];
  s[2] ^= t;
  s[3] = rotl64(s[3], 45);
  return out;
}

/* Rng.nextIndex(n) = intRangeLessThan(usize, 0, n) (rng.zig:35-38):
 * Lemire's multiply-shift with the rejection threshold -n mod n. */
uint64_t orc_rng_index(orc_rng* r, uint64_t n) {
  uint64_t x = orc_rng_next(r);
  __uint128_t m = (__uint128_t)x * n;
  uint64_t l = (uint64_t)m;
  if (l < n) {
    uint64_t t = (uint64_t)0 - n;
    if (t >= n) {
      t -= n;
      if (t >= n) t %= n;
    }
    while (l < t) {
      x = orc_rng_next(r);
      m = (__uint128_t)x * n;
      l = (uint64_t)m;
    }
  }
  return (uint64_t)(m >> 64);
}

static int clz64(uint64_t x) { return x ? __builtin_clzll(x) : 64; }

/* Random.float(f64): 52 mantissa bits, exponent from leading zeros. */
double orc_rng_f64(orc_rng* r) {
  const uint64_t rnd = orc_rng_next(r);
  uint64_t lz = (uint64_t)clz64(rnd);
  if (lz >= 12) {
    lz = 12;
    for (;;) {
      const uint64_t add = (uint64_t)clz64(orc_rng_next(r));
      lz += add;
      if (add != 64) break;
      if (lz >= 1022) {
        lz = 1022;
        break;
      }
    }
  }
  const uint64_t bits = ((1022 - lz) << 52) | (rnd & 0xFFFFFFFFFFFFFULL);
  double d;
  memcpy(&d, &bits, 8);
  return d;
}

/* Random.float(f32): 23 mantissa bits, exponent from leading zeros. */
float orc_rng_f32(orc_rng* r) {
  const uint64_t rnd = orc_rng_next(r);
  uint32_t lz = (uint32_t)clz64(rnd);
  if (lz >= 41) {
    lz = 41 + (uint32_t)clz64(orc_rng_next(r));
    if (lz == 41 + 64) {
      const uint32_t x = (uint32_t)orc_rng_next(r) | 0x7FFu;
      lz += (uint32_t)__builtin_clz(x);
    }
  }
  const uint32_t bits = ((126u - lz) << 23) | ((uint32_t)rnd & 0x7FFFFFu);
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

/* rng.weightedSample (src/util/rng.zig:57-82). */
int orc_weighted_sample(orc_rng* r, const float* w, uint64_t n, uint64_t* out) {
  if (n == 0) return MVR_E_EMPTY_DISTRIBUTION;
  double total = 0.0;
  for (uint64_t i = 0; i < n; ++i) {
    if (!isfinite(w[i]) || w[i] < 0.0f) return MVR_E_NON_FINITE;
    total += (double)w[i];
  }
  if (total <= 0.0) return MVR_E_ALL_ZERO;
  const double u = orc_rng_f64(r) * total;
  double cum = 0.0;
  for (uint64_t i = 0; i < n; ++i) {
    cum += (double)w[i];
    if (u < cum) {
      *out = i;
      return MVR_OK;
    }
  }
  uint64_t last = n - 1;
  while (last > 0 && w[last] == 0.0f) --last;
  *out = last;
  return MVR_OK;
}

/* ------------------------------------------------------------------------
 * kmeans.zig
 * ------------------------------------------------------------------------ */

typedef struct assign_job {
  const float* vectors;
  const float* centroids;
  uint32_t* assignments;
  float* min_to_any;
  uint64_t lo, hi, d, k;
} assign_job;

/* kmeans.assignSlice (src/tac/kmeans.zig:344-365). */
static void assign_slice(const assign_job* j) {
  float* dists = (float*)malloc(sizeof(float) * j->k);
  for (uint64_t i = j->lo; i < j->hi; ++i) {
    const float* v = j->vectors + i * j->d;
    for (uint64_t c = 0; c < j->k; ++c)
      dists[c] = orc_l2sq(v, j->centroids + c * j->d, (uint32_t)j->d);
    const int64_t a = orc_argmin(dists, j->k);
    j->assignments[i] = (uint32_t)a;
    j->min_to_any[i] = dists[a];
  }
  free(dists);
}

static void* assign_thread(void* p) {
  assign_slice((const assign_job*)p);
  return NULL;
}

/* kmeans.assignVectors (src/tac/kmeans.zig:244-340): static chunks. */
static void assign_vectors(const float* vectors, uint64_t n, uint64_t d,
                           uint64_t k, const float* centroids,
                           uint32_t* assignments, float* min_to_any,
                           uint32_t n_threads) {
  uint64_t t = n_threads <= 1 ? 1 : (n_threads < n ? n_threads : n);
  if (t <= 1) {
    assign_job j = {vectors, centroids, assignments, min_to_any, 0, n, d, k};
    assign_slice(&j);
    return;
  }
  assign_job* jobs = (assign_job*)calloc(t, sizeof(assign_job));
  pthread_t* th = (pthread_t*)calloc(t, sizeof(pthread_t));
  const uint64_t chunk = (n + t - 1) / t;
  for (uint64_t i = 0; i < t; ++i) {
    uint64_t lo = i * chunk, hi = lo + chunk;
    if (lo > n) lo = n;
    if (hi > n) hi = n;
    jobs[i] = (assign_job){vectors, centroids, assignments, min_to_any, lo, hi, d, k};
    pthread_create(&th[i], NULL, assign_thread, &jobs[i]);
  }
  for (uint64_t i = 0; i < t; ++i) pthread_join(th[i], NULL);
  free(jobs);
  free(th);
}

/* One Lloyd iteration body shared by kmeans.fit and the timing helper:
 * assign, serial in-order accumulation, update with reseed
 * (src/tac/kmeans.zig:156-212). Returns the WCSS of the assignment step. */
static float lloyd_step(const float* vectors, uint64_t n, uint64_t d,
                        uint64_t k, float* centroids, uint32_t* assignments,
                        float* min_to_any, float* sums, uint32_t* counts,
                        uint32_t n_threads) {
  float wcss = 0.0f;
  memset(sums, 0, sizeof(float) * k * d);
  memset(counts, 0, sizeof(uint32_t) * k);
  assign_vectors(vectors, n, d, k, centroids, assignments, min_to_any, n_threads);
  for (uint64_t i = 0; i < n; ++i) {
    const uint32_t a = assignments[i];
    wcss += min_to_any[i];
    const float* v = vectors + i * d;
    float* s = sums + (uint64_t)a * d;
    for (uint64_t dd = 0; dd < d; ++dd) s[dd] += v[dd];
    counts[a] += 1;
  }
  for (uint64_t c = 0; c < k; ++c) {
    if (counts[c] > 0) {
      const float inv = 1.0f / (float)counts[c];
      float* slot = centroids + c * d;
      const float* s = sums + c * d;
      for (uint64_t dd = 0; dd < d; ++dd) slot[dd] = s[dd] * inv;
    } else {
      const int64_t far = orc_argmax(min_to_any, n);
      memcpy(centroids + c * d, vectors + (uint64_t)far * d, sizeof(float) * d);
      min_to_any[far] = -INFINITY;
    }
  }
  return wcss;
}

/* The k-means++ weight update of one step (kmeans.zig:128-135): per row,
 * independent of the others, so static row chunks on n_threads threads give
 * the same bytes as the serial loop (the reference runs it serially). */
typedef struct seed_job {
  const float* vectors;
  const float* cc;
  float* min_dist;
  uint64_t lo, hi, d;
} seed_job;

static void seed_slice(const seed_job* j) {
  for (uint64_t i = j->lo; i < j->hi; ++i) {
    const float dist = orc_l2sq(j->vectors + i * j->d, j->cc, (uint32_t)j->d);
    if (dist < j->min_dist[i]) j->min_dist[i] = dist;
  }
}

static void* seed_thread(void* p) {
  seed_slice((const seed_job*)p);
  return NULL;
}

static void seed_update(const float* vectors, uint64_t n, uint64_t d, const float* cc, float* min_dist,
                        uint32_t n_threads) {
  uint64_t t = n_threads <= 1 || n < 8192 ? 1 : (n_threads < n ? n_threads : n);
  if (t <= 1) {
    seed_job j = {vectors, cc, min_dist, 0, n, d};
    seed_slice(&j);
    return;
  }
  seed_job jobs[64];
  pthread_t th[64];
  if (t > 64) t = 64;
  const uint64_t chunk = (n + t - 1) / t;
  for (uint64_t i = 0; i < t; ++i) {
    uint64_t lo = i * chunk, hi = lo + chunk;
    if (lo > n) lo = n;
    if (hi > n) hi = n;
    jobs[i] = (seed_job){vectors, cc, min_dist, lo, hi, d};
    pthread_create(&th[i], NULL, seed_thread, &jobs[i]);
  }
  for (uint64_t i = 0; i < t; ++i) pthread_join(th[i], NULL);
}

/* kmeans.fit (src/tac/kmeans.zig:67-232). `trace`, if not NULL, receives
 * the assignments of every Lloyd iteration (max_iters * n u32). */
int orc_kmeans_fit(const float* vectors, uint64_t vectors_len, uint32_t dim,
                   uint32_t k, uint32_t max_iters, float tol, uint64_t seed,
                   uint32_t n_threads, float* centroids, uint32_t* assignments,
                   float* wcss_out, uint32_t* iters_out, uint32_t* trace) {
  if (k == 0) return MVR_E_KMEANS_BUDGET_TOO_SMALL;
  if (dim == 0) return MVR_E_DIM_MISMATCH;
  if (vectors_len == 0) return MVR_E_EMPTY_VECTOR_SET;
  if (vectors_len % dim != 0) return MVR_E_DIM_MISMATCH;
  const uint64_t n = vectors_len / dim, d = dim, K = k;

  if (K >= n) { /* degenerate (:88-104) */
    memcpy(centroids, vectors, sizeof(float) * n * d);
    for (uint64_t c = n; c < K; ++c)
      memcpy(centroids + c * d, vectors + (n - 1) * d, sizeof(float) * d);
    for (uint64_t i = 0; i < n; ++i) assignments[i] = (uint32_t)i;
    if (wcss_out) *wcss_out = 0.0f;
    if (iters_out) *iters_out = 0;
    return MVR_OK;
  }

  orc_rng rng;
  orc_rng_init(&rng, seed);
  float* min_dist = (float*)malloc(sizeof(float) * n);
  if (!min_dist) return MVR_E_OUT_OF_MEMORY;
  { /* k-means++ (:113-136) */
    const uint64_t idx0 = orc_rng_index(&rng, n);
    memcpy(centroids, vectors + idx0 * d, sizeof(float) * d);
    for (uint64_t i = 0; i < n; ++i)
      min_dist[i] = orc_l2sq(vectors + i * d, centroids, dim);
  }
  for (uint64_t c = 1; c < K; ++c) {
    uint64_t idx = 0;
    const int st = orc_weighted_sample(&rng, min_dist, n, &idx);
    if (st != MVR_OK) {
      free(min_dist);
      return st;
    }
    memcpy(centroids + c * d, vectors + idx * d, sizeof(float) * d);
    seed_update(vectors, n, d, centroids + c * d, min_dist, n_threads);
  }
  free(min_dist);

  float* sums = (float*)malloc(sizeof(float) * K * d);
  uint32_t* counts = (uint32_t*)malloc(sizeof(uint32_t) * K);
  float* min_to_any = (float*)malloc(sizeof(float) * n);
  if (!sums || !counts || !min_to_any) {
    free(sums);
    free(counts);
    free(min_to_any);
    return MVR_E_OUT_OF_MEMORY;
  }
  float prev = INFINITY, wcss = 0.0f;
  uint32_t iters = 0;
  for (uint32_t it = 0; it < max_iters; ++it) {
    wcss = lloyd_step(vectors, n, d, K, centroids, assignments, min_to_any,
                      sums, counts, n_threads);
    if (trace) memcpy(trace + (uint64_t)it * n, assignments, sizeof(uint32_t) * n);
    iters = it + 1;
    if (it > 0) { /* (:217-221) */
      const float denom = prev > 0.0f ? prev : 1.0f;
      const float rel = (prev - wcss) / denom;
      if (rel < tol) break;
    }
    prev = wcss;
  }
  free(sums);
  free(counts);
  free(min_to_any);
  if (wcss_out) *wcss_out = wcss;
  if (iters_out) *iters_out = iters;
  return MVR_OK;
}

/* ------------------------------------------------------------------------
 * pq.zig
 * ------------------------------------------------------------------------ */

typedef struct pq_ctx {
  const float* residuals;
  uint64_t n;
  uint32_t dim, sub_dim, pq_m, max_iters, inner_threads;
  float tol;
  uint64_t seed;
  float* codebooks;
  atomic_uint next_m;
  int* status; /* per subspace */
} pq_ctx;

/* trainOneSubspace (src/index/pq.zig:301-336). */
static int train_one_subspace(pq_ctx* c, uint32_t m, float* sub_buf,
                              uint32_t* assign_buf) {
  const uint64_t s = c->sub_dim;
  for (uint64_t i = 0; i < c->n; ++i)
    memcpy(sub_buf + i * s, c->residuals + i * c->dim + m * s, sizeof(float) * s);
  float* cent = (float*)malloc(sizeof(float) * MVR_PQ_CENTROIDS * s);
  const int st = orc_kmeans_fit(sub_buf, c->n * s, (uint32_t)s, MVR_PQ_CENTROIDS,
                                c->max_iters, c->tol, c->seed + (uint64_t)m,
                                c->inner_threads, cent, assign_buf, NULL, NULL, NULL);
  if (st == MVR_OK)
    memcpy(c->codebooks + (uint64_t)m * MVR_PQ_CENTROIDS * s, cent,
           sizeof(float) * MVR_PQ_CENTROIDS * s);
  free(cent);
  return st;
}

static void* pq_worker(void* p) {
  pq_ctx* c = (pq_ctx*)p;
  float* sub_buf = (float*)malloc(sizeof(float) * c->n * c->sub_dim);
  uint32_t* assign_buf = (uint32_t*)malloc(sizeof(uint32_t) * c->n);
  for (;;) {
    const unsigned m = atomic_fetch_add(&c->next_m, 1u);
    if (m >= c->pq_m) break;
    c->status[m] = train_one_subspace(c, m, sub_buf, assign_buf);
  }
  free(sub_buf);
  free(assign_buf);
  return NULL;
}

/* pq.train (src/index/pq.zig:158-291), parametric in the subspace count.
 * Work-stealing over subspaces when n_threads > 1 (:192-284); inner
 * k-means threads only when n_threads > pq_m (:250-253). The reported
 * error is that of the smallest failing subspace. */
int orc_pq_train(const float* residuals, uint64_t residuals_len, uint32_t dim,
                 uint64_t seed, uint32_t n_threads, uint32_t pq_m,
                 uint32_t max_iters, float tol, float* codebooks) {
  if (dim == 0) return MVR_E_DIM_MISMATCH;
  if (pq_m == 0 || dim % pq_m != 0) return MVR_E_DIM_NOT_DIVISIBLE_BY_M;
  if (residuals_len == 0) return MVR_E_EMPTY_CORPUS;
  if (residuals_len % dim != 0) return MVR_E_DIM_MISMATCH;
  pq_ctx c;
  c.residuals = residuals;
  c.n = residuals_len / dim;
  c.dim = dim;
  c.sub_dim = dim / pq_m;
  c.pq_m = pq_m;
  c.max_iters = max_iters;
  c.tol = tol;
  c.seed = seed;
  c.codebooks = codebooks;
  atomic_init(&c.next_m, 0u);
  c.status = (int*)calloc(pq_m, sizeof(int));
  const uint32_t real = n_threads <= 1 ? 1 : (n_threads < pq_m ? n_threads : pq_m);
  c.inner_threads = (n_threads <= real) ? 1 : (n_threads / real > 1 ? n_threads / real : 1);
  if (real <= 1) {
    c.inner_threads = n_threads;
    pq_worker(&c);
  } else {
    pthread_t* th = (pthread_t*)calloc(real, sizeof(pthread_t));
    for (uint32_t t = 0; t < real; ++t) pthread_create(&th[t], NULL, pq_worker, &c);
    for (uint32_t t = 0; t < real; ++t) pthread_join(th[t], NULL);
    free(th);
  }
  int st = MVR_OK;
  for (uint32_t m = 0; m < pq_m; ++m)
    if (c.status[m] != MVR_OK) {
      st = c.status[m];
      break;
    }
  free(c.status);
  return st;
}

typedef struct enc_job {
  const float* codebooks;
  const float* residuals;
  uint8_t* codes;
  uint64_t lo, hi;
  uint32_t dim, pq_m;
} enc_job;

/* PQ.encode (src/index/pq.zig:59-76) for rows [lo, hi). */
static void* enc_thread(void* p) {
  const enc_job* j = (const enc_job*)p;
  const uint32_t s = j->dim / j->pq_m;
  for (uint64_t i = j->lo; i < j->hi; ++i) {
    const float* r = j->residuals + i * j->dim;
    for (uint32_t m = 0; m < j->pq_m; ++m) {
      const float* sub = r + m * s;
      uint32_t best_c = 0;
      float best_d = INFINITY;
      for (uint32_t c = 0; c < MVR_PQ_CENTROIDS; ++c) {
        const float d = orc_l2sq(sub, j->codebooks + ((uint64_t)m * MVR_PQ_CENTROIDS + c) * s, s);
        if (d < best_d) {
          best_d = d;
          best_c = c;
        }
      }
      j->codes[i * j->pq_m + m] = (uint8_t)best_c;
    }
  }
  return NULL;
}

/* storage.pqEncodeChunk over parallelTokenLoop (src/index/storage.zig:
 * 201-244, 287-295): static chunks, serial below 1024 rows. */
int orc_pq_encode(const float* codebooks, uint32_t dim, uint32_t pq_m,
                  const float* residuals, uint64_t n, uint8_t* codes,
                  uint32_t n_threads) {
  if (dim == 0) return MVR_E_DIM_MISMATCH;
  if (pq_m == 0 || dim % pq_m != 0) return MVR_E_DIM_NOT_DIVISIBLE_BY_M;
  if (n_threads <= 1 || n < 1024) {
    enc_job j = {codebooks, residuals, codes, 0, n, dim, pq_m};
    enc_thread(&j);
    return MVR_OK;
  }
  const uint64_t t = n_threads < n ? n_threads : n;
  enc_job* jobs = (enc_job*)calloc(t, sizeof(enc_job));
  pthread_t* th = (pthread_t*)calloc(t, sizeof(pthread_t));
  const uint64_t chunk = (n + t - 1) / t;
  for (uint64_t i = 0; i < t; ++i) {
    uint64_t lo = i * chunk, hi = lo + chunk;
    if (lo > n) lo = n;
    if (hi > n) hi = n;
    jobs[i] = (enc_job){codebooks, residuals, codes, lo, hi, dim, pq_m};
    pthread_create(&th[i], NULL, enc_thread, &jobs[i]);
  }
  for (uint64_t i = 0; i < t; ++i) pthread_join(th[i], NULL);
  free(jobs);
  free(th);
  return MVR_OK;
}

typedef struct lloyd_job {
  const float* residuals;
  uint64_t n;
  uint32_t dim, sub_dim, pq_m, iters, inner;
  float* codebooks;
  atomic_uint next_m;
} lloyd_job;

static void* lloyd_worker(void* p) {
  lloyd_job* j = (lloyd_job*)p;
  const uint64_t s = j->sub_dim, n = j->n, K = MVR_PQ_CENTROIDS;
  float* sub = (float*)malloc(sizeof(float) * n * s);
  uint32_t* asg = (uint32_t*)malloc(sizeof(uint32_t) * n);
  float* mta = (float*)malloc(sizeof(float) * n);
  float* sums = (float*)malloc(sizeof(float) * K * s);
  uint32_t* counts = (uint32_t*)malloc(sizeof(uint32_t) * K);
  for (;;) {
    const unsigned m = atomic_fetch_add(&j->next_m, 1u);
    if (m >= j->pq_m) break;
    for (uint64_t i = 0; i < n; ++i)
      memcpy(sub + i * s, j->residuals + i * j->dim + m * s, sizeof(float) * s);
    float* cb = j->codebooks + (uint64_t)m * K * s;
    for (uint32_t it = 0; it < j->iters; ++it)
      (void)lloyd_step(sub, n, s, K, cb, asg, mta, sums, counts, j->inner);
  }
  free(sub);
  free(asg);
  free(mta);
  free(sums);
  free(counts);
  return NULL;
}

int orc_pq_lloyd_iters(const float* residuals, uint64_t n, uint32_t dim,
                       uint32_t pq_m, uint32_t iters, uint32_t n_threads,
                       float* codebooks_inout) {
  if (dim == 0 || pq_m == 0 || dim % pq_m != 0) return MVR_E_DIM_NOT_DIVISIBLE_BY_M;
  lloyd_job j;
  j.residuals = residuals;
  j.n = n;
  j.dim = dim;
  j.sub_dim = dim / pq_m;
  j.pq_m = pq_m;
  j.iters = iters;
  j.codebooks = codebooks_inout;
  atomic_init(&j.next_m, 0u);
  const uint32_t t = n_threads <= 1 ? 1 : (n_threads < pq_m ? n_threads : pq_m);
  /* inner assignment threads when the budget exceeds the subspace count,
   * as in pq.train (src/index/pq.zig:250-253) */
  j.inner = n_threads > t ? n_threads / t : 1;
  pthread_t* th = (pthread_t*)calloc(t, sizeof(pthread_t));
  for (uint32_t i = 0; i < t; ++i) pthread_create(&th[i], NULL, lloyd_worker, &j);
  for (uint32_t i = 0; i < t; ++i) pthread_join(th[i], NULL);
  free(th);
  return MVR_OK;
}

/* ------------------------------------------------------------------------
 * storage.zig residuals
 * ------------------------------------------------------------------------ */

/* residualsAndNormsChunk (src/index/storage.zig:255-278). */
int orc_residuals_norms(const float* vectors, const float* centroids,
                        const uint32_t* assignments, uint64_t n, uint32_t dim,
                        float* residuals, float* norms) {
  for (uint64_t i = 0; i < n; ++i) {
    const float* v = vectors + i * dim;
    const float* c = centroids + (uint64_t)assignments[i] * dim;
    float* r = residuals + i * dim;
    float sum_sq = 0.0f;
    for (uint32_t dd = 0; dd < dim; ++dd) {
      const float diff = v[dd] - c[dd];
      r[dd] = diff;
      sum_sq += diff * diff;
    }
    const float norm = sqrtf(sum_sq);
    norms[i] = norm;
    if (norm > 0.0f) {
      const float inv = 1.0f / norm;
      for (uint32_t dd = 0; dd < dim; ++dd) r[dd] *= inv;
    }
  }
  return MVR_OK;
}

/* ------------------------------------------------------------------------
 * tac.zig
 * ------------------------------------------------------------------------ */

enum { TIER_EMPTY, TIER_MICRO, TIER_SMALL, TIER_ACTIVE };

/* classifyToken (src/tac/tac.zig:80-85). */
static int classify(uint32_t n_j, uint32_t mu, uint32_t tau) {
  if (n_j == 0) return TIER_EMPTY;
  if (n_j < mu) return TIER_MICRO;
  if (n_j < tau) return TIER_SMALL;
  return TIER_ACTIVE;
}

/* allocateTail (src/tac/tac.zig:97-125). */
int orc_tac_allocate_tail(const uint32_t* freqs, uint32_t* kappa, uint64_t n,
                          uint32_t mu, uint32_t tau, uint32_t kappa_total,
                          uint32_t* budget_out) {
  if (mu == 0 || tau == 0 || mu >= tau) return MVR_E_INVALID_THRESHOLDS;
  uint32_t tail = 0;
  for (uint64_t j = 0; j < n; ++j) {
    switch (classify(freqs[j], mu, tau)) {
      case TIER_MICRO: kappa[j] = 1; tail += 1; break;
      case TIER_SMALL: kappa[j] = 2; tail += 2; break;
      default: kappa[j] = 0; break;
    }
  }
  if (tail > kappa_total) return MVR_E_BUDGET_TOO_SMALL;
  *budget_out = kappa_total - tail;
  return MVR_OK;
}

/* dampedWeight (src/tac/tac.zig:133-135). */
static float damped_weight(uint32_t n_j, float s_j) {
  return sqrtf((float)n_j) * s_j;
}

/* dampedPhase2 (src/tac/tac.zig:157-210). */
int orc_tac_damped_phase2(const uint32_t* freqs, const float* spreads,
                          uint32_t* kappa, float* frac, uint64_t n,
                          uint32_t budget, uint32_t mu, uint32_t tau) {
  for (uint64_t j = 0; j < n; ++j) frac[j] = 0.0f;
  double sum_w = 0.0;
  uint32_t n_active = 0;
  for (uint64_t j = 0; j < n; ++j) {
    if (classify(freqs[j], mu, tau) != TIER_ACTIVE) continue;
    const float w = damped_weight(freqs[j], spreads[j]);
    if (!isfinite(w) || w < 0.0f) return MVR_E_INVALID_THRESHOLDS;
    sum_w += (double)w;
    n_active += 1;
  }
  if (n_active == 0) return MVR_OK;
  if (sum_w <= 0.0) {
    const uint32_t base = budget / n_active;
    uint32_t left = budget - base * n_active;
    for (uint64_t j = 0; j < n; ++j) {
      if (classify(freqs[j], mu, tau) != TIER_ACTIVE) continue;
      kappa[j] = base;
      if (left > 0) {
        kappa[j] += 1;
        left -= 1;
      }
    }
    return MVR_OK;
  }
  const double bf = (double)budget;
  for (uint64_t j = 0; j < n; ++j) {
    if (classify(freqs[j], mu, tau) != TIER_ACTIVE) continue;
    const double w = (double)damped_weight(freqs[j], spreads[j]);
    const double target = (w / sum_w) * bf;
    const uint32_t fl = (uint32_t)floor(target);
    kappa[j] = fl;
    frac[j] = (float)(target - (double)fl);
  }
  return MVR_OK;
}

/* boundPhase3 (src/tac/tac.zig:228-248). */
int orc_tac_bound_phase3(const uint32_t* freqs, uint32_t* kappa, uint64_t n,
                         uint32_t mu, uint32_t tau, uint32_t eps,
                         uint32_t theta) {
  if (eps == 0 || theta == 0) return MVR_E_INVALID_THRESHOLDS;
  if ((uint64_t)tau < (uint64_t)eps * theta) return MVR_E_INVALID_THRESHOLDS;
  for (uint64_t j = 0; j < n; ++j) {
    if (classify(freqs[j], mu, tau) != TIER_ACTIVE) continue;
    const uint32_t cap = freqs[j] / theta;
    if (kappa[j] < eps) kappa[j] = eps;
    if (kappa[j] > cap) kappa[j] = cap;
  }
  return MVR_OK;
}

/* reconcilePhase4 (src/tac/tac.zig:281-376). */
int orc_tac_reconcile_phase4(const uint32_t* freqs, uint32_t* kappa,
                             const float* frac, uint64_t n,
                             uint32_t kappa_total, uint32_t mu, uint32_t tau,
                             uint32_t eps, uint32_t theta) {
  uint64_t cur = 0;
  for (uint64_t j = 0; j < n; ++j) cur += kappa[j];
  if (cur == kappa_total) return MVR_OK;
  if (cur < kappa_total) {
    uint32_t remaining = (uint32_t)(kappa_total - cur);
    while (remaining > 0) {
      int64_t best = -1;
      float bf = -INFINITY;
      for (uint64_t j = 0; j < n; ++j) {
        if (classify(freqs[j], mu, tau) != TIER_ACTIVE) continue;
        const uint32_t cap = freqs[j] / theta;
        if (kappa[j] >= cap) continue;
        if (frac[j] > bf || (frac[j] == bf && best < 0)) {
          best = (int64_t)j;
          bf = frac[j];
        }
      }
      if (best < 0) return MVR_E_BUDGET_TOO_LARGE;
      kappa[best] += 1;
      remaining -= 1;
    }
    return MVR_OK;
  }
  uint32_t excess = (uint32_t)(cur - kappa_total);
  while (excess > 0) {
    int64_t best = -1;
    float bf = INFINITY;
    for (uint64_t j = 0; j < n; ++j) {
      if (classify(freqs[j], mu, tau) != TIER_ACTIVE) continue;
      if (kappa[j] <= eps) continue;
      if (frac[j] < bf) {
        best = (int64_t)j;
        bf = frac[j];
      }
    }
    if (best >= 0) {
      kappa[best] -= 1;
      excess -= 1;
      continue;
    }
    int64_t found = -1;
    for (uint64_t j = 0; j < n; ++j)
      if (classify(freqs[j], mu, tau) == TIER_SMALL && kappa[j] == 2) {
        found = (int64_t)j;
        break;
      }
    if (found >= 0) {
      kappa[found] = 1;
      excess -= 1;
      continue;
    }
    for (uint64_t j = 0; j < n; ++j)
      if (classify(freqs[j], mu, tau) == TIER_MICRO && kappa[j] == 1) {
        found = (int64_t)j;
        break;
      }
    if (found >= 0) {
      kappa[found] = 0;
      excess -= 1;
      continue;
    }
    return MVR_E_BUDGET_TOO_SMALL;
  }
  return MVR_OK;
}

/* allocateBudgets (src/tac/tac.zig:390-402). */
int orc_tac_allocate_budgets(const uint32_t* freqs, const float* spreads,
                             uint32_t* kappa, float* frac, uint64_t n,
                             uint32_t kappa_total, uint32_t mu, uint32_t tau,
                             uint32_t eps, uint32_t theta) {
  uint32_t budget = 0;
  int st = orc_tac_allocate_tail(freqs, kappa, n, mu, tau, kappa_total, &budget);
  if (st) return st;
  st = orc_tac_damped_phase2(freqs, spreads, kappa, frac, n, budget, mu, tau);
  if (st) return st;
  st = orc_tac_bound_phase3(freqs, kappa, n, mu, tau, eps, theta);
  if (st) return st;
  return orc_tac_reconcile_phase4(freqs, kappa, frac, n, kappa_total, mu, tau, eps, theta);
}

/* Steps 0-2 of clusterFlat (src/tac/tac.zig:576-644): frequencies, CSR
 * grouping in ascending row order, Welford spread per token. */
static void group_tokens(const uint32_t* ids, uint64_t n_tokens, uint64_t nd,
                         uint32_t* freqs, uint32_t* offsets, uint32_t* indices) {
  memset(freqs, 0, sizeof(uint32_t) * nd);
  for (uint64_t i = 0; i < n_tokens; ++i) freqs[ids[i]] += 1;
  offsets[0] = 0;
  for (uint64_t j = 0; j < nd; ++j) offsets[j + 1] = offsets[j] + freqs[j];
  uint32_t* cursor = (uint32_t*)malloc(sizeof(uint32_t) * nd);
  memcpy(cursor, offsets, sizeof(uint32_t) * nd);
  for (uint64_t i = 0; i < n_tokens; ++i) indices[cursor[ids[i]]++] = (uint32_t)i;
  free(cursor);
}

static void welford_spreads(const float* vectors, uint32_t dim, uint64_t nd,
                            const uint32_t* offsets, const uint32_t* indices,
                            float* spreads) {
  float* mean = (float*)malloc(sizeof(float) * dim);
  float* m2 = (float*)malloc(sizeof(float) * dim);
  for (uint64_t j = 0; j < nd; ++j) {
    spreads[j] = 0.0f;
    const uint32_t start = offsets[j], end = offsets[j + 1];
    const uint32_t n_j = end - start;
    if (n_j == 0) continue;
    memset(mean, 0, sizeof(float) * dim);
    memset(m2, 0, sizeof(float) * dim);
    float count = 0.0f;
    for (uint32_t q = start; q < end; ++q) {
      const float* v = vectors + (uint64_t)indices[q] * dim;
      count += 1.0f;
      const float inv = 1.0f / count;
      for (uint32_t dd = 0; dd < dim; ++dd) {
        const float x = v[dd];
        const float old = mean[dd];
        const float delta = x - old;
        mean[dd] = old + delta * inv;
        m2[dd] += delta * (x - mean[dd]);
      }
    }
    float trace = 0.0f;
    for (uint32_t dd = 0; dd < dim; ++dd) trace += m2[dd];
    spreads[j] = trace / (float)n_j;
  }
  free(mean);
  free(m2);
}

int orc_tac_spreads(const uint32_t* token_ids, uint64_t n_tokens,
                    const float* vectors, uint32_t dim, uint64_t nd,
                    uint32_t* freqs, float* spreads) {
  uint32_t* offsets = (uint32_t*)malloc(sizeof(uint32_t) * (nd + 1));
  uint32_t* indices = (uint32_t*)malloc(sizeof(uint32_t) * n_tokens);
  group_tokens(token_ids, n_tokens, nd, freqs, offsets, indices);
  welford_spreads(vectors, dim, nd, offsets, indices, spreads);
  free(offsets);
  free(indices);
  return MVR_OK;
}

static int g_workers = 1;
void orc_set_workers(int n) { g_workers = n > 1 ? n : 1; }

/* runOneTokenKmeans (src/tac/tac.zig:458-514): gather the token's rows in
 * index order, kmeans.fit(k_j, seed ^ j), scatter centroids and global
 * assignments. */
static int cluster_one_token(const float* vectors, uint32_t dim, uint64_t j, const uint32_t* offsets,
                             const uint32_t* indices, const uint32_t* kappa_per_token, const uint32_t* goff,
                             uint32_t max_iters, float tol, uint64_t seed, uint32_t inner, float* gather,
                             float* cent, uint32_t* asg, float* centroids, uint32_t* assignments, float* w) {
  const uint32_t k_j = kappa_per_token[j];
  const uint32_t n_j = offsets[j + 1] - offsets[j];
  *w = 0.0f;
  if (k_j == 0 || n_j == 0) return MVR_OK;
  for (uint32_t q = 0; q < n_j; ++q)
    memcpy(gather + (uint64_t)q * dim, vectors + (uint64_t)indices[offsets[j] + q] * dim, sizeof(float) * dim);
  const int st = orc_kmeans_fit(gather, (uint64_t)n_j * dim, dim, k_j, max_iters, tol, seed ^ (uint64_t)j, inner,
                                cent, asg, w, NULL, NULL);
  if (st) return st;
  memcpy(centroids + (uint64_t)goff[j] * dim, cent, sizeof(float) * (uint64_t)k_j * dim);
  for (uint32_t q = 0; q < n_j; ++q) assignments[indices[offsets[j] + q]] = goff[j] + asg[q];
  return MVR_OK;
}

typedef struct token_pool {
  const float* vectors;
  uint32_t dim;
  const uint32_t* offsets;
  const uint32_t* indices;
  const uint32_t* kappa;
  const uint32_t* goff;
  uint32_t max_iters;
  float tol;
  uint64_t seed;
  const uint64_t* order;
  uint64_t count;
  uint64_t next;
  uint32_t max_n, max_k;
  float* centroids;
  uint32_t* assignments;
  float* token_wcss;
  int status;
  pthread_mutex_t mu;
} token_pool;

static void* token_worker(void* p) {
  token_pool* tp = (token_pool*)p;
  float* gather = (float*)malloc(sizeof(float) * (uint64_t)(tp->max_n ? tp->max_n : 1) * tp->dim);
  float* cent = (float*)malloc(sizeof(float) * (uint64_t)(tp->max_k ? tp->max_k : 1) * tp->dim);
  uint32_t* asg = (uint32_t*)malloc(sizeof(uint32_t) * (tp->max_n ? tp->max_n : 1));
  for (;;) {
    pthread_mutex_lock(&tp->mu);
    const uint64_t q = tp->next++;
    const int stop = tp->status != MVR_OK;
    pthread_mutex_unlock(&tp->mu);
    if (stop || q >= tp->count) break;
    const uint64_t j = tp->order[q];
    float w = 0.0f;
    const int st = cluster_one_token(tp->vectors, tp->dim, j, tp->offsets, tp->indices, tp->kappa, tp->goff,
                                     tp->max_iters, tp->tol, tp->seed, 1, gather, cent, asg, tp->centroids,
                                     tp->assignments, &w);
    tp->token_wcss[j] = w;
    if (st) {
      pthread_mutex_lock(&tp->mu);
      if (tp->status == MVR_OK) tp->status = st;
      pthread_mutex_unlock(&tp->mu);
    }
  }
  free(gather);
  free(cent);
  free(asg);
  return NULL;
}

static const uint64_t* g_sort_work;
static int cmp_work_desc(const void* a, const void* b) {
  const uint64_t x = g_sort_work[*(const uint64_t*)a], y = g_sort_work[*(const uint64_t*)b];
  if (x != y) return x > y ? -1 : 1;
  const uint64_t i = *(const uint64_t*)a, k = *(const uint64_t*)b;
  return i < k ? -1 : (i > k);
}

static int cluster_tokens_parallel(const float* vectors, uint32_t dim, uint64_t nd, const uint32_t* freqs,
                                   const uint32_t* offsets, const uint32_t* indices, const uint32_t* kappa,
                                   const uint32_t* goff, uint32_t max_iters, float tol, uint64_t seed,
                                   float* centroids, uint32_t* assignments, float* token_wcss) {
  uint64_t* work = (uint64_t*)calloc(nd ? nd : 1, sizeof(uint64_t));
  uint64_t* order = (uint64_t*)malloc(sizeof(uint64_t) * (nd ? nd : 1));
  uint64_t total = 0, cnt = 0;
  uint32_t max_n = 0, max_k = 0;
  for (uint64_t j = 0; j < nd; ++j) {
    if (!freqs[j] || !kappa[j]) continue;
    work[j] = (uint64_t)freqs[j] * ((uint64_t)kappa[j] + 1);
    total += work[j];
    order[cnt++] = j;
  }
  g_sort_work = work;
  qsort(order, cnt, sizeof(uint64_t), cmp_work_desc);
  int st = MVR_OK;
  uint64_t first_small = 0;
  /* big tokens one at a time with all workers inside kmeans.fit */
  while (first_small < cnt && work[order[first_small]] * (uint64_t)g_workers >= total) {
    const uint64_t j = order[first_small++];
    const uint32_t n_j = offsets[j + 1] - offsets[j];
    float* gather = (float*)malloc(sizeof(float) * (uint64_t)n_j * dim);
    float* cent = (float*)malloc(sizeof(float) * (uint64_t)kappa[j] * dim);
    uint32_t* asg = (uint32_t*)malloc(sizeof(uint32_t) * n_j);
    float w = 0.0f;
    st = cluster_one_token(vectors, dim, j, offsets, indices, kappa, goff, max_iters, tol, seed,
                           (uint32_t)g_workers, gather, cent, asg, centroids, assignments, &w);
    token_wcss[j] = w;
    free(gather);
    free(cent);
    free(asg);
    if (st) break;
  }
  if (st == MVR_OK && first_small < cnt) {
    for (uint64_t q = first_small; q < cnt; ++q) {
      const uint64_t j = order[q];
      const uint32_t n_j = offsets[j + 1] - offsets[j];
      if (n_j > max_n) max_n = n_j;
      if (kappa[j] > max_k) max_k = kappa[j];
    }
    token_pool tp = {vectors, dim, offsets, indices, kappa, goff, max_iters, tol, seed, order + first_small,
                     cnt - first_small, 0, max_n, max_k, centroids, assignments, token_wcss, MVR_OK,
                     PTHREAD_MUTEX_INITIALIZER};
    pthread_t th[256];
    const int t = g_workers < 256 ? g_workers : 256;
    for (int i = 0; i < t; ++i) pthread_create(&th[i], NULL, token_worker, &tp);
    for (int i = 0; i < t; ++i) pthread_join(th[i], NULL);
    st = tp.status;
  }
  free(work);
  free(order);
  return st;
}

/* clusterFlat (src/tac/tac.zig:563-838) with runOneTokenKmeans
 * (:458-514). wcss_total follows the reference's static per-thread token
 * chunks (:712-825) when n_threads > 1. */
int orc_tac_cluster_flat(const uint32_t* token_ids, uint64_t n_tokens,
                         const float* vectors, uint64_t vectors_len,
                         uint32_t dim, uint32_t kappa_total, uint32_t mu,
                         uint32_t tau, uint32_t eps, uint32_t theta,
                         uint32_t max_iters, float tol, uint64_t seed,
                         uint32_t n_threads, float* centroids,
                         uint32_t* assignments, uint32_t* kappa_per_token,
                         uint64_t kappa_cap, uint64_t* nd_out,
                         float* wcss_total) {
  if (n_tokens == 0) return MVR_E_EMPTY_TOKEN_DUMP;
  if (dim == 0) return MVR_E_INVALID_THRESHOLDS;
  if (vectors_len != n_tokens * (uint64_t)dim) return MVR_E_INVALID_THRESHOLDS;
  if (kappa_total == 0) return MVR_E_BUDGET_TOO_SMALL;
  uint32_t max_id = 0;
  for (uint64_t i = 0; i < n_tokens; ++i)
    if (token_ids[i] > max_id) max_id = token_ids[i];
  const uint64_t nd = (uint64_t)max_id + 1;
  if (nd_out) *nd_out = nd;
  if (kappa_cap < nd) return MVR_E_OUT_BUFFER_WRONG_SIZE;

  uint32_t* freqs = (uint32_t*)malloc(sizeof(uint32_t) * nd);
  uint32_t* offsets = (uint32_t*)malloc(sizeof(uint32_t) * (nd + 1));
  uint32_t* indices = (uint32_t*)malloc(sizeof(uint32_t) * n_tokens);
  float* spreads = (float*)malloc(sizeof(float) * nd);
  float* frac = (float*)malloc(sizeof(float) * nd);
  uint32_t* goff = (uint32_t*)malloc(sizeof(uint32_t) * (nd + 1));
  int st = MVR_OK;
  float* gather = NULL;
  float* cent = NULL;
  uint32_t* asg = NULL;
  float* token_wcss = NULL;
  group_tokens(token_ids, n_tokens, nd, freqs, offsets, indices);
  welford_spreads(vectors, dim, nd, offsets, indices, spreads);
  st = orc_tac_allocate_budgets(freqs, spreads, kappa_per_token, frac, nd,
                                kappa_total, mu, tau, eps, theta);
  if (st) goto done;
  for (uint64_t j = 0; j < nd; ++j)
    if (freqs[j] > 0 && kappa_per_token[j] == 0) {
      st = MVR_E_BUDGET_TOO_SMALL;
      goto done;
    }
  goff[0] = 0;
  for (uint64_t j = 0; j < nd; ++j) goff[j + 1] = goff[j] + kappa_per_token[j];
  if (goff[nd] != kappa_total) {
    st = MVR_E_BUDGET_TOO_SMALL;
    goto done;
  }
  uint32_t max_n = 0, max_k = 0;
  for (uint64_t j = 0; j < nd; ++j) {
    if (freqs[j] > max_n) max_n = freqs[j];
    if (kappa_per_token[j] > max_k) max_k = kappa_per_token[j];
  }
  token_wcss = (float*)calloc(nd, sizeof(float));
  if (g_workers > 1) {
    /* Test-speed path, same bytes: tokens are independent k-means problems
     * writing disjoint outputs, so they run on g_workers threads; a token
     * with a large share of the work runs alone with its assignment and
     * seeding loops split over all workers (per-row work: identical). */
    st = cluster_tokens_parallel(vectors, dim, nd, freqs, offsets, indices, kappa_per_token, goff,
                                 max_iters, tol, seed, centroids, assignments, token_wcss);
    if (st) goto done;
  } else {
    gather = (float*)malloc(sizeof(float) * (uint64_t)max_n * dim);
    cent = (float*)malloc(sizeof(float) * (uint64_t)(max_k ? max_k : 1) * dim);
    asg = (uint32_t*)malloc(sizeof(uint32_t) * (max_n ? max_n : 1));
    for (uint64_t j = 0; j < nd; ++j) {
      float w = 0.0f;
      st = cluster_one_token(vectors, dim, j, offsets, indices, kappa_per_token, goff, max_iters, tol, seed, 1,
                             gather, cent, asg, centroids, assignments, &w);
      if (st) goto done;
      token_wcss[j] = w;
    }
  }
  {
    float total = 0.0f;
    if (n_threads <= 1) {
      for (uint64_t j = 0; j < nd; ++j)
        if (kappa_per_token[j] && freqs[j]) total += token_wcss[j];
    } else {
      const uint64_t chunk = (nd + n_threads - 1) / n_threads;
      for (uint64_t t = 0; t < n_threads; ++t) {
        const uint64_t lo = t * chunk;
        uint64_t hi = (t + 1) * chunk;
        if (hi > nd) hi = nd;
        float w = 0.0f;
        for (uint64_t j = lo; j < hi; ++j)
          if (kappa_per_token[j] && freqs[j]) w += token_wcss[j];
        total += w;
      }
    }
    if (wcss_total) *wcss_total = total;
  }
  for (uint64_t i = 0; i < n_tokens; ++i)
    if (assignments[i] >= kappa_total) {
      st = MVR_E_INVALID_THRESHOLDS;
      goto done;
    }
done:
  free(freqs);
  free(offsets);
  free(indices);
  free(spreads);
  free(frac);
  free(goff);
  free(gather);
  free(cent);
  free(asg);
  free(token_wcss);
  return st;
}

/* ------------------------------------------------------------------------
 * storage.zig — per-doc layouts (:705-749)
 * ------------------------------------------------------------------------ */
static uint64_t align_up8(uint64_t v) { return (v + 7u) & ~(uint64_t)7u; }

uint64_t orc_write_doc_layouts(const uint64_t* doc_offsets, uint64_t n_docs,
                               const uint32_t* assignments, const uint8_t* codes,
                               uint32_t pq_m, uint8_t* out, uint64_t out_len) {
  const uint64_t idx_bytes = (n_docs + 1) * 8;
  if (out_len < idx_bytes) return 0;
  uint64_t cur = idx_bytes, payload_off = 0;
  for (uint64_t d = 0; d < n_docs; ++d) {
    memcpy(out + d * 8, &payload_off, 8);
    const uint64_t n_d = doc_offsets[d + 1] - doc_offsets[d];
    const uint64_t tok_lo = doc_offsets[d];
    const uint64_t unpadded = 4 + n_d * 4 + n_d * (uint64_t)pq_m;
    const uint64_t this_doc = align_up8(unpadded);
    if (out_len < cur + this_doc) return 0;
    const uint32_t n32 = (uint32_t)n_d;
    memcpy(out + cur, &n32, 4);
    uint64_t w = cur + 4;
    memcpy(out + w, assignments + tok_lo, n_d * 4);
    w += n_d * 4;
    memcpy(out + w, codes + tok_lo * pq_m, n_d * pq_m);
    w += n_d * pq_m;
    memset(out + w, 0, cur + this_doc - w);
    payload_off += this_doc;
    cur += this_doc;
  }
  memcpy(out + n_docs * 8, &payload_off, 8);
  return cur;
}

/* ------------------------------------------------------------------------
 * vec.dot, PQ.buildDistanceTable, refine.refine
 * ------------------------------------------------------------------------ */
float orc_dot(const float* a, const float* b, uint32_t len) {
  if (len == 2) return a[0] * b[0] + a[1] * b[1]; /* vec.zig:50 */
  if (len == 4) {                                 /* dotComptime, dim <= 4 */
    float s = 0.0f;
    for (int i = 0; i < 4; ++i) s += a[i] * b[i];
    return s;
  }
  if (len == 64 || len == 128) { /* dotComptime: 4 lanes, ordered @reduce */
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (uint32_t off = 0; off < len; off += 4)
      for (int l = 0; l < 4; ++l) acc[l] = acc[l] + a[off + l] * b[off + l];
    return reduce_lanes(acc, 4);
  }
  const int L = g_lane_count; /* dotGeneric */
  float acc[64] = {0.0f};
  uint32_t i = 0;
  while (i + (uint32_t)L <= len) {
    for (int l = 0; l < L; ++l) acc[l] = acc[l] + a[i + l] * b[i + l];
    i += (uint32_t)L;
  }
  float sum = reduce_lanes(acc, L);
  while (i < len) {
    sum += a[i] * b[i];
    ++i;
  }
  return sum;
}

int orc_pq_distance_table(const float* codebooks, uint32_t dim, uint32_t pq_m,
                          const float* query, uint64_t query_len, uint32_t n_q,
                          float* out, uint64_t out_len) {
  if (n_q == 0) return MVR_E_NQ_MISMATCH;
  if (query_len != (uint64_t)n_q * dim) return MVR_E_NQ_MISMATCH;
  if (out_len != (uint64_t)pq_m * 256u * n_q) return MVR_E_OUT_BUFFER_WRONG_SIZE;
  const uint32_t s = dim / pq_m;
  for (uint32_t m = 0; m < pq_m; ++m)
    for (uint32_t c = 0; c < 256; ++c) {
      const float* cv = codebooks + ((uint64_t)m * 256 + c) * s;
      const uint64_t base = ((uint64_t)m * 256 + c) * n_q;
      for (uint32_t i = 0; i < n_q; ++i)
        out[base + i] = orc_dot(query + (uint64_t)i * dim + (uint64_t)m * s, cv, s);
    }
  return MVR_OK;
}

int orc_refine(const float* centroids, uint32_t dim, uint32_t pq_m,
               const uint8_t* doc_section, uint64_t n_docs,
               const uint64_t* doc_token_offsets, const float* residual_norms,
               const float* table, uint64_t table_len, const float* query,
               uint64_t query_len, uint32_t n_q, uint32_t doc_id, float* score) {
  if (n_q == 0 || query_len != (uint64_t)n_q * dim) return MVR_E_QUERY_SHAPE_MISMATCH;
  if (table_len != (uint64_t)pq_m * 256u * n_q) return MVR_E_TABLE_SIZE_MISMATCH;
  if (doc_id >= n_docs) return MVR_E_DOC_OUT_OF_RANGE;
  const uint64_t* idx = (const uint64_t*)doc_section;
  const uint8_t* payload = doc_section + (n_docs + 1) * 8;
  const uint64_t lo = idx[doc_id], hi = idx[doc_id + 1];
  if (hi - lo < 4) return MVR_E_DOC_LAYOUT_CORRUPT;
  uint32_t n_d;
  memcpy(&n_d, payload + lo, 4);
  if (hi - lo < 4 + (uint64_t)n_d * 4 + (uint64_t)n_d * pq_m) return MVR_E_DOC_LAYOUT_CORRUPT;
  const uint64_t t_lo = doc_token_offsets[doc_id], t_hi = doc_token_offsets[doc_id + 1];
  if (t_hi - t_lo != n_d) return MVR_E_DOC_LAYOUT_CORRUPT;
  const uint8_t* ids = payload + lo + 4;
  const uint8_t* codes = ids + (uint64_t)n_d * 4;
  float* best = (float*)malloc(sizeof(float) * n_q);
  for (uint32_t i = 0; i < n_q; ++i) best[i] = -INFINITY;
  for (uint32_t k = 0; k < n_d; ++k) {
    uint32_t cid;
    memcpy(&cid, ids + (uint64_t)k * 4, 4);
    const float* cv = centroids + (uint64_t)cid * dim;
    const float norm_k = residual_norms[t_lo + k];
    for (uint32_t i = 0; i < n_q; ++i) {
      const float cent = orc_dot(query + (uint64_t)i * dim, cv, dim);
      float res = 0.0f;
      for (uint32_t m = 0; m < pq_m; ++m)
        res += table[((uint64_t)m * 256 + codes[(uint64_t)k * pq_m + m]) * n_q + i];
      const float sc = cent + norm_k * res;
      if (sc > best[i]) best[i] = sc;
    }
  }
  float sum = 0.0f;
  if (n_d > 0)
    for (uint32_t i = 0; i < n_q; ++i) sum += best[i];
  free(best);
  *score = sum;
  return MVR_OK;
}
