/*
 * hnsw_oracle.c — TEST INFRASTRUCTURE, NOT PRODUCT CODE.
 *
 * Plain-C restatement of the reference's HNSW build over the TAC centroids
 * (src/index/hnsw.zig) — the parity checker for the CUDA build in
 * hnsw.cu. Loaded by tests/ and bench.py's CPU-baseline leg only.
 *
 * What is restated, with the reference lines it follows:
 *   build           hnsw.zig:314-475   levels[0] drawn first, entry point 0
 *   buildParallel   hnsw.zig:639-946   chunks of min(256, q_base) nodes, every
 *                                      node of a chunk planned against the
 *                                      graph as it stood at the chunk's start,
 *                                      then committed in node order
 *   buildSerial     hnsw.zig:477-625   (n_threads <= 1) the same loop with
 *                                      chunks of one node: the plan of node q
 *                                      sees every commit before it, which is
 *                                      exactly the serial loop
 *   pickLevel       hnsw.zig:949-956   floor(-ln(1 - nextFloat) / ln(M)), <= 31
 *   greedySearchLayer hnsw.zig:969-991 strict improvements, list order
 *   searchLayer     hnsw.zig:995-1043  best-first beam of width ef
 *   selectHeuristic hnsw.zig:1048-1083 stable sort by similarity, keep a
 *                                      candidate unless an already chosen
 *                                      neighbour is strictly more similar to it
 *   shrinkNeighbours hnsw.zig:1090-1107
 *   search          hnsw.zig:1117-1150 (query side, for the recall tests)
 *
 * Parity status: UNPINNED. The reference's tests hold no golden graph (they
 * check recall@10 >= 0.9 on 1024 random unit vectors and byte-equal graphs
 * across runs and across thread counts >= 2; tests/test_hnsw.py replays
 * those on this restatement). The reference's two heaps are Zig std's
 * PriorityQueue ordered by similarity alone (Zig 0.16 std, not vendored
 * with the reference and not runnable here), so among candidates with
 * exactly equal similarity its pop order follows the heap's internal
 * layout. This restatement — and the CUDA build — order equal similarities
 * by node id instead (the smaller id is popped first from the frontier,
 * the larger id is evicted first from the beam, and ranks first in the
 * beam's output): graphs can differ from the reference's only after two
 * candidates of one search tie exactly at a point where the order matters.
 * Everything else (the comparisons, which all use similarity alone, the
 * stable sorts, list orders, vec.dot order) follows the reference.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "../include/mvr.h"
#include "mvr_oracle.h"

#define HNSW_CHUNK 256u  /* CHUNK_SIZE, hnsw.zig:272 */
#define HNSW_MAX_LAYERS 32u

typedef struct {
  float sim;
  uint32_t node;
} cand_t;

/* the frontier's and the beam's order: higher similarity first, equal
 * similarities by the smaller node id */
static inline int better(cand_t a, cand_t b) { return a.sim > b.sim || (a.sim == b.sim && a.node < b.node); }

/* ---- binary heaps (any correct heap gives the same pops under a total
 * order) ---- */
typedef struct {
  cand_t* v;
  uint32_t n, cap;
  int max_first; /* 1: pop the best; 0: pop the worst */
} heap_t;

static inline int h_before(const heap_t* h, cand_t a, cand_t b) { return h->max_first ? better(a, b) : better(b, a); }

static int h_push(heap_t* h, cand_t c) {
  if (h->n == h->cap) {
    uint32_t nc = h->cap ? h->cap * 2 : 64;
    cand_t* nv = (cand_t*)realloc(h->v, (size_t)nc * sizeof(cand_t));
    if (!nv) return 0;
    h->v = nv;
    h->cap = nc;
  }
  uint32_t i = h->n++;
  while (i > 0) {
    uint32_t p = (i - 1) >> 1;
    if (!h_before(h, c, h->v[p])) break;
    h->v[i] = h->v[p];
    i = p;
  }
  h->v[i] = c;
  return 1;
}

static cand_t h_pop(heap_t* h) {
  cand_t top = h->v[0];
  cand_t last = h->v[--h->n];
  uint32_t i = 0;
  for (;;) {
    uint32_t c = 2 * i + 1;
    if (c >= h->n) break;
    if (c + 1 < h->n && h_before(h, h->v[c + 1], h->v[c])) ++c;
    if (!h_before(h, h->v[c], last)) break;
    h->v[i] = h->v[c];
    i = c;
  }
  if (h->n) h->v[i] = last;
  return top;
}

/* ---- growable per-(node, layer) adjacency with fixed capacity ----
 * A list never holds more than cap + 1 entries (append, then shrink when it
 * exceeds cap), cap = 2M on layer 0 and M above (hnsw.zig:327-330). */
typedef struct {
  uint32_t n, m, max_level;
  uint32_t cap[HNSW_MAX_LAYERS];
  uint32_t* ids[HNSW_MAX_LAYERS]; /* n x (cap + 1) */
  uint32_t* len[HNSW_MAX_LAYERS];
} adj_t;

static int adj_ensure(adj_t* a, uint32_t level) {
  for (uint32_t L = 0; L <= level; ++L) {
    if (a->ids[L]) continue;
    a->cap[L] = L == 0 ? 2 * a->m : a->m;
    a->ids[L] = (uint32_t*)malloc((size_t)a->n * (a->cap[L] + 1) * sizeof(uint32_t));
    a->len[L] = (uint32_t*)calloc(a->n, sizeof(uint32_t));
    if (!a->ids[L] || !a->len[L]) return 0;
  }
  if (level > a->max_level) a->max_level = level;
  return 1;
}

static inline const uint32_t* adj_list(const adj_t* a, uint32_t node, uint32_t L, uint32_t* cnt) {
  *cnt = a->len[L][node];
  return a->ids[L] + (size_t)node * (a->cap[L] + 1);
}

/* ---- statistics of the last build (design aid) ---- */
static orc_hnsw_stats g_stats;

void orc_hnsw_last_stats(orc_hnsw_stats* out) { *out = g_stats; }

typedef struct {
  uint64_t searches, expansions, sims, accepted, heur_examined, heur_dots;
} local_stats;

/* ---- pickLevel (hnsw.zig:949-956) ---- */
static uint8_t pick_level(orc_rng* r, float m_l) {
  const float u = 1.0f - orc_rng_f32(r);
  const float lvl = floorf(-logf(u) * m_l);
  if (lvl < 0.0f) return 0;
  if (lvl > 31.0f) return 31;
  return (uint8_t)lvl;
}

typedef struct {
  const float* x;
  uint32_t dim;
} vecs_t;

static inline const float* row(const vecs_t* v, uint32_t id) { return v->x + (size_t)id * v->dim; }

/* greedySearchLayer (hnsw.zig:969-991) */
static uint32_t greedy(const vecs_t* v, const adj_t* a, uint32_t entry, const float* q, uint32_t L,
                       local_stats* st) {
  uint32_t cur = entry;
  float cur_sim = orc_dot(q, row(v, cur), v->dim);
  for (;;) {
    int improved = 0;
    uint32_t cnt;
    const uint32_t* list = adj_list(a, cur, L, &cnt);
    for (uint32_t i = 0; i < cnt; ++i) {
      const uint32_t e = list[i];
      const float s = orc_dot(q, row(v, e), v->dim);
      st->sims++;
      if (s > cur_sim) {
        cur_sim = s;
        cur = e;
        improved = 1;
      }
    }
    if (!improved) break;
  }
  return cur;
}

/* searchLayer (hnsw.zig:995-1043): the beam, best first, into out[] (at
 * most ef); returns its size, or -1 when out of memory. */
static int64_t search_layer(const vecs_t* v, const adj_t* a, uint32_t entry, const float* q, uint32_t ef,
                            uint32_t L, uint32_t* visited, uint32_t gen, cand_t* out, local_stats* st) {
  heap_t C = {0}, W = {0};
  C.max_first = 1;
  W.max_first = 0;
  int ok = 1;
  const cand_t e0 = {orc_dot(q, row(v, entry), v->dim), entry};
  st->sims++;
  visited[entry] = gen;
  ok &= h_push(&C, e0);
  ok &= h_push(&W, e0);
  while (ok && C.n) {
    const cand_t c = h_pop(&C);
    const cand_t worst = W.v[0];
    if (c.sim < worst.sim && W.n >= ef) break;
    st->expansions++;
    uint32_t cnt;
    const uint32_t* list = adj_list(a, c.node, L, &cnt);
    for (uint32_t i = 0; i < cnt && ok; ++i) {
      const uint32_t e = list[i];
      if (visited[e] == gen) continue;
      visited[e] = gen;
      const float s = orc_dot(q, row(v, e), v->dim);
      st->sims++;
      if (W.n < ef || s > W.v[0].sim) {
        const cand_t ce = {s, e};
        ok &= h_push(&C, ce);
        ok &= h_push(&W, ce);
        st->accepted++;
        if (W.n > ef) (void)h_pop(&W);
      }
    }
  }
  int64_t n = -1;
  if (ok) {
    n = W.n;
    for (int64_t i = n - 1; i >= 0; --i) out[i] = h_pop(&W); /* worst first -> best at 0 */
  }
  free(C.v);
  free(W.v);
  return n;
}

/* std.mem.sort with candDescSim (stable): insertion sort */
static void sort_desc_stable(cand_t* c, uint32_t n) {
  for (uint32_t i = 1; i < n; ++i) {
    const cand_t x = c[i];
    uint32_t j = i;
    while (j > 0 && c[j - 1].sim < x.sim) {
      c[j] = c[j - 1];
      --j;
    }
    c[j] = x;
  }
}

/* selectHeuristic (hnsw.zig:1048-1083); `c` is sorted in place */
static uint32_t select_heuristic(const vecs_t* v, cand_t* c, uint32_t n, uint32_t m, uint32_t* out,
                                 local_stats* st) {
  sort_desc_stable(c, n);
  uint32_t k = 0;
  for (uint32_t i = 0; i < n; ++i) {
    if (k >= m) break;
    if (st) st->heur_examined++;
    int keep = 1;
    const float* cv = row(v, c[i].node);
    for (uint32_t j = 0; j < k; ++j) {
      const float s = orc_dot(cv, row(v, out[j]), v->dim);
      if (st) st->heur_dots++;
      if (s > c[i].sim) {
        keep = 0;
        break;
      }
    }
    if (keep) out[k++] = c[i].node;
  }
  return k;
}

/* shrinkNeighbours (hnsw.zig:1090-1107) */
static void shrink(const vecs_t* v, uint32_t node, uint32_t* list, uint32_t* len, uint32_t cap, cand_t* scratch,
                   uint32_t* kept) {
  const float* nv = row(v, node);
  for (uint32_t i = 0; i < *len; ++i) {
    scratch[i].sim = orc_dot(nv, row(v, list[i]), v->dim);
    scratch[i].node = list[i];
  }
  const uint32_t k = select_heuristic(v, scratch, *len, cap, kept, NULL);
  memcpy(list, kept, k * sizeof(uint32_t));
  *len = k;
}

/* ---- one node's plan: greedy descent, then per layer the beam and the
 * heuristic (hnsw.zig:735-802) ---- */
typedef struct {
  uint32_t top_layer, l_new;
  uint32_t n_chosen[HNSW_MAX_LAYERS];
  uint32_t* chosen; /* (top_layer + 1) x m */
} plan_t;

typedef struct {
  const vecs_t* v;
  const adj_t* a;
  const uint8_t* levels;
  uint32_t ef, m, snap_entry, snap_max;
  uint32_t q_base, lo, hi;
  plan_t* plans;
  uint32_t* visited;
  uint32_t gen;
  cand_t* beam;
  int err;
  local_stats st;
} worker_t;

static void plan_one(worker_t* w, uint32_t q) {
  const vecs_t* v = w->v;
  const float* qv = row(v, q);
  const uint32_t l_new = w->levels[q];
  uint32_t cur = w->snap_entry;
  if (w->snap_max > l_new)
    for (uint32_t L = w->snap_max; L > l_new; --L) cur = greedy(v, w->a, cur, qv, L, &w->st);
  const uint32_t top = w->snap_max < l_new ? w->snap_max : l_new;
  plan_t* p = &w->plans[q - w->q_base];
  p->top_layer = top;
  p->l_new = l_new;
  for (int L = (int)top; L >= 0; --L) {
    w->gen += 1;
    if (w->gen == 0) {
      memset(w->visited, 0, sizeof(uint32_t) * w->a->n);
      w->gen = 1;
    }
    w->st.searches++;
    const int64_t nb = search_layer(v, w->a, cur, qv, w->ef, (uint32_t)L, w->visited, w->gen, w->beam, &w->st);
    if (nb < 0) {
      w->err = MVR_E_OUT_OF_MEMORY;
      return;
    }
    if (nb > 0) cur = w->beam[0].node; /* first strict maximum = beam[0] */
    p->n_chosen[L] = select_heuristic(v, w->beam, (uint32_t)nb, w->m, p->chosen + (size_t)L * w->m, &w->st);
  }
}

static void* worker_run(void* arg) {
  worker_t* w = (worker_t*)arg;
  for (uint32_t i = w->lo; i < w->hi && !w->err; ++i) plan_one(w, w->q_base + i);
  return NULL;
}

struct orc_hnsw {
  uint32_t n, dim, entry_point, max_level;
  uint8_t* levels;
  uint32_t* offsets[HNSW_MAX_LAYERS]; /* n + 1 each */
  uint32_t* nbrs[HNSW_MAX_LAYERS];
  const float* centroids; /* borrowed copy owned below */
  float* own;
};

void orc_hnsw_free(orc_hnsw* h) {
  if (!h) return;
  for (uint32_t L = 0; L < HNSW_MAX_LAYERS; ++L) {
    free(h->offsets[L]);
    free(h->nbrs[L]);
  }
  free(h->levels);
  free(h->own);
  free(h);
}

static void adj_free(adj_t* a) {
  for (uint32_t L = 0; L < HNSW_MAX_LAYERS; ++L) {
    free(a->ids[L]);
    free(a->len[L]);
  }
}

int orc_hnsw_build(const float* centroids, uint64_t n_floats, uint32_t dim, uint64_t seed, uint32_t ef_c,
                   uint32_t m, uint32_t n_threads, uint32_t workers, orc_hnsw** out) {
  *out = NULL;
  if (dim == 0 || n_floats % dim) return MVR_E_DIM_MISMATCH;
  const uint64_t n64 = n_floats / dim;
  if (n64 == 0) return MVR_E_EMPTY_CORPUS;
  if (n64 > 0xFFFFFFFFull || m == 0) return MVR_E_INVALID_ARGUMENT;
  const uint32_t n = (uint32_t)n64;
  if (workers == 0) workers = 1;

  orc_hnsw* h = (orc_hnsw*)calloc(1, sizeof(orc_hnsw));
  if (!h) return MVR_E_OUT_OF_MEMORY;
  h->n = n;
  h->dim = dim;
  h->own = (float*)malloc(n_floats * sizeof(float));
  h->levels = (uint8_t*)calloc(n, 1);
  if (!h->own || !h->levels) {
    orc_hnsw_free(h);
    return MVR_E_OUT_OF_MEMORY;
  }
  memcpy(h->own, centroids, n_floats * sizeof(float));
  h->centroids = h->own;
  vecs_t v = {h->own, dim};

  const float m_l = 1.0f / logf((float)m);
  orc_rng rng;
  orc_rng_init(&rng, seed);
  adj_t a;
  memset(&a, 0, sizeof a);
  a.n = n;
  a.m = m;
  int st = MVR_OK;
  uint32_t entry = 0, max_level = 0;
  h->levels[0] = pick_level(&rng, m_l);
  max_level = h->levels[0];
  if (!adj_ensure(&a, max_level)) st = MVR_E_OUT_OF_MEMORY;

  worker_t* ws = (worker_t*)calloc(workers, sizeof(worker_t));
  plan_t* plans = (plan_t*)calloc(HNSW_CHUNK, sizeof(plan_t));
  uint32_t* chosen = (uint32_t*)malloc((size_t)HNSW_CHUNK * HNSW_MAX_LAYERS * m * sizeof(uint32_t));
  cand_t* scratch = (cand_t*)malloc((size_t)(2 * m + 2) * sizeof(cand_t));
  uint32_t* kept = (uint32_t*)malloc((size_t)(2 * m + 2) * sizeof(uint32_t));
  pthread_t* th = (pthread_t*)calloc(workers, sizeof(pthread_t));
  if (!ws || !plans || !chosen || !scratch || !kept || !th) st = MVR_E_OUT_OF_MEMORY;
  for (uint32_t t = 0; t < workers && st == MVR_OK; ++t) {
    ws[t].visited = (uint32_t*)calloc(n, sizeof(uint32_t));
    ws[t].beam = (cand_t*)malloc((size_t)(ef_c + 1) * sizeof(cand_t));
    if (!ws[t].visited || !ws[t].beam) st = MVR_E_OUT_OF_MEMORY;
  }
  for (uint32_t i = 0; i < HNSW_CHUNK && st == MVR_OK; ++i) plans[i].chosen = chosen + (size_t)i * HNSW_MAX_LAYERS * m;
  memset(&g_stats, 0, sizeof g_stats);

  uint32_t q_base = 1;
  while (st == MVR_OK && q_base < n) {
    const uint32_t csz = n_threads <= 1 ? 1u : (q_base < HNSW_CHUNK ? q_base : HNSW_CHUNK);
    const uint32_t q_end = (uint64_t)q_base + csz < n ? q_base + csz : n;
    const uint32_t len = q_end - q_base;
    uint32_t max_in_chunk = 0;
    for (uint32_t i = 0; i < len; ++i) {
      h->levels[q_base + i] = pick_level(&rng, m_l);
      if (h->levels[q_base + i] > max_in_chunk) max_in_chunk = h->levels[q_base + i];
    }
    if (!adj_ensure(&a, max_in_chunk > max_level ? max_in_chunk : max_level)) {
      st = MVR_E_OUT_OF_MEMORY;
      break;
    }
    /* plan: the workers split the chunk into contiguous slices */
    const uint32_t nw = workers < len ? workers : len;
    const uint32_t per = (len + nw - 1) / nw;
    for (uint32_t t = 0; t < nw; ++t) {
      worker_t* w = &ws[t];
      w->v = &v;
      w->a = &a;
      w->levels = h->levels;
      w->ef = ef_c;
      w->m = m;
      w->snap_entry = entry;
      w->snap_max = max_level;
      w->q_base = q_base;
      w->lo = t * per;
      w->hi = (t + 1) * per < len ? (t + 1) * per : len;
      w->plans = plans;
      w->err = 0;
    }
    if (nw == 1) {
      worker_run(&ws[0]);
    } else {
      for (uint32_t t = 0; t < nw; ++t) pthread_create(&th[t], NULL, worker_run, &ws[t]);
      for (uint32_t t = 0; t < nw; ++t) pthread_join(th[t], NULL);
    }
    for (uint32_t t = 0; t < nw; ++t)
      if (ws[t].err) st = ws[t].err;
    if (st != MVR_OK) break;
    /* commit in node order (hnsw.zig:891-929) */
    for (uint32_t i = 0; i < len; ++i) {
      const uint32_t q = q_base + i;
      const plan_t* p = &plans[i];
      for (int L = (int)p->top_layer; L >= 0; --L) {
        const uint32_t cap = a.cap[L];
        const uint32_t* ch = p->chosen + (size_t)L * m;
        const uint32_t nc = p->n_chosen[L];
        uint32_t* ql = a.ids[L] + (size_t)q * (cap + 1);
        memcpy(ql + a.len[L][q], ch, nc * sizeof(uint32_t));
        a.len[L][q] += nc;
        for (uint32_t j = 0; j < nc; ++j) {
          const uint32_t r = ch[j];
          uint32_t* rl = a.ids[L] + (size_t)r * (cap + 1);
          rl[a.len[L][r]++] = q;
          if (a.len[L][r] > cap) shrink(&v, r, rl, &a.len[L][r], cap, scratch, kept);
        }
      }
      if (p->l_new > max_level) {
        max_level = p->l_new;
        entry = q;
      }
    }
    q_base = q_end;
  }
  for (uint32_t t = 0; t < workers && ws; ++t) {
    g_stats.searches += ws[t].st.searches;
    g_stats.expansions += ws[t].st.expansions;
    g_stats.sims += ws[t].st.sims;
    g_stats.accepted += ws[t].st.accepted;
    g_stats.heur_examined += ws[t].st.heur_examined;
    g_stats.heur_dots += ws[t].st.heur_dots;
    memset(&ws[t].st, 0, sizeof ws[t].st);
  }
  /* freeze to per-layer CSR (hnsw.zig:427-462) */
  for (uint32_t L = 0; st == MVR_OK && L <= max_level; ++L) {
    h->offsets[L] = (uint32_t*)malloc(((size_t)n + 1) * sizeof(uint32_t));
    uint64_t tot = 0;
    for (uint32_t i = 0; i < n; ++i) tot += a.len[L][i];
    h->nbrs[L] = (uint32_t*)malloc((tot ? tot : 1) * sizeof(uint32_t));
    if (!h->offsets[L] || !h->nbrs[L]) {
      st = MVR_E_OUT_OF_MEMORY;
      break;
    }
    h->offsets[L][0] = 0;
    for (uint32_t i = 0; i < n; ++i) {
      const uint32_t c = a.len[L][i];
      memcpy(h->nbrs[L] + h->offsets[L][i], a.ids[L] + (size_t)i * (a.cap[L] + 1), c * sizeof(uint32_t));
      h->offsets[L][i + 1] = h->offsets[L][i] + c;
    }
  }
  h->entry_point = entry;
  h->max_level = max_level;
  for (uint32_t t = 0; t < workers && ws; ++t) {
    free(ws[t].visited);
    free(ws[t].beam);
  }
  free(ws);
  free(plans);
  free(chosen);
  free(scratch);
  free(kept);
  free(th);
  adj_free(&a);
  if (st != MVR_OK) {
    orc_hnsw_free(h);
    return st;
  }
  *out = h;
  return MVR_OK;
}

void orc_hnsw_info(const orc_hnsw* h, uint32_t* n, uint32_t* entry_point, uint32_t* max_level) {
  *n = h->n;
  *entry_point = h->entry_point;
  *max_level = h->max_level;
}

void orc_hnsw_levels(const orc_hnsw* h, uint8_t* out) { memcpy(out, h->levels, h->n); }

uint64_t orc_hnsw_layer_size(const orc_hnsw* h, uint32_t L) {
  return L <= h->max_level ? h->offsets[L][h->n] : 0;
}

void orc_hnsw_layer(const orc_hnsw* h, uint32_t L, uint32_t* offsets, uint32_t* nbrs) {
  memcpy(offsets, h->offsets[L], ((size_t)h->n + 1) * sizeof(uint32_t));
  memcpy(nbrs, h->nbrs[L], (size_t)h->offsets[L][h->n] * sizeof(uint32_t));
}

/* ---- search over a frozen CSR graph (hnsw.zig:1117-1237) ----
 * The graph is given as plain arrays so the tests can search the CUDA
 * build's output with the same code. */
int orc_hnsw_search_csr(const float* centroids, uint32_t n, uint32_t dim, uint32_t entry_point, uint32_t max_level,
                        const uint32_t* const* offsets, const uint32_t* const* nbrs, const float* query,
                        uint32_t k, uint32_t ef, uint32_t* out, uint32_t* written) {
  *written = 0;
  if (k == 0) return MVR_OK;
  const uint32_t ef_eff = ef > k ? ef : k;
  vecs_t v = {centroids, dim};
  /* a read-only adj_t view over the CSR: the list of node i at layer L is
   * nbrs[L][offsets[L][i] .. offsets[L][i+1]] */
  uint32_t cur = entry_point;
  for (uint32_t L = max_level; L > 0; --L) {
    float cur_sim = orc_dot(query, row(&v, cur), dim);
    for (;;) {
      int improved = 0;
      const uint32_t b = offsets[L][cur], e = offsets[L][cur + 1];
      for (uint32_t i = b; i < e; ++i) {
        const float s = orc_dot(query, row(&v, nbrs[L][i]), dim);
        if (s > cur_sim) {
          cur_sim = s;
          cur = nbrs[L][i];
          improved = 1;
        }
      }
      if (!improved) break;
    }
  }
  uint32_t* visited = (uint32_t*)calloc(n, sizeof(uint32_t));
  heap_t C = {0}, W = {0};
  C.max_first = 1;
  int ok = visited != NULL;
  if (ok) {
    const cand_t e0 = {orc_dot(query, row(&v, cur), dim), cur};
    visited[cur] = 1;
    ok &= h_push(&C, e0);
    ok &= h_push(&W, e0);
  }
  while (ok && C.n) {
    const cand_t c = h_pop(&C);
    if (c.sim < W.v[0].sim && W.n >= ef_eff) break;
    const uint32_t b = offsets[0][c.node], e = offsets[0][c.node + 1];
    for (uint32_t i = b; i < e && ok; ++i) {
      const uint32_t x = nbrs[0][i];
      if (visited[x]) continue;
      visited[x] = 1;
      const float s = orc_dot(query, row(&v, x), dim);
      if (W.n < ef_eff || s > W.v[0].sim) {
        const cand_t cx = {s, x};
        ok &= h_push(&C, cx);
        ok &= h_push(&W, cx);
        if (W.n > ef_eff) (void)h_pop(&W);
      }
    }
  }
  if (ok) {
    const uint32_t nb = W.n;
    cand_t* tmp = (cand_t*)malloc((size_t)(nb ? nb : 1) * sizeof(cand_t));
    if (!tmp) ok = 0;
    for (int64_t i = (int64_t)nb - 1; ok && i >= 0; --i) tmp[i] = h_pop(&W);
    const uint32_t want = k < nb ? k : nb;
    for (uint32_t i = 0; ok && i < want; ++i) out[i] = tmp[i].node;
    if (ok) *written = want;
    free(tmp);
  }
  free(C.v);
  free(W.v);
  free(visited);
  return ok ? MVR_OK : MVR_E_OUT_OF_MEMORY;
}

int orc_hnsw_search(const orc_hnsw* h, const float* query, uint32_t k, uint32_t ef, uint32_t* out,
                    uint32_t* written) {
  return orc_hnsw_search_csr(h->centroids, h->n, h->dim, h->entry_point, h->max_level,
                             (const uint32_t* const*)h->offsets, (const uint32_t* const*)h->nbrs, query, k, ef, out,
                             written);
}

/* vec.normalizeRowsInPlace (src/util/vec.zig:185-230): |v|^2 in the dot
 * order, then v * (1 / sqrt(|v|^2)); zero rows stay zero */
void orc_normalize_rows(float* v, uint64_t n_rows, uint32_t dim) {
  for (uint64_t r = 0; r < n_rows; ++r) {
    float* x = v + r * dim;
    const float ns = orc_dot(x, x, dim);
    if (ns == 0.0f) continue;
    const float inv = 1.0f / sqrtf(ns);
    for (uint32_t i = 0; i < dim; ++i) x[i] = x[i] * inv;
  }
}
