// tac_budget.cpp — TAC budget phases 1-4 (host integer/float logic).
//
// Reference: src/tac/tac.zig:80-402 (classifyToken, allocateTail,
// dampedWeight, dampedPhase2, boundPhase3, reconcilePhase4,
// allocateBudgets). O(vocabulary) work that runs once per build between the
// device spread pass and the device per-token k-means.
#include <cmath>
#include <algorithm>
#include <cstdint>
#include <vector>

#include "../../include/mvr.h"
#include "tac_engine.h"

namespace mvr {
namespace {

enum Tier { kEmpty, kMicro, kSmall, kActive };

inline Tier classify(uint32_t n, uint32_t mu, uint32_t tau) {
  if (n == 0) return kEmpty;
  if (n < mu) return kMicro;
  if (n < tau) return kSmall;
  return kActive;
}

}  // namespace

int tac_allocate_budgets_host(const uint32_t* freqs, const float* spreads, uint32_t* kappa,
                              float* frac, uint64_t n, uint32_t kappa_total, uint32_t mu,
                              uint32_t tau, uint32_t eps, uint32_t theta) {
  // Phase 1 — tail (tac.zig:97-125)
  if (mu == 0 || tau == 0 || mu >= tau) return MVR_E_INVALID_THRESHOLDS;
  uint32_t tail = 0;
  for (uint64_t j = 0; j < n; ++j) {
    switch (classify(freqs[j], mu, tau)) {
      case kMicro: kappa[j] = 1; tail += 1; break;
      case kSmall: kappa[j] = 2; tail += 2; break;
      default: kappa[j] = 0; break;
    }
  }
  if (tail > kappa_total) return MVR_E_BUDGET_TOO_SMALL;
  const uint32_t budget = kappa_total - tail;

  // Phase 2 — damped proportional allocation (tac.zig:157-210)
  for (uint64_t j = 0; j < n; ++j) frac[j] = 0.f;
  double sum_w = 0.0;
  uint32_t n_active = 0;
  for (uint64_t j = 0; j < n; ++j) {
    if (classify(freqs[j], mu, tau) != kActive) continue;
    const float w = std::sqrt((float)freqs[j]) * spreads[j];
    if (!std::isfinite(w) || w < 0.f) return MVR_E_INVALID_THRESHOLDS;
    sum_w += (double)w;
    ++n_active;
  }
  if (n_active > 0) {
    if (sum_w <= 0.0) {
      const uint32_t base = budget / n_active;
      uint32_t left = budget - base * n_active;
      for (uint64_t j = 0; j < n; ++j) {
        if (classify(freqs[j], mu, tau) != kActive) continue;
        kappa[j] = base + (left > 0 ? 1u : 0u);
        if (left > 0) --left;
      }
    } else {
      const double bf = (double)budget;
      for (uint64_t j = 0; j < n; ++j) {
        if (classify(freqs[j], mu, tau) != kActive) continue;
        const double w = (double)(std::sqrt((float)freqs[j]) * spreads[j]);
        const double target = (w / sum_w) * bf;
        const uint32_t fl = (uint32_t)std::floor(target);
        kappa[j] = fl;
        frac[j] = (float)(target - (double)fl);
      }
    }
  }

  // Phase 3 — floor and cap (tac.zig:228-248)
  if (eps == 0 || theta == 0) return MVR_E_INVALID_THRESHOLDS;
  if ((uint64_t)tau < (uint64_t)eps * theta) return MVR_E_INVALID_THRESHOLDS;
  for (uint64_t j = 0; j < n; ++j) {
    if (classify(freqs[j], mu, tau) != kActive) continue;
    const uint32_t cap = freqs[j] / theta;
    if (kappa[j] < eps) kappa[j] = eps;
    if (kappa[j] > cap) kappa[j] = cap;
  }

  // Phase 4 — largest-remainder reconciliation (tac.zig:281-376). The
  // reference moves one unit per round to the arg-max (surplus) or arg-min
  // (deficit) fractional remainder among the eligible active tokens, first
  // index on ties. A round never changes frac, so the same token wins every
  // round until it leaves the eligible set (reaches its cap, or its floor
  // eps); visiting the eligible tokens once in (frac, index) order and
  // moving all their units at once gives the same result in O(n log n).
  uint64_t cur = 0;
  for (uint64_t j = 0; j < n; ++j) cur += kappa[j];
  if (cur == kappa_total) return MVR_OK;
  std::vector<uint32_t> order;
  if (cur < kappa_total) {
    uint64_t remaining = kappa_total - cur;
    for (uint64_t j = 0; j < n; ++j)
      if (classify(freqs[j], mu, tau) == kActive && kappa[j] < freqs[j] / theta && !std::isnan(frac[j]))
        order.push_back((uint32_t)j);
    std::stable_sort(order.begin(), order.end(), [&](uint32_t a, uint32_t b) { return frac[a] > frac[b]; });
    for (uint32_t j : order) {
      if (remaining == 0) break;
      const uint64_t room = freqs[j] / theta - kappa[j];
      const uint64_t take = room < remaining ? room : remaining;
      kappa[j] += (uint32_t)take;
      remaining -= take;
    }
    return remaining == 0 ? MVR_OK : MVR_E_BUDGET_TOO_LARGE;
  }
  uint64_t excess = cur - kappa_total;
  for (uint64_t j = 0; j < n; ++j)
    if (classify(freqs[j], mu, tau) == kActive && kappa[j] > eps && frac[j] < INFINITY)
      order.push_back((uint32_t)j);
  std::stable_sort(order.begin(), order.end(), [&](uint32_t a, uint32_t b) { return frac[a] < frac[b]; });
  for (uint32_t j : order) {
    if (excess == 0) break;
    const uint64_t room = kappa[j] - eps;
    const uint64_t take = room < excess ? room : excess;
    kappa[j] -= (uint32_t)take;
    excess -= take;
  }
  // then small tokens 2 -> 1, then micro tokens 1 -> 0, in index order
  for (uint64_t j = 0; j < n && excess > 0; ++j)
    if (classify(freqs[j], mu, tau) == kSmall && kappa[j] == 2) {
      kappa[j] = 1;
      --excess;
    }
  for (uint64_t j = 0; j < n && excess > 0; ++j)
    if (classify(freqs[j], mu, tau) == kMicro && kappa[j] == 1) {
      kappa[j] = 0;
      --excess;
    }
  return excess == 0 ? MVR_OK : MVR_E_BUDGET_TOO_SMALL;
}

uint64_t tac_token_work(uint32_t n, uint32_t k) {
  if (n == 0 || k == 0) return 0;
  return k < n ? (uint64_t)n * ((uint64_t)k + 1) : (uint64_t)n;
}

void tac_partition_tokens_host(const uint32_t* freqs, const uint32_t* kappa, uint64_t n, uint32_t ranks,
                               uint32_t* owner) {
  std::vector<uint32_t> order;
  for (uint64_t j = 0; j < n; ++j) {
    owner[j] = 0;
    if (tac_token_work(freqs[j], kappa[j]) > 0) order.push_back((uint32_t)j);
  }
  // heaviest first, ties in token order; each to the least-loaded rank
  // (ties: the lowest rank)
  std::stable_sort(order.begin(), order.end(), [&](uint32_t a, uint32_t b) {
    return tac_token_work(freqs[a], kappa[a]) > tac_token_work(freqs[b], kappa[b]);
  });
  std::vector<uint64_t> load(ranks, 0);
  for (uint32_t j : order) {
    uint32_t best = 0;
    for (uint32_t r = 1; r < ranks; ++r)
      if (load[r] < load[best]) best = r;
    owner[j] = best;
    load[best] += tac_token_work(freqs[j], kappa[j]);
  }
}

}  // namespace mvr

extern "C" {

void mvr_clustering_params_default(mvr_clustering_params* p, uint32_t kappa_total, uint64_t seed) {
  if (!p) return;
  p->kappa_total = kappa_total;
  p->mu = 128;   // constants.TAC_MU
  p->tau = 256;  // constants.TAC_TAU
  p->epsilon = 4;
  p->theta = 39;
  p->max_iters = 25;
  p->tol = 1e-4f;
  p->seed = seed;
  p->n_threads = 1;
}

int mvr_tac_allocate_budgets(const uint32_t* freqs, const float* spreads, uint32_t* kappa,
                             float* frac, uint64_t n, uint32_t kappa_total,
                             const mvr_clustering_params* p) {
  if (!p || (n > 0 && (!freqs || !spreads || !kappa || !frac))) return MVR_E_INVALID_ARGUMENT;
  return mvr::tac_allocate_budgets_host(freqs, spreads, kappa, frac, n, kappa_total, p->mu, p->tau,
                                        p->epsilon, p->theta);
}

int mvr_tac_partition_tokens(const uint32_t* freqs, const uint32_t* kappa, uint64_t n, uint32_t n_ranks,
                             uint32_t* owner_out) {
  if (n_ranks == 0 || (n > 0 && (!freqs || !kappa || !owner_out))) return MVR_E_INVALID_ARGUMENT;
  mvr::tac_partition_tokens_host(freqs, kappa, n, n_ranks, owner_out);
  return MVR_OK;
}

}  // extern "C"
