// Seeded synthetic tensors for the benchmark configurations.
//
// Coordinates: the first `nnz` DISTINCT linear keys of a counter-based draw
// sequence (draw d uses counter d), so duplicates never occur (the order-3
// dense-tile kernel of the reference stores rather than sums, so parity
// requires distinct coordinates).  Values are a pure function of the key.
// Output nonzeros are sorted by linear key (mode 0 slowest).
#include <omp.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <functional>
#include <parallel/algorithm>
#include <string>
#include <vector>

#include "coo.hpp"
#include "rng.hpp"

namespace cptc {

static thread_local std::string g_host_err;

static int host_fail(int code, const std::string& msg) {
  g_host_err = msg;
  return code;
}

void set_host_error(const char* msg) { g_host_err = msg ? msg : ""; }

int host_threads() {
  if (const char* e = std::getenv("CPTC_HOST_THREADS")) {
    const int n = std::atoi(e);
    if (n > 0) return n;
  }
  return omp_get_num_procs();
}

bool coo_alloc(cptc_coo* t, int order, uint64_t nnz) {
  std::memset(t, 0, sizeof(*t));
  t->order = order;
  t->nnz = nnz;
  const size_t n = nnz ? (size_t)nnz : 1;
  for (int m = 0; m < order; ++m) {
    t->idx[m] = (uint32_t*)std::malloc(n * sizeof(uint32_t));
    if (!t->idx[m]) return false;
  }
  t->vals = (double*)std::malloc(n * sizeof(double));
  return t->vals != nullptr;
}

// ---------------------------------------------------------------------------
// Distinct-key engine: keeps (key, first draw id) sorted by key; draws in
// batches until at least `target` distinct keys exist, then keeps the
// `target` keys whose first occurrence came earliest.  `draw(d)` returns the
// key of draw d, or UINT64_MAX to reject the draw.
// ---------------------------------------------------------------------------
struct KeyId {
  uint64_t key, id;
};

static std::vector<uint64_t> first_distinct(
    uint64_t target, const std::function<uint64_t(uint64_t)>& draw,
    uint64_t key_space) {
  if (target == 0) return {};
  if (key_space != 0 && target > key_space) return {};
  const uint64_t batch = std::max<uint64_t>((target + 3) / 4, 65536);
  const int nt = host_threads();
  // Buffers are sized once: repeated allocation of multi-GB vectors costs
  // more in page faults than the sort itself.
  std::vector<KeyId> have, merged, b;
  have.reserve(target + batch);
  merged.reserve(target + batch);
  b.resize(batch);
  uint64_t d0 = 0;
  int guard = 0;
  while (have.size() < target && guard++ < 4096) {
    b.resize(batch);
#pragma omp parallel for num_threads(nt) schedule(static)
    for (int64_t i = 0; i < (int64_t)batch; ++i)
      b[i] = KeyId{draw(d0 + (uint64_t)i), d0 + (uint64_t)i};
    d0 += batch;
    b.erase(std::remove_if(b.begin(), b.end(),
                           [](const KeyId& x) { return x.key == UINT64_MAX; }),
            b.end());
    __gnu_parallel::sort(b.begin(), b.end(), [](const KeyId& x, const KeyId& y) {
      return x.key != y.key ? x.key < y.key : x.id < y.id;
    });
    b.erase(std::unique(b.begin(), b.end(),
                        [](const KeyId& x, const KeyId& y) { return x.key == y.key; }),
            b.end());
    merged.clear();
    size_t i = 0, j = 0;
    while (i < have.size() || j < b.size()) {
      if (j == b.size() || (i < have.size() && have[i].key < b[j].key)) {
        merged.push_back(have[i++]);
      } else if (i == have.size() || b[j].key < have[i].key) {
        merged.push_back(b[j++]);
      } else {  // same key: the earlier batch holds the smaller draw id
        merged.push_back(have[i++]);
        ++j;
      }
    }
    have.swap(merged);
  }
  if (have.size() < target) return {};
  if (have.size() > target) {
    std::vector<uint64_t> ids(have.size());
    for (size_t i = 0; i < have.size(); ++i) ids[i] = have[i].id;
    std::nth_element(ids.begin(), ids.begin() + (target - 1), ids.end());
    const uint64_t cut = ids[target - 1];
    have.erase(std::remove_if(have.begin(), have.end(),
                              [cut](const KeyId& x) { return x.id > cut; }),
               have.end());
  }
  std::vector<uint64_t> keys(have.size());
  for (size_t i = 0; i < have.size(); ++i) keys[i] = have[i].key;
  return keys;
}

// Mixed-radix decode of sorted keys into coordinate arrays.
static void decode_keys(const std::vector<uint64_t>& keys, cptc_coo* t) {
  const int N = t->order;
  const int nt = host_threads();
#pragma omp parallel for num_threads(nt) schedule(static)
  for (int64_t e = 0; e < (int64_t)keys.size(); ++e) {
    uint64_t k = keys[e];
    for (int m = N - 1; m >= 0; --m) {
      t->idx[m][e] = (uint32_t)(k % t->dims[m]);
      k /= t->dims[m];
    }
  }
}

// Zipf(alpha) sampler over n ranks mapped through a random permutation.
struct ZipfMode {
  std::vector<double> cum;  // unnormalised cumulative weights
  std::vector<uint32_t> perm;
  double total = 0.0;
  void init(uint64_t n, double alpha, uint64_t seed, uint64_t perm_stream) {
    cum.resize(n);
    double s = 0.0;
    for (uint64_t k = 0; k < n; ++k) {
      s += std::pow((double)(k + 1), -alpha);
      cum[k] = s;
    }
    total = s;
    perm.resize(n);
    for (uint64_t i = 0; i < n; ++i) perm[i] = (uint32_t)i;
    for (uint64_t i = n - 1; i > 0; --i) {  // Fisher-Yates
      const uint64_t j = rng_below(seed, perm_stream, i, i + 1);
      std::swap(perm[i], perm[j]);
    }
  }
  uint32_t sample(double u) const {
    const double x = u * total;
    size_t r = (size_t)(std::upper_bound(cum.begin(), cum.end(), x) - cum.begin());
    if (r >= cum.size()) r = cum.size() - 1;
    return perm[r];
  }
};

static uint64_t key_space_of(const cptc_coo* t) {
  unsigned __int128 s = 1;
  for (int m = 0; m < t->order; ++m) s *= t->dims[m];
  if (s > (unsigned __int128)UINT64_MAX / 2) return 0;
  return (uint64_t)s;
}

// Values of a planted rank-Rp CP model at each key, plus Gaussian noise with
// standard deviation noise_frac * rms(model values).
static void planted_values(cptc_coo* t, const std::vector<uint64_t>& keys, int Rp,
                           double noise_frac, uint64_t seed) {
  const int N = t->order;
  std::vector<std::vector<double>> F(N);
  for (int m = 0; m < N; ++m) {
    F[m].resize(t->dims[m] * (size_t)Rp);
    for (size_t i = 0; i < F[m].size(); ++i) F[m][i] = rng_unit(seed, 300 + m, i);
  }
  const int nt = host_threads();
  // Sum of squares over fixed blocks, then the block sums in order: the
  // result does not depend on the thread count.
  const int64_t nnz = (int64_t)t->nnz, blk = 65536;
  std::vector<double> part((size_t)((nnz + blk - 1) / blk), 0.0);
#pragma omp parallel for num_threads(nt) schedule(static)
  for (int64_t b = 0; b < (int64_t)part.size(); ++b) {
    double s = 0.0;
    for (int64_t e = b * blk; e < std::min(nnz, (b + 1) * blk); ++e) {
      double x = 0.0;
      for (int r = 0; r < Rp; ++r) {
        double p = 1.0;
        for (int m = 0; m < N; ++m) p *= F[m][(size_t)t->idx[m][e] * Rp + r];
        x += p;
      }
      t->vals[e] = x;
      s += x * x;
    }
    part[b] = s;
  }
  double ss = 0.0;
  for (double s : part) ss += s;
  const double sigma = noise_frac * std::sqrt(ss / (double)(t->nnz ? t->nnz : 1));
#pragma omp parallel for num_threads(nt) schedule(static)
  for (int64_t e = 0; e < (int64_t)t->nnz; ++e)
    t->vals[e] += sigma * rng_normal(seed, 400, keys[e]);
}

static void kind_values(cptc_coo* t, const std::vector<uint64_t>& keys, int kind,
                        uint64_t seed) {
  const int nt = host_threads();
#pragma omp parallel for num_threads(nt) schedule(static)
  for (int64_t e = 0; e < (int64_t)t->nnz; ++e) {
    const uint64_t k = keys[e];
    double v;
    switch (kind) {
      case 1: v = std::exp(rng_normal(seed, 200, k)); break;
      case 2: v = rng_normal(seed, 200, k); break;
      case 3: v = 1.0 + (double)rng_poisson(seed, 200, k, 3.0); break;
      default: v = 1.0 - rng_unit(seed, 200, k); break;  // (0, 1]
    }
    t->vals[e] = v;
  }
}

static int finish(cptc_coo* out, int order, const uint64_t* dims,
                  const std::vector<uint64_t>& keys) {
  if (!coo_alloc(out, order, keys.size())) {
    cptc_coo_free(out);
    return host_fail(-3, "out of host memory");
  }
  for (int m = 0; m < order; ++m) out->dims[m] = dims[m];
  decode_keys(keys, out);
  return 0;
}

}  // namespace cptc

using namespace cptc;

extern "C" {

const char* cptc_host_last_error(void) { return g_host_err.c_str(); }

void cptc_coo_free(cptc_coo* t) {
  if (!t) return;
  for (int m = 0; m < CPTC_MAX_ORDER; ++m) {
    std::free(t->idx[m]);
    t->idx[m] = nullptr;
  }
  std::free(t->vals);
  t->vals = nullptr;
  t->nnz = 0;
}

int cptc_gen_uniform(int order, const uint64_t* dims, uint64_t nnz, uint64_t seed,
                     int value_kind, cptc_coo* out) {
  return host_guard(out, [&]() -> int {
    if (!out || !dims || order < 1 || order > CPTC_MAX_ORDER)
      return host_fail(-2, "bad order");
    std::memset(out, 0, sizeof(*out));
    cptc_coo shape{};
    shape.order = order;
    for (int m = 0; m < order; ++m) {
      if (dims[m] == 0 || dims[m] > UINT32_MAX) return host_fail(-2, "bad dims");
      shape.dims[m] = dims[m];
    }
    const uint64_t space = key_space_of(&shape);
    if (space == 0) return host_fail(-2, "key space exceeds 2^63");
    if (nnz > space) return host_fail(-2, "nnz exceeds the number of cells");
    auto keys = first_distinct(
        nnz, [&](uint64_t d) { return rng_below(seed, 1, d, space); }, space);
    if (keys.size() != nnz) return host_fail(-4, "generator did not converge");
    int rc = finish(out, order, dims, keys);
    if (rc) return rc;
    kind_values(out, keys, value_kind, seed);
    return 0;
  });
}

int cptc_gen_config(int cfg, double nnz_scale, uint64_t seed, cptc_coo* out) {
  return host_guard(out, [&]() -> int {
    if (!out) return host_fail(-2, "null output");
    std::memset(out, 0, sizeof(*out));
    if (!(nnz_scale > 0.0)) return host_fail(-2, "nnz_scale must be positive");
    auto scaled = [&](double n) { return (uint64_t)std::llround(n * nnz_scale); };
  
    if (cfg == 1 || cfg == 2) {
      // Uniform distinct cells, planted low-rank values plus Gaussian noise.
      const uint64_t n = (cfg == 1) ? 128 : 256;
      const uint64_t dims[3] = {n, n, n};
      const uint64_t nnz = scaled(cfg == 1 ? 200000.0 : 15100000.0);
      const uint64_t space = n * n * n;
      if (nnz > space) return host_fail(-2, "nnz exceeds cells");
      auto keys = first_distinct(
          nnz, [&](uint64_t d) { return rng_below(seed, 1, d, space); }, space);
      if (keys.size() != nnz) return host_fail(-4, "generator did not converge");
      int rc = finish(out, 3, dims, keys);
      if (rc) return rc;
      planted_values(out, keys, cfg == 1 ? 8 : 32, cfg == 1 ? 0.01 : 0.05, seed);
      return 0;
    }
  
    if (cfg == 3) {
      // 40% of nonzeros inside random aligned 16^3 tiles with per-tile fill
      // U[0.05, 0.6]; 60% uniform residual outside those cells; values U(0,1].
      const uint64_t n = 512, nb = n / 16, space = n * n * n;
      const uint64_t dims[3] = {n, n, n};
      const uint64_t n_tile = scaled(8000000.0), n_res = scaled(12000000.0);
      std::vector<uint64_t> tile_keys;
      tile_keys.reserve(n_tile);
      std::vector<char> used(nb * nb * nb, 0);
      std::vector<uint16_t> pos(4096);
      for (uint64_t t = 0; tile_keys.size() < n_tile && t < 100 * nb * nb * nb; ++t) {
        const uint64_t tid = rng_below(seed, 20, t, nb * nb * nb);
        if (used[tid]) continue;
        used[tid] = 1;
        const double f = 0.05 + 0.55 * rng_unit(seed, 21, t);
        uint64_t cnt = (uint64_t)std::max<long long>(1, std::llround(f * 4096.0));
        cnt = std::min<uint64_t>(cnt, n_tile - tile_keys.size());
        for (int i = 0; i < 4096; ++i) pos[i] = (uint16_t)i;
        const uint64_t bi = tid / (nb * nb), bj = (tid / nb) % nb, bk = tid % nb;
        for (uint64_t i = 0; i < cnt; ++i) {  // partial Fisher-Yates
          const uint64_t j = i + rng_below(seed, 22, t * 4096 + i, 4096 - i);
          std::swap(pos[i], pos[j]);
          const uint64_t li = pos[i] >> 8, lj = (pos[i] >> 4) & 15, lk = pos[i] & 15;
          tile_keys.push_back(((bi * 16 + li) * n + (bj * 16 + lj)) * n + bk * 16 + lk);
        }
      }
      __gnu_parallel::sort(tile_keys.begin(), tile_keys.end());
      auto res = first_distinct(
          n_res,
          [&](uint64_t d) {
            const uint64_t k = rng_below(seed, 23, d, space);
            return std::binary_search(tile_keys.begin(), tile_keys.end(), k) ? UINT64_MAX
                                                                              : k;
          },
          space);
      if (res.size() != n_res) return host_fail(-4, "generator did not converge");
      std::vector<uint64_t> keys(tile_keys.size() + res.size());
      std::merge(tile_keys.begin(), tile_keys.end(), res.begin(), res.end(), keys.begin());
      int rc = finish(out, 3, dims, keys);
      if (rc) return rc;
      kind_values(out, keys, 0, seed);
      return 0;
    }
  
    if (cfg == 4 || cfg == 5) {
      // Per-mode Zipf indices over a random permutation of each mode.
      const int N = (cfg == 4) ? 3 : 4;
      const uint64_t d4[3] = {12092, 9184, 28818};
      const uint64_t d5[4] = {183, 24, 1140, 1717};
      const uint64_t* dims = (cfg == 4) ? d4 : d5;
      const double alpha = (cfg == 4) ? 1.1 : 1.2;
      const uint64_t nnz = scaled(cfg == 4 ? 76900000.0 : 3300000.0);
      std::vector<ZipfMode> z(N);
      for (int m = 0; m < N; ++m) z[m].init(dims[m], alpha, seed, 100 + m);
      cptc_coo shape{};
      shape.order = N;
      for (int m = 0; m < N; ++m) shape.dims[m] = dims[m];
      const uint64_t space = key_space_of(&shape);
      auto keys = first_distinct(
          nnz,
          [&](uint64_t d) {
            uint64_t k = 0;
            for (int m = 0; m < N; ++m) k = k * dims[m] + z[m].sample(rng_unit(seed, 10 + m, d));
            return k;
          },
          space);
      if (keys.size() != nnz) return host_fail(-4, "generator did not converge");
      int rc = finish(out, N, dims, keys);
      if (rc) return rc;
      kind_values(out, keys, cfg == 4 ? 1 : 3, seed);
      return 0;
    }
    return host_fail(-2, "unknown config (1..5)");
  });
}

}  // extern "C"
