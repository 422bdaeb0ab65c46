// Index relabelling: CADR (degree descending) and HITS hub scores.
#include "reorder.hpp"

#include <omp.h>

#include <algorithm>
#include <cstdio>
#include <numeric>
#include <unordered_map>

#include "coo.hpp"

namespace cptc {

namespace {

inline uint64_t splitbit_hash(uint64_t x) {  // 64-bit finaliser (splitmix64)
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

// Per-mode degree counts with all host threads.
std::vector<size_t> degrees(uint64_t dim, uint64_t nnz, const uint32_t* idx) {
  const int nt = host_threads();
  std::vector<std::vector<size_t>> part(nt, std::vector<size_t>(dim, 0));
#pragma omp parallel num_threads(nt)
  {
    std::vector<size_t>& d = part[omp_get_thread_num()];
#pragma omp for schedule(static)
    for (int64_t e = 0; e < (int64_t)nnz; ++e) d[idx[e]]++;
  }
  std::vector<size_t> deg(dim, 0);
  for (auto& p : part)
    for (uint64_t i = 0; i < dim; ++i) deg[i] += p[i];
  return deg;
}

void cadr_tiebreak(uint64_t dim, uint64_t nnz, const uint32_t* idx, std::vector<uint32_t>& rank) {
  const std::vector<size_t> d = degrees(dim, nnz, idx);
  std::vector<uint32_t> ord(dim);
  for (uint64_t i = 0; i < dim; ++i) ord[i] = (uint32_t)i;
  std::sort(ord.begin(), ord.end(),
            [&](uint32_t a, uint32_t b) { return d[a] != d[b] ? d[a] > d[b] : a < b; });
  rank.assign(dim, 0);
  for (uint64_t i = 0; i < dim; ++i) rank[ord[i]] = (uint32_t)i;
}

// HITS scores: s_m(i) = sum over sampled nonzeros at i of prod_{q != m}
// s_q(o_q), max-normalised, T rounds; sort desc, ties by index.  Sums run in
// the reference's order (sample stride, modes ascending), sequentially, so
// the scores and hence the ranks are bit-identical to it.
void hits(int N, const uint64_t* dims, uint64_t nnz, const uint32_t* const* idx, int rounds,
          uint64_t budget, std::vector<std::vector<uint32_t>>& rank) {
  const uint64_t stride = (nnz > budget && budget > 0) ? (nnz / budget) : 1;
  std::vector<std::vector<double>> s(N), ns(N);
  for (int m = 0; m < N; ++m) s[m].assign(dims[m], 1.0);
  for (int it = 0; it < rounds; ++it) {
    for (int m = 0; m < N; ++m) ns[m].assign(dims[m], 0.0);
    for (uint64_t e = 0; e < nnz; e += stride)
      for (int m = 0; m < N; ++m) {
        double p = 1.0;
        for (int q = 0; q < N; ++q)
          if (q != m) p *= s[q][idx[q][e]];
        ns[m][idx[m][e]] += p;
      }
    for (int m = 0; m < N; ++m) {
      double mx = 0.0;
      for (double v : ns[m]) mx = std::max(mx, v);
      if (mx > 0.0)
        for (double& v : ns[m]) v /= mx;
      s[m].swap(ns[m]);
    }
  }
  rank.assign(N, {});
  for (int m = 0; m < N; ++m) {
    std::vector<uint32_t> ord(dims[m]);
    for (uint64_t i = 0; i < dims[m]; ++i) ord[i] = (uint32_t)i;
    std::sort(ord.begin(), ord.end(), [&](uint32_t a, uint32_t b) {
      const double sa = s[m][a], sb = s[m][b];
      return (sa != sb) ? (sa > sb) : (a < b);
    });
    rank[m].assign(dims[m], 0);
    for (uint64_t i = 0; i < dims[m]; ++i) rank[m][ord[i]] = (uint32_t)i;
  }
}

// Probed dense-tile fill of the (optionally relabelled) tensor over modes
// 0,1,2 with the outer modes folded into the key (src/generic.cu:1208-1233).
double probe_fill(int N, const uint64_t* dims, uint64_t nnz, const uint32_t* const* idx,
                  const std::vector<std::vector<uint32_t>>* rk) {
  const uint64_t budget = 2000000;
  const uint64_t st = (nnz > budget) ? (nnz / budget) : 1;
  const uint64_t nbj = (dims[1] + 15) / 16, nbk = (dims[2] + 15) / 16;
  auto at = [&](int m, uint64_t e) -> uint64_t {
    return rk ? (*rk)[m][idx[m][e]] : idx[m][e];
  };
  std::unordered_map<uint64_t, uint32_t> cnt;
  cnt.reserve(budget / 2 + 1);
  for (uint64_t e = 0; e < nnz; e += st) {
    const uint64_t tile = ((at(0, e) / 16) * nbj + at(1, e) / 16) * nbk + at(2, e) / 16;
    uint64_t o = 0;
    for (int m = 3; m < N; ++m) o = o * 1000003ull + at(m, e);
    ++cnt[splitbit_hash(tile ^ (o * 0x9E3779B97F4A7C15ull))];
  }
  long long tiles = 0, nnz_in = 0;
  for (const auto& kv : cnt)
    if ((long long)kv.second * (long long)st >= 122) {
      ++tiles;
      nnz_in += (long long)kv.second * (long long)st;
    }
  return tiles ? (double)nnz_in / ((double)tiles * 4096.0) : 0.0;
}

}  // namespace

void cadr_perm_ref(uint64_t dim, uint64_t nnz, const uint32_t* idx, std::vector<uint32_t>& perm) {
  const std::vector<size_t> deg = degrees(dim, nnz, idx);
  std::vector<int> sorted_indices(deg.size());
  std::iota(sorted_indices.begin(), sorted_indices.end(), 0);
  std::sort(sorted_indices.begin(), sorted_indices.end(),
            [&](int a, int b) { return deg[a] > deg[b]; });
  perm.assign(dim, 0);
  for (int new_idx = 0; new_idx < (int)sorted_indices.size(); ++new_idx)
    perm[sorted_indices[new_idx]] = (uint32_t)new_idx;
}

void reorder_generic(int N, const uint64_t* dims, uint64_t nnz, const uint32_t* const* idx,
                     int kind, int rounds, uint64_t sample_budget,
                     std::vector<std::vector<uint32_t>>& rank, std::string* note) {
  rank.clear();
  char buf[256];
  if (kind == 1) {
    rank.resize(N);
    for (int m = 0; m < N; ++m) cadr_tiebreak(dims[m], nnz, idx[m], rank[m]);
  } else if (kind == 2) {
    hits(N, dims, nnz, idx, rounds, sample_budget, rank);
  } else if (kind == 3 && N >= 3) {
    const double f_raw = probe_fill(N, dims, nnz, idx, nullptr);
    if (f_raw < 0.02) {
      std::snprintf(buf, sizeof buf, "[GEN] reorder=auto -> none (raw probe fill %g < 0.02)", f_raw);
      if (note) *note = buf;
      return;
    }
    std::vector<std::vector<uint32_t>> rk;
    hits(N, dims, nnz, idx, rounds, sample_budget, rk);
    const double f_hits = probe_fill(N, dims, nnz, idx, &rk);
    if (f_hits >= 0.11) {
      rank.swap(rk);
      std::snprintf(buf, sizeof buf, "[GEN] reorder=auto -> hits (probe fill %g -> %g >= 0.11)",
                    f_raw, f_hits);
    } else {
      std::snprintf(buf, sizeof buf, "[GEN] reorder=auto -> none (probe fill %g -> %g < 0.11)",
                    f_raw, f_hits);
    }
    if (note) *note = buf;
  }
}

}  // namespace cptc
