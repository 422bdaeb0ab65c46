// =============================================================================
// cptc oracle — TEST INFRASTRUCTURE ONLY.
//
// A plain C++ restatement, on the host, of the CP-ALS / MTTKRP arithmetic of
// zhixianzhu/cpTC.  It is the checker for the CUDA engine and the CPU
// baseline of the benchmark; the engine never links or calls it.  Every
// function cites the reference lines it follows (paths inside the reference
// project).  Built by oracle/Makefile into oracle/_build/liboracle.so.
//
// Parity pins: tests/golden/ holds per-iteration fits printed by the
// reference itself (rebuilt for sm_100a by oracle/build_ref.sh and run on a
// B200) together with the script that produced them.
// =============================================================================
#include <omp.h>

#include <algorithm>
#include <cfloat>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <numeric>
#include <random>
#include <unordered_map>
#include <vector>

namespace {

using u32 = uint32_t;
using u64 = uint64_t;

// ---------------------------------------------------------------------------
// COO MTTKRP, FP64.
// prod = v * F_m1[o_m1] * F_m2[o_m2] * ... over the non-target modes in
// increasing mode order, as in src/sparse.cu:666-669 (order 3: v*F1*F2 with
// F1 the lower mode, :741-755) and src/generic.cu:308-318 (order N).
// Each output row is summed in input order (rows split over threads).
// `skip` (nullable) excludes flagged nonzeros (src/generic.cu:305-306).
// ---------------------------------------------------------------------------
void mttkrp_fp64(int N, const u64* dims, u64 nnz, const u32* const* idx, const double* vals,
                 int R, const double* const* F, int n, double* out, const uint8_t* skip,
                 int nthreads) {
  const u64 In = dims[n];
  std::fill(out, out + In * (u64)R, 0.0);
  // CSR by target row, stable in input order.
  std::vector<u64> start(In + 1, 0);
  for (u64 e = 0; e < nnz; ++e) ++start[idx[n][e] + 1];
  for (u64 i = 0; i < In; ++i) start[i + 1] += start[i];
  std::vector<u64> order(nnz);
  {
    std::vector<u64> cur(start.begin(), start.end() - 1);
    for (u64 e = 0; e < nnz; ++e) order[cur[idx[n][e]]++] = e;
  }
  std::vector<double> prod((size_t)R * (nthreads > 0 ? nthreads : 1));
#pragma omp parallel for num_threads(nthreads) schedule(dynamic, 64)
  for (int64_t i = 0; i < (int64_t)In; ++i) {
    double* o = out + (u64)i * R;
    for (u64 p = start[i]; p < start[i + 1]; ++p) {
      const u64 e = order[p];
      if (skip && skip[e]) continue;
      for (int r = 0; r < R; ++r) {
        double q = vals[e];
        for (int m = 0; m < N; ++m)
          if (m != n) q *= F[m][(u64)idx[m][e] * R + r];
        o[r] += q;
      }
    }
  }
}

// TF32 operand as read by the tensor core from an FP32 register: the low 13
// mantissa bits are ignored.
inline float tf32(float x) {
  u32 b;
  std::memcpy(&b, &x, 4);
  b &= 0xFFFFE000u;
  std::memcpy(&x, &b, 4);
  return x;
}

inline float to_f32_clamped(double v) {  // src/dense.cu:248-252
  if (v > FLT_MAX) v = FLT_MAX;
  if (v < -FLT_MAX) v = -FLT_MAX;
  return (float)v;
}

// ---------------------------------------------------------------------------
// Order-3 dense-tile MTTKRP (TF32 slabs, FP64 weighting), restating
// dense_tile_mttkrp_wmma (src/dense.cu:89-1076): per 16^3 tile, per slab s
// of the F2 mode, P[t, r] = fp32( sum_c tf32(x[t,c,s]) * tf32(F1[c, r]) )
// and out[t, r] += sum_s double(P[t, r]) * F2[s, r]  (mode 0: t=i c=j s=k;
// mode 1: t=j c=i s=k; mode 2: t=k c=i s=j).  Tiles store values (last
// write wins, src/dense.cu:266-271).
// tiles: list of (tile origin b0,b1,b2) with element lists.
// ---------------------------------------------------------------------------
struct Tile3 {
  int b[3];
  std::vector<u64> elems;
};

void mttkrp_dense_tiles3(const u64* dims, const u32* const* idx, const double* vals, int R,
                         const double* const* F, int n, const std::vector<Tile3>& tiles,
                         double* out, int nthreads) {
  const int tmode = n;
  const int cmode = (n == 0) ? 1 : 0;
  const int smode = (n == 2) ? 1 : 2;
  const double* F1 = F[cmode];
  const double* F2 = F[smode];
  std::vector<std::vector<double>> part(nthreads > 0 ? nthreads : 1);
#pragma omp parallel num_threads(nthreads)
  {
    std::vector<float> x(4096);
    std::vector<double> acc(16 * (size_t)R);
    std::vector<double>& mine = part[omp_get_thread_num()];
    mine.assign(dims[n] * (u64)R, 0.0);
#pragma omp for schedule(dynamic, 16)
    for (int64_t ti = 0; ti < (int64_t)tiles.size(); ++ti) {
      const Tile3& T = tiles[ti];
      std::fill(x.begin(), x.end(), 0.0f);
      for (u64 e : T.elems) {
        const int li = (int)(idx[0][e] - (u32)T.b[0]);
        const int lj = (int)(idx[1][e] - (u32)T.b[1]);
        const int lk = (int)(idx[2][e] - (u32)T.b[2]);
        x[li * 256 + lj * 16 + lk] = to_f32_clamped(vals[e]);
      }
      std::fill(acc.begin(), acc.end(), 0.0);
      for (int s = 0; s < 16; ++s) {
        const u64 sg = (u64)T.b[smode] + s;
        if (sg >= dims[smode]) continue;
        for (int t = 0; t < 16; ++t) {
          const u64 tg = (u64)T.b[tmode] + t;
          if (tg >= dims[tmode]) continue;
          for (int r = 0; r < R; ++r) {
            float p = 0.0f;
            for (int c = 0; c < 16; ++c) {
              const u64 cg = (u64)T.b[cmode] + c;
              const float f = (cg < dims[cmode]) ? (float)F1[cg * R + r] : 0.0f;
              int li, lj, lk;
              if (n == 0) { li = t; lj = c; lk = s; }
              else if (n == 1) { li = c; lj = t; lk = s; }
              else { li = c; lj = s; lk = t; }
              p += tf32(x[li * 256 + lj * 16 + lk]) * tf32(f);
            }
            acc[t * (size_t)R + r] += (double)p * F2[sg * R + r];
          }
        }
      }
      for (int t = 0; t < 16; ++t) {
        const u64 tg = (u64)T.b[tmode] + t;
        if (tg >= dims[tmode]) continue;
        for (int r = 0; r < R; ++r) mine[tg * R + r] += acc[t * (size_t)R + r];
      }
    }
  }
  for (auto& p : part)
    if (!p.empty())
      for (u64 i = 0; i < dims[n] * (u64)R; ++i) out[i] += p[i];
}

// ---------------------------------------------------------------------------
// Order-3 hybrid partition (src/partition.cu:581-1493): tiles of 16^3 keyed
// by block id; dense when count >= cutoff, cutoff = int(4096*thr) clamped to
// [1, 4096]; thr <= 0 selects the auto-balance cutoff of :1030-1098.
// ---------------------------------------------------------------------------
int partition3(const u64* dims, u64 nnz, const u32* const* idx, double thr, int sm_count,
               std::vector<uint8_t>& is_dense, std::vector<Tile3>& tiles) {
  const u64 nbj = (dims[1] + 15) / 16, nbk = (dims[2] + 15) / 16;
  std::vector<std::pair<u64, u64>> key(nnz);
  for (u64 e = 0; e < nnz; ++e)
    key[e] = {((u64)(idx[0][e] / 16) * nbj + idx[1][e] / 16) * nbk + idx[2][e] / 16, e};
  std::stable_sort(key.begin(), key.end(),
                   [](const std::pair<u64, u64>& a, const std::pair<u64, u64>& b) {
                     return a.first < b.first;
                   });
  std::vector<std::pair<u64, u64>> runs;  // (start, count)
  for (u64 s = 0; s < nnz;) {
    u64 t = s;
    while (t < nnz && key[t].first == key[s].first) ++t;
    runs.push_back({s, t - s});
    s = t;
  }
  int cutoff = 0;
  if (thr > 0.0) {
    cutoff = (int)(4096.0 * thr);
    if (cutoff < 1) cutoff = 1;
    if (cutoff > 4096) cutoff = 4096;
  } else {
    const double sm_scale = (double)sm_count / 24.0;
    const double rate_wmma = 1.20 / sm_scale, rate_cuda = 0.688 / sm_scale;
    const double frac_dense = rate_cuda / (rate_wmma + rate_cuda);
    const u64 target = (u64)((double)nnz * frac_dense);
    std::vector<int> cs;
    for (auto& r : runs) cs.push_back((int)r.second);
    std::sort(cs.begin(), cs.end(), std::greater<int>());
    u64 acc = 0;
    cutoff = 1;
    for (int c : cs) {
      acc += (u64)c;
      if (acc >= target) {
        cutoff = c;
        break;
      }
    }
  }
  is_dense.assign(nnz, 0);
  tiles.clear();
  for (auto& r : runs) {
    if ((int)r.second < cutoff) continue;
    const u64 bid = key[r.first].first;
    Tile3 T;
    T.b[2] = (int)((bid % nbk) * 16);
    T.b[1] = (int)(((bid / nbk) % nbj) * 16);
    T.b[0] = (int)((bid / nbk / nbj) * 16);
    for (u64 p = r.first; p < r.first + r.second; ++p) {
      T.elems.push_back(key[p].second);
      is_dense[key[p].second] = 1;
    }
    tiles.push_back(std::move(T));
  }
  return cutoff;
}

// ---------------------------------------------------------------------------
// Symmetric eigendecomposition by the cyclic Jacobi method (Golub & Van Loan,
// Alg. 8.5.3).  A (R x R, row-major) is destroyed; eigenvalues to w, vectors
// as columns of V.
// ---------------------------------------------------------------------------
void jacobi_eig(int n, std::vector<double>& A, std::vector<double>& w, std::vector<double>& V) {
  V.assign((size_t)n * n, 0.0);
  for (int i = 0; i < n; ++i) V[(size_t)i * n + i] = 1.0;
  for (int sweep = 0; sweep < 100; ++sweep) {
    double off = 0.0, tot = 0.0;
    for (int i = 0; i < n; ++i)
      for (int j = 0; j < n; ++j) {
        const double a = A[(size_t)i * n + j] * A[(size_t)i * n + j];
        tot += a;
        if (i != j) off += a;
      }
    if (off <= 1e-30 * tot || off == 0.0) break;
    for (int p = 0; p < n - 1; ++p)
      for (int q = p + 1; q < n; ++q) {
        const double apq = A[(size_t)p * n + q];
        if (apq == 0.0) continue;
        const double app = A[(size_t)p * n + p], aqq = A[(size_t)q * n + q];
        const double tau = (aqq - app) / (2.0 * apq);
        const double t = (tau >= 0 ? 1.0 : -1.0) / (std::fabs(tau) + std::sqrt(1.0 + tau * tau));
        const double c = 1.0 / std::sqrt(1.0 + t * t), s = t * c;
        for (int k = 0; k < n; ++k) {  // A <- J^T A J
          const double akp = A[(size_t)k * n + p], akq = A[(size_t)k * n + q];
          A[(size_t)k * n + p] = c * akp - s * akq;
          A[(size_t)k * n + q] = s * akp + c * akq;
        }
        for (int k = 0; k < n; ++k) {
          const double apk = A[(size_t)p * n + k], aqk = A[(size_t)q * n + k];
          A[(size_t)p * n + k] = c * apk - s * aqk;
          A[(size_t)q * n + k] = s * apk + c * aqk;
        }
        for (int k = 0; k < n; ++k) {
          const double vkp = V[(size_t)k * n + p], vkq = V[(size_t)k * n + q];
          V[(size_t)k * n + p] = c * vkp - s * vkq;
          V[(size_t)k * n + q] = s * vkp + c * vkq;
        }
      }
  }
  w.resize(n);
  for (int i = 0; i < n; ++i) w[i] = A[(size_t)i * n + i];
}

// Truncated pseudo-inverse of symmetric FtF (src/solver.cu:900-1003):
// singular values sigma = |lambda|; sigma <= R*ulp(sigma_max) is dropped
// (tol of :952-954); pinv = sum_k v_k v_k^T / lambda_k.
void pinv_sym(int R, const double* FtF, std::vector<double>& P) {
  std::vector<double> A(FtF, FtF + (size_t)R * R), w, V;
  jacobi_eig(R, A, w, V);
  double smax = 0.0;
  for (double x : w) smax = std::max(smax, std::fabs(x));
  const double tol = (double)R * (std::nextafter(smax, smax + 1.0) - smax);
  P.assign((size_t)R * R, 0.0);
  for (int k = 0; k < R; ++k) {
    if (!(std::fabs(w[k]) > tol)) continue;
    const double inv = 1.0 / w[k];
    for (int a = 0; a < R; ++a)
      for (int b = 0; b < R; ++b)
        P[(size_t)a * R + b] += V[(size_t)a * R + k] * inv * V[(size_t)b * R + k];
  }
}

// Cholesky solve with relative ridge (src/generic.cu:746-819).
void chol_solve(int R, const double* FtF, const double* FtV, double* F, u64 dim, int nthreads) {
  std::vector<double> L((size_t)R * R, 0.0);
  double tr = 0.0;
  for (int i = 0; i < R; ++i) tr += FtF[i * R + i];
  const double eps = 1e-12 * ((tr > 0.0) ? tr / (double)R : 1.0) + 1e-300;
  for (int i = 0; i < R; ++i)
    for (int j = 0; j <= i; ++j) {
      double s = FtF[i * R + j];
      if (i == j) s += eps;
      for (int k = 0; k < j; ++k) s -= L[i * R + k] * L[j * R + k];
      if (i == j) L[i * R + j] = (s > 0.0) ? std::sqrt(s) : std::sqrt(eps);
      else L[i * R + j] = s / L[j * R + j];
    }
#pragma omp parallel for num_threads(nthreads) schedule(static)
  for (int64_t row = 0; row < (int64_t)dim; ++row) {
    const double* b = FtV + (u64)row * R;
    double y[256], x[256];
    for (int i = 0; i < R; ++i) {
      double s = b[i];
      for (int k = 0; k < i; ++k) s -= L[i * R + k] * y[k];
      y[i] = s / L[i * R + i];
    }
    for (int i = R - 1; i >= 0; --i) {
      double s = y[i];
      for (int k = i + 1; k < R; ++k) s -= L[k * R + i] * x[k];
      x[i] = s / L[i * R + i];
    }
    for (int i = 0; i < R; ++i) F[(u64)row * R + i] = x[i];
  }
}

void gram(const double* F, u64 rows, int R, double* G) {
  std::fill(G, G + (size_t)R * R, 0.0);
  for (u64 i = 0; i < rows; ++i)
    for (int a = 0; a < R; ++a) {
      const double fa = F[i * R + a];
      for (int b = 0; b < R; ++b) G[a * R + b] += fa * F[i * R + b];
    }
}

// CADR permutation of one mode (src/cadr.cu:31-51): degree-descending order
// by std::sort with the reference's comparator on the same input sequence
// (ties unbroken, so the same libstdc++ gives the same order).
void cadr_perm(u64 dim, u64 nnz, const u32* idx, std::vector<int>& perm) {
  std::vector<size_t> deg(dim, 0);
  for (u64 e = 0; e < nnz; ++e) deg[idx[e]]++;
  std::vector<int> sorted_indices(deg.size());
  std::iota(sorted_indices.begin(), sorted_indices.end(), 0);
  std::sort(sorted_indices.begin(), sorted_indices.end(),
            [&](int a, int b) { return deg[a] > deg[b]; });
  perm.assign(dim, 0);
  for (int new_idx = 0; new_idx < (int)sorted_indices.size(); ++new_idx)
    perm[sorted_indices[new_idx]] = new_idx;
}

// N-order dense units (src/generic.cu:578-725): key of (inner 16^3 tile,
// outer tuple); elements of keys with count >= int(4096*thr) are dense.
inline u64 splitbit_hash(u64 x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

struct UnitN {
  u32 b[3];
  std::vector<u32> outer;
  std::vector<u64> elems;
};

void build_units(int N, u64 nnz, const u32* const* idx, double thr, const int* inner,
                 std::vector<UnitN>& units, std::vector<uint8_t>& is_dense) {
  const int cutoff = (int)(4096.0 * thr);
  std::vector<u64> key(nnz);
  std::unordered_map<u64, u32> cnt;
  for (u64 e = 0; e < nnz; ++e) {
    const u32 a = idx[inner[0]][e], b = idx[inner[1]][e], c = idx[inner[2]][e];
    u64 o = 0;
    for (int m = 0; m < N; ++m)
      if (m != inner[0] && m != inner[1] && m != inner[2]) o = o * 1000003ull + idx[m][e];
    const u64 tile = ((u64)(a / 16) << 40) | ((u64)(b / 16) << 20) | (u64)(c / 16);
    key[e] = splitbit_hash(tile ^ (o * 0x9E3779B97F4A7C15ull));
    ++cnt[key[e]];
  }
  std::unordered_map<u64, u32> index;
  units.clear();
  is_dense.assign(nnz, 0);
  for (u64 e = 0; e < nnz; ++e) {
    if (cnt[key[e]] < (u32)cutoff) continue;
    auto it = index.find(key[e]);
    u32 ui;
    if (it == index.end()) {
      UnitN u;
      u.b[0] = idx[inner[0]][e] / 16;
      u.b[1] = idx[inner[1]][e] / 16;
      u.b[2] = idx[inner[2]][e] / 16;
      for (int m = 0; m < N; ++m)
        if (m != inner[0] && m != inner[1] && m != inner[2]) u.outer.push_back(idx[m][e]);
      ui = (u32)units.size();
      index[key[e]] = ui;
      units.push_back(std::move(u));
    } else {
      ui = it->second;
    }
    units[ui].elems.push_back(e);
    is_dense[e] = 1;
  }
}

// N-order dense-unit MTTKRP for inner target slot t (src/generic.cu:429-561):
// tile x[slot0][slot1][slot2] (duplicates summed in fp32); folded factor
// p = (t+1)%3 in TF32, weight q = (t+2)%3 and outer w_r in FP64:
// out[t_row, r] += sum_lk double(P[li, r]) * F_q[q_row, r] * w[r].
void mttkrp_units(int N, const u64* dims, const u32* const* idx, const double* vals, int R,
                  const double* const* F, const int* inner, int tslot,
                  const std::vector<UnitN>& units, double* out) {
  std::vector<int> outer_modes;
  for (int m = 0; m < N; ++m)
    if (m != inner[0] && m != inner[1] && m != inner[2]) outer_modes.push_back(m);
  const int ps = (tslot + 1) % 3, qs = (tslot + 2) % 3;
  const int stride[3] = {256, 16, 1};
  std::vector<float> x(4096);
  std::vector<double> w(R), acc(16 * (size_t)R);
  for (const UnitN& u : units) {
    std::fill(x.begin(), x.end(), 0.0f);
    for (u64 e : u.elems) {
      const u32 l0 = idx[inner[0]][e] % 16, l1 = idx[inner[1]][e] % 16, l2 = idx[inner[2]][e] % 16;
      x[l0 * 256 + l1 * 16 + l2] += (float)vals[e];
    }
    for (int r = 0; r < R; ++r) w[r] = 1.0;
    for (size_t q = 0; q < outer_modes.size(); ++q)
      for (int r = 0; r < R; ++r) w[r] *= F[outer_modes[q]][(u64)u.outer[q] * R + r];
    std::fill(acc.begin(), acc.end(), 0.0);
    const int pm = inner[ps], qm = inner[qs], tm = inner[tslot];
    for (int lk = 0; lk < 16; ++lk) {
      const u64 qrow = (u64)u.b[qs] * 16 + lk;
      const bool q_ok = qrow < dims[qm];
      for (int li = 0; li < 16; ++li)
        for (int r = 0; r < R; ++r) {
          float p = 0.0f;
          for (int lj = 0; lj < 16; ++lj) {
            const u64 prow = (u64)u.b[ps] * 16 + lj;
            const float f = (prow < dims[pm]) ? (float)F[pm][prow * R + r] : 0.0f;
            p += tf32(x[li * stride[tslot] + lj * stride[ps] + lk * stride[qs]]) * tf32(f);
          }
          if (q_ok) acc[li * (size_t)R + r] += (double)p * F[qm][qrow * R + r] * w[r];
        }
    }
    for (int li = 0; li < 16; ++li) {
      const u64 trow = (u64)u.b[tslot] * 16 + li;
      if (trow >= dims[tm]) continue;
      for (int r = 0; r < R; ++r) out[trow * R + r] += acc[li * (size_t)R + r];
    }
  }
}

}  // namespace

extern "C" {

// ---------------------------------------------------------------------------
// Plain FP64 MTTKRP over all nonzeros (the FP64-only path of the reference).
// ---------------------------------------------------------------------------
int or_mttkrp(int order, const u64* dims, u64 nnz, const u32* const* idx, const double* vals,
              int R, const double* const* factors, int mode, double* out, int nthreads) {
  if (order < 2 || order > 8 || mode < 0 || mode >= order || R < 1) return -1;
  mttkrp_fp64(order, dims, nnz, idx, vals, R, factors, mode, out, nullptr,
              nthreads > 0 ? nthreads : 1);
  return 0;
}

// Order-3 hybrid MTTKRP on coordinates as given (no reordering): tiles with
// count >= cutoff(thr) through the TF32 tile arithmetic, the rest in FP64.
// Returns the number of dense tiles (>= 0) or a negative error.
int or_mttkrp_hybrid3(const u64* dims, u64 nnz, const u32* const* idx, const double* vals,
                      int R, const double* const* factors, int mode, double thr, int sm_count,
                      double* out, int nthreads) {
  if (mode < 0 || mode > 2) return -1;
  std::vector<uint8_t> dense;
  std::vector<Tile3> tiles;
  partition3(dims, nnz, idx, thr, sm_count, dense, tiles);
  const int nt = nthreads > 0 ? nthreads : 1;
  mttkrp_fp64(3, dims, nnz, idx, vals, R, factors, mode, out, dense.data(), nt);
  mttkrp_dense_tiles3(dims, idx, vals, R, factors, mode, tiles, out, nt);
  return (int)tiles.size();
}

// Partition statistics of the reference's fill-rate selector
// (src/main.cu:336-416): out[0] dense_nnz, out[1] sparse_nnz,
// out[2] dense tiles, out[3] cutoff, out[4] avg_fill.
int or_partition_stats3(const u64* dims, u64 nnz, const u32* const* idx, double thr,
                        int sm_count, double* out5) {
  std::vector<uint8_t> dense;
  std::vector<Tile3> tiles;
  const int cutoff = partition3(dims, nnz, idx, thr, sm_count, dense, tiles);
  u64 dn = 0;
  for (auto& t : tiles) dn += t.elems.size();
  out5[0] = (double)dn;
  out5[1] = (double)(nnz - dn);
  out5[2] = (double)tiles.size();
  out5[3] = (double)cutoff;
  out5[4] = tiles.empty() ? 0.0 : (double)dn / ((double)tiles.size() * 4096.0);
  return 0;
}

// CADR relabelling of one mode: perm[old] = new.
int or_cadr_perm(u64 dim, u64 nnz, const u32* idx, int* perm_out) {
  std::vector<int> p;
  cadr_perm(dim, nnz, idx, p);
  std::copy(p.begin(), p.end(), perm_out);
  return 0;
}

// Order-3 initial factors (src/common.cu:83-101): mt19937(42),
// uniform_real_distribution<double>(0,1), modes 0,1,2 in turn, row-major.
int or_init_factors3(const u64* dims, int R, double* const* out) {
  std::mt19937 gen(42);
  std::uniform_real_distribution<double> dis(0.0, 1.0);
  for (int m = 0; m < 3; ++m)
    for (u64 i = 0; i < dims[m] * (u64)R; ++i) out[m][i] = dis(gen);
  return 0;
}

// ---------------------------------------------------------------------------
// Order-3 CP-ALS as main.cu:176-517 + als.cu:362-761:
//  CADR relabel -> mt19937(42) factors in relabelled space -> partition ->
//  per iteration, for modes 0,1,2: Grams of the other two factors, Hadamard,
//  MTTKRP (hybrid when use_tf32), truncated-pinv solve, divide by lambda,
//  normalise and absorb norms into lambda (norm < 1e-14 -> column and
//  lambda zero), then the Gram-based fit (als.cu:659-715).
// path: 0 = FP64 only (ALS_FORCE_CUDA), 1 = TF32 tiles + FP64 residual.
// factors_out (nullable): unpermuted factors (original index space).
// ---------------------------------------------------------------------------
int or_cp_als3(const u64* dims_in, u64 nnz, const u32* const* idx_in, const double* vals, int R,
               int iters, double thr, int path, int sm_count, double* fits, double* lambda_out,
               double* const* factors_out, int nthreads) {
  if (R < 1 || iters < 1) return -1;
  const int nt = nthreads > 0 ? nthreads : 1;
  u64 dims[3] = {dims_in[0], dims_in[1], dims_in[2]};
  std::vector<std::vector<int>> perm(3);
  std::vector<std::vector<u32>> idx(3);
  for (int m = 0; m < 3; ++m) {
    cadr_perm(dims[m], nnz, idx_in[m], perm[m]);
    idx[m].resize(nnz);
    for (u64 e = 0; e < nnz; ++e) idx[m][e] = (u32)perm[m][idx_in[m][e]];
  }
  const u32* ip[3] = {idx[0].data(), idx[1].data(), idx[2].data()};
  std::vector<std::vector<double>> F(3);
  for (int m = 0; m < 3; ++m) F[m].resize(dims[m] * (u64)R);
  double* fp[3] = {F[0].data(), F[1].data(), F[2].data()};
  or_init_factors3(dims, R, fp);

  std::vector<uint8_t> dense;
  std::vector<Tile3> tiles;
  if (path == 1) partition3(dims, nnz, ip, thr, sm_count, dense, tiles);

  double X2 = 0.0;
  for (u64 e = 0; e < nnz; ++e) X2 += vals[e] * vals[e];
  const double Xn = std::sqrt(X2);

  std::vector<double> lambda(R, 1.0);
  std::vector<std::vector<double>> G(3, std::vector<double>((size_t)R * R));
  std::vector<double> FtF((size_t)R * R), Ainv;
  u64 maxd = std::max({dims[0], dims[1], dims[2]});
  std::vector<double> FtV(maxd * (u64)R);
  const double* cfp[3] = {fp[0], fp[1], fp[2]};

  for (int it = 0; it < iters; ++it) {
    for (int n = 0; n < 3; ++n) {
      const int p = (n == 0) ? 1 : 0, q = (n == 2) ? 1 : 2;
      gram(fp[p], dims[p], R, G[p].data());
      gram(fp[q], dims[q], R, G[q].data());
      for (size_t i = 0; i < (size_t)R * R; ++i) FtF[i] = G[p][i] * G[q][i];
      mttkrp_fp64(3, dims, nnz, ip, vals, R, cfp, n, FtV.data(),
                  path == 1 ? dense.data() : nullptr, nt);
      if (path == 1) mttkrp_dense_tiles3(dims, ip, vals, R, cfp, n, tiles, FtV.data(), nt);
      pinv_sym(R, FtF.data(), Ainv);
      double* Fn = fp[n];
#pragma omp parallel for num_threads(nt) schedule(static)
      for (int64_t i = 0; i < (int64_t)dims[n]; ++i)
        for (int r = 0; r < R; ++r) {
          double s = 0.0;
          for (int k = 0; k < R; ++k) s += Ainv[(size_t)r * R + k] * FtV[(u64)i * R + k];
          Fn[(u64)i * R + r] = s;
        }
      for (u64 i = 0; i < dims[n] * (u64)R; ++i) Fn[i] /= lambda[i % R];
      std::vector<double> nr(R, 0.0);
      for (u64 i = 0; i < dims[n]; ++i)
        for (int r = 0; r < R; ++r) nr[r] += Fn[i * R + r] * Fn[i * R + r];
      for (int r = 0; r < R; ++r) nr[r] = std::sqrt(nr[r]);
      for (u64 i = 0; i < dims[n] * (u64)R; ++i) {
        const double v = nr[i % R];
        Fn[i] = (v < 1e-14) ? 0.0 : Fn[i] / v;
      }
      for (int r = 0; r < R; ++r) lambda[r] = (nr[r] < 1e-14) ? 0.0 : lambda[r] * nr[r];
      gram(Fn, dims[n], R, G[n].data());
    }
    double iprod = 0.0;
    for (int r = 0; r < R; ++r) {
      double d = 0.0;
      for (u64 k = 0; k < dims[2]; ++k) d += fp[2][k * R + r] * FtV[k * R + r];
      iprod += lambda[r] * d;
    }
    double model2 = 0.0;
    for (int r = 0; r < R; ++r)
      for (int s = 0; s < R; ++s)
        model2 += lambda[r] * lambda[s] * G[0][r * R + s] * G[1][r * R + s] * G[2][r * R + s];
    const double res2 = std::max(X2 - 2.0 * iprod + model2, 0.0);
    fits[it] = (Xn > 0.0) ? 1.0 - std::sqrt(res2) / Xn : 0.0;
  }
  if (lambda_out) std::copy(lambda.begin(), lambda.end(), lambda_out);
  if (factors_out)
    for (int m = 0; m < 3; ++m)
      if (factors_out[m])
        for (u64 a = 0; a < dims[m]; ++a)
          std::memcpy(factors_out[m] + a * R, fp[m] + (u64)perm[m][a] * R, R * sizeof(double));
  return (int)tiles.size();
}

// ---------------------------------------------------------------------------
// N-order reordering (src/generic.cu:1180-1376). kind: 0 none, 1 cadr
// (degree desc, tie a<b), 2 hits (T rounds on a strided sample).
// rank_out[m][old] = new.
// ---------------------------------------------------------------------------
int or_reorder(int N, const u64* dims, u64 nnz, const u32* const* idx, int kind, int rounds,
               u64 sample_budget, u32* const* rank_out) {
  for (int m = 0; m < N; ++m)
    for (u64 i = 0; i < dims[m]; ++i) rank_out[m][i] = (u32)i;
  if (kind == 2) {
    const u64 stride = (nnz > sample_budget && sample_budget > 0) ? nnz / sample_budget : 1;
    std::vector<std::vector<double>> s(N), ns(N);
    for (int m = 0; m < N; ++m) s[m].assign(dims[m], 1.0);
    for (int it = 0; it < rounds; ++it) {
      for (int m = 0; m < N; ++m) ns[m].assign(dims[m], 0.0);
      for (u64 e = 0; e < nnz; e += stride)
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
    for (int m = 0; m < N; ++m) {
      std::vector<u32> ord(dims[m]);
      for (u64 i = 0; i < dims[m]; ++i) ord[i] = (u32)i;
      std::sort(ord.begin(), ord.end(), [&](u32 a, u32 b) {
        const double sa = s[m][a], sb = s[m][b];
        return (sa != sb) ? (sa > sb) : (a < b);
      });
      for (u64 i = 0; i < dims[m]; ++i) rank_out[m][ord[i]] = (u32)i;
    }
  } else if (kind == 1) {
    for (int m = 0; m < N; ++m) {
      std::vector<u32> deg(dims[m], 0);
      for (u64 e = 0; e < nnz; ++e) ++deg[idx[m][e]];
      std::vector<u32> ord(dims[m]);
      for (u64 i = 0; i < dims[m]; ++i) ord[i] = (u32)i;
      std::sort(ord.begin(), ord.end(),
                [&](u32 a, u32 b) { return deg[a] != deg[b] ? deg[a] > deg[b] : a < b; });
      for (u64 i = 0; i < dims[m]; ++i) rank_out[m][ord[i]] = (u32)i;
    }
  }
  return 0;
}

// N-order dense-unit MTTKRP for inner target `tslot` with the FP64 residual
// of all non-unit elements (the reference's combined dense + segment pass,
// src/generic.cu:2061-2105).  Returns number of units.
int or_mttkrp_units(int N, const u64* dims, u64 nnz, const u32* const* idx, const double* vals,
                    int R, const double* const* F, const int* inner, int tslot, double thr,
                    double* out, int nthreads) {
  std::vector<UnitN> units;
  std::vector<uint8_t> dense;
  build_units(N, nnz, idx, thr, inner, units, dense);
  const int n = inner[tslot];
  mttkrp_fp64(N, dims, nnz, idx, vals, R, F, n, out, dense.data(), nthreads > 0 ? nthreads : 1);
  mttkrp_units(N, dims, idx, vals, R, F, inner, tslot, units, out);
  return (int)units.size();
}

// ---------------------------------------------------------------------------
// Generic N-order CP-ALS (src/generic.cu:1639-2251).
// reorder: 0 none, 1 cadr, 2 hits.  solver: 0 Cholesky, 1 truncated pinv.
// dense_thr > 0 with N >= 4 enables TF32 units over inner modes (0,1,2).
// factors_out (nullable): factors in ORIGINAL index space.
// ---------------------------------------------------------------------------
int or_cp_als_generic(int N, const u64* dims, u64 nnz, const u32* const* idx_in,
                      const double* vals, int R, int iters, unsigned seed, int reorder,
                      int rounds, u64 sample_budget, double dense_thr, int solver,
                      double* fits, double* lambda_out, double* const* factors_out,
                      int nthreads) {
  if (N < 2 || N > 8 || R < 1 || iters < 1) return -1;
  const int nt = nthreads > 0 ? nthreads : 1;
  std::vector<std::vector<u32>> rank(N), idx(N);
  std::vector<u32*> rp(N);
  for (int m = 0; m < N; ++m) {
    rank[m].resize(dims[m]);
    rp[m] = rank[m].data();
  }
  or_reorder(N, dims, nnz, idx_in, reorder, rounds, sample_budget, rp.data());
  for (int m = 0; m < N; ++m) {
    idx[m].resize(nnz);
    for (u64 e = 0; e < nnz; ++e) idx[m][e] = rank[m][idx_in[m][e]];
  }
  std::vector<const u32*> ip(N);
  for (int m = 0; m < N; ++m) ip[m] = idx[m].data();

  std::mt19937 gen(seed);  // :1755-1783, rows carried through the relabelling
  std::uniform_real_distribution<double> dis(0.0, 1.0);
  std::vector<std::vector<double>> F(N);
  for (int m = 0; m < N; ++m) {
    std::vector<double> u(dims[m] * (u64)R);
    for (auto& x : u) x = dis(gen);
    F[m].resize(u.size());
    for (u64 a = 0; a < dims[m]; ++a)
      std::memcpy(F[m].data() + (u64)rank[m][a] * R, u.data() + a * R, R * sizeof(double));
  }
  std::vector<double*> fp(N);
  std::vector<const double*> cfp(N);
  for (int m = 0; m < N; ++m) {
    fp[m] = F[m].data();
    cfp[m] = F[m].data();
  }

  const int inner[3] = {0, 1, 2};
  std::vector<UnitN> units;
  std::vector<uint8_t> dense;
  const bool use_dense = (N >= 4 && dense_thr > 0.0);
  if (use_dense) build_units(N, nnz, ip.data(), dense_thr, inner, units, dense);

  std::vector<std::vector<double>> G(N, std::vector<double>((size_t)R * R));
  for (int m = 0; m < N; ++m) gram(fp[m], dims[m], R, G[m].data());
  double X2 = 0.0;
  for (u64 e = 0; e < nnz; ++e) X2 += vals[e] * vals[e];
  const double Xn = std::sqrt(X2);
  std::vector<double> lambda(R, 1.0), FtF((size_t)R * R), P;
  u64 maxd = 0;
  for (int m = 0; m < N; ++m) maxd = std::max(maxd, dims[m]);
  std::vector<double> FtV(maxd * (u64)R);

  for (int it = 0; it < iters; ++it) {
    for (int n = 0; n < N; ++n) {
      std::fill(FtF.begin(), FtF.end(), 1.0);
      for (int m = 0; m < N; ++m)
        if (m != n)
          for (size_t i = 0; i < FtF.size(); ++i) FtF[i] *= G[m][i];
      const bool inner_mode = use_dense && n < 3;
      mttkrp_fp64(N, dims, nnz, ip.data(), vals, R, cfp.data(), n, FtV.data(),
                  inner_mode ? dense.data() : nullptr, nt);
      if (inner_mode)
        mttkrp_units(N, dims, ip.data(), vals, R, cfp.data(), inner, n, units, FtV.data());
      if (solver == 1) {
        pinv_sym(R, FtF.data(), P);
        for (u64 i = 0; i < dims[n]; ++i)
          for (int r = 0; r < R; ++r) {
            double s = 0.0;
            for (int k = 0; k < R; ++k) s += P[(size_t)r * R + k] * FtV[i * R + k];
            fp[n][i * R + r] = s;
          }
      } else {
        chol_solve(R, FtF.data(), FtV.data(), fp[n], dims[n], nt);
      }
      std::vector<double> nr(R, 0.0);  // :2144-2159
      for (u64 i = 0; i < dims[n]; ++i)
        for (int r = 0; r < R; ++r) nr[r] += fp[n][i * R + r] * fp[n][i * R + r];
      for (int r = 0; r < R; ++r) {
        double v = std::sqrt(nr[r]);
        if (!std::isfinite(v) || v < 1e-14) v = 1.0;
        nr[r] = v;
      }
      for (u64 i = 0; i < dims[n] * (u64)R; ++i) fp[n][i] /= nr[i % R];
      for (int r = 0; r < R; ++r) lambda[r] = nr[r];
      gram(fp[n], dims[n], R, G[n].data());
    }
    double model2 = 0.0;
    for (int r = 0; r < R; ++r)
      for (int s = 0; s < R; ++s) {
        double v = lambda[r] * lambda[s];
        for (int m = 0; m < N; ++m) v *= G[m][r * R + s];
        model2 += v;
      }
    double iprod = 0.0;
    for (int r = 0; r < R; ++r) {
      double d = 0.0;
      for (u64 i = 0; i < dims[N - 1]; ++i) d += fp[N - 1][i * R + r] * FtV[i * R + r];
      iprod += lambda[r] * d;
    }
    const double res2 = std::max(X2 - 2.0 * iprod + model2, 0.0);
    fits[it] = (Xn > 0.0) ? 1.0 - std::sqrt(res2) / Xn : 0.0;
  }
  if (lambda_out) std::copy(lambda.begin(), lambda.end(), lambda_out);
  if (factors_out)
    for (int m = 0; m < N; ++m)
      if (factors_out[m])
        for (u64 a = 0; a < dims[m]; ++a)
          std::memcpy(factors_out[m] + a * R, fp[m] + (u64)rank[m][a] * R, R * sizeof(double));
  return (int)units.size();
}

}  // extern "C"
