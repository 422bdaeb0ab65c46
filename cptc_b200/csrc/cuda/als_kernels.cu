// Small on-device kernels of the CP-ALS update: Gram, Hadamard, the R x R
// inverse (truncated pseudo-inverse or ridge Cholesky), the solve applied to
// all rows with its Gram fused in, column normalisation and the Gram fit.
//
// Reference counterparts: compute_gram_matrix (cuBLAS Dgemm, src/als.cu:
// 115-134), g_gram_kernel (src/generic.cu:203-258), solve_als_system_svd
// (cuSOLVER gesvdj + 2 Dgemm, src/solver.cu:900-1003), g_chol_solve_kernel
// (src/generic.cu:746-819), update_mode normalisation (src/als.cu:480-517),
// the N-order normalisation (src/generic.cu:2139-2159) and the Gram fit
// (src/als.cu:659-715, src/generic.cu:2174-2214).
//
// Every reduction is two-stage with a fixed order (per-block partials, then
// one block sums them in block order), so these kernels are deterministic.
#include <cfloat>

#include "kernels.hpp"

namespace cptc {

namespace {

constexpr int kGramRows = 32;  // rows staged per block iteration

__host__ __device__ inline int padded_rank(int R) {
  return R <= 16 ? 16 : R <= 32 ? 32 : R <= 64 ? 64 : 128;
}

// acc[x][y] += sum_i tile[i][a0+x] * tile[i][b0+y] over nrows staged rows.
template <int TM>
__device__ __forceinline__ void gram_tile(const double* tile, int nrows, int Rp, int a0, int b0,
                                          double (&acc)[TM][TM]) {
  for (int i = 0; i < nrows; ++i) {
    double av[TM], bv[TM];
#pragma unroll
    for (int x = 0; x < TM; ++x) av[x] = tile[i * Rp + a0 + x];
#pragma unroll
    for (int y = 0; y < TM; ++y) bv[y] = tile[i * Rp + b0 + y];
#pragma unroll
    for (int x = 0; x < TM; ++x)
#pragma unroll
      for (int y = 0; y < TM; ++y) acc[x][y] = fma(av[x], bv[y], acc[x][y]);
  }
}

template <int TM>
__device__ __forceinline__ void store_partial(double* part, int R, int a0, int b0,
                                              const double (&acc)[TM][TM]) {
#pragma unroll
  for (int x = 0; x < TM; ++x)
#pragma unroll
    for (int y = 0; y < TM; ++y)
      if (a0 + x < R && b0 + y < R) part[(a0 + x) * R + b0 + y] = acc[x][y];
}

template <int TM>
__global__ void __launch_bounds__(256) k_gram_partial(const double* __restrict__ F, uint64_t rows,
                                                      int R, double* __restrict__ part) {
  constexpr int Rp = 16 * TM;
  __shared__ double tile[kGramRows * Rp];
  const int tid = threadIdx.x;
  const int a0 = (tid / 16) * TM, b0 = (tid % 16) * TM;
  double acc[TM][TM];
#pragma unroll
  for (int x = 0; x < TM; ++x)
#pragma unroll
    for (int y = 0; y < TM; ++y) acc[x][y] = 0.0;
  for (uint64_t r0 = (uint64_t)blockIdx.x * kGramRows; r0 < rows;
       r0 += (uint64_t)gridDim.x * kGramRows) {
    const int nr = (int)((rows - r0 < (uint64_t)kGramRows) ? rows - r0 : kGramRows);
    __syncthreads();
    for (int k = tid; k < kGramRows * Rp; k += 256) {
      const int i = k / Rp, c = k % Rp;
      tile[k] = (i < nr && c < R) ? F[(r0 + i) * (uint64_t)R + c] : 0.0;
    }
    __syncthreads();
    gram_tile<TM>(tile, nr, Rp, a0, b0, acc);
  }
  store_partial<TM>(part + (uint64_t)blockIdx.x * R * R, R, a0, b0, acc);
}

// out[i] = sum_b part[b * len + i] for b < nblk, in a fixed order: warp w of
// the block adds partials w, w + 8, w + 16, ... for 32 consecutive entries
// (coalesced), then the 8 warp sums are added in warp order.  One block per
// 32 entries, so an R x R Gram (R = 128: 512 blocks) is reduced across the GPU.
// out[i] = (add ? out[i] : 0) + sum over the nblk partials, in a fixed order.
__global__ void __launch_bounds__(256) k_partial_sum(const double* __restrict__ part, int nblk,
                                                     int len, double* __restrict__ out, int add) {
  __shared__ double sh[8][32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int i = blockIdx.x * 32 + lane;
  double s = 0.0;
  if (i < len)
    for (int b = w; b < nblk; b += 8) s += part[(uint64_t)b * len + i];
  sh[w][lane] = s;
  __syncthreads();
  if (w == 0 && i < len) {
    double t = 0.0;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += sh[k][lane];
    out[i] = add ? out[i] + t : t;
  }
}

struct GPtrs {
  const double* p[CPTC_MAX_ORDER];
};

__global__ void k_hadamard(GPtrs g, int ng, int R, double* __restrict__ out) {
  const int RR = R * R;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < RR; i += gridDim.x * blockDim.x) {
    double v = 1.0;
    for (int k = 0; k < ng; ++k) v *= g.p[k][i];
    out[i] = v;
  }
}

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---------------------------------------------------------------------------
// Truncated pseudo-inverse of a symmetric positive semi-definite A (R <= 128)
// by one-sided Jacobi (Hestenes 1958): W = A is rotated in column pairs
// until its columns are mutually orthogonal, W = A V = U Sigma.  A is PSD
// (a Hadamard product of Gram matrices, Schur product theorem), so U = V and
// pinv(A) = sum_k u_k u_k^T / sigma_k = sum_k w_k w_k^T / sigma_k^3.
// sigma_k <= R*ulp(sigma_max) is dropped, the truncation rule of the
// reference (src/solver.cu:952-954).  Convergence test and sweep cap follow
// the reference's gesvdj settings (tolerance 1e-14, 15 sweeps,
// src/solver.cu:837-838).  Pairs follow a round-robin schedule: R/2
// disjoint rotations per step, one warp per pair, R-1 steps per sweep.  Only
// W lives in shared memory (R*R doubles), so R = 128 fits one CTA.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) k_pinv_jacobi(const double* __restrict__ A, int R,
                                                      double* __restrict__ Ainv,
                                                      int* __restrict__ status,
                                                      const int* __restrict__ gate) {
  if (gate != nullptr && *gate == 0) return;  // the Cholesky inverse was accepted
  extern __shared__ double smem[];
  double* W = smem;                        // column-major, W[c*R + r]
  double* wgt = smem + R * R;              // R
  __shared__ int rotated;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  for (int k = tid; k < R * R; k += blockDim.x) {
    const int r = k % R, c = k / R;
    W[k] = A[r * R + c];
  }
  const int n = (R + 1) & ~1;  // players, with a dummy when R is odd
  for (int sweep = 0; sweep < 15; ++sweep) {
    if (tid == 0) rotated = 0;
    __syncthreads();
    for (int step = 0; step < n - 1; ++step) {
      for (int k = warp; k < n / 2; k += nwarps) {
        const int a = (k == 0) ? 0 : ((k - 1 + step) % (n - 1)) + 1;
        const int bpos = n - 1 - k;
        const int b = ((bpos - 1 + step) % (n - 1)) + 1;
        int p = a < b ? a : b, q = a < b ? b : a;
        if (q >= R) continue;
        double al = 0.0, be = 0.0, ga = 0.0;
        for (int i = lane; i < R; i += 32) {
          const double wp = W[p * R + i], wq = W[q * R + i];
          al = fma(wp, wp, al);
          be = fma(wq, wq, be);
          ga = fma(wp, wq, ga);
        }
        al = warp_sum(al);
        be = warp_sum(be);
        ga = warp_sum(ga);
        if (fabs(ga) > 1e-14 * sqrt(al * be) && ga != 0.0) {
          const double zeta = (be - al) / (2.0 * ga);
          const double t = (zeta >= 0.0 ? 1.0 : -1.0) / (fabs(zeta) + sqrt(1.0 + zeta * zeta));
          const double c = 1.0 / sqrt(1.0 + t * t), s = c * t;
          for (int i = lane; i < R; i += 32) {
            const double wp = W[p * R + i], wq = W[q * R + i];
            W[p * R + i] = c * wp - s * wq;
            W[q * R + i] = s * wp + c * wq;
          }
          if (lane == 0) rotated = 1;
        }
      }
      __syncthreads();
    }
    if (!rotated) break;
    __syncthreads();
  }
  for (int k = warp; k < R; k += nwarps) {
    double s2 = 0.0;
    for (int i = lane; i < R; i += 32) s2 = fma(W[k * R + i], W[k * R + i], s2);
    s2 = warp_sum(s2);
    if (lane == 0) wgt[k] = sqrt(s2);
  }
  __syncthreads();
  double smax = 0.0;
  for (int k = 0; k < R; ++k) smax = fmax(smax, wgt[k]);
  const double tol = (double)R * (nextafter(smax, smax + 1.0) - smax);
  __syncthreads();
  for (int k = tid; k < R; k += blockDim.x) {
    const double sk = wgt[k];
    wgt[k] = (sk > tol && isfinite(sk)) ? 1.0 / (sk * sk * sk) : 0.0;
  }
  __syncthreads();
  for (int o = tid; o < R * R; o += blockDim.x) {
    const int a = o / R, b = o % R;
    double s = 0.0;
    for (int k = 0; k < R; ++k) s = fma(W[k * R + a] * wgt[k], W[k * R + b], s);
    Ainv[o] = s;
    if (!isfinite(s)) atomicOr(status, 1);
  }
}

// ---------------------------------------------------------------------------
// FtF = Hadamard product of the Gram matrices Gs (written out for the
// pseudo-inverse kernel) and its inverse by the symmetric sweep operator
// (Gauss-Jordan elimination in place; Goodnight 1979): for pivot j with
// d = M[j][j],  M[i][k] -= M[i][j] M[j][k] / d,  M[i][j] = M[i][j] / d,
// M[j][j] = -1 / d;  after all R pivots M = -A^-1.  The pivot d of step j is
// the Schur complement that a Cholesky factorisation would take the square
// root of, so the reference's rules carry over unchanged:
//  ridge = 1 (N-order path, src/generic.cu:757-783): A + eps*I with
//    eps = 1e-12 * tr(A)/R + 1e-300, a pivot d <= 0 becomes eps;
//  ridge = 0: a pivot d <= 1e-11 * max diag (condition beyond ~1e11) rejects
//    the inverse: *fail is set and the pseudo-inverse kernel that follows
//    computes Ainv instead.
// One CTA; all R*R entries are updated in parallel per pivot from registers,
// one barrier per pivot.
// ---------------------------------------------------------------------------
template <int NWARP, int RM, int RC>
__global__ void __launch_bounds__(NWARP * 32) k_sweep_inverse(GPtrs g, int ng, int R, int ridge,
                                                        double* __restrict__ FtF,
                                                        double* __restrict__ Ainv,
                                                        int* __restrict__ status,
                                                        int* __restrict__ fail) {
  // The matrix lives in registers: thread (warp w, lane l) holds entries
  // (w + NWARP*m, l + 32c), m < RM, c < RC.  Per pivot the warp owning row j writes
  // it to shared memory (two buffers, so one barrier per pivot suffices) and
  // every thread updates its own entries: no shared-memory read-modify-write.
  __shared__ double prow[2][128];
  __shared__ double diag[128];
  __shared__ double eps_s, dmax_s;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  double M[RM][RC];
#pragma unroll
  for (int m = 0; m < RM; ++m)
#pragma unroll
    for (int c = 0; c < RC; ++c) {
      const int i = w + NWARP * m, k = lane + 32 * c;
      double v = 0.0;
      if (i < R && k < R) {
        v = 1.0;
#pragma unroll
        for (int q = 0; q < CPTC_MAX_ORDER; ++q)
          if (q < ng) v *= g.p[q][i * R + k];
        FtF[i * R + k] = v;
        if (i == k) diag[i] = v;
      }
      M[m][c] = v;
    }
  __syncthreads();
  if (tid == 0) {
    double tr = 0.0, dm = 0.0;
    for (int i = 0; i < R; ++i) {
      tr += diag[i];
      dm = fmax(dm, diag[i]);
    }
    eps_s = ridge ? 1e-12 * ((tr > 0.0) ? tr / (double)R : 1.0) + 1e-300 : 0.0;
    dmax_s = dm;
  }
  __syncthreads();
  const double eps = eps_s, dmax = dmax_s;
  if (ridge) {
#pragma unroll
    for (int m = 0; m < RM; ++m)
#pragma unroll
      for (int c = 0; c < RC; ++c)
        if (w + NWARP * m == lane + 32 * c && w + NWARP * m < R) M[m][c] += eps;
  }
  for (int j = 0; j < R; ++j) {
    double* pr = prow[j & 1];
    if (w == (j % NWARP)) {
      // Select chain over the compile-time row index (a runtime index would
      // move M to local memory).
      const int mj = j / NWARP;
#pragma unroll
      for (int c = 0; c < RC; ++c) {
        double val = M[0][c];
#pragma unroll
        for (int m = 1; m < RM; ++m) val = (m == mj) ? M[m][c] : val;
        if (lane + 32 * c < R) pr[lane + 32 * c] = val;
      }
    }
    __syncthreads();
    double d = pr[j];
    if (ridge) {
      if (!(d > 0.0)) d = eps;
    } else if (!(d > 1e-11 * dmax)) {
      if (tid == 0 && fail) *fail = 1;
      return;  // every thread sees the same d: uniform exit
    }
    const double inv = 1.0 / d;
    double pks[RC];
#pragma unroll
    for (int c = 0; c < RC; ++c) {
      const int k = lane + 32 * c;
      pks[c] = (k < R) ? pr[k] * inv : 0.0;
    }
#pragma unroll
    for (int m = 0; m < RM; ++m) {
      const int i = w + NWARP * m;
      const double pi = (i < R) ? pr[i] : 0.0;
#pragma unroll
      for (int c = 0; c < RC; ++c) {
        const int k = lane + 32 * c;
        double v;
        if (i == j) v = (k == j) ? -inv : pks[c];
        else if (k == j) v = pi * inv;
        else v = fma(-pi, pks[c], M[m][c]);
        M[m][c] = v;
      }
    }
  }
  if (tid == 0 && fail) *fail = 0;
#pragma unroll
  for (int m = 0; m < RM; ++m)
#pragma unroll
    for (int c = 0; c < RC; ++c) {
      const int i = w + NWARP * m, k = lane + 32 * c;
      if (i < R && k < R) {
        const double v = -M[m][c];
        Ainv[i * R + k] = v;
        if (!isfinite(v)) atomicOr(status, 1);
      }
    }
}

// ---------------------------------------------------------------------------
// F[i, r] = sum_s FtV[i, s] * Ainv[s, r]  (Ainv symmetric), optionally divided
// by lambda[r] (src/als.cu:496-500), with the Gram of the written rows
// accumulated per block and, when dots is set, the fit's column dot products
// sum_i F[i, r] * FtV[i, r] of the written rows (src/als.cu:659-715) per block
// as well.  Rows are staged kGramRows at a time; Ainv lives in shared memory.
// Thread layout: 16 x 16 threads, each a TM x TM tile of the 32-row x Rp
// output slab's Gram and of the product; every output a thread writes is in
// column tid % Rp (Rp divides 256), so its dot partial is one column's.
// ---------------------------------------------------------------------------
template <int TM>
__global__ void __launch_bounds__(256) k_apply_solve(const double* __restrict__ FtV,
                                                     const double* __restrict__ Ainv,
                                                     const double* __restrict__ lambda,
                                                     int divide_lambda, uint64_t rows, int R,
                                                     double* __restrict__ F,
                                                     double* __restrict__ part,
                                                     double* __restrict__ dots) {
  constexpr int Rp = 16 * TM;
  static_assert(256 % Rp == 0, "a thread's outputs share one column");
  extern __shared__ double sm[];
  double* sA = sm;                      // Rp * Rp
  double* sX = sA + Rp * Rp;            // kGramRows * Rp  (FtV slab)
  double* sY = sX + kGramRows * Rp;     // kGramRows * Rp  (result slab)
  const int tid = threadIdx.x;
  for (int k = tid; k < Rp * Rp; k += 256) {
    const int a = k / Rp, b = k % Rp;
    sA[k] = (a < R && b < R) ? Ainv[a * R + b] : 0.0;
  }
  const int a0 = (tid / 16) * TM, b0 = (tid % 16) * TM;
  double acc[TM][TM];
#pragma unroll
  for (int x = 0; x < TM; ++x)
#pragma unroll
    for (int y = 0; y < TM; ++y) acc[x][y] = 0.0;
  double dacc = 0.0;
  for (uint64_t r0 = (uint64_t)blockIdx.x * kGramRows; r0 < rows;
       r0 += (uint64_t)gridDim.x * kGramRows) {
    const int nr = (int)((rows - r0 < (uint64_t)kGramRows) ? rows - r0 : kGramRows);
    __syncthreads();
    for (int k = tid; k < kGramRows * Rp; k += 256) {
      const int i = k / Rp, c = k % Rp;
      sX[k] = (i < nr && c < R) ? FtV[(r0 + i) * (uint64_t)R + c] : 0.0;
    }
    __syncthreads();
    // Product: thread handles rows i = tid / (Rp/ TM) ... flattened outputs.
    for (int o = tid; o < kGramRows * Rp; o += 256) {
      const int i = o / Rp, r = o % Rp;
      double s = 0.0;
      if (i < nr && r < R) {
        for (int k = 0; k < R; ++k) s = fma(sX[i * Rp + k], sA[k * Rp + r], s);
        if (divide_lambda) s /= lambda[r];
        F[(r0 + i) * (uint64_t)R + r] = s;
        dacc = fma(s, sX[i * Rp + r], dacc);
      }
      sY[o] = s;
    }
    __syncthreads();
    gram_tile<TM>(sY, nr, Rp, a0, b0, acc);
  }
  store_partial<TM>(part + (uint64_t)blockIdx.x * R * R, R, a0, b0, acc);
  if (dots != nullptr) {
    __syncthreads();  // sX is free
    sX[tid] = dacc;
    __syncthreads();
    if (tid < R) {
      double t = 0.0;
      for (int k = 0; k < 256 / Rp; ++k) t += sX[k * Rp + tid];
      dots[(uint64_t)blockIdx.x * R + tid] = t;
    }
  }
}

__global__ void k_norm_finalize(const double* __restrict__ part, int nblk, int R,
                                int generic_norm, double* __restrict__ lambda,
                                double* __restrict__ G, double* __restrict__ scale) {
  extern __shared__ double sh[];  // R scales
  const int RR = R * R;
  for (int r = threadIdx.x; r < R; r += blockDim.x) {
    double s = 0.0;
    for (int b = 0; b < nblk; ++b) s += part[(uint64_t)b * RR + r * R + r];
    double nrm = sqrt(s);
    double sc;
    if (generic_norm) {
      if (!isfinite(nrm) || nrm < 1e-14) nrm = 1.0;
      lambda[r] = nrm;
      sc = 1.0 / nrm;
    } else {
      if (nrm < 1e-14) {
        lambda[r] = 0.0;
        sc = 0.0;
      } else {
        lambda[r] = lambda[r] * nrm;
        sc = 1.0 / nrm;
      }
    }
    scale[r] = sc;
    sh[r] = sc;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < RR; i += blockDim.x) {
    double s = 0.0;
    for (int b = 0; b < nblk; ++b) s += part[(uint64_t)b * RR + i];
    G[i] = sh[i / R] * s * sh[i % R];
  }
}

__global__ void k_scale_cols(double* __restrict__ F, uint64_t n, int R,
                             const double* __restrict__ scale) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    F[i] *= scale[i % R];
}

__global__ void k_fit_final(const double* __restrict__ dot_part, int nblk,
                            const double* __restrict__ scale, const double* __restrict__ lambda,
                            GPtrs g, int ng, int R, double* __restrict__ out) {
  __shared__ double sh[1024];
  const int tid = threadIdx.x;
  double ip = 0.0, m2 = 0.0;
  for (int r = tid; r < R; r += blockDim.x) {
    double d = 0.0;
    for (int b = 0; b < nblk; ++b) d += dot_part[(uint64_t)b * R + r];
    if (scale) d *= scale[r];
    ip += lambda[r] * d;
  }
  for (int i = tid; i < R * R; i += blockDim.x) {
    double v = lambda[i / R] * lambda[i % R];
    for (int k = 0; k < ng; ++k) v *= g.p[k][i];
    m2 += v;
  }
  sh[tid] = ip;
  __syncthreads();
  for (int o = blockDim.x / 2; o > 0; o >>= 1) {
    if (tid < o) sh[tid] += sh[tid + o];
    __syncthreads();
  }
  if (tid == 0) out[0] = sh[0];
  __syncthreads();
  sh[tid] = m2;
  __syncthreads();
  for (int o = blockDim.x / 2; o > 0; o >>= 1) {
    if (tid < o) sh[tid] += sh[tid + o];
    __syncthreads();
  }
  if (tid == 0) out[1] = sh[0];
}

__global__ void k_sumsq_partial(const double* __restrict__ v, uint64_t n, double* __restrict__ part) {
  __shared__ double sh[256];
  double s = 0.0;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    s = fma(v[i], v[i], s);
  sh[threadIdx.x] = s;
  __syncthreads();
  for (int o = 128; o > 0; o >>= 1) {
    if (threadIdx.x < o) sh[threadIdx.x] += sh[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) part[blockIdx.x] = sh[0];
}

__global__ void k_residual_partial(ResidualArgs a, double* __restrict__ part) {
  __shared__ double sh[256];
  double s = 0.0;
  for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < a.nnz;
       e += (uint64_t)gridDim.x * blockDim.x) {
    double xhat = 0.0;
    for (int r = 0; r < a.R; ++r) {
      double p = a.lambda[r];
      for (int m = 0; m < a.N; ++m) p *= a.F[m][(uint64_t)a.idx[m][e] * a.R + r];
      xhat += p;
    }
    const double d = a.val[e] - xhat;
    s = fma(d, d, s);
  }
  sh[threadIdx.x] = s;
  __syncthreads();
  for (int o = 128; o > 0; o >>= 1) {
    if (threadIdx.x < o) sh[threadIdx.x] += sh[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) part[blockIdx.x] = sh[0];
}

__global__ void k_sum_serial(const double* __restrict__ part, int n, double* __restrict__ out) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    double s = 0.0;
    for (int i = 0; i < n; ++i) s += part[i];
    out[0] = s;
  }
}

}  // namespace

int launch_gram_partial(const double* F, uint64_t rows, int R, double* part, int max_blocks,
                        cudaStream_t s) {
  CPTC_REQUIRE(R >= 1 && R <= 128, CPTC_E_UNSUP, "rank must be in [1, 128]");
  int nblk = (int)((rows + kGramRows - 1) / kGramRows);
  if (nblk > max_blocks) nblk = max_blocks;
  if (nblk < 1) nblk = 1;
  switch (padded_rank(R)) {
    case 16: k_gram_partial<1><<<nblk, 256, 0, s>>>(F, rows, R, part); break;
    case 32: k_gram_partial<2><<<nblk, 256, 0, s>>>(F, rows, R, part); break;
    case 64: k_gram_partial<4><<<nblk, 256, 0, s>>>(F, rows, R, part); break;
    default: k_gram_partial<8><<<nblk, 256, 0, s>>>(F, rows, R, part); break;
  }
  CPTC_LAUNCH_CHECK();
  return nblk;
}

void launch_partial_sum(const double* part, int nblk, int len, double* out, cudaStream_t s) {
  k_partial_sum<<<(unsigned)((len + 31) / 32), 256, 0, s>>>(part, nblk, len, out, 0);
  CPTC_LAUNCH_CHECK();
}

void launch_partial_sum_add(const double* part, int nblk, int len, double* out, cudaStream_t s) {
  k_partial_sum<<<(unsigned)((len + 31) / 32), 256, 0, s>>>(part, nblk, len, out, 1);
  CPTC_LAUNCH_CHECK();
}

void launch_gram_reduce(const double* part, int nblk, int R, double* G, cudaStream_t s) {
  launch_partial_sum(part, nblk, R * R, G, s);
}

void launch_sym_inverse(const double* const* Gs, int ng, int R, int mode, double* FtF,
                        double* Ainv, int* status, cudaStream_t s) {
  CPTC_REQUIRE(R >= 1 && R <= 128, CPTC_E_UNSUP, "rank must be in [1, 128]");
  CPTC_REQUIRE(ng >= 1 && ng <= CPTC_MAX_ORDER, CPTC_E_ARG, "bad Gram count");
  // Ainv holds 2*R*R doubles (+1 int flag after them): the flag gates the
  // pseudo-inverse kernel on the sweep's outcome.
  int* gate = reinterpret_cast<int*>(Ainv + 2 * (size_t)R * R);
  GPtrs g{};
  for (int k = 0; k < ng; ++k) g.p[k] = Gs[k];
  if (mode != kInvPinv) {
    // (warps, rows per warp, 32-column slices per lane): the R x R matrix
    // stays in registers (R = 128: 32 doubles per thread, 512 threads).
    const int rdg = mode == kInvCholRidge ? 1 : 0;
    int* fl = mode == kInvAuto ? gate : nullptr;
    if (R <= 32) k_sweep_inverse<32, 1, 1><<<1, 1024, 0, s>>>(g, ng, R, rdg, FtF, Ainv, status, fl);
    else if (R <= 64) k_sweep_inverse<16, 4, 2><<<1, 512, 0, s>>>(g, ng, R, rdg, FtF, Ainv, status, fl);
    else if (R <= 96) k_sweep_inverse<16, 6, 3><<<1, 512, 0, s>>>(g, ng, R, rdg, FtF, Ainv, status, fl);
    else k_sweep_inverse<16, 8, 4><<<1, 512, 0, s>>>(g, ng, R, rdg, FtF, Ainv, status, fl);
    CPTC_LAUNCH_CHECK();
    if (mode == kInvCholRidge) return;
  } else {
    k_hadamard<<<grid_for((uint64_t)R * R, 256), 256, 0, s>>>(g, ng, R, FtF);
    CPTC_LAUNCH_CHECK();
  }
  const int n = (R + 1) & ~1;
  int threads = 32 * (n / 2);
  if (threads > 1024) threads = 1024;
  if (threads < 64) threads = 64;
  const size_t smem = ((size_t)R * R + R) * sizeof(double);
  CPTC_CUDA(cudaFuncSetAttribute(k_pinv_jacobi, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem));
  k_pinv_jacobi<<<1, threads, smem, s>>>(FtF, R, Ainv, status, mode == kInvAuto ? gate : nullptr);
  CPTC_LAUNCH_CHECK();
}

int launch_apply_solve(const double* FtV, const double* Ainv, const double* lambda,
                       int divide_lambda, uint64_t rows, int R, double* F, double* part,
                       int max_blocks, cudaStream_t s, double* dots) {
  int nblk = (int)((rows + kGramRows - 1) / kGramRows);
  if (nblk > max_blocks) nblk = max_blocks;
  if (nblk < 1) nblk = 1;
  const int Rp = padded_rank(R);
  const size_t smem = ((size_t)Rp * Rp + 2 * (size_t)kGramRows * Rp) * sizeof(double);
#define CPTC_APPLY(TM)                                                                       \
  do {                                                                                       \
    CPTC_CUDA(cudaFuncSetAttribute(k_apply_solve<TM>,                                        \
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)); \
    k_apply_solve<TM><<<nblk, 256, smem, s>>>(FtV, Ainv, lambda, divide_lambda, rows, R, F,  \
                                              part, dots);                                   \
  } while (0)
  switch (Rp) {
    case 16: CPTC_APPLY(1); break;
    case 32: CPTC_APPLY(2); break;
    case 64: CPTC_APPLY(4); break;
    default: CPTC_APPLY(8); break;
  }
#undef CPTC_APPLY
  CPTC_LAUNCH_CHECK();
  return nblk;
}

void launch_norm_finalize(const double* part, int nblk, int R, int generic_norm,
                          double* lambda, double* G, double* scale, cudaStream_t s) {
  k_norm_finalize<<<1, 1024, R * sizeof(double), s>>>(part, nblk, R, generic_norm, lambda, G,
                                                      scale);
  CPTC_LAUNCH_CHECK();
}

void launch_scale_cols(double* F, uint64_t rows, int R, const double* scale, cudaStream_t s) {
  const uint64_t n = rows * (uint64_t)R;
  k_scale_cols<<<grid_for(n, 256, 148 * 32), 256, 0, s>>>(F, n, R, scale);
  CPTC_LAUNCH_CHECK();
}

void launch_fit_final(const double* dot_part, int nblk, const double* scale, const double* lambda,
                      const double* const* Gs, int ng, int R, double* out, cudaStream_t s) {
  GPtrs g{};
  for (int k = 0; k < ng; ++k) g.p[k] = Gs[k];
  k_fit_final<<<1, 1024, 0, s>>>(dot_part, nblk, scale, lambda, g, ng, R, out);
  CPTC_LAUNCH_CHECK();
}

void launch_residual(const ResidualArgs& a, double* part, int max_blocks, double* out,
                     cudaStream_t s) {
  const int nblk = (int)grid_for(a.nnz, 256, (unsigned)max_blocks);
  k_residual_partial<<<nblk, 256, 0, s>>>(a, part);
  CPTC_LAUNCH_CHECK();
  k_sum_serial<<<1, 32, 0, s>>>(part, nblk, out);
  CPTC_LAUNCH_CHECK();
}

void launch_sumsq(const double* v, uint64_t n, double* part, int max_blocks, double* out,
                  cudaStream_t s) {
  int nblk = (int)grid_for(n, 256, (unsigned)max_blocks);
  k_sumsq_partial<<<nblk, 256, 0, s>>>(v, n, part);
  CPTC_LAUNCH_CHECK();
  k_sum_serial<<<1, 32, 0, s>>>(part, nblk, out);
  CPTC_LAUNCH_CHECK();
}

}  // namespace cptc
