// FP64 sparse MTTKRP over a sorted view (the residual of the hybrid path, or
// every nonzero on the FP64 path).
//
// Computes, for target mode n, FtV[t, r] += sum_e v_e * prod_{m != n} F_m[o_m(e), r]
// (reference: mttkrp_rowsorted_coalesced_kernel, src/sparse.cu:614-711, and
// g_mttkrp_seg_pack_kernel, src/generic.cu:271-343).
//
// B200 design:
//  * nonzero-balanced tasks of kTask elements per lane group (a warp for
//    R >= 32, R lanes for R < 32); row boundaries come from flags in the
//    element word, so heavy (Zipf head) rows need no host-side segmenting;
//  * lane = rank slice: 1, 2 or 4 consecutive ranks per lane, loaded as
//    8- or 16-byte vectors, so one factor row is one coalesced request;
//  * the view is sorted by (target, outer modes, gathered mode): along a
//    fiber of equal outer indices the outer rows are loaded once and the
//    fiber sum  sum_e v_e F_g[g_e]  is multiplied by them at the fiber end,
//    so ~1/fiber-length of the second gather disappears (N-order kernel,
//    and the order-3 record kernel at R >= 64 where it measures faster);
//  * order 3: the record stream is staged through shared memory by cp.async
//    (L2 only), N-order: element words/values are streamed with evict-first
//    loads, so the factor matrices stay resident in L1/L2; gathers of U
//    elements are issued before any of them is consumed;
//  * a row that starts and ends inside one task is written with a plain
//    read-modify-write (it has no other writer in this launch); rows cut by
//    a task boundary are combined with FP64 atomicAdd.
#include <cstdlib>
#include <cstring>

#include "engine.hpp"
#include "kernels.hpp"

namespace cptc {

namespace {

struct FoPtrs {
  const double* p[4];
};

// Ranks held by lane `glane` of a GW-lane group.  Vector paths: 1 or 2
// consecutive ranks, or with 4 ranks two pairs, one in each half of the row
// (ranks 2g, 2g+1 and 2GW+2g, 2GW+2g+1), so that each 16-byte load
// instruction of the group reads one contiguous half row: every sector it
// touches is used whole.  Scalar paths: ranks glane + k*GW.
template <int GW, int RPL, bool VEC>
struct Lanes {
  int r[RPL];
  bool ok[RPL];
  __device__ Lanes(int glane, int R) {
#pragma unroll
    for (int k = 0; k < RPL; ++k) {
      if (VEC && RPL == 4) r[k] = (k < 2) ? 2 * glane + k : 2 * GW + 2 * glane + (k - 2);
      else r[k] = VEC ? glane * RPL + k : glane + k * GW;
      ok[k] = r[k] < R;
    }
  }
};

template <int GW, int RPL, bool VEC>
__device__ __forceinline__ void load_row(const double* __restrict__ F, uint64_t row, int R,
                                         int glane, const Lanes<GW, RPL, VEC>& L, double (&x)[RPL]) {
  const double* base = F + row * (uint64_t)R;
  if constexpr (VEC && RPL == 1) {
    x[0] = __ldg(base + glane);
  } else if constexpr (VEC && RPL == 2) {
    const double2 a = __ldg(reinterpret_cast<const double2*>(base) + glane);
    x[0] = a.x;
    x[1] = a.y;
  } else if constexpr (VEC && RPL == 4) {
    const double2 a = __ldg(reinterpret_cast<const double2*>(base) + glane);
    const double2 b = __ldg(reinterpret_cast<const double2*>(base) + GW + glane);
    x[0] = a.x;
    x[1] = a.y;
    x[2] = b.x;
    x[3] = b.y;
  } else {
#pragma unroll
    for (int k = 0; k < RPL; ++k) x[k] = L.ok[k] ? __ldg(base + L.r[k]) : 0.0;
  }
}

// Software pipeline per lane group: element words of batch b+1 are loaded
// while batch b is processed, and the factor rows of sub-batch k+1 are
// gathered before sub-batch k is consumed (two register buffers, selected
// at compile time by the sub-batch parity, so U*GW/U must be even).
template <int GW, int RPL, bool VEC, int U>
__global__ void __launch_bounds__(256, 2) k_mttkrp_view(MttkrpArgs a) {
  constexpr int GPW = 32 / GW;
  constexpr int SUBS = GW / U;
  static_assert(SUBS % 2 == 0, "an even number of sub-batches per batch");
  const int lane = threadIdx.x & 31;
  const int glane = lane % GW;
  const int gid = lane / GW;
  const unsigned gmask = (GW == 32) ? 0xffffffffu : (((1u << GW) - 1u) << (gid * GW));
  const uint64_t task =
      a.task0 + ((uint64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * GPW + gid;
  if (task >= a.ntasks) return;
  const int R = a.R;
  const Lanes<GW, RPL, VEC> L(glane, R);
  const uint64_t p0 = task * (uint64_t)a.task;
  const uint64_t p1 = (p0 + a.task < a.nnz) ? p0 + a.task : a.nnz;

  uint32_t rowi = a.task_row[task];
  uint32_t row = a.rows[rowi];
  bool row_began_here = (a.gw[p0] & kRowFlag) != 0;
  const bool last_row_ends_here = (p1 == a.nnz) || (a.gw[p1] & kRowFlag);

  double accr[RPL], accf[RPL], ff[RPL];
#pragma unroll
  for (int k = 0; k < RPL; ++k) accr[k] = accf[k] = ff[k] = 0.0;

  auto write_row = [&](bool owned) {
    double* dst = a.out + (uint64_t)row * (uint64_t)R;
#pragma unroll
    for (int k = 0; k < RPL; ++k) {
      if (!L.ok[k]) continue;
      if (owned) dst[L.r[k]] += accr[k];
      else atomicAdd(dst + L.r[k], accr[k]);
      accr[k] = 0.0;
    }
  };
  auto load_batch = [&](uint64_t b, uint32_t& w, uint32_t& o, double& v) {
    const uint64_t p = b + glane;
    w = 0u;
    o = 0u;
    v = 0.0;
    if (p < p1) {
      w = __ldcs(a.gw + p);
      v = __ldcs(a.val + p);
      if (a.nout > 0) o = __ldcs(a.oidx + p);
    }
  };
  auto gather = [&](uint32_t wsrc, int j0, int cnt, double (&g)[U][RPL]) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t w = __shfl_sync(gmask, wsrc, j0 + u, GW);
      if (j0 + u < cnt) {
        load_row<GW, RPL, VEC>(a.Fg, w & kIdxMask, R, glane, L, g[u]);
      } else {
#pragma unroll
        for (int k = 0; k < RPL; ++k) g[u][k] = 0.0;
      }
    }
  };

  uint32_t cw, co, nw = 0u, no = 0u;
  double cv, nv = 0.0;
  load_batch(p0, cw, co, cv);
  if (glane == 0) cw = (cw & ~kRowFlag) | kFibFlag;  // row state is set; open a fiber
  if (p0 + GW < p1) load_batch(p0 + GW, nw, no, nv);
  double gA[U][RPL], gB[U][RPL];
  gather(cw, 0, (p1 - p0 < (uint64_t)GW) ? (int)(p1 - p0) : GW, gA);

  for (uint64_t b = p0; b < p1; b += GW) {
    const int cnt = (p1 - b < (uint64_t)GW) ? (int)(p1 - b) : GW;
    const bool has_next = b + GW < p1;
    const int cnt_next = has_next ? ((p1 - b - GW < (uint64_t)GW) ? (int)(p1 - b - GW) : GW) : 0;
#pragma unroll
    for (int sb = 0; sb < SUBS; ++sb) {
      const int j0 = sb * U;
      if (j0 >= cnt) break;
      double (&cur)[U][RPL] = (sb & 1) ? gB : gA;
      double (&nxt)[U][RPL] = (sb & 1) ? gA : gB;
      if (j0 + U < cnt) gather(cw, j0 + U, cnt, nxt);
      else if (has_next) gather(nw, 0, cnt_next, nxt);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int j = j0 + u;
        if (j >= cnt) break;
        const uint32_t ww = __shfl_sync(gmask, cw, j, GW);
        const double vj = __shfl_sync(gmask, cv, j, GW);
        if (ww & kFibFlag) {
          const uint32_t oj = __shfl_sync(gmask, co, j, GW);
#pragma unroll
          for (int k = 0; k < RPL; ++k) {
            accr[k] = fma(accf[k], ff[k], accr[k]);
            accf[k] = 0.0;
          }
          if (ww & kRowFlag) {
            write_row(row_began_here);
            row = a.rows[++rowi];
            row_began_here = true;
          }
          if (a.nout == 0) {
#pragma unroll
            for (int k = 0; k < RPL; ++k) ff[k] = 1.0;
          } else {
            load_row<GW, RPL, VEC>(a.Fo[0], oj, R, glane, L, ff);
            for (int q = 1; q < a.nout; ++q) {
              const uint32_t oq = a.oidx[(uint64_t)q * a.nnz + b + j];
              double t[RPL];
              load_row<GW, RPL, VEC>(a.Fo[q], oq, R, glane, L, t);
#pragma unroll
              for (int k = 0; k < RPL; ++k) ff[k] *= t[k];
            }
          }
        }
#pragma unroll
        for (int k = 0; k < RPL; ++k) accf[k] = fma(vj, cur[u][k], accf[k]);
      }
    }
    cw = nw;
    co = no;
    cv = nv;
    if (b + 2 * GW < p1) load_batch(b + 2 * GW, nw, no, nv);
  }
#pragma unroll
  for (int k = 0; k < RPL; ++k) accr[k] = fma(accf[k], ff[k], accr[k]);
  write_row(row_began_here && last_row_ends_here);
}

// Order 3: one 16-byte record per nonzero {index word, outer index, value},
// read by every lane of the group with a single uniform 128-bit load (no
// shuffles); the two factor rows of the nonzero are 8/16-byte vector loads
// across the group.  U nonzeros are in flight per group and the records of
// the next U are loaded before the current U are consumed.  The kernel
// keeps few registers so that many warps hide the gather latency.
// Per nonzero acc += (v * F_g[g, r]) * F_o[o, r], the reference's product
// v * F1 * F2 (src/sparse.cu:666-669).
template <int GW, int RPL, bool VEC, int U>
__global__ void __launch_bounds__(256) k_mttkrp_rec3(const uint4* __restrict__ rec,
                                                     const uint32_t* __restrict__ rows,
                                                     const uint32_t* __restrict__ task_row,
                                                     uint64_t nnz, uint64_t task0,
                                                     uint64_t ntasks,
                                                     uint32_t tsize, int R,
                                                     const double* __restrict__ Fg,
                                                     const double* __restrict__ Fo,
                                                     double* __restrict__ out) {
  constexpr int GPW = 32 / GW;
  const int lane = threadIdx.x & 31;
  const int glane = lane % GW;
  const uint64_t task =
      task0 + ((uint64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * GPW + lane / GW;
  if (task >= ntasks) return;
  const Lanes<GW, RPL, VEC> L(glane, R);
  const uint64_t p0 = task * (uint64_t)tsize;
  const uint64_t p1 = (p0 + tsize < nnz) ? p0 + tsize : nnz;

  uint32_t rowi = task_row[task];
  uint32_t row = rows[rowi];
  bool began = (rec[p0].x & kRowFlag) != 0;
  const bool ends = (p1 == nnz) || (rec[p1].x & kRowFlag);

  double acc[RPL];
#pragma unroll
  for (int k = 0; k < RPL; ++k) acc[k] = 0.0;
  auto write_row = [&](bool owned) {
    double* dst = out + (uint64_t)row * (uint64_t)R;
#pragma unroll
    for (int k = 0; k < RPL; ++k) {
      if (!L.ok[k]) continue;
      if (owned) dst[L.r[k]] += acc[k];
      else atomicAdd(dst + L.r[k], acc[k]);
      acc[k] = 0.0;
    }
  };
  auto step = [&](const uint4& e, const double (&g)[RPL], const double (&f)[RPL], bool first) {
    if ((e.x & kRowFlag) && !first) {
      write_row(began);
      row = rows[++rowi];
      began = true;
    }
    const double v = __hiloint2double((int)e.w, (int)e.z);
#pragma unroll
    for (int k = 0; k < RPL; ++k) acc[k] = fma(v * g[k], f[k], acc[k]);
  };

  uint64_t p = p0;
  const uint64_t pfull = p0 + ((p1 - p0) / U) * U;
  uint4 cur[U];
  if (p < pfull) {
#pragma unroll
    for (int u = 0; u < U; ++u) cur[u] = __ldcs(rec + p + u);
  }
#pragma unroll 1
  for (; p < pfull; p += U) {
    double g[U][RPL], f[U][RPL];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      load_row<GW, RPL, VEC>(Fg, cur[u].x & kIdxMask, R, glane, L, g[u]);
      load_row<GW, RPL, VEC>(Fo, cur[u].y, R, glane, L, f[u]);
    }
    uint4 nxt[U];
    if (p + U < pfull) {
#pragma unroll
      for (int u = 0; u < U; ++u) nxt[u] = __ldcs(rec + p + U + u);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) step(cur[u], g[u], f[u], p + u == p0);
#pragma unroll
    for (int u = 0; u < U; ++u) cur[u] = nxt[u];
  }
  for (; p < p1; ++p) {  // tail of fewer than U nonzeros
    const uint4 e = __ldcs(rec + p);
    double g[RPL], f[RPL];
    load_row<GW, RPL, VEC>(Fg, e.x & kIdxMask, R, glane, L, g);
    load_row<GW, RPL, VEC>(Fo, e.y, R, glane, L, f);
    step(e, g, f, p == p0);
  }
  write_row(began && ends);
}

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  const unsigned sa = (unsigned)__cvta_generic_to_shared(smem_dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(sa), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// Order 3 with the record stream staged through shared memory: each lane
// group double-buffers chunks of 2*GW records, copied with cp.async (16
// bytes per lane, L2 only, so the stream leaves L1 to the factor rows) one
// chunk ahead; no registers hold prefetched records.  The factor rows are
// register loads, U nonzeros issued together (staging them in shared memory
// as well measured 2x slower: it triples traffic on the L1/shared path).
// Same arithmetic and row/atomic rules as k_mttkrp_rec3.  MINB: minimum
// resident CTAs per SM asked of the register allocator.
template <int GW, int RPL, int U, int MINB, bool FIB>
__global__ void __launch_bounds__(256, MINB) k_mttkrp_rec3s(const uint4* __restrict__ rec,
                                                           const uint32_t* __restrict__ rows,
                                                           const uint32_t* __restrict__ task_row,
                                                           uint64_t nnz, uint64_t task0,
                                                           uint64_t ntasks, uint32_t tsize, int R,
                                                           const double* __restrict__ Fg,
                                                           const double* __restrict__ Fo,
                                                           double* __restrict__ out) {
  constexpr int GPW = 32 / GW;
  constexpr int CH = 2 * GW;  // records per chunk: two per lane
  static_assert(CH % U == 0, "chunk holds whole batches");
  __shared__ __align__(16) uint4 sbuf[8 * GPW][2][CH];
  const int lane = threadIdx.x & 31, glane = lane % GW, gw = lane / GW;
  const int warp = threadIdx.x >> 5;
  const int grp = warp * GPW + gw;
  const unsigned gmask = (GW == 32) ? 0xffffffffu : (((1u << GW) - 1u) << (gw * GW));
  const uint64_t task = task0 + ((uint64_t)blockIdx.x * 8 + warp) * GPW + gw;
  if (task >= ntasks) return;
  const Lanes<GW, RPL, true> L(glane, R);
  const uint64_t p0 = task * (uint64_t)tsize;
  const uint64_t p1 = (p0 + tsize < nnz) ? p0 + tsize : nnz;
  const int n = (int)(p1 - p0);
  uint4 (*buf)[CH] = sbuf[grp];

  uint32_t rowi = task_row[task];
  uint32_t row = rows[rowi];
  bool began = (rec[p0].x & kRowFlag) != 0;
  const bool ends = (p1 == nnz) || (rec[p1].x & kRowFlag);

  auto fetch = [&](int c) {  // chunk c -> buffer c & 1 (records past the task end skipped)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int q = c * CH + h * GW + glane;
      if (q < n) cp_async16(&buf[c & 1][h * GW + glane], rec + p0 + q);
    }
    cp_async_commit();
  };

  double acc[RPL], fs[RPL], fo[RPL];
#pragma unroll
  for (int k = 0; k < RPL; ++k) acc[k] = fs[k] = fo[k] = 0.0;
  auto write_row = [&](bool owned) {
    double* dst = out + (uint64_t)row * (uint64_t)R;
#pragma unroll
    for (int k = 0; k < RPL; ++k) {
      if (!L.ok[k]) continue;
      if (owned) dst[L.r[k]] += acc[k];
      else atomicAdd(dst + L.r[k], acc[k]);
      acc[k] = 0.0;
    }
  };
  // One nonzero: row change, then acc += (v*g)*f; with FIB the view's sort
  // order (target, outer, gathered) is used: the outer row is loaded only
  // for a fiber's first nonzero and the fiber sum sum v*g is multiplied by
  // it once, at the fiber end (acc += (sum_e v_e g_e) * f).
  auto step = [&](uint32_t ex, const uint4& e, const double (&g)[RPL], const double (&f)[RPL],
                  bool first) {
    const bool fib = (ex & kFibFlag) != 0;
    if (FIB && fib && !first) {
#pragma unroll
      for (int k = 0; k < RPL; ++k) {
        acc[k] = fma(fs[k], fo[k], acc[k]);
        fs[k] = 0.0;
      }
    }
    if ((ex & kRowFlag) && !first) {
      write_row(began);
      row = rows[++rowi];
      began = true;
    }
    const double v = __hiloint2double((int)e.w, (int)e.z);
    if (FIB) {
      if (fib || first) {
#pragma unroll
        for (int k = 0; k < RPL; ++k) fo[k] = f[k];
      }
#pragma unroll
      for (int k = 0; k < RPL; ++k) fs[k] = fma(v, g[k], fs[k]);
    } else {
#pragma unroll
      for (int k = 0; k < RPL; ++k) acc[k] = fma(v * g[k], f[k], acc[k]);
    }
  };

  const int nch = (n + CH - 1) / CH;
  fetch(0);
  if (nch > 1) fetch(1);
  else cp_async_commit();
#pragma unroll 1
  for (int c = 0; c < nch; ++c) {
    cp_async_wait<1>();  // chunk c has landed (chunk c + 1 may be in flight)
    __syncwarp(gmask);
    const int q0 = c * CH;
    const int qe = (q0 + CH < n) ? q0 + CH : n;
    const uint4* cb = buf[c & 1];
    int q = q0;
#pragma unroll 1
    for (; q + U <= qe; q += U) {
      double g[U][RPL], f[U][RPL];
      uint32_t ex[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const uint4 e = cb[q - q0 + u];
        ex[u] = e.x;
        load_row<GW, RPL, true>(Fg, e.x & kIdxMask, R, glane, L, g[u]);
        if (!FIB || (e.x & kFibFlag) || q + u == 0) {
          load_row<GW, RPL, true>(Fo, e.y, R, glane, L, f[u]);
        } else {
#pragma unroll
          for (int k = 0; k < RPL; ++k) f[u][k] = 0.0;
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) step(ex[u], cb[q - q0 + u], g[u], f[u], q + u == 0);
    }
    for (; q < qe; ++q) {
      const uint4 e = cb[q - q0];
      double g[RPL], f[RPL];
      load_row<GW, RPL, true>(Fg, e.x & kIdxMask, R, glane, L, g);
      if (!FIB || (e.x & kFibFlag) || q == 0) {
        load_row<GW, RPL, true>(Fo, e.y, R, glane, L, f);
      } else {
#pragma unroll
        for (int k = 0; k < RPL; ++k) f[k] = 0.0;
      }
      step(e.x, e, g, f, q == 0);
    }
    __syncwarp(gmask);  // every lane is done with buffer c & 1
    if (c + 2 < nch) fetch(c + 2);
    else cp_async_commit();
  }
  cp_async_wait<0>();
  if (FIB) {
#pragma unroll
    for (int k = 0; k < RPL; ++k) acc[k] = fma(fs[k], fo[k], acc[k]);
  }
  write_row(began && ends);
}

template <int GW, int RPL, int U, int MINB, bool FIB = false>
void launch_rec3s(const MttkrpArgs& a, cudaStream_t s) {
  constexpr int GPW = 32 / GW;
  if (GW * RPL <= 32) {
    // R <= 32: the largest shared-memory carveout measured fastest on config 4
    // (R = 32: 0.955 -> 0.92 ms per mode against the driver's default; the
    // factor-row gathers mostly miss L1 whatever its size).
    CPTC_CUDA(cudaFuncSetAttribute(k_mttkrp_rec3s<GW, RPL, U, MINB, FIB>,
                                   cudaFuncAttributePreferredSharedMemoryCarveout, 100));
  }
  const uint64_t warps = (a.ntasks - a.task0 + GPW - 1) / GPW;
  const unsigned blocks = (unsigned)((warps + 7) / 8);
  k_mttkrp_rec3s<GW, RPL, U, MINB, FIB><<<blocks, 256, 0, s>>>(a.rec, a.rows, a.task_row, a.nnz,
                                                                a.task0, a.ntasks, a.task, a.R,
                                                                a.Fg, a.Fo[0], a.out);
  CPTC_LAUNCH_CHECK();
}

// Orders 4-6 (NOUT = 2..4 outer modes): 32-byte records {word, o0, o1, o2}
// {o3, 0, value} staged through shared memory by cp.async as in
// k_mttkrp_rec3s (one record per lane per chunk).  The outer rows of a
// fiber are loaded with the batch, only for the fiber's first nonzero, and
// multiplied together; per fiber acc += (sum_e v_e g_e) * prod_q F_q[o_q] —
// the association of k_mttkrp_view, whose outer-row loads at a fiber start
// wait on a shuffle and a further index load.
template <int GW, int RPL, int U, int NOUT>
__global__ void __launch_bounds__(256) k_mttkrp_recns(const uint4* __restrict__ rec,
                                                     const uint32_t* __restrict__ rows,
                                                     const uint32_t* __restrict__ task_row,
                                                     uint64_t nnz, uint64_t task0,
                                                     uint64_t ntasks, uint32_t tsize, int R,
                                                     const double* __restrict__ Fg, FoPtrs fo_p,
                                                     double* __restrict__ out) {
  constexpr int GPW = 32 / GW;
  constexpr int CH = GW;  // records per chunk: one per lane
  static_assert(CH % U == 0, "chunk holds whole batches");
  __shared__ __align__(16) uint4 sbuf[8 * GPW][2][2 * CH];
  const int lane = threadIdx.x & 31, glane = lane % GW, gw = lane / GW;
  const int warp = threadIdx.x >> 5;
  const int grp = warp * GPW + gw;
  const unsigned gmask = (GW == 32) ? 0xffffffffu : (((1u << GW) - 1u) << (gw * GW));
  const uint64_t task = task0 + ((uint64_t)blockIdx.x * 8 + warp) * GPW + gw;
  if (task >= ntasks) return;
  const Lanes<GW, RPL, true> L(glane, R);
  const uint64_t p0 = task * (uint64_t)tsize;
  const uint64_t p1 = (p0 + tsize < nnz) ? p0 + tsize : nnz;
  const int n = (int)(p1 - p0);
  uint4 (*buf)[2 * CH] = sbuf[grp];

  uint32_t rowi = task_row[task];
  uint32_t row = rows[rowi];
  bool began = (rec[2 * p0].x & kRowFlag) != 0;
  const bool ends = (p1 == nnz) || (rec[2 * p1].x & kRowFlag);

  auto fetch = [&](int c) {
    const int q = c * CH + glane;
    if (q < n) {
      cp_async16(&buf[c & 1][2 * glane], rec + 2 * (p0 + q));
      cp_async16(&buf[c & 1][2 * glane + 1], rec + 2 * (p0 + q) + 1);
    }
    cp_async_commit();
  };

  double acc[RPL], fs[RPL], fo[RPL];
#pragma unroll
  for (int k = 0; k < RPL; ++k) acc[k] = fs[k] = fo[k] = 0.0;
  auto write_row = [&](bool owned) {
    double* dst = out + (uint64_t)row * (uint64_t)R;
#pragma unroll
    for (int k = 0; k < RPL; ++k) {
      if (!L.ok[k]) continue;
      if (owned) dst[L.r[k]] += acc[k];
      else atomicAdd(dst + L.r[k], acc[k]);
      acc[k] = 0.0;
    }
  };
  auto outer_rows = [&](const uint4& r0, const uint4& r1, double (&f)[RPL]) {
    const uint32_t o[4] = {r0.y, r0.z, r0.w, r1.x};
    load_row<GW, RPL, true>(fo_p.p[0], o[0], R, glane, L, f);
#pragma unroll
    for (int q = 1; q < NOUT; ++q) {
      double t[RPL];
      load_row<GW, RPL, true>(fo_p.p[q], o[q], R, glane, L, t);
#pragma unroll
      for (int k = 0; k < RPL; ++k) f[k] *= t[k];
    }
  };
  auto step = [&](const uint4& r0, const uint4& r1, const double (&g)[RPL],
                  const double (&f)[RPL], bool first) {
    const bool fib = (r0.x & kFibFlag) != 0;
    if (fib && !first) {
#pragma unroll
      for (int k = 0; k < RPL; ++k) {
        acc[k] = fma(fs[k], fo[k], acc[k]);
        fs[k] = 0.0;
      }
    }
    if ((r0.x & kRowFlag) && !first) {
      write_row(began);
      row = rows[++rowi];
      began = true;
    }
    if (fib || first) {
#pragma unroll
      for (int k = 0; k < RPL; ++k) fo[k] = f[k];
    }
    const double v = __hiloint2double((int)r1.w, (int)r1.z);
#pragma unroll
    for (int k = 0; k < RPL; ++k) fs[k] = fma(v, g[k], fs[k]);
  };

  const int nch = (n + CH - 1) / CH;
  fetch(0);
  if (nch > 1) fetch(1);
  else cp_async_commit();
#pragma unroll 1
  for (int c = 0; c < nch; ++c) {
    cp_async_wait<1>();
    __syncwarp(gmask);
    const int q0 = c * CH;
    const int qe = (q0 + CH < n) ? q0 + CH : n;
    const uint4* cb = buf[c & 1];
    int q = q0;
#pragma unroll 1
    for (; q + U <= qe; q += U) {
      double g[U][RPL], f[U][RPL];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const uint4 r0 = cb[2 * (q - q0 + u)], r1 = cb[2 * (q - q0 + u) + 1];
        load_row<GW, RPL, true>(Fg, r0.x & kIdxMask, R, glane, L, g[u]);
        if ((r0.x & kFibFlag) || q + u == 0) {
          outer_rows(r0, r1, f[u]);
        } else {
#pragma unroll
          for (int k = 0; k < RPL; ++k) f[u][k] = 0.0;
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u)
        step(cb[2 * (q - q0 + u)], cb[2 * (q - q0 + u) + 1], g[u], f[u], q + u == 0);
    }
    for (; q < qe; ++q) {
      const uint4 r0 = cb[2 * (q - q0)], r1 = cb[2 * (q - q0) + 1];
      double g[RPL], f[RPL];
      load_row<GW, RPL, true>(Fg, r0.x & kIdxMask, R, glane, L, g);
      if ((r0.x & kFibFlag) || q == 0) {
        outer_rows(r0, r1, f);
      } else {
#pragma unroll
        for (int k = 0; k < RPL; ++k) f[k] = 0.0;
      }
      step(r0, r1, g, f, q == 0);
    }
    __syncwarp(gmask);
    if (c + 2 < nch) fetch(c + 2);
    else cp_async_commit();
  }
  cp_async_wait<0>();
#pragma unroll
  for (int k = 0; k < RPL; ++k) acc[k] = fma(fs[k], fo[k], acc[k]);
  write_row(began && ends);
}

template <int GW, int RPL, int U, int NOUT>
void launch_recns(const MttkrpArgs& a, cudaStream_t s) {
  constexpr int GPW = 32 / GW;
  const uint64_t warps = (a.ntasks - a.task0 + GPW - 1) / GPW;
  const unsigned blocks = (unsigned)((warps + 7) / 8);
  FoPtrs fo{};
  for (int q = 0; q < NOUT; ++q) fo.p[q] = a.Fo[q];
  k_mttkrp_recns<GW, RPL, U, NOUT><<<blocks, 256, 0, s>>>(a.rec, a.rows, a.task_row, a.nnz,
                                                           a.task0, a.ntasks, a.task, a.R, a.Fg,
                                                           fo, a.out);
  CPTC_LAUNCH_CHECK();
}

template <int NOUT>
void launch_recns_r(const MttkrpArgs& a, cudaStream_t s) {
  switch (a.R) {
    case 8: launch_recns<8, 1, 2, NOUT>(a, s); return;
    case 16: launch_recns<8, 2, 2, NOUT>(a, s); return;
    case 32: launch_recns<16, 2, 2, NOUT>(a, s); return;
    case 64: launch_recns<16, 4, 2, NOUT>(a, s); return;
    case 128: launch_recns<32, 4, 1, NOUT>(a, s); return;
    default: throw CptcError(CPTC_E_UNSUP, "N-order records are built for R in {8,16,32,64,128}");
  }
}

template <int GW, int RPL, bool VEC, int U>
void launch_rec3(const MttkrpArgs& a, cudaStream_t s) {
  constexpr int GPW = 32 / GW;
  const uint64_t warps = (a.ntasks - a.task0 + GPW - 1) / GPW;
  const unsigned blocks = (unsigned)((warps + 7) / 8);
  k_mttkrp_rec3<GW, RPL, VEC, U><<<blocks, 256, 0, s>>>(a.rec, a.rows, a.task_row, a.nnz,
                                                         a.task0, a.ntasks, a.task, a.R, a.Fg,
                                                         a.Fo[0], a.out);
  CPTC_LAUNCH_CHECK();
}

template <int GW, int RPL, bool VEC, int U>
void launch(const MttkrpArgs& a, cudaStream_t s) {
  constexpr int GPW = 32 / GW;
  const uint64_t warps = (a.ntasks - a.task0 + GPW - 1) / GPW;
  const unsigned blocks = (unsigned)((warps + 7) / 8);
  k_mttkrp_view<GW, RPL, VEC, U><<<blocks, 256, 0, s>>>(a);
  CPTC_LAUNCH_CHECK();
}

// Lane groups of kernel `kern` (256 threads, GW-lane groups) resident on
// the whole GPU at once.
template <class K>
uint64_t slots_of(K kern, int GW, bool carve, int device) {
  if (carve)
    CPTC_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
  int sms = 148, per_sm = 0;
  CPTC_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
  CPTC_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 256, 0));
  if (per_sm < 1) per_sm = 1;
  return (uint64_t)sms * per_sm * 8 * (32 / GW);
}

}  // namespace

uint64_t mttkrp_view_slots(bool rec, int recw, int nout, int R, int device) {
  if (rec && recw == 2) {
    switch (nout * 1000 + R) {
      case 2008: return slots_of(k_mttkrp_recns<8, 1, 2, 2>, 8, false, device);
      case 2016: return slots_of(k_mttkrp_recns<8, 2, 2, 2>, 8, false, device);
      case 2032: return slots_of(k_mttkrp_recns<16, 2, 2, 2>, 16, false, device);
      case 2064: return slots_of(k_mttkrp_recns<16, 4, 2, 2>, 16, false, device);
      case 2128: return slots_of(k_mttkrp_recns<32, 4, 1, 2>, 32, false, device);
      case 3008: return slots_of(k_mttkrp_recns<8, 1, 2, 3>, 8, false, device);
      case 3016: return slots_of(k_mttkrp_recns<8, 2, 2, 3>, 8, false, device);
      case 3032: return slots_of(k_mttkrp_recns<16, 2, 2, 3>, 16, false, device);
      case 3064: return slots_of(k_mttkrp_recns<16, 4, 2, 3>, 16, false, device);
      case 3128: return slots_of(k_mttkrp_recns<32, 4, 1, 3>, 32, false, device);
      case 4008: return slots_of(k_mttkrp_recns<8, 1, 2, 4>, 8, false, device);
      case 4016: return slots_of(k_mttkrp_recns<8, 2, 2, 4>, 8, false, device);
      case 4032: return slots_of(k_mttkrp_recns<16, 2, 2, 4>, 16, false, device);
      case 4064: return slots_of(k_mttkrp_recns<16, 4, 2, 4>, 16, false, device);
      default: return slots_of(k_mttkrp_recns<32, 4, 1, 4>, 32, false, device);
    }
  }
  if (rec) {
    switch (R) {
      case 8: return slots_of(k_mttkrp_rec3s<8, 1, 4, 1, false>, 8, true, device);
      case 16: return slots_of(k_mttkrp_rec3s<8, 2, 2, 4, false>, 8, true, device);
      case 32: return slots_of(k_mttkrp_rec3s<16, 2, 2, 4, false>, 16, true, device);
      case 64: return slots_of(k_mttkrp_rec3s<16, 4, 2, 1, true>, 16, false, device);
      case 128: return slots_of(k_mttkrp_rec3s<32, 4, 1, 1, true>, 32, false, device);
      default: break;
    }
    if (R <= 32) return slots_of(k_mttkrp_rec3<32, 1, false, 4>, 32, false, device);
    if (R <= 64) return slots_of(k_mttkrp_rec3<32, 2, false, 2>, 32, false, device);
    return slots_of(k_mttkrp_rec3<32, 4, false, 2>, 32, false, device);
  }
  switch (R) {
    case 8: return slots_of(k_mttkrp_view<8, 1, true, 4>, 8, false, device);
    case 16: return slots_of(k_mttkrp_view<16, 1, true, 8>, 16, false, device);
    case 32: return slots_of(k_mttkrp_view<32, 1, true, 8>, 32, false, device);
    case 64: return slots_of(k_mttkrp_view<32, 2, true, 4>, 32, false, device);
    case 128: return slots_of(k_mttkrp_view<32, 4, true, 2>, 32, false, device);
    default: break;
  }
  if (R <= 32) return slots_of(k_mttkrp_view<32, 1, false, 8>, 32, false, device);
  if (R <= 64) return slots_of(k_mttkrp_view<32, 2, false, 4>, 32, false, device);
  return slots_of(k_mttkrp_view<32, 4, false, 2>, 32, false, device);
}

void launch_mttkrp_view(const MttkrpArgs& a, cudaStream_t s) {
  if (a.nnz == 0 || a.ntasks <= a.task0) return;
  if (a.rec != nullptr && a.recw == 2) {
    switch (a.nout) {
      case 2: launch_recns_r<2>(a, s); return;
      case 3: launch_recns_r<3>(a, s); return;
      case 4: launch_recns_r<4>(a, s); return;
      default: throw CptcError(CPTC_E_UNSUP, "32-byte records hold 2 to 4 outer modes");
    }
  }
  if (a.rec != nullptr) {
    // Record kernel per rank, measured on config 4 (B200, ms per mode of the
    // FP64 residual): staging the record stream through shared memory with
    // cp.async beats register prefetch at every rank (R=16 0.70 -> 0.58,
    // R=32 1.10 -> 0.95, R=64 2.27 -> 1.82 with fiber reuse, R=128
    // 3.75 -> 3.49 with fiber reuse); fiber reuse costs registers and loses
    // at R <= 32, where the kernel is latency-bound.
    switch (a.R) {
      case 8: launch_rec3s<8, 1, 4, 1>(a, s); return;
      case 16: launch_rec3s<8, 2, 2, 4>(a, s); return;
      case 32: launch_rec3s<16, 2, 2, 4>(a, s); return;
      case 64: launch_rec3s<16, 4, 2, 1, true>(a, s); return;
      case 128: launch_rec3s<32, 4, 1, 1, true>(a, s); return;
      default: break;
    }
    if (a.R <= 32) launch_rec3<32, 1, false, 4>(a, s);
    else if (a.R <= 64) launch_rec3<32, 2, false, 2>(a, s);
    else if (a.R <= 128) launch_rec3<32, 4, false, 2>(a, s);
    else throw CptcError(CPTC_E_UNSUP, "rank > 128 is not supported");
    return;
  }
  switch (a.R) {
    case 8: launch<8, 1, true, 4>(a, s); return;
    case 16: launch<16, 1, true, 8>(a, s); return;
    case 32: launch<32, 1, true, 8>(a, s); return;
    case 64: launch<32, 2, true, 4>(a, s); return;
    case 128: launch<32, 4, true, 2>(a, s); return;
    default: break;
  }
  if (a.R <= 32) launch<32, 1, false, 8>(a, s);
  else if (a.R <= 64) launch<32, 2, false, 4>(a, s);
  else if (a.R <= 128) launch<32, 4, false, 2>(a, s);
  else throw CptcError(CPTC_E_UNSUP, "rank > 128 is not supported");
}

}  // namespace cptc
