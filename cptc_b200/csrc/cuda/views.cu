// GPU construction of the per-mode MTTKRP views.
//
// Replaces build_mttkrp_views (reference src/partition.cu:1865-2329) and the
// N-order host counting sort (src/generic.cu:1842-1958).  Differences by
// design: coordinates are not packed into 15-bit fields (any dims < 2^30 for
// the gathered mode, < 2^32 otherwise); the sort key is a stable LSD radix
// sort over as many 64-bit passes as the index widths need; rows are not cut
// into fixed segments on the host — the kernel walks nonzero-balanced tasks
// and finds row boundaries from per-element flags.
#include <cub/cub.cuh>

#include <algorithm>
#include <numeric>

#include "engine.hpp"
#include "kernels.hpp"

namespace cptc {

namespace {

struct KeyGroup {
  int ncomp = 0;
  int mode[CPTC_MAX_ORDER];
  int shift[CPTC_MAX_ORDER];
  int bits = 0;
};

struct IdxPtrs {
  const uint32_t* p[CPTC_MAX_ORDER];
};

__global__ void k_iota_sel(const uint32_t* __restrict__ sel, uint64_t n, uint32_t* __restrict__ out) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    out[i] = sel ? sel[i] : (uint32_t)i;
}

__global__ void k_group_keys(IdxPtrs idx, KeyGroup g, const uint32_t* __restrict__ perm,
                             uint64_t n, uint64_t* __restrict__ key) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t e = perm[i];
    uint64_t k = 0;
    for (int c = 0; c < g.ncomp; ++c) k |= (uint64_t)idx.p[g.mode[c]][e] << g.shift[c];
    key[i] = k;
  }
}

// Gathers the sorted element data and marks row / fiber starts.
__global__ void k_gather_view(IdxPtrs idx, const double* __restrict__ vals,
                              const uint32_t* __restrict__ perm, uint64_t n, int target,
                              int nout, IdxPtrs omode_src, int gmode_unused,
                              const uint32_t* __restrict__ gsrc, uint32_t* __restrict__ gw,
                              uint32_t* __restrict__ oidx, double* __restrict__ val,
                              uint8_t* __restrict__ rowflag, unsigned long long* __restrict__ nfib) {
  unsigned long long fibs = 0;
  for (uint64_t p = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; p < n;
       p += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t e = perm[p];
    const uint32_t t = idx.p[target][e];
    bool row = (p == 0);
    bool fib = row;
    if (p > 0) {
      const uint32_t ep = perm[p - 1];
      row = idx.p[target][ep] != t;
      fib = row;
      for (int q = 0; q < nout && !fib; ++q) fib = omode_src.p[q][ep] != omode_src.p[q][e];
    }
    for (int q = 0; q < nout; ++q) oidx[(uint64_t)q * n + p] = omode_src.p[q][e];
    gw[p] = gsrc[e] | (row ? kRowFlag : 0u) | (fib ? kFibFlag : 0u);
    val[p] = vals[e];
    rowflag[p] = row ? 1 : 0;
    fibs += fib ? 1 : 0;
  }
  for (int o = 16; o > 0; o >>= 1) fibs += __shfl_down_sync(0xffffffffu, fibs, o);
  if ((threadIdx.x & 31) == 0 && fibs) atomicAdd(nfib, fibs);
}

// Orders 4-6: two uint4 per nonzero, {word, o0, o1, o2} {o3, 0, value}.
__global__ void k_pack_records2(const uint32_t* __restrict__ gw, const uint32_t* __restrict__ oidx,
                                const double* __restrict__ val, uint64_t n, int nout,
                                uint4* __restrict__ rec) {
  for (uint64_t p = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; p < n;
       p += (uint64_t)gridDim.x * blockDim.x) {
    uint32_t o[4] = {0u, 0u, 0u, 0u};
    for (int q = 0; q < nout; ++q) o[q] = oidx[(uint64_t)q * n + p];
    const unsigned long long vb = __double_as_longlong(val[p]);
    rec[2 * p] = make_uint4(gw[p], o[0], o[1], o[2]);
    rec[2 * p + 1] = make_uint4(o[3], 0u, (uint32_t)vb, (uint32_t)(vb >> 32));
  }
}

__global__ void k_pack_records(const uint32_t* __restrict__ gw, const uint32_t* __restrict__ oidx,
                               const double* __restrict__ val, uint64_t n, uint4* __restrict__ rec) {
  for (uint64_t p = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; p < n;
       p += (uint64_t)gridDim.x * blockDim.x) {
    const unsigned long long vb = __double_as_longlong(val[p]);
    rec[p] = make_uint4(gw[p], oidx[p], (uint32_t)vb, (uint32_t)(vb >> 32));
  }
}

__global__ void k_rows_from_pos(const uint32_t* __restrict__ pos, uint64_t nrows,
                                const uint32_t* __restrict__ tsrc, const uint32_t* __restrict__ perm,
                                uint32_t* __restrict__ rows) {
  for (uint64_t k = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; k < nrows;
       k += (uint64_t)gridDim.x * blockDim.x)
    rows[k] = tsrc[perm[pos[k]]];
}

// task_row[k] = index of the last row start at or before element k*task.
__global__ void k_task_rows(const uint32_t* __restrict__ pos, uint64_t nrows, uint64_t ntasks,
                            uint32_t task, uint32_t* __restrict__ task_row) {
  for (uint64_t k = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; k < ntasks;
       k += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t e0 = k * (uint64_t)task;
    uint64_t lo = 0, hi = nrows;  // first pos > e0
    while (lo < hi) {
      const uint64_t mid = (lo + hi) >> 1;
      if ((uint64_t)pos[mid] <= e0) lo = mid + 1;
      else hi = mid;
    }
    task_row[k] = (uint32_t)(lo - 1);
  }
}

}  // namespace

// Builds `v` for target mode n with the other modes ordered as `order`
// (outer modes first, gathered mode last) over the selected elements.
void build_view_order(Engine& E, View& v, int n, const int* order, int nother,
                      const uint32_t* d_sel, uint64_t nsel) {
  cudaStream_t s = E.stream;
  v = View{};
  v.target = n;
  v.nout = nother - 1;
  for (int q = 0; q < nother; ++q) v.omode[q] = order[q];
  v.gmode = order[nother - 1];
  v.nnz = nsel;
  CPTC_REQUIRE(E.dims[v.gmode] <= kMaxGatherDim, CPTC_E_UNSUP,
               "mode length >= 2^30 is not supported for the gathered mode");
  if (nsel == 0) {
    v.gw.alloc(1);
    v.val.alloc(1);
    v.oidx.alloc(1);
    v.rows.alloc(1);
    v.task_row.alloc(1);
    return;
  }
  CPTC_REQUIRE(nsel < (1ull << 32), CPTC_E_UNSUP, "more than 2^32-1 nonzeros per view");

  IdxPtrs ip{};
  for (int m = 0; m < E.N; ++m) ip.p[m] = E.idx[m].p;

  // Key components from most to least significant: target, order[0..].
  std::vector<int> comp;
  comp.push_back(n);
  for (int q = 0; q < nother; ++q) comp.push_back(order[q]);
  // Group from the least significant end into <= 64-bit keys.
  std::vector<KeyGroup> groups;
  {
    KeyGroup g{};
    for (int c = (int)comp.size() - 1; c >= 0; --c) {
      const int b = bits_for(E.dims[comp[c]]);
      if (g.bits + b > 64) {
        groups.push_back(g);
        g = KeyGroup{};
      }
      g.mode[g.ncomp] = comp[c];
      g.shift[g.ncomp] = g.bits;
      g.bits += b;
      ++g.ncomp;
    }
    groups.push_back(g);
  }

  DArray<uint32_t> perm_a(nsel), perm_b(nsel);
  DArray<uint64_t> key_a(nsel), key_b(nsel);
  const unsigned gb = grid_for(nsel, 256, 148 * 16);
  k_iota_sel<<<gb, 256, 0, s>>>(d_sel, nsel, perm_a.p);
  CPTC_LAUNCH_CHECK();
  size_t temp_bytes = 0;
  CPTC_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, temp_bytes, key_a.p, key_b.p, perm_a.p,
                                            perm_b.p, (int64_t)nsel, 0, 64, s));
  DArray<unsigned char> temp(temp_bytes);
  for (const KeyGroup& g : groups) {
    k_group_keys<<<gb, 256, 0, s>>>(ip, g, perm_a.p, nsel, key_a.p);
    CPTC_LAUNCH_CHECK();
    size_t tb = temp_bytes;
    CPTC_CUDA(cub::DeviceRadixSort::SortPairs(temp.p, tb, key_a.p, key_b.p, perm_a.p, perm_b.p,
                                              (int64_t)nsel, 0, g.bits, s));
    std::swap(perm_a, perm_b);
  }
  key_b.release();

  v.gw.alloc(nsel);
  v.val.alloc(nsel);
  v.oidx.alloc(std::max<uint64_t>(1, (uint64_t)v.nout * nsel));
  DArray<uint8_t> rowflag(nsel);
  DArray<unsigned long long> nfib(1);
  CPTC_CUDA(cudaMemsetAsync(nfib.p, 0, sizeof(unsigned long long), s));
  IdxPtrs osrc{};
  for (int q = 0; q < v.nout; ++q) osrc.p[q] = E.idx[order[q]].p;
  k_gather_view<<<gb, 256, 0, s>>>(ip, E.vals.p, perm_a.p, nsel, n, v.nout, osrc, v.gmode,
                                   E.idx[v.gmode].p, v.gw.p, v.oidx.p, v.val.p, rowflag.p,
                                   nfib.p);
  CPTC_LAUNCH_CHECK();

  // Row starts -> compact positions -> row ids and task rows.
  DArray<uint32_t> pos(nsel);
  DArray<unsigned long long> npos(1);
  size_t sel_bytes = 0;
  cub::CountingInputIterator<uint32_t> cnt(0);
  CPTC_CUDA(cub::DeviceSelect::Flagged(nullptr, sel_bytes, cnt, rowflag.p, pos.p, npos.p,
                                       (int64_t)nsel, s));
  if (sel_bytes > temp.bytes()) temp.alloc(sel_bytes);
  CPTC_CUDA(cub::DeviceSelect::Flagged(temp.p, sel_bytes, cnt, rowflag.p, pos.p, npos.p,
                                       (int64_t)nsel, s));
  unsigned long long h_npos = 0, h_nfib = 0;
  CPTC_CUDA(cudaMemcpyAsync(&h_npos, npos.p, sizeof(h_npos), cudaMemcpyDeviceToHost, s));
  CPTC_CUDA(cudaMemcpyAsync(&h_nfib, nfib.p, sizeof(h_nfib), cudaMemcpyDeviceToHost, s));
  CPTC_CUDA(cudaStreamSynchronize(s));
  v.nrows = h_npos;
  v.fibers = h_nfib;
  v.rows.alloc(v.nrows);
  k_rows_from_pos<<<grid_for(v.nrows, 256, 148 * 16), 256, 0, s>>>(pos.p, v.nrows, E.idx[n].p,
                                                                    perm_a.p, v.rows.p);
  CPTC_LAUNCH_CHECK();
  // Tasks in whole waves of the kernel's resident lane groups.
  const bool recs = (v.nout == 1) ||
                    (v.nout >= 2 && v.nout <= 4 &&
                     (E.R == 8 || E.R == 16 || E.R == 32 || E.R == 64 || E.R == 128));
  v.task = task_size_for(nsel, mttkrp_view_slots(recs, v.nout == 1 ? 1 : 2, v.nout, E.R,
                                                 E.device));
  v.ntasks = (nsel + v.task - 1) / v.task;
  v.task_row.alloc(v.ntasks);
  k_task_rows<<<grid_for(v.ntasks, 256, 148 * 16), 256, 0, s>>>(pos.p, v.nrows, v.ntasks,
                                                                 v.task, v.task_row.p);
  CPTC_LAUNCH_CHECK();
  if (v.nout == 1) {
    // Order 3: one 16-byte record per nonzero for the MTTKRP stream; the
    // separate arrays are released (only the row-start flags are read
    // elsewhere, from the records).
    v.rec.alloc(nsel);
    k_pack_records<<<gb, 256, 0, s>>>(v.gw.p, v.oidx.p, v.val.p, nsel, v.rec.p);
    CPTC_LAUNCH_CHECK();
    CPTC_CUDA(cudaStreamSynchronize(s));
    v.oidx.release();
    v.val.release();
    v.gw.release();
    v.recw = 1;
  } else if (v.nout >= 2 && v.nout <= 4 &&
             (E.R == 8 || E.R == 16 || E.R == 32 || E.R == 64 || E.R == 128)) {
    // Orders 4-6 at the ranks the staged record kernel is built for: two
    // uint4 per nonzero (32 bytes), the separate arrays released.
    v.rec.alloc(2 * nsel);
    k_pack_records2<<<gb, 256, 0, s>>>(v.gw.p, v.oidx.p, v.val.p, nsel, v.nout, v.rec.p);
    CPTC_LAUNCH_CHECK();
    CPTC_CUDA(cudaStreamSynchronize(s));
    v.oidx.release();
    v.val.release();
    v.gw.release();
    v.recw = 2;
  }
  CPTC_CUDA(cudaStreamSynchronize(s));
}

// Chooses the order of the other modes for target n and builds the view.
// Order 3: both orders are built and the one with fewer fibers is kept.
// Order > 3: outer modes by ascending length, the longest mode gathered.
void build_view(Engine& E, View& v, int n, const uint32_t* d_sel, uint64_t nsel) {
  std::vector<int> others;
  for (int m = 0; m < E.N; ++m)
    if (m != n) others.push_back(m);
  if (others.size() == 1) {
    build_view_order(E, v, n, others.data(), 1, d_sel, nsel);
    return;
  }
  if (others.size() == 2) {
    int a[2] = {others[0], others[1]}, b[2] = {others[1], others[0]};
    const bool a_ok = E.dims[a[1]] <= kMaxGatherDim, b_ok = E.dims[b[1]] <= kMaxGatherDim;
    if (!b_ok) {
      build_view_order(E, v, n, a, 2, d_sel, nsel);
      return;
    }
    if (!a_ok) {
      build_view_order(E, v, n, b, 2, d_sel, nsel);
      return;
    }
    View va, vb;
    build_view_order(E, va, n, a, 2, d_sel, nsel);
    build_view_order(E, vb, n, b, 2, d_sel, nsel);
    v = (vb.fibers < va.fibers) ? std::move(vb) : std::move(va);
    return;
  }
  std::stable_sort(others.begin(), others.end(),
                   [&](int x, int y) { return E.dims[x] < E.dims[y]; });
  build_view_order(E, v, n, others.data(), (int)others.size(), d_sel, nsel);
}

}  // namespace cptc
