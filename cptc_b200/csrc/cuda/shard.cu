// Row-slab sharding of the MTTKRP over G ranks (one process per GPU).
//
// Rows of every mode are owned in contiguous slabs of 16-row blocks, cut so
// that the ranks' estimated MTTKRP costs are equal, and each rank stores only
// the nonzeros (residual records and dense tiles) whose target row it owns.
// A slab can only be cut between blocks, so blocks above an eighth of a
// rank's share would unbalance it (a Zipf head row holds ~15% of a mode,
// config 4's first block ~45%); the relabelling puts them first, so the
// prefix of blocks that ends with the last such block is "heavy": its
// residual nonzeros are dealt to the ranks by a hash of their fiber, its
// tiles in turn, and its rows' partial MTTKRPs are summed by
// an all-reduce of the heavy prefix (at most kMaxHeavyRows rows), which every
// rank then solves itself.  The estimate (residual nonzeros and rows, tile
// nonzeros and tiles, with fixed relative costs) misses how locality varies
// along a mode: the residual nonzeros of the light tail rows, whose fibers
// are short, cost more each than those of the head rows.  So the engine
// builds twice: each rank times its own MTTKRP of every mode after the first
// pass (shard_calibrate), and the second pass weighs every block by the time
// per unit of estimated cost measured on the rank that held it.
//
// Reference: cpTC runs on one GPU (src/common.cu:43-46); this is the
// partition the north star asks for (row slabs, nonzeros sharded to match,
// factor all-gather + Gram all-reduce), with the heavy-row split proposed
// for Zipf heads.
#include <cub/cub.cuh>

#include <algorithm>
#include <vector>

#include "comm.hpp"
#include "kernels.hpp"

namespace cptc {

namespace {

// Rows of the heavy prefix are all-reduced every mode update: bounded so
// that the all-reduce stays small (4096 rows = 1 MB at R = 32).
constexpr uint64_t kMaxHeavyRows = 4096;

__global__ void k_block_hist(const uint32_t* __restrict__ idx, const uint32_t* __restrict__ sel,
                             uint64_t n, unsigned long long* __restrict__ cnt) {
  for (uint64_t k = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; k < n;
       k += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t e = sel ? sel[k] : (uint32_t)k;
    atomicAdd(cnt + (idx[e] >> 4), 1ull);
  }
}

// Nonzeros per target row (residual elements).
__global__ void k_row_hist(const uint32_t* __restrict__ idx, const uint32_t* __restrict__ sel,
                           uint64_t n, uint32_t* __restrict__ cnt) {
  for (uint64_t k = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; k < n;
       k += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t e = sel ? sel[k] : (uint32_t)k;
    atomicAdd(cnt + idx[e], 1u);
  }
}

// Non-empty rows per 16-row block.
__global__ void k_block_rows(const uint32_t* __restrict__ cnt, uint64_t dim,
                             unsigned long long* __restrict__ rows) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < dim;
       i += (uint64_t)gridDim.x * blockDim.x)
    if (cnt[i]) atomicAdd(rows + (i >> 4), 1ull);
}

__global__ void k_tile_hist(const int4* __restrict__ tile, uint64_t n, int slot,
                            unsigned long long* __restrict__ nz, unsigned long long* __restrict__ nt) {
  for (uint64_t k = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; k < n;
       k += (uint64_t)gridDim.x * blockDim.x) {
    const int4 T = tile[k];
    const int b = slot == 0 ? T.x : slot == 1 ? T.y : T.z;
    atomicAdd(nz + b, (unsigned long long)T.w);
    atomicAdd(nt + b, 1ull);
  }
}

// Index arrays of the modes that, with the target, key a fiber of the
// target's view (the modes other than the gathered one).
struct FiberModes {
  const uint32_t* p[CPTC_MAX_ORDER];
  int n;
};

__device__ __forceinline__ uint32_t mix32(uint32_t h) {
  h ^= h >> 16;
  h *= 0x7feb352du;
  h ^= h >> 15;
  h *= 0x846ca68bu;
  h ^= h >> 16;
  return h;
}

// Elements of this rank: heavy ones by a hash of their fiber (target index
// and the view's outer indices) modulo G, so that a fiber's nonzeros, which
// share the outer factor rows, stay on one rank; the others by owned block
// range [blo, bhi).
__global__ void k_mine_flag(const uint32_t* __restrict__ idx, const uint32_t* __restrict__ sel,
                            uint64_t n, FiberModes fm, uint32_t hblocks, uint32_t blo,
                            uint32_t bhi, int G, int rank, uint8_t* __restrict__ mine) {
  for (uint64_t k = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; k < n;
       k += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t e = sel ? sel[k] : (uint32_t)k;
    const uint32_t t = idx[e];
    const uint32_t b = t >> 4;
    if (b < hblocks) {
      uint32_t h = mix32(t + 0x9e3779b9u);
      for (int q = 0; q < fm.n; ++q) h = mix32(h ^ (fm.p[q][e] + 0x9e3779b9u));
      mine[k] = (int)(h % (uint32_t)G) == rank ? 1 : 0;
    } else {
      mine[k] = (b >= blo && b < bhi) ? 1 : 0;
    }
  }
}

// Same for tiles in visiting order: tile block of `slot`.
__global__ void k_tile_heavy_flag(const int4* __restrict__ tile, const uint32_t* __restrict__ order,
                                  uint64_t n, int slot, uint32_t hblocks, uint32_t* __restrict__ hf) {
  for (uint64_t k = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; k < n;
       k += (uint64_t)gridDim.x * blockDim.x) {
    const int4 T = tile[order[k]];
    const uint32_t b = (uint32_t)(slot == 0 ? T.x : slot == 1 ? T.y : T.z);
    hf[k] = b < hblocks ? 1u : 0u;
  }
}

__global__ void k_tile_mine_flag(const int4* __restrict__ tile, const uint32_t* __restrict__ order,
                                 uint64_t n, int slot, const uint32_t* __restrict__ hord,
                                 uint32_t hblocks, uint32_t blo, uint32_t bhi, int G, int rank,
                                 uint8_t* __restrict__ mine) {
  for (uint64_t k = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; k < n;
       k += (uint64_t)gridDim.x * blockDim.x) {
    const int4 T = tile[order[k]];
    const uint32_t b = (uint32_t)(slot == 0 ? T.x : slot == 1 ? T.y : T.z);
    mine[k] = b < hblocks ? ((int)(hord[k] % (uint32_t)G) == rank ? 1 : 0)
                          : (b >= blo && b < bhi ? 1 : 0);
  }
}

template <class In>
uint64_t select_flagged(In in, const uint8_t* flags, uint64_t n, uint32_t* out, cudaStream_t s) {
  DArray<unsigned long long> cnt(1);
  size_t tb = 0;
  CPTC_CUDA(cub::DeviceSelect::Flagged(nullptr, tb, in, flags, out, cnt.p, (int64_t)n, s));
  DArray<unsigned char> temp(tb);
  CPTC_CUDA(cub::DeviceSelect::Flagged(temp.p, tb, in, flags, out, cnt.p, (int64_t)n, s));
  unsigned long long h = 0;
  CPTC_CUDA(cudaMemcpyAsync(&h, cnt.p, sizeof(h), cudaMemcpyDeviceToHost, s));
  CPTC_CUDA(cudaStreamSynchronize(s));
  return h;
}

void exclusive_scan_u32(const uint32_t* in, uint32_t* out, uint64_t n, cudaStream_t s) {
  size_t tb = 0;
  CPTC_CUDA(cub::DeviceScan::ExclusiveSum(nullptr, tb, in, out, (int64_t)n, s));
  DArray<unsigned char> temp(tb);
  CPTC_CUDA(cub::DeviceScan::ExclusiveSum(temp.p, tb, in, out, (int64_t)n, s));
}

}  // namespace

// Cost of one tile-kernel unit (a dense nonzero, or 1/tile3w_fixed_cost of
// a tile's fixed part) in residual-nonzero units.  Measured on config 4 (one
// B200, ms per mode): R=32 tiles 0.45 ms for 39.1M nonzeros in 81,886 tiles
// against the residual's 0.95 ms for 37.8M nonzeros gives 0.10; R=128
// (1.42 against 3.16 ms) 0.029; about 3.2 / R.
static double tile_cost_ratio(int R) { return std::min(0.5, 3.2 / (double)R); }

// Cost of one non-empty target row of the residual view (the row's write,
// its row-index load and the task boundary work) in residual-nonzero units.
static double row_cost(int R) { return 0.0 * R; }

void shard_plan(Engine& E, const uint32_t* sel, uint64_t nsel) {
  const int G = E.nranks;
  cudaStream_t s = E.stream;
  for (int n = 0; n < E.N; ++n) {
    E.slab[n].assign(G + 1, 0);
    E.heavy_rows[n] = 0;
    const uint64_t nb = (E.dims[n] + 15) / 16;
    // Residual elements of this target mode: the selection when the dense
    // tiles cover the mode, every nonzero otherwise.
    int ts = -1;
    if (E.dense_active)
      for (int q = 0; q < 3; ++q)
        if (E.units.inner[q] == n && E.units.nunits > 0) ts = q;
    const uint32_t* msel = ts >= 0 ? sel : nullptr;
    const uint64_t mn = ts >= 0 ? nsel : E.nnz;
    DArray<unsigned long long> rc(nb), dz(nb), dt(nb), rr(nb);
    DArray<uint32_t> rowc(E.dims[n]);
    CPTC_CUDA(cudaMemsetAsync(rc.p, 0, nb * 8, s));
    CPTC_CUDA(cudaMemsetAsync(dz.p, 0, nb * 8, s));
    CPTC_CUDA(cudaMemsetAsync(dt.p, 0, nb * 8, s));
    CPTC_CUDA(cudaMemsetAsync(rr.p, 0, nb * 8, s));
    CPTC_CUDA(cudaMemsetAsync(rowc.p, 0, E.dims[n] * 4, s));
    if (mn) {
      k_block_hist<<<grid_for(mn, 256, 148 * 16), 256, 0, s>>>(E.idx[n].p, msel, mn, rc.p);
      CPTC_LAUNCH_CHECK();
      k_row_hist<<<grid_for(mn, 256, 148 * 16), 256, 0, s>>>(E.idx[n].p, msel, mn, rowc.p);
      CPTC_LAUNCH_CHECK();
      k_block_rows<<<grid_for(E.dims[n], 256, 148 * 8), 256, 0, s>>>(rowc.p, E.dims[n], rr.p);
      CPTC_LAUNCH_CHECK();
    }
    if (ts >= 0) {
      k_tile_hist<<<grid_for(E.units.nunits, 256, 148 * 16), 256, 0, s>>>(
          E.units.unit.p, E.units.nunits, ts, dz.p, dt.p);
      CPTC_LAUNCH_CHECK();
    }
    std::vector<unsigned long long> hrc(nb), hdz(nb), hdt(nb), hrr(nb);
    CPTC_CUDA(cudaMemcpyAsync(hrc.data(), rc.p, nb * 8, cudaMemcpyDeviceToHost, s));
    CPTC_CUDA(cudaMemcpyAsync(hrr.data(), rr.p, nb * 8, cudaMemcpyDeviceToHost, s));
    CPTC_CUDA(cudaMemcpyAsync(hdz.data(), dz.p, nb * 8, cudaMemcpyDeviceToHost, s));
    CPTC_CUDA(cudaMemcpyAsync(hdt.data(), dt.p, nb * 8, cudaMemcpyDeviceToHost, s));
    CPTC_CUDA(cudaStreamSynchronize(s));
    const double rho = tile_cost_ratio(E.R);
    const double fixed = E.generic ? 512.0 : (double)tile3w_fixed_cost(E.R);
    const double crow = row_cost(E.R);
    std::vector<double> w(nb);
    double W = 0.0;
    for (uint64_t b = 0; b < nb; ++b) {
      w[b] = (double)hrc[b] + crow * (double)hrr[b] +
             rho * ((double)hdz[b] + fixed * (double)hdt[b]);
      W += w[b];
    }
    // Heavy prefix: up to the last block above an eighth of a rank's share.
    uint64_t h = 0;
    for (uint64_t b = 0; b < nb; ++b)
      if (w[b] > W / (8.0 * G)) h = b + 1;
    h = std::min<uint64_t>(h, kMaxHeavyRows / 16);
    double Wh = 0.0;
    for (uint64_t b = 0; b < h; ++b) Wh += w[b];
    // Second pass: the blocks each rank held in the first pass weigh its
    // measured time per unit of estimated cost (mean 1).
    std::vector<double> raw = w;
    const auto& sp = E.shard_speed[n];
    const auto& pb = E.prev_blocks[n];
    if ((int)sp.size() == G && (int)pb.size() == G + 1) {
      for (int r = 0; r < G; ++r)
        for (uint64_t b = std::max<uint64_t>(pb[r], h); b < std::min<uint64_t>(pb[r + 1], nb); ++b)
          w[b] *= sp[r];
    }
    double Wn = 0.0;
    for (uint64_t b = h; b < nb; ++b) Wn += w[b];
    // Slab cuts over the remaining blocks at equal cost, each at the block
    // boundary nearest to its target.
    std::vector<uint64_t> cb(G + 1, nb);
    cb[0] = h;
    double acc = 0.0;
    uint64_t b = h;
    for (int r = 1; r < G; ++r) {
      const double target = Wn * (double)r / (double)G;
      while (b < nb && acc + 0.5 * w[b] <= target) acc += w[b++];
      cb[r] = b;
    }
    // Estimated (uncorrected) cost of each rank's share: its slab and an
    // equal part of the heavy prefix.
    E.slab_cost[n].assign(G, Wh / G);
    for (int r = 0; r < G; ++r)
      for (uint64_t q = cb[r]; q < cb[r + 1]; ++q) E.slab_cost[n][r] += raw[q];
    E.heavy_rows[n] = std::min<uint64_t>(h * 16, E.dims[n]);
    E.slab[n][0] = 0;
    for (int r = 1; r < G; ++r) E.slab[n][r] = std::min<uint64_t>(cb[r] * 16, E.dims[n]);
    E.slab[n][G] = E.dims[n];
    E.slab_blocks[n] = cb;
  }
}

void shard_calibrate(Engine& E) {
  const int G = E.nranks, N = E.N;
  std::vector<double> t(N, 0.0), all((size_t)G * N, 0.0);
  cudaEvent_t e0 = E.ev[0], e1 = E.ev[1];
  constexpr int kReps = 3;
  for (int n = 0; n < N; ++n) {
    E.mttkrp(n);  // warm-up
    CPTC_CUDA(cudaEventRecord(e0, E.stream));
    for (int r = 0; r < kReps; ++r) E.mttkrp(n);
    CPTC_CUDA(cudaEventRecord(e1, E.stream));
    CPTC_CUDA(cudaEventSynchronize(e1));
    float ms = 0.f;
    CPTC_CUDA(cudaEventElapsedTime(&ms, e0, e1));
    t[n] = ms / kReps;
  }
  comm_allgather_host(E, t.data(), N, all.data());
  for (int n = 0; n < N; ++n) {
    const auto& est = E.slab_cost[n];
    std::vector<double> k(G, 1.0);
    double mean = 0.0;
    bool ok = (int)est.size() == G;
    for (int r = 0; ok && r < G; ++r) {
      const double tr = all[(size_t)r * N + n];
      ok = est[r] > 0.0 && tr > 0.0;
      if (ok) k[r] = tr / est[r];
      mean += k[r];
    }
    if (!ok) {
      E.shard_speed[n].clear();
      E.prev_blocks[n].clear();
      continue;
    }
    mean /= G;
    for (auto& x : k) x /= mean;
    E.shard_speed[n] = k;
    E.prev_blocks[n] = E.slab_blocks[n];
  }
}

uint64_t shard_select(Engine& E, int n, const uint32_t* sel, uint64_t nsel, DArray<uint32_t>& out) {
  cudaStream_t s = E.stream;
  const uint64_t mn = sel ? nsel : E.nnz;
  out.alloc(mn);
  if (mn == 0) return 0;
  const uint32_t hb = (uint32_t)(E.heavy_rows[n] + 15) / 16;
  // Fibers are keyed by the target and every other mode but the longest:
  // the view's gathered mode for order > 3, and for order 3 usually (that
  // view keeps whichever order has fewer fibers, in practice the one with
  // the shorter outer mode; otherwise fibers are split, which costs only
  // locality).
  std::vector<int> others;
  for (int m = 0; m < E.N; ++m)
    if (m != n) others.push_back(m);
  std::stable_sort(others.begin(), others.end(),
                   [&](int x, int y) { return E.dims[x] < E.dims[y]; });
  FiberModes fm{};
  fm.n = (int)others.size() - 1;
  for (int q = 0; q < fm.n; ++q) fm.p[q] = E.idx[others[q]].p;
  DArray<uint8_t> mine(mn);
  const unsigned gb = grid_for(mn, 256, 148 * 16);
  k_mine_flag<<<gb, 256, 0, s>>>(E.idx[n].p, sel, mn, fm, hb, (uint32_t)E.slab_blocks[n][E.rank],
                                 (uint32_t)E.slab_blocks[n][E.rank + 1], E.nranks, E.rank, mine.p);
  CPTC_LAUNCH_CHECK();
  if (sel) return select_flagged(sel, mine.p, mn, out.p, s);
  return select_flagged(cub::CountingInputIterator<uint32_t>(0), mine.p, mn, out.p, s);
}

uint64_t shard_tiles(Engine& E, int slot, DArray<uint32_t>& local_order) {
  cudaStream_t s = E.stream;
  UnitPool& U = E.units;
  const int n = U.inner[slot];
  const uint64_t cnt = U.nunits;
  local_order.alloc(cnt);
  if (cnt == 0) return 0;
  const uint32_t hb = (uint32_t)(E.heavy_rows[n] + 15) / 16;
  DArray<uint32_t> hf(cnt), hord(cnt);
  DArray<uint8_t> mine(cnt);
  const unsigned gb = grid_for(cnt, 256, 148 * 16);
  k_tile_heavy_flag<<<gb, 256, 0, s>>>(U.unit.p, U.order[slot].p, cnt, slot, hb, hf.p);
  CPTC_LAUNCH_CHECK();
  exclusive_scan_u32(hf.p, hord.p, cnt, s);
  k_tile_mine_flag<<<gb, 256, 0, s>>>(U.unit.p, U.order[slot].p, cnt, slot, hord.p, hb,
                                      (uint32_t)E.slab_blocks[n][E.rank],
                                      (uint32_t)E.slab_blocks[n][E.rank + 1], E.nranks, E.rank,
                                      mine.p);
  CPTC_LAUNCH_CHECK();
  return select_flagged(U.order[slot].p, mine.p, cnt, local_order.p, s);
}

}  // namespace cptc
