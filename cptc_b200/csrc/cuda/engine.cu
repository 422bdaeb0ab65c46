// The CP-ALS engine: load, build (relabel, partition, views, path choice),
// factor initialisation, MTTKRP and the ALS loop, plus the C ABI.
//
// Reference drivers: main (src/main.cu:22-680), execute_als_decomposition
// (src/als.cu:362-821) and run_generic_cp (src/generic.cu:1639-2366).
#include <omp.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <random>
#include <thread>

#include "../host/coo.hpp"
#include "../host/reorder.hpp"
#include "comm.hpp"
#include <cstdlib>
#include "kernels.hpp"

namespace cptc {

std::atomic<unsigned long long> g_launches{0};
thread_local unsigned long long t_launches = 0;

namespace {

__global__ void k_relabel(uint32_t* __restrict__ idx, uint64_t n, const uint32_t* __restrict__ map) {
  for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < n;
       e += (uint64_t)gridDim.x * blockDim.x)
    idx[e] = map[idx[e]];
}

// Row permutation between the caller's labels and the relabelled space,
// on the device.  to_relabelled: out[map[a]] = in[a]; otherwise
// out[a] = in[map[a]] (map[old] = new).  One thread per (row, column pair).
__global__ void k_permute_rows(const double* __restrict__ in, const uint32_t* __restrict__ map,
                               uint64_t rows, int R, int to_relabelled, double* __restrict__ out) {
  const int h = R >> 1;  // R is even for every vector-width path; odd R uses h = 0
  if (h > 0 && (R & 1) == 0) {
    const uint64_t n = rows * (uint64_t)h;
    for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < n;
         e += (uint64_t)gridDim.x * blockDim.x) {
      const uint64_t a = e / h, c = e - a * h;
      const uint64_t b = map[a];
      const uint64_t src = to_relabelled ? a : b, dst = to_relabelled ? b : a;
      reinterpret_cast<double2*>(out)[dst * h + c] =
          reinterpret_cast<const double2*>(in)[src * h + c];
    }
  } else {
    const uint64_t n = rows * (uint64_t)R;
    for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < n;
         e += (uint64_t)gridDim.x * blockDim.x) {
      const uint64_t a = e / R, c = e - a * R;
      const uint64_t b = map[a];
      const uint64_t src = to_relabelled ? a : b, dst = to_relabelled ? b : a;
      out[dst * R + c] = in[src * R + c];
    }
  }
}

}  // namespace

double b200_fill_min(int R) {
  if (R <= 32) return 0.07;
  if (R >= 128) return 0.04;
  return 0.07 - 0.03 * (double)(R - 32) / 96.0;
}

Engine::Engine(int dev) : device(dev) {
  int n = 0;
  CPTC_CUDA(cudaGetDeviceCount(&n));
  CPTC_REQUIRE(dev >= 0 && dev < n, CPTC_E_ARG, "no such CUDA device");
  CPTC_CUDA(cudaSetDevice(dev));
  CPTC_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
  CPTC_CUDA(cudaStreamCreateWithFlags(&side, cudaStreamNonBlocking));
  for (auto& e : ev) CPTC_CUDA(cudaEventCreate(&e));
  for (auto& e : ev1) CPTC_CUDA(cudaEventCreate(&e));
  evc = ev;
  CPTC_CUDA(cudaEventCreateWithFlags(&ev_fork, cudaEventDisableTiming));
  CPTC_CUDA(cudaEventCreateWithFlags(&ev_join, cudaEventDisableTiming));
  CPTC_CUDA(cudaMallocHost((void**)&h_scal, 16 * sizeof(double)));
}

Engine::~Engine() {
  cudaSetDevice(device);
  if (stream) cudaStreamSynchronize(stream);
  if (side) cudaStreamSynchronize(side);
  release_graph();  // before the communicator its NCCL nodes use
  comm_destroy(*this);
  for (auto& e : ev)
    if (e) cudaEventDestroy(e);
  for (auto& e : ev1)
    if (e) cudaEventDestroy(e);
  for (auto& sl : evp)
    for (auto& md : sl)
      for (auto& e : md)
        if (e) cudaEventDestroy(e);
  if (ev_fork) cudaEventDestroy(ev_fork);
  if (ev_join) cudaEventDestroy(ev_join);
  if (h_scal) cudaFreeHost(h_scal);
  if (side) cudaStreamDestroy(side);
  if (stream) cudaStreamDestroy(stream);
}

uint64_t Engine::device_bytes() const {
  uint64_t b = vals.bytes();
  for (int m = 0; m < N; ++m) b += idx[m].bytes() + F[m].bytes() + G[m].bytes();
  for (const View& v : views)
    b += v.gw.bytes() + v.oidx.bytes() + v.val.bytes() + v.rec.bytes() + v.rows.bytes() +
         v.task_row.bytes();
  b += units.unit.bytes() + units.start.bytes() + units.lid.bytes() + units.val.bytes() +
       units.outer_idx.bytes() + units.words.bytes() + units.pstart.bytes();
  for (int m = 0; m < 3; ++m)
    b += units.order[m].bytes() + units.vtile[m].bytes() + units.vstart[m].bytes();
  b += Ftf.bytes();
  b += FtV.bytes() + FtF.bytes() + Ainv.bytes() + gpart.bytes() + dots.bytes() +
       lambda.bytes();
  return b;
}

void Engine::load(const cptc_coo* t) {
  CPTC_REQUIRE(t && t->order >= 2 && t->order <= CPTC_MAX_ORDER, CPTC_E_ARG,
               "tensor order must be in [2, 8]");
  CPTC_REQUIRE(t->nnz < (1ull << 32), CPTC_E_UNSUP, "more than 2^32-1 nonzeros");
  CPTC_CUDA(cudaSetDevice(device));
  release_graph();
  built = false;
  have_factors = false;
  views.clear();
  N = t->order;
  nnz = t->nnz;
  for (int m = 0; m < N; ++m) {
    CPTC_REQUIRE(t->dims[m] >= 1 && t->dims[m] <= 0xFFFFFFFFull, CPTC_E_ARG, "bad mode length");
    dims[m] = t->dims[m];
    CPTC_REQUIRE(t->idx[m] != nullptr || nnz == 0, CPTC_E_ARG, "null index array");
  }
  CPTC_REQUIRE(t->vals != nullptr || nnz == 0, CPTC_E_ARG, "null value array");
  // Host-side bounds check: an index beyond its mode length would make
  // every later kernel read out of bounds.
  for (int m = 0; m < N; ++m) {
    const uint32_t* ix = t->idx[m];
    const uint64_t d = dims[m];
    int bad = 0;
#pragma omp parallel for reduction(| : bad) schedule(static)
    for (int64_t e = 0; e < (int64_t)nnz; ++e) bad |= (ix[e] >= d);
    CPTC_REQUIRE(!bad, CPTC_E_ARG, "index out of range for its mode length");
  }
  for (int m = 0; m < N; ++m) {
    idx[m].alloc(nnz);
    if (nnz) CPTC_CUDA(cudaMemcpyAsync(idx[m].p, t->idx[m], nnz * 4, cudaMemcpyHostToDevice, stream));
  }
  vals.alloc(nnz);
  if (nnz) CPTC_CUDA(cudaMemcpyAsync(vals.p, t->vals, nnz * 8, cudaMemcpyHostToDevice, stream));
  // Host copy of the coordinates for the relabelling (degree sort / HITS).
  host_idx.assign(N, {});
  for (int m = 0; m < N; ++m) host_idx[m].assign(t->idx[m], t->idx[m] + nnz);
  CPTC_CUDA(cudaStreamSynchronize(stream));
}

void Engine::reorder() {
  const auto t0 = std::chrono::steady_clock::now();
  perm.assign(N, {});
  int kind = opts.reorder;
  if (!generic && kind == CPTC_REORDER_DEFAULT) kind = CPTC_REORDER_CADR;
  if (generic && kind == CPTC_REORDER_DEFAULT)
    kind = (N >= 4) ? CPTC_REORDER_HITS : CPTC_REORDER_CADR;
  if (!generic && kind == CPTC_REORDER_CADR) {
    // Order-3 CADR: the reference's unstable std::sort decides the order of
    // equal degrees, so the permutation is made by the same call on the host.
    for (int m = 0; m < N; ++m) cadr_perm_ref(dims[m], nnz, host_idx[m].data(), perm[m]);
  } else if (kind == CPTC_REORDER_HITS) {
    gpu_hits(*this, opts.reorder_rounds, opts.reorder_sample, perm);
  } else if (kind == CPTC_REORDER_CADR) {
    gpu_degree_rank(*this, perm);  // N-order CADR: ties by index
  } else if (kind == CPTC_REORDER_AUTO) {
    // probe of the tile fill before and after HITS (host, sampled)
    std::vector<const uint32_t*> ip(N);
    for (int m = 0; m < N; ++m) ip[m] = host_idx[m].data();
    reorder_generic(N, dims, nnz, ip.data(), kind, opts.reorder_rounds, opts.reorder_sample,
                    perm, &reorder_note);
    perm.resize(N);
  }
  for (int m = 0; m < N; ++m) {
    dperm[m].release();
    if (perm[m].empty()) continue;
    dperm[m].alloc(dims[m]);
    CPTC_CUDA(cudaMemcpyAsync(dperm[m].p, perm[m].data(), dims[m] * 4, cudaMemcpyHostToDevice,
                              stream));
    k_relabel<<<grid_for(nnz, 256, 148 * 16), 256, 0, stream>>>(idx[m].p, nnz, dperm[m].p);
    CPTC_LAUNCH_CHECK();
    CPTC_CUDA(cudaStreamSynchronize(stream));
  }
  reorder_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
}

// Factor-shaped buffers hold nranks equal slabs (padding rows past I_m are
// never read as factor rows); FtV is shared by all modes.
uint64_t Engine::padded_rows(int m) const {
  return nranks > 1 ? slab_rows(*this, m) * (uint64_t)nranks : dims[m];
}

void Engine::alloc_workspace() {
  uint64_t maxd = 0;
  for (int m = 0; m < N; ++m) maxd = std::max<uint64_t>(maxd, padded_rows(m));
  // FtV holds the MTTKRP of a mode; on several ranks its rows past the
  // mode's length also carry the exchange's Gram and dot sums (R + 1 rows).
  FtV.alloc((maxd + R + 1) * (uint64_t)R);
  FtF.alloc((uint64_t)R * R);
  Ainv.alloc(2 * (uint64_t)R * R + 1);
  gpart_blocks = 148;
  gpart.alloc((uint64_t)gpart_blocks * R * R);
  dots.alloc((uint64_t)gpart_blocks * R);
  comm_buf.alloc((uint64_t)R * R + R);
  cscale.alloc(R);
  scal.alloc(8);
  status.alloc(1);
  lambda.alloc(R);
  if (dense_active && !generic) Ftf.alloc(((maxd + 15) / 16) * 16 * (uint64_t)R);
  else Ftf.release();
  for (int m = 0; m < N; ++m) {
    F[m].alloc(padded_rows(m) * (uint64_t)R);
    CPTC_CUDA(cudaMemsetAsync(F[m].p, 0, padded_rows(m) * (uint64_t)R * sizeof(double), stream));
    G[m].alloc((uint64_t)R * R);
  }
}

// With several ranks the slabs are cut twice: the first pass cuts them at
// equal estimated cost, each rank then times its own MTTKRP of every mode,
// and the second pass cuts again with each rank's measured time per unit of
// estimated cost applied to the blocks it held (shard_calibrate).
void Engine::build(int R_, double threshold, const cptc_opts* o) {
  for (int m = 0; m < CPTC_MAX_ORDER; ++m) {
    shard_speed[m].clear();
    prev_blocks[m].clear();
  }
  const auto t0 = std::chrono::steady_clock::now();
  build_pass(R_, threshold, o);
  if (nranks > 1 && nnz > 0) {
    shard_calibrate(*this);
    build_pass(R_, threshold, o);
  }
  build_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
}

void Engine::build_pass(int R_, double threshold, const cptc_opts* o) {
  CPTC_REQUIRE(N >= 2, CPTC_E_ARG, "load a tensor first");
  CPTC_REQUIRE(R_ >= 1 && R_ <= 128, CPTC_E_UNSUP, "rank must be in [1, 128]");
  CPTC_CUDA(cudaSetDevice(device));
  const auto t0 = std::chrono::steady_clock::now();
  if (o) opts = *o;
  else cptc_opts_default(&opts);
  R = R_;
  generic = (N != 3) || opts.generic;
  release_graph();
  CPTC_REQUIRE(opts.exchange == CPTC_EXCHANGE_NCCL || opts.exchange == CPTC_EXCHANGE_PEER,
               CPTC_E_ARG, "unknown exchange");
  CPTC_REQUIRE(opts.exchange == CPTC_EXCHANGE_NCCL || nranks == 1, CPTC_E_UNSUP,
               "the ranks exchange through NCCL (one grouped call per mode update)");
  built = false;
  have_factors = false;
  views.clear();
  units = UnitPool{};
  dense_active = false;
  tf32 = false;
  avg_fill = 0.0;
  cutoff = 0;

  // Relabel from the original coordinates (the permutation depends on the
  // path: CADR for order 3, HITS/CADR with tie-break for the N-order path).
  for (int m = 0; m < N; ++m)
    if (nnz)
      CPTC_CUDA(cudaMemcpyAsync(idx[m].p, host_idx[m].data(), nnz * 4, cudaMemcpyHostToDevice,
                                stream));
  reorder();
  {
    DArray<double> part(148 * 16);
    launch_sumsq(vals.p, nnz, part.p, 148 * 16, scal_tmp(), stream);
    CPTC_CUDA(cudaMemcpyAsync(&x_norm_sq, scal_tmp(), sizeof(double), cudaMemcpyDeviceToHost,
                              stream));
    CPTC_CUDA(cudaStreamSynchronize(stream));
  }

  // Fill-rate selector re-derived on B200 (the reference's rule,
  // max(0.08, 0.11/sqrt(SMs/24)) from src/main.cu:369-381, was calibrated on
  // a 24-SM RTX 4060).  Measured per-tile cost a + b*nnz of the TF32 tile
  // kernel against c*nnz of the FP64 kernel on configs 2-4 gives the
  // break-even fill a / (4096 (c - b)): R=16 a~4.1 ns, b~0.0053, c~0.0195
  // -> 0.068; R=32 a~6, b~0.005, c~0.029 -> 0.061; R=128 a~20, b~0.012,
  // c~0.13 -> 0.041 (ns per tile / per nonzero).
  fill_min = opts.fill_min > 0.0 ? opts.fill_min : b200_fill_min(R);

  DArray<uint32_t> sel;
  uint64_t nsel = nnz;
  if (!generic && opts.path != CPTC_PATH_FP64 && nnz > 0) {
    partition_tiles3(*this, threshold, sel, nsel);
    avg_fill = units.nunits ? (double)units.nnz / ((double)units.nunits * 4096.0) : 0.0;
    if (opts.path == CPTC_PATH_TF32) tf32 = true;
    else tf32 = (avg_fill >= fill_min) && units.nunits > 0 && (R % 8 == 0);
    CPTC_REQUIRE(!tf32 || R % 8 == 0, CPTC_E_UNSUP,
                 "the TF32 tile path needs the rank to be a multiple of 8");
  } else if (generic && N >= 4 && opts.dense_generic && opts.dense_thr_generic > 0.0 &&
             R % 8 == 0 && nnz > 0) {
    // N-order dense units over the inner modes (src/generic.cu:1808-1840).
    partition_units(*this, opts.dense_thr_generic, sel, nsel);
    units.store_dups = false;
    cutoff = (int)(4096.0 * opts.dense_thr_generic);
    avg_fill = units.nunits ? (double)units.nnz / ((double)units.nunits * 4096.0) : 0.0;
    tf32 = units.nunits > 0;
  }
  if (!tf32) {
    units = UnitPool{};
    sel.release();
    nsel = nnz;
  }
  dense_active = tf32;
  views.resize(N);
  comm_prepare(*this);  // transfer slabs; one rank: the whole modes
  // Several ranks: rows of every mode in slabs, each rank keeping only the
  // nonzeros and tiles of its rows and its share of the heavy prefix.
  if (nranks > 1) shard_plan(*this, sel.p, nsel);
  alloc_workspace();
  for (int t = 0; t < 3; ++t) units.cnt[t] = units.nunits;
  if (dense_active && nranks > 1) {
    for (int t = 0; t < 3; ++t) {
      DArray<uint32_t> mine;
      units.cnt[t] = shard_tiles(*this, t, mine);
      units.order[t] = std::move(mine);
    }
  }
  uint64_t most = 0;
  for (int t = 0; t < 3; ++t) most = std::max<uint64_t>(most, units.cnt[t]);
  if (dense_active && !generic) {
    // order 3: the packed word pool (tiles_pool.cu)
    units.blocks = tile3w_blocks_for(R, device, most);
    for (int t = 0; t < 3; ++t) {
      tile_cuts(*this, t, tile3w_fixed_cost(R));
      tile_visit_lists(*this, t);
      if (nranks > 1) compact_slot_pool(*this, t);
    }
    if (nranks > 1) {
      units.words.release();
      units.pstart.release();
    }
  } else if (dense_active) {
    // N-order units: a tile weighs its nonzeros plus 512 (zeroing the tile
    // and the 16 slab products, in nonzero units)
    units.blocks = tile_blocks_for(R, device, most);
    for (int t = 0; t < 3; ++t) tile_cuts(*this, t, 512ull);
  }
  for (int n = 0; n < N; ++n) {
    // Residual-only views for modes the dense tiles cover as a target.
    const bool covered = dense_active &&
                         (n == units.inner[0] || n == units.inner[1] || n == units.inner[2]);
    const uint32_t* base = covered ? sel.p : nullptr;
    const uint64_t nbase = covered ? nsel : nnz;
    if (nranks > 1) {
      DArray<uint32_t> mine;
      const uint64_t nm = shard_select(*this, n, base, nbase, mine);
      build_view(*this, views[n], n, mine.p, nm);
    } else {
      build_view(*this, views[n], n, base, nbase);
    }
    views[n].t0 = 0;
    views[n].t1 = views[n].ntasks;
  }
  CPTC_CUDA(cudaStreamSynchronize(stream));
  build_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
  built = true;
}

double* Engine::scal_tmp() {
  if (!scal.p) scal.alloc(8);
  return scal.p;
}

void Engine::init_factors() {
  CPTC_REQUIRE(built, CPTC_E_ARG, "call cptc_build first");
  if (!generic) {
    // src/common.cu:83-101: mt19937(42), U[0,1), modes in order, row-major,
    // in the relabelled index space.
    std::mt19937 gen(42);
    std::uniform_real_distribution<double> dis(0.0, 1.0);
    for (int m = 0; m < N; ++m) {
      std::vector<double> h(dims[m] * (uint64_t)R);
      for (auto& x : h) x = dis(gen);
      CPTC_CUDA(cudaMemcpyAsync(F[m].p, h.data(), h.size() * 8, cudaMemcpyHostToDevice, stream));
      CPTC_CUDA(cudaStreamSynchronize(stream));
    }
  } else {
    // src/generic.cu:1754-1783: mt19937(seed) in original order, each row
    // carried to its relabelled position.
    std::mt19937 gen(opts.seed);
    std::uniform_real_distribution<double> dis(0.0, 1.0);
    for (int m = 0; m < N; ++m) {
      std::vector<double> u(dims[m] * (uint64_t)R), h(u.size());
      for (auto& x : u) x = dis(gen);
      for (uint64_t a = 0; a < dims[m]; ++a) {
        const uint64_t nw = perm[m].empty() ? a : perm[m][a];
        std::memcpy(h.data() + nw * R, u.data() + a * R, R * sizeof(double));
      }
      CPTC_CUDA(cudaMemcpyAsync(F[m].p, h.data(), h.size() * 8, cudaMemcpyHostToDevice, stream));
      CPTC_CUDA(cudaStreamSynchronize(stream));
    }
  }
  std::vector<double> one(R, 1.0);
  CPTC_CUDA(cudaMemcpyAsync(lambda.p, one.data(), R * 8, cudaMemcpyHostToDevice, stream));
  CPTC_CUDA(cudaStreamSynchronize(stream));
  have_factors = true;
  grams_valid = false;
}

// Host factors in the caller's labels <-> device factors in relabelled rows.
// The rows are permuted on the device (through `stage`), so a transfer is one
// copy at PCIe speed (DMA when the caller's buffer is pinned).
double* Engine::stage_rows() {
  uint64_t maxd = 0;
  for (int m = 0; m < N; ++m) maxd = std::max<uint64_t>(maxd, padded_rows(m));
  if (stage.n < maxd * (uint64_t)R) stage.alloc(maxd * (uint64_t)R);
  return stage.p;
}

void Engine::permute_rows(const double* in, int m, bool to_relabelled, double* out) {
  const uint64_t n = dims[m] * (uint64_t)R;
  k_permute_rows<<<grid_for(n / 2 + 1, 256, 148 * 16), 256, 0, stream>>>(
      in, dperm[m].p, dims[m], R, to_relabelled ? 1 : 0, out);
  CPTC_LAUNCH_CHECK();
}

void Engine::set_factor(int m, const double* host) {
  CPTC_REQUIRE(built && m >= 0 && m < N && host, CPTC_E_ARG, "bad mode or call order");
  const uint64_t bytes = dims[m] * (uint64_t)R * sizeof(double);
  if (dperm[m].p) {
    double* st = stage_rows();
    CPTC_CUDA(cudaMemcpyAsync(st, host, bytes, cudaMemcpyHostToDevice, stream));
    permute_rows(st, m, true, F[m].p);
  } else {
    CPTC_CUDA(cudaMemcpyAsync(F[m].p, host, bytes, cudaMemcpyHostToDevice, stream));
  }
  if (!have_factors) {
    std::vector<double> one(R, 1.0);
    CPTC_CUDA(cudaMemcpyAsync(lambda.p, one.data(), R * 8, cudaMemcpyHostToDevice, stream));
  }
  // The caller may reuse `host` once this returns.
  CPTC_CUDA(cudaStreamSynchronize(stream));
  have_factors = true;
  grams_valid = false;
}

// Collective: rank r copies rows [r*s, (r+1)*s) of `host` (original index
// space, s = ceil(I_m / G)) and the pieces are all-gathered on the device.
void Engine::set_factor_sharded(int m, const double* host) {
  CPTC_REQUIRE(built && m >= 0 && m < N && host, CPTC_E_ARG, "bad mode or call order");
  if (nranks == 1) {
    set_factor(m, host);
    return;
  }
  const uint64_t s = slab_rows(*this, m);
  const uint64_t lo = std::min<uint64_t>(s * (uint64_t)rank, dims[m]);
  const uint64_t hi = std::min<uint64_t>(s * (uint64_t)(rank + 1), dims[m]);
  double* dst = dperm[m].p ? stage_rows() : F[m].p;
  if (hi > lo)
    CPTC_CUDA(cudaMemcpyAsync(dst + lo * R, host + lo * R, (hi - lo) * (uint64_t)R * sizeof(double),
                              cudaMemcpyHostToDevice, stream));
  comm_allgather_rows(*this, m, dst);
  if (dperm[m].p) permute_rows(dst, m, true, F[m].p);
  if (!have_factors) {
    std::vector<double> one(R, 1.0);
    CPTC_CUDA(cudaMemcpyAsync(lambda.p, one.data(), R * 8, cudaMemcpyHostToDevice, stream));
  }
  CPTC_CUDA(cudaStreamSynchronize(stream));
  have_factors = true;
  grams_valid = false;
}

void Engine::get_factor(int m, double* host) {
  CPTC_REQUIRE(built && have_factors && m >= 0 && m < N && host, CPTC_E_ARG,
               "bad mode or call order");
  fetch_rows(F[m].p, m, host);
}

// Local: rows [r*s, (r+1)*s) of the factor (original index space) into the
// same rows of `host`; the other rows of `host` are not written.
void Engine::get_factor_sharded(int m, double* host) {
  CPTC_REQUIRE(built && have_factors && m >= 0 && m < N && host, CPTC_E_ARG,
               "bad mode or call order");
  if (nranks == 1) {
    fetch_rows(F[m].p, m, host);
    return;
  }
  const uint64_t s = slab_rows(*this, m);
  const uint64_t lo = std::min<uint64_t>(s * (uint64_t)rank, dims[m]);
  const uint64_t hi = std::min<uint64_t>(s * (uint64_t)(rank + 1), dims[m]);
  const double* src = F[m].p;
  if (dperm[m].p) {
    double* st = stage_rows();
    permute_rows(F[m].p, m, false, st);
    src = st;
  }
  if (hi > lo)
    CPTC_CUDA(cudaMemcpyAsync(host + lo * R, src + lo * R, (hi - lo) * (uint64_t)R * sizeof(double),
                              cudaMemcpyDeviceToHost, stream));
  CPTC_CUDA(cudaStreamSynchronize(stream));
}

void Engine::fetch_rows(const double* dev, int m, double* host) {
  const uint64_t bytes = dims[m] * (uint64_t)R * sizeof(double);
  const double* src = dev;
  if (dperm[m].p) {
    double* st = stage_rows();
    permute_rows(dev, m, false, st);
    src = st;
  }
  CPTC_CUDA(cudaMemcpyAsync(host, src, bytes, cudaMemcpyDeviceToHost, stream));
  CPTC_CUDA(cudaStreamSynchronize(stream));
}

bool Engine::tiles_target(int mode) const {
  if (!dense_active) return false;
  for (int q = 0; q < 3; ++q)
    if (units.inner[q] == mode && units.cnt[q] > 0) return true;
  return false;
}

// FtV = MTTKRP of `mode` (relabelled rows): zero, dense tiles, residual.
void Engine::mttkrp(int mode) {
  if (nranks == 1) {
    CPTC_CUDA(cudaMemsetAsync(FtV.p, 0, dims[mode] * (uint64_t)R * sizeof(double), stream));
  } else {
    // the rows this rank's nonzeros can reach: the heavy prefix and its slab
    const uint64_t H = heavy_rows[mode], lo = row_lo(mode), hi = row_hi(mode);
    if (H > 0) CPTC_CUDA(cudaMemsetAsync(FtV.p, 0, H * (uint64_t)R * sizeof(double), stream));
    if (hi > lo)
      CPTC_CUDA(cudaMemsetAsync(FtV.p + lo * (uint64_t)R, 0,
                                (hi - lo) * (uint64_t)R * sizeof(double), stream));
  }
  // The residual kernel first: its many short CTAs rebalance around an SM
  // that the side stream's inverse may hold; the persistent tile grid is
  // launched once that SM is free again.
  mttkrp_sparse(mode);
  mttkrp_tiles(mode);
}

void Engine::mttkrp_tiles(int mode, double* out, cudaStream_t s) {
  if (!dense_active) return;
  int ts = -1;
  for (int q = 0; q < 3; ++q)
    if (units.inner[q] == mode) ts = q;
  if (ts < 0 || units.cnt[ts] == 0) return;
  cudaStream_t st = s ? s : stream;
  double* dst = out ? out : FtV.p;
  const uint32_t* cut = units.cut[ts].p;
  if (!generic) {
    // Order-3 roles (src/dense.cu:339-1075): mode 0 contracts j in TF32
    // and weights k-slabs; mode 1 contracts i, weights k; mode 2 contracts
    // i, weights j.
    Tile3Args ta{};
    ta.vtile = units.vtile[ts].p;
    ta.vstart = units.vstart[ts].p;
    ta.words = units.swords[ts].p ? units.swords[ts].p : units.words.p;
    ta.ntiles = units.cnt[ts];
    ta.R = R;
    ta.tslot = ts;
    ta.cslot = (ts == 0) ? 1 : 0;
    ta.sslot = (ts == 2) ? 1 : 2;
    for (int q = 0; q < 3; ++q) ta.dims[q] = dims[q];
    launch_to_tf32_blocks(F[ta.cslot].p, dims[ta.cslot], R, Ftf.p, st);
    ta.Fct = Ftf.p;
    ta.Fs = F[ta.sslot].p;
    ta.out = dst;
    launch_tiles3w(ta, cut, units.blocks, st);
    return;
  }
  TileArgs ta{};
  ta.tile = units.unit.p;
  ta.start = units.start.p;
  ta.lid = units.lid.p;
  ta.val = units.val.p;
  ta.ntiles = units.cnt[ts];
  ta.R = R;
  ta.tslot = ts;
  // N-order roles (src/generic.cu:486-487): fold slot t+1, weight t+2.
  ta.cslot = (ts + 1) % 3;
  ta.sslot = (ts + 2) % 3;
  for (int q = 0; q < 3; ++q) ta.dims[q] = dims[units.inner[q]];
  ta.Fc = F[units.inner[ta.cslot]].p;
  ta.Fs = F[units.inner[ta.sslot]].p;
  ta.nouter = units.nouter;
  ta.outer_idx = units.outer_idx.p;
  for (int q = 0; q < units.nouter; ++q) ta.Fout[q] = F[units.outer[q]].p;
  ta.store_dups = units.store_dups ? 1 : 0;
  ta.out = dst;
  launch_mttkrp_tiles3(ta, units.order[ts].p, cut, units.blocks, st);
}

void Engine::mttkrp_sparse(int mode) {
  const View& v = views[mode];
  MttkrpArgs a{};
  a.rec = v.rec.p;
  a.recw = v.recw;
  a.gw = v.gw.p;
  a.oidx = v.oidx.p;
  a.val = v.val.p;
  a.rows = v.rows.p;
  a.task_row = v.task_row.p;
  a.nnz = v.nnz;
  a.task0 = v.t0;
  a.ntasks = v.t1;
  a.task = v.task;
  a.nout = v.nout;
  a.R = R;
  a.Fg = F[v.gmode].p;
  for (int q = 0; q < v.nout; ++q) a.Fo[q] = F[v.omode[q]].p;
  a.out = FtV.p;
  launch_mttkrp_view(a, stream);
}

void Engine::gram_of(int m) {
  const int nb = launch_gram_partial(F[m].p, dims[m], R, gpart.p, gpart_blocks, stream);
  launch_gram_reduce(gpart.p, nb, R, G[m].p, stream);
}

// One mode update: Hadamard of the other Grams, MTTKRP, inverse, apply,
// normalisation.  Order-3 semantics (src/als.cu:480-517): pseudo-inverse,
// divide by lambda, norm < 1e-14 zeroes the column, lambda *= norm.
// N-order semantics (src/generic.cu:2109-2170): ridge Cholesky (default),
// lambda = norms with norm < 1e-14 -> 1.
void Engine::update_mode(int n, bool last) {
  const double* gs[CPTC_MAX_ORDER];
  int ng = 0;
  for (int m = 0; m < N; ++m)
    if (m != n) gs[ng++] = G[m].p;
  // Order 3: the reference solves with a truncated SVD pseudo-inverse; by
  // default the same result is obtained by the sweep inverse when FtF is
  // well conditioned (the pseudo-inverse kernel runs only when it is not).
  // N-order: the reference's ridge rule.  The inverse needs only the other
  // modes' Grams, so it runs on the side stream during this mode's MTTKRP;
  // it is launched first so that its single CTA is placed before the
  // MTTKRP fills the GPU.
  int inv = generic ? kInvCholRidge : kInvAuto;
  if (opts.solver == CPTC_SOLVER_CHOL) inv = kInvCholRidge;
  if (opts.solver == CPTC_SOLVER_PINV) inv = kInvPinv;
  CPTC_CUDA(cudaEventRecord(ev_fork, stream));
  CPTC_CUDA(cudaStreamWaitEvent(side, ev_fork, 0));
  launch_sym_inverse(gs, ng, R, inv, FtF.p, Ainv.p, status.p, side);
  CPTC_CUDA(cudaEventRecord(ev_join, side));
  // Per-mode MTTKRP timing; while the iteration is being captured the
  // records must be External so that the graph performs them.
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  CPTC_CUDA(cudaStreamIsCapturing(stream, &cs));
  const unsigned rf = (cs == cudaStreamCaptureStatusActive) ? cudaEventRecordExternal
                                                            : cudaEventRecordDefault;
  auto phase_end = [&](int k) {
    if (phase_timing) CPTC_CUDA(cudaEventRecordWithFlags(evp[cur_slot][n][k], stream, rf));
  };
  CPTC_CUDA(cudaEventRecordWithFlags(evc[2 * n], stream, rf));
  mttkrp(n);
  CPTC_CUDA(cudaEventRecordWithFlags(evc[2 * n + 1], stream, rf));
  CPTC_CUDA(cudaStreamWaitEvent(stream, ev_join, 0));
  phase_end(0);
  const int div = generic ? 0 : 1;
  const uint64_t lo = row_lo(n), rows = row_hi(n) - lo;
  // The last mode also yields the fit's column dot products, taken on the
  // solved (not yet normalised) rows in the same pass and scaled with the
  // column scales.
  const int nb = launch_apply_solve(FtV.p + lo * R, Ainv.p, lambda.p, div, rows, R,
                                    F[n].p + lo * R, gpart.p, gpart_blocks, stream,
                                    last ? dots.p : nullptr);
  const int nd = last ? nb : 0;
  phase_end(1);
  // The Gram partial (and fit dots) summed over blocks and ranks; with
  // several ranks grouped with the all-reduce of the heavy prefix's partial
  // MTTKRP and the all-reduce that shares every rank's solved slab.
  double* gsum = comm_exchange_mode(*this, n, nb, last ? nd : -1);
  const uint64_t H = heavy_rows[n];
  if (H > 0) {
    // The heavy prefix, now summed over the ranks, is solved by every rank
    // (the same bits everywhere) and its Gram and dots added once.
    const int nbh = launch_apply_solve(FtV.p, Ainv.p, lambda.p, div, H, R, F[n].p, gpart.p,
                                       gpart_blocks, stream, last ? dots.p : nullptr);
    launch_partial_sum_add(gpart.p, nbh, R * R, gsum, stream);
    if (last) launch_partial_sum_add(dots.p, nbh, R, gsum + (size_t)R * R, stream);
  }
  phase_end(2);
  launch_norm_finalize(gsum, 1, R, generic ? 1 : 0, lambda.p, G[n].p, colscale(), stream);
  launch_scale_cols(F[n].p, dims[n], R, colscale(), stream);
  if (last) {
    const double* gall[CPTC_MAX_ORDER];
    for (int m = 0; m < N; ++m) gall[m] = G[m].p;
    launch_fit_final(gsum + (size_t)R * R, 1, colscale(), lambda.p, gall, N, R, scal.p, stream);
  }
  phase_end(3);
}

void Engine::set_phase_timing(bool on) {
  CPTC_CUDA(cudaSetDevice(device));
  if (on && !evp[0][0][0])
    for (auto& sl : evp)
      for (auto& md : sl)
        for (auto& e : md) CPTC_CUDA(cudaEventCreate(&e));
  if (on != phase_timing) {
    CPTC_CUDA(cudaStreamSynchronize(stream));
    release_graph();  // the captured iteration has (or lacks) the events
  }
  phase_timing = on;
  phase_valid = false;
}

double* Engine::colscale() { return cscale.p; }

void Engine::release_graph() {
  for (int k = 0; k < 2; ++k) {
    if (iter_exec[k]) cudaGraphExecDestroy(iter_exec[k]);
    if (iter_graph[k]) cudaGraphDestroy(iter_graph[k]);
    iter_exec[k] = nullptr;
    iter_graph[k] = nullptr;
  }
}

// One ALS iteration on the stream: every mode update, then the fit and the
// solve status copied to readback slot `slot` of the pinned host buffer.
void Engine::enqueue_iteration(int slot) {
  evc = slot ? ev1 : ev;
  cur_slot = slot;
  for (int n = 0; n < N; ++n) update_mode(n, n == N - 1);
  double* hs = h_scal + 8 * slot;
  CPTC_CUDA(cudaMemcpyAsync(hs, scal.p, 2 * sizeof(double), cudaMemcpyDeviceToHost, stream));
  CPTC_CUDA(cudaMemcpyAsync(hs + 4, status.p, sizeof(int), cudaMemcpyDeviceToHost, stream));
  evc = ev;
}

// The iteration is captured once into a CUDA graph (kernels, the side
// stream's inverse, NCCL calls, the readback) and replayed with one launch,
// so host launch overhead does not gap the GPU between the short solve
// kernels; set CPTC_GRAPH=0 to launch it stream-ordered instead.
void Engine::launch_iteration(int slot) {
  static const bool use_graph = [] {
    const char* e = std::getenv("CPTC_GRAPH");
    return !(e && e[0] == '0');
  }();
  cudaEvent_t* E = slot ? ev1 : ev;
  // The iteration's start and end events are recorded outside the graph:
  // the host waits on the end event for the fit.
  CPTC_CUDA(cudaEventRecord(E[2 * CPTC_MAX_ORDER], stream));
  if (!use_graph) {
    enqueue_iteration(slot);
    CPTC_CUDA(cudaEventRecord(E[2 * CPTC_MAX_ORDER + 1], stream));
    return;
  }
  if (!iter_exec[slot]) {
    // Kernels enqueued during capture are counted when the graph runs.
    const unsigned long long l0 = t_launches;
    CPTC_CUDA(cudaStreamBeginCapture(stream, cudaStreamCaptureModeRelaxed));
    try {
      enqueue_iteration(slot);
    } catch (...) {
      cudaGraph_t g = nullptr;
      cudaStreamEndCapture(stream, &g);
      if (g) cudaGraphDestroy(g);
      cudaGetLastError();
      g_launches.fetch_sub(t_launches - l0);
      t_launches = l0;
      evc = ev;
      throw;
    }
    iter_kernels = t_launches - l0;
    g_launches.fetch_sub(iter_kernels);  // counted when the graph runs
    t_launches = l0;
    CPTC_CUDA(cudaStreamEndCapture(stream, &iter_graph[slot]));
    CPTC_CUDA(cudaGraphInstantiate(&iter_exec[slot], iter_graph[slot], 0));
  }
  CPTC_CUDA(cudaGraphLaunch(iter_exec[slot], stream));
  g_launches.fetch_add(iter_kernels);
  CPTC_CUDA(cudaEventRecord(E[2 * CPTC_MAX_ORDER + 1], stream));
}

// Waits for iteration `it` (readback slot `slot`), checks the solve status,
// computes the fit and reports it.
void Engine::finish_iteration(int it, int slot, cptc_iter_cb cb, void* user) {
  cudaEvent_t* E = slot ? ev1 : ev;
  const double* hs = h_scal + 8 * slot;
  CPTC_CUDA(cudaEventSynchronize(E[2 * CPTC_MAX_ORDER + 1]));
  int h_status = 0;
  std::memcpy(&h_status, hs + 4, sizeof(int));
  if (h_status != 0) {
    cudaStreamSynchronize(stream);  // the next iteration may be in flight
    throw CptcError(CPTC_E_NUMERIC, "non-finite values in the R x R solve");
  }
  const double xn = std::sqrt(x_norm_sq);
  const double iprod = hs[0], model2 = hs[1];
  const double res2 = std::max(x_norm_sq - 2.0 * iprod + model2, 0.0);
  const double fit = (xn > 0.0) ? 1.0 - std::sqrt(res2) / xn : 0.0;
  float ms_it = 0.f;
  cudaEventElapsedTime(&ms_it, E[2 * CPTC_MAX_ORDER], E[2 * CPTC_MAX_ORDER + 1]);
  double mode_ms[CPTC_MAX_ORDER] = {0};
  for (int n = 0; n < N; ++n) {
    float t = 0.f;
    cudaEventElapsedTime(&t, E[2 * n], E[2 * n + 1]);
    mode_ms[n] = t;
  }
  if (phase_timing) {
    for (int n = 0; n < N; ++n) {
      const cudaEvent_t b[5] = {E[2 * n + 1], evp[slot][n][0], evp[slot][n][1],
                                evp[slot][n][2], evp[slot][n][3]};
      phase_ms[n][0] = mode_ms[n];
      for (int k = 0; k < 4; ++k) {
        float t = 0.f;
        CPTC_CUDA(cudaEventElapsedTime(&t, b[k], b[k + 1]));
        phase_ms[n][k + 1] = t;
      }
    }
    phase_valid = true;
  }
  last_iprod = iprod;
  last_model2 = model2;
  last_fit = fit;
  if (cb) cb(it + 1, (double)ms_it, fit, mode_ms, N, user);
}

void Engine::als(int iters, cptc_iter_cb cb, void* user) {
  CPTC_REQUIRE(built && have_factors, CPTC_E_ARG, "call cptc_build and cptc_init_factors first");
  CPTC_CUDA(cudaSetDevice(device));
  if (!grams_valid) {
    for (int m = 0; m < N; ++m) gram_of(m);
    grams_valid = true;
  }
  CPTC_CUDA(cudaMemsetAsync(status.p, 0, sizeof(int), stream));
  // One iteration stays in flight: iteration it + 1 is launched before the
  // fit of iteration it is read, so the GPU does not wait for the host
  // between iterations (the iterations do not depend on host decisions).
  for (int it = 0; it < iters; ++it) {
    launch_iteration(it & 1);
    if (it > 0) finish_iteration(it - 1, (it - 1) & 1, cb, user);
  }
  if (iters > 0) finish_iteration(iters - 1, (iters - 1) & 1, cb, user);
}

}  // namespace cptc

// ===========================================================================
// C ABI
// ===========================================================================
using cptc::CptcError;
using cptc::Engine;

struct cptc_ctx {
  Engine* e = nullptr;
  std::string err;
};

namespace {

template <class F>
int guarded(cptc_ctx* c, F&& f) {
  if (!c || !c->e) return CPTC_E_ARG;
  try {
    f(*c->e);
    c->err.clear();
    return CPTC_OK;
  } catch (const CptcError& x) {
    c->err = x.what();
    return x.code;
  } catch (const std::bad_alloc&) {
    c->err = "host allocation failed";
    return CPTC_E_NOMEM;
  } catch (const std::exception& x) {
    c->err = x.what();
    return CPTC_E_ARG;
  } catch (...) {
    c->err = "unknown error";
    return CPTC_E_ARG;
  }
}

}  // namespace

extern "C" {

int cptc_opts_default(cptc_opts* o) {
  if (!o) return CPTC_E_ARG;
  std::memset(o, 0, sizeof(*o));
  o->path = CPTC_PATH_AUTO;
  o->fill_min = 0.0;
  o->generic = 0;
  o->reorder = CPTC_REORDER_DEFAULT;
  o->reorder_rounds = 3;
  o->reorder_sample = 8000000ull;
  o->solver = CPTC_SOLVER_DEFAULT;
  o->seed = 42u;
  o->dense_generic = 1;
  o->dense_thr_generic = 0.03;
  o->dense_inner[0] = 0;
  o->dense_inner[1] = 1;
  o->dense_inner[2] = 2;
  o->verbose = 0;
  o->exchange = CPTC_EXCHANGE_NCCL;
  return CPTC_OK;
}

int cptc_create(cptc_ctx** out, int device, int flags) {
  (void)flags;
  if (!out) return CPTC_E_ARG;
  *out = nullptr;
  cptc_ctx* c = new (std::nothrow) cptc_ctx;
  if (!c) return CPTC_E_NOMEM;
  try {
    c->e = new Engine(device);
  } catch (const CptcError& x) {
    const int code = x.code;
    delete c;
    return code;
  } catch (const std::bad_alloc&) {
    delete c;
    return CPTC_E_NOMEM;
  } catch (...) {
    delete c;
    return CPTC_E_CUDA;
  }
  *out = c;
  return CPTC_OK;
}

int cptc_destroy(cptc_ctx* c) {
  if (!c) return CPTC_E_ARG;
  delete c->e;
  delete c;
  return CPTC_OK;
}

const char* cptc_last_error(const cptc_ctx* c) { return c ? c->err.c_str() : "null context"; }

int cptc_load_coo(cptc_ctx* c, const cptc_coo* t) {
  return guarded(c, [&](Engine& e) { e.load(t); });
}

int cptc_comm_init(cptc_ctx* c, const unsigned char id[128], int rank, int nranks) {
  return guarded(c, [&](Engine& e) {
    CPTC_REQUIRE(id != nullptr, CPTC_E_ARG, "null id");
    cptc::comm_init(e, id, rank, nranks);
  });
}

int cptc_build(cptc_ctx* c, int R, double threshold, const cptc_opts* o) {
  return guarded(c, [&](Engine& e) { e.build(R, threshold, o); });
}

int cptc_init_factors(cptc_ctx* c) {
  return guarded(c, [&](Engine& e) { e.init_factors(); });
}

int cptc_set_factors(cptc_ctx* c, int mode, const double* host) {
  return guarded(c, [&](Engine& e) { e.set_factor(mode, host); });
}

int cptc_set_factors_sharded(cptc_ctx* c, int mode, const double* host) {
  return guarded(c, [&](Engine& e) { e.set_factor_sharded(mode, host); });
}

int cptc_get_factors_sharded(cptc_ctx* c, int mode, double* host) {
  return guarded(c, [&](Engine& e) { e.get_factor_sharded(mode, host); });
}

int cptc_get_factors(cptc_ctx* c, int mode, double* host) {
  return guarded(c, [&](Engine& e) { e.get_factor(mode, host); });
}

int cptc_get_lambda(cptc_ctx* c, double* host) {
  return guarded(c, [&](Engine& e) {
    CPTC_REQUIRE(e.built && e.have_factors && host, CPTC_E_ARG, "no factors yet");
    CPTC_CUDA(cudaMemcpyAsync(host, e.lambda.p, e.R * sizeof(double), cudaMemcpyDeviceToHost,
                              e.stream));
    CPTC_CUDA(cudaStreamSynchronize(e.stream));
  });
}

int cptc_mttkrp(cptc_ctx* c, int mode, double* host_out) {
  return guarded(c, [&](Engine& e) {
    CPTC_REQUIRE(e.built && e.have_factors && mode >= 0 && mode < e.N && host_out, CPTC_E_ARG,
                 "bad mode or call order");
    CPTC_CUDA(cudaSetDevice(e.device));
    e.mttkrp(mode);
    cptc::comm_reduce_ftv(e, mode);
    e.fetch_rows(e.FtV.p, mode, host_out);
  });
}

int cptc_mttkrp_timed(cptc_ctx* c, int mode, int reps, double* ms) {
  return guarded(c, [&](Engine& e) {
    CPTC_REQUIRE(e.built && e.have_factors && mode >= 0 && mode < e.N && reps > 0, CPTC_E_ARG,
                 "bad mode or call order");
    CPTC_CUDA(cudaSetDevice(e.device));
    cudaEvent_t a = e.ev[0], b = e.ev[1];
    CPTC_CUDA(cudaEventRecord(a, e.stream));
    for (int r = 0; r < reps; ++r) e.mttkrp(mode);
    CPTC_CUDA(cudaEventRecord(b, e.stream));
    CPTC_CUDA(cudaEventSynchronize(b));
    float t = 0.f;
    CPTC_CUDA(cudaEventElapsedTime(&t, a, b));
    if (ms) *ms = (double)t / reps;
  });
}

int cptc_profile_gather(cptc_ctx* c, int mode, int reps, double* ms2) {
  return guarded(c, [&](Engine& e) {
    CPTC_REQUIRE(e.built && e.have_factors && mode >= 0 && mode < e.N && reps > 0 && ms2,
                 CPTC_E_ARG, "bad mode or call order");
    CPTC_CUDA(cudaSetDevice(e.device));
    const cptc::View& v = e.views[mode];
    ms2[0] = cptc::time_gather_replay(v, e.R, e.F[v.gmode].p, e.F[v.omode[0]].p, reps, e.stream);
    CPTC_CUDA(cudaMemsetAsync(e.FtV.p, 0, e.dims[mode] * (uint64_t)e.R * sizeof(double),
                              e.stream));
    e.mttkrp_sparse(mode);  // warm-up
    CPTC_CUDA(cudaEventRecord(e.ev[0], e.stream));
    for (int r = 0; r < reps; ++r) e.mttkrp_sparse(mode);
    CPTC_CUDA(cudaEventRecord(e.ev[1], e.stream));
    CPTC_CUDA(cudaEventSynchronize(e.ev[1]));
    float b = 0.f;
    CPTC_CUDA(cudaEventElapsedTime(&b, e.ev[0], e.ev[1]));
    ms2[1] = b / reps;
  });
}

int cptc_profile_mttkrp(cptc_ctx* c, int mode, int reps, double* ms3) {
  return guarded(c, [&](Engine& e) {
    CPTC_REQUIRE(e.built && e.have_factors && mode >= 0 && mode < e.N && reps > 0 && ms3,
                 CPTC_E_ARG, "bad mode or call order");
    CPTC_CUDA(cudaSetDevice(e.device));
    cudaEvent_t* ev = e.ev;
    CPTC_CUDA(cudaMemsetAsync(e.FtV.p, 0, e.dims[mode] * (uint64_t)e.R * sizeof(double),
                              e.stream));
    CPTC_CUDA(cudaEventRecord(ev[0], e.stream));
    for (int r = 0; r < reps; ++r) e.mttkrp_tiles(mode);
    CPTC_CUDA(cudaEventRecord(ev[1], e.stream));
    for (int r = 0; r < reps; ++r) e.mttkrp_sparse(mode);
    CPTC_CUDA(cudaEventRecord(ev[2], e.stream));
    for (int r = 0; r < reps; ++r) e.mttkrp(mode);
    CPTC_CUDA(cudaEventRecord(ev[3], e.stream));
    CPTC_CUDA(cudaEventSynchronize(ev[3]));
    float a = 0.f, b = 0.f, t = 0.f;
    CPTC_CUDA(cudaEventElapsedTime(&a, ev[0], ev[1]));
    CPTC_CUDA(cudaEventElapsedTime(&b, ev[1], ev[2]));
    CPTC_CUDA(cudaEventElapsedTime(&t, ev[2], ev[3]));
    ms3[0] = a / reps;
    ms3[1] = b / reps;
    ms3[2] = t / reps;
  });
}

unsigned long long cptc_launch_count(void) { return cptc::g_launches.load(); }

int cptc_get_relabel(cptc_ctx* c, int mode, uint32_t* perm_out) {
  return guarded(c, [&](Engine& e) {
    CPTC_REQUIRE(e.built && mode >= 0 && mode < e.N && perm_out, CPTC_E_ARG, "call order");
    if (e.perm[mode].empty())
      for (uint64_t a = 0; a < e.dims[mode]; ++a) perm_out[a] = (uint32_t)a;
    else
      std::memcpy(perm_out, e.perm[mode].data(), e.dims[mode] * sizeof(uint32_t));
  });
}

int cptc_phase_timing(cptc_ctx* c, int on) {
  return guarded(c, [&](Engine& e) { e.set_phase_timing(on != 0); });
}

int cptc_phase_times(cptc_ctx* c, double* out, int cap) {
  int written = 0;
  const int rc = guarded(c, [&](Engine& e) {
    CPTC_REQUIRE(out != nullptr || cap == 0, CPTC_E_ARG, "null output");
    if (!e.phase_timing || !e.phase_valid) return;
    for (int n = 0; n < e.N; ++n)
      for (int p = 0; p < CPTC_NPHASES; ++p)
        if (written < cap) out[written++] = e.phase_ms[n][p];
  });
  return rc != 0 ? rc : written;
}

int cptc_fit_terms(cptc_ctx* c, double* out3) {
  return guarded(c, [&](Engine& e) {
    CPTC_REQUIRE(out3 != nullptr, CPTC_E_ARG, "null output");
    out3[0] = e.last_iprod;
    out3[1] = e.last_model2;
    out3[2] = e.last_fit;
  });
}

int cptc_residual(cptc_ctx* c, double* out2) {
  return guarded(c, [&](Engine& e) {
    CPTC_REQUIRE(e.built && e.have_factors && out2, CPTC_E_ARG, "call order");
    CPTC_CUDA(cudaSetDevice(e.device));
    cptc::ResidualArgs a{};
    for (int m = 0; m < e.N; ++m) {
      a.idx[m] = e.idx[m].p;
      a.F[m] = e.F[m].p;
    }
    a.val = e.vals.p;
    a.lambda = e.lambda.p;
    a.nnz = e.nnz;
    a.N = e.N;
    a.R = e.R;
    cptc::DArray<double> part(148 * 8);
    cptc::launch_residual(a, part.p, 148 * 8, e.scal.p + 4, e.stream);
    CPTC_CUDA(cudaMemcpyAsync(out2, e.scal.p + 4, sizeof(double), cudaMemcpyDeviceToHost, e.stream));
    CPTC_CUDA(cudaStreamSynchronize(e.stream));
    out2[1] = e.x_norm_sq;
  });
}

int cptc_als(cptc_ctx* c, int iters, cptc_iter_cb cb, void* user) {
  return guarded(c, [&](Engine& e) { e.als(iters, cb, user); });
}

int cptc_get_stats(cptc_ctx* c, cptc_stats* s) {
  return guarded(c, [&](Engine& e) {
    CPTC_REQUIRE(s != nullptr, CPTC_E_ARG, "null stats");
    std::memset(s, 0, sizeof(*s));
    s->order = e.N;
    for (int m = 0; m < e.N; ++m) s->dims[m] = e.dims[m];
    s->nnz = e.nnz;
    s->rank = e.R;
    s->tf32_path = e.tf32 ? 1 : 0;
    s->dense_nnz = e.tf32 ? e.units.nnz : 0;
    s->sparse_nnz = e.nnz - s->dense_nnz;
    s->dense_tiles = e.tf32 ? e.units.nunits : 0;
    s->avg_fill = e.avg_fill;
    s->fill_min = e.fill_min;
    s->cutoff = e.cutoff;
    s->x_norm_sq = e.x_norm_sq;
    s->build_ms = e.build_ms;
    s->device_bytes = e.device_bytes();
    for (int m = 0; m < e.N && m < (int)e.views.size(); ++m)
      s->fiber_mode[m] = e.views[m].nout > 0 ? e.views[m].omode[0] : -1;
    s->nranks = e.nranks;
    s->rank_id = e.rank;
    s->reorder_ms = e.reorder_ms;
    for (int m = 0; m < e.N && m < (int)e.views.size(); ++m) {
      s->local_sparse_nnz[m] = e.views[m].nnz;
      s->local_rows[m] = e.views[m].nrows;
      for (int t = 0; t < 3; ++t)
        if (e.dense_active && e.units.inner[t] == m) {
          s->local_tiles[m] = e.units.cnt[t];
          s->local_tile_words[m] = e.generic ? 0 : e.units.wcnt[t];
        }
    }
  });
}

}  // extern "C"
