// N-order dense units: 16^3 tiles over the inner modes with every outer
// mode fixed (reference build_dense_nd, src/generic.cu:578-725, and
// g_dense_tile_mttkrp_kernel, :429-561).
//
// The reference keys a unit by a 64-bit hash of (tile, outer tuple) in a
// host unordered_map; here elements are radix-sorted on the device by the
// exact (inner tile, outer tuple) key and units are the runs with at least
// int(4096 * threshold) nonzeros.  The arithmetic runs through the shared
// tile kernel (tiles.cu) with the outer modes folded into the FP64 weight.
#include <cub/cub.cuh>

#include "kernels.hpp"

namespace cptc {

namespace {

struct UnitKeyArgs {
  const uint32_t* in[3];
  uint64_t nb1, nb2;  // tile counts of inner modes 1, 2
  int nout;
  const uint32_t* out[CPTC_MAX_ORDER];
  uint64_t odim[CPTC_MAX_ORDER];
};

__global__ void k_unit_keys(UnitKeyArgs a, uint64_t n, uint64_t* __restrict__ tkey,
                            uint64_t* __restrict__ okey, uint32_t* __restrict__ id) {
  for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < n;
       e += (uint64_t)gridDim.x * blockDim.x) {
    tkey[e] = ((uint64_t)(a.in[0][e] >> 4) * a.nb1 + (a.in[1][e] >> 4)) * a.nb2 + (a.in[2][e] >> 4);
    uint64_t o = 0;
    for (int q = 0; q < a.nout; ++q) o = o * a.odim[q] + a.out[q][e];
    okey[e] = o;
    id[e] = (uint32_t)e;
  }
}

__global__ void k_gather_u64(const uint64_t* __restrict__ src, const uint32_t* __restrict__ perm,
                             uint64_t n, uint64_t* __restrict__ dst) {
  for (uint64_t p = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; p < n;
       p += (uint64_t)gridDim.x * blockDim.x)
    dst[p] = src[perm[p]];
}

__global__ void k_unit_flags(const uint64_t* __restrict__ tk, const uint64_t* __restrict__ ok,
                             uint64_t n, uint32_t* __restrict__ flag) {
  for (uint64_t p = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; p < n;
       p += (uint64_t)gridDim.x * blockDim.x)
    flag[p] = (p == 0 || tk[p] != tk[p - 1] || ok[p] != ok[p - 1]) ? 1u : 0u;
}

// Run lengths from run starts: counts[k] = start[k+1] - start[k].
__global__ void k_run_counts(const uint32_t* __restrict__ start, uint64_t nruns, uint64_t n,
                             int* __restrict__ counts) {
  for (uint64_t k = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; k < nruns;
       k += (uint64_t)gridDim.x * blockDim.x)
    counts[k] = (int)(((k + 1 < nruns) ? (uint64_t)start[k + 1] : n) - start[k]);
}

__global__ void k_elem_dense_u(const uint32_t* __restrict__ runid, const int* __restrict__ counts,
                               uint64_t n, int cutoff, uint32_t* __restrict__ dflag) {
  for (uint64_t p = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; p < n;
       p += (uint64_t)gridDim.x * blockDim.x)
    dflag[p] = counts[runid[p] - 1] >= cutoff ? 1u : 0u;
}

__global__ void k_scatter_units(const uint32_t* __restrict__ perm, const uint32_t* __restrict__ dflag,
                                const uint64_t* __restrict__ dpos, uint64_t n, UnitKeyArgs a,
                                const double* __restrict__ vals, uint16_t* __restrict__ lid,
                                double* __restrict__ pval, uint32_t* __restrict__ sel) {
  for (uint64_t p = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; p < n;
       p += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t e = perm[p];
    if (dflag[p]) {
      const uint64_t d = dpos[p];
      lid[d] = (uint16_t)(((a.in[0][e] & 15u) << 8) | ((a.in[1][e] & 15u) << 4) |
                          (a.in[2][e] & 15u));
      pval[d] = vals[e];
    } else {
      sel[p - dpos[p]] = e;
    }
  }
}

__global__ void k_units_from_runs(const uint32_t* __restrict__ runs_sel, uint64_t nunits,
                                  const uint32_t* __restrict__ run_start,
                                  const uint32_t* __restrict__ perm, const int* __restrict__ counts,
                                  UnitKeyArgs a, int4* __restrict__ unit,
                                  uint64_t* __restrict__ cnt64, uint32_t* __restrict__ outer_idx) {
  for (uint64_t k = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; k < nunits;
       k += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t r = runs_sel[k];
    const uint32_t e = perm[run_start[r]];
    unit[k] = make_int4((int)(a.in[0][e] >> 4), (int)(a.in[1][e] >> 4), (int)(a.in[2][e] >> 4),
                        counts[r]);
    cnt64[k] = (uint64_t)counts[r];
    for (int q = 0; q < a.nout; ++q) outer_idx[k * a.nout + q] = a.out[q][e];
  }
}

__global__ void k_unit_slot_keys(const int4* __restrict__ u, uint64_t n, int slot,
                                 uint32_t* __restrict__ key, uint32_t* __restrict__ id) {
  for (uint64_t k = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; k < n;
       k += (uint64_t)gridDim.x * blockDim.x) {
    const int4 t = u[k];
    key[k] = (uint32_t)(slot == 0 ? t.x : slot == 1 ? t.y : t.z);
    id[k] = (uint32_t)k;
  }
}

struct AtLeast {
  int c;
  __host__ __device__ uint8_t operator()(int x) const { return x >= c ? 1 : 0; }
};

template <class F>
void cub_call(DArray<unsigned char>& temp, F&& f) {
  size_t b = 0;
  CPTC_CUDA(f((void*)nullptr, b));
  if (b > temp.bytes()) temp.alloc(b);
  CPTC_CUDA(f((void*)temp.p, b));
}

}  // namespace

void partition_units(Engine& E, double threshold, DArray<uint32_t>& sel, uint64_t& nsel) {
  cudaStream_t s = E.stream;
  UnitPool& U = E.units;
  U = UnitPool{};
  const uint64_t n = E.nnz;
  for (int q = 0; q < 3; ++q) U.inner[q] = E.opts.dense_inner[q];
  U.nouter = 0;
  for (int m = 0; m < E.N; ++m)
    if (m != U.inner[0] && m != U.inner[1] && m != U.inner[2]) U.outer[U.nouter++] = m;
  UnitKeyArgs ka{};
  for (int q = 0; q < 3; ++q) ka.in[q] = E.idx[U.inner[q]].p;
  ka.nb1 = (E.dims[U.inner[1]] + 15) / 16;
  ka.nb2 = (E.dims[U.inner[2]] + 15) / 16;
  ka.nout = U.nouter;
  unsigned __int128 ospace = 1;
  for (int q = 0; q < U.nouter; ++q) {
    ka.out[q] = E.idx[U.outer[q]].p;
    ka.odim[q] = E.dims[U.outer[q]];
    ospace *= ka.odim[q];
  }
  CPTC_REQUIRE(ospace < ((unsigned __int128)1 << 63), CPTC_E_UNSUP,
               "outer-mode tuple does not fit a 64-bit key");
  const int obits = bits_for((uint64_t)ospace);
  const int tbits = bits_for(((E.dims[U.inner[0]] + 15) / 16) * ka.nb1 * ka.nb2);

  const unsigned gb = grid_for(n, 256, 148 * 16);
  DArray<uint64_t> tk(n), ok(n), ktmp(n);
  DArray<uint32_t> id_a(n), id_b(n);
  k_unit_keys<<<gb, 256, 0, s>>>(ka, n, tk.p, ok.p, id_a.p);
  CPTC_LAUNCH_CHECK();
  DArray<unsigned char> temp;
  // LSD: outer key, then tile key (both stable).
  cub_call(temp, [&](void* t, size_t& b) {
    return cub::DeviceRadixSort::SortPairs(t, b, ok.p, ktmp.p, id_a.p, id_b.p, (int64_t)n, 0,
                                           obits, s);
  });
  k_gather_u64<<<gb, 256, 0, s>>>(tk.p, id_b.p, n, ok.p);  // tile keys in outer order
  CPTC_LAUNCH_CHECK();
  cub_call(temp, [&](void* t, size_t& b) {
    return cub::DeviceRadixSort::SortPairs(t, b, ok.p, tk.p, id_b.p, id_a.p, (int64_t)n, 0,
                                           tbits, s);
  });
  // tk = sorted tile keys, id_a = permutation; outer keys in sorted order:
  k_unit_keys<<<gb, 256, 0, s>>>(ka, n, ktmp.p, ok.p, id_b.p);  // ok = outer key by element
  CPTC_LAUNCH_CHECK();
  k_gather_u64<<<gb, 256, 0, s>>>(ok.p, id_a.p, n, ktmp.p);
  CPTC_LAUNCH_CHECK();
  DArray<uint32_t> flag(n), runid(n);
  k_unit_flags<<<gb, 256, 0, s>>>(tk.p, ktmp.p, n, flag.p);
  CPTC_LAUNCH_CHECK();
  cub_call(temp, [&](void* t, size_t& b) {
    return cub::DeviceScan::InclusiveSum(t, b, flag.p, runid.p, (int64_t)n, s);
  });
  DArray<uint32_t> rstart(n);
  DArray<unsigned long long> nr_d(1);
  cub::CountingInputIterator<uint32_t> cnt(0);
  {
    auto asbool = cub::TransformInputIterator<bool, cub::CastOp<bool>, const uint32_t*>(
        flag.p, cub::CastOp<bool>());
    cub_call(temp, [&](void* t, size_t& b) {
      return cub::DeviceSelect::Flagged(t, b, cnt, asbool, rstart.p, nr_d.p, (int64_t)n, s);
    });
  }
  unsigned long long nruns = 0;
  CPTC_CUDA(cudaMemcpyAsync(&nruns, nr_d.p, sizeof(nruns), cudaMemcpyDeviceToHost, s));
  CPTC_CUDA(cudaStreamSynchronize(s));
  DArray<int> counts(nruns);
  k_run_counts<<<grid_for(nruns, 256, 148 * 16), 256, 0, s>>>(rstart.p, nruns, n, counts.p);
  CPTC_LAUNCH_CHECK();
  const int cutoff = (int)(4096.0 * threshold);  // src/generic.cu:584, no clamp
  k_elem_dense_u<<<gb, 256, 0, s>>>(runid.p, counts.p, n, cutoff, flag.p);
  CPTC_LAUNCH_CHECK();
  DArray<uint64_t> dpos(n + 1);
  {
    auto conv = cub::TransformInputIterator<uint64_t, cub::CastOp<uint64_t>, const uint32_t*>(
        flag.p, cub::CastOp<uint64_t>());
    cub_call(temp, [&](void* t, size_t& b) {
      return cub::DeviceScan::ExclusiveSum(t, b, conv, dpos.p, (int64_t)n, s);
    });
  }
  uint64_t last_pos = 0;
  uint32_t last_flag = 0;
  CPTC_CUDA(cudaMemcpyAsync(&last_pos, dpos.p + (n - 1), 8, cudaMemcpyDeviceToHost, s));
  CPTC_CUDA(cudaMemcpyAsync(&last_flag, flag.p + (n - 1), 4, cudaMemcpyDeviceToHost, s));
  CPTC_CUDA(cudaStreamSynchronize(s));
  U.nnz = last_pos + last_flag;
  nsel = n - U.nnz;
  U.lid.alloc(U.nnz + 8);  // the tile kernel copies whole 4-byte words
  U.val.alloc(U.nnz);
  sel.alloc(nsel);
  k_scatter_units<<<gb, 256, 0, s>>>(id_a.p, flag.p, dpos.p, n, ka, E.vals.p, U.lid.p, U.val.p,
                                     sel.p);
  CPTC_LAUNCH_CHECK();

  // Units = runs with count >= cutoff, in key order.
  {
    DArray<uint32_t> rsel(nruns);
    DArray<unsigned long long> nu_d(1);
    cub::TransformInputIterator<uint8_t, AtLeast, const int*> fl(counts.p, AtLeast{cutoff});
    cub_call(temp, [&](void* t, size_t& b) {
      return cub::DeviceSelect::Flagged(t, b, cnt, fl, rsel.p, nu_d.p, (int64_t)nruns, s);
    });
    unsigned long long nunits = 0;
    CPTC_CUDA(cudaMemcpyAsync(&nunits, nu_d.p, sizeof(nunits), cudaMemcpyDeviceToHost, s));
    CPTC_CUDA(cudaStreamSynchronize(s));
    U.nunits = nunits;
    U.unit.alloc(nunits);
    U.start.alloc(nunits);
    U.outer_idx.alloc(std::max<uint64_t>(1, nunits * (uint64_t)U.nouter));
    if (nunits) {
      DArray<uint64_t> c64(nunits);
      k_units_from_runs<<<grid_for(nunits, 256, 148 * 16), 256, 0, s>>>(
          rsel.p, nunits, rstart.p, id_a.p, counts.p, ka, U.unit.p, c64.p, U.outer_idx.p);
      CPTC_LAUNCH_CHECK();
      cub_call(temp, [&](void* t, size_t& b) {
        return cub::DeviceScan::ExclusiveSum(t, b, c64.p, U.start.p, (int64_t)nunits, s);
      });
      for (int slot = 0; slot < 3; ++slot) {
        DArray<uint32_t> ka2(nunits), kb2(nunits), ia(nunits);
        U.order[slot].alloc(nunits);
        k_unit_slot_keys<<<grid_for(nunits, 256, 148 * 16), 256, 0, s>>>(U.unit.p, nunits, slot,
                                                                          ka2.p, ia.p);
        CPTC_LAUNCH_CHECK();
        cub_call(temp, [&](void* t, size_t& b) {
          return cub::DeviceRadixSort::SortPairs(t, b, ka2.p, kb2.p, ia.p, U.order[slot].p,
                                                 (int64_t)nunits, 0, 32, s);
        });
      }
    }
  }
  CPTC_CUDA(cudaStreamSynchronize(s));
}

}  // namespace cptc
