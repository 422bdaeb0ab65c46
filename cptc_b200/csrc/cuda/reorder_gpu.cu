// N-order relabelling on the device: HITS hub scores and degree order with
// ties by index (reference apply_reordering, src/generic.cu:1180-1376).
//
// HITS: T rounds over a strided sample of the nonzeros (every
// max(1, nnz / budget)-th); in each round every mode's score of index i is
// the sum, over the sampled nonzeros at i, of the product of the other
// modes' previous scores (modes ascending), then divided by the mode's
// maximum; indices are ranked by score descending, ties by index
// (src/generic.cu:1290-1341).  The reference sums sequentially in sample
// order, and a tie or a near-tie decides unit membership, so the device
// reproduces its bits: each mode's sample is sorted once by index with a
// stable sort (sample order kept within an index), the products are formed
// with round-to-nearest multiplies in mode order, and each index's products
// are added one after another by one thread (no reassociation, no fused
// multiply-add).  Only the ranking is order-independent (a stable sort on
// the score bits, descending, over indices in ascending order).
//
// Degree order with ties by index (the N-order path's CADR): integer
// histograms and the same stable descending sort.
#include <cub/cub.cuh>

#include <vector>

#include "kernels.hpp"

namespace cptc {

namespace {

struct IdxSet {
  const uint32_t* p[CPTC_MAX_ORDER];
};
struct ScoreSet {
  const double* p[CPTC_MAX_ORDER];
};

__global__ void k_sample_keys(const uint32_t* __restrict__ idx, uint64_t ns, uint64_t stride,
                              uint32_t* __restrict__ key, uint32_t* __restrict__ id) {
  for (uint64_t k = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; k < ns;
       k += (uint64_t)gridDim.x * blockDim.x) {
    key[k] = idx[k * stride];
    id[k] = (uint32_t)k;
  }
}

// prod[p] = product over q != m (ascending) of s_q[idx_q[e]], e the sample at
// sorted position p; each multiply rounded to nearest.
__global__ void k_hits_products(IdxSet idx, ScoreSet s, int N, int m, const uint32_t* __restrict__ ord,
                                uint64_t ns, uint64_t stride, double* __restrict__ prod) {
  for (uint64_t p = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; p < ns;
       p += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t e = (uint64_t)ord[p] * stride;
    double v = 1.0;
    for (int q = 0; q < N; ++q)
      if (q != m) v = __dmul_rn(v, s.p[q][idx.p[q][e]]);
    prod[p] = v;
  }
}

// One thread per index run: out[uidx[j]] = ((0 + prod[o]) + prod[o+1]) + ...
__global__ void k_hits_run_sums(const uint32_t* __restrict__ uidx, const uint32_t* __restrict__ off,
                                const uint32_t* __restrict__ cnt, uint64_t nruns,
                                const double* __restrict__ prod, double* __restrict__ out) {
  for (uint64_t j = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; j < nruns;
       j += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t o = off[j], n = cnt[j];
    double acc = 0.0;
    for (uint64_t p = 0; p < n; ++p) acc = __dadd_rn(acc, prod[o + p]);
    out[uidx[j]] = acc;
  }
}

__global__ void k_div_by_max(double* __restrict__ v, uint64_t n, const double* __restrict__ mx) {
  const double m = mx[0];
  if (!(m > 0.0)) return;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    v[i] = __ddiv_rn(v[i], m);
}

// Descending keys of non-negative doubles: the bit pattern inverted.
__global__ void k_desc_keys_f64(const double* __restrict__ v, uint64_t n,
                                unsigned long long* __restrict__ key, uint32_t* __restrict__ id) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    key[i] = ~(unsigned long long)__double_as_longlong(v[i]);
    id[i] = (uint32_t)i;
  }
}

__global__ void k_desc_keys_u32(const uint32_t* __restrict__ v, uint64_t n,
                                uint32_t* __restrict__ key, uint32_t* __restrict__ id) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    key[i] = ~v[i];
    id[i] = (uint32_t)i;
  }
}

__global__ void k_rank_of(const uint32_t* __restrict__ ord, uint64_t n, uint32_t* __restrict__ rank) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    rank[ord[i]] = (uint32_t)i;
}

__global__ void k_degrees(const uint32_t* __restrict__ idx, uint64_t n, uint32_t* __restrict__ deg) {
  for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < n;
       e += (uint64_t)gridDim.x * blockDim.x)
    atomicAdd(deg + idx[e], 1u);
}

__global__ void k_fill_f64(double* __restrict__ v, uint64_t n, double x) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    v[i] = x;
}

// Stable ascending sort of (key, index) pairs, then rank[index] = position.
template <class K>
void rank_from_keys(DArray<K>& key, DArray<uint32_t>& id, uint64_t n, int bits,
                    std::vector<uint32_t>& rank, cudaStream_t s) {
  DArray<K> key2(n);
  DArray<uint32_t> id2(n), rk(n);
  size_t tb = 0;
  CPTC_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, tb, key.p, key2.p, id.p, id2.p, (int64_t)n,
                                            0, bits, s));
  DArray<unsigned char> temp(tb);
  CPTC_CUDA(cub::DeviceRadixSort::SortPairs(temp.p, tb, key.p, key2.p, id.p, id2.p, (int64_t)n,
                                            0, bits, s));
  k_rank_of<<<grid_for(n, 256, 148 * 16), 256, 0, s>>>(id2.p, n, rk.p);
  CPTC_LAUNCH_CHECK();
  rank.assign(n, 0);
  CPTC_CUDA(cudaMemcpyAsync(rank.data(), rk.p, n * sizeof(uint32_t), cudaMemcpyDeviceToHost, s));
  CPTC_CUDA(cudaStreamSynchronize(s));
}

}  // namespace

void gpu_hits(Engine& E, int rounds, uint64_t budget, std::vector<std::vector<uint32_t>>& rank) {
  cudaStream_t s = E.stream;
  const int N = E.N;
  const uint64_t nnz = E.nnz;
  const uint64_t stride = (nnz > budget && budget > 0) ? (nnz / budget) : 1;
  const uint64_t ns = nnz ? (nnz + stride - 1) / stride : 0;
  IdxSet ip{};
  for (int m = 0; m < N; ++m) ip.p[m] = E.idx[m].p;
  DArray<double> sc[CPTC_MAX_ORDER], nx[CPTC_MAX_ORDER];
  for (int m = 0; m < N; ++m) {
    sc[m].alloc(E.dims[m]);
    nx[m].alloc(E.dims[m]);
    k_fill_f64<<<grid_for(E.dims[m], 256, 148 * 8), 256, 0, s>>>(sc[m].p, E.dims[m], 1.0);
    CPTC_LAUNCH_CHECK();
  }
  if (ns > 0 && rounds > 0) {
    // Per mode: the sample sorted by index (stable) and its index runs.
    DArray<uint32_t> ord[CPTC_MAX_ORDER], uidx[CPTC_MAX_ORDER], off[CPTC_MAX_ORDER],
        cnt[CPTC_MAX_ORDER];
    uint64_t nruns[CPTC_MAX_ORDER] = {0};
    {
      DArray<uint32_t> key(ns), key2(ns), id(ns);
      DArray<unsigned long long> nr(1);
      size_t tb = 0, rb = 0, sb = 0;
      CPTC_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, tb, key.p, key2.p, id.p, id.p,
                                                (int64_t)ns, 0, 32, s));
      CPTC_CUDA(cub::DeviceRunLengthEncode::Encode(nullptr, rb, key2.p, key.p, id.p, nr.p,
                                                   (int64_t)ns, s));
      CPTC_CUDA(cub::DeviceScan::ExclusiveSum(nullptr, sb, id.p, id.p, (int64_t)ns, s));
      DArray<unsigned char> temp(std::max(tb, std::max(rb, sb)));
      for (int m = 0; m < N; ++m) {
        ord[m].alloc(ns);
        k_sample_keys<<<grid_for(ns, 256, 148 * 16), 256, 0, s>>>(E.idx[m].p, ns, stride, key.p,
                                                                  id.p);
        CPTC_LAUNCH_CHECK();
        size_t t1 = temp.bytes();
        CPTC_CUDA(cub::DeviceRadixSort::SortPairs(temp.p, t1, key.p, key2.p, id.p, ord[m].p,
                                                  (int64_t)ns, 0, bits_for(E.dims[m]), s));
        uidx[m].alloc(ns);
        cnt[m].alloc(ns);
        size_t t2 = temp.bytes();
        CPTC_CUDA(cub::DeviceRunLengthEncode::Encode(temp.p, t2, key2.p, uidx[m].p, cnt[m].p, nr.p,
                                                     (int64_t)ns, s));
        unsigned long long h = 0;
        CPTC_CUDA(cudaMemcpyAsync(&h, nr.p, sizeof(h), cudaMemcpyDeviceToHost, s));
        CPTC_CUDA(cudaStreamSynchronize(s));
        nruns[m] = h;
        off[m].alloc(h);
        size_t t3 = temp.bytes();
        CPTC_CUDA(cub::DeviceScan::ExclusiveSum(temp.p, t3, cnt[m].p, off[m].p, (int64_t)h, s));
      }
    }
    DArray<double> prod(ns), mx(1);
    size_t xb = 0;
    CPTC_CUDA(cub::DeviceReduce::Max(nullptr, xb, nx[0].p, mx.p, (int64_t)E.dims[0], s));
    for (int m = 1; m < N; ++m) {
      size_t b = 0;
      CPTC_CUDA(cub::DeviceReduce::Max(nullptr, b, nx[m].p, mx.p, (int64_t)E.dims[m], s));
      xb = std::max(xb, b);
    }
    DArray<unsigned char> xtemp(xb);
    for (int it = 0; it < rounds; ++it) {
      ScoreSet sp{};
      for (int m = 0; m < N; ++m) sp.p[m] = sc[m].p;
      for (int m = 0; m < N; ++m) {
        CPTC_CUDA(cudaMemsetAsync(nx[m].p, 0, E.dims[m] * sizeof(double), s));
        k_hits_products<<<grid_for(ns, 256, 148 * 16), 256, 0, s>>>(ip, sp, N, m, ord[m].p, ns,
                                                                     stride, prod.p);
        CPTC_LAUNCH_CHECK();
        k_hits_run_sums<<<grid_for(nruns[m], 128, 148 * 16), 128, 0, s>>>(
            uidx[m].p, off[m].p, cnt[m].p, nruns[m], prod.p, nx[m].p);
        CPTC_LAUNCH_CHECK();
        size_t b = xtemp.bytes();
        CPTC_CUDA(cub::DeviceReduce::Max(xtemp.p, b, nx[m].p, mx.p, (int64_t)E.dims[m], s));
        k_div_by_max<<<grid_for(E.dims[m], 256, 148 * 8), 256, 0, s>>>(nx[m].p, E.dims[m], mx.p);
        CPTC_LAUNCH_CHECK();
      }
      for (int m = 0; m < N; ++m) std::swap(sc[m], nx[m]);
    }
  }
  rank.assign(N, {});
  for (int m = 0; m < N; ++m) {
    const uint64_t d = E.dims[m];
    DArray<unsigned long long> key(d);
    DArray<uint32_t> id(d);
    k_desc_keys_f64<<<grid_for(d, 256, 148 * 8), 256, 0, s>>>(sc[m].p, d, key.p, id.p);
    CPTC_LAUNCH_CHECK();
    rank_from_keys(key, id, d, 64, rank[m], s);
  }
}

void gpu_degree_rank(Engine& E, std::vector<std::vector<uint32_t>>& rank) {
  cudaStream_t s = E.stream;
  rank.assign(E.N, {});
  for (int m = 0; m < E.N; ++m) {
    const uint64_t d = E.dims[m];
    DArray<uint32_t> deg(d), key(d), id(d);
    CPTC_CUDA(cudaMemsetAsync(deg.p, 0, d * sizeof(uint32_t), s));
    k_degrees<<<grid_for(E.nnz, 256, 148 * 16), 256, 0, s>>>(E.idx[m].p, E.nnz, deg.p);
    CPTC_LAUNCH_CHECK();
    k_desc_keys_u32<<<grid_for(d, 256, 148 * 8), 256, 0, s>>>(deg.p, d, key.p, id.p);
    CPTC_LAUNCH_CHECK();
    rank_from_keys(key, id, d, 32, rank[m], s);
  }
}

}  // namespace cptc
