// Order-3 hybrid partition into dense 16^3 tiles and an FP64 residual, and
// the dense-tile MTTKRP on the tensor cores (TF32 slabs, FP64 weighting).
//
// Partition: reference partition_tensor_hybrid_gpu (src/partition.cu:
// 581-1493).  Same tile ids, cutoff rule (count >= int(4096*thr), clamped to
// [1, 4096]; thr <= 0 auto-balance of :1030-1098) and classification, but
// the classification, offsets and scatter stay on the device (one readback
// of four scalars) instead of the reference's host classify loop.
//
// Dense-tile MTTKRP: reference dense_tile_mttkrp_wmma (src/dense.cu:89-1076).
// Per tile and slab s of the weighting mode, P = X_s (16 x 16) * F1_block
// (16 x R) in TF32 with FP32 accumulation, then out += double(P) * F2[s, :]
// in FP64 — the reference's numerics.  B200 mapping:
//  * mma.sync m16n8k8 TF32: a tile slab is a single 16x16x(R) product, far
//    below the 128-row M of tcgen05.mma, and the kernel is bound by loading
//    the tile pool and building the tile in shared memory, not by the
//    tensor pipe (ncu on config 4: tensor pipe ~10% active, issue- and
//    latency-bound while the tile is built);
//  * the tile is scattered into shared memory in a per-mode (s, t, c) layout
//    with a row stride of 20 floats, which makes every A-fragment load
//    bank-conflict free; F1 (TF32) and F2 (FP64) rows of the tile sit in
//    shared memory; B fragments stay in registers across the 16 slabs;
//  * tiles are visited in target-block order, so a CTA accumulates
//    consecutive tiles of the same 16 output rows in shared memory and
//    issues the FP64 atomics once per row block instead of once per tile.
#include <cfloat>
#include <cstdlib>
#include <cstring>

#include <cub/cub.cuh>

#include "kernels.hpp"

namespace cptc {

namespace {

__global__ void k_tile_keys(const uint32_t* __restrict__ i0, const uint32_t* __restrict__ i1,
                            const uint32_t* __restrict__ i2, uint64_t n, uint64_t nbj,
                            uint64_t nbk, uint64_t* __restrict__ key, uint32_t* __restrict__ id) {
  for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < n;
       e += (uint64_t)gridDim.x * blockDim.x) {
    key[e] = ((uint64_t)(i0[e] >> 4) * nbj + (i1[e] >> 4)) * nbk + (i2[e] >> 4);
    id[e] = (uint32_t)e;
  }
}

__global__ void k_run_start_flags(const uint64_t* __restrict__ key, uint64_t n,
                                  uint32_t* __restrict__ flag) {
  for (uint64_t p = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; p < n;
       p += (uint64_t)gridDim.x * blockDim.x)
    flag[p] = (p == 0 || key[p] != key[p - 1]) ? 1u : 0u;
}

// Per element in sorted order: dense flag from its run's count.
__global__ void k_elem_dense(const uint32_t* __restrict__ runid, const int* __restrict__ counts,
                             uint64_t n, int cutoff, uint32_t* __restrict__ dflag) {
  for (uint64_t p = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; p < n;
       p += (uint64_t)gridDim.x * blockDim.x)
    dflag[p] = counts[runid[p] - 1] >= cutoff ? 1u : 0u;
}

__global__ void k_scatter_split(const uint32_t* __restrict__ perm, const uint32_t* __restrict__ dflag,
                                const uint64_t* __restrict__ dpos, uint64_t n,
                                const uint32_t* __restrict__ i0, const uint32_t* __restrict__ i1,
                                const uint32_t* __restrict__ i2, const double* __restrict__ vals,
                                uint16_t* __restrict__ lid, double* __restrict__ pval,
                                uint32_t* __restrict__ sel) {
  for (uint64_t p = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; p < n;
       p += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t e = perm[p];
    if (dflag[p]) {
      const uint64_t d = dpos[p];
      lid[d] = (uint16_t)(((i0[e] & 15u) << 8) | ((i1[e] & 15u) << 4) | (i2[e] & 15u));
      pval[d] = vals[e];
    } else {
      sel[p - dpos[p]] = e;
    }
  }
}

__global__ void k_tiles_from_runs(const uint32_t* __restrict__ runs_sel, uint64_t ntiles,
                                  const uint64_t* __restrict__ ukeys, const int* __restrict__ counts,
                                  uint64_t nbj, uint64_t nbk, int4* __restrict__ tile,
                                  uint64_t* __restrict__ cnt64) {
  for (uint64_t k = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; k < ntiles;
       k += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t r = runs_sel[k];
    const uint64_t key = ukeys[r];
    const uint64_t bk = key % nbk, t = key / nbk, bj = t % nbj, bi = t / nbj;
    tile[k] = make_int4((int)bi, (int)bj, (int)bk, counts[r]);
    cnt64[k] = (uint64_t)counts[r];
  }
}

__global__ void k_run_dense_flags(const int* __restrict__ counts, uint64_t nruns, int cutoff,
                                  uint8_t* __restrict__ f) {
  for (uint64_t k = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; k < nruns;
       k += (uint64_t)gridDim.x * blockDim.x)
    f[k] = counts[k] >= cutoff ? 1 : 0;
}

// First index whose inclusive prefix reaches target (prefix is monotone).
__global__ void k_auto_cutoff(const unsigned long long* __restrict__ prefix,
                              const int* __restrict__ sorted_desc, uint64_t n,
                              unsigned long long target, int* __restrict__ out) {
  if (threadIdx.x || blockIdx.x) return;
  uint64_t lo = 0, hi = n;
  while (lo < hi) {
    const uint64_t mid = (lo + hi) >> 1;
    if (prefix[mid] >= target) hi = mid;
    else lo = mid + 1;
  }
  out[0] = (lo < n) ? sorted_desc[lo] : 1;
}

__global__ void k_tile_target_keys(const int4* __restrict__ tile, uint64_t n, int mode,
                                   uint32_t* __restrict__ key, uint32_t* __restrict__ id) {
  for (uint64_t k = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; k < n;
       k += (uint64_t)gridDim.x * blockDim.x) {
    const int4 t = tile[k];
    key[k] = (uint32_t)(mode == 0 ? t.x : mode == 1 ? t.y : t.z);
    id[k] = (uint32_t)k;
  }
}

// ---------------------------------------------------------------------------
// Dense-tile TF32 MTTKRP.
// ---------------------------------------------------------------------------
constexpr int kSt = 20;               // t stride (floats) of the slab layout
constexpr int kSs = 16 * kSt;         // s stride
constexpr int kTileFloats = 16 * kSs; // 5120 floats = 20 KB
constexpr int kScU = 4;               // nonzeros per thread per scatter round
constexpr int kStage = 1024;          // nonzeros of the next tile staged by cp.async

__device__ __forceinline__ void cp_async4(void* smem_dst, const void* gsrc) {
  const unsigned sa = (unsigned)__cvta_generic_to_shared(smem_dst);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(sa), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async8(void* smem_dst, const void* gsrc) {
  const unsigned sa = (unsigned)__cvta_generic_to_shared(smem_dst);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(sa), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_group 0;\n" ::: "memory");
}

__device__ __forceinline__ uint32_t tf32_bits(float x) {
  return __float_as_uint(x) & 0xFFFFE000u;  // low 13 mantissa bits ignored
}

__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Block of 4 warps, persistent over a contiguous range of the visiting
// order.  Slot roles (target TS, TF32-contracted CS, FP64-weighted SS) are
// compile-time constants.  The R/8 n-tiles (8 ranks each) are cut into
// ng = ceil(NT/NW) groups of NW; the 4 warps are (n-tile group, slab group)
// pairs, each slab group taking every SG-th of the 16 slabs (SG = 4/ng).  A
// warp loads an A fragment (a 16x8 piece of one slab) once and uses it for
// all NW of its n-tiles, so each slab is read ng times per tile (R=32: once).
// Per tile: zero + scatter the 16^3 tile in (s, t, c) layout as TF32 bit
// patterns, load the c-slot rows (TF32) and the s-slot rows times the outer
// weights (FP64), then per slab 2 k-steps of m16n8k8 and the FP64 epilogue.
// The FP64 results stay in registers across consecutive tiles of the same
// target block; when the block changes they are added into shared memory
// slab group by slab group (fixed order) and flushed with FP64 atomics.
// Row loops are (warp, lane)-strided: no integer division in the kernel.
template <int TS, int CS, int SS, int NW, int MINB>
__global__ void __launch_bounds__(128, MINB) k_tiles(TileArgs a,
                                                     const uint32_t* __restrict__ order,
                                                     const uint32_t* __restrict__ cut) {
  extern __shared__ __align__(16) unsigned char smraw[];
  const int R = a.R;
  const int Rs = R + 8;                                         // fB row stride (floats)
  float* X = reinterpret_cast<float*>(smraw);                  // kTileFloats (TF32)
  float* fB = X + kTileFloats;                                  // 16 * Rs (TF32)
  double* F2s = reinterpret_cast<double*>(fB + 16 * Rs);       // 16 * R
  double* accS = F2s + 16 * R;                                  // 16 * R
  double* wS = accS + 16 * R;                                   // R (outer weights)
  double* sv = wS + R;                                          // kStage staged values
  uint32_t* sl = reinterpret_cast<uint32_t*>(sv + kStage);     // staged local ids (words)
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t4 = lane & 3;
  const int NT = R >> 3;
  const int ng = (NT + NW - 1) / NW;
  const int SG = 4 / ng;
  const bool active = warp < ng * SG;
  const int ntg = warp % ng, my_sg = warp / ng;
  const int nt_base = ntg * NW;
  const uint64_t dimT = a.dims[TS], dimC = a.dims[CS], dimS = a.dims[SS];

  const uint64_t k0 = cut[blockIdx.x];
  const uint64_t k1 = cut[blockIdx.x + 1];
  if (k0 >= k1) return;

  for (int t = warp; t < 16; t += 4)
    for (int r = lane; r < R; r += 32) accS[t * R + r] = 0.0;
  double acc[NW][4];
#pragma unroll
  for (int q = 0; q < NW; ++q)
#pragma unroll
    for (int x = 0; x < 4; ++x) acc[q][x] = 0.0;
  int cur_tb = -1;

  // Called by all threads at the same point.
  auto flush = [&](int tb) {
    for (int sgi = 0; sgi < SG; ++sgi) {
      if (active && my_sg == sgi) {
#pragma unroll
        for (int q = 0; q < NW; ++q) {
          const int nt = nt_base + q;
          if (nt >= NT) break;
          const int r = nt * 8 + 2 * t4;
          accS[g * R + r] += acc[q][0];
          accS[g * R + r + 1] += acc[q][1];
          accS[(g + 8) * R + r] += acc[q][2];
          accS[(g + 8) * R + r + 1] += acc[q][3];
        }
      }
      __syncthreads();
    }
#pragma unroll
    for (int q = 0; q < NW; ++q)
#pragma unroll
      for (int x = 0; x < 4; ++x) acc[q][x] = 0.0;
    for (int t = warp; t < 16; t += 4) {
      const uint64_t row = (uint64_t)tb * 16 + t;
      for (int r = lane; r < R; r += 32) {
        const double v = accS[t * R + r];
        if (row < dimT && v != 0.0) atomicAdd(a.out + row * (uint64_t)R + r, v);
        accS[t * R + r] = 0.0;
      }
    }
  };

  // The first kStage nonzeros of a tile are copied into shared memory with
  // cp.async while the previous tile is on the tensor cores: values as
  // 8-byte copies, local ids as the aligned 4-byte words that hold them.
  auto stage = [&](uint64_t st, int cnt) {
    const int c = cnt < a.stage_max ? cnt : a.stage_max;
    const uint64_t w0 = st >> 1;
    const int nw = (int)(((st + (uint64_t)c + 1) >> 1) - w0);
    const uint32_t* lw = reinterpret_cast<const uint32_t*>(a.lid);
    for (int j = tid; j < nw; j += 128) cp_async4(sl + j, lw + w0 + j);
    for (int j = tid; j < c; j += 128) cp_async8(sv + j, a.val + st + j);
    cp_async_commit();
  };

  // Tile metadata is fetched one tile ahead (three dependent loads).
  uint32_t ti_next = order[k0];
  int4 T_next = a.tile[ti_next];
  uint64_t st_next = a.start[ti_next];
  stage(st_next, T_next.w);
  for (uint64_t k = k0; k < k1; ++k) {
    const uint32_t ti = ti_next;
    const int4 T = T_next;
    const uint64_t st = st_next;
    if (k + 1 < k1) {
      ti_next = order[k + 1];
      T_next = a.tile[ti_next];
      st_next = a.start[ti_next];
    }
    const int tb = TS == 0 ? T.x : TS == 1 ? T.y : T.z;
    const int cb = CS == 0 ? T.x : CS == 1 ? T.y : T.z;
    const int sb = SS == 0 ? T.x : SS == 1 ? T.y : T.z;
    __syncthreads();  // previous tile's shared-memory reads are done
    if (tb != cur_tb) {
      if (cur_tb >= 0) flush(cur_tb);
      cur_tb = tb;
    }
    for (int i = tid; i < kTileFloats / 4; i += 128)
      reinterpret_cast<float4*>(X)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (a.nouter > 0) {
      for (int r = tid; r < R; r += 128) {
        double w = 1.0;
        for (int q = 0; q < a.nouter; ++q)
          w *= a.Fout[q][(uint64_t)a.outer_idx[(uint64_t)ti * a.nouter + q] * R + r];
        wS[r] = w;
      }
    }
    cp_async_wait_all();  // this tile's staged nonzeros (own copies) ...
    __syncthreads();      // ... and everyone else's
    // Factor rows of the tile; every load of this thread is issued before
    // the first is used (the c loop is unrolled).
#pragma unroll
    for (int ci = 0; ci < 4; ++ci) {
      const int c = warp + 4 * ci;
      const uint64_t cg = (uint64_t)cb * 16 + c, sg = (uint64_t)sb * 16 + c;
      const bool cok = cg < dimC, sok = sg < dimS;
      for (int r = lane; r < R; r += 32) {
        fB[c * Rs + r] = cok ? __uint_as_float(tf32_bits((float)a.Fc[cg * R + r])) : 0.0f;
        double f2 = sok ? a.Fs[sg * R + r] : 0.0;
        if (a.nouter > 0) f2 *= wS[r];
        F2s[c * R + r] = f2;
      }
    }
    // Scatter of the tile's nonzeros, kScU per thread loaded at once.  Order-3
    // tiles store each cell once (duplicates: last write wins) and keep TF32
    // bit patterns; N-order units sum duplicates in FP32 and are truncated to
    // TF32 after the scatter.
    for (int j0 = 0; j0 < T.w; j0 += 128 * kScU) {
      uint32_t lq[kScU];
      double vq[kScU];
#pragma unroll
      for (int u = 0; u < kScU; ++u) {
        const int j = j0 + u * 128 + tid;
        if (j < T.w) {
          if (j < a.stage_max) {
            lq[u] = reinterpret_cast<const uint16_t*>(sl)[(st & 1) + j];
            vq[u] = sv[j];
          } else {
            lq[u] = a.lid[st + j];
            vq[u] = a.val[st + j];
          }
        }
      }
#pragma unroll
      for (int u = 0; u < kScU; ++u) {
        const int j = j0 + u * 128 + tid;
        if (j < T.w) {
          const uint32_t l = lq[u];
          const int l0 = (int)(l >> 8), l1 = (int)((l >> 4) & 15), l2 = (int)(l & 15);
          const int lt = TS == 0 ? l0 : TS == 1 ? l1 : l2;
          const int lc = CS == 0 ? l0 : CS == 1 ? l1 : l2;
          const int ls = SS == 0 ? l0 : SS == 1 ? l1 : l2;
          double v = vq[u];
          v = v > FLT_MAX ? FLT_MAX : (v < -FLT_MAX ? -FLT_MAX : v);
          float* dst = X + ls * kSs + lt * kSt + lc;
          if (a.store_dups) *dst = __uint_as_float(tf32_bits((float)v));
          else atomicAdd(dst, (float)v);
        }
      }
    }
    __syncthreads();
    if (!a.store_dups) {
      for (int i = tid; i < kTileFloats / 4; i += 128) {
        float4 x = reinterpret_cast<float4*>(X)[i];
        x.x = __uint_as_float(tf32_bits(x.x));
        x.y = __uint_as_float(tf32_bits(x.y));
        x.z = __uint_as_float(tf32_bits(x.z));
        x.w = __uint_as_float(tf32_bits(x.w));
        reinterpret_cast<float4*>(X)[i] = x;
      }
      __syncthreads();
    }
    // Everyone is past the scatter: the staging buffer takes the next tile.
    if (k + 1 < k1) stage(st_next, T_next.w);

    if (active) {
      uint32_t bf[NW][2][2];
#pragma unroll
      for (int q = 0; q < NW; ++q) {
        const int nt = nt_base + q;
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {
          bf[q][ks][0] = bf[q][ks][1] = 0u;
          if (nt < NT) {
            bf[q][ks][0] = __float_as_uint(fB[(ks * 8 + t4) * Rs + nt * 8 + g]);
            bf[q][ks][1] = __float_as_uint(fB[(ks * 8 + t4 + 4) * Rs + nt * 8 + g]);
          }
        }
      }
      for (int s = my_sg; s < 16; s += SG) {
        uint32_t af[2][4];
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {
          const float* base = X + s * kSs + ks * 8;
          af[ks][0] = __float_as_uint(base[g * kSt + t4]);
          af[ks][1] = __float_as_uint(base[(g + 8) * kSt + t4]);
          af[ks][2] = __float_as_uint(base[g * kSt + t4 + 4]);
          af[ks][3] = __float_as_uint(base[(g + 8) * kSt + t4 + 4]);
        }
#pragma unroll
        for (int q = 0; q < NW; ++q) {
          const int nt = nt_base + q;
          if (nt >= NT) break;
          float d[4] = {0.f, 0.f, 0.f, 0.f};
          mma_tf32(d, af[0], bf[q][0][0], bf[q][0][1]);
          mma_tf32(d, af[1], bf[q][1][0], bf[q][1][1]);
          const double2 w = *reinterpret_cast<const double2*>(F2s + s * R + nt * 8 + 2 * t4);
          acc[q][0] = fma((double)d[0], w.x, acc[q][0]);
          acc[q][1] = fma((double)d[1], w.y, acc[q][1]);
          acc[q][2] = fma((double)d[2], w.x, acc[q][2]);
          acc[q][3] = fma((double)d[3], w.y, acc[q][3]);
        }
      }
    }
  }
  __syncthreads();
  flush(cur_tb);
}

}  // namespace

// Builds the dense tile pool (tiles with >= cutoff nonzeros) and the list of
// residual elements.  Returns the residual selection in `sel` (device).
void partition_tiles3(Engine& E, double threshold, DArray<uint32_t>& sel, uint64_t& nsel) {
  cudaStream_t s = E.stream;
  const uint64_t n = E.nnz;
  const uint64_t nbj = (E.dims[1] + 15) / 16, nbk = (E.dims[2] + 15) / 16;
  UnitPool& P = E.units;
  P = UnitPool{};
  P.store_dups = true;
  const unsigned gb = grid_for(n, 256, 148 * 16);
  DArray<uint64_t> key_a(n), key_b(n);
  DArray<uint32_t> id_a(n), id_b(n);
  k_tile_keys<<<gb, 256, 0, s>>>(E.idx[0].p, E.idx[1].p, E.idx[2].p, n, nbj, nbk, key_a.p, id_a.p);
  CPTC_LAUNCH_CHECK();
  const int kbits = bits_for(((E.dims[0] + 15) / 16) * nbj * nbk);
  size_t tb = 0;
  CPTC_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, tb, key_a.p, key_b.p, id_a.p, id_b.p,
                                            (int64_t)n, 0, kbits, s));
  DArray<unsigned char> temp(tb);
  CPTC_CUDA(cub::DeviceRadixSort::SortPairs(temp.p, tb, key_a.p, key_b.p, id_a.p, id_b.p,
                                            (int64_t)n, 0, kbits, s));
  // Runs.
  DArray<uint64_t> ukeys(n);
  DArray<int> counts(n);
  DArray<unsigned long long> nruns_d(1);
  size_t rb = 0;
  CPTC_CUDA(cub::DeviceRunLengthEncode::Encode(nullptr, rb, key_b.p, ukeys.p, counts.p,
                                               nruns_d.p, (int64_t)n, s));
  if (rb > temp.bytes()) temp.alloc(rb);
  CPTC_CUDA(cub::DeviceRunLengthEncode::Encode(temp.p, rb, key_b.p, ukeys.p, counts.p,
                                               nruns_d.p, (int64_t)n, s));
  unsigned long long nruns = 0;
  CPTC_CUDA(cudaMemcpyAsync(&nruns, nruns_d.p, sizeof(nruns), cudaMemcpyDeviceToHost, s));
  CPTC_CUDA(cudaStreamSynchronize(s));

  // Cutoff.
  int cutoff;
  if (threshold > 0.0) {
    cutoff = (int)(4096.0 * threshold);
    if (cutoff < 1) cutoff = 1;
    if (cutoff > 4096) cutoff = 4096;
  } else {
    // Auto-balance of the reference: dense share rate_cuda/(rate_wmma +
    // rate_cuda) with its RTX 4060 rates scaled by SMs/24.
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, E.device);
    const double sm_scale = (double)sms / 24.0;
    const double rw = 1.20 / sm_scale, rc = 0.688 / sm_scale;
    const unsigned long long target = (unsigned long long)((double)n * (rc / (rw + rc)));
    DArray<int> cdesc(nruns);
    DArray<unsigned long long> pref(nruns);
    size_t sb = 0;
    CPTC_CUDA(cub::DeviceRadixSort::SortKeysDescending(nullptr, sb, counts.p, cdesc.p,
                                                       (int64_t)nruns, 0, 13, s));
    if (sb > temp.bytes()) temp.alloc(sb);
    CPTC_CUDA(cub::DeviceRadixSort::SortKeysDescending(temp.p, sb, counts.p, cdesc.p,
                                                       (int64_t)nruns, 0, 13, s));
    size_t scb = 0;
    auto conv = cub::TransformInputIterator<unsigned long long, cub::CastOp<unsigned long long>,
                                            const int*>(cdesc.p, cub::CastOp<unsigned long long>());
    CPTC_CUDA(cub::DeviceScan::InclusiveSum(nullptr, scb, conv, pref.p, (int64_t)nruns, s));
    if (scb > temp.bytes()) temp.alloc(scb);
    CPTC_CUDA(cub::DeviceScan::InclusiveSum(temp.p, scb, conv, pref.p, (int64_t)nruns, s));
    DArray<int> cut_d(1);
    k_auto_cutoff<<<1, 32, 0, s>>>(pref.p, cdesc.p, nruns, target, cut_d.p);
    CPTC_LAUNCH_CHECK();
    CPTC_CUDA(cudaMemcpyAsync(&cutoff, cut_d.p, sizeof(int), cudaMemcpyDeviceToHost, s));
    CPTC_CUDA(cudaStreamSynchronize(s));
  }
  E.cutoff = cutoff;

  // Per-element run id (1-based) and dense flag; dense positions by scan.
  DArray<uint32_t> flag(n), runid(n);
  k_run_start_flags<<<gb, 256, 0, s>>>(key_b.p, n, flag.p);
  CPTC_LAUNCH_CHECK();
  size_t sc = 0;
  CPTC_CUDA(cub::DeviceScan::InclusiveSum(nullptr, sc, flag.p, runid.p, (int64_t)n, s));
  if (sc > temp.bytes()) temp.alloc(sc);
  CPTC_CUDA(cub::DeviceScan::InclusiveSum(temp.p, sc, flag.p, runid.p, (int64_t)n, s));
  k_elem_dense<<<gb, 256, 0, s>>>(runid.p, counts.p, n, cutoff, flag.p);
  CPTC_LAUNCH_CHECK();
  DArray<uint64_t> dpos(n + 1);
  {
    auto conv = cub::TransformInputIterator<uint64_t, cub::CastOp<uint64_t>, const uint32_t*>(
        flag.p, cub::CastOp<uint64_t>());
    size_t eb = 0;
    CPTC_CUDA(cub::DeviceScan::ExclusiveSum(nullptr, eb, conv, dpos.p, (int64_t)n, s));
    if (eb > temp.bytes()) temp.alloc(eb);
    CPTC_CUDA(cub::DeviceScan::ExclusiveSum(temp.p, eb, conv, dpos.p, (int64_t)n, s));
  }
  uint64_t dense_nnz = 0;
  {
    uint64_t last_pos = 0;
    uint32_t last_flag = 0;
    CPTC_CUDA(cudaMemcpyAsync(&last_pos, dpos.p + (n - 1), sizeof(uint64_t),
                              cudaMemcpyDeviceToHost, s));
    CPTC_CUDA(cudaMemcpyAsync(&last_flag, flag.p + (n - 1), sizeof(uint32_t),
                              cudaMemcpyDeviceToHost, s));
    CPTC_CUDA(cudaStreamSynchronize(s));
    dense_nnz = last_pos + last_flag;
  }
  P.nnz = dense_nnz;
  nsel = n - dense_nnz;
  P.lid.alloc(dense_nnz + 8);  // the tile kernel copies whole 4-byte words
  P.val.alloc(dense_nnz);
  sel.alloc(nsel);
  k_scatter_split<<<gb, 256, 0, s>>>(id_b.p, flag.p, dpos.p, n, E.idx[0].p, E.idx[1].p,
                                     E.idx[2].p, E.vals.p, P.lid.p, P.val.p, sel.p);
  CPTC_LAUNCH_CHECK();

  // Dense tiles, in tile-id order.
  DArray<uint8_t> rflag(nruns);
  k_run_dense_flags<<<grid_for(nruns, 256, 148 * 16), 256, 0, s>>>(counts.p, nruns, cutoff,
                                                                   rflag.p);
  CPTC_LAUNCH_CHECK();
  DArray<uint32_t> rsel(nruns);
  DArray<unsigned long long> nt_d(1);
  cub::CountingInputIterator<uint32_t> cnt(0);
  size_t fb = 0;
  CPTC_CUDA(cub::DeviceSelect::Flagged(nullptr, fb, cnt, rflag.p, rsel.p, nt_d.p, (int64_t)nruns, s));
  if (fb > temp.bytes()) temp.alloc(fb);
  CPTC_CUDA(cub::DeviceSelect::Flagged(temp.p, fb, cnt, rflag.p, rsel.p, nt_d.p, (int64_t)nruns, s));
  unsigned long long ntiles = 0;
  CPTC_CUDA(cudaMemcpyAsync(&ntiles, nt_d.p, sizeof(ntiles), cudaMemcpyDeviceToHost, s));
  CPTC_CUDA(cudaStreamSynchronize(s));
  P.nunits = ntiles;
  P.unit.alloc(ntiles);
  P.start.alloc(ntiles);
  if (ntiles > 0) {
    DArray<uint64_t> c64(ntiles);
    k_tiles_from_runs<<<grid_for(ntiles, 256, 148 * 16), 256, 0, s>>>(rsel.p, ntiles, ukeys.p,
                                                                      counts.p, nbj, nbk,
                                                                      P.unit.p, c64.p);
    CPTC_LAUNCH_CHECK();
    size_t xb = 0;
    CPTC_CUDA(cub::DeviceScan::ExclusiveSum(nullptr, xb, c64.p, P.start.p, (int64_t)ntiles, s));
    if (xb > temp.bytes()) temp.alloc(xb);
    CPTC_CUDA(cub::DeviceScan::ExclusiveSum(temp.p, xb, c64.p, P.start.p, (int64_t)ntiles, s));
    // Per-mode visiting order: by target block (stable).  (The order-3 pool
    // is packed into words after this, pack_tile_words.)
    for (int m = 0; m < 3; ++m) {
      DArray<uint32_t> ka(ntiles), kb(ntiles), ia(ntiles);
      P.order[m].alloc(ntiles);
      k_tile_target_keys<<<grid_for(ntiles, 256, 148 * 16), 256, 0, s>>>(P.unit.p, ntiles, m,
                                                                          ka.p, ia.p);
      CPTC_LAUNCH_CHECK();
      size_t ob = 0;
      CPTC_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, ob, ka.p, kb.p, ia.p, P.order[m].p,
                                                (int64_t)ntiles, 0, 32, s));
      if (ob > temp.bytes()) temp.alloc(ob);
      CPTC_CUDA(cub::DeviceRadixSort::SortPairs(temp.p, ob, ka.p, kb.p, ia.p, P.order[m].p,
                                                (int64_t)ntiles, 0, 32, s));
    }
  }
  CPTC_CUDA(cudaStreamSynchronize(s));
  pack_tile_words(E);
}

namespace {

size_t tile_smem(int R) {
  return (size_t)kTileFloats * 4 + (size_t)16 * (R + 8) * 4 + (size_t)(2 * 16 * R + R) * 8 +
         (size_t)kStage * 8 + (size_t)(kStage / 2 + 2) * 4;
}

// Weight of a tile in the CTA (and rank) balance: its nonzeros plus a fixed
// cost for zeroing the tile and the 16 slab products, in nonzero units.
__global__ void k_tile_weights(const int4* __restrict__ tile, const uint32_t* __restrict__ order,
                               uint64_t n, unsigned long long fixed,
                               unsigned long long* __restrict__ w) {
  for (uint64_t k = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; k < n;
       k += (uint64_t)gridDim.x * blockDim.x)
    w[k] = (unsigned long long)tile[order[k]].w + fixed;
}

// cut[c] = first k whose inclusive prefix exceeds c * total / blocks.
__global__ void k_tile_cuts(const unsigned long long* __restrict__ pre, uint64_t n,
                            uint32_t blocks, uint32_t* __restrict__ cut) {
  const unsigned long long total = n ? pre[n - 1] : 0ull;
  for (uint32_t c = blockIdx.x * blockDim.x + threadIdx.x; c <= blocks;
       c += gridDim.x * blockDim.x) {
    if (c == 0) { cut[0] = 0; continue; }
    if (c == blocks) { cut[c] = (uint32_t)n; continue; }
    const unsigned long long target = (total * c) / blocks;
    uint64_t lo = 0, hi = n;  // first k with pre[k] > target
    while (lo < hi) {
      const uint64_t mid = (lo + hi) >> 1;
      if (pre[mid] <= target) lo = mid + 1;
      else hi = mid;
    }
    cut[c] = (uint32_t)lo;
  }
}

}  // namespace

// k_tiles splits the R/8 n-tiles into ceil(NT/NW) groups over its 4 warps;
// more than 4 groups would leave every warp without a slab group.
static void require_tile_shape(int R, int NW) {
  const int NT = R / 8;
  CPTC_REQUIRE(NW >= 1 && (NT + NW - 1) / NW <= 4, CPTC_E_UNSUP,
               "tile kernel shape: more n-tile groups than warps");
}

uint32_t tile_blocks_for(int R, int device, uint64_t ntiles) {
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  // A whole number of waves of the CTAs the SMs hold at once (registers
  // and shared memory both limit it; all role instances share the same
  // resources), about 16 tiles per CTA, 1 to 8 waves: the static CTA ranges
  // are balanced by nonzero count, and when tile costs vary (config 4's
  // Zipf tiles) several short waves let the block scheduler even out the
  // rest (config 4, R=32: 0.91 ms per mode at 1 wave, 0.70 at 8; config 2's
  // uniform tiles: 0.09 at 1 wave, 0.11 at 4).
  const size_t smem = tile_smem(R);
  const int NT = R / 8;
  const int ntm = NT < 4 ? NT : 4;
  auto kern = ntm == 1  ? k_tiles<0, 1, 2, 1, 4>
              : ntm == 2  ? k_tiles<0, 1, 2, 2, 4>
              : ntm == 3  ? k_tiles<0, 1, 2, 3, 4>
                          : k_tiles<0, 1, 2, 4, 4>;
  CPTC_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  CPTC_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
  int per_sm = 0;
  CPTC_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 128, smem));
  if (per_sm < 1) per_sm = 1;
  const uint64_t wave = (uint64_t)sms * per_sm;
  uint64_t waves = ntiles / (wave * 16);
  if (waves < 1) waves = 1;
  if (waves > 8) waves = 8;
  return (uint32_t)(wave * waves);
}

void tile_cuts(Engine& E, int slot, unsigned long long fixed) {
  UnitPool& U = E.units;
  const uint64_t n = U.cnt[slot];
  // `blocks` CTA ranges over this rank's visiting order (with several ranks
  // it lists only the rank's own tiles).
  const uint32_t total = U.blocks;
  U.cut[slot].alloc((uint64_t)total + 1);
  if (n == 0) {
    CPTC_CUDA(cudaMemsetAsync(U.cut[slot].p, 0, ((uint64_t)total + 1) * 4, E.stream));
    return;
  }
  DArray<unsigned long long> w(n), pre(n);
  k_tile_weights<<<grid_for(n, 256, 148 * 16), 256, 0, E.stream>>>(U.unit.p, U.order[slot].p, n,
                                                                   fixed, w.p);
  CPTC_LAUNCH_CHECK();
  size_t tb = 0;
  CPTC_CUDA(cub::DeviceScan::InclusiveSum(nullptr, tb, w.p, pre.p, (int64_t)n, E.stream));
  DArray<unsigned char> temp(tb);
  CPTC_CUDA(cub::DeviceScan::InclusiveSum(temp.p, tb, w.p, pre.p, (int64_t)n, E.stream));
  k_tile_cuts<<<grid_for((uint64_t)total + 1, 256), 256, 0, E.stream>>>(pre.p, n, total,
                                                                      U.cut[slot].p);
  CPTC_LAUNCH_CHECK();
  CPTC_CUDA(cudaStreamSynchronize(E.stream));
}

void launch_mttkrp_tiles3(const TileArgs& a_in, const uint32_t* order, const uint32_t* cut,
                          uint32_t blocks, cudaStream_t s) {
  TileArgs a = a_in;
  a.stage_max = kStage;
  if (a.ntiles == 0) return;
  CPTC_REQUIRE(a.R % 8 == 0 && a.R <= 128, CPTC_E_UNSUP,
               "the TF32 tile path needs R a multiple of 8, <= 128");
  const int R = a.R;
  const size_t smem = tile_smem(R);
  const int NT = R / 8;
  const int ntm = NT < 4 ? NT : 4;  // n-tiles per warp
  const int roles = a.tslot * 100 + a.cslot * 10 + a.sslot;
  // 4 resident CTAs per SM (<= 128 registers): measured against 5 (96
  // registers, spills at 4 n-tiles per warp) on config 4, 4 is faster.
#define CPTC_TILES(TS_, CS_, SS_, NTM, MINB_)                                              \
  do {                                                                                     \
    require_tile_shape(R, NTM);                                                            \
    auto kern = k_tiles<TS_, CS_, SS_, NTM, MINB_>;                                        \
    CPTC_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,      \
                                   (int)smem));                                            \
    CPTC_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,   \
                                   100));                                                  \
    kern<<<blocks, 128, smem, s>>>(a, order, cut);                                         \
  } while (0)
#define CPTC_TILES_R(TS_, CS_, SS_)                          \
  do {                                                       \
    if (ntm == 1) CPTC_TILES(TS_, CS_, SS_, 1, 4);           \
    else if (ntm == 2) CPTC_TILES(TS_, CS_, SS_, 2, 4);      \
    else if (ntm == 3) CPTC_TILES(TS_, CS_, SS_, 3, 4);      \
    else CPTC_TILES(TS_, CS_, SS_, 4, 4);                    \
  } while (0)
  switch (roles) {
    case 12: CPTC_TILES_R(0, 1, 2); break;   // order-3 mode 0; N-order slot 0
    case 102: CPTC_TILES_R(1, 0, 2); break;  // order-3 mode 1
    case 201: CPTC_TILES_R(2, 0, 1); break;  // order-3 mode 2
    case 120: CPTC_TILES_R(1, 2, 0); break;  // N-order slot 1 (slot 2 is 201)
    default: throw CptcError(CPTC_E_ARG, "unsupported tile slot roles");
  }
#undef CPTC_TILES_R
#undef CPTC_TILES
  CPTC_LAUNCH_CHECK();
}

}  // namespace cptc
