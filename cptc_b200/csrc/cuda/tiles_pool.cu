// Order-3 dense-tile MTTKRP from a packed word pool, pipelined through
// shared memory with cp.async.
//
// Reference numerics (dense_tile_mttkrp_wmma, src/dense.cu:339-1075): per
// tile and slab s of the weighting mode, P_s = X_s (16 x 16) * F_c block
// (16 x R) with TF32 operands and FP32 accumulation, then
// out[t, :] += double(P_s[t, :]) * F_s[s, :] in FP64.  The operands are the
// reference's: a value is clamped to +-FLT_MAX, cast to float and its low 13
// mantissa bits are ignored; a factor entry is cast to float, low bits
// ignored.
//
// B200 layout and schedule:
//  * the pool holds one 32-bit word per nonzero: the TF32 bit pattern of
//    its value, whose low 13 bits are zero, carries the 12-bit local id in
//    those bits, so a nonzero is 4 bytes (the reference's pool: 12) and the
//    kernel never converts a value; each tile's words start on a 16-byte
//    boundary.  The local coordinates are stored permuted, p = cpos(l) (the
//    order 0,4,8,12, 1,5,9,13, ...; cpos is its own inverse), which is the
//    order the shared-memory tile uses, and a tile's words are stored in a
//    strided order (element j at (a*j) mod count) so that the 32 nonzeros
//    a warp scatters at once are spread over the banks;
//  * per target mode the tiles are listed in visiting order (sorted by
//    target block) with their word offsets, so a CTA reads its tile list
//    as a contiguous stream;
//  * while the tensor cores work on tile k, the CTA copies tile k+1 into
//    the other half of a double buffer with cp.async (16 bytes per copy,
//    L2 only): its words, its 16 contracted-factor rows (TF32 bit patterns,
//    converted once per launch by k_to_tf32) and its 16 weighting-factor
//    rows (FP64); rows past the end of a mode are zero-filled by the copy;
//  * the tile is scattered into a zero tile in shared memory laid out per
//    mode as (s, t, c) in the permuted coordinates: a 16-float row per
//    (s, t), slabs 260 floats apart; the four A-fragment values a lane needs
//    from a row (columns t4, t4+4, t4+8, t4+12 of both k-steps) are then
//    one 16-byte load, bank-conflict free; the weighting rows are staged in
//    the permuted slab order and the 16 output rows are put back in order
//    when a target block is flushed; after the products the tile is zeroed
//    again by writing zero to the cells it set (or by clearing the whole
//    tile when it holds more nonzeros than the stage);
//  * the contracted factor is converted once per launch (k_to_tf32_blocks)
//    into 16-row blocks stored rank-major with the same column order, so a
//    lane's B-fragment values of one n-tile are one 16-byte load, and a
//    block is one contiguous copy (rows past the mode's end are zeros);
//  * warps are (n-tile group, slab group) pairs, an A fragment is loaded
//    once per warp and used for all of its n-tiles; FP64 results stay in
//    registers across the consecutive tiles of one target block and are
//    combined in shared memory (aliasing the zero tile) and added to the
//    output with FP64 atomics when the block changes.
// mma.sync rather than tcgen05: one slab product is 16 x 16 x R, far below
// tcgen05.mma's 64/128-row M, and the tile build bounds the kernel.
#include <cfloat>

#include <cub/cub.cuh>

#include "kernels.hpp"

namespace cptc {

namespace {

constexpr int kSt = 16;                // t stride (floats) of the slab layout
constexpr int kSs = 16 * kSt + 4;      // s stride: slabs 4 banks apart
constexpr int kTileFloats = 16 * kSs;  // 4160 floats = 16.25 KB

// Position of column c in a 16-float row: columns c, c+4, c+8, c+12 are
// adjacent, so the fragment values of lane t4 are one 16-byte chunk.
__host__ __device__ constexpr int cpos(int c) { return (c & 3) * 4 + (c >> 2); }
constexpr uint32_t kValMask = 0xFFFFE000u;

__device__ __forceinline__ uint32_t tf32_of(double v) {
  v = v > FLT_MAX ? FLT_MAX : (v < -FLT_MAX ? -FLT_MAX : v);
  return __float_as_uint((float)v) & kValMask;
}

__global__ void k_pad_counts(const int4* __restrict__ tile, uint64_t n, uint64_t* __restrict__ pc) {
  for (uint64_t k = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; k < n;
       k += (uint64_t)gridDim.x * blockDim.x)
    pc[k] = ((uint64_t)tile[k].w + 3) & ~3ull;
}

// One CTA per tile (grid-stride over tiles): the packed words of the tile's
// nonzeros at its padded offset, coordinates permuted (cpos), element j at
// position (a*j) mod cnt with a = 101 (103 when 101 divides cnt): a
// bijection, so every nonzero is stored once.
__global__ void k_pack_words(const int4* __restrict__ tile, const uint64_t* __restrict__ start,
                             const uint64_t* __restrict__ pst, const uint16_t* __restrict__ lid,
                             const double* __restrict__ val, uint64_t ntiles,
                             uint32_t* __restrict__ words, uint32_t* __restrict__ pst32) {
  for (uint64_t k = blockIdx.x; k < ntiles; k += gridDim.x) {
    const int cnt = tile[k].w;
    const uint64_t s0 = start[k], d0 = pst[k];
    const uint32_t a = (cnt % 101 == 0) ? 103u : 101u;
    for (int j = threadIdx.x; j < cnt; j += blockDim.x) {
      const uint32_t l = lid[s0 + j];
      const uint32_t pl = ((uint32_t)cpos((int)(l >> 8) & 15) << 8) |
                          ((uint32_t)cpos((int)(l >> 4) & 15) << 4) | (uint32_t)cpos((int)l & 15);
      words[d0 + (uint64_t)((a * (uint32_t)j) % (uint32_t)cnt)] = tf32_of(val[s0 + j]) | pl;
    }
    if (threadIdx.x == 0) pst32[k] = (uint32_t)d0;
  }
}

__global__ void k_visit(const uint32_t* __restrict__ order, const int4* __restrict__ tile,
                        const uint32_t* __restrict__ pst, uint64_t n, int4* __restrict__ vt,
                        uint32_t* __restrict__ vs) {
  for (uint64_t k = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; k < n;
       k += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t t = order[k];
    vt[k] = tile[t];
    vs[k] = pst[t];
  }
}

// Words of the listed tiles (visiting order) copied to consecutive padded
// offsets: dst[nst[k] + j] = src[vs[k] + j], j < padded count.
__global__ void k_copy_tile_words(const int4* __restrict__ vt, const uint32_t* __restrict__ vs,
                                  const uint64_t* __restrict__ nst, uint64_t n,
                                  const uint32_t* __restrict__ src, uint32_t* __restrict__ dst,
                                  uint32_t* __restrict__ vs_new) {
  for (uint64_t k = blockIdx.x; k < n; k += gridDim.x) {
    const int cnt = (vt[k].w + 3) & ~3;
    const uint64_t s0 = vs[k], d0 = nst[k];
    for (int j = threadIdx.x; j < cnt; j += blockDim.x) dst[d0 + j] = src[s0 + j];
    if (threadIdx.x == 0) vs_new[k] = (uint32_t)d0;
  }
}

// The contracted factor as TF32 bit patterns in 16-row blocks: block b holds
// rows 16b..16b+15 rank-major, out[b*16R + r*16 + cpos(c)] = F[16b + c, r],
// zero for rows past `dim`.  n = ceil(dim/16)*16*R entries.
__global__ void k_to_tf32_blocks(const double* __restrict__ F, uint64_t dim, int R, uint64_t n,
                                 float* __restrict__ out) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t row = i / (uint64_t)R;
    const int r = (int)(i - row * R);
    const uint64_t b = row >> 4;
    const int c = (int)(row & 15);
    const float v = row < dim ? (float)F[i] : 0.0f;
    out[b * 16 * (uint64_t)R + (uint64_t)r * 16 + cpos(c)] =
        __uint_as_float(__float_as_uint(v) & kValMask);
  }
}

__device__ __forceinline__ void cp16(void* sdst, const void* gsrc, bool ok) {
  const unsigned sa = (unsigned)__cvta_generic_to_shared(sdst);
  const int sz = ok ? 16 : 0;  // 0: nothing is read, 16 zero bytes are written
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(sa), "l"(gsrc), "r"(sz)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::: "memory"); }

__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <int SLOT>
__device__ __forceinline__ int blk(const int4& T) {
  return SLOT == 0 ? T.x : SLOT == 1 ? T.y : T.z;
}

// Bytes of one stage: words, the contracted-factor block (16 x R floats),
// the weighting-factor rows (16 x R doubles).
__host__ __device__ constexpr size_t stage_bytes(int capw, int R) {
  return (size_t)capw * 4 + (size_t)16 * R * 4 + (size_t)16 * R * 8;
}

// TS/CS/SS: target, contracted and weighting slots; NW: n-tiles (8 ranks
// each) per warp; CAPW: words staged per tile; MINB: resident CTAs per SM
// asked of the register allocator.
template <int TS, int CS, int SS, int NW, int CAPW, int MINB>
__global__ void __launch_bounds__(128, MINB) k_tiles3w(Tile3Args a, const uint32_t* __restrict__ cut) {
  constexpr int NTH = 128, WARPS = 4;
  extern __shared__ __align__(16) unsigned char smraw[];
  const int R = a.R;
  float* X = reinterpret_cast<float*>(smraw);
  double* accS = reinterpret_cast<double*>(smraw);  // 16 x R, only while X is all zero
  unsigned char* stg = smraw + (size_t)kTileFloats * 4;
  const size_t sb = stage_bytes(CAPW, R);
  auto s_words = [&](int b) { return reinterpret_cast<uint32_t*>(stg + b * sb); };
  auto s_fc = [&](int b) { return reinterpret_cast<float*>(stg + b * sb + CAPW * 4); };
  auto s_fs = [&](int b) {
    return reinterpret_cast<double*>(stg + b * sb + CAPW * 4 + (size_t)16 * R * 4);
  };
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t4 = lane & 3;
  const int NT = R >> 3;
  const int ng = (NT + NW - 1) / NW;  // n-tile groups (<= WARPS, checked by the launcher)
  const int SG = WARPS / ng;           // slab groups
  const bool active = warp < ng * SG;
  const int ntg = warp % ng, my_sg = warp / ng;
  const int nt_base = ntg * NW;
  const uint64_t dimT = a.dims[TS], dimC = a.dims[CS], dimS = a.dims[SS];
  // 16-byte chunks per weighting row (R/2); row = chunk / per-row by a
  // float reciprocal, exact for these sizes.
  const int cps = R >> 1;
  const float icps = 1.0f / (float)cps;

  const uint64_t k0 = cut[blockIdx.x], k1 = cut[blockIdx.x + 1];
  if (k0 >= k1) return;

  double acc[NW][4];
#pragma unroll
  for (int q = 0; q < NW; ++q)
#pragma unroll
    for (int x = 0; x < 4; ++x) acc[q][x] = 0.0;

  // Copies of tile T (word offset ws) into stage b; one commit group.
  auto issue = [&](int b, const int4& T, uint32_t ws) {
    const int nw = T.w < CAPW ? T.w : CAPW;
    uint32_t* dw = s_words(b);
    for (int q = tid; q < ((nw + 3) >> 2); q += NTH)
      cp16(dw + 4 * q, a.words + (uint64_t)ws + 4 * q, true);
    const uint64_t cb = (uint64_t)blk<CS>(T) * 16, sbk = (uint64_t)blk<SS>(T) * 16;
    float* dfc = s_fc(b);
    const float* sfc = a.Fct + cb * (uint64_t)R;  // block cb/16, padded with zero rows
    for (int q = tid; q < 4 * R; q += NTH) cp16(dfc + 4 * q, sfc + 4 * q, true);
    double* dfs = s_fs(b);
    for (int q = tid; q < 16 * cps; q += NTH) {
      const int row = (int)(((float)q + 0.5f) * icps), ch = q - row * cps;
      const uint64_t gr = sbk + row;
      const bool ok = gr < dimS;
      // stored at the tile's (permuted) slab position of this row
      cp16(dfs + cpos(row) * R + 2 * ch, a.Fs + (ok ? gr : 0) * (uint64_t)R + 2 * ch, ok);
    }
    cp_commit();
  };

  // Combines the slab groups' registers in shared memory (fixed order) and
  // adds the block's 16 rows to the output; X is all zero on entry and on
  // return.  Called by every thread at the same point.
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
    for (int t = warp; t < 16; t += WARPS) {
      const uint64_t row = (uint64_t)tb * 16 + cpos(t);  // stored row t holds row cpos(t)
      for (int r = lane; r < R; r += 32) {
        const double v = accS[t * R + r];
        if (row < dimT && v != 0.0) atomicAdd(a.out + row * (uint64_t)R + r, v);
        accS[t * R + r] = 0.0;
      }
    }
    __syncthreads();
  };

  auto cell = [&](uint32_t w) {
    const int l0 = (int)((w >> 8) & 15u), l1 = (int)((w >> 4) & 15u), l2 = (int)(w & 15u);
    const int lt = TS == 0 ? l0 : TS == 1 ? l1 : l2;
    const int lc = CS == 0 ? l0 : CS == 1 ? l1 : l2;
    const int ls = SS == 0 ? l0 : SS == 1 ? l1 : l2;
    return ls * kSs + lt * kSt + lc;  // the word's coordinates are already permuted
  };

  // Tile metadata two tiles ahead: T1 is the next tile, T2 the one after.
  int4 T1 = a.vtile[k0];
  uint32_t w1 = a.vstart[k0];
  int4 T2 = T1;
  uint32_t w2 = w1;
  if (k0 + 1 < k1) {
    T2 = a.vtile[k0 + 1];
    w2 = a.vstart[k0 + 1];
  }
  issue(0, T1, w1);
  // Shared memory starts undefined: the tile (and the flush buffer it
  // holds) is cleared once here, and after that by each tile's own cells.
  for (int i = tid; i < kTileFloats / 4; i += NTH)
    reinterpret_cast<float4*>(X)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  int cur_tb = -1;
#pragma unroll 1
  for (uint64_t k = k0; k < k1; ++k) {
    const int b = (int)((k - k0) & 1);
    const int4 T = T1;
    const uint32_t ws = w1;
    T1 = T2;
    w1 = w2;
    if (k + 2 < k1) {
      T2 = a.vtile[k + 2];
      w2 = a.vstart[k + 2];
    }
    cp_wait_all();    // this tile's stage (the only group in flight) has landed ...
    __syncthreads();  // ... for every thread; the previous tile's zeroing is visible
    if (k + 1 < k1) issue(b ^ 1, T1, w1);
    const int tb = blk<TS>(T);
    if (tb != cur_tb) {
      if (cur_tb >= 0) flush(cur_tb);
      cur_tb = tb;
    }
    // Scatter: staged words, then (tiles above CAPW) the rest from global.
    const uint32_t* sw = s_words(b);
    const int cnt = T.w;
#pragma unroll 4
    for (int j = tid; j < cnt; j += NTH) {
      const uint32_t w = j < CAPW ? sw[j] : __ldg(a.words + (uint64_t)ws + j);
      X[cell(w)] = __uint_as_float(w & kValMask);
    }
    __syncthreads();
    if (active) {
      const float* fc = s_fc(b);
      const double* fs = s_fs(b);
      uint32_t bf[NW][2][2];
#pragma unroll
      for (int q = 0; q < NW; ++q) {
        const int nt = nt_base + q;
        bf[q][0][0] = bf[q][0][1] = bf[q][1][0] = bf[q][1][1] = 0u;
        if (nt < NT) {
          // rows t4, t4+4 (k-step 0) and t4+8, t4+12 (k-step 1) of column
          // nt*8 + g of the contracted block
          const uint4 v = *reinterpret_cast<const uint4*>(fc + (nt * 8 + g) * 16 + 4 * t4);
          bf[q][0][0] = v.x;
          bf[q][0][1] = v.y;
          bf[q][1][0] = v.z;
          bf[q][1][1] = v.w;
        }
      }
#pragma unroll 2
      for (int s = my_sg; s < 16; s += SG) {
        // rows g and g+8 of slab s, columns t4, t4+4, t4+8, t4+12
        const uint4 lo = *reinterpret_cast<const uint4*>(X + s * kSs + g * kSt + 4 * t4);
        const uint4 hi = *reinterpret_cast<const uint4*>(X + s * kSs + (g + 8) * kSt + 4 * t4);
        const uint32_t af[2][4] = {{lo.x, hi.x, lo.y, hi.y}, {lo.z, hi.z, lo.w, hi.w}};
#pragma unroll
        for (int q = 0; q < NW; ++q) {
          const int nt = nt_base + q;
          if (nt >= NT) break;
          float d[4] = {0.f, 0.f, 0.f, 0.f};
          mma_tf32(d, af[0], bf[q][0][0], bf[q][0][1]);
          mma_tf32(d, af[1], bf[q][1][0], bf[q][1][1]);
          const double2 wv = *reinterpret_cast<const double2*>(fs + s * R + nt * 8 + 2 * t4);
          acc[q][0] = fma((double)d[0], wv.x, acc[q][0]);
          acc[q][1] = fma((double)d[1], wv.y, acc[q][1]);
          acc[q][2] = fma((double)d[2], wv.x, acc[q][2]);
          acc[q][3] = fma((double)d[3], wv.y, acc[q][3]);
        }
      }
    }
    __syncthreads();  // every read of X is done
    if (cnt <= CAPW) {
#pragma unroll 4
      for (int j = tid; j < cnt; j += NTH) X[cell(sw[j])] = 0.0f;
    } else {
      for (int i = tid; i < kTileFloats / 4; i += NTH)
        reinterpret_cast<float4*>(X)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  __syncthreads();
  flush(cur_tb);
}

// Launch shape per rank: n-tiles per warp, staged words per tile, resident
// CTAs per SM (registers and shared memory are sized for that many).
struct Shape {
  int nw, capw, minb;
};
Shape shape_for(int R) {
  const int NT = R / 8;
  const int nw = NT < 4 ? NT : 4;
  if (R <= 32) return {nw, 1024, 5};
  if (R <= 64) return {nw, 1024, 4};
  return {nw, 512, 3};
}

size_t smem_for(int R, int capw) { return (size_t)kTileFloats * 4 + 2 * stage_bytes(capw, R); }

template <int TS, int CS, int SS, int NW, int CAPW, int MINB>
void launch_one(const Tile3Args& a, const uint32_t* cut, uint32_t blocks, cudaStream_t s) {
  auto kern = k_tiles3w<TS, CS, SS, NW, CAPW, MINB>;
  const size_t smem = smem_for(a.R, CAPW);
  CPTC_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  CPTC_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
  kern<<<blocks, 128, smem, s>>>(a, cut);
}

template <int TS, int CS, int SS>
void launch_roles(const Tile3Args& a, const Shape& sh, const uint32_t* cut, uint32_t blocks,
                  cudaStream_t s) {
  if (sh.capw == 512) {
    launch_one<TS, CS, SS, 4, 512, 3>(a, cut, blocks, s);
  } else if (sh.minb == 4) {
    launch_one<TS, CS, SS, 4, 1024, 4>(a, cut, blocks, s);
  } else {
    switch (sh.nw) {
      case 1: launch_one<TS, CS, SS, 1, 1024, 5>(a, cut, blocks, s); break;
      case 2: launch_one<TS, CS, SS, 2, 1024, 5>(a, cut, blocks, s); break;
      case 3: launch_one<TS, CS, SS, 3, 1024, 5>(a, cut, blocks, s); break;
      default: launch_one<TS, CS, SS, 4, 1024, 5>(a, cut, blocks, s); break;
    }
  }
}

}  // namespace

// Packs the order-3 tile pool into words (UnitPool::words, pstart) and
// releases the separate local-id and value arrays.
void pack_tile_words(Engine& E) {
  UnitPool& P = E.units;
  cudaStream_t s = E.stream;
  const uint64_t n = P.nunits;
  if (n == 0) {
    P.words.alloc(4);
    P.pstart.alloc(1);
    return;
  }
  DArray<uint64_t> pc(n), pst(n);
  k_pad_counts<<<grid_for(n, 256, 148 * 16), 256, 0, s>>>(P.unit.p, n, pc.p);
  CPTC_LAUNCH_CHECK();
  size_t tb = 0;
  CPTC_CUDA(cub::DeviceScan::ExclusiveSum(nullptr, tb, pc.p, pst.p, (int64_t)n, s));
  DArray<unsigned char> temp(tb);
  CPTC_CUDA(cub::DeviceScan::ExclusiveSum(temp.p, tb, pc.p, pst.p, (int64_t)n, s));
  uint64_t last[2] = {0, 0};
  CPTC_CUDA(cudaMemcpyAsync(&last[0], pst.p + n - 1, 8, cudaMemcpyDeviceToHost, s));
  CPTC_CUDA(cudaMemcpyAsync(&last[1], pc.p + n - 1, 8, cudaMemcpyDeviceToHost, s));
  CPTC_CUDA(cudaStreamSynchronize(s));
  const uint64_t total = last[0] + last[1];
  CPTC_REQUIRE(total < (1ull << 32), CPTC_E_UNSUP, "dense tile pool above 2^32 words");
  for (int t = 0; t < 3; ++t) P.wcnt[t] = total;
  P.words.alloc(total + 4);
  CPTC_CUDA(cudaMemsetAsync(P.words.p, 0, (total + 4) * sizeof(uint32_t), s));
  P.pstart.alloc(n);
  k_pack_words<<<grid_for(n, 1, 148 * 32), 128, 0, s>>>(P.unit.p, P.start.p, pst.p, P.lid.p,
                                                          P.val.p, n, P.words.p, P.pstart.p);
  CPTC_LAUNCH_CHECK();
  CPTC_CUDA(cudaStreamSynchronize(s));
  P.lid.release();
  P.val.release();
}

// Tiles and word starts of target slot `slot` in a visiting order of n
// tile indices.
void tile_visit_lists_from(Engine& E, int slot, const uint32_t* order, uint64_t n) {
  UnitPool& P = E.units;
  P.vtile[slot].alloc(n);
  P.vstart[slot].alloc(n);
  if (n == 0) return;
  k_visit<<<grid_for(n, 256, 148 * 16), 256, 0, E.stream>>>(order, P.unit.p, P.pstart.p, n,
                                                            P.vtile[slot].p, P.vstart[slot].p);
  CPTC_LAUNCH_CHECK();
}

void tile_visit_lists(Engine& E, int slot) {
  tile_visit_lists_from(E, slot, E.units.order[slot].p, E.units.cnt[slot]);
}

void compact_slot_pool(Engine& E, int slot) {
  UnitPool& P = E.units;
  cudaStream_t s = E.stream;
  const uint64_t n = P.cnt[slot];
  if (n == 0) {
    P.swords[slot].alloc(4);
    P.wcnt[slot] = 0;
    return;
  }
  DArray<uint64_t> pc(n), nst(n);
  k_pad_counts<<<grid_for(n, 256, 148 * 16), 256, 0, s>>>(P.vtile[slot].p, n, pc.p);
  CPTC_LAUNCH_CHECK();
  size_t tb = 0;
  CPTC_CUDA(cub::DeviceScan::ExclusiveSum(nullptr, tb, pc.p, nst.p, (int64_t)n, s));
  DArray<unsigned char> temp(tb);
  CPTC_CUDA(cub::DeviceScan::ExclusiveSum(temp.p, tb, pc.p, nst.p, (int64_t)n, s));
  uint64_t last[2] = {0, 0};
  CPTC_CUDA(cudaMemcpyAsync(&last[0], nst.p + n - 1, 8, cudaMemcpyDeviceToHost, s));
  CPTC_CUDA(cudaMemcpyAsync(&last[1], pc.p + n - 1, 8, cudaMemcpyDeviceToHost, s));
  CPTC_CUDA(cudaStreamSynchronize(s));
  const uint64_t total = last[0] + last[1];
  P.wcnt[slot] = total;
  P.swords[slot].alloc(total + 4);
  CPTC_CUDA(cudaMemsetAsync(P.swords[slot].p, 0, (total + 4) * sizeof(uint32_t), s));
  DArray<uint32_t> vs_new(n);
  k_copy_tile_words<<<grid_for(n, 1, 148 * 32), 128, 0, s>>>(P.vtile[slot].p, P.vstart[slot].p,
                                                             nst.p, n, P.words.p,
                                                             P.swords[slot].p, vs_new.p);
  CPTC_LAUNCH_CHECK();
  CPTC_CUDA(cudaStreamSynchronize(s));
  P.vstart[slot] = std::move(vs_new);
}

// Per-tile cost of k_tiles3w in nonzero units, for balancing CTA ranges:
// the products and FP64 weighting of a tile (16 slabs x R/8 n-tiles x about
// 11 warp instructions, plus the A-fragment loads of each n-tile group)
// against about half a warp instruction per nonzero (scatter + clear).
unsigned long long tile3w_fixed_cost(int R) {
  const int NT = R / 8, ng = (NT + 3) / 4;
  return (unsigned long long)(44 * R + 256 * ng);
}

void launch_to_tf32_blocks(const double* F, uint64_t dim, int R, float* out, cudaStream_t s) {
  const uint64_t n = ((dim + 15) / 16) * 16 * (uint64_t)R;
  k_to_tf32_blocks<<<grid_for(n, 256, 148 * 8), 256, 0, s>>>(F, dim, R, n, out);
  CPTC_LAUNCH_CHECK();
}

uint32_t tile3w_blocks_for(int R, int device, uint64_t ntiles) {
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  const Shape sh = shape_for(R);
  const size_t smem = smem_for(R, sh.capw);
  int per_sm = 0;
  // every role and shape instance of a rank has the same resources
  auto kern = sh.capw == 512  ? k_tiles3w<0, 1, 2, 4, 512, 3>
              : sh.minb == 4  ? k_tiles3w<0, 1, 2, 4, 1024, 4>
              : sh.nw == 1    ? k_tiles3w<0, 1, 2, 1, 1024, 5>
              : sh.nw == 2    ? k_tiles3w<0, 1, 2, 2, 1024, 5>
              : sh.nw == 3    ? k_tiles3w<0, 1, 2, 3, 1024, 5>
                              : k_tiles3w<0, 1, 2, 4, 1024, 5>;
  CPTC_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  CPTC_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
  CPTC_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 128, smem));
  if (per_sm < 1) per_sm = 1;
  // Whole waves of resident CTAs, about 16 tiles per CTA, 1 to 8 waves: the
  // static CTA ranges are balanced by estimated cost, and several short
  // waves let the block scheduler even out what the estimate misses.
  const uint64_t wave = (uint64_t)sms * per_sm;
  uint64_t waves = ntiles / (wave * 16);
  if (waves < 1) waves = 1;
  if (waves > 8) waves = 8;
  return (uint32_t)(wave * waves);
}

void launch_tiles3w(const Tile3Args& a, const uint32_t* cut, uint32_t blocks, cudaStream_t s) {
  if (a.ntiles == 0) return;
  CPTC_REQUIRE(a.R % 8 == 0 && a.R >= 8 && a.R <= 128, CPTC_E_UNSUP,
               "the TF32 tile path needs R a multiple of 8, <= 128");
  const Shape sh = shape_for(a.R);
  const int NT = a.R / 8;
  CPTC_REQUIRE((NT + sh.nw - 1) / sh.nw <= 4, CPTC_E_UNSUP,
               "tile kernel shape: more n-tile groups than warps");
  const int roles = a.tslot * 100 + a.cslot * 10 + a.sslot;
  switch (roles) {
    case 12: launch_roles<0, 1, 2>(a, sh, cut, blocks, s); break;   // mode 0
    case 102: launch_roles<1, 0, 2>(a, sh, cut, blocks, s); break;  // mode 1
    case 201: launch_roles<2, 0, 1>(a, sh, cut, blocks, s); break;  // mode 2
    default: throw CptcError(CPTC_E_ARG, "unsupported order-3 tile roles");
  }
  CPTC_LAUNCH_CHECK();
}

}  // namespace cptc
