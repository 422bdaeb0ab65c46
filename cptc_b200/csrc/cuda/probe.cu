// Random-row gather bandwidth of this GPU: the ceiling of the FP64 sparse
// MTTKRP's factor-row gathers.
//
// The residual kernel reads, per nonzero, one row of the gathered mode's
// factor (8R bytes at a data-dependent row) and one row of the outer mode's
// factor (reused along a fiber, so mostly an L1 hit).  The factor matrices
// are a few MB (config 4 at R = 32: 2.3-7.4 MB), resident in the 126 MB L2,
// so the gathers are served by L2 rather than HBM and their rate is bounded
// by how many scattered row requests the SMs and L2 sustain, not by DRAM.
// This probe measures that bound with the same row layout as the kernel
// (a lane group per row, 16-byte vector loads, whole 32-byte sectors used)
// and no other work: uniformly random rows of an L2-resident matrix, many
// rows in flight per lane group, one double per thread written at the end.
//
// No counterpart in the reference (measurement only).
#include <cstdint>

#include "engine.hpp"
#include "kernels.hpp"

namespace cptc {

namespace {

__device__ __forceinline__ uint32_t hash32(uint64_t x) {
  uint32_t h = (uint32_t)x ^ (uint32_t)(x >> 32) * 0x9e3779b9u;
  h ^= h >> 16;
  h *= 0x7feb352du;
  h ^= h >> 15;
  h *= 0x846ca68bu;
  h ^= h >> 16;
  return h;
}

__global__ void k_fill_probe(double* __restrict__ F, uint64_t n) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    F[i] = 1.0 + (double)(i & 1023) * 1e-3;
}

// GW lanes per row, 2 * PAIRS doubles per lane (PAIRS 16-byte loads), U rows
// in flight per group; row q of the sequence is hash(q) mod rows.
template <int GW, int PAIRS, int U>
__global__ void __launch_bounds__(256) k_gather_probe(const double* __restrict__ F, uint64_t rows,
                                                      int R, uint64_t n, double* __restrict__ out) {
  constexpr int GPB = 256 / GW;
  const int glane = threadIdx.x % GW;
  const uint64_t group = (uint64_t)blockIdx.x * GPB + threadIdx.x / GW;
  const uint64_t ngroups = (uint64_t)gridDim.x * GPB;
  double acc = 0.0;
  for (uint64_t base = group * U; base < n; base += ngroups * U) {
    double2 v[U][PAIRS];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint64_t row = (base + u < n) ? hash32(base + u) % rows : 0;
      const double2* p = reinterpret_cast<const double2*>(F + row * (uint64_t)R);
#pragma unroll
      for (int k = 0; k < PAIRS; ++k) v[u][k] = __ldg(p + k * GW + glane);
    }
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int k = 0; k < PAIRS; ++k) acc += v[u][k].x + v[u][k].y;
  }
  out[(uint64_t)blockIdx.x * blockDim.x + threadIdx.x] = acc;
}

template <int GW, int PAIRS, int U>
float time_probe(const double* F, uint64_t rows, int R, uint64_t n, int reps, double* out,
                 unsigned blocks, cudaStream_t s) {
  cudaEvent_t e0, e1;
  CPTC_CUDA(cudaEventCreate(&e0));
  CPTC_CUDA(cudaEventCreate(&e1));
  k_gather_probe<GW, PAIRS, U><<<blocks, 256, 0, s>>>(F, rows, R, n, out);  // warm-up
  CPTC_LAUNCH_CHECK();
  CPTC_CUDA(cudaEventRecord(e0, s));
  for (int r = 0; r < reps; ++r) k_gather_probe<GW, PAIRS, U><<<blocks, 256, 0, s>>>(F, rows, R, n, out);
  CPTC_LAUNCH_CHECK();
  CPTC_CUDA(cudaEventRecord(e1, s));
  CPTC_CUDA(cudaEventSynchronize(e1));
  float ms = 0.f;
  CPTC_CUDA(cudaEventElapsedTime(&ms, e0, e1));
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  return ms / reps;
}

// Replay of the order-3 residual kernel's memory accesses: the same tasks
// (lane group = task of `tsize` records), the same records streamed, the
// same factor rows gathered with the same lane layout (the outer row only
// at fiber starts when FIB, as the kernel does at R >= 64), U records in
// flight per group and no arithmetic besides a running sum.
template <int GW, int PAIRS, int U, bool FIB>
__global__ void __launch_bounds__(256) k_gather_replay(const uint4* __restrict__ rec, uint64_t nnz,
                                                       uint64_t task0, uint64_t ntasks,
                                                       uint32_t tsize, int R,
                                                       const double* __restrict__ Fg,
                                                       const double* __restrict__ Fo,
                                                       double* __restrict__ out) {
  constexpr int GPW = 32 / GW;
  const int lane = threadIdx.x & 31, glane = lane % GW, gw = lane / GW;
  const int warp = threadIdx.x >> 5;
  const uint64_t task = task0 + ((uint64_t)blockIdx.x * 8 + warp) * GPW + gw;
  double acc = 0.0;
  if (task < ntasks) {
    const uint64_t p0 = task * (uint64_t)tsize;
    const uint64_t p1 = (p0 + tsize < nnz) ? p0 + tsize : nnz;
    for (uint64_t p = p0; p < p1; p += U) {
      uint4 e[U];
#pragma unroll
      for (int u = 0; u < U; ++u) e[u] = (p + u < p1) ? __ldcs(rec + p + u) : make_uint4(0, 0, 0, 0);
      double2 g[U][PAIRS], f[U][PAIRS];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const bool ok = p + u < p1;
        const double2* pg = reinterpret_cast<const double2*>(Fg + (uint64_t)(e[u].x & kIdxMask) * R);
        const double2* po = reinterpret_cast<const double2*>(Fo + (uint64_t)e[u].y * R);
        const bool lo = ok && (!FIB || (e[u].x & kFibFlag) || p + u == p0);
#pragma unroll
        for (int k = 0; k < PAIRS; ++k) {
          g[u][k] = ok ? __ldg(pg + k * GW + glane) : make_double2(0.0, 0.0);
          f[u][k] = lo ? __ldg(po + k * GW + glane) : make_double2(0.0, 0.0);
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int k = 0; k < PAIRS; ++k) acc += (g[u][k].x + g[u][k].y) + (f[u][k].x + f[u][k].y);
    }
  }
  out[(uint64_t)blockIdx.x * blockDim.x + threadIdx.x] = acc;
}

template <int GW, int PAIRS, int U, bool FIB>
float time_replay(const View& v, int R, const double* Fg, const double* Fo, int reps, double* out,
                  unsigned blocks, cudaEvent_t e0, cudaEvent_t e1, cudaStream_t s) {
  if (GW * PAIRS * 2 <= 32)  // the residual kernel's carveout at R <= 32
    CPTC_CUDA(cudaFuncSetAttribute(k_gather_replay<GW, PAIRS, U, FIB>,
                                   cudaFuncAttributePreferredSharedMemoryCarveout, 100));
  auto launch = [&] {
    k_gather_replay<GW, PAIRS, U, FIB><<<blocks, 256, 0, s>>>(v.rec.p, v.nnz, v.t0, v.t1, v.task,
                                                              R, Fg, Fo, out);
  };
  launch();  // warm-up
  CPTC_LAUNCH_CHECK();
  CPTC_CUDA(cudaEventRecord(e0, s));
  for (int r = 0; r < reps; ++r) launch();
  CPTC_LAUNCH_CHECK();
  CPTC_CUDA(cudaEventRecord(e1, s));
  CPTC_CUDA(cudaEventSynchronize(e1));
  float ms = 0.f;
  CPTC_CUDA(cudaEventElapsedTime(&ms, e0, e1));
  return ms / reps;
}

}  // namespace

// Fastest of a few depths (records in flight per lane group) of the replay
// of view `v`'s residual MTTKRP accesses; ms per launch.
double time_gather_replay(const View& v, int R, const double* Fg, const double* Fo, int reps,
                          cudaStream_t s) {
  CPTC_REQUIRE(v.rec.p != nullptr && v.recw == 1, CPTC_E_UNSUP,
               "the gather replay covers order-3 record views");
  CPTC_REQUIRE(R == 16 || R == 32 || R == 64 || R == 128, CPTC_E_UNSUP,
               "the gather replay covers R in {16, 32, 64, 128}");
  if (v.t1 <= v.t0) return 0.0;
  const int GW = R >= 64 ? (R == 64 ? 16 : 32) : R / 2;
  const int GPW = 32 / GW;
  const uint64_t warps = (v.t1 - v.t0 + GPW - 1) / GPW;
  const unsigned blocks = (unsigned)((warps + 7) / 8);
  DArray<double> out((uint64_t)blocks * 256);
  cudaEvent_t e0, e1;
  CPTC_CUDA(cudaEventCreate(&e0));
  CPTC_CUDA(cudaEventCreate(&e1));
  float best = 0.f;
  auto keep = [&](float ms) {
    if (best == 0.f || ms < best) best = ms;
  };
  switch (R) {
    case 16:
      keep(time_replay<8, 1, 2, false>(v, R, Fg, Fo, reps, out.p, blocks, e0, e1, s));
      keep(time_replay<8, 1, 4, false>(v, R, Fg, Fo, reps, out.p, blocks, e0, e1, s));
      keep(time_replay<8, 1, 8, false>(v, R, Fg, Fo, reps, out.p, blocks, e0, e1, s));
      break;
    case 32:
      keep(time_replay<16, 1, 2, false>(v, R, Fg, Fo, reps, out.p, blocks, e0, e1, s));
      keep(time_replay<16, 1, 4, false>(v, R, Fg, Fo, reps, out.p, blocks, e0, e1, s));
      keep(time_replay<16, 1, 8, false>(v, R, Fg, Fo, reps, out.p, blocks, e0, e1, s));
      break;
    case 64:
      keep(time_replay<16, 2, 1, true>(v, R, Fg, Fo, reps, out.p, blocks, e0, e1, s));
      keep(time_replay<16, 2, 2, true>(v, R, Fg, Fo, reps, out.p, blocks, e0, e1, s));
      keep(time_replay<16, 2, 4, true>(v, R, Fg, Fo, reps, out.p, blocks, e0, e1, s));
      break;
    default:
      keep(time_replay<32, 2, 1, true>(v, R, Fg, Fo, reps, out.p, blocks, e0, e1, s));
      keep(time_replay<32, 2, 2, true>(v, R, Fg, Fo, reps, out.p, blocks, e0, e1, s));
      keep(time_replay<32, 2, 4, true>(v, R, Fg, Fo, reps, out.p, blocks, e0, e1, s));
      break;
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  return best;
}

}  // namespace cptc

extern "C" int cptc_gather_peak(int device, uint64_t rows, int R, uint64_t n, int reps,
                                double* gbs) {
  using namespace cptc;
  try {
    CPTC_REQUIRE(rows > 0 && n > 0 && reps > 0 && gbs &&
                     (R == 16 || R == 32 || R == 64 || R == 128),
                 CPTC_E_ARG, "gather probe: rows, n, reps > 0 and R in {16, 32, 64, 128}");
    CPTC_CUDA(cudaSetDevice(device));
    int sms = 148;
    CPTC_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
    const unsigned blocks = (unsigned)sms * 8;
    struct Stream {
      cudaStream_t s = nullptr;
      ~Stream() {
        if (s) cudaStreamDestroy(s);
      }
    } st;
    CPTC_CUDA(cudaStreamCreateWithFlags(&st.s, cudaStreamNonBlocking));
    cudaStream_t s = st.s;
    DArray<double> F(rows * (uint64_t)R), out((uint64_t)blocks * 256);
    k_fill_probe<<<grid_for(rows * (uint64_t)R, 256, 148 * 8), 256, 0, s>>>(F.p, rows * (uint64_t)R);
    CPTC_LAUNCH_CHECK();
    float ms = 0.f;
    switch (R) {  // lane groups as in the residual kernel: R/2 lanes up to a warp
      case 16: ms = time_probe<8, 1, 8>(F.p, rows, R, n, reps, out.p, blocks, s); break;
      case 32: ms = time_probe<16, 1, 8>(F.p, rows, R, n, reps, out.p, blocks, s); break;
      case 64: ms = time_probe<16, 2, 4>(F.p, rows, R, n, reps, out.p, blocks, s); break;
      default: ms = time_probe<32, 2, 4>(F.p, rows, R, n, reps, out.p, blocks, s); break;
    }
    CPTC_CUDA(cudaStreamSynchronize(s));
    *gbs = (double)n * 8.0 * R / (ms * 1e-3) / 1e9;
    return CPTC_OK;
  } catch (const CptcError& e) {
    return e.code;
  } catch (...) {
    return CPTC_E_CUDA;
  }
}
