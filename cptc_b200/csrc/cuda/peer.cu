// Peer-memory exchange of a multi-GPU mode update (opt-in, cptc_opts.exchange
// = CPTC_EXCHANGE_PEER; the default exchange is the NCCL collectives of
// comm.cu).  Same row slabs, same work split, same arithmetic; only the two
// exchanges of a mode update change:
//
//   reduce-scatter  every rank stores each owner's slab rows of its partial
//                   MTTKRP into that owner's receive buffer (region `rank`)
//                   right after its MTTKRP; one barrier; each owner sums the
//                   G partials of its slab in rank order 0..G-1;
//   all-reduce +    every rank stores its solved slab rows into every peer's
//   all-gather      replica of the factor and its Gram (+ fit dot) partial
//                   sums into slot `rank` of every peer's slot area; one
//                   barrier; each rank sums the G slots in rank order.
//
// Sums run in a fixed rank order, so every rank computes the same bits.  The
// data moves as plain stores over NVLink (no TMA, no multicast).  A barrier is
// one CTA: it stores an epoch into flag `rank` of every peer with release
// semantics at system scope, then waits with acquire loads until all peers'
// flags reach the epoch.  Every wait is bounded (default 5 s of
// %globaltimer, plus an iteration cap); a wait that runs out sets bit
// kStatusPeerTimeout of the status word the host reads after each iteration
// and marks the exchange broken, after which later barriers return at once.
//
// Buffers are shared with CUDA IPC: the handles are all-gathered with NCCL
// when the build maps them (the all-gather also orders every rank's zeroed
// flags before any signal), and teardown closes them, then holds an NCCL
// barrier before anything exported is freed.
#include <nccl.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "comm.hpp"
#include "kernels.hpp"

namespace cptc {

namespace {

#define CPTC_NCCL_P(call)                                                         \
  do {                                                                            \
    ncclResult_t r_ = (call);                                                     \
    if (r_ != ncclSuccess)                                                        \
      throw CptcError(CPTC_E_COMM, std::string(#call " failed: ") + ncclGetErrorString(r_)); \
  } while (0)

constexpr uint64_t kArenaHeader = 128;  // flags (kMaxPeers u32) | epoch, broken (u32)
constexpr uint64_t kCtlOffset = 64;

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
  return t;
}

struct BarrierArgs {
  uint32_t* flags[kMaxPeers];  // every rank's flag array; entry q is written by rank q
  uint32_t* ctl;               // own: ctl[0] epoch, ctl[1] broken
  int* status;
  int rank, G;
  unsigned long long timeout_ns;
  unsigned long long max_spins;
};

// Entry i of a kernel-parameter pointer table without indexing the
// parameter space dynamically (which would copy the table to local memory).
template <typename T>
__device__ __forceinline__ T* pick(T* const (&tab)[kMaxPeers], int i) {
  T* r = nullptr;
#pragma unroll
  for (int q = 0; q < kMaxPeers; ++q)
    if (q == i) r = tab[q];
  return r;
}

// One CTA of 32 threads; thread t signals rank t and waits for rank t.
__global__ void __launch_bounds__(32) k_peer_barrier(BarrierArgs a) {
  __shared__ uint32_t s_epoch;
  __shared__ int s_skip;
  const int t = threadIdx.x;
  if (t == 0) {
    s_skip = a.ctl[1] != 0u;
    s_epoch = a.ctl[0] + 1u;
    if (!s_skip) a.ctl[0] = s_epoch;
  }
  __syncthreads();
  if (s_skip) return;
  const uint32_t e = s_epoch;
  // This GPU's earlier writes (earlier kernels of the stream, the peer
  // stores among them) are ordered before the signal.
  __threadfence_system();
  if (t < a.G) st_release_sys(pick(a.flags, t) + a.rank, e);
  if (t < a.G && t != a.rank) {
    const uint32_t* f = pick(a.flags, a.rank) + t;
    const unsigned long long t0 = global_ns();
    unsigned ns = 32;
    unsigned long long spins = 0;
    while ((int)(ld_acquire_sys(f) - e) < 0) {
      ++spins;
      if (spins > a.max_spins || global_ns() - t0 > a.timeout_ns) {
        atomicOr(a.status, kStatusPeerTimeout);
        atomicExch(a.ctl + 1, 1u);
        break;
      }
      __nanosleep(ns);
      if (ns < 1024) ns <<= 1;
    }
  }
}

struct PushArgs {
  const double* src;          // own partial MTTKRP (all padded rows)
  double* recv[kMaxPeers];    // every rank's receive buffer
  uint64_t per;               // elements of one slab (slab rows x R)
  uint64_t lo, hi;            // elements this rank's share can write: [lo, hi)
  int rank;
};

// blockIdx.y = owner o; the part of owner o's slab that this rank's share can
// have written (its touched rows) goes to region `rank` of o's receive
// buffer, at the same offsets.  The owner's own slab is summed in place.
template <bool VEC>
__global__ void __launch_bounds__(256) k_peer_push(PushArgs a) {
  const int o = blockIdx.y;
  if (o == a.rank) return;
  const uint64_t s0 = (uint64_t)o * a.per;
  const uint64_t b = a.lo > s0 ? a.lo : s0;
  const uint64_t e = a.hi < s0 + a.per ? a.hi : s0 + a.per;
  if (b < e) {
    const double* s = a.src + b;
    double* d = pick(a.recv, o) + (uint64_t)a.rank * a.per + (b - s0);
    const uint64_t n = e - b;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    if (VEC) {  // b and n even: 16-byte aligned on both sides
      const double2* s2 = reinterpret_cast<const double2*>(s);
      double2* d2 = reinterpret_cast<double2*>(d);
      for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n / 2; i += stride)
        d2[i] = s2[i];
    } else {
      for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += stride)
        d[i] = s[i];
    }
  }
  __threadfence_system();  // the stores reach the peer before the barrier's signal
}

struct SlabSumArgs {
  double* own;                 // own slab of FtV
  const double* recv;          // own receive buffer
  uint64_t per;
  uint64_t lo[kMaxPeers];      // rank r's region holds data in [lo[r], hi[r]) (slab offsets)
  uint64_t hi[kMaxPeers];
  int rank, G;
};

// own[i] = sum over r = 0..G-1 (rank order) of rank r's partial of this slab;
// outside rank r's touched rows its partial is zero and is not read.
__global__ void __launch_bounds__(256) k_peer_slab_sum(SlabSumArgs a) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < a.per; i += stride) {
    double s = 0.0;
#pragma unroll
    for (int r = 0; r < kMaxPeers; ++r) {
      if (r < a.G) {
        if (r == a.rank) s += a.own[i];
        else if (i >= a.lo[r] && i < a.hi[r]) s += a.recv[(uint64_t)r * a.per + i];
        else s += 0.0;  // the zero a full-slab copy would have added
      }
    }
    a.own[i] = s;
  }
}

struct PublishArgs {
  const double* slab;          // own solved rows (F[n] + rank * per)
  double* F[kMaxPeers];        // every rank's F[n]
  const double* part;          // own partial sums: Gram (R x R) [+ R dots]
  double* slots[kMaxPeers];    // every rank's slot area
  uint64_t per;
  int len, slot_stride, rank;
};

// blockIdx.y = destination rank q: the solved slab into q's replica (q !=
// rank) and the partial sums into q's slot `rank` (every q).
template <bool VEC>
__global__ void __launch_bounds__(256) k_peer_publish(PublishArgs a) {
  const int q = blockIdx.y;
  const uint64_t tid = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  if (tid < (uint64_t)a.len) pick(a.slots, q)[(uint64_t)a.rank * a.slot_stride + tid] = a.part[tid];
  if (q == a.rank) return;
  double* d = pick(a.F, q) + (uint64_t)a.rank * a.per;
  if (VEC) {
    const uint64_t n2 = a.per >> 1;
    const double2* s2 = reinterpret_cast<const double2*>(a.slab);
    double2* d2 = reinterpret_cast<double2*>(d);
    for (uint64_t i = tid; i < n2; i += stride) d2[i] = s2[i];
  } else {
    for (uint64_t i = tid; i < a.per; i += stride) d[i] = a.slab[i];
  }
  __threadfence_system();
}

// out[i] = sum over r = 0..G-1 (rank order) of slot r.
__global__ void __launch_bounds__(256) k_peer_slot_sum(const double* __restrict__ slots,
                                                       int slot_stride, int len, int G,
                                                       double* __restrict__ out) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < len; i += gridDim.x * blockDim.x) {
    double s = 0.0;
    for (int r = 0; r < G; ++r) s += slots[(uint64_t)r * slot_stride + i];
    out[i] = s;
  }
}

inline ncclComm_t comm_of(const Engine& E) { return (ncclComm_t)E.nccl; }

uint32_t* flags_of(unsigned char* arena) { return reinterpret_cast<uint32_t*>(arena); }
double* slots_of(unsigned char* arena) {
  return reinterpret_cast<double*>(arena + kArenaHeader);
}

unsigned long long timeout_ns_from_env() {
  if (const char* e = std::getenv("CPTC_PEER_TIMEOUT_MS")) {
    const long long ms = std::atoll(e);
    if (ms > 0) return (unsigned long long)ms * 1000000ull;
  }
  return 5000000000ull;
}

void launch_barrier(Engine& E) {
  PeerState& P = E.peer;
  BarrierArgs a{};
  for (int q = 0; q < P.G; ++q) a.flags[q] = flags_of(P.arena_of[q]);
  a.ctl = reinterpret_cast<uint32_t*>(P.arena.p + kCtlOffset);
  a.status = E.status.p;
  a.rank = E.rank;
  a.G = P.G;
  a.timeout_ns = P.timeout_ns;
  // __nanosleep backs off to 1 us: the cap is above the time limit's spins
  a.max_spins = P.timeout_ns / 256ull + 1000000ull;
  k_peer_barrier<<<1, 32, 0, E.stream>>>(a);
  CPTC_LAUNCH_CHECK();
}

unsigned copy_grid(uint64_t n) {
  uint64_t g = (n + 255) / 256;
  if (g < 1) g = 1;
  if (g > 148 * 4) g = 148 * 4;
  return (unsigned)g;
}

}  // namespace

// Rows [lo, hi) of mode n that this rank's share of the MTTKRP can write:
// the rows of its residual tasks and the target blocks of its dense tiles
// (both visited in row order), as one hull.
static void touched_rows(Engine& E, int n, uint64_t& lo, uint64_t& hi) {
  lo = UINT64_MAX;
  hi = 0;
  auto get32 = [&](const uint32_t* p, uint64_t i) {
    uint32_t v = 0;
    CPTC_CUDA(cudaMemcpy(&v, p + i, sizeof(v), cudaMemcpyDeviceToHost));
    return v;
  };
  const View& v = E.views[n];
  if (v.nnz > 0 && v.t1 > v.t0) {
    const uint32_t first = get32(v.rows.p, get32(v.task_row.p, v.t0));
    // the row holding task t1's first element bounds task t1 - 1's last row
    const uint32_t last = v.t1 < v.ntasks ? get32(v.rows.p, get32(v.task_row.p, v.t1))
                                          : get32(v.rows.p, v.nrows - 1);
    lo = first;
    hi = (uint64_t)last + 1;
  }
  if (E.dense_active) {
    const UnitPool& U = E.units;
    for (int ts = 0; ts < 3; ++ts) {
      if (U.inner[ts] != n || U.cnt[ts] == 0) continue;
      const uint32_t k0 = get32(U.cut[ts].p, (uint64_t)E.rank * U.blocks);
      const uint32_t k1 = get32(U.cut[ts].p, (uint64_t)(E.rank + 1) * U.blocks);
      if (k1 <= k0) continue;
      int4 u0, u1;
      CPTC_CUDA(cudaMemcpy(&u0, U.unit.p + get32(U.order[ts].p, k0), sizeof(int4),
                           cudaMemcpyDeviceToHost));
      CPTC_CUDA(cudaMemcpy(&u1, U.unit.p + get32(U.order[ts].p, k1 - 1), sizeof(int4),
                           cudaMemcpyDeviceToHost));
      const int b0 = ts == 0 ? u0.x : ts == 1 ? u0.y : u0.z;
      const int b1 = ts == 0 ? u1.x : ts == 1 ? u1.y : u1.z;
      lo = std::min<uint64_t>(lo, (uint64_t)b0 * 16);
      hi = std::max<uint64_t>(hi, std::min<uint64_t>((uint64_t)b1 * 16 + 16, E.dims[n]));
    }
  }
  if (lo >= hi) lo = hi = 0;
}

void peer_map(Engine& E) {
  PeerState& P = E.peer;
  CPTC_REQUIRE(!P.on, CPTC_E_ARG, "peer buffers are already mapped");
  CPTC_REQUIRE(E.nranks >= 2 && E.nranks <= kMaxPeers && E.nccl, CPTC_E_UNSUP,
               "the peer exchange needs 2 to 8 ranks and an initialised communicator");
  CPTC_CUDA(cudaSetDevice(E.device));
  const int G = E.nranks;
  uint64_t max_per = 0;
  for (int m = 0; m < E.N; ++m) max_per = std::max<uint64_t>(max_per, slab_rows(E, m) * E.R);
  P.G = G;
  P.slot_stride = E.R * E.R + E.R;
  P.recv.alloc((uint64_t)G * max_per);
  const uint64_t arena_bytes = kArenaHeader + (uint64_t)G * P.slot_stride * sizeof(double);
  P.arena.alloc(arena_bytes);
  CPTC_CUDA(cudaMemsetAsync(P.arena.p, 0, arena_bytes, E.stream));
  P.timeout_ns = timeout_ns_from_env();

  // Handles of every exported buffer: F[0..N-1], the receive buffer, the arena.
  constexpr int kH = CPTC_MAX_ORDER + 2;
  struct Ex {
    cudaIpcMemHandle_t h[kH];
  };
  Ex mine{};
  for (int m = 0; m < E.N; ++m) CPTC_CUDA(cudaIpcGetMemHandle(&mine.h[m], E.F[m].p));
  CPTC_CUDA(cudaIpcGetMemHandle(&mine.h[CPTC_MAX_ORDER], P.recv.p));
  CPTC_CUDA(cudaIpcGetMemHandle(&mine.h[CPTC_MAX_ORDER + 1], P.arena.p));
  DArray<unsigned char> dex((uint64_t)G * sizeof(Ex));
  CPTC_CUDA(cudaMemcpyAsync(dex.p + (uint64_t)E.rank * sizeof(Ex), &mine, sizeof(Ex),
                            cudaMemcpyHostToDevice, E.stream));
  // In place; it completes on a rank only after every rank zeroed its arena
  // (stream order), so no signal can reach an arena before its zeroing.
  CPTC_NCCL_P(ncclAllGather(dex.p + (uint64_t)E.rank * sizeof(Ex), dex.p, sizeof(Ex), ncclChar,
                            comm_of(E), E.stream));
  std::vector<Ex> all(G);
  CPTC_CUDA(cudaMemcpyAsync(all.data(), dex.p, (uint64_t)G * sizeof(Ex), cudaMemcpyDeviceToHost,
                            E.stream));
  CPTC_CUDA(cudaStreamSynchronize(E.stream));

  // Every rank's touched rows per mode, so owners read only what was pushed.
  CPTC_CUDA(cudaStreamSynchronize(E.stream));
  std::vector<uint64_t> hl(2 * CPTC_MAX_ORDER, 0);
  for (int m = 0; m < E.N; ++m) touched_rows(E, m, hl[2 * m], hl[2 * m + 1]);
  DArray<uint64_t> dh((uint64_t)G * 2 * CPTC_MAX_ORDER);
  CPTC_CUDA(cudaMemcpyAsync(dh.p + (uint64_t)E.rank * 2 * CPTC_MAX_ORDER, hl.data(),
                            hl.size() * sizeof(uint64_t), cudaMemcpyHostToDevice, E.stream));
  CPTC_NCCL_P(ncclAllGather(dh.p + (uint64_t)E.rank * 2 * CPTC_MAX_ORDER, dh.p,
                            2 * CPTC_MAX_ORDER, ncclUint64, comm_of(E), E.stream));
  std::vector<uint64_t> allh((uint64_t)G * 2 * CPTC_MAX_ORDER);
  CPTC_CUDA(cudaMemcpyAsync(allh.data(), dh.p, allh.size() * sizeof(uint64_t),
                            cudaMemcpyDeviceToHost, E.stream));
  CPTC_CUDA(cudaStreamSynchronize(E.stream));
  for (int q = 0; q < G; ++q)
    for (int m = 0; m < E.N; ++m) {
      P.rows_lo[m][q] = allh[(uint64_t)q * 2 * CPTC_MAX_ORDER + 2 * m];
      P.rows_hi[m][q] = allh[(uint64_t)q * 2 * CPTC_MAX_ORDER + 2 * m + 1];
    }

  auto open = [&](const cudaIpcMemHandle_t& h) {
    void* p = nullptr;
    CPTC_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
    P.opened.push_back(p);
    return p;
  };
  try {
    for (int q = 0; q < G; ++q) {
      if (q == E.rank) {
        for (int m = 0; m < E.N; ++m) P.F_of[m][q] = E.F[m].p;
        P.recv_of[q] = P.recv.p;
        P.arena_of[q] = P.arena.p;
        continue;
      }
      for (int m = 0; m < E.N; ++m) P.F_of[m][q] = static_cast<double*>(open(all[q].h[m]));
      P.recv_of[q] = static_cast<double*>(open(all[q].h[CPTC_MAX_ORDER]));
      P.arena_of[q] = static_cast<unsigned char*>(open(all[q].h[CPTC_MAX_ORDER + 1]));
    }
  } catch (...) {
    for (void* p : P.opened) cudaIpcCloseMemHandle(p);
    P.opened.clear();
    throw;
  }
  P.on = true;
}

void peer_unmap(Engine& E) {
  PeerState& P = E.peer;
  if (!P.on) return;
  cudaSetDevice(E.device);
  cudaStreamSynchronize(E.stream);
  cudaStreamSynchronize(E.side);
  for (void* p : P.opened) cudaIpcCloseMemHandle(p);
  P.opened.clear();
  P.on = false;
  // Nothing exported may be freed before every rank has closed its mappings.
  if (E.nccl) {
    DArray<int> one(1);
    cudaMemsetAsync(one.p, 0, sizeof(int), E.stream);
    if (ncclAllReduce(one.p, one.p, 1, ncclInt, ncclSum, comm_of(E), E.stream) == ncclSuccess)
      cudaStreamSynchronize(E.stream);
  }
  P.recv.release();
  P.arena.release();
  std::memset(P.F_of, 0, sizeof(P.F_of));
  std::memset(P.recv_of, 0, sizeof(P.recv_of));
  std::memset(P.arena_of, 0, sizeof(P.arena_of));
}

void peer_reduce_scatter_ftv(Engine& E, int n) {
  PeerState& P = E.peer;
  const uint64_t R = (uint64_t)E.R;
  const uint64_t per = slab_rows(E, n) * R;
  PushArgs a{};
  a.src = E.FtV.p;
  for (int q = 0; q < P.G; ++q) a.recv[q] = P.recv_of[q];
  a.per = per;
  a.lo = P.rows_lo[n][E.rank] * R;
  a.hi = P.rows_hi[n][E.rank] * R;
  a.rank = E.rank;
  // even R: every slab, every row and so every copied range start on 16 bytes
  const bool vec = (R % 2) == 0;
  const uint64_t span = a.hi > a.lo ? a.hi - a.lo : 1;
  const dim3 grid(copy_grid(vec ? span / 2 : span), (unsigned)P.G);
  if (vec) k_peer_push<true><<<grid, 256, 0, E.stream>>>(a);
  else k_peer_push<false><<<grid, 256, 0, E.stream>>>(a);
  CPTC_LAUNCH_CHECK();
  launch_barrier(E);
  SlabSumArgs b{};
  b.own = E.FtV.p + (uint64_t)E.rank * per;
  b.recv = P.recv.p;
  b.per = per;
  const uint64_t s0 = (uint64_t)E.rank * per;
  for (int q = 0; q < P.G; ++q) {  // rank q's touched elements inside this slab
    const uint64_t lo = P.rows_lo[n][q] * R, hi = P.rows_hi[n][q] * R;
    b.lo[q] = lo > s0 ? std::min(lo - s0, per) : 0;
    b.hi[q] = hi > s0 ? std::min(hi - s0, per) : 0;
  }
  b.rank = E.rank;
  b.G = P.G;
  k_peer_slab_sum<<<copy_grid(per), 256, 0, E.stream>>>(b);
  CPTC_LAUNCH_CHECK();
}

const double* peer_reduce_gram_gather(Engine& E, int n, int nblk, int ndots) {
  PeerState& P = E.peer;
  const int RR = E.R * E.R;
  double* out = E.comm_buf.p;
  launch_partial_sum(E.gpart.p, nblk, RR, out, E.stream);
  if (ndots > 0) launch_partial_sum(E.dots.p, ndots, E.R, out + RR, E.stream);
  const int len = RR + (ndots > 0 ? E.R : 0);
  const uint64_t per = slab_rows(E, n) * (uint64_t)E.R;
  PublishArgs a{};
  a.slab = E.F[n].p + (uint64_t)E.rank * per;
  for (int q = 0; q < P.G; ++q) {
    a.F[q] = P.F_of[n][q];
    a.slots[q] = slots_of(P.arena_of[q]);
  }
  a.part = out;
  a.per = per;
  a.len = len;
  a.slot_stride = P.slot_stride;
  a.rank = E.rank;
  const bool vec = (per % 2) == 0;
  uint64_t work = vec ? per / 2 : per;
  if (work < (uint64_t)len) work = (uint64_t)len;
  const dim3 grid(copy_grid(work), (unsigned)P.G);
  if (vec) k_peer_publish<true><<<grid, 256, 0, E.stream>>>(a);
  else k_peer_publish<false><<<grid, 256, 0, E.stream>>>(a);
  CPTC_LAUNCH_CHECK();
  launch_barrier(E);
  k_peer_slot_sum<<<(unsigned)((len + 255) / 256), 256, 0, E.stream>>>(
      slots_of(P.arena.p), P.slot_stride, len, P.G, out);
  CPTC_LAUNCH_CHECK();
  return out;
}

}  // namespace cptc
