// Row-slab partition and NCCL collectives (see comm.hpp).
#include <nccl.h>

#include <cub/cub.cuh>

#include "comm.hpp"
#include "kernels.hpp"

namespace cptc {

namespace {

#define CPTC_NCCL(call)                                                           \
  do {                                                                            \
    ncclResult_t r_ = (call);                                                     \
    if (r_ != ncclSuccess)                                                        \
      throw CptcError(CPTC_E_COMM, std::string(#call " failed: ") + ncclGetErrorString(r_)); \
  } while (0)

inline ncclComm_t comm_of(const Engine& E) { return (ncclComm_t)E.nccl; }

__global__ void k_row_hist(const uint32_t* __restrict__ idx, uint64_t n, unsigned* __restrict__ h) {
  for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < n;
       e += (uint64_t)gridDim.x * blockDim.x)
    atomicAdd(h + idx[e], 1u);
}

}  // namespace

int comm_unique_id(unsigned char out[128]) {
  ncclUniqueId id;
  if (ncclGetUniqueId(&id) != ncclSuccess) return CPTC_E_COMM;
  static_assert(sizeof(id) == 128, "ncclUniqueId is 128 bytes");
  std::memcpy(out, &id, 128);
  return CPTC_OK;
}

void comm_init(Engine& E, const unsigned char idb[128], int rank, int nranks) {
  CPTC_REQUIRE(nranks >= 1 && rank >= 0 && rank < nranks, CPTC_E_ARG, "bad rank / nranks");
  CPTC_CUDA(cudaSetDevice(E.device));
  comm_destroy(E);
  if (nranks == 1) {
    E.nranks = 1;
    E.rank = 0;
    return;
  }
  ncclUniqueId id;
  std::memcpy(&id, idb, 128);
  ncclComm_t c = nullptr;
  CPTC_NCCL(ncclCommInitRank(&c, nranks, id, rank));
  E.nccl = (void*)c;
  E.nranks = nranks;
  E.rank = rank;
}

void comm_destroy(Engine& E) {
  if (E.nccl) {
    ncclCommDestroy(comm_of(E));
    E.nccl = nullptr;
  }
}

void comm_prepare(Engine& E) {
  for (int m = 0; m < E.N; ++m) E.slab[m].clear();
  if (E.nranks == 1) return;
  for (int m = 0; m < E.N; ++m) {
    DArray<unsigned> h(E.dims[m]);
    CPTC_CUDA(cudaMemsetAsync(h.p, 0, E.dims[m] * sizeof(unsigned), E.stream));
    k_row_hist<<<grid_for(E.nnz, 256, 148 * 16), 256, 0, E.stream>>>(E.idx[m].p, E.nnz, h.p);
    CPTC_LAUNCH_CHECK();
    std::vector<uint32_t> hh(E.dims[m]);
    CPTC_CUDA(cudaMemcpyAsync(hh.data(), h.p, E.dims[m] * sizeof(unsigned),
                              cudaMemcpyDeviceToHost, E.stream));
    CPTC_CUDA(cudaStreamSynchronize(E.stream));
    std::vector<uint64_t> cuts(E.nranks + 1, 0);
    CPTC_REQUIRE(cptc_slab_cuts(hh.data(), E.dims[m], E.nnz, E.nranks, cuts.data()) == 0,
                 CPTC_E_ARG, "slab cuts");
    E.slab[m] = cuts;
  }
}

void comm_allreduce_gram(Engine& E, int nblk) {
  if (E.nranks == 1) return;
  const int RR = E.R * E.R;
  if (E.comm_buf.n < (size_t)RR) E.comm_buf.alloc(RR);
  launch_partial_sum(E.gpart.p, nblk, RR, E.comm_buf.p, E.stream);
  CPTC_NCCL(ncclAllReduce(E.comm_buf.p, E.gpart.p, RR, ncclDouble, ncclSum, comm_of(E), E.stream));
}

int comm_gram_blocks(const Engine& E, int nblk) { return E.nranks == 1 ? nblk : 1; }

void comm_allreduce_dots(Engine& E, int nblk) {
  if (E.nranks == 1) return;
  if (E.comm_buf.n < (size_t)E.R * E.R) E.comm_buf.alloc((size_t)E.R * E.R);
  launch_partial_sum(E.dots.p, nblk, E.R, E.comm_buf.p, E.stream);
  CPTC_NCCL(ncclAllReduce(E.comm_buf.p, E.dots.p, E.R, ncclDouble, ncclSum, comm_of(E), E.stream));
}

int comm_dot_blocks(const Engine& E, int nblk) { return E.nranks == 1 ? nblk : 1; }

namespace {

struct InSlab {
  const uint32_t* idx;
  uint32_t lo, hi;
  __host__ __device__ bool operator()(uint32_t e) const {
    const uint32_t t = idx[e];
    return t >= lo && t < hi;
  }
};

struct TileInSlab {
  const int4* tile;
  int mode;
  int lo, hi;  // target block range
  __host__ __device__ bool operator()(uint32_t k) const {
    const int4 t = tile[k];
    const int b = mode == 0 ? t.x : mode == 1 ? t.y : t.z;
    return b >= lo && b < hi;
  }
};

}  // namespace

void slab_select(Engine& E, int n, const uint32_t* base, uint64_t nbase, DArray<uint32_t>& out,
                 uint64_t& nout) {
  InSlab pred{E.idx[n].p, (uint32_t)E.row_lo(n), (uint32_t)E.row_hi(n)};
  out.alloc(nbase);
  DArray<unsigned long long> cnt(1);
  size_t tb = 0;
  if (base) {
    CPTC_CUDA(cub::DeviceSelect::If(nullptr, tb, base, out.p, cnt.p, (int64_t)nbase, pred, E.stream));
    DArray<unsigned char> temp(tb);
    CPTC_CUDA(cub::DeviceSelect::If(temp.p, tb, base, out.p, cnt.p, (int64_t)nbase, pred, E.stream));
  } else {
    cub::CountingInputIterator<uint32_t> it(0);
    CPTC_CUDA(cub::DeviceSelect::If(nullptr, tb, it, out.p, cnt.p, (int64_t)nbase, pred, E.stream));
    DArray<unsigned char> temp(tb);
    CPTC_CUDA(cub::DeviceSelect::If(temp.p, tb, it, out.p, cnt.p, (int64_t)nbase, pred, E.stream));
  }
  unsigned long long h = 0;
  CPTC_CUDA(cudaMemcpyAsync(&h, cnt.p, sizeof(h), cudaMemcpyDeviceToHost, E.stream));
  CPTC_CUDA(cudaStreamSynchronize(E.stream));
  nout = h;
}

void slab_tiles(Engine& E) {
  UnitPool& U = E.units;
  for (int t = 0; t < 3; ++t) U.cnt[t] = U.nunits;
  if (E.nranks == 1 || U.nunits == 0) return;
  for (int t = 0; t < 3; ++t) {
    const int m = U.inner[t];
    TileInSlab pred{U.unit.p, t, (int)(E.row_lo(m) / 16), (int)((E.row_hi(m) + 15) / 16)};
    DArray<uint32_t> out(U.nunits);
    DArray<unsigned long long> cnt(1);
    size_t tb = 0;
    CPTC_CUDA(cub::DeviceSelect::If(nullptr, tb, U.order[t].p, out.p, cnt.p, (int64_t)U.nunits,
                                    pred, E.stream));
    DArray<unsigned char> temp(tb);
    CPTC_CUDA(cub::DeviceSelect::If(temp.p, tb, U.order[t].p, out.p, cnt.p, (int64_t)U.nunits,
                                    pred, E.stream));
    unsigned long long h = 0;
    CPTC_CUDA(cudaMemcpyAsync(&h, cnt.p, sizeof(h), cudaMemcpyDeviceToHost, E.stream));
    CPTC_CUDA(cudaStreamSynchronize(E.stream));
    U.order[t] = std::move(out);
    U.cnt[t] = h;
  }
}

static void allgather_rows(Engine& E, int n, double* base) {
  if (E.nranks == 1) return;
  const uint64_t R = (uint64_t)E.R;
  CPTC_NCCL(ncclGroupStart());
  for (int r = 0; r < E.nranks; ++r) {
    const uint64_t lo = E.slab[n][r], hi = E.slab[n][r + 1];
    if (hi <= lo) continue;
    CPTC_NCCL(ncclBroadcast(base + lo * R, base + lo * R, (hi - lo) * R, ncclDouble, r, comm_of(E),
                            E.stream));
  }
  CPTC_NCCL(ncclGroupEnd());
}

void comm_allgather_factor(Engine& E, int n) { allgather_rows(E, n, E.F[n].p); }

void comm_reduce_ftv(Engine& E, int n) { allgather_rows(E, n, E.FtV.p); }

}  // namespace cptc

extern "C" {

int cptc_comm_unique_id(unsigned char out_id[128]) {
  try {
    return cptc::comm_unique_id(out_id);
  } catch (...) {
    return CPTC_E_COMM;
  }
}

}  // extern "C"
