// Row-slab partition and NCCL collectives (see comm.hpp).
#include <nccl.h>

#include <algorithm>
#include <cstring>

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
  E.release_graph();  // it may hold NCCL calls on the old communicator
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

uint64_t slab_rows(const Engine& E, int m) {
  const uint64_t n = (uint64_t)E.nranks;
  return (E.dims[m] + n - 1) / n;
}

void comm_prepare(Engine& E) {
  for (int m = 0; m < E.N; ++m) {
    E.slab[m].clear();
    E.slab_blocks[m].clear();
    E.heavy_rows[m] = 0;
  }
}

namespace {

// The rows past the heavy prefix that this rank does not own, cleared: a
// row of `base` summed over the ranks then has one nonzero term, so its sum
// is the owner's values exactly (x + 0 = x) and every replica holds the same
// bits.
void clear_unowned(Engine& E, int n, double* base) {
  const uint64_t H = E.heavy_rows[n], I = E.dims[n], R = (uint64_t)E.R;
  const uint64_t lo = E.row_lo(n), hi = E.row_hi(n);
  if (I <= H) return;
  if (lo > H) CPTC_CUDA(cudaMemsetAsync(base + H * R, 0, (lo - H) * R * sizeof(double), E.stream));
  if (I > hi) CPTC_CUDA(cudaMemsetAsync(base + hi * R, 0, (I - hi) * R * sizeof(double), E.stream));
}

}  // namespace

// With several ranks the mode update's whole exchange is ONE all-reduce over
// FtV, whose rows are free once the own slab is solved:
//   rows [0, H)    the heavy prefix's partial MTTKRP (summed: the full rows),
//   rows [H, I)    this rank's solved slab rows, zeros elsewhere (summed:
//                  every rank's rows, exactly),
//   past row I     the Gram partial sum and fit dots (summed: the totals);
// then rows [H, I) are copied into F[n].  Against G in-place broadcasts of
// unequal slabs, which ran one after another, this cut mode 2's exchange
// on config 4 from 0.145 to 0.10 ms on 4 B200s (0.17 ms on 8 with the
// broadcasts); against three grouped all-reduces it measured the same.
double* comm_exchange_mode(Engine& E, int n, int nblk, int ndots) {
  const int RR = E.R * E.R;
  const uint64_t R = (uint64_t)E.R, I = E.dims[n], H = E.heavy_rows[n];
  double* out = E.nranks > 1 ? E.FtV.p + I * R : E.comm_buf.p;
  launch_partial_sum(E.gpart.p, nblk, RR, out, E.stream);
  if (ndots >= 0) launch_partial_sum(E.dots.p, ndots, E.R, out + RR, E.stream);
  if (E.nranks > 1) {
    const uint64_t lo = E.row_lo(n), hi = E.row_hi(n);
    if (hi > lo)
      CPTC_CUDA(cudaMemcpyAsync(E.FtV.p + lo * R, E.F[n].p + lo * R, (hi - lo) * R * sizeof(double),
                                cudaMemcpyDeviceToDevice, E.stream));
    clear_unowned(E, n, E.FtV.p);
    CPTC_NCCL(ncclAllReduce(E.FtV.p, E.FtV.p, I * R + RR + (ndots >= 0 ? R : 0), ncclDouble,
                            ncclSum, comm_of(E), E.stream));
    if (I > H)
      CPTC_CUDA(cudaMemcpyAsync(E.F[n].p + H * R, E.FtV.p + H * R, (I - H) * R * sizeof(double),
                                cudaMemcpyDeviceToDevice, E.stream));
  }
  return out;
}

void comm_reduce_ftv(Engine& E, int n) {
  if (E.nranks == 1) return;
  clear_unowned(E, n, E.FtV.p);
  CPTC_NCCL(ncclAllReduce(E.FtV.p, E.FtV.p, E.dims[n] * (uint64_t)E.R, ncclDouble, ncclSum,
                          comm_of(E), E.stream));
}

void comm_allgather_rows(Engine& E, int n, double* base) {
  if (E.nranks == 1) return;
  const uint64_t cnt = slab_rows(E, n) * (uint64_t)E.R;
  CPTC_NCCL(ncclAllGather(base + (uint64_t)E.rank * cnt, base, cnt, ncclDouble, comm_of(E),
                          E.stream));
}

void comm_allgather_host(Engine& E, const double* in, int count, double* out) {
  const int G = E.nranks;
  if (G == 1) {
    std::memcpy(out, in, sizeof(double) * count);
    return;
  }
  DArray<double> d(((size_t)G + 1) * count);
  CPTC_CUDA(cudaMemcpyAsync(d.p, in, sizeof(double) * count, cudaMemcpyHostToDevice, E.stream));
  CPTC_NCCL(ncclAllGather(d.p, d.p + count, count, ncclDouble, comm_of(E), E.stream));
  CPTC_CUDA(cudaMemcpyAsync(out, d.p + count, sizeof(double) * G * count, cudaMemcpyDeviceToHost,
                            E.stream));
  CPTC_CUDA(cudaStreamSynchronize(E.stream));
}

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
