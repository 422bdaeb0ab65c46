// Multi-GPU plumbing of the engine: one process per GPU, NCCL over NVLink.
//
// Work and ownership are split separately.  The nonzeros of every mode are
// shared out by count: each rank walks an equal range of the view's
// nonzero-balanced tasks and an equal-weight range of the dense tiles, so a
// Zipf head row (or a 16-row block holding half of all nonzeros) is spread
// over all ranks.  Rows are owned in equal-size slabs: after the MTTKRP the
// partial results are reduce-scattered into the slabs, each rank solves and
// normalises its slab (Gram partials all-reduced), and the slabs are
// all-gathered into every rank's replica of the factor.
#pragma once
#include "engine.hpp"

namespace cptc {

// Row slabs of every mode (single rank: whole modes).
void comm_prepare(Engine& E);
void comm_destroy(Engine& E);
// Aborts the communicator (its unfinished collectives return) and drops it:
// cptc_comm_init has to run again before the next collective.
void comm_abort(Engine& E);
void comm_init(Engine& E, const unsigned char id[128], int rank, int nranks);
int comm_unique_id(unsigned char out[128]);
// Rows per slab of mode m (slab r = rows [r * s, min((r + 1) * s, I_m))).
uint64_t slab_rows(const Engine& E, int m);

// Sums, in a fixed order over blocks and ranks, the nblk per-block Gram
// partials (R x R) and, when ndots > 0, the ndots per-block column dot
// products (R, stored after the Gram); with several ranks the all-reduce is
// grouped with the all-gather of this rank's solved slab of F[n] into every
// rank's replica.  Returns the device address of the summed Gram.
const double* comm_reduce_gram_gather(Engine& E, int n, int nblk, int ndots);
// Partial MTTKRP rows of every rank summed into each rank's slab of FtV.
void comm_reduce_scatter_ftv(Engine& E, int n);
// The full reduced FtV on every rank (reduce-scatter + all-gather).
void comm_reduce_ftv(Engine& E, int n);
// In place: every rank's slab r of `base` (I_n rows padded to G slabs)
// gathered into every rank's copy.
void comm_allgather_rows(Engine& E, int n, double* base);

// Peer-memory exchange (peer.cu).  peer_map / peer_unmap are collective:
// map after the factor buffers are allocated, unmap before any of them is
// freed.  The two others replace comm_reduce_scatter_ftv and
// comm_reduce_gram_gather with the same results (sums in rank order).
void peer_map(Engine& E);
void peer_unmap(Engine& E);
void peer_reduce_scatter_ftv(Engine& E, int n);
const double* peer_reduce_gram_gather(Engine& E, int n, int nblk, int ndots);

}  // namespace cptc
