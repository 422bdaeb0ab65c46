// Multi-GPU plumbing of the engine: one process per GPU, NCCL over NVLink.
//
// Rows of every mode are owned in slabs and each rank holds only the
// nonzeros of its rows, plus an equal share of a heavy prefix of rows whose
// partial MTTKRPs are all-reduced (shard.cu).  A mode update then needs one
// NCCL all-reduce, over [the heavy prefix's partial MTTKRP | every rank's
// solved slab, each rank contributing its own rows and zeros elsewhere |
// Gram partial and fit dots].
#pragma once
#include "engine.hpp"

namespace cptc {

// Clears the MTTKRP partition (one rank: whole modes; shard_plan fills it).
void comm_prepare(Engine& E);
void comm_destroy(Engine& E);
void comm_init(Engine& E, const unsigned char id[128], int rank, int nranks);
int comm_unique_id(unsigned char out[128]);
// Rows per transfer slab of mode m for the sharded factor upload and
// read-back (slab r = rows [r * s, min((r + 1) * s, I_m)) of the caller's
// index space).
uint64_t slab_rows(const Engine& E, int m);

// Sums, in a fixed order over blocks, the nblk per-block Gram partials
// (R x R) and, when ndots >= 0, the ndots per-block column dot products (R,
// stored after the Gram).  One rank: into E.comm_buf.  Several ranks: into
// FtV's rows past I_n, then one all-reduce of FtV = [heavy prefix's partial
// MTTKRP | this rank's solved rows of F[n], zeros elsewhere | those sums],
// and rows [H, I_n) copied back into F[n].  Returns where the sums are.
double* comm_exchange_mode(Engine& E, int n, int nblk, int ndots);
// The full MTTKRP of mode n in every rank's FtV (one all-reduce: heavy
// prefix partials, own slab rows, zeros elsewhere).
void comm_reduce_ftv(Engine& E, int n);
// In place: every rank's transfer slab r of `base` (I_n rows padded to G
// slabs) gathered into every rank's copy.
void comm_allgather_rows(Engine& E, int n, double* base);
// Host values: out[r * count + i] = rank r's in[i], for every rank
// (synchronous; every rank calls it at the same point).
void comm_allgather_host(Engine& E, const double* in, int count, double* out);

}  // namespace cptc
