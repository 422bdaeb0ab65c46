// Multi-GPU plumbing of the engine: one process per GPU, NCCL over NVLink.
//
// Rows of every mode are owned in slabs and each rank holds only the
// nonzeros of its rows, plus an equal share of a heavy prefix of rows whose
// partial MTTKRPs are all-reduced (shard.cu).  A mode update then needs one
// grouped NCCL call: the all-reduce of [Gram partial | fit dots], the
// all-reduce of the heavy prefix and the all-reduce that puts every rank's
// solved slab into every replica of the factor (each rank contributes its
// own rows and zeros elsewhere).
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
// stored after the Gram) into E.comm_buf; with several ranks, in one NCCL
// group, all-reduces that buffer and the heavy prefix of FtV and shares
// every rank's solved rows of F[n] with the others (its unowned rows past the
// prefix cleared, then one all-reduce of rows [H, I)).  Returns E.comm_buf.
double* comm_exchange_mode(Engine& E, int n, int nblk, int ndots);
// The full MTTKRP of mode n in every rank's FtV (heavy prefix all-reduced,
// slabs shared as in comm_exchange_mode).
void comm_reduce_ftv(Engine& E, int n);
// In place: every rank's transfer slab r of `base` (I_n rows padded to G
// slabs) gathered into every rank's copy.
void comm_allgather_rows(Engine& E, int n, double* base);
// Host values: out[r * count + i] = rank r's in[i], for every rank
// (synchronous; every rank calls it at the same point).
void comm_allgather_host(Engine& E, const double* in, int count, double* out);

}  // namespace cptc
