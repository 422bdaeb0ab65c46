// Multi-GPU plumbing of the engine: one process per GPU, mode-n rows split
// into contiguous slabs of equal nonzero count, NCCL over NVLink for the two
// collectives of a mode update (Gram all-reduce, factor all-gather).
#pragma once
#include "engine.hpp"

namespace cptc {

// Computes the row slabs of every mode for this rank (single rank: whole
// modes).  Slab cuts are multiples of 16 so dense tiles have one owner.
void comm_prepare(Engine& E);
void comm_destroy(Engine& E);
void comm_init(Engine& E, const unsigned char id[128], int rank, int nranks);
int comm_unique_id(unsigned char out[128]);

// Sum of the per-block Gram partials over blocks and ranks into gpart[0];
// returns the number of partial blocks left for launch_norm_finalize.
void comm_allreduce_gram(Engine& E, int nblk);
int comm_gram_blocks(const Engine& E, int nblk);
void comm_allreduce_dots(Engine& E, int nblk);
int comm_dot_blocks(const Engine& E, int nblk);
// Every rank's slab of F[n] (or FtV) to every rank.
void comm_allgather_factor(Engine& E, int n);
void comm_reduce_ftv(Engine& E, int n);
// Elements of `base` (all when null) whose mode-n index lies in this rank's
// slab; and the per-mode tile lists restricted to this rank's row blocks.
void slab_select(Engine& E, int n, const uint32_t* base, uint64_t nbase, DArray<uint32_t>& out,
                 uint64_t& nout);
void slab_tiles(Engine& E);

}  // namespace cptc
