// Launch interfaces of the engine's kernels.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

#include "engine.hpp"

namespace cptc {

struct MttkrpArgs {
  const uint4* rec;  // records (null: the SoA arrays below): order 3 one
                     // uint4 {word, outer, value}; orders 4-6 two uint4
                     // {word, o0, o1, o2}{o3, 0, value}
  int recw;          // uint4 per record (1 or 2)
  const uint32_t* gw;
  const uint32_t* oidx;
  const double* val;
  const uint32_t* rows;
  const uint32_t* task_row;
  uint64_t nnz;
  uint64_t task0, ntasks;  // this launch walks tasks [task0, ntasks)
  uint32_t task;
  int nout, R;
  const double* Fg;
  const double* Fo[CPTC_MAX_ORDER];
  double* out;
};

void launch_mttkrp_view(const MttkrpArgs& a, cudaStream_t s);
// Lane groups the kernel launch_mttkrp_view picks for a view (records of
// recw uint4 or SoA arrays, nout outer modes, rank R) keeps resident on the
// whole of `device` at once.
uint64_t mttkrp_view_slots(bool rec, int recw, int nout, int R, int device);
// ms per launch of a gather-only replay of view v's order-3 residual MTTKRP
// accesses (probe.cu): the same records and factor rows, no arithmetic.
double time_gather_replay(const View& v, int R, const double* Fg, const double* Fo, int reps,
                          cudaStream_t s);

// Dense 16^3 tiles on the tensor cores: TF32 slabs with FP64 weighting.
// Slots 0,1,2 are the tile's three modes (order 3: modes 0,1,2; N-order
// units: the inner modes).  For target slot t the contraction runs over
// slot c in TF32 and each slab of slot s is weighted in FP64 by
// Fs[s-row, r] * prod_q Fout_q[outer_q, r].
struct TileArgs {
  const int4* tile;         // x,y,z = block coords of slots 0,1,2, w = count
  const uint64_t* start;
  const uint16_t* lid;      // (l0 << 8) | (l1 << 4) | l2
  const double* val;
  uint64_t ntiles;
  int R;
  int tslot, cslot, sslot;
  uint64_t dims[3];         // lengths of slots 0,1,2
  const double* Fc;
  const double* Fs;
  int nouter;
  const uint32_t* outer_idx;  // ntiles x nouter (tile-major), may be null
  const double* Fout[CPTC_MAX_ORDER];
  int store_dups;           // 1: last write wins (order-3), 0: duplicates sum
  double* out;
  int stage_max;  // nonzeros of the next tile staged ahead (0: none)
};
// order: tile visiting order for this mode (sorted by target block);
// cut: blocks+1 CTA range starts over `order` (balanced by nonzeros).
// N-order units (outer weights, duplicates summed).
void launch_mttkrp_tiles3(const TileArgs& a, const uint32_t* order, const uint32_t* cut,
                          uint32_t blocks, cudaStream_t s);

// Order-3 dense tiles from the packed word pool (UnitPool::words): the
// tiles of target slot `tslot` in visiting order (vtile, vstart), CTA
// ranges `cut` over that order.  Fct is the contracted factor as TF32 bit
// patterns, Fs the FP64 weighting factor.
struct Tile3Args {
  const int4* vtile;       // x,y,z = block coords of modes 0,1,2, w = count
  const uint32_t* vstart;  // first word of each tile (a multiple of 4)
  const uint32_t* words;   // TF32 value bits | (l0 << 8) | (l1 << 4) | l2
  uint64_t ntiles;
  int R;
  int tslot, cslot, sslot;
  uint64_t dims[3];
  const float* Fct;        // contracted factor in 16-row TF32 blocks (launch_to_tf32_blocks)
  const double* Fs;
  double* out;
};
void launch_tiles3w(const Tile3Args& a, const uint32_t* cut, uint32_t blocks, cudaStream_t s);
// CTAs of one launch of launch_tiles3w (waves of what the SMs hold at once).
uint32_t tile3w_blocks_for(int R, int device, uint64_t ntiles);
// The first `dim` rows of F (R columns) as TF32 bit patterns in 16-row
// blocks, each block rank-major with the tile kernel's column order; rows up
// to the next multiple of 16 are zero.  out holds ceil(dim/16)*16*R floats.
void launch_to_tf32_blocks(const double* F, uint64_t dim, int R, float* out, cudaStream_t s);
// Per-tile cost of launch_tiles3w in nonzero units (CTA range balancing).
unsigned long long tile3w_fixed_cost(int R);
// Order-3 pool packing (after partition_tiles3) and visit lists per slot.
void pack_tile_words(Engine& E);
void tile_visit_lists(Engine& E, int slot);
// Visit lists of `slot` from a visiting order of n tile indices.
void tile_visit_lists_from(Engine& E, int slot, const uint32_t* order, uint64_t n);
// CTAs the N-order unit kernel runs for rank R (occupancy x SMs, waves).
uint32_t tile_blocks_for(int R, int device, uint64_t ntiles);
// Balanced CTA ranges over E.units.order[slot] (fills E.units.cut[slot]),
// a tile weighing its nonzeros plus `fixed`.
void tile_cuts(Engine& E, int slot, unsigned long long fixed);
// Partition of Engine::tiles + residual selection (tiles.cu).
void partition_tiles3(Engine& E, double threshold, DArray<uint32_t>& sel, uint64_t& nsel);
// Device relabelling (reorder_gpu.cu): HITS scores with the reference's
// summation order, and degree order with ties by index; rank[m][old] = new.
void gpu_hits(Engine& E, int rounds, uint64_t budget, std::vector<std::vector<uint32_t>>& rank);
void gpu_degree_rank(Engine& E, std::vector<std::vector<uint32_t>>& rank);
// Row-slab sharding (shard.cu): the plan (E.slab, E.slab_blocks,
// E.heavy_rows) from the residual selection and the dense tiles; this rank's
// residual elements of target mode n (out; the selection or every nonzero
// when sel is null); this rank's tiles of a target slot in visiting order.
void shard_plan(Engine& E, const uint32_t* sel, uint64_t nsel);
// Times this rank's MTTKRP of every mode, gathers the times of all ranks and
// sets E.shard_speed / E.prev_blocks for the next shard_plan (every rank
// must call it at the same point).
void shard_calibrate(Engine& E);
uint64_t shard_select(Engine& E, int n, const uint32_t* sel, uint64_t nsel, DArray<uint32_t>& out);
uint64_t shard_tiles(Engine& E, int slot, DArray<uint32_t>& local_order);
// Copies the tiles listed in E.units.vtile/vstart[slot] into swords[slot]
// and points vstart[slot] into it.
void compact_slot_pool(Engine& E, int slot);
// Views (views.cu).
void build_view(Engine& E, View& v, int n, const uint32_t* d_sel, uint64_t nsel);

// N-order dense units (units.cu): partition over the inner modes with the
// outer modes fixed; fills E.units, returns residual selection.
void partition_units(Engine& E, double threshold, DArray<uint32_t>& sel, uint64_t& nsel);

// ---- ALS kernels (als_kernels.cu) ----
// Per-block partial Grams of F (rows x R) into part[nblk][R][R]; returns nblk.
int launch_gram_partial(const double* F, uint64_t rows, int R, double* part, int max_blocks,
                        cudaStream_t s);
// out[i] = sum_b part[b*len + i], i < len (fixed order).
void launch_partial_sum(const double* part, int nblk, int len, double* out, cudaStream_t s);
// out[i] += sum_b part[b*len + i], i < len (fixed order).
void launch_partial_sum_add(const double* part, int nblk, int len, double* out, cudaStream_t s);
// G = sum of nblk partials (fixed order).
void launch_gram_reduce(const double* part, int nblk, int R, double* G, cudaStream_t s);
// FtF = prod of the ng Grams Gs (elementwise, written out) and Ainv = its
// inverse; status[0] != 0 on non-finite results.  Ainv must hold
// 2*R*R + 1 doubles (scratch).
//   kInvPinv:      truncated pseudo-inverse (Jacobi, tol R*ulp(smax))
//   kInvCholRidge: ridge rule of the N-order reference path (sweep inverse)
//   kInvAuto:      sweep inverse when well conditioned, else the pseudo-inverse
enum { kInvPinv = 0, kInvCholRidge = 1, kInvAuto = 2 };
void launch_sym_inverse(const double* const* Gs, int ng, int R, int mode, double* FtF,
                        double* Ainv, int* status, cudaStream_t s);
// F[i,:] = (FtV[i,:] * Ainv) ./ (divide_lambda ? lambda : 1) for rows
// [0, rows); partial Grams of the written rows into part and, when dots is
// given, partials of the fit's column dots sum_i F[i,r] * FtV[i,r] into
// dots (nblk x R); returns nblk.
int launch_apply_solve(const double* FtV, const double* Ainv, const double* lambda,
                       int divide_lambda, uint64_t rows, int R, double* F, double* part,
                       int max_blocks, cudaStream_t s, double* dots = nullptr);
// From the Gram partials of the solved factor: column norms, new lambda and
// the Gram of the normalised factor; scale[r] = multiplier for column r.
//   generic_norm = 0: order-3 rule (norm < 1e-14 -> column 0, lambda 0,
//                     else lambda *= norm)
//   generic_norm = 1: N-order rule (norm < 1e-14 or non-finite -> 1,
//                     lambda = norm)
void launch_norm_finalize(const double* part, int nblk, int R, int generic_norm,
                          double* lambda, double* G, double* scale, cudaStream_t s);
void launch_scale_cols(double* F, uint64_t rows, int R, const double* scale, cudaStream_t s);
// out[0] = iprod = sum_r lambda_r dot_r (dot_r * scale[r] when scale is
// given), out[1] = model^2.
void launch_fit_final(const double* dot_part, int nblk, const double* scale, const double* lambda,
                      const double* const* Gs, int ng, int R, double* out, cudaStream_t s);
// part[b] = partial sums of (v - sum_r lambda_r prod_m F_m[i_m, r])^2.
struct ResidualArgs {
  const uint32_t* idx[CPTC_MAX_ORDER];
  const double* val;
  const double* F[CPTC_MAX_ORDER];
  const double* lambda;
  uint64_t nnz;
  int N, R;
};
void launch_residual(const ResidualArgs& a, double* part, int max_blocks, double* out,
                     cudaStream_t s);
// out[0] = sum v^2 (two-stage, deterministic).
void launch_sumsq(const double* v, uint64_t n, double* part, int max_blocks, double* out,
                  cudaStream_t s);

}  // namespace cptc
