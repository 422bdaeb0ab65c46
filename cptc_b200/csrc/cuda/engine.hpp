// Engine state: the device-resident tensor, per-mode MTTKRP views, the dense
// 16^3 tile pool, factors and the ALS workspace.
#pragma once
#include <cuda_runtime.h>

#include <algorithm>
#include <string>
#include <vector>

#include "../../../include/cptc.h"
#include "common.cuh"

namespace cptc {

// Element word of a view: bits 0..29 gathered-mode index, bit 30 starts a
// fiber (a run of equal target and outer-mode indices), bit 31 starts a row.
constexpr uint32_t kRowFlag = 0x80000000u;
constexpr uint32_t kFibFlag = 0x40000000u;
constexpr uint32_t kIdxMask = 0x3FFFFFFFu;
constexpr uint64_t kMaxGatherDim = (1ull << 30);

// Nonzeros of one lane-group task in the sparse MTTKRP: at most 1024, and
// sized so that the tasks fill whole waves of the resident lane groups
// (`slots`): a view of nnz nonzeros runs in ceil(nnz / (1024 slots)) waves of
// equal tasks, so no wave is left almost empty (on 8 GPUs a rank with 5.1M
// residual nonzeros in 256-nonzero tasks ran 2.1 waves and took 35% longer
// than one with 4.6M); at least 64 nonzeros per task.
constexpr int kTask = 1024;
inline uint32_t task_size_for(uint64_t nnz, uint64_t slots) {
  if (slots == 0) slots = 148ull * 64;
  const uint64_t waves = (nnz + kTask * slots - 1) / (kTask * slots);
  uint64_t t = (nnz + waves * slots - 1) / (waves ? waves * slots : 1);
  if (t < 64) t = 64;
  if (t > (uint64_t)kTask) t = kTask;
  return (uint32_t)t;
}

// Sorted view of the nonzeros for one target mode, in the order
// (target, outer modes..., gathered mode).  The rows of the outer modes are
// reused along a fiber; the gathered mode's row is read per nonzero.
struct View {
  int target = -1;
  int nout = 0;                  // number of outer (fiber) modes
  int omode[CPTC_MAX_ORDER] = {0};  // outer modes then the gathered mode
  int gmode = -1;
  uint64_t nnz = 0;
  uint64_t fibers = 0;
  DArray<uint32_t> gw;           // element word (gathered index + flags)
  DArray<uint32_t> oidx;         // nout * nnz outer indices (SoA)
  DArray<double> val;
  // The same data as records: order 3 one 16-byte record per nonzero
  // {word, outer index, value} (x, y = word, outer; zw = value bits);
  // orders 4-6 two uint4 {word, o0, o1, o2} {o3, 0, value}.
  DArray<uint4> rec;
  int recw = 0;                  // uint4 per record (0: SoA arrays only)
  DArray<uint32_t> rows;         // non-empty target rows, in order
  DArray<uint32_t> task_row;     // index into `rows` of each task's first row
  uint64_t nrows = 0, ntasks = 0;
  uint32_t task = kTask;         // nonzeros per task
  uint64_t t0 = 0, t1 = 0;       // tasks [t0, t1) are this rank's share
};

// Dense 16^3 tiles: order 3 (inner = modes 0,1,2, no outer modes) or the
// N-order units (a tile over the inner modes with every outer mode fixed,
// src/generic.cu:406-561).  Elements of tiles with at least `cutoff`
// nonzeros, grouped by tile.
struct UnitPool {
  uint64_t nunits = 0, nnz = 0;
  int inner[3] = {0, 1, 2};
  int nouter = 0;
  int outer[CPTC_MAX_ORDER] = {0};
  bool store_dups = true;      // order-3 tiles store (last write wins)
  DArray<int4> unit;           // x,y,z tile block coords of the inner modes, w = count
  DArray<uint64_t> start;      // first element of each tile in the pool
  DArray<uint32_t> outer_idx;  // nunits x nouter (unit-major)
  DArray<uint16_t> lid;        // N-order units: (l0 << 8) | (l1 << 4) | l2
  DArray<double> val;          // N-order units: values
  // Order-3 tiles: one word per nonzero, the value as TF32 bits (sign,
  // exponent, top 10 mantissa bits) with the 12-bit local id in the low bits
  // the TF32 truncation clears; each tile's words start on a 16-byte
  // boundary (pstart, in words; the gap words are zero and never read as
  // nonzeros).
  DArray<uint32_t> words;
  DArray<uint32_t> pstart;
  // Per target slot, the tiles and their word starts in visiting order.
  DArray<int4> vtile[3];
  DArray<uint32_t> vstart[3];
  // Several ranks: each slot's own tiles copied into a pool of their own
  // (vstart[slot] then indexes swords[slot]); one rank: the shared pool.
  DArray<uint32_t> swords[3];
  DArray<uint32_t> order[3];   // visiting order per inner target slot
  uint64_t cnt[3] = {0, 0, 0}; // tiles per inner target slot
  uint64_t wcnt[3] = {0, 0, 0};  // words of those tiles (order 3, padded to 4 per tile)
  // CTA ranges over each visiting order with balanced estimated costs:
  // blocks + 1 cut points.
  DArray<uint32_t> cut[3];
  uint32_t blocks = 0;
};

// Default fill-rate threshold of the dense-tile path on B200 for rank R.
double b200_fill_min(int R);

struct Engine {
  int device = 0;
  cudaStream_t stream = nullptr;
  // Side stream for the R x R inverse of a mode update, which needs only the
  // other modes' Grams and so runs beside that mode's MTTKRP.
  cudaStream_t side = nullptr;
  cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
  // One ALS iteration captured as a CUDA graph (rebuilt after load, build
  // and communicator changes).
  // Two of them, for two iterations in flight (slot = iteration parity),
  // each with its own timing events (ev, ev1) and readback slot in h_scal.
  cudaGraph_t iter_graph[2] = {nullptr, nullptr};
  cudaGraphExec_t iter_exec[2] = {nullptr, nullptr};
  cudaEvent_t ev1[2 * CPTC_MAX_ORDER + 2] = {};
  cudaEvent_t* evc = nullptr;  // events of the iteration being enqueued
  unsigned long long iter_kernels = 0;  // this library's kernels in the graph
  // Phase timing (off by default; the events are extra graph nodes): per
  // slot and mode, events after the reduce-scatter, the solve, the
  // all-reduce + all-gather and the normalisation.
  bool phase_timing = false;
  int cur_slot = 0;
  cudaEvent_t evp[2][CPTC_MAX_ORDER][4] = {};
  double phase_ms[CPTC_MAX_ORDER][CPTC_NPHASES] = {};
  bool phase_valid = false;
  std::string err;

  // Tensor (device COO, relabelled in place by the build).
  int N = 0;
  uint64_t dims[CPTC_MAX_ORDER] = {0};
  uint64_t nnz = 0;
  DArray<uint32_t> idx[CPTC_MAX_ORDER];
  DArray<double> vals;
  double x_norm_sq = 0.0;

  // Relabelling: perm[m][old] = new (host); identity when empty.
  std::vector<std::vector<uint32_t>> perm;
  DArray<uint32_t> dperm[CPTC_MAX_ORDER];  // device copy of perm (unset when identity)
  DArray<double> stage;                    // max_m I_m x R rows for host transfers
  std::vector<std::vector<uint32_t>> host_idx;  // original coordinates
  std::string reorder_note;

  // Build results.
  bool built = false;
  int R = 0;
  cptc_opts opts{};
  bool generic = false;  // N-order ALS semantics (Cholesky, lambda = norms)
  bool tf32 = false;
  std::vector<View> views;
  UnitPool units;               // dense tiles (order 3) or units (N-order)
  bool dense_active = false;
  double avg_fill = 0.0, fill_min = 0.0;
  int cutoff = 0;
  double build_ms = 0.0;
  double reorder_ms = 0.0;

  // Factors (relabelled space) and ALS workspace.
  bool have_factors = false;
  bool grams_valid = false;
  DArray<double> F[CPTC_MAX_ORDER];
  DArray<double> G[CPTC_MAX_ORDER];
  DArray<double> lambda;
  DArray<double> FtV, FtF, Ainv, gpart, dots, scal, cscale;
  // The contracted factor of an order-3 tile launch as TF32 bit patterns in
  // 16-row blocks (launch_to_tf32_blocks), written just before the launch.
  DArray<float> Ftf;
  DArray<int> status;
  double* h_scal = nullptr;  // pinned, 16 doubles: two readback slots of 8
  int gpart_blocks = 0;
  double last_iprod = 0.0, last_model2 = 0.0, last_fit = 0.0;

  // Multi-GPU (shard.cu, comm.cu): mode-n rows [slab[n][r], slab[n][r+1])
  // belong to rank r, in 16-row blocks [slab_blocks[n][r], ..[r+1]); the
  // first heavy_rows[n] rows (inside rank 0's slab) are a heavy prefix
  // whose nonzeros every rank shares and whose rows every rank solves.
  void* nccl = nullptr;  // ncclComm_t
  int nranks = 1, rank = 0;
  std::vector<uint64_t> slab[CPTC_MAX_ORDER];
  std::vector<uint64_t> slab_blocks[CPTC_MAX_ORDER];
  uint64_t heavy_rows[CPTC_MAX_ORDER] = {0};
  // Estimated MTTKRP cost of every rank's share of mode n (the heavy
  // prefix's share plus its slab), and the measured speed correction per
  // rank that the second build pass applies to the first pass's slabs.
  std::vector<double> slab_cost[CPTC_MAX_ORDER];
  std::vector<double> shard_speed[CPTC_MAX_ORDER];
  std::vector<uint64_t> prev_blocks[CPTC_MAX_ORDER];
  DArray<double> comm_buf;

  cudaEvent_t ev[2 * CPTC_MAX_ORDER + 2] = {};

  explicit Engine(int dev);
  ~Engine();

  void load(const cptc_coo* t);
  void build(int R, double threshold, const cptc_opts* o);
  void init_factors();
  void set_factor(int m, const double* host);
  void set_factor_sharded(int m, const double* host);
  void get_factor_sharded(int m, double* host);
  void get_factor(int m, double* host);
  void fetch_rows(const double* dev, int m, double* host);
  double* stage_rows();
  void release_graph();
  void set_phase_timing(bool on);
  void enqueue_iteration(int slot);
  void launch_iteration(int slot);
  void finish_iteration(int it, int slot, cptc_iter_cb cb, void* user);
  uint64_t padded_rows(int m) const;
  void permute_rows(const double* in, int m, bool to_relabelled, double* out);
  void mttkrp(int mode);  // into FtV (relabelled rows), stream-ordered
  void mttkrp_tiles(int mode, double* out = nullptr, cudaStream_t s = nullptr);
                                 // dense-tile TF32 part only (accumulates into out, FtV
                                 // by default, on s, the engine stream by default)
  bool tiles_target(int mode) const;  // the dense tiles contribute to this mode
  void mttkrp_sparse(int mode);  // FP64 view part only (accumulates)
  void als(int iters, cptc_iter_cb cb, void* user);
  uint64_t device_bytes() const;
  // Rows this rank solves and publishes: its slab without the heavy prefix.
  uint64_t row_lo(int m) const {
    return slab[m].empty() ? 0 : std::max<uint64_t>(slab[m][rank], heavy_rows[m]);
  }
  uint64_t row_hi(int m) const {
    return slab[m].empty() ? dims[m] : std::max<uint64_t>(slab[m][rank + 1], heavy_rows[m]);
  }
  double* scal_tmp();
  double* colscale();

 private:
  void reorder();
  void alloc_workspace();
  void build_pass(int R, double threshold, const cptc_opts* o);
  void update_mode(int n, bool last);
  void gram_of(int m);
};

}  // namespace cptc
