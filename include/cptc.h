/*
 * cptc.h — C ABI of the cptc-b200 CP-ALS engine (sm_100a).
 *
 * The reference (zhixianzhu/cpTC) has no library interface: its operator
 * boundary is a set of C++ functions over its HybridCOOTensor, called only by
 * its own main().  Each entry point below names the reference function whose
 * role it takes over (paths inside the reference project):
 *
 *   cptc_load_coo     <- load_tns_file / COO upload (src/tensor.cu:39-271)
 *   cptc_build        <- compute/apply_cadr_reordering (src/cadr.cu:23-81),
 *                        partition_tensor_hybrid (include/partition.hpp:335),
 *                        build_mttkrp_views (include/partition.hpp:369),
 *                        build_dense_mttkrp_views (:375), the fill-rate
 *                        selector (src/main.cu:336-426); for the N-order path
 *                        apply_reordering / build_dense_nd / ModeView build
 *                        (src/generic.cu:1180-1376, 578-725, 1842-1958)
 *   cptc_init_factors <- init_factors_random (src/common.cu:66-126) and the
 *                        generic init (src/generic.cu:1754-1788)
 *   cptc_mttkrp       <- run_mttkrp_mode (src/als.cu:535-604):
 *                        zero FtV, compute_dense_mttkrp_async
 *                        (include/dense.hpp:7) + compute_sparse_mttkrp_async
 *                        (include/sparse.hpp:77)
 *   cptc_als          <- execute_als_decomposition (include/als.hpp:7) and
 *                        run_generic_cp (include/generic.hpp:42)
 *   cptc_get_factors  <- unpermute_factor_matrices (include/cadr.hpp:21-32)
 *
 * Conventions: status 0 = OK, negative = error (message from
 * cptc_last_error); the library never exits the process.  Host arrays are
 * copied; factors are row-major FP64 I_n x R in the caller's original index
 * space.  One context per host thread; a context is not thread-safe.
 */
#ifndef CPTC_H
#define CPTC_H

#include <stdint.h>

#include "cptc_host.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct cptc_ctx cptc_ctx;

enum {
  CPTC_OK = 0,
  CPTC_E_ARG = -1,      /* invalid argument or call order */
  CPTC_E_CUDA = -2,     /* CUDA runtime / kernel launch failure */
  CPTC_E_NOMEM = -3,    /* device or host allocation failed */
  CPTC_E_UNSUP = -4,    /* configuration not supported */
  CPTC_E_COMM = -5,     /* NCCL failure or timeout */
  CPTC_E_NUMERIC = -6   /* solve failed (non-finite) */
};

/* Path selection (ALS_FORCE_WMMA / ALS_FORCE_CUDA of src/main.cu:395-402). */
enum { CPTC_PATH_AUTO = 0, CPTC_PATH_TF32 = 1, CPTC_PATH_FP64 = 2 };
/* Index relabelling before the build (src/generic.cu:1162-1169). */
enum { CPTC_REORDER_NONE = 0, CPTC_REORDER_CADR = 1, CPTC_REORDER_HITS = 2,
       CPTC_REORDER_AUTO = 3, CPTC_REORDER_DEFAULT = -1 };
/* R x R solve (GEN_SOLVER of src/generic.cu:2114-2136). */
enum { CPTC_SOLVER_DEFAULT = 0, CPTC_SOLVER_CHOL = 1, CPTC_SOLVER_PINV = 2 };
/* How the ranks of a multi-GPU context combine a mode update (no
 * counterpart in the reference, which runs on one GPU).
 *   NCCL: one NCCL all-reduce per mode update, of one buffer holding the
 *         heavy prefix's partial MTTKRP rows, the factor rows past that
 *         prefix (each rank contributing its solved slab and zeros
 *         elsewhere) and the Gram partials (and fit dots) (the default).
 *   PEER: reserved (a peer-memory exchange); cptc_build returns
 *         CPTC_E_UNSUP for it on several ranks. */
enum { CPTC_EXCHANGE_NCCL = 0, CPTC_EXCHANGE_PEER = 1 };

typedef struct cptc_opts {
  int path;                 /* CPTC_PATH_*                                   */
  double fill_min;          /* <= 0: B200 default; else ALS_FILL_MIN         */
  int generic;              /* 1: order-3 through the N-order path
                               (ALS_GENERIC_FORCE)                           */
  int reorder;              /* CPTC_REORDER_* (GEN_REORDER)                  */
  int reorder_rounds;       /* HITS rounds (GEN_REORDER_T, 3)                */
  uint64_t reorder_sample;  /* HITS sample budget (GEN_REORDER_SAMPLE, 8e6)  */
  int solver;               /* CPTC_SOLVER_*                                 */
  uint32_t seed;            /* N-order init seed (GEN_SEED, 42)              */
  int dense_generic;        /* 0 disables N-order dense units (GEN_DENSE=0)  */
  double dense_thr_generic; /* GEN_DENSE_THRESHOLD (0.03)                    */
  int dense_inner[3];       /* GEN_DENSE_INNER (0,1,2)                       */
  int verbose;              /* print the reference's progress lines          */
  int exchange;             /* CPTC_EXCHANGE_*: how ranks combine a mode
                               update (several GPUs only)                    */
} cptc_opts;

/* Per-iteration report: iteration number (1-based), device time of the
 * iteration in ms, Gram fit, and MTTKRP device ms per mode. */
typedef void (*cptc_iter_cb)(int iter, double ms, double fit,
                             const double* mttkrp_ms, int nmodes, void* user);

typedef struct cptc_stats {
  int order;
  uint64_t dims[CPTC_MAX_ORDER];
  uint64_t nnz;
  int rank;
  int tf32_path;            /* 1 if the dense-tile TF32 path is active       */
  uint64_t dense_nnz;       /* nonzeros in dense tiles / units               */
  uint64_t sparse_nnz;      /* nonzeros in the FP64 residual                 */
  uint64_t dense_tiles;
  double avg_fill;          /* dense_nnz / (tiles * 4096)                    */
  double fill_min;          /* threshold used by the selector                */
  int cutoff;               /* nonzeros per 16^3 tile to be dense            */
  double x_norm_sq;         /* ||X||_F^2                                     */
  double build_ms;          /* reorder + partition + views                   */
  uint64_t device_bytes;    /* device memory held by the context             */
  int fiber_mode[CPTC_MAX_ORDER]; /* per target mode: mode whose rows are
                                     reused along a sorted run               */
  int nranks, rank_id;
  double reorder_ms;        /* relabelling share of build_ms (HITS, degree
                               order: on the device; order-3 CADR: host)     */
  /* Per target mode, this rank's share of the MTTKRP (the whole mode on one
   * rank): residual nonzeros, non-empty target rows of the residual view,
   * dense tiles and the words of those tiles (nonzeros, each tile padded to
   * a multiple of 4; order-3 tiles only). */
  uint64_t local_sparse_nnz[CPTC_MAX_ORDER];
  uint64_t local_rows[CPTC_MAX_ORDER];
  uint64_t local_tiles[CPTC_MAX_ORDER];
  uint64_t local_tile_words[CPTC_MAX_ORDER];
} cptc_stats;

int cptc_opts_default(cptc_opts* o);

/* Creates a context on CUDA device `device` (flags reserved, pass 0). */
int cptc_create(cptc_ctx** out, int device, int flags);
int cptc_destroy(cptc_ctx* ctx);
const char* cptc_last_error(const cptc_ctx* ctx);

/* Multi-GPU (one process per GPU): rank 0 calls cptc_comm_unique_id and
 * shares the 128 bytes; every rank then calls cptc_comm_init before
 * cptc_build.  cptc_comm_init, cptc_build, cptc_als, cptc_mttkrp and
 * cptc_set_factors_sharded are collective: every rank calls them, in the
 * same order; the other functions are local (for example one rank alone may
 * read the replicated factors).  The rows of every mode are owned in slabs
 * of equal estimated MTTKRP cost and each rank keeps only the nonzeros (FP64
 * residual and dense tiles) of its rows; a heavy prefix of rows (a Zipf
 * head) has its nonzeros dealt to all ranks and its partial rows
 * all-reduced.  Each mode update is one NCCL all-reduce (see
 * CPTC_EXCHANGE_NCCL) and every rank ends with the whole factor.  The
 * reference runs on one GPU.  A rank that stops calling leaves the others'
 * next collective waiting on the GPU: callers detect a lost rank on the host
 * (their own heartbeat or store) before the next collective call and end
 * the job, as the CLI does (CPTC_NGPU). */
int cptc_comm_unique_id(unsigned char out_id[128]);
int cptc_comm_init(cptc_ctx* ctx, const unsigned char id[128], int rank, int nranks);

/* Copies a host COO tensor (order 2..8) to the device. */
int cptc_load_coo(cptc_ctx* ctx, const cptc_coo* t);

/* Reorders, partitions, builds per-mode views and selects the path for rank
 * R.  threshold: dense 16^3 tile cutoff fraction (<= 0: auto balance). */
int cptc_build(cptc_ctx* ctx, int R, double threshold, const cptc_opts* opts);

/* The reference's initial factors (order-3: mt19937(42) in relabelled
 * space; N-order: mt19937(seed) carried through the relabelling), lambda=1. */
int cptc_init_factors(cptc_ctx* ctx);

/* Factors in the caller's original index space, row-major I_n x R.  The
 * copy is complete when cptc_set_factors returns (the buffer may be reused;
 * pinned memory makes it a single DMA).  With several ranks every rank sets
 * the same factors (each holds a replica). */
int cptc_set_factors(cptc_ctx* ctx, int mode, const double* host);
/* The same result with the host-to-device copy shared out (no counterpart in
 * the reference, which runs on one GPU). Collective: rank r of G copies only
 * rows [r*s, min((r+1)*s, I)) of `host`, s = ceil(I / G), in the original
 * index space (the other rows of `host` are not read), and the pieces are
 * all-gathered over NVLink into every rank's replica. One rank: the same as
 * cptc_set_factors. */
int cptc_set_factors_sharded(cptc_ctx* ctx, int mode, const double* host);
/* Local counterpart for reading: rank r copies only rows [r*s, (r+1)*s) of
 * the factor (original index space) into the same rows of `host`; the other
 * rows are not written. One rank: the same as cptc_get_factors. */
int cptc_get_factors_sharded(cptc_ctx* ctx, int mode, double* host);
int cptc_get_factors(cptc_ctx* ctx, int mode, double* host);
int cptc_get_lambda(cptc_ctx* ctx, double* host_R);

/* One MTTKRP of `mode` on the current factors (the path selected by
 * cptc_build), result in original index space (I_mode x R, host).  With
 * several ranks it is collective: every rank calls it and receives the
 * whole result. */
int cptc_mttkrp(cptc_ctx* ctx, int mode, double* host_out);

/* Device-resident MTTKRP into the context's FtV buffer; *ms = device time of
 * `reps` back-to-back launches divided by reps (CUDA events on the
 * context's stream). */
int cptc_mttkrp_timed(cptc_ctx* ctx, int mode, int reps, double* ms);

/* Device times (ms, mean of `reps` back-to-back launches on the context's
 * stream) of one mode's MTTKRP parts on this rank's share: ms3[0] dense-tile
 * TF32 kernel, ms3[1] FP64 residual kernel, ms3[2] the whole MTTKRP (zero +
 * both). */
int cptc_profile_mttkrp(cptc_ctx* ctx, int mode, int reps, double ms3[3]);

/* Number of kernels this library has launched since it was loaded (a
 * replayed CUDA graph of an ALS iteration counts the kernels it holds). */
unsigned long long cptc_launch_count(void);

/* The order-3 FP64 residual MTTKRP of `mode` against the floor set by its own
 * memory accesses (no counterpart in the reference; measurement only):
 * ms2[0] = ms per launch of a gather-only replay (the same tasks, records and
 * factor rows with the same lane layout, the fastest of three depths of
 * records in flight, no arithmetic), ms2[1] = ms per launch of the kernel
 * itself. Order-3 record views, R in {16, 32, 64, 128}; else CPTC_E_UNSUP. */
int cptc_profile_gather(cptc_ctx* ctx, int mode, int reps, double ms2[2]);

/* Measured ceiling of the FP64 MTTKRP's factor-row gathers on `device` (no
 * counterpart in the reference; measurement only): gathers n uniformly
 * random rows of an L2-resident rows x R FP64 matrix with the residual
 * kernel's row layout (R/2 lanes up to a warp per row, 16-byte loads) and
 * nothing else, and writes the rate in GB/s (n * 8R bytes per launch over
 * its CUDA-event time, mean of `reps` launches). R in {16, 32, 64, 128}.
 * Allocates and frees its own buffers. */
int cptc_gather_peak(int device, uint64_t rows, int R, uint64_t n, int reps, double* gbs);

/* Per-phase device times of each mode update (no counterpart in the
 * reference, whose ALS_PROFILE reports the MTTKRP only: src/als.cu:535-604).
 * cptc_phase_timing(ctx, 1) adds timing events after each phase of every
 * mode update from the next cptc_als on (off by default: the events are
 * extra nodes in the iteration's graph). cptc_phase_times then writes, for
 * the last iteration that finished, out[n * CPTC_NPHASES + p] in ms for
 * mode n < order and phase p:
 *   0  MTTKRP (zero, residual kernel, dense tiles)
 *   1  wait for the R x R inverse (computed beside the MTTKRP)
 *   2  apply the inverse to this rank's rows, Gram partials (and the fit's
 *      column dots on the last mode)
 *   3  the exchange: partial sums, and on several GPUs one NCCL group
 *      (one all-reduce of the heavy prefix's MTTKRP, every rank's solved
 *      rows, Gram and dots), then the solve of
 *      the heavy prefix
 *   4  normalisation (and the fit on the last mode)
 * Writes at most `cap` values and returns how many (0 when phase timing is
 * off or no iteration has run since it was turned on), or a negative
 * status. On several GPUs each rank reports its own times: a phase that
 * waits for the slowest rank shows that wait. */
#define CPTC_NPHASES 5
int cptc_phase_timing(cptc_ctx* ctx, int on);
int cptc_phase_times(cptc_ctx* ctx, double* out, int cap);

/* Runs `iters` CP-ALS iterations; cb (nullable) is called once per
 * iteration, in order, with that iteration's device time, fit and per-mode
 * MTTKRP times.  Iteration k+1 is already on the GPU when the callback of
 * iteration k runs (the iterations do not depend on the host), and all
 * iterations have finished when cptc_als returns. */
int cptc_als(cptc_ctx* ctx, int iters, cptc_iter_cb cb, void* user);

int cptc_get_stats(cptc_ctx* ctx, cptc_stats* out);

/* The build's index relabelling of `mode`: perm_out[old] = new
 * (dims[mode] entries; the identity when no relabelling ran). */
int cptc_get_relabel(cptc_ctx* ctx, int mode, uint32_t* perm_out);

/* Terms of the last iteration's Gram fit: out3 = {iprod, model^2, fit}
 * (src/als.cu:668-715, src/generic.cu:2174-2214). */
int cptc_fit_terms(cptc_ctx* ctx, double out3[3]);

/* Exact residual over the stored nonzeros with the current factors and
 * lambda: out2 = {sum (v - xhat)^2, sum v^2}.  Replaces
 * compute_residual_and_norm_sq (src/common.cu:517-650) and
 * g_exact_residual_kernel (src/generic.cu:936-967). */
int cptc_residual(cptc_ctx* ctx, double out2[2]);

/* Residual sum of squares of a CP model against a sparse tensor,
 *   d_out[0] = sum_e (v_e - sum_r lambda_r prod_m F_m[i_m(e), r])^2,
 * computed on buffers the caller already holds on the current device,
 * WITHOUT ALLOCATING: no cudaMalloc, no cudaFree, no allocating library
 * routine.  It is for callers that cannot let a library allocate device
 * memory: processes whose device memory belongs to their own pool or to a
 * reservation made at start-up (a serving process that pre-allocates
 * everything, a framework that permits no allocation outside its caching
 * allocator), and tight loops that cannot afford the device-wide
 * synchronisation a cudaFree implies.  It has no counterpart in the
 * reference; cptc_residual is the allocating equivalent.
 *   d_idx[m]     host array of `order` device pointers: u32 indices, nnz each
 *   d_vals       device, nnz doubles
 *   d_factors[m] host array of `order` device pointers: row-major I_m x R
 *   d_lambda     device, R doubles;  d_out  device, 1 double (written)
 *   stream       cudaStream_t on the current device (NULL = default stream)
 * Limits: 1 <= order <= 8 and 1 <= R <= 128, else CPTC_E_UNSUP and a
 * message in cptc_host_last_error(); nnz is unrestricted.  The per-block
 * partial sums live in a fixed array inside the library, 2048 doubles
 * (16 KiB) on every GPU that loads it, held until the process exits.  The
 * first call on each device sets up that device's address of the array
 * (cudaGetSymbolAddress, with the device current): make that first call
 * before any stream capture.  The address is kept for the life of the
 * process, so a cudaDeviceReset of a device after its first call is not
 * supported (the library's module, and the array, are gone with the
 * context).  All calls share the array, which keeps the
 * last call's contents; each call writes every slot it later reads, so no
 * clearing is needed.  Calls that overlap on the GPU (concurrent streams,
 * or host threads sharing a device) race on the array: serialise them. */
int cptc_residual_noalloc(int order, uint64_t nnz, const uint32_t* const* d_idx,
                          const double* d_vals, int R, const double* const* d_factors,
                          const double* d_lambda, double* d_out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CPTC_H */
