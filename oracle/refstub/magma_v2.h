/* Stand-in for MAGMA's header, used only to compile the reference CP-ALS
 * sources (oracle/build_ref.sh).  The reference calls MAGMA only from solver
 * paths that its driver never reaches; these stubs report failure if called. */
#pragma once
#include <cstdint>
typedef int magma_int_t;
typedef enum { MagmaLower = 122, MagmaUpper = 121 } magma_uplo_t;
typedef enum { MagmaNoTrans = 111, MagmaTrans = 112 } magma_trans_t;
static inline int magma_init() { return 0; }
static inline int magma_finalize() { return 0; }
static inline int magma_dpotrf_gpu(magma_uplo_t, magma_int_t, double*, magma_int_t,
                                   magma_int_t* info) { *info = -1; return -1; }
static inline int magma_dpotrs_gpu(magma_uplo_t, magma_int_t, magma_int_t, double*,
                                   magma_int_t, double*, magma_int_t, magma_int_t* info) {
  *info = -1; return -1; }
static inline int magma_dgetrf_gpu(magma_int_t, magma_int_t, double*, magma_int_t,
                                   magma_int_t*, magma_int_t* info) { *info = -1; return -1; }
static inline int magma_dgetrs_gpu(magma_trans_t, magma_int_t, magma_int_t, double*,
                                   magma_int_t, magma_int_t*, double*, magma_int_t,
                                   magma_int_t* info) { *info = -1; return -1; }
