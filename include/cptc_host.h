/*
 * cptc_host.h — host-only C ABI of cptc-b200: sparse tensor container,
 * FROSTT .tns reader/writer and the seeded synthetic generators.
 *
 * Nothing here touches a GPU; the library that exports it (libcptc_host.so,
 * and the same symbols inside libcptc.so) loads on a machine without CUDA.
 *
 * Reference interfaces replaced (paths inside zhixianzhu/cpTC):
 *   cptc_tns_read        <- load_tns_file (include/tensor.hpp:346,
 *                           src/tensor.cu:39-271) and load_tns_generic
 *                           (include/generic.hpp:34, src/generic.cu:1023-1155)
 *   cptc_tns_probe_order <- probe_tns_nmodes (include/generic.hpp:30,
 *                           src/generic.cu:983-1021)
 *   cptc_gen_config      <- scripts/gen_synth.py, gen_norder.py (the configs
 *                           of this project's benchmark replace them)
 */
#ifndef CPTC_HOST_H
#define CPTC_HOST_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CPTC_MAX_ORDER 8

/* Sparse tensor in coordinate form. idx[m][e] is the 0-based index of
 * nonzero e along mode m; vals[e] its value. Arrays are malloc'ed by the
 * library and released with cptc_coo_free. */
typedef struct cptc_coo {
  int order;
  uint64_t dims[CPTC_MAX_ORDER];
  uint64_t nnz;
  uint32_t* idx[CPTC_MAX_ORDER];
  double* vals;
} cptc_coo;

void cptc_coo_free(cptc_coo* t);

/* Reads a FROSTT .tns file with the reference's parse rules: '#' lines and
 * lines without a parseable value are skipped, indices are 1-based (an index
 * of 0 maps to 0), dims[m] = max 0-based index + 1 (at least 1).
 * order_hint <= 0 probes the order from the first data line.
 * Returns 0, or a negative code (-1 open failed, -2 bad order, -3 no memory). */
int cptc_tns_read(const char* path, int order_hint, cptc_coo* out);

/* Order of a .tns file (columns of the first data line minus one), or -1. */
int cptc_tns_probe_order(const char* path);

/* Writes `t` as 1-based .tns text, values with %.17g (exact round trip). */
int cptc_tns_write(const char* path, const cptc_coo* t);

/* Binary tensor cache (no counterpart in the reference, which parses the
 * text on every run: src/tensor.cu:39-271, src/generic.cu:1023-1155).
 * The file holds the arrays of `t` as they are in memory plus the size and
 * modification time (ns) of the .tns they came from, and a hash of the
 * arrays; it is written under a temporary name and renamed into place.
 * Returns 0 or -1 (cannot create / write). */
int cptc_bin_write(const char* path, const cptc_coo* t, uint64_t src_size,
                   int64_t src_mtime_ns);

/* Reads a cache written by cptc_bin_write; src_size / src_mtime_ns (may be
 * NULL) receive the recorded stamp of the source text. Returns 0, -1 (cannot
 * open), -3 (no memory) or -4 (not a cache, truncated, hash mismatch, or an
 * index outside the recorded dims). */
int cptc_bin_read(const char* path, cptc_coo* out, uint64_t* src_size,
                  int64_t* src_mtime_ns);

/* cptc_tns_read through a cache at cache_path (NULL or "": path +
 * ".cptcbin"). The cache is used when its recorded stamp equals the .tns
 * file's current size and modification time and its order is the one the
 * text would be read with (order_hint, or the probed order when
 * order_hint <= 0); otherwise the text is parsed and the cache
 * rewritten — a cache that cannot be written leaves just the parse result.
 * *from_cache (may be NULL) is 1 when the cache was used. Same results and
 * return codes as cptc_tns_read. */
int cptc_tns_read_cached(const char* path, int order_hint, const char* cache_path,
                         cptc_coo* out, int* from_cache);

/* Synthetic workloads of the benchmark (cfg 1..5: 128^3 planted rank 8;
 * 256^3 block-dense planted rank 32; 512^3 dense blocks + uniform residual;
 * 12092x9184x28818 Zipf(1.1) lognormal; 183x24x1140x1717 Zipf(1.2)
 * Poisson+1), scaled
 * to round(nnz * nnz_scale) nonzeros with the same dims. Every tensor is a
 * pure function of (cfg, nnz_scale, seed): coordinates are the first nnz
 * distinct draws of a counter-based RNG, sorted by linear index. */
int cptc_gen_config(int cfg, double nnz_scale, uint64_t seed, cptc_coo* out);

/* Uniform distinct coordinates of any order <= 8.
 * value_kind: 0 = U(0,1], 1 = lognormal(0,1), 2 = N(0,1), 3 = Poisson(3)+1. */
int cptc_gen_uniform(int order, const uint64_t* dims, uint64_t nnz,
                     uint64_t seed, int value_kind, cptc_coo* out);

/* Last host-side error message (thread-local). */
const char* cptc_host_last_error(void);


#ifdef __cplusplus
}
#endif

#endif /* CPTC_HOST_H */
