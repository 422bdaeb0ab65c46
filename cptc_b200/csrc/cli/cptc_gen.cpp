// cptc_gen — writes a seeded benchmark tensor as a FROSTT .tns file.
//
//   cptc_gen <cfg 1..5> <nnz_scale> <out.tns> [seed]
//
// The same tensors as cptc_gen_config (include/cptc_host.h), for programs
// that read .tns text, such as the reference's own driver.  The generator and
// writer sources are compiled into this executable, so a process that runs it
// loads no library of this project.  On success it prints one JSON line with
// the order, dims (max 0-based index + 1 per mode, the reference loader's
// rule, src/tensor.cu:247-254), nnz and the generator's nominal dims.
#include <cinttypes>
#include <cstdio>
#include <cstdlib>

#include "cptc_host.h"

int main(int argc, char** argv) {
  if (argc < 4) {
    std::fprintf(stderr, "usage: %s <cfg 1..5> <nnz_scale> <out.tns> [seed]\n", argv[0]);
    return 2;
  }
  const int cfg = std::atoi(argv[1]);
  const double scale = std::atof(argv[2]);
  const uint64_t seed = argc > 4 ? std::strtoull(argv[4], nullptr, 10) : 0ull;
  cptc_coo t{};
  if (cptc_gen_config(cfg, scale, seed, &t) != 0) {
    std::fprintf(stderr, "cptc_gen: %s\n", cptc_host_last_error());
    return 1;
  }
  if (cptc_tns_write(argv[3], &t) != 0) {
    std::fprintf(stderr, "cptc_gen: cannot write %s: %s\n", argv[3], cptc_host_last_error());
    cptc_coo_free(&t);
    return 1;
  }
  uint64_t seen[CPTC_MAX_ORDER] = {0};
  for (int m = 0; m < t.order; ++m) {
    uint32_t mx = 0;
    for (uint64_t e = 0; e < t.nnz; ++e)
      if (t.idx[m][e] > mx) mx = t.idx[m][e];
    seen[m] = t.nnz ? (uint64_t)mx + 1 : 1;
  }
  std::printf("{\"order\": %d, \"nnz\": %" PRIu64 ", \"dims\": [", t.order, t.nnz);
  for (int m = 0; m < t.order; ++m) std::printf("%s%" PRIu64, m ? ", " : "", seen[m]);
  std::printf("], \"nominal_dims\": [");
  for (int m = 0; m < t.order; ++m) std::printf("%s%" PRIu64, m ? ", " : "", t.dims[m]);
  std::printf("]}\n");
  cptc_coo_free(&t);
  return 0;
}
