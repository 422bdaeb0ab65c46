// Row-slab cuts for the multi-GPU partition (cptc_slab_cuts in cptc_host.h).
#include <cstdint>

#include "coo.hpp"

extern "C" int cptc_slab_cuts(const uint32_t* counts, uint64_t dim, uint64_t nnz, int nranks,
                              uint64_t* cuts) {
  if (nranks < 1 || !cuts || (dim > 0 && !counts)) {
    cptc::set_host_error("cptc_slab_cuts: nranks < 1 or null pointer");
    return -1;
  }
  for (int r = 0; r <= nranks; ++r) cuts[r] = 0;
  cuts[nranks] = dim;
  uint64_t acc = 0;
  int r = 1;
  for (uint64_t i = 0; i < dim && r < nranks; ++i) {
    acc += counts[i];
    // Rank r starts after the row where the running count reaches r/nranks.
    while (r < nranks && acc * (uint64_t)nranks >= (uint64_t)r * nnz) {
      uint64_t c = (i + 1 + 15) / 16 * 16;
      if (c > dim) c = dim;
      if (c < cuts[r - 1]) c = cuts[r - 1];
      cuts[r++] = c;
    }
  }
  for (; r < nranks; ++r) cuts[r] = dim;
  cptc::set_host_error("");
  return 0;
}
