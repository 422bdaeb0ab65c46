// Index relabelling before the build (host side; only mode-length arrays and
// a strided sample of the nonzeros are touched).
#pragma once
#include <cstdint>
#include <string>
#include <vector>

namespace cptc {

// Order-3 CADR (reference src/cadr.cu:31-51): degree-descending order by
// std::sort with the reference's comparator on the reference's input
// sequence, so ties land where the reference puts them.  perm[old] = new.
void cadr_perm_ref(uint64_t dim, uint64_t nnz, const uint32_t* idx,
                   std::vector<uint32_t>& perm);

// N-order relabelling (reference src/generic.cu:1180-1376).
// kind: 0 none, 1 cadr (ties by index), 2 hits (T rounds on a strided
// sample of <= sample_budget nonzeros), 3 auto (probe fill, keep HITS only
// if it lifts the probed tile fill to >= 0.11).  rank[m][old] = new; empty
// vectors mean identity.  `note` receives the reference's log text.
void reorder_generic(int N, const uint64_t* dims, uint64_t nnz, const uint32_t* const* idx,
                     int kind, int rounds, uint64_t sample_budget,
                     std::vector<std::vector<uint32_t>>& rank, std::string* note);

}  // namespace cptc
