// Residual of a CP model on caller-owned device buffers, with no device
// allocation inside the library (cptc_residual_noalloc in include/cptc.h).
//
// The per-block partial sums that cptc_residual keeps in memory it
// allocates live here in one fixed array in device global memory, declared
// at file scope: every GPU that loads this library holds it until the
// process exits.  Host code cannot use the array's name as a device address
// (it names a host-side stand-in), so the address is looked up once per
// device with cudaGetSymbolAddress and passed to the kernels.
#include <mutex>

#include "../host/coo.hpp"
#include "kernels.hpp"

namespace cptc {

namespace {

// Partial sums the entry point can hold: at most this many blocks per call.
constexpr int kNoAllocPartials = 2048;  // 16 KiB per GPU

static __device__ __align__(256) double g_noalloc_partials[kNoAllocPartials];

constexpr int kMaxDevices = 64;

struct ScratchTable {
  std::mutex mu;
  double* ptr[kMaxDevices] = {};
};

ScratchTable& table() {
  static ScratchTable t;
  return t;
}

// Device address of the scratch array on the current device (set up on
// the first call on each device, with that device current).
double* scratch_on_current_device() {
  int dev = 0;
  CPTC_CUDA(cudaGetDevice(&dev));
  CPTC_REQUIRE(dev >= 0 && dev < kMaxDevices, CPTC_E_UNSUP, "device index beyond 63");
  ScratchTable& t = table();
  std::lock_guard<std::mutex> lock(t.mu);
  if (!t.ptr[dev]) {
    double* p = nullptr;
    const cudaError_t rc = cudaGetSymbolAddress((void**)&p, g_noalloc_partials);
    if (rc != cudaSuccess || p == nullptr)
      throw CptcError(CPTC_E_CUDA, std::string("cudaGetSymbolAddress of the residual scratch: ") +
                                       cudaGetErrorString(rc));
    t.ptr[dev] = p;
  }
  return t.ptr[dev];
}

}  // namespace

}  // namespace cptc

extern "C" int cptc_residual_noalloc(int order, uint64_t nnz, const uint32_t* const* d_idx,
                                     const double* d_vals, int R,
                                     const double* const* d_factors, const double* d_lambda,
                                     double* d_out, void* stream) {
  using namespace cptc;
  if (order < 1 || order > CPTC_MAX_ORDER) {
    set_host_error("cptc_residual_noalloc: order must be in [1, 8]");
    return CPTC_E_UNSUP;
  }
  if (R < 1 || R > 128) {
    set_host_error("cptc_residual_noalloc: R must be in [1, 128]");
    return CPTC_E_UNSUP;
  }
  if (!d_idx || !d_factors || !d_out || !d_lambda || (nnz > 0 && !d_vals)) {
    set_host_error("cptc_residual_noalloc: null pointer argument");
    return CPTC_E_ARG;
  }
  try {
    ResidualArgs a{};
    for (int m = 0; m < order; ++m) {
      if (!d_idx[m] || !d_factors[m]) {
        set_host_error("cptc_residual_noalloc: null index or factor pointer");
        return CPTC_E_ARG;
      }
      a.idx[m] = d_idx[m];
      a.F[m] = d_factors[m];
    }
    a.val = d_vals;
    a.lambda = d_lambda;
    a.nnz = nnz;
    a.N = order;
    a.R = R;
    double* scratch = scratch_on_current_device();
    // Every block writes its own partial and the final pass reads exactly
    // those, so nothing left in the array by an earlier call is read.
    launch_residual(a, scratch, kNoAllocPartials, d_out, (cudaStream_t)stream);
    set_host_error("");
    return CPTC_OK;
  } catch (const CptcError& x) {
    set_host_error(x.what());
    return x.code;
  } catch (...) {  // std::mutex or the per-device cache
    set_host_error("cptc_residual_noalloc: host error");
    return CPTC_E_ARG;
  }
}
