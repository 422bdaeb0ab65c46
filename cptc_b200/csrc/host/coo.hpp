// Host-side sparse tensor in coordinate form, shared by the generators, the
// .tns reader/writer and the engine's loader.
#pragma once
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <new>

#include "../../../include/cptc_host.h"

namespace cptc {

// Allocates the index and value arrays of `t` for `nnz` entries.
bool coo_alloc(cptc_coo* t, int order, uint64_t nnz);

// Number of worker threads for host loops (CPTC_HOST_THREADS, else all cores).
int host_threads();

// Sets the thread-local message returned by cptc_host_last_error().
void set_host_error(const char* msg);

// Runs the body of a C entry point: a C++ exception never crosses the C ABI
// (out of memory -> -3, anything else -> -2, message kept).  `out`, when
// given, is zeroed first and released on that path.
template <class F>
int host_guard(cptc_coo* out, F&& body) {
  if (out) std::memset(out, 0, sizeof(*out));
  try {
    return body();
  } catch (const std::bad_alloc&) {
    set_host_error("out of host memory");
    if (out) cptc_coo_free(out);
    return -3;
  } catch (const std::exception& e) {
    set_host_error(e.what());
    if (out) cptc_coo_free(out);
    return -2;
  } catch (...) {
    set_host_error("unknown host error");
    if (out) cptc_coo_free(out);
    return -2;
  }
}

}  // namespace cptc
