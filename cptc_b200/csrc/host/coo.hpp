// Host-side sparse tensor in coordinate form, shared by the generators, the
// .tns reader/writer and the engine's loader.
#pragma once
#include <cstdint>
#include <cstdlib>

#include "../../../include/cptc_host.h"

namespace cptc {

// Allocates the index and value arrays of `t` for `nnz` entries.
bool coo_alloc(cptc_coo* t, int order, uint64_t nnz);

// Number of worker threads for host loops (CPTC_HOST_THREADS, else all cores).
int host_threads();

// Sets the thread-local message returned by cptc_host_last_error().
void set_host_error(const char* msg);

}  // namespace cptc
