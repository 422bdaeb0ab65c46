// Shared helpers of the cptc-b200 engine: error plumbing, owning device
// arrays and small launch utilities.
#pragma once
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstdio>
#include <stdexcept>
#include <string>
#include <utility>

namespace cptc {

// Errors inside the engine are thrown as CptcError and turned into a status
// code at the C ABI boundary; nothing in the library exits the process.
struct CptcError : std::runtime_error {
  int code;
  CptcError(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

[[noreturn]] inline void throw_cuda(cudaError_t e, const char* what, const char* file,
                                    int line) {
  char buf[512];
  std::snprintf(buf, sizeof(buf), "%s failed: %s (%s:%d)", what, cudaGetErrorString(e), file,
                line);
  throw CptcError(e == cudaErrorMemoryAllocation ? -3 : -2, buf);
}

#define CPTC_CUDA(call)                                                 \
  do {                                                                  \
    cudaError_t e_ = (call);                                            \
    if (e_ != cudaSuccess) ::cptc::throw_cuda(e_, #call, __FILE__, __LINE__); \
  } while (0)

// Kernels launched by this library (all host threads), and by this host
// thread (used to count the kernels a graph capture records).
extern std::atomic<unsigned long long> g_launches;
extern thread_local unsigned long long t_launches;

#define CPTC_LAUNCH_CHECK()                                          \
  do {                                                               \
    CPTC_CUDA(cudaGetLastError());                                   \
    ::cptc::g_launches.fetch_add(1, std::memory_order_relaxed);      \
    ++::cptc::t_launches;                                            \
  } while (0)

#define CPTC_REQUIRE(cond, code, msg)                 \
  do {                                                \
    if (!(cond)) throw ::cptc::CptcError(code, msg);  \
  } while (0)

// Owning device array (cudaMalloc / cudaFree); movable, not copyable.
template <class T>
struct DArray {
  T* p = nullptr;
  size_t n = 0;
  DArray() = default;
  explicit DArray(size_t count) { alloc(count); }
  DArray(const DArray&) = delete;
  DArray& operator=(const DArray&) = delete;
  DArray(DArray&& o) noexcept : p(o.p), n(o.n) {
    o.p = nullptr;
    o.n = 0;
  }
  DArray& operator=(DArray&& o) noexcept {
    if (this != &o) {
      release();
      p = o.p;
      n = o.n;
      o.p = nullptr;
      o.n = 0;
    }
    return *this;
  }
  ~DArray() { release(); }
  void alloc(size_t count) {
    release();
    if (count == 0) count = 1;
    CPTC_CUDA(cudaMalloc((void**)&p, count * sizeof(T)));
    n = count;
  }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    n = 0;
  }
  size_t bytes() const { return n * sizeof(T); }
  T* get() const { return p; }
};

inline unsigned grid_for(uint64_t n, unsigned block, unsigned cap = 1u << 30) {
  uint64_t g = (n + block - 1) / block;
  if (g < 1) g = 1;
  if (g > cap) g = cap;
  return (unsigned)g;
}

inline int bits_for(uint64_t n) {  // bits needed to hold values in [0, n)
  int b = 0;
  while (b < 64 && (n - 1) >> b) ++b;
  return b ? b : 1;
}

}  // namespace cptc
