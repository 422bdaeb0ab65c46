// Binary tensor cache beside a .tns file.
//
// Parsing config 4's 2.7 GB text takes seconds on all cores; the cache holds
// the parsed arrays as they sit in memory, so a later run copies them back at
// memory speed.  The cache records the size and modification time (ns) of
// the text it was made from and is used only while both still match.
//
// File layout (little-endian; every array starts on a 64-byte boundary):
//   0    char[8]  magic "CPTCBIN1"
//   8    u32      order N (1..8)
//   12   u32      reserved (0)
//   16   u64      nnz
//   24   u64      source .tns size in bytes
//   32   i64      source .tns modification time, ns since the epoch
//   40   u64[8]   dims (unused entries 0)
//   104  u64      payload hash
//   112  u64[2]   reserved (0)
//   128  u32[nnz] idx[0], then idx[1] .. idx[N-1], then f64[nnz] vals
// The payload hash is FNV-1a (64-bit) over the hashes of consecutive 4 MiB
// chunks of each array in order (a chunk hash is FNV-1a over its 8-byte
// words, a ragged end zero-padded), so it is computed by many threads and
// does not depend on how many.
#include <fcntl.h>
#include <omp.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "coo.hpp"

namespace cptc {
namespace {

constexpr char kMagic[8] = {'C', 'P', 'T', 'C', 'B', 'I', 'N', '1'};
constexpr uint64_t kHeader = 128;
constexpr uint64_t kChunk = 4ull << 20;
constexpr uint64_t kFnvOffset = 0xcbf29ce484222325ull;
constexpr uint64_t kFnvPrime = 0x100000001b3ull;

struct Header {
  char magic[8];
  uint32_t order;
  uint32_t reserved0;
  uint64_t nnz;
  uint64_t src_size;
  int64_t src_mtime_ns;
  uint64_t dims[CPTC_MAX_ORDER];
  uint64_t hash;
  uint64_t reserved1[2];
};
static_assert(sizeof(Header) == kHeader, "cache header is 128 bytes");

uint64_t align64(uint64_t x) { return (x + 63) & ~63ull; }

uint64_t fnv_words(const unsigned char* p, uint64_t n) {
  uint64_t h = kFnvOffset;
  uint64_t i = 0;
  for (; i + 8 <= n; i += 8) {
    uint64_t w;
    std::memcpy(&w, p + i, 8);
    h = (h ^ w) * kFnvPrime;
  }
  if (i < n) {
    uint64_t w = 0;
    std::memcpy(&w, p + i, (size_t)(n - i));
    h = (h ^ w) * kFnvPrime;
  }
  return h;
}

// One array of the payload: where it lives in the file and in memory.
struct Span {
  uint64_t off;  // file offset
  uint64_t bytes;
  unsigned char* mem;
};

std::vector<Span> spans_of(const cptc_coo* t) {
  std::vector<Span> s;
  uint64_t off = kHeader;
  for (int m = 0; m < t->order; ++m) {
    s.push_back({off, t->nnz * 4, (unsigned char*)t->idx[m]});
    off = align64(off + t->nnz * 4);
  }
  s.push_back({off, t->nnz * 8, (unsigned char*)t->vals});
  return s;
}

uint64_t file_bytes(int order, uint64_t nnz) {
  uint64_t off = kHeader;
  for (int m = 0; m < order; ++m) off = align64(off + nnz * 4);
  return off + nnz * 8;
}

struct Piece {
  int span;
  uint64_t begin, end;  // byte range inside the span
};

std::vector<Piece> pieces_of(const std::vector<Span>& s) {
  std::vector<Piece> p;
  for (int k = 0; k < (int)s.size(); ++k)
    for (uint64_t b = 0; b < s[k].bytes; b += kChunk)
      p.push_back({k, b, std::min(s[k].bytes, b + kChunk)});
  return p;
}

uint64_t combine(const std::vector<uint64_t>& h) {
  uint64_t x = kFnvOffset;
  for (uint64_t v : h) x = (x ^ v) * kFnvPrime;
  return x;
}

bool write_all(int fd, const void* p, uint64_t n, uint64_t off) {
  const char* c = (const char*)p;
  while (n > 0) {
    const ssize_t w = ::pwrite(fd, c, (size_t)std::min<uint64_t>(n, 1ull << 30), (off_t)off);
    if (w <= 0) return false;
    c += w;
    n -= (uint64_t)w;
    off += (uint64_t)w;
  }
  return true;
}

}  // namespace

// Size and modification time (ns) of a file; false if it cannot be stat'ed.
static bool file_stamp(const char* path, uint64_t* size, int64_t* mtime_ns) {
  struct stat st;
  if (::stat(path, &st) != 0) return false;
  *size = (uint64_t)st.st_size;
  *mtime_ns = (int64_t)st.st_mtim.tv_sec * 1000000000ll + (int64_t)st.st_mtim.tv_nsec;
  return true;
}

}  // namespace cptc

using namespace cptc;

extern "C" {

int cptc_bin_write(const char* path, const cptc_coo* t, uint64_t src_size, int64_t src_mtime_ns) {
  return host_guard(nullptr, [&]() -> int {
    if (!path || !t || t->order < 1 || t->order > CPTC_MAX_ORDER) {
      set_host_error("cptc_bin_write: bad tensor");
      return -2;
    }
    Header h{};
    std::memcpy(h.magic, kMagic, 8);
    h.order = (uint32_t)t->order;
    h.nnz = t->nnz;
    h.src_size = src_size;
    h.src_mtime_ns = src_mtime_ns;
    for (int m = 0; m < t->order; ++m) h.dims[m] = t->dims[m];
    const std::vector<Span> sp = spans_of(t);
    const std::vector<Piece> pc = pieces_of(sp);
    std::vector<uint64_t> ph(pc.size());
    const int nt = std::max(1, std::min<int>(host_threads(), (int)pc.size()));
  #pragma omp parallel for num_threads(nt) schedule(static)
    for (int64_t i = 0; i < (int64_t)pc.size(); ++i)
      ph[i] = fnv_words(sp[pc[i].span].mem + pc[i].begin, pc[i].end - pc[i].begin);
    h.hash = combine(ph);
  
    // Written under a temporary name and renamed into place, so a reader (say
    // another rank of the same job) sees the old file or the whole new one.
    const std::string tmp = std::string(path) + ".tmp." + std::to_string((long)::getpid());
    const int fd = ::open(tmp.c_str(), O_WRONLY | O_CREAT | O_TRUNC, 0644);
    if (fd < 0) {
      set_host_error("cptc_bin_write: cannot create the cache file");
      return -1;
    }
    const uint64_t total = file_bytes(t->order, t->nnz);
    bool ok = ::ftruncate(fd, (off_t)total) == 0 && write_all(fd, &h, sizeof(h), 0);
    int bad = 0;
    // Chunks written by all threads at their offsets (the padding between
    // arrays stays the zeros of the ftruncate); on the 200 MB/s disk of the
    // build machine this took 8.5 s for config 4, one sequential stream 22 s.
  #pragma omp parallel for num_threads(nt) schedule(static) reduction(| : bad)
    for (int64_t i = 0; i < (int64_t)pc.size(); ++i) {
      const Span& s = sp[pc[i].span];
      if (!write_all(fd, s.mem + pc[i].begin, pc[i].end - pc[i].begin, s.off + pc[i].begin))
        bad |= 1;
    }
    ok = ok && !bad;
    ok = (::close(fd) == 0) && ok;
    if (!ok || std::rename(tmp.c_str(), path) != 0) {
      ::unlink(tmp.c_str());
      set_host_error("cptc_bin_write: write failed");
      return -1;
    }
    return 0;
  });
}

int cptc_bin_read(const char* path, cptc_coo* out, uint64_t* src_size, int64_t* src_mtime_ns) {
  return host_guard(out, [&]() -> int {
    if (!out) return -2;
    std::memset(out, 0, sizeof(*out));
    const int fd = ::open(path, O_RDONLY);
    if (fd < 0) {
      set_host_error("cptc_bin_read: cannot open the cache file");
      return -1;
    }
    struct stat st;
    if (::fstat(fd, &st) != 0 || (uint64_t)st.st_size < kHeader) {
      ::close(fd);
      set_host_error("cptc_bin_read: not a tensor cache (too short)");
      return -4;
    }
    const uint64_t fsz = (uint64_t)st.st_size;
    void* mp = ::mmap(nullptr, (size_t)fsz, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (mp == MAP_FAILED) {
      set_host_error("cptc_bin_read: mmap failed");
      return -1;
    }
    struct Unmap {
      void* p;
      size_t n;
      ~Unmap() { ::munmap(p, n); }
    } unmap{mp, (size_t)fsz};
    const unsigned char* base = (const unsigned char*)mp;
    Header h;
    std::memcpy(&h, base, sizeof(h));
    if (std::memcmp(h.magic, kMagic, 8) != 0 || h.order < 1 || h.order > CPTC_MAX_ORDER ||
        h.nnz > (fsz / 12) || file_bytes((int)h.order, h.nnz) != fsz) {
      set_host_error("cptc_bin_read: not a tensor cache, or truncated");
      return -4;
    }
    if (!coo_alloc(out, (int)h.order, h.nnz)) {
      cptc_coo_free(out);
      set_host_error("cptc_bin_read: out of host memory");
      return -3;
    }
    for (int m = 0; m < (int)h.order; ++m) out->dims[m] = h.dims[m];
    ::madvise(mp, (size_t)fsz, MADV_SEQUENTIAL);
    const std::vector<Span> sp = spans_of(out);
    const std::vector<Piece> pc = pieces_of(sp);
    std::vector<uint64_t> ph(pc.size());
    const int nt = std::max(1, std::min<int>(host_threads(), (int)pc.size()));
    // Copy and hash chunk by chunk (the destination pages are first touched by
    // the thread that fills them).
  #pragma omp parallel for num_threads(nt) schedule(static)
    for (int64_t i = 0; i < (int64_t)pc.size(); ++i) {
      const Span& s = sp[pc[i].span];
      const uint64_t n = pc[i].end - pc[i].begin;
      std::memcpy(s.mem + pc[i].begin, base + s.off + pc[i].begin, (size_t)n);
      ph[i] = fnv_words(s.mem + pc[i].begin, n);
    }
    if (combine(ph) != h.hash) {
      cptc_coo_free(out);
      std::memset(out, 0, sizeof(*out));
      set_host_error("cptc_bin_read: payload hash mismatch (corrupt cache)");
      return -4;
    }
    // Indices must lie inside the recorded dims (a consumer indexes factor
    // rows with them).
    uint64_t viol = 0;
    for (int m = 0; m < (int)h.order; ++m) {
      const uint32_t* ix = out->idx[m];
      const uint64_t d = h.dims[m];
  #pragma omp parallel for num_threads(nt) schedule(static) reduction(+ : viol)
      for (int64_t e = 0; e < (int64_t)h.nnz; ++e) viol += (uint64_t)(ix[e] >= d);
    }
    if (viol) {
      cptc_coo_free(out);
      std::memset(out, 0, sizeof(*out));
      set_host_error("cptc_bin_read: index outside the recorded dims");
      return -4;
    }
    if (src_size) *src_size = h.src_size;
    if (src_mtime_ns) *src_mtime_ns = h.src_mtime_ns;
    return 0;
  });
}

int cptc_tns_read_cached(const char* path, int order_hint, const char* cache_path,
                         cptc_coo* out, int* from_cache) {
  return host_guard(out, [&]() -> int {
    if (!path || !out) return -2;
    if (from_cache) *from_cache = 0;
    const std::string cp = cache_path && *cache_path ? std::string(cache_path)
                                                     : std::string(path) + ".cptcbin";
    uint64_t size = 0;
    int64_t mtime = 0;
    if (!file_stamp(path, &size, &mtime)) {
      std::memset(out, 0, sizeof(*out));
      set_host_error("cptc_tns_read_cached: cannot stat the .tns file");
      return -1;
    }
    // The order the text would be parsed with (the cache may have been made
    // with another hint).
    const int order = order_hint > 0 ? order_hint : cptc_tns_probe_order(path);
    uint64_t csize = 0;
    int64_t cmtime = 0;
    if (cptc_bin_read(cp.c_str(), out, &csize, &cmtime) == 0) {
      if (csize == size && cmtime == mtime && out->order == order) {
        if (from_cache) *from_cache = 1;
        return 0;
      }
      cptc_coo_free(out);  // stale: made from another version of the text
    }
    const int rc = cptc_tns_read(path, order_hint, out);
    if (rc != 0) return rc;
    // Best effort: a cache that cannot be written leaves the parse result.
    (void)cptc_bin_write(cp.c_str(), out, size, mtime);
    return 0;
  });
}

}  // extern "C"
