// FROSTT .tns reader and writer.
//
// Parse rules follow the reference loaders (src/tensor.cu:98-185 and
// src/generic.cu:1064-1099): lines starting with '#' are comments; blanks
// and tabs separate fields; a line whose coordinates are not all digit
// strings or whose value does not parse is skipped; indices are 1-based and
// an index of 0 maps to 0; dims[m] = largest 0-based index + 1.
// The file is mapped read-only and parsed by all host threads on
// newline-aligned chunks (a last line without a newline is parsed from a
// small padded copy, so no parse reads past the mapping); the per-thread
// results are copied into the output arrays in parallel, and the nonzeros
// keep file order.
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

static thread_local std::string g_tns_err;

static inline bool is_blank(char c) { return c == ' ' || c == '\t'; }

// Number of whitespace-separated fields of the first data line, minus one.
static int probe_order(const char* p, const char* end) {
  while (p < end) {
    const char* nl = (const char*)std::memchr(p, '\n', (size_t)(end - p));
    if (!nl) nl = end;
    const char* q = p;
    while (q < nl && is_blank(*q)) ++q;
    if (q < nl && *q != '#' && *q != '\r' && *q >= '0' && *q <= '9') {
      int fields = 0;
      while (q < nl && *q != '\r') {
        while (q < nl && is_blank(*q)) ++q;
        if (q >= nl || *q == '\r') break;
        ++fields;
        while (q < nl && !is_blank(*q) && *q != '\r') ++q;
      }
      return fields - 1;
    }
    p = nl + 1;
  }
  return -1;
}

struct Part {
  std::vector<uint32_t> idx[CPTC_MAX_ORDER];
  std::vector<double> val;
  uint64_t mx[CPTC_MAX_ORDER] = {0};
};

static void parse_range(const char* p, const char* end, int N, Part& out) {
  // Lines in the range bound the nonzeros: reserve once.
  size_t lines = 0;
  for (const char* c = p; c < end;) {
    const char* nl = (const char*)std::memchr(c, '\n', (size_t)(end - c));
    ++lines;
    if (!nl) break;
    c = nl + 1;
  }
  for (int m = 0; m < N; ++m) out.idx[m].reserve(lines);
  out.val.reserve(lines);
  uint32_t ix[CPTC_MAX_ORDER];
  while (p < end) {
    const char* nl = (const char*)std::memchr(p, '\n', (size_t)(end - p));
    if (!nl) nl = end;
    const char* q = p;
    p = nl + 1;
    if (q >= nl || *q == '#') continue;
    bool ok = true;
    for (int m = 0; m < N && ok; ++m) {
      while (q < nl && is_blank(*q)) ++q;
      if (q >= nl || *q < '0' || *q > '9') {
        ok = false;
        break;
      }
      uint64_t v = 0;
      while (q < nl && *q >= '0' && *q <= '9') v = v * 10 + (uint64_t)(*q++ - '0');
      ix[m] = v > 0 ? (uint32_t)(v - 1) : 0u;
    }
    if (!ok) continue;
    while (q < nl && is_blank(*q)) ++q;
    if (q >= nl || *q == '\r') continue;  // no value on this line
    char* endc = nullptr;
    const double val = std::strtod(q, &endc);
    if (endc == q) continue;
    for (int m = 0; m < N; ++m) {
      out.idx[m].push_back(ix[m]);
      if (ix[m] > out.mx[m]) out.mx[m] = ix[m];
    }
    out.val.push_back(val);
  }
}

}  // namespace cptc

using namespace cptc;

extern "C" {

int cptc_tns_probe_order(const char* path) {
  return host_guard(nullptr, [&]() -> int {
    FILE* f = std::fopen(path, "rb");
    if (!f) return -1;
    std::vector<char> buf(1 << 16);
    const size_t got = std::fread(buf.data(), 1, buf.size(), f);
    std::fclose(f);
    return probe_order(buf.data(), buf.data() + got);
  });
}

int cptc_tns_read(const char* path, int order_hint, cptc_coo* out) {
  return host_guard(out, [&]() -> int {
    if (!out) return -2;
    std::memset(out, 0, sizeof(*out));
    const int fd = ::open(path, O_RDONLY);
    if (fd < 0) return -1;
    struct stat st;
    if (::fstat(fd, &st) != 0) {
      ::close(fd);
      return -1;
    }
    const size_t fsz = (size_t)st.st_size;
    const char* map = nullptr;
    if (fsz > 0) {
      void* mp = ::mmap(nullptr, fsz, PROT_READ, MAP_PRIVATE, fd, 0);
      if (mp == MAP_FAILED) {
        ::close(fd);
        return -1;
      }
      map = (const char*)mp;
      ::madvise(mp, fsz, MADV_SEQUENTIAL);
    }
    ::close(fd);
    struct Unmap {
      const char* p;
      size_t n;
      ~Unmap() {
        if (p) ::munmap((void*)p, n);
      }
    } unmap{map, fsz};
    // Everything up to the last newline is parsed in place; a final line
    // without a newline goes through a copy that ends with one.
    size_t body = fsz;
    while (body > 0 && map[body - 1] != '\n') --body;
    std::vector<char> tail(map + body, map + fsz);
    tail.push_back('\n');
    const char* b = map;
    const char* e = map + body;
    int N = order_hint;
    if (N <= 0) {
      N = probe_order(b, e);
      if (N < 0) N = probe_order(tail.data(), tail.data() + tail.size());
    }
    if (N < 1 || N > CPTC_MAX_ORDER) return -2;
  
    const int nt = std::max(1, std::min(host_threads(), (int)(body >> 20) + 1));
    std::vector<const char*> cut(nt + 1);
    cut[0] = b;
    cut[nt] = e;
    for (int t = 1; t < nt; ++t) {
      const char* c = b + (body * (size_t)t) / (size_t)nt;
      if (c < cut[t - 1]) c = cut[t - 1];
      const char* nl = (const char*)std::memchr(c, '\n', (size_t)(e - c));
      cut[t] = nl ? nl + 1 : e;
    }
    std::vector<Part> parts(nt + 1);
  #pragma omp parallel for num_threads(nt) schedule(static, 1)
    for (int t = 0; t < nt; ++t) parse_range(cut[t], cut[t + 1], N, parts[t]);
    parse_range(tail.data(), tail.data() + tail.size(), N, parts[nt]);
  
    uint64_t nnz = 0;
    std::vector<uint64_t> off(parts.size() + 1, 0);
    for (size_t t = 0; t < parts.size(); ++t) off[t + 1] = off[t] + parts[t].val.size();
    nnz = off[parts.size()];
    if (!coo_alloc(out, N, nnz)) {
      cptc_coo_free(out);
      return -3;
    }
    // Parallel copy: the output pages are first touched by many threads.
  #pragma omp parallel for num_threads(nt) schedule(dynamic, 1)
    for (int t = 0; t < (int)parts.size(); ++t) {
      const Part& p = parts[t];
      if (p.val.empty()) continue;
      for (int m = 0; m < N; ++m)
        std::memcpy(out->idx[m] + off[t], p.idx[m].data(), p.val.size() * sizeof(uint32_t));
      std::memcpy(out->vals + off[t], p.val.data(), p.val.size() * sizeof(double));
    }
    for (const Part& p : parts)
      for (int m = 0; m < N; ++m)
        if (!p.val.empty()) out->dims[m] = std::max<uint64_t>(out->dims[m], p.mx[m] + 1);
    for (int m = 0; m < N; ++m)
      if (out->dims[m] == 0) out->dims[m] = 1;
    return 0;
  });
}

int cptc_tns_write(const char* path, const cptc_coo* t) {
  return host_guard(nullptr, [&]() -> int {
    if (!t || t->order < 1 || t->order > CPTC_MAX_ORDER) return -2;
    FILE* f = std::fopen(path, "wb");
    if (!f) return -1;
    const int N = t->order;
    const uint64_t nnz = t->nnz;
    const uint64_t block = 1 << 20;
    const int nt = host_threads();
    std::vector<std::string> out((size_t)nt);
    for (uint64_t s = 0; s < nnz; s += block * (uint64_t)nt) {
  #pragma omp parallel for num_threads(nt) schedule(static, 1)
      for (int th = 0; th < nt; ++th) {
        std::string& o = out[th];
        o.clear();
        const uint64_t a = s + (uint64_t)th * block;
        const uint64_t z = std::min(nnz, a + block);
        char line[256];
        for (uint64_t e = a; e < z; ++e) {
          int n = 0;
          for (int m = 0; m < N; ++m)
            n += std::snprintf(line + n, sizeof(line) - n, "%u ", t->idx[m][e] + 1u);
          n += std::snprintf(line + n, sizeof(line) - n, "%.17g\n", t->vals[e]);
          o.append(line, (size_t)n);
        }
      }
      for (int th = 0; th < nt; ++th) std::fwrite(out[th].data(), 1, out[th].size(), f);
    }
    return std::fclose(f) == 0 ? 0 : -1;
  });
}

}  // extern "C"
