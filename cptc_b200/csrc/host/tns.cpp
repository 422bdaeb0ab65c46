// FROSTT .tns reader and writer.
//
// Parse rules follow the reference loaders (src/tensor.cu:98-185 and
// src/generic.cu:1064-1099): lines starting with '#' are comments; blanks
// and tabs separate fields; a line whose coordinates are not all digit
// strings or whose value does not parse is skipped; indices are 1-based and
// an index of 0 maps to 0; dims[m] = largest 0-based index + 1.
// The file is parsed by all host threads on newline-aligned chunks and the
// nonzeros keep file order.
#include <omp.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "coo.hpp"

namespace cptc {

static thread_local std::string g_tns_err;

static bool read_file(const char* path, std::vector<char>& buf) {
  FILE* f = std::fopen(path, "rb");
  if (!f) return false;
  std::fseek(f, 0, SEEK_END);
  const long sz = std::ftell(f);
  std::fseek(f, 0, SEEK_SET);
  buf.resize((size_t)(sz > 0 ? sz : 0) + 1);
  const size_t got = sz > 0 ? std::fread(buf.data(), 1, (size_t)sz, f) : 0;
  std::fclose(f);
  buf.resize(got + 1);
  buf[got] = '\n';  // sentinel: every line ends with '\n'
  return true;
}

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
  FILE* f = std::fopen(path, "rb");
  if (!f) return -1;
  std::vector<char> buf(1 << 16);
  const size_t got = std::fread(buf.data(), 1, buf.size(), f);
  std::fclose(f);
  return probe_order(buf.data(), buf.data() + got);
}

int cptc_tns_read(const char* path, int order_hint, cptc_coo* out) {
  if (!out) return -2;
  std::memset(out, 0, sizeof(*out));
  std::vector<char> buf;
  if (!read_file(path, buf)) return -1;
  const char* b = buf.data();
  const char* e = b + buf.size();
  const int N = order_hint > 0 ? order_hint : probe_order(b, e);
  if (N < 1 || N > CPTC_MAX_ORDER) return -2;

  const int nt = std::max(1, std::min(host_threads(), (int)(buf.size() >> 20) + 1));
  std::vector<const char*> cut(nt + 1);
  cut[0] = b;
  cut[nt] = e;
  for (int t = 1; t < nt; ++t) {
    const char* c = b + (buf.size() * (size_t)t) / (size_t)nt;
    if (c < cut[t - 1]) c = cut[t - 1];
    const char* nl = (const char*)std::memchr(c, '\n', (size_t)(e - c));
    cut[t] = nl ? nl + 1 : e;
  }
  std::vector<Part> parts(nt);
#pragma omp parallel for num_threads(nt) schedule(static, 1)
  for (int t = 0; t < nt; ++t) parse_range(cut[t], cut[t + 1], N, parts[t]);

  uint64_t nnz = 0;
  for (auto& p : parts) nnz += p.val.size();
  if (!coo_alloc(out, N, nnz)) {
    cptc_coo_free(out);
    return -3;
  }
  uint64_t off = 0;
  for (auto& p : parts) {
    for (int m = 0; m < N; ++m) {
      if (!p.val.empty())
        std::memcpy(out->idx[m] + off, p.idx[m].data(), p.val.size() * sizeof(uint32_t));
      out->dims[m] = std::max<uint64_t>(out->dims[m], p.mx[m] + 1);
    }
    if (!p.val.empty())
      std::memcpy(out->vals + off, p.val.data(), p.val.size() * sizeof(double));
    off += p.val.size();
  }
  for (int m = 0; m < N; ++m)
    if (out->dims[m] == 0) out->dims[m] = 1;
  return 0;
}

int cptc_tns_write(const char* path, const cptc_coo* t) {
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
}

}  // extern "C"
