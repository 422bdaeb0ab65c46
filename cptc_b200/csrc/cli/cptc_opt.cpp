// cptc_opt — command-line driver with the reference's surface
// (src/main.cu:22-680):
//
//   cptc_opt <tns> [iters=20] [R=32] [threshold=0.03]
//
// Order-3 tensors run the hybrid pipeline (CADR, dense 16^3 tiles in TF32 +
// FP64 residual, or FP64 only, chosen by the fill-rate selector); any other
// order, or ALS_GENERIC_FORCE=1, runs the N-order path.  Switches honoured:
//   ALS_FORCE_WMMA, ALS_FORCE_CUDA, ALS_FILL_MIN, ALS_GENERIC_FORCE,
//   ALS_EXPORT_FACTORS, ALS_PROFILE,
//   GEN_DENSE, GEN_DENSE_THRESHOLD, GEN_DENSE_INNER, GEN_REORDER,
//   GEN_REORDER_T, GEN_REORDER_SAMPLE, GEN_SOLVER, GEN_SEED, GEN_DUMP,
//   GEN_PROFILE, GEN_SELFTEST (the N-order dense-path known-answer test,
//   src/generic.cu:1389-1637, then exit), CPTC_DEVICE, CPTC_TNS_CACHE
//   (binary copy of the parsed tensor beside the .tns, used while the text
//   is unchanged), CPTC_NGPU (one process per GPU on devices CPTC_DEVICE..,
//   NCCL between them).
// Output lines keep the reference's formats ("[ALS] iter i/N time=<ms> ms
// fit=<f>", "[GEN] iter ... fit=", "[ALS] Lambda:", export files).
#include <signal.h>
#include <sys/prctl.h>
#include <sys/wait.h>
#include <unistd.h>

#include <chrono>
#include <cmath>
#include <random>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "cptc.h"

namespace {

const char* env(const char* k) { return std::getenv(k); }

// Several GPUs from the command line (CPTC_NGPU=G > 1; the reference runs on
// one GPU): one process per GPU, forked at the start of main, before any
// OpenMP thread pool or CUDA context exists (neither survives a fork).
// Rank 0 makes the NCCL id and writes it into a pipe per child; every rank
// runs the same calls (the ALS is collective), rank 0 alone prints and
// exports.  A rank that fails ends the job: rank 0 watches its children and
// stops the others, and children die with rank 0.
std::vector<pid_t> g_kids;  // rank 0 only
std::thread g_watch;
int g_watch_rc = 0;

void stop_kids() {
  for (pid_t k : g_kids) kill(k, SIGTERM);
}

// Reaps every child; the first one that fails stops the rest and ends rank 0.
void watch_kids() {
  size_t left = g_kids.size();
  while (left > 0) {
    int st = 0;
    const pid_t p = waitpid(-1, &st, 0);
    if (p < 0) break;
    --left;
    if (!WIFEXITED(st) || WEXITSTATUS(st) != 0) {
      std::fprintf(stderr, "[cptc] a rank (pid %d) failed; stopping the job\n", (int)p);
      stop_kids();
      std::fflush(stdout);
      _exit(1);
    }
  }
}

bool write_all(int fd, const void* p, size_t n) {
  const char* c = (const char*)p;
  while (n > 0) {
    const ssize_t w = write(fd, c, n);
    if (w <= 0) return false;
    c += w;
    n -= (size_t)w;
  }
  return true;
}

bool read_all(int fd, void* p, size_t n) {
  char* c = (char*)p;
  while (n > 0) {
    const ssize_t r = read(fd, c, n);
    if (r <= 0) return false;
    c += r;
    n -= (size_t)r;
  }
  return true;
}

// Forks ranks 1..G-1; returns this process's rank (-1 on failure) and, in the
// children, the read end of their id pipe; in rank 0 the write ends.
int fork_ranks(int G, std::vector<int>& id_out, int& id_in) {
  std::fflush(stdout);
  std::fflush(stderr);
  const pid_t parent = getpid();
  for (int r = 1; r < G; ++r) {
    int fd[2];
    if (pipe(fd) != 0) return -1;
    const pid_t pid = fork();
    if (pid < 0) return -1;
    if (pid == 0) {
      prctl(PR_SET_PDEATHSIG, SIGKILL);
      if (getppid() != parent) _exit(1);
      close(fd[1]);
      for (int w : id_out) close(w);
      id_out.clear();
      g_kids.clear();
      id_in = fd[0];
      if (!std::freopen("/dev/null", "w", stdout)) _exit(1);
      return r;
    }
    close(fd[0]);
    id_out.push_back(fd[1]);
    g_kids.push_back(pid);
  }
  g_watch = std::thread(watch_kids);
  return 0;
}

struct IterLog {
  bool generic = false;
  int iters = 0;
  bool profile = false;
  cptc_ctx* ctx = nullptr;
};

void on_iter(int it, double ms, double fit, const double* mode_ms, int nm, void* user) {
  IterLog* L = (IterLog*)user;
  if (!L->generic) {
    std::printf("[ALS] iter %d/%d time=%g ms fit=%g\n", it, L->iters, ms, fit);
    if (L->profile) {
      std::printf("[ALS][profile] iter %d mttkrp=", it);
      for (int m = 0; m < nm; ++m) std::printf("%s%g", m ? "/" : "", mode_ms[m]);
      std::printf(" ms (iter=%g)\n", ms);
    }
  } else {
    double t[3] = {0, 0, 0};
    cptc_fit_terms(L->ctx, t);
    std::printf("[GEN] iter %d/%d time=%g ms iprod=%g model2=%g fit=%g\n", it, L->iters, ms,
                t[0], t[1], fit);
    if (L->profile) {
      std::printf("[GEN][profile] iter %d mttkrp=", it);
      for (int m = 0; m < nm; ++m) std::printf("%s%g", m ? "/" : "", mode_ms[m]);
      std::printf(" ms\n");
    }
  }
  std::fflush(stdout);
}

int fail(cptc_ctx* c, const char* what, int rc) {
  std::fprintf(stderr, "[cptc] %s failed (%d): %s\n", what, rc, c ? cptc_last_error(c) : "");
  std::fflush(stdout);
  if (!g_kids.empty()) {  // rank 0: the other ranks cannot finish without it
    stop_kids();
    _exit(1);
  }
  return 1;
}

int reorder_of(const char* s) {
  if (!s) return CPTC_REORDER_DEFAULT;
  if (!std::strcmp(s, "none")) return CPTC_REORDER_NONE;
  if (!std::strcmp(s, "cadr")) return CPTC_REORDER_CADR;
  if (!std::strcmp(s, "hits")) return CPTC_REORDER_HITS;
  if (!std::strcmp(s, "auto")) return CPTC_REORDER_AUTO;
  std::fprintf(stderr, "[GEN] unknown GEN_REORDER=%s -> falling back to cadr\n", s);
  return CPTC_REORDER_CADR;
}

// GEN_SELFTEST: the reference's known-answer test of the N-order dense path
// (src/generic.cu:1389-1637).  The same order-4 tensor (40 x 24 x 36 x 3,
// drawn from mt19937(1234) in the reference's order: two ~50%-full tiles per
// outer slice, the partial corner tile at ~60%, 4000 scattered nonzeros),
// the same factors, R = 8; for each inner-mode set and each pass (every
// nonzero in dense units, then units at cutoff 0.01 plus the FP64 residual)
// the engine's MTTKRP of every inner mode is compared with an exact host
// MTTKRP by relative L2 error, bound 2e-3.  Returns the exit status.
int run_selftest(int dev) {
  const int N = 4, R = 8;
  const int dims[4] = {40, 24, 36, 3};
  std::vector<uint32_t> co[4];
  std::vector<double> vals;
  std::mt19937 gen(1234);
  std::uniform_real_distribution<double> uv(0.0, 1.0);
  auto add = [&](int i, int j, int k, int l, double v) {
    co[0].push_back((uint32_t)i);
    co[1].push_back((uint32_t)j);
    co[2].push_back((uint32_t)k);
    co[3].push_back((uint32_t)l);
    vals.push_back(v);
  };
  const int tb[2][3] = {{0, 0, 0}, {1, 0, 1}};
  for (int l = 0; l < dims[3]; ++l)
    for (int t = 0; t < 2; ++t)
      for (int a = 0; a < 16; ++a)
        for (int b = 0; b < 16; ++b)
          for (int c = 0; c < 16; ++c)
            if (uv(gen) < 0.5) add(tb[t][0] * 16 + a, tb[t][1] * 16 + b, tb[t][2] * 16 + c, l, 1.0 + uv(gen));
  for (int l = 0; l < dims[3]; ++l)
    for (int a = 32; a < dims[0]; ++a)
      for (int b = 16; b < dims[1]; ++b)
        for (int c = 32; c < dims[2]; ++c)
          if (uv(gen) < 0.6) add(a, b, c, l, 1.0 + uv(gen));
  // The reference draws these five numbers as the arguments of one call,
  // which its host compiler (g++) evaluates last argument first: the value,
  // then the indices from the last mode to the first.
  for (int e = 0; e < 4000; ++e) {
    const double v = 1.0 + uv(gen);
    const int l = (int)(uv(gen) * dims[3]) % dims[3];
    const int k = (int)(uv(gen) * dims[2]) % dims[2];
    const int j = (int)(uv(gen) * dims[1]) % dims[1];
    const int i = (int)(uv(gen) * dims[0]) % dims[0];
    add(i, j, k, l, v);
  }
  const size_t nnz = vals.size();
  std::printf("[SELFTEST] N=%d dims=%d,%d,%d,%d nnz=%zu R=%d\n", N, dims[0], dims[1], dims[2],
              dims[3], nnz, R);
  std::vector<double> F[4];
  for (int m = 0; m < N; ++m) {
    F[m].resize((size_t)dims[m] * R);
    for (double& x : F[m]) x = uv(gen);
  }
  std::vector<double> exact[4];
  for (int n = 0; n < N; ++n) {
    exact[n].assign((size_t)dims[n] * R, 0.0);
    for (size_t e = 0; e < nnz; ++e)
      for (int r = 0; r < R; ++r) {
        double q = vals[e];
        for (int m = 0; m < N; ++m)
          if (m != n) q *= F[m][(size_t)co[m][e] * R + r];
        exact[n][(size_t)co[n][e] * R + r] += q;
      }
  }
  cptc_coo t{};
  t.order = N;
  t.nnz = nnz;
  for (int m = 0; m < N; ++m) {
    t.dims[m] = (uint64_t)dims[m];
    t.idx[m] = co[m].data();
  }
  t.vals = vals.data();
  cptc_ctx* c = nullptr;
  int rc = cptc_create(&c, dev, 0);
  if (rc) return fail(c, "cptc_create", rc);
  if ((rc = cptc_load_coo(c, &t))) return fail(c, "load", rc);
  int fails = 0;
  const int sets[4][3] = {{0, 1, 2}, {1, 2, 3}, {0, 1, 3}, {0, 2, 3}};
  for (int si = 0; si < 4; ++si)
    for (int pass = 0; pass < 2; ++pass) {
      const int* in = sets[si];
      std::printf("[SELFTEST] --- inner=(%d,%d,%d) pass %d (%s) ---\n", in[0], in[1], in[2], pass,
                  pass == 0 ? "dense-only" : "mixed dense+FP64");
      cptc_opts o;
      cptc_opts_default(&o);
      o.generic = 1;
      o.reorder = CPTC_REORDER_NONE;
      o.dense_generic = 1;
      // cutoff int(4096 * thr): 0 puts every unit on the dense path
      o.dense_thr_generic = pass == 0 ? 1e-12 : 0.01;
      for (int q = 0; q < 3; ++q) o.dense_inner[q] = in[q];
      if ((rc = cptc_build(c, R, 0.03, &o))) return fail(c, "build", rc);
      for (int m = 0; m < N; ++m)
        if ((rc = cptc_set_factors(c, m, F[m].data()))) return fail(c, "set_factors", rc);
      cptc_stats st;
      cptc_get_stats(c, &st);
      std::printf("[SELFTEST]   units=%llu dense_nnz=%llu (%.1f%%)\n",
                  (unsigned long long)st.dense_tiles, (unsigned long long)st.dense_nnz,
                  100.0 * (double)st.dense_nnz / (double)nnz);
      for (int q = 0; q < 3; ++q) {
        const int n = in[q];
        std::vector<double> got((size_t)dims[n] * R);
        if ((rc = cptc_mttkrp(c, n, got.data()))) return fail(c, "mttkrp", rc);
        double num = 0.0, den = 0.0;
        for (size_t i = 0; i < got.size(); ++i) {
          const double d = got[i] - exact[n][i];
          num += d * d;
          den += exact[n][i] * exact[n][i];
        }
        const double rel = den > 0.0 ? std::sqrt(num / den) : 0.0;
        const bool ok = rel < 2e-3;
        std::printf("[SELFTEST]   mode %d: relative L2 error = %.3e  %s\n", n, rel,
                    ok ? "OK" : "FAIL");
        if (!ok) ++fails;
      }
    }
  std::printf("[SELFTEST] %s (%d failures)\n", fails ? "FAILED" : "PASSED", fails);
  std::fflush(stdout);
  cptc_destroy(c);
  return fails ? 1 : 0;
}

}  // namespace

int main(int argc, char** argv) {
  std::string filename = "nell-2.tns";
  int iters = 20, R = 32;
  double threshold = 0.03;
  if (argc > 1) filename = argv[1];
  if (argc > 2) iters = std::atoi(argv[2]);
  if (argc > 3) R = std::atoi(argv[3]);
  if (argc > 4) threshold = std::atof(argv[4]);
  if (iters <= 0) iters = 1;
  if (R <= 0) R = 1;
  if (env("GEN_SELFTEST"))  // src/main.cu:89-91: the known-answer test, then exit
    return run_selftest(env("CPTC_DEVICE") ? std::atoi(env("CPTC_DEVICE")) : 0);

  // The ranks are forked before anything else runs (no OpenMP pool, no CUDA
  // context exists yet); each parses the tensor itself.
  const int ngpu = env("CPTC_NGPU") ? std::max(1, std::atoi(env("CPTC_NGPU"))) : 1;
  int rank = 0;
  std::vector<int> id_out;
  int id_in = -1;
  if (ngpu > 1) {
    rank = fork_ranks(ngpu, id_out, id_in);
    if (rank < 0) {
      std::fprintf(stderr, "[cptc] cannot start %d ranks\n", ngpu);
      return fail(nullptr, "fork", -1);
    }
  }

  const int order = cptc_tns_probe_order(filename.c_str());
  if (order < 0) {
    std::fprintf(stderr, "[Main] cannot determine tensor order of: %s\n", filename.c_str());
    return fail(nullptr, "probe", -1);
  }
  const bool generic = (order != 3) || env("ALS_GENERIC_FORCE");

  const auto t0 = std::chrono::steady_clock::now();
  cptc_coo t{};
  // CPTC_TNS_CACHE=1 keeps a binary copy beside the text (<tns>.cptcbin);
  // any other non-empty value names the copy.
  const char* cache = env("CPTC_TNS_CACHE");
  const bool use_cache = cache && *cache && std::strcmp(cache, "0") != 0;
  int from_cache = 0;
  const int lrc = use_cache ? cptc_tns_read_cached(filename.c_str(), order,
                                                   std::strcmp(cache, "1") ? cache : nullptr,
                                                   &t, &from_cache)
                            : cptc_tns_read(filename.c_str(), order, &t);
  if (lrc != 0) {
    std::fprintf(stderr, "[Error] Cannot open file: %s\n", filename.c_str());
    return fail(nullptr, "read", lrc);
  }
  const double load_ms =
      std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
  if (generic) {
    std::printf("[Main] order-%d tensor -> generic N-order CP-ALS\n", order);
    std::printf("[Main] Load time = %g ms | dims = ", load_ms);
    for (int m = 0; m < order; ++m) std::printf("%s%llu", m ? " x " : "", (unsigned long long)t.dims[m]);
    std::printf(" | NNZ = %llu\n", (unsigned long long)t.nnz);
  } else {
    std::printf("[Main] Load time = %g ms\n", load_ms);
    std::printf("[Main] Tensor Dimensions: %llu x %llu x %llu | NNZ: %llu\n",
                (unsigned long long)t.dims[0], (unsigned long long)t.dims[1],
                (unsigned long long)t.dims[2], (unsigned long long)t.nnz);
  }
  if (use_cache)
    std::printf("[Main] binary cache: %s\n", from_cache ? "read" : "written from the text");

  cptc_opts o;
  cptc_opts_default(&o);
  o.generic = generic ? 1 : 0;
  if (env("ALS_FORCE_WMMA")) o.path = CPTC_PATH_TF32;
  else if (env("ALS_FORCE_CUDA")) o.path = CPTC_PATH_FP64;
  if (env("ALS_FILL_MIN")) o.fill_min = std::atof(env("ALS_FILL_MIN"));
  if (generic) {
    o.reorder = reorder_of(env("GEN_REORDER"));
    if (env("GEN_REORDER_T")) o.reorder_rounds = std::max(1, std::atoi(env("GEN_REORDER_T")));
    if (env("GEN_REORDER_SAMPLE"))
      o.reorder_sample = std::strtoull(env("GEN_REORDER_SAMPLE"), nullptr, 10);
    if (env("GEN_SOLVER") && !std::strcmp(env("GEN_SOLVER"), "svd")) o.solver = CPTC_SOLVER_PINV;
    if (env("GEN_SEED")) o.seed = (uint32_t)std::atoi(env("GEN_SEED"));
    if (env("GEN_DENSE")) o.dense_generic = std::atoi(env("GEN_DENSE")) != 0;
    if (env("GEN_DENSE_THRESHOLD")) o.dense_thr_generic = std::atof(env("GEN_DENSE_THRESHOLD"));
    if (const char* s = env("GEN_DENSE_INNER")) {
      int k = 0;
      const char* q = s;
      while (*q && k < 3) {
        o.dense_inner[k++] = std::atoi(q);
        while (*q && *q != ',') ++q;
        if (*q == ',') ++q;
      }
    }
  }

  unsigned char id[128];
  if (ngpu > 1) {
    if (rank == 0) {
      const int irc = cptc_comm_unique_id(id);
      for (int w : id_out) {
        if (irc == 0) write_all(w, id, sizeof(id));
        close(w);  // a child that reads nothing gives up
      }
      if (irc) return fail(nullptr, "cptc_comm_unique_id", irc);
    } else {
      const bool ok = read_all(id_in, id, sizeof(id));
      close(id_in);
      if (!ok) return 1;
    }
  }
  int dev = (env("CPTC_DEVICE") ? std::atoi(env("CPTC_DEVICE")) : 0) + rank;
  cptc_ctx* c = nullptr;
  int rc = cptc_create(&c, dev, 0);
  if (rc) return fail(c, "cptc_create", rc);
  if (ngpu > 1 && (rc = cptc_comm_init(c, id, rank, ngpu))) return fail(c, "comm_init", rc);
  if ((rc = cptc_load_coo(c, &t))) return fail(c, "load", rc);
  if ((rc = cptc_build(c, R, threshold, &o))) return fail(c, "build", rc);
  cptc_stats st;
  cptc_get_stats(c, &st);
  std::printf("[Main] build (reorder + partition + views) = %g ms\n", st.build_ms);
  if (!generic) {
    // The reference's selector line (src/main.cu:408-416), same labels and
    // texts: dense/sparse nonzeros, tiles, mean tile fill, dense nonzeros
    // weighted by the fill, the dense share, the threshold, the chosen path
    // (TF32 tiles + FP64 residual, or FP64 only).
    const double eff_dense = (double)st.dense_nnz * st.avg_fill;
    const double dense_ratio =
        st.nnz > 0 ? (double)st.dense_nnz / (double)(st.dense_nnz + st.sparse_nnz) : 0.0;
    std::printf("[Main] 稠密度检测: dense_nnz=%llu sparse_nnz=%llu "
                "tiles=%llu avg_fill=%g eff_dense=%g dense_ratio=%g (阈值 %g) -> %s\n",
                (unsigned long long)st.dense_nnz, (unsigned long long)st.sparse_nnz,
                (unsigned long long)st.dense_tiles, st.avg_fill, eff_dense, dense_ratio,
                st.fill_min,
                st.tf32_path ? "双流串行(WMMA+FP64)"
                             : "纯 CUDA core(全 FP64)");
    std::printf("[ALS] Starting CP-ALS: rank=%d, max_iters=%d\n", R, iters);
  } else {
    std::printf("[GEN] N-order CP-ALS: order=%d R=%d iters=%d nnz=%llu\n", order, R, iters,
                (unsigned long long)t.nnz);
    if (st.tf32_path)
      std::printf("[GEN] dense: units=%llu dense_nnz=%llu cutoff=%d\n",
                  (unsigned long long)st.dense_tiles, (unsigned long long)st.dense_nnz,
                  st.cutoff);
  }
  if ((rc = cptc_init_factors(c))) return fail(c, "init_factors", rc);
  IterLog L;
  L.generic = generic;
  L.iters = iters;
  L.ctx = c;
  L.profile = env(generic ? "GEN_PROFILE" : "ALS_PROFILE") != nullptr;
  const auto ta = std::chrono::steady_clock::now();
  if ((rc = cptc_als(c, iters, on_iter, &L))) return fail(c, "als", rc);
  const double als_ms =
      std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - ta).count();

  if (rank != 0) {  // the replicated results are reported and exported by rank 0
    cptc_destroy(c);
    cptc_coo_free(&t);
    return 0;
  }
  std::vector<double> lam(R);
  cptc_get_lambda(c, lam.data());
  double res[2] = {0, 0};
  cptc_residual(c, res);
  const double xn = std::sqrt(res[1]);
  const double rmse = t.nnz ? std::sqrt(std::max(res[0], 0.0) / (double)t.nnz) : 0.0;
  if (!generic) {
    std::printf("[ALS] Final RMSE=%g\n", rmse);
    std::printf("[ALS] Lambda:");
    for (int r = 0; r < R; ++r) std::printf(" %g", lam[r]);
    std::printf("\n[ALS] Total time=%g ms\n", als_ms);
  } else {
    const double rn = std::sqrt(std::max(res[0], 0.0));
    std::printf("[GEN] ALS total = %g ms\n", als_ms);
    std::printf("[GEN] exact: ||X-Xhat||_F=%g RMSE=%g fit=%g (||X||_F=%g)\n", rn, rmse,
                xn > 0 ? 1.0 - rn / xn : 0.0, xn);
    std::printf("[GEN] lambda = ");
    for (int r = 0; r < R; ++r) std::printf("%s%g", r ? " " : "", lam[r]);
    std::printf("\n");
  }

  if (const char* exp = env("ALS_EXPORT_FACTORS"); exp && !generic) {
    // src/main.cu:595-621: <p>.{0,1,2}.out (row-major, %.20lf) and <p>.lambda.out
    for (int n = 0; n < 3; ++n) {
      std::vector<double> f(t.dims[n] * (size_t)R);
      cptc_get_factors(c, n, f.data());
      std::string path = std::string(exp) + "." + std::to_string(n) + ".out";
      FILE* fp = std::fopen(path.c_str(), "w");
      if (!fp) continue;
      std::fprintf(fp, "matrix\n2\n%llu %d\n", (unsigned long long)t.dims[n], R);
      for (double v : f) std::fprintf(fp, "%.20lf\n", v);
      std::fclose(fp);
    }
    FILE* lf = std::fopen((std::string(exp) + ".lambda.out").c_str(), "w");
    if (lf) {
      std::fprintf(lf, "vector\n1\n%d\n", R);
      for (double v : lam) std::fprintf(lf, "%.20lf\n", v);
      std::fclose(lf);
    }
    std::printf("[Main] factors exported to %s\n", exp);
  }
  if (const char* dump = env("GEN_DUMP"); dump && generic) {
    // src/generic.cu:2253-2287: factors in the relabelled row order, 17 digits
    std::string path = std::string(dump) + ".factors.txt";
    FILE* fo = std::fopen(path.c_str(), "w");
    if (fo) {
      std::fprintf(fo, "# cpTC factor dump (factors are column-normalised; lambda holds the norms)\n");
      std::fprintf(fo, "order %d\nrank %d\ndims", order, R);
      for (int m = 0; m < order; ++m) std::fprintf(fo, " %llu", (unsigned long long)t.dims[m]);
      std::fprintf(fo, "\n");
      for (int m = 0; m < order; ++m) {
        const size_t d = t.dims[m];
        std::vector<double> f(d * R), g(d * R);
        std::vector<uint32_t> perm(d);
        cptc_get_factors(c, m, f.data());
        cptc_get_relabel(c, m, perm.data());
        for (size_t a = 0; a < d; ++a)
          std::memcpy(g.data() + (size_t)perm[a] * R, f.data() + a * R, R * sizeof(double));
        std::fprintf(fo, "mode %d %zu %d\n", m, d, R);
        for (size_t i = 0; i < d; ++i) {
          for (int r = 0; r < R; ++r) std::fprintf(fo, "%s%.17g", r ? " " : "", g[i * R + r]);
          std::fprintf(fo, "\n");
        }
      }
      std::fprintf(fo, "lambda %d\n", R);
      for (int r = 0; r < R; ++r) std::fprintf(fo, "%s%.17g", r ? " " : "", lam[r]);
      std::fprintf(fo, "\n");
      std::fclose(fo);
      std::printf("[GEN] factors dumped to %s\n", path.c_str());
    }
  }
  std::fflush(stdout);
  cptc_destroy(c);
  cptc_coo_free(&t);
  if (g_watch.joinable()) g_watch.join();  // every other rank has finished
  return 0;
}
