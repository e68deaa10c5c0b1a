// Shared helpers for the oracle/_ref wrappers (test and baseline infrastructure).
//
// Each wrapper translation unit #includes one of the reference's CPU driver
// files from the reference checkout (its main() renamed so it does not clash),
// then exports extern "C" entry points that call the driver's own tiled AVX2
// compute template exactly as the driver's testBlockSize() does: page-aligned
// per-thread A/B/C caches, C zero-initialised (the templates accumulate into C),
// and the template's own chrono window reported as the kernel time.
#pragma once
#include <cstdlib>
#include <cstring>
#include <unistd.h>
#include <omp.h>

namespace refwrap {

// Per-thread scratch caches, sized the way the reference drivers size them
// (gemm_benchmark.cpp:206-219): one page-rounded buffer per OpenMP thread.
struct ThreadCaches {
  int n = 0;
  float** a = nullptr;
  float** b = nullptr;
  float** c = nullptr;
  ThreadCaches(size_t a_elems, size_t b_elems, size_t c_elems) {
    n = omp_get_max_threads();
    long pg = sysconf(_SC_PAGESIZE);
    auto round = [pg](size_t bytes) { return ((bytes + pg - 1) / pg) * pg; };
    a = new float*[n];
    b = new float*[n];
    c = new float*[n];
    for (int t = 0; t < n; ++t) {
      a[t] = (float*)aligned_alloc(pg, round(a_elems * sizeof(float)));
      b[t] = (float*)aligned_alloc(pg, round(b_elems * sizeof(float)));
      c[t] = (float*)aligned_alloc(pg, round(c_elems * sizeof(float)));
    }
  }
  ~ThreadCaches() {
    for (int t = 0; t < n; ++t) {
      free(a[t]);
      free(b[t]);
      free(c[t]);
    }
    delete[] a;
    delete[] b;
    delete[] c;
  }
};

}  // namespace refwrap
