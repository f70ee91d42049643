// CPU oracle for strict-FP32 SGEMM -- TEST INFRASTRUCTURE ONLY (see oracle.h).
//
// Restates the FP64 oracle of the reference's device correctness test,
// tests/cuda/correctness.cu:373-392 (AG0708/sgBLAS), and its input generator,
// tests/cuda/correctness.cu:170-174. Built with -ffp-contract=off so that the
// compiler cannot fuse the double multiply-add into an FMA: the reference loop
// rounds the product and the sum separately.
#include "oracle.h"

#include <algorithm>
#include <cmath>
#include <random>
#include <thread>
#include <vector>

namespace {

inline double loadA(const float *a, int lda, bool t, int row, int r) {
  // op(A)(row, r): A(row, r) when not transposed, A(r, row) when transposed.
  return t ? static_cast<double>(a[static_cast<size_t>(r) + static_cast<size_t>(row) * lda])
           : static_cast<double>(a[static_cast<size_t>(row) + static_cast<size_t>(r) * lda]);
}

inline double loadB(const float *b, int ldb, bool t, int r, int col) {
  return t ? static_cast<double>(b[static_cast<size_t>(col) + static_cast<size_t>(r) * ldb])
           : static_cast<double>(b[static_cast<size_t>(r) + static_cast<size_t>(col) * ldb]);
}

// One output entry: correctness.cu:373-392, in the same order.
inline void entry(bool ta, bool tb, int k, float alpha, const float *a, int lda,
                  const float *b, int ldb, float beta, const float *c0, int ldc,
                  int row, int col, double *ref, double *mag) {
  double dot = 0.0, abs_sum = 0.0;
  for (int r = 0; r < k; ++r) {
    const double p = loadA(a, lda, ta, row, r) * loadB(b, ldb, tb, r, col);
    dot += p;
    abs_sum += std::abs(p);
  }
  const double product = static_cast<double>(alpha) * dot;
  double reference = product;
  double magnitude = std::abs(static_cast<double>(alpha)) * abs_sum;
  if (beta != 0.0F) {
    const double cv = c0[static_cast<size_t>(row) + static_cast<size_t>(col) * ldc];
    reference = product + static_cast<double>(beta) * cv;
    magnitude += std::abs(static_cast<double>(beta) * cv);
  }
  *ref = reference;
  *mag = magnitude;
}

int resolveThreads(int threads) {
  if (threads > 0) return threads;
  const unsigned hc = std::thread::hardware_concurrency();
  return hc == 0 ? 1 : static_cast<int>(hc);
}

template <typename F>
void parallelFor(int begin, int end, int threads, F body) {
  const int count = end - begin;
  if (count <= 0) return;
  threads = std::min(resolveThreads(threads), count);
  if (threads <= 1) {
    for (int i = begin; i < end; ++i) body(i);
    return;
  }
  std::vector<std::thread> pool;
  pool.reserve(threads);
  for (int t = 0; t < threads; ++t) {
    pool.emplace_back([=] {
      // Round-robin columns so that threads finish together.
      for (int i = begin + t; i < end; i += threads) body(i);
    });
  }
  for (auto &th : pool) th.join();
}

}  // namespace

extern "C" {

void *oracle_rng_new(uint32_t seed) { return new std::mt19937(seed); }

void oracle_rng_free(void *rng) { delete static_cast<std::mt19937 *>(rng); }

void oracle_rng_uniform(void *rng, float *out, size_t count) {
  auto &g = *static_cast<std::mt19937 *>(rng);
  std::uniform_real_distribution<float> dist(-1.0F, 1.0F);
  for (size_t i = 0; i < count; ++i) out[i] = dist(g);
}

void oracle_rng_normal(void *rng, float *out, size_t count) {
  auto &g = *static_cast<std::mt19937 *>(rng);
  std::normal_distribution<float> dist(0.0F, 1.0F);
  for (size_t i = 0; i < count; ++i) out[i] = dist(g);
}

void oracle_sgemm_f64(int transa, int transb, int m, int /*n*/, int k, float alpha,
                      const float *a, int lda, const float *b, int ldb,
                      float beta, const float *c0, int ldc, int j0, int j1,
                      double *ref, double *mag, int threads) {
  parallelFor(j0, j1, threads, [&](int col) {
    const size_t base = static_cast<size_t>(col - j0) * m;
    for (int row = 0; row < m; ++row)
      entry(transa != 0, transb != 0, k, alpha, a, lda, b, ldb, beta, c0, ldc,
            row, col, ref + base + row, mag + base + row);
  });
}

void oracle_sgemm_f64_points(int transa, int transb, int k, float alpha,
                             const float *a, int lda, const float *b, int ldb,
                             float beta, const float *c0, int ldc,
                             const int *rows, const int *cols, int count,
                             double *ref, double *mag, int threads) {
  parallelFor(0, count, threads, [&](int i) {
    entry(transa != 0, transb != 0, k, alpha, a, lda, b, ldb, beta, c0, ldc,
          rows[i], cols[i], ref + i, mag + i);
  });
}

void oracle_sgemm_cpu(int transa, int transb, int m, int k, float alpha,
                      const float *a, int lda, const float *b, int ldb,
                      float beta, float *c, int ldc, int j0, int j1,
                      int threads) {
  parallelFor(j0, j1, threads, [&](int col) {
    for (int row = 0; row < m; ++row) {
      double ref, mag;
      entry(transa != 0, transb != 0, k, alpha, a, lda, b, ldb, beta, c, ldc,
            row, col, &ref, &mag);
      c[static_cast<size_t>(row) + static_cast<size_t>(col) * ldc] =
          static_cast<float>(ref);
    }
  });
}

int oracle_hardware_threads(void) { return resolveThreads(0); }

}  // extern "C"
