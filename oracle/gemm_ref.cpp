// CPU GEMM oracle -- TEST INFRASTRUCTURE ONLY (see oracle.h).
//
// Restates the reference's GEMM validation arithmetic
// (5.GEMM/gemm256_tma_tcgen05_bench.cu:1115-1137): C[row, col] is the double
// sum over k of double(A[row, k]) * double(B[k, col]) in ascending k, with A
// and B the bf16 inputs widened exactly.  The reference's fills
// (5.GEMM/gemm256_tma_tcgen05_bench.cu:1013-1023) are restated as well.
#include <algorithm>
#include <atomic>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "oracle.h"

namespace {

double bf16_to_f64(uint16_t bits) {
  const uint32_t w = static_cast<uint32_t>(bits) << 16;
  float f;
  std::memcpy(&f, &w, sizeof(f));
  return static_cast<double>(f);
}

float gemm_a_value(bool ones, int row, int col) {
  if (ones) return 1.0f;
  return (static_cast<float>((row % 17) - 8) * 0.015625f) +
         (static_cast<float>((col % 11) - 5) * 0.0078125f);
}

float gemm_b_value(bool ones, int row, int col) {
  if (ones) return 1.0f;
  return (static_cast<float>((row % 13) - 6) * 0.01171875f) -
         (static_cast<float>((col % 19) - 9) * 0.005859375f);
}

}  // namespace

extern "C" {

void oracle_gemm_f64(const uint16_t* A, const uint16_t* Bm, int M, int N, int K, int b_col_major,
                     int row_begin, int row_end, double* out, int threads) {
  (void)M;
  const int rows = row_end - row_begin;
  if (rows <= 0) return;
  if (threads <= 0) threads = static_cast<int>(std::max(1u, std::thread::hardware_concurrency()));
  threads = std::min(threads, rows);
  // B as doubles in [N][K] order so the inner loop walks both operands contiguously.
  std::vector<double> bt(static_cast<size_t>(N) * K);
  for (int n = 0; n < N; ++n)
    for (int kk = 0; kk < K; ++kk)
      bt[static_cast<size_t>(n) * K + kk] =
          bf16_to_f64(b_col_major ? Bm[static_cast<size_t>(n) * K + kk]
                                  : Bm[static_cast<size_t>(kk) * N + n]);
  std::atomic<int> next{row_begin};
  auto work = [&] {
    std::vector<double> arow(K);
    for (int row = next.fetch_add(1); row < row_end; row = next.fetch_add(1)) {
      for (int kk = 0; kk < K; ++kk) arow[kk] = bf16_to_f64(A[static_cast<size_t>(row) * K + kk]);
      double* orow = out + static_cast<size_t>(row - row_begin) * N;
      for (int col = 0; col < N; ++col) {
        const double* bc = &bt[static_cast<size_t>(col) * K];
        double ref = 0.0;
        for (int kk = 0; kk < K; ++kk) ref += arow[kk] * bc[kk];
        orow[col] = ref;
      }
    }
  };
  std::vector<std::thread> pool;
  for (int t = 1; t < threads; ++t) pool.emplace_back(work);
  work();
  for (auto& th : pool) th.join();
}

void oracle_gemm_fill_bf16(uint16_t* dst, char which, const char* pattern, int rows, int cols) {
  const bool ones = std::string(pattern) == "ones";
  for (int r = 0; r < rows; ++r)
    for (int c = 0; c < cols; ++c)
      dst[static_cast<size_t>(r) * cols + c] =
          oracle_f32_to_bf16(which == 'a' ? gemm_a_value(ones, r, c) : gemm_b_value(ones, r, c));
}

}  // extern "C"
