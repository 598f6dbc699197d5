// gemm_bench -- C++ host harness for the bf16 GEMM over the C ABI.
//
// Mirrors 5.GEMM/gemm256_tma_tcgen05_bench.cu's CLI (main :1276-1348):
//   --sizes 4096,8192,... --warmup N --iters N --csv PATH --device N
//   --validate --validate-size N --validate-pattern pattern|ones
// plus --impl tcgen05|cublas (the 6.cuBLAS comparator, cublas_gemm_bench.cu
// :226-231) and --b-layout col|row (B stored [N,K] or [K,N]).  Benchmark
// inputs are seeded U(-1,1) (BASELINE's GEMM data); validation uses the
// reference's fills (:1013-1023) and compares against the library's fp32
// reference GEMM with the reference tolerance (abs 2e-2 AND rel 2e-2,
// :1113-1127) and BASELINE's relative Frobenius error <= 1e-2.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <sstream>
#include <string>
#include <vector>

#include "b200attn.h"

namespace {

struct Args {
  std::vector<int> sizes{4096, 8192, 16384};
  int warmup = 2, iters = 5, device = 0, validate_size = 256;
  bool validate = false, b_col = true, cublas = false;
  std::string validate_pattern = "pattern", csv;
};

bool parse(int argc, char** argv, Args* a) {
  for (int i = 1; i < argc; ++i) {
    const std::string f = argv[i];
    auto next = [&]() -> std::string {
      if (i + 1 >= argc) {
        std::fprintf(stderr, "%s needs a value\n", f.c_str());
        std::exit(2);
      }
      return argv[++i];
    };
    if (f == "--help") {
      std::printf("gemm_bench [--sizes a,b] [--warmup N] [--iters N] [--csv PATH] [--device N]\n"
                  "           [--validate --validate-size N --validate-pattern pattern|ones]\n"
                  "           [--impl tcgen05|cublas] [--b-layout col|row]\n");
      std::exit(0);
    } else if (f == "--sizes") {
      a->sizes.clear();
      std::stringstream ss(next());
      std::string tok;
      while (std::getline(ss, tok, ',')) a->sizes.push_back(std::atoi(tok.c_str()));
    } else if (f == "--warmup") a->warmup = std::atoi(next().c_str());
    else if (f == "--iters") a->iters = std::atoi(next().c_str());
    else if (f == "--device") a->device = std::atoi(next().c_str());
    else if (f == "--csv") a->csv = next();
    else if (f == "--validate") a->validate = true;
    else if (f == "--validate-size") a->validate_size = std::atoi(next().c_str());
    else if (f == "--validate-pattern") a->validate_pattern = next();
    else if (f == "--impl") {
      const std::string v = next();
      if (v != "tcgen05" && v != "cublas") return false;
      a->cublas = v == "cublas";
    } else if (f == "--b-layout") {
      const std::string v = next();
      if (v != "col" && v != "row") return false;
      a->b_col = v == "col";
    } else {
      std::fprintf(stderr, "unknown argument %s\n", f.c_str());
      return false;
    }
  }
  for (int s : a->sizes)
    if (s < 8 || s % 8) return false;
  return a->iters >= 1 && a->warmup >= 0 && a->validate_size >= 8 && a->validate_size % 8 == 0 &&
         (a->validate_pattern == "pattern" || a->validate_pattern == "ones");
}

uint16_t to_bf16(float v) {
  uint32_t b;
  std::memcpy(&b, &v, 4);
  b += 0x7fffu + ((b >> 16) & 1u);
  return static_cast<uint16_t>(b >> 16);
}

float bf16_to_f32(uint16_t h) {
  const uint32_t w = static_cast<uint32_t>(h) << 16;
  float f;
  std::memcpy(&f, &w, 4);
  return f;
}

b200_status gemm(const Args& a, const void* A, const void* B, void* C, int M, int N, int K) {
  return a.cublas ? gemm_bf16_cublas(A, B, C, M, N, K, a.b_col ? 1 : 0, nullptr)
                  : gemm_bf16(A, B, C, M, N, K, a.b_col ? 1 : 0, nullptr);
}

int run_validation(const Args& a) {
  const int n = a.validate_size;
  const bool ones = a.validate_pattern == "ones";
  std::vector<uint16_t> ha(static_cast<size_t>(n) * n), hb(static_cast<size_t>(n) * n);
  for (int r = 0; r < n; ++r)
    for (int c = 0; c < n; ++c) {
      // A[r][c] and B[k=r][n=c] as the reference's validation_a/b_value.
      const float av = ones ? 1.0f : static_cast<float>((r % 17) - 8) * 0.015625f +
                                         static_cast<float>((c % 11) - 5) * 0.0078125f;
      const float bv = ones ? 1.0f : static_cast<float>((r % 13) - 6) * 0.01171875f -
                                         static_cast<float>((c % 19) - 9) * 0.005859375f;
      ha[static_cast<size_t>(r) * n + c] = to_bf16(av);
      if (a.b_col)
        hb[static_cast<size_t>(c) * n + r] = to_bf16(bv);  // stored [N,K]
      else
        hb[static_cast<size_t>(r) * n + c] = to_bf16(bv);  // stored [K,N]
    }
  const size_t bytes = static_cast<size_t>(n) * n * 2;
  void *dA, *dB, *dC, *dR;
  cudaMalloc(&dA, bytes);
  cudaMalloc(&dB, bytes);
  cudaMalloc(&dC, bytes);
  cudaMalloc(&dR, bytes * 2);
  cudaMemcpy(dA, ha.data(), bytes, cudaMemcpyHostToDevice);
  cudaMemcpy(dB, hb.data(), bytes, cudaMemcpyHostToDevice);
  b200_status st = gemm(a, dA, dB, dC, n, n, n);
  if (st == B200_OK) st = gemm_f32_reference(dA, dB, dR, n, n, n, a.b_col ? 1 : 0, nullptr);
  if (st == B200_OK) st = b200_check(nullptr);
  if (st != B200_OK) {
    std::fprintf(stderr, "validation failed to run: %s\n", b200_last_error());
    return 1;
  }
  std::vector<uint16_t> hc(static_cast<size_t>(n) * n);
  std::vector<float> hr(static_cast<size_t>(n) * n);
  cudaMemcpy(hc.data(), dC, bytes, cudaMemcpyDeviceToHost);
  cudaMemcpy(hr.data(), dR, bytes * 2, cudaMemcpyDeviceToHost);
  double max_abs = 0, max_rel = 0, num = 0, den = 0;
  size_t bad = 0;
  for (size_t i = 0; i < hc.size(); ++i) {
    const double got = bf16_to_f32(hc[i]), ref = hr[i];
    const double d = std::fabs(got - ref), rel = d / std::max(1.0e-12, std::fabs(ref));
    max_abs = std::max(max_abs, d);
    max_rel = std::max(max_rel, rel);
    num += d * d;
    den += ref * ref;
    if (!std::isfinite(got) || (d > 2.0e-2 && rel > 2.0e-2)) ++bad;
  }
  const double frob = std::sqrt(num / std::max(den, 1e-300));
  const bool ok = bad == 0 && frob <= 1e-2;
  std::printf("validation size=%d pattern=%s impl=%s b_layout=%s status=%s max_abs=%g max_rel=%g "
              "bad=%zu rel_frob=%g\n",
              n, a.validate_pattern.c_str(), a.cublas ? "cublas" : "tcgen05",
              a.b_col ? "col" : "row", ok ? "ok" : "fail", max_abs, max_rel, bad, frob);
  cudaFree(dA);
  cudaFree(dB);
  cudaFree(dC);
  cudaFree(dR);
  return ok ? 0 : 1;
}

int run_bench(const Args& a) {
  FILE* csv = a.csv.empty() ? nullptr : std::fopen(a.csv.c_str(), "w");
  if (csv)
    std::fprintf(csv, "size,m,n,k,impl,b_layout,warmup,iters,event_ms,min_ms,event_TFLOPS,"
                      "status,device\n");
  int rc = 0;
  for (int s : a.sizes) {
    const size_t bytes = static_cast<size_t>(s) * s * 2;
    void *dA = nullptr, *dB = nullptr, *dC = nullptr;
    const char* status = "ok";
    if (cudaMalloc(&dA, bytes) != cudaSuccess || cudaMalloc(&dB, bytes) != cudaSuccess ||
        cudaMalloc(&dC, bytes) != cudaSuccess) {
      status = "alloc_failed";
    } else {
      b200_fill_uniform_bf16(dA, static_cast<uint64_t>(s) * s, 5, 10, 0, -1.0f, 1.0f, nullptr);
      b200_fill_uniform_bf16(dB, static_cast<uint64_t>(s) * s, 5, 11, 0, -1.0f, 1.0f, nullptr);
    }
    float ms = 0, mn = 1e30f;
    if (std::strcmp(status, "ok") == 0) {
      for (int i = 0; i < a.warmup; ++i)
        if (gemm(a, dA, dB, dC, s, s, s) != B200_OK) status = "warmup_failed";
      cudaEvent_t t0, t1;
      cudaEventCreate(&t0);
      cudaEventCreate(&t1);
      cudaDeviceSynchronize();
      // event_ms: mean of per-launch event times; min_ms: fastest launch
      for (int i = 0; i < a.iters; ++i) {
        cudaEventRecord(t0);
        if (gemm(a, dA, dB, dC, s, s, s) != B200_OK) status = "timed_failed";
        cudaEventRecord(t1);
        cudaEventSynchronize(t1);
        float one = 0;
        cudaEventElapsedTime(&one, t0, t1);
        mn = std::min(mn, one);
        ms += one;
      }
      ms /= static_cast<float>(a.iters);
      if (b200_check(nullptr) != B200_OK) status = "runtime_failed";
      cudaEventDestroy(t0);
      cudaEventDestroy(t1);
    }
    const double tflops = ms > 0 ? 2.0 * s * static_cast<double>(s) * s / (ms * 1e-3) / 1e12 : 0;
    std::printf("size=%d impl=%s b_layout=%s event_ms=%.6f min_ms=%.6f event_TFLOPS=%.3f "
                "status=%s\n",
                s, a.cublas ? "cublas" : "tcgen05", a.b_col ? "col" : "row", ms, mn, tflops,
                status);
    if (csv)
      std::fprintf(csv, "%d,%d,%d,%d,%s,%s,%d,%d,%.6f,%.6f,%.3f,%s,%d\n", s, s, s, s,
                   a.cublas ? "cublas" : "tcgen05", a.b_col ? "col" : "row", a.warmup, a.iters,
                   ms, mn, tflops, status, a.device);
    if (std::strcmp(status, "ok") != 0) rc = 1;
    if (dA) cudaFree(dA);
    if (dB) cudaFree(dB);
    if (dC) cudaFree(dC);
  }
  if (csv) std::fclose(csv);
  return rc;
}

}  // namespace

int main(int argc, char** argv) {
  Args a;
  if (!parse(argc, argv, &a)) {
    std::fprintf(stderr, "invalid arguments (see --help)\n");
    return 2;
  }
  cudaDeviceProp prop{};
  if (cudaSetDevice(a.device) != cudaSuccess ||
      cudaGetDeviceProperties(&prop, a.device) != cudaSuccess) {
    std::fprintf(stderr, "no CUDA device %d\n", a.device);
    return 77;
  }
  if (prop.major < 10) {
    std::fprintf(stderr, "this build requires sm_100a; got sm_%d%d\n", prop.major, prop.minor);
    return 77;
  }
  return a.validate ? run_validation(a) : run_bench(a);
}
