// cublas_bench -- the reference's cuBLAS GEMM benchmark over the C ABI.
//
// Mirrors 6.cuBLAS/cublas_gemm_bench.cu (flags :68-128, modes :145-166,
// output :283-298): --device --m --n --k --repeat --warmup
// --mode fp16|bf16|tf32|fp32, inputs ((i % 251) - 125) * 1e-3 in the mode's
// type, event- and wall-timed mean over `repeat` back-to-back calls, and the
// same key=value and csv lines.  Exit codes: 0 ok, 1 failure, 2 bad arguments.
#include <cuda_runtime.h>

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

#include "b200attn.h"

namespace {

struct Options {
  int device = 0, m = 16384, n = 16384, k = 16384, repeat = 20, warmup = 5;
  std::string mode = "bf16";
};

int mode_id(const std::string& m) {
  if (m == "fp16") return B200_CUBLAS_FP16;
  if (m == "bf16") return B200_CUBLAS_BF16;
  if (m == "tf32") return B200_CUBLAS_TF32;
  if (m == "fp32") return B200_CUBLAS_FP32;
  return -1;
}

const char* mode_label(int id) {
  switch (id) {
    case B200_CUBLAS_FP16: return "FP16 input/output, FP32 accumulate";
    case B200_CUBLAS_BF16: return "BF16 input/output, FP32 accumulate";
    case B200_CUBLAS_TF32: return "TF32 tensor cores, FP32 input/output";
    default: return "FP32 CUDA cores, FP32 input/output";
  }
}

bool parse(int argc, char** argv, Options* o) {
  for (int i = 1; i < argc; ++i) {
    const std::string f = argv[i];
    auto next = [&]() -> const char* {
      if (i + 1 >= argc) {
        std::fprintf(stderr, "%s needs a value\n", f.c_str());
        std::exit(2);
      }
      return argv[++i];
    };
    if (f == "--help") {
      std::printf("Usage: %s [--device N] [--m M] [--n N] [--k K] [--repeat R] [--warmup W] "
                  "[--mode fp16|bf16|tf32|fp32]\n", argv[0]);
      std::exit(0);
    } else if (f == "--device") o->device = std::atoi(next());
    else if (f == "--m") o->m = std::atoi(next());
    else if (f == "--n") o->n = std::atoi(next());
    else if (f == "--k") o->k = std::atoi(next());
    else if (f == "--repeat") o->repeat = std::atoi(next());
    else if (f == "--warmup") o->warmup = std::atoi(next());
    else if (f == "--mode") o->mode = next();
    else {
      std::fprintf(stderr, "unknown argument %s\n", f.c_str());
      return false;
    }
  }
  return o->m > 0 && o->n > 0 && o->k > 0 && o->repeat > 0 && o->warmup >= 0 &&
         mode_id(o->mode) >= 0;
}

}  // namespace

int main(int argc, char** argv) {
  Options o;
  if (!parse(argc, argv, &o)) {
    std::fprintf(stderr, "invalid arguments (see --help)\n");
    return 2;
  }
  cudaDeviceProp prop{};
  if (cudaSetDevice(o.device) != cudaSuccess ||
      cudaGetDeviceProperties(&prop, o.device) != cudaSuccess) {
    std::fprintf(stderr, "no CUDA device %d\n", o.device);
    return 77;
  }
  const int mode = mode_id(o.mode);
  const size_t es = (mode == B200_CUBLAS_FP16 || mode == B200_CUBLAS_BF16) ? 2 : 4;
  const size_t a = static_cast<size_t>(o.m) * o.k, b = static_cast<size_t>(o.k) * o.n,
               c = static_cast<size_t>(o.m) * o.n;
  void *dA = nullptr, *dB = nullptr, *dC = nullptr;
  if (cudaMalloc(&dA, a * es) != cudaSuccess || cudaMalloc(&dB, b * es) != cudaSuccess ||
      cudaMalloc(&dC, c * es) != cudaSuccess) {
    std::fprintf(stderr, "allocation failed\n");
    return 1;
  }
  if (b200_fill_cublas_pattern(dA, a, mode, 1.0e-3f, nullptr) != B200_OK ||
      b200_fill_cublas_pattern(dB, b, mode, 1.0e-3f, nullptr) != B200_OK ||
      b200_fill_cublas_pattern(dC, c, mode, 0.0f, nullptr) != B200_OK) {
    std::fprintf(stderr, "%s\n", b200_last_error());
    return 1;
  }
  auto run = [&]() { return gemm_cublas_mode(dA, dB, dC, o.m, o.n, o.k, mode, nullptr); };
  for (int i = 0; i < o.warmup; ++i)
    if (run() != B200_OK) {
      std::fprintf(stderr, "%s\n", b200_last_error());
      return 1;
    }
  cudaDeviceSynchronize();
  cudaEvent_t start, stop;
  cudaEventCreate(&start);
  cudaEventCreate(&stop);
  const auto w0 = std::chrono::steady_clock::now();
  cudaEventRecord(start);
  for (int i = 0; i < o.repeat; ++i)
    if (run() != B200_OK) {
      std::fprintf(stderr, "%s\n", b200_last_error());
      return 1;
    }
  cudaEventRecord(stop);
  cudaEventSynchronize(stop);
  const auto w1 = std::chrono::steady_clock::now();
  float ev_ms = 0.0f;
  cudaEventElapsedTime(&ev_ms, start, stop);
  if (b200_check(nullptr) != B200_OK) return 1;
  const double wall_ms = std::chrono::duration<double, std::milli>(w1 - w0).count();
  const double flops = 2.0 * o.m * static_cast<double>(o.n) * o.k;
  const double ev_avg = ev_ms / o.repeat, wall_avg = wall_ms / o.repeat;
  const double ev_tf = flops / (ev_avg * 1e-3) / 1e12, wall_tf = flops / (wall_avg * 1e-3) / 1e12;
  std::printf("device=%d name=\"%s\" cc=%d.%d\n", o.device, prop.name, prop.major, prop.minor);
  std::printf("mode=%s (%s)\n", o.mode.c_str(), mode_label(mode));
  std::printf("m=%d n=%d k=%d repeat=%d warmup=%d\n", o.m, o.n, o.k, o.repeat, o.warmup);
  std::printf("memory=%.2f GiB\n", static_cast<double>((a + b + c) * es) / (1024.0 * 1024 * 1024));
  std::printf("event_total_ms=%.3f event_avg_ms=%.6f event_TFLOPS=%.3f\n", ev_ms, ev_avg, ev_tf);
  std::printf("wall_total_ms=%.3f wall_avg_ms=%.6f wall_TFLOPS=%.3f\n", wall_ms, wall_avg, wall_tf);
  std::printf("csv,%s,%d,%d,%d,%d,%d,%.6f,%.3f,%.6f,%.3f,%s\n", o.mode.c_str(), o.m, o.n, o.k,
              o.repeat, o.warmup, ev_avg, ev_tf, wall_avg, wall_tf, prop.name);
  cudaFree(dA);
  cudaFree(dB);
  cudaFree(dC);
  return 0;
}
