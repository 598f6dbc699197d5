// Same-box timing of the reference's own fused attention kernel
// (qk_tma_mma_ld_kernel, 0.attention/attention.cu:1503-1974) on seeded
// N(0, sigma^2) bf16 inputs, through the reference's own launch and timing
// function run_kernel (0.attention/main.cu:506-598) and TMA encoders
// (0.attention/main.cu:372-460).  The reference's benchmark binary fills its
// inputs with near-constant values (fill_packed_bf16,
// 0.attention/attention.cu:142-147); this driver gives its kernel the data
// distribution of BASELINE config 2 instead.
//
// MEASUREMENT INFRASTRUCTURE ONLY: compiled from the reference's sources into
// oracle/_ref by oracle/Makefile (target `ref`), never part of the product.
//
//   attention_ref_bench_data [--blocks N] [--k-tiles N] [--warmup N] [--iters N] [--sigma S]
#define main reference_main
#include "0.attention/main.cu"
#undef main

#include <cstdlib>
#include <cstring>

namespace shim {

// splitmix64 counter -> two uniforms -> Box-Muller -> bf16 (round to nearest
// even); one value per element.
__global__ void fill_normal_bf16(uint16_t* p, size_t n, uint64_t seed, float sigma) {
  const size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  if (i >= n) return;
  uint64_t z = seed + 0x9E3779B97F4A7C15ull * (i + 1);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  const float u1 = (static_cast<float>(z >> 40) + 1.0f) * (1.0f / 16777217.0f);
  const float u2 = static_cast<float>((z >> 16) & 0xffffff) * (1.0f / 16777216.0f);
  const float v = sigma * sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
  uint32_t b = __float_as_uint(v);
  b += 0x7fffu + ((b >> 16) & 1u);
  p[i] = static_cast<uint16_t>(b >> 16);
}

}  // namespace shim

int main(int argc, char** argv) {
  Args args;
  float sigma = 1.0f;
  for (int i = 1; i + 1 < argc; i += 2) {
    if (!std::strcmp(argv[i], "--blocks")) args.blocks = std::atoi(argv[i + 1]);
    else if (!std::strcmp(argv[i], "--k-tiles")) args.k_tiles = std::atoi(argv[i + 1]);
    else if (!std::strcmp(argv[i], "--warmup")) args.warmup = std::atoi(argv[i + 1]);
    else if (!std::strcmp(argv[i], "--iters")) args.iters = std::atoi(argv[i + 1]);
    else if (!std::strcmp(argv[i], "--sigma")) sigma = static_cast<float>(std::atof(argv[i + 1]));
    else {
      std::fprintf(stderr, "unknown argument %s\n", argv[i]);
      return 2;
    }
  }
  if (args.blocks < 1 || args.k_tiles < 1 || args.iters < 1 || args.warmup < 0) return 2;
  args.repeats = args.k_tiles;
  driver_check(cuInit(0), "cuInit");
  const int kv_tiles = ((args.blocks + args.k_tiles - 1) / args.k_tiles) * args.k_tiles;
  const size_t q_elems = static_cast<size_t>(args.blocks) * kTileWords * 2;
  const size_t kv_elems = static_cast<size_t>(kv_tiles) * kTileWords * 2;
  uint16_t *q = nullptr, *k = nullptr, *v = nullptr, *o = nullptr;
  CUDA_CHECK(cudaMalloc(&q, q_elems * 2));
  CUDA_CHECK(cudaMalloc(&k, kv_elems * 2));
  CUDA_CHECK(cudaMalloc(&v, kv_elems * 2));
  CUDA_CHECK(cudaMalloc(&o, q_elems * 2));
  const int t = 256;
  shim::fill_normal_bf16<<<static_cast<unsigned>((q_elems + t - 1) / t), t>>>(q, q_elems, 101, sigma);
  shim::fill_normal_bf16<<<static_cast<unsigned>((kv_elems + t - 1) / t), t>>>(k, kv_elems, 202, sigma);
  shim::fill_normal_bf16<<<static_cast<unsigned>((kv_elems + t - 1) / t), t>>>(v, kv_elems, 303, sigma);
  CUDA_CHECK(cudaDeviceSynchronize());
  CUtensorMap q_map{}, k_map{}, v_map{}, o_map{};
  encode_qk_contiguous_sw128_tma_map(&q_map, q, static_cast<uint64_t>(args.blocks));
  encode_qk_contiguous_sw128_tma_map(&k_map, k, static_cast<uint64_t>(kv_tiles));
#if ATTENTION_SPLIT_V_TMA
  encode_contiguous_sw128_k16_half_tma_map(&v_map, v, static_cast<uint64_t>(kv_tiles));
#else
  encode_contiguous_sw128_k16_tma_map(&v_map, v, static_cast<uint64_t>(kv_tiles));
#endif
  encode_bf16_output_tma_map(&o_map, o, static_cast<uint64_t>(args.blocks));
  int active = 0;
  const RunResult r =
      run_kernel(args, q_map, k_map, v_map, o_map, resolved_score_to_exp2_scale(args), o, &active);
  const double flops = 2.0 * static_cast<double>(args.blocks) * args.repeats * kMmasPerTile *
                       kFlopsPerMma;
  std::printf("blocks=%d k_tiles=%d sigma=%g iters=%d elapsed_ms=%.6f total_TFLOP_per_s=%.3f "
              "status=%s cuda_error=%s\n",
              args.blocks, args.k_tiles, sigma, args.iters, r.ms,
              r.ms > 0 ? flops / (r.ms * 1e-3) / 1e12 : 0.0, r.status, cudaGetErrorString(r.error));
  cudaFree(q);
  cudaFree(k);
  cudaFree(v);
  cudaFree(o);
  return r.error == cudaSuccess ? 0 : 1;
}
