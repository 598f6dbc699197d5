// Validation-only GPU kernels and seeded input generators.
//
// attention_scalar_kernel: plain CUDA-core attention used to check the fused
// kernel on full-size tensors (where the CPU oracle is too slow).  Same
// semantics and arithmetic shape as the harness's CPU reference
// (0.attention/main.cu:1333-1388) and its scalar GPU kernel
// (0.attention/attention.cu:210-274): fp32 dot product, score = dot * scale,
// exact two-pass softmax with expf, fully masked rows -> 0, bf16 RNE output.
// Unlike the reference kernel it handles head_dim 64 as well as 128 and uses
// one warp per query row instead of a block-wide tree reduction per key.
//
// gemm_f32_reference_kernel: fp32 CUDA-core GEMM for full-size GEMM checks.
//
// fill_*: counter-based generators keyed on (seed, tensor id, element index):
// splitmix64 -> uniforms -> (Box-Muller for normals) -> bf16 RNE.  A value
// depends only on its global index, never on the launch shape or on how a
// tensor is sharded across GPUs.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>

namespace b200 {
namespace ref {

__host__ __device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
  x += 0x9e3779b97f4a7c15ull;
  uint64_t z = x;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

__host__ __device__ __forceinline__ uint64_t stream_key(uint64_t seed, uint32_t tensor_id) {
  return splitmix64(seed ^ (0xd1b54a32d192ed03ull * (static_cast<uint64_t>(tensor_id) + 1)));
}

__device__ __forceinline__ uint16_t f32_to_bf16_rne(float v) {
  uint32_t bits = __float_as_uint(v);
  if ((bits & 0x7fffffffu) > 0x7f800000u) return 0x7fc0;  // NaN stays NaN
  bits += 0x7fffu + ((bits >> 16) & 1u);
  return static_cast<uint16_t>(bits >> 16);
}

__device__ __forceinline__ float bf16_to_f32(uint16_t h) {
  return __uint_as_float(static_cast<uint32_t>(h) << 16);
}

// Normal(mean, sigma): element 2p uses the cosine branch and 2p+1 the sine
// branch of one Box-Muller pair drawn from splitmix64(key + p).
__global__ void fill_normal_bf16_kernel(uint16_t* __restrict__ dst, uint64_t n, uint64_t key,
                                        uint64_t index_base, float mean, float sigma) {
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
  for (uint64_t t = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < n;
       t += stride) {
    const uint64_t g = index_base + t;
    const uint64_t r = splitmix64(key + (g >> 1));
    const float u1 = (static_cast<float>(r >> 40) + 1.0f) * (1.0f / 16777216.0f);  // (0, 1]
    const float u2 = static_cast<float>((r >> 16) & 0xffffffull) * (1.0f / 16777216.0f);
    const float rad = sqrtf(-2.0f * logf(u1));
    float sn, cs;
    sincospif(2.0f * u2, &sn, &cs);
    const float z = (g & 1ull) ? rad * sn : rad * cs;
    dst[t] = f32_to_bf16_rne(mean + sigma * z);
  }
}

// Uniform[lo, hi): 24-bit uniform from the top bits of splitmix64(key + g).
__global__ void fill_uniform_bf16_kernel(uint16_t* __restrict__ dst, uint64_t n, uint64_t key,
                                         uint64_t index_base, float lo, float hi) {
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
  for (uint64_t t = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < n;
       t += stride) {
    const uint64_t g = index_base + t;
    const uint64_t r = splitmix64(key + g);
    const float u = static_cast<float>(r >> 40) * (1.0f / 16777216.0f);
    dst[t] = f32_to_bf16_rne(lo + (hi - lo) * u);
  }
}

struct ScalarParams {
  const uint16_t* q;
  const uint16_t* k;
  const uint16_t* v;
  uint16_t* o;
  int B, Hq, Hkv, Sq, Skv, group, causal;
  float scale;
};

// grid (ceil(Sq / 4), B * Hq), 128 threads: warp w handles query row
// blockIdx.x * 4 + w; lane l holds head dims [l * D/32, (l + 1) * D/32).
template <int D>
__global__ void __launch_bounds__(128) attention_scalar_kernel(const ScalarParams p) {
  constexpr int kPer = D / 32;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int qi = blockIdx.x * 4 + warp;
  const int bh = blockIdx.y;
  if (qi >= p.Sq) return;
  const int b = bh / p.Hq;
  const int hq = bh - b * p.Hq;
  const int hkv = hq / p.group;
  const size_t q_off = (static_cast<size_t>(bh) * p.Sq + qi) * D;
  const size_t kv_off = (static_cast<size_t>(b) * p.Hkv + hkv) * static_cast<size_t>(p.Skv) * D;
  float qv[kPer];
#pragma unroll
  for (int e = 0; e < kPer; ++e) qv[e] = bf16_to_f32(p.q[q_off + lane * kPer + e]);
  const int limit = p.causal ? min(p.Skv, qi + (p.Skv - p.Sq) + 1) : p.Skv;

  auto score = [&](int key) {
    const uint16_t* kr = p.k + kv_off + static_cast<size_t>(key) * D + lane * kPer;
    float dot = 0.0f;
#pragma unroll
    for (int e = 0; e < kPer; ++e) dot += qv[e] * bf16_to_f32(kr[e]);
#pragma unroll
    for (int sh = 16; sh > 0; sh >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, sh);
    return dot * p.scale;
  };

  float mx = -INFINITY;
  for (int key = 0; key < limit; ++key) mx = fmaxf(mx, score(key));
  float acc[kPer];
#pragma unroll
  for (int e = 0; e < kPer; ++e) acc[e] = 0.0f;
  float denom = 0.0f;
  if (limit > 0 && mx != -INFINITY) {
    for (int key = 0; key < limit; ++key) {
      const float w = expf(score(key) - mx);
      denom += w;
      const uint16_t* vr = p.v + kv_off + static_cast<size_t>(key) * D + lane * kPer;
#pragma unroll
      for (int e = 0; e < kPer; ++e) acc[e] += w * bf16_to_f32(vr[e]);
    }
  }
#pragma unroll
  for (int e = 0; e < kPer; ++e)
    p.o[q_off + lane * kPer + e] = f32_to_bf16_rne(denom > 0.0f ? acc[e] / denom : 0.0f);
}

// C[M,N] (fp32, row-major) = A[M,K] (row-major) * B, with B either [N,K]
// (b_col_major = 1) or [K,N] (b_col_major = 0).  16x16 threads, 64x64 tile.
__global__ void __launch_bounds__(256) gemm_f32_reference_kernel(const uint16_t* __restrict__ A,
                                                                 const uint16_t* __restrict__ Bm,
                                                                 float* __restrict__ C, int M,
                                                                 int N, int K, int b_col_major) {
  __shared__ float as[16][65];
  __shared__ float bs[16][65];
  const int tx = threadIdx.x & 15;
  const int ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * 64;
  const int n0 = blockIdx.x * 64;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += 16) {
    for (int t = threadIdx.x; t < 64 * 16; t += 256) {
      const int r = t >> 4, kk = t & 15;
      const int gm = m0 + r, gk = k0 + kk;
      as[kk][r] = (gm < M && gk < K) ? bf16_to_f32(A[static_cast<size_t>(gm) * K + gk]) : 0.0f;
      const int gn = n0 + r;
      float bv = 0.0f;
      if (gn < N && gk < K)
        bv = bf16_to_f32(b_col_major ? Bm[static_cast<size_t>(gn) * K + gk]
                                     : Bm[static_cast<size_t>(gk) * N + gn]);
      bs[kk][r] = bv;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] += as[kk][ty * 4 + i] * bs[kk][tx * 4 + j];
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gm = m0 + ty * 4 + i, gn = n0 + tx * 4 + j;
      if (gm < M && gn < N) C[static_cast<size_t>(gm) * N + gn] = acc[i][j];
    }
}

}  // namespace ref
}  // namespace b200
