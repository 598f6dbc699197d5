// peak_probe -- throughput probes behind the rooflines this library reports.
//
// Stands in for the reference's microbenchmarks 1.mma (tcgen05.mma rate),
// 2.TMEM_LDST (TMEM load/store rate) and the exp/MUFU rate its softmax
// design assumes, plus a plain HBM copy:
//
//   peak_probe [--probe mma|issue|tile|tmem|mufu|softmax|hbm|all] [--iters N] [--device N]
//
// One CTA per SM.  Each probe prints one line `probe=... value=... unit=...`
// with the per-SM cycle count behind it.  Operand values do not matter for a
// rate: shared-memory operands are zero, TMEM operands are whatever the
// accumulators hold.  Every wait is bounded (ptx.cuh); exit code 1 if one ran
// out or a CUDA call failed, 2 on bad arguments, 77 without an sm_100 device.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

#include "ptx.cuh"

using namespace b200;

namespace {

constexpr int kSmemProbe = 120 * 1024;  // keeps one CTA (and its 512 TMEM columns) per SM

// tcgen05.mma M=128, N (128 or 256), K=16, bf16 -> fp32, A from shared memory
// (ts = 0), TMEM (ts = 1) or alternating (ts = 2: shared-A MMAs into one
// accumulator, TMEM-A MMAs into another, the attention kernel's S/PV mix),
// issued back to back by one warp.  accs = 2 alternates the accumulator
// between columns [0, N) and [128, 128 + N) (N = 128 only).  fill = 0: zero
// operands; fill = 1: bf16 near 1.0 (the reference probe's fill).
__global__ void __launch_bounds__(128, 1)
    mma_probe(int n, int ts, int accs, int fill, int iters, unsigned long long* cycles) {
  extern __shared__ uint8_t raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* a = smem;                         // 128 x 64 bf16, K-major SW128 (16 KiB)
  uint8_t* b = smem + 16384;                 // 256 x 64 bf16, K-major SW128 (32 KiB)
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + 16384 + 32768);
  uint32_t* slot = reinterpret_cast<uint32_t*>(smem + 16384 + 32768 + 16);
  for (int i = threadIdx.x; i < (16384 + 32768) / 4; i += blockDim.x)
    reinterpret_cast<uint32_t*>(smem)[i] =
        fill ? 0x3f803f80u ^ (static_cast<uint32_t>(i) & 0x000f000fu) : 0u;
  fence_proxy_async_smem();
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  if (warp_id() == 0) {
    tmem_alloc(slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *slot;
  if (warp_id() == 0) {
    // The whole warp runs the loop and one elected lane issues, as the
    // kernels issue their MMAs.
    const uint32_t idesc = idesc_bf16_f32(128, n, false, false);
    const uint64_t da = sdesc_sw128(smem_u32(a), 16, 1024);
    const uint64_t db = sdesc_sw128(smem_u32(b), 16, 1024);
    const unsigned long long t0 = clock64();
    for (int it = 0; it < iters; ++it) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t d = tmem + ((accs == 2 && (k & 1)) ? 128u : 0u);
        if (ts == 1 || (ts == 2 && (k & 1)))
          mma_ts_warp(d, tmem + 256 + k * 8, db + k * 2, idesc, 1u);
        else
          mma_ss_warp(d, da + k * 2, db + k * 2, idesc, 1u);
      }
    }
    mma_commit_warp(bar);
    const bool ok = __all_sync(0xffffffffu, mbar_wait(bar, 0, 0x51));
    const unsigned long long t1 = clock64();
    if (lane_id() == 0) cycles[blockIdx.x] = ok ? t1 - t0 : 0ull;
  }
  tc_fence_before();
  __syncthreads();
  if (warp_id() == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// tcgen05.mma.cta_group::2 M=256 (128 rows per CTA), N (128 or 256), K=16,
// both operands from shared memory, issued by the even CTA of each pair.
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(128, 1)
    mma_pair_probe(int n, int iters, unsigned long long* cycles) {
  extern __shared__ uint8_t raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* a = smem;           // this CTA's 128 x 64 A rows (16 KiB)
  uint8_t* b = smem + 16384;   // this CTA's N/2 x 64 B rows (up to 16 KiB)
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + 32768);
  uint32_t* slot = reinterpret_cast<uint32_t*>(smem + 32768 + 16);
  const bool leader = cluster_ctarank() == 0;
  for (int i = threadIdx.x; i < 32768 / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
  fence_proxy_async_smem();
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  if (warp_id() == 0) {
    tmem_alloc_pair(slot, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = *slot;
  if (warp_id() == 0 && leader) {
    const uint32_t idesc = idesc_bf16_f32(256, n, false, false);
    const uint64_t da = sdesc_sw128(smem_u32(a), 16, 1024);
    const uint64_t db = sdesc_sw128(smem_u32(b), 16, 1024);
    const unsigned long long t0 = clock64();
    for (int it = 0; it < iters; ++it) {
#pragma unroll
      for (int k = 0; k < 4; ++k) mma_ss_pair_warp(tmem, da + k * 2, db + k * 2, idesc, 1u);
    }
    if (lane_id() == 0) mma_commit_pair_local(bar);
    __syncwarp();
    const bool ok = __all_sync(0xffffffffu, mbar_wait(bar, 0, 0x52));
    const unsigned long long t1 = clock64();
    if (lane_id() == 0) cycles[blockIdx.x >> 1] = ok ? t1 - t0 : 0ull;
  }
  tc_fence_before();
  cluster_sync_all();
  if (warp_id() == 0) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

// tcgen05.mma M=128 N=128 K=16, both operands in shared memory, issued by
// `issuers` warps of each CTA (several CTAs per SM when the grid asks for
// them), each warp into its own 128-column accumulator.  reuse = 1 repeats
// the same A and B descriptors for every MMA, the pattern of the reference's
// issue-rate probe (1.mma/mma_throughput_bench.cu:404-460); reuse = 0 walks
// four K slices of distinct operands, as a kernel's K loop does.  Operands
// are bf16 near 1.0 (fill = 1, the reference probe's fill) or zero (fill = 0).
__global__ void __launch_bounds__(128) mma_issue_probe(int issuers, int reuse, int fill,
                                                       int iters, unsigned long long* cycles) {
  __shared__ __align__(1024) uint8_t smem[32768];  // A 128x64 | B 128x64 (K-major SW128)
  __shared__ uint64_t bar;
  __shared__ uint32_t slot;
  for (int i = threadIdx.x; i < 32768 / 4; i += blockDim.x)
    reinterpret_cast<uint32_t*>(smem)[i] =
        fill ? 0x3f803f80u ^ (static_cast<uint32_t>(i) & 0x000f000fu) : 0u;
  fence_proxy_async_smem();
  if (threadIdx.x == 0) {
    mbar_init(&bar, static_cast<uint32_t>(issuers));
    fence_mbar_init();
  }
  const uint32_t cols = issuers == 1 ? 128u : (issuers == 2 ? 256u : 512u);
  if (warp_id() == 0) {
    tmem_alloc(&slot, cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = slot;
  unsigned long long t0 = clock64();
  if (static_cast<int>(warp_id()) < issuers) {
    const uint32_t idesc = idesc_bf16_f32(128, 128, false, false);
    const uint64_t da = sdesc_sw128(smem_u32(smem), 16, 1024);
    const uint64_t db = sdesc_sw128(smem_u32(smem + 16384), 16, 1024);
    const uint32_t d = tmem + warp_id() * 128u;
    const uint32_t step = reuse ? 0u : 2u;
    for (int it = 0; it < iters; ++it) {
#pragma unroll
      for (int k = 0; k < 4; ++k) mma_ss_warp(d, da + k * step, db + k * step, idesc, 1u);
    }
    mma_commit_warp(&bar);
  }
  const bool ok = mbar_wait(&bar, 0, 0x53);
  const unsigned long long t1 = clock64();
  if (threadIdx.x == 0) cycles[blockIdx.x] = ok ? t1 - t0 : 0ull;
  tc_fence_before();
  __syncthreads();
  if (warp_id() == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, cols);
  }
}

// The attention kernel's per-tile MMA stream for d=128: S = Q K^T as eight
// M128 N128 K16 SS MMAs into one of three 128-column S buffers (Q and K
// 128 x 128 bf16, K-major SW128 in two 64-column boxes), then O += P V as
// eight M128 N128 K16 TS MMAs with P read from that S buffer and V (keys x D,
// MN-major SW128) from shared memory, O in columns 384-511.  mode:
//   0  one issuing warp, MMAs only
//   1  one issuing warp, plus the kernel's four commits per tile
//   2  one issuing warp, commits, and before each group the kernel's grouped
//      barrier test (three try_waits, warp vote, fence) on phases that have
//      already completed
//   3  two issuing warps (S groups / PV groups), each with its commits and
//      grouped test before each of its groups
//   4  two issuing warps, MMAs only
// Values are whatever the operands hold (timing only).
__global__ void __launch_bounds__(128, 1) tile_issue_probe(int mode, int iters,
                                                           unsigned long long* cycles) {
  extern __shared__ uint8_t raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  constexpr uint32_t kBox = 16384, kTile = 32768;
  uint8_t* q = smem;
  uint8_t* k = smem + kTile;
  uint8_t* v = smem + 2 * kTile;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 3 * kTile);  // 0 final, 1-4 commits, 5 idle
  uint32_t* slot = reinterpret_cast<uint32_t*>(smem + 3 * kTile + 64);
  const int issuers = mode >= 3 ? 2 : 1;
  for (int i = threadIdx.x; i < 3 * static_cast<int>(kTile) / 4; i += blockDim.x)
    reinterpret_cast<uint32_t*>(smem)[i] = 0x3f803f80u ^ (static_cast<uint32_t>(i) & 0x000f000fu);
  fence_proxy_async_smem();
  if (threadIdx.x == 0) {
    mbar_init(&bars[0], static_cast<uint32_t>(issuers));
    for (int b = 1; b < 6; ++b) mbar_init(&bars[b], 1);
    fence_mbar_init();
  }
  if (warp_id() == 0) {
    tmem_alloc(slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *slot;
  const unsigned long long t0 = clock64();
  const int w = static_cast<int>(warp_id());
  if (w < issuers) {
    constexpr uint32_t idesc_s = idesc_bf16_f32(128, 128, false, false);
    constexpr uint32_t idesc_o = idesc_bf16_f32(128, 128, false, true);
    const uint64_t dq = sdesc_sw128(smem_u32(q), 16, 1024);
    const uint64_t dk = sdesc_sw128(smem_u32(k), 16, 1024);
    const uint64_t dv = sdesc_sw128(smem_u32(v), kBox, 1024);
    const uint32_t idle = smem_u32(&bars[5]);
    const bool do_s = issuers == 1 || w == 0;
    const bool do_pv = issuers == 1 || w == 1;
    const bool commits = mode == 1 || mode == 2 || mode == 3;
    const bool waits = mode == 2 || mode == 3;
    bool ok = true;
    for (int t = 0; t < iters && ok; ++t) {
      const uint32_t sbuf = tmem + static_cast<uint32_t>((t % 3) * 128);
      if (do_s) {
        if (waits) {
          ok = __all_sync(0xffffffffu, mbar_wait3(idle, 1u, idle, 1u, idle, 1u, 0x54));
          tc_fence_after();
        }
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * (kBox >> 4) + (kk & 3) * 2;
          mma_ss_warp(sbuf, dq + off, dk + off, idesc_s, kk > 0 ? 1u : 0u);
        }
        if (commits) {
          mma_commit_warp(&bars[1]);
          mma_commit_warp(&bars[2]);
        }
      }
      if (do_pv) {
        if (waits) {
          ok = ok && __all_sync(0xffffffffu, mbar_wait3(idle, 1u, idle, 1u, idle, 1u, 0x55));
          tc_fence_after();
        }
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          mma_ts_warp(tmem + 384u, sbuf + kk * 8, dv + kk * (2048 >> 4), idesc_o, 1u);
        if (commits) {
          mma_commit_warp(&bars[3]);
          mma_commit_warp(&bars[4]);
        }
      }
    }
    mma_commit_warp(&bars[0]);
  }
  const bool ok = mbar_wait(&bars[0], 0, 0x56);
  const unsigned long long t1 = clock64();
  if (threadIdx.x == 0) cycles[blockIdx.x] = ok ? t1 - t0 : 0ull;
  tc_fence_before();
  __syncthreads();
  if (warp_id() == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// tcgen05.ld / tcgen05.st 32x32b.x32 by four warps (each its lane quadrant).
__global__ void __launch_bounds__(128, 1) tmem_probe(int store, int iters,
                                                     unsigned long long* cycles,
                                                     uint32_t* sink) {
  extern __shared__ uint8_t raw[];
  uint32_t* slot = reinterpret_cast<uint32_t*>(
      (reinterpret_cast<uintptr_t>(raw) + 15) & ~static_cast<uintptr_t>(15));
  if (warp_id() == 0) {
    tmem_alloc(slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *slot + ((warp_id() * 32u) << 16);
  uint32_t v[32];
#pragma unroll
  for (int e = 0; e < 32; ++e) v[e] = threadIdx.x + e;
  uint32_t acc = 0;
  __syncthreads();
  const unsigned long long t0 = clock64();
  for (int it = 0; it < iters; ++it) {
    const uint32_t col = static_cast<uint32_t>((it & 15) * 32);
    if (store) {
      tmem_st32(tmem + col, v);
    } else {
      tmem_ld32(tmem + col, v);
      tmem_wait_ld(v);
      acc ^= v[it & 31];
    }
  }
  if (store) tmem_wait_st();
  __syncthreads();
  const unsigned long long t1 = clock64();
  if (threadIdx.x == 0) cycles[blockIdx.x] = t1 - t0;
  sink[blockIdx.x * blockDim.x + threadIdx.x] = acc;
  tc_fence_before();
  __syncthreads();
  if (warp_id() == 0) {
    tc_fence_after();
    tmem_dealloc(*slot, 512);
  }
}

// MUFU ex2.approx.ftz.f32: eight independent chains per thread, 8 warps.
__global__ void mufu_probe(int iters, unsigned long long* cycles, float* sink) {
  float x[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) x[i] = -1e-3f * (threadIdx.x + i);
  __syncthreads();
  const unsigned long long t0 = clock64();
  for (int it = 0; it < iters; ++it) {
#pragma unroll
    for (int i = 0; i < 8; ++i) asm volatile("ex2.approx.ftz.f32 %0, %0;" : "+f"(x[i]));
  }
  __syncthreads();
  const unsigned long long t1 = clock64();
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) s += x[i];
  sink[blockIdx.x * blockDim.x + threadIdx.x] = s;
  if (threadIdx.x == 0) cycles[blockIdx.x] = t1 - t0;
}

// The per-element work of the softmax P loop, in pairs, 16 pairs per thread
// per iteration, 8 warps (two per scheduler, as in the attention kernel):
//   mode 0  2 ex2
//   mode 1  2 ex2 + cvt.rn.bf16x2.f32
//   mode 2  cvt.rn.bf16x2.f32 alone
//   mode 3  2 ex2 + round-to-nearest-even bf16 packing on the integer pipe
//   mode 4  the whole pair: fma.f32x2 (scale, subtract max), 2 ex2,
//           add.f32x2 (row sums), cvt.rn.bf16x2.f32
//   mode 5  mode 4 with the integer packing of mode 3
//   mode 6  ex2.approx.ftz.bf16x2 (two bf16 exponentials per instruction)
//   mode 7  ex2.approx.f16x2
// Every value is carried from one iteration to the next (ex2 and fma update
// their own inputs, the cvt of mode 2 feeds its word back as the next input,
// packed words are folded into one xor), so the assembler can hoist none of
// them out of the loop.  Elements per cycle per SM = 32 * threads * iters /
// cycles (pairs of modes 2, 6 and 7 count as 2).
__device__ __forceinline__ uint32_t probe_pack_rne_int(float a, float b) {
  // Round-to-nearest-even of two non-negative finite floats to bf16 by
  // integer arithmetic: add 0x7FFF plus the lowest kept bit, keep the top
  // halves (bytes 2-3 of each word).
  const uint32_t ua = __float_as_uint(a), ub = __float_as_uint(b);
  const uint32_t ta = ua + 0x7FFFu + ((ua >> 16) & 1u);
  const uint32_t tb = ub + 0x7FFFu + ((ub >> 16) & 1u);
  return __byte_perm(ta, tb, 0x7632);
}

template <int kMode>
__global__ void softmax_mix_probe(int iters, unsigned long long* cycles, uint32_t* sink) {
  float x[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) x[i] = -1e-3f * (threadIdx.x + i);
  uint32_t acc = 0;
  uint64_t rs = 0;
  const uint64_t sc2 = (static_cast<uint64_t>(__float_as_uint(0.125f)) << 32) |
                       __float_as_uint(0.125f);
  const uint64_t nm2 = (static_cast<uint64_t>(__float_as_uint(-2.0f)) << 32) |
                       __float_as_uint(-2.0f);
  __syncthreads();
  const unsigned long long t0 = clock64();
  for (int it = 0; it < iters; ++it) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      float& a = x[2 * j];
      float& b = x[2 * j + 1];
      if (kMode == 6 || kMode == 7) {
        uint32_t r = __float_as_uint(a);
        if (kMode == 6)
          asm volatile("ex2.approx.ftz.bf16x2 %0, %0;" : "+r"(r));
        else
          asm volatile("ex2.approx.f16x2 %0, %0;" : "+r"(r));
        a = __uint_as_float(r);
        continue;
      }
      if (kMode == 2) {
        uint32_t r;
        asm volatile("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
        a = __uint_as_float(r);
        continue;
      }
      float pa = a, pb = b;
      if (kMode >= 4) {
        // s <- s * 0.125 - 2 (carried), p = 2^s
        uint64_t s2 = (static_cast<uint64_t>(__float_as_uint(b)) << 32) | __float_as_uint(a);
        asm volatile("fma.rn.f32x2 %0, %0, %1, %2;" : "+l"(s2) : "l"(sc2), "l"(nm2));
        a = __uint_as_float(static_cast<uint32_t>(s2));
        b = __uint_as_float(static_cast<uint32_t>(s2 >> 32));
        asm volatile("ex2.approx.ftz.f32 %0, %1;" : "=f"(pa) : "f"(a));
        asm volatile("ex2.approx.ftz.f32 %0, %1;" : "=f"(pb) : "f"(b));
        const uint64_t p2 =
            (static_cast<uint64_t>(__float_as_uint(pb)) << 32) | __float_as_uint(pa);
        asm volatile("add.rn.f32x2 %0, %0, %1;" : "+l"(rs) : "l"(p2));
      } else {
        asm volatile("ex2.approx.ftz.f32 %0, %0;" : "+f"(a));
        asm volatile("ex2.approx.ftz.f32 %0, %0;" : "+f"(b));
        pa = a;
        pb = b;
      }
      if (kMode == 1 || kMode == 4) {
        uint32_t r;
        asm volatile("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(pb), "f"(pa));
        acc ^= r;
      } else if (kMode == 3 || kMode == 5) {
        acc ^= probe_pack_rne_int(pa, pb);
      }
    }
  }
  __syncthreads();
  const unsigned long long t1 = clock64();
  uint32_t fold = acc ^ static_cast<uint32_t>(rs) ^ static_cast<uint32_t>(rs >> 32);
#pragma unroll
  for (int i = 0; i < 32; ++i) fold ^= __float_as_uint(x[i]);
  sink[blockIdx.x * blockDim.x + threadIdx.x] = fold;
  if (threadIdx.x == 0) cycles[blockIdx.x] = t1 - t0;
}

__global__ void copy_probe(const uint4* __restrict__ src, uint4* __restrict__ dst, size_t n) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    dst[i] = src[i];
}

double mean_cycles(const unsigned long long* d, int n) {
  unsigned long long h[1024];
  cudaMemcpy(h, d, n * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
  double s = 0;
  int k = 0;
  for (int i = 0; i < n; ++i)
    if (h[i]) {
      s += static_cast<double>(h[i]);
      ++k;
    }
  return k ? s / k : 0.0;
}

bool status_ok() {
  uint32_t st = 0;
  cudaMemcpyFromSymbol(&st, g_status, sizeof(st));
  if (st != 0) {
    std::fprintf(stderr, "device wait timed out (status 0x%08x)\n", st);
    const uint32_t zero = 0;
    cudaMemcpyToSymbol(g_status, &zero, sizeof(zero));
    return false;
  }
  return cudaGetLastError() == cudaSuccess;
}

}  // namespace

int main(int argc, char** argv) {
  std::string probe = "all";
  int iters = 4096, device = 0;
  for (int i = 1; i < argc; ++i) {
    const std::string f = argv[i];
    auto next = [&]() -> const char* {
      if (i + 1 >= argc) std::exit(2);
      return argv[++i];
    };
    if (f == "--help") {
      std::printf("peak_probe [--probe mma|issue|tile|tmem|mufu|softmax|hbm|all] [--iters N] [--device N]\n");
      return 0;
    } else if (f == "--probe") probe = next();
    else if (f == "--iters") iters = std::atoi(next());
    else if (f == "--device") device = std::atoi(next());
    else {
      std::fprintf(stderr, "unknown argument %s\n", f.c_str());
      return 2;
    }
  }
  if (iters < 16 || iters > (1 << 20) ||
      (probe != "mma" && probe != "issue" && probe != "tile" && probe != "tmem" && probe != "mufu" && probe != "softmax" &&
       probe != "hbm" && probe != "all")) {
    std::fprintf(stderr, "invalid arguments (see --help)\n");
    return 2;
  }
  cudaDeviceProp prop{};
  if (cudaSetDevice(device) != cudaSuccess ||
      cudaGetDeviceProperties(&prop, device) != cudaSuccess || prop.major < 10) {
    std::fprintf(stderr, "no sm_100 device %d\n", device);
    return 77;
  }
  const int sms = prop.multiProcessorCount;
  int clock_khz = 0;
  cudaDeviceGetAttribute(&clock_khz, cudaDevAttrClockRate, device);
  unsigned long long* cyc = nullptr;
  uint32_t* sink = nullptr;
  cudaMalloc(&cyc, 1024 * sizeof(unsigned long long));
  cudaMalloc(&sink, 1024 * 1024 * sizeof(uint32_t));
  cudaFuncSetAttribute(mma_probe, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemProbe);
  cudaFuncSetAttribute(tmem_probe, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemProbe);
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  int rc = 0;
  auto timed = [&](auto launch) {
    launch();  // warm-up
    cudaDeviceSynchronize();
    cudaMemset(cyc, 0, 1024 * sizeof(unsigned long long));
    cudaEventRecord(e0);
    launch();
    cudaEventRecord(e1);
    cudaEventSynchronize(e1);
    float ms = 0;
    cudaEventElapsedTime(&ms, e0, e1);
    if (!status_ok()) rc = 1;
    return static_cast<double>(ms);
  };
  if (probe == "mma" || probe == "all") {
    // {N, A source, accumulators}
    const int shapes[6][3] = {{256, 0, 1}, {128, 0, 1}, {128, 1, 1},
                              {128, 0, 2}, {128, 1, 2}, {128, 2, 2}};
    const char* src_name[3] = {"ss", "ts", "ss_ts"};
    for (int fill = 0; fill < 2; ++fill) {
      for (const auto& sh : shapes) {
        const int n = sh[0], ts = sh[1], accs = sh[2];
        const double ms = timed([&] {
          mma_probe<<<sms, 128, kSmemProbe>>>(n, ts, accs, fill, iters, cyc);
        });
        const double per_mma = mean_cycles(cyc, sms) / (4.0 * iters);
        const double flops = 2.0 * 128 * n * 16 * 4.0 * iters * sms;
        std::printf("probe=mma_m128_n%d_%s_%dacc%s cycles_per_mma=%.2f value=%.1f "
                    "unit=TFLOP/s ms=%.4f\n", n, src_name[ts], accs, fill ? "_ones" : "",
                    per_mma, flops / (ms * 1e-3) / 1e12, ms);
      }
    }
  }
  if (probe == "mma" || probe == "all") {
    cudaFuncSetAttribute(mma_pair_probe, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kSmemProbe);
    for (int n : {128, 256}) {
      const int pairs = sms / 2;
      const double ms = timed([&] {
        mma_pair_probe<<<2 * pairs, 128, kSmemProbe>>>(n, iters, cyc);
      });
      const double per_mma = mean_cycles(cyc, pairs) / (4.0 * iters);
      const double flops = 2.0 * 256 * n * 16 * 4.0 * iters * pairs;
      std::printf("probe=mma_pair_m256_n%d_ss cycles_per_mma=%.2f value=%.1f unit=TFLOP/s "
                  "ms=%.4f\n", n, per_mma, flops / (ms * 1e-3) / 1e12, ms);
    }
  }
  if (probe == "issue" || probe == "all") {
    // M128 N128 SS: issue warps per CTA x CTAs per SM (at most four 128-column
    // accumulators per SM), same or distinct operands.
    const int combos[6][2] = {{1, 1}, {2, 1}, {4, 1}, {1, 2}, {1, 4}, {2, 2}};
    for (int fill = 1; fill >= 0; --fill) {
      for (int reuse = 1; reuse >= 0; --reuse) {
        for (const auto& c : combos) {
          const int issuers = c[0], per_sm = c[1];
          const int grid = sms * per_sm;
          if (grid > 1024) continue;
          if (fill == 0 && (issuers != 1 || per_sm != 1)) continue;
          const double ms = timed([&] {
            mma_issue_probe<<<grid, 128>>>(issuers, reuse, fill, iters, cyc);
          });
          unsigned long long h[1024];
          cudaMemcpy(h, cyc, grid * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
          unsigned long long mx = 0;
          for (int i = 0; i < grid; ++i) mx = h[i] > mx ? h[i] : mx;
          const double mmas_per_sm = 4.0 * iters * issuers * per_sm;
          const double flops = 2.0 * 128 * 128 * 16 * mmas_per_sm * sms;
          std::printf("probe=issue_m128_n128_ss_%s%s issuers_per_cta=%d ctas_per_sm=%d "
                      "cycles_per_mma_per_sm=%.2f value=%.1f unit=TFLOP/s ms=%.4f\n",
                      reuse ? "same_operands" : "distinct_operands", fill ? "" : "_zeros",
                      issuers, per_sm, static_cast<double>(mx) / mmas_per_sm,
                      flops / (ms * 1e-3) / 1e12, ms);
        }
      }
    }
  }
  if (probe == "tile" || probe == "all") {
    cudaFuncSetAttribute(tile_issue_probe, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kSmemProbe);
    const char* names[5] = {"mma_only", "commits", "commits_waits", "two_issuers_commits_waits",
                            "two_issuers_mma_only"};
    const int tiles = iters / 4 > 16 ? iters / 4 : 16;
    for (int mode = 0; mode < 5; ++mode) {
      const double ms = timed([&] {
        tile_issue_probe<<<sms, 128, kSmemProbe>>>(mode, tiles, cyc);
      });
      const double per_tile = mean_cycles(cyc, sms) / tiles;
      const double flops = 4.0 * 128 * 128 * 128 * tiles * sms;
      std::printf("probe=tile_issue_d128_%s cycles_per_tile=%.1f value=%.1f unit=TFLOP/s "
                  "ms=%.4f\n", names[mode], per_tile, flops / (ms * 1e-3) / 1e12, ms);
    }
  }
  if (probe == "tmem" || probe == "all") {
    for (int store = 0; store < 2; ++store) {
      const double ms = timed([&] {
        tmem_probe<<<sms, 128, kSmemProbe>>>(store, iters, cyc, sink);
      });
      const double c = mean_cycles(cyc, sms);
      const double bytes_per_sm = 128.0 * 32 * 4 * iters;
      std::printf("probe=tmem_%s_32x32b_x32 bytes_per_cycle_per_sm=%.1f value=%.1f unit=TB/s "
                  "ms=%.4f\n", store ? "st" : "ld", bytes_per_sm / c,
                  bytes_per_sm * sms / (ms * 1e-3) / 1e12, ms);
    }
  }
  if (probe == "mufu" || probe == "all") {
    const double ms = timed([&] {
      mufu_probe<<<sms, 256>>>(iters, cyc, reinterpret_cast<float*>(sink));
    });
    const double c = mean_cycles(cyc, sms);
    const double ops = 256.0 * 8 * iters;
    std::printf("probe=mufu_ex2_f32 lanes_per_cycle_per_sm=%.2f value=%.1f unit=Gop/s ms=%.4f\n",
                ops / c, ops * sms / (ms * 1e-3) / 1e9, ms);
  }
  if (probe == "softmax" || probe == "all") {
    // The ninth line repeats pair_cvt with one warp per scheduler (128
    // threads): what a lone softmax warp can draw from MUFU.
    static const char* kNames[9] = {"ex2",          "ex2_cvt",      "cvt",
                                    "ex2_intpack",  "pair_cvt",     "pair_intpack",
                                    "ex2_bf16x2",   "ex2_f16x2",    "pair_cvt_1warp"};
    for (int mode = 0; mode < 9 && rc == 0; ++mode) {
      const int threads = mode == 8 ? 128 : 256;
      const double ms = timed([&] {
        switch (mode) {
          case 8: softmax_mix_probe<4><<<sms, 128>>>(iters, cyc, sink); break;
          case 0: softmax_mix_probe<0><<<sms, 256>>>(iters, cyc, sink); break;
          case 1: softmax_mix_probe<1><<<sms, 256>>>(iters, cyc, sink); break;
          case 2: softmax_mix_probe<2><<<sms, 256>>>(iters, cyc, sink); break;
          case 3: softmax_mix_probe<3><<<sms, 256>>>(iters, cyc, sink); break;
          case 4: softmax_mix_probe<4><<<sms, 256>>>(iters, cyc, sink); break;
          case 5: softmax_mix_probe<5><<<sms, 256>>>(iters, cyc, sink); break;
          case 6: softmax_mix_probe<6><<<sms, 256>>>(iters, cyc, sink); break;
          default: softmax_mix_probe<7><<<sms, 256>>>(iters, cyc, sink); break;
        }
      });
      const double c = mean_cycles(cyc, sms);
      const double elems = static_cast<double>(threads) * 32 * iters;
      std::printf("probe=softmax_%s elements_per_cycle_per_sm=%.2f value=%.1f unit=Gelem/s "
                  "ms=%.4f\n", kNames[mode], elems / c, elems * sms / (ms * 1e-3) / 1e9, ms);
    }
  }
  if (probe == "hbm" || probe == "all") {
    const size_t bytes = static_cast<size_t>(1) << 30;
    void *src = nullptr, *dst = nullptr;
    if (cudaMalloc(&src, bytes) != cudaSuccess || cudaMalloc(&dst, bytes) != cudaSuccess) {
      std::fprintf(stderr, "hbm probe: allocation failed\n");
      rc = 1;
    } else {
      cudaMemset(src, 1, bytes);
      const size_t n = bytes / 16;
      const double ms = timed([&] {
        copy_probe<<<sms * 8, 512>>>(static_cast<const uint4*>(src), static_cast<uint4*>(dst),
                                     n);
      });
      std::printf("probe=hbm_copy_1GiB value=%.1f unit=GB/s (read+write) ms=%.4f\n",
                  2.0 * bytes / (ms * 1e-3) / 1e9, ms);
    }
    cudaFree(src);
    cudaFree(dst);
  }
  std::printf("device=\"%s\" sms=%d clock_khz=%d\n", prop.name, sms, clock_khz);
  cudaFree(cyc);
  cudaFree(sink);
  return rc;
}
