// bf16 GEMM for sm_100a: C[M,N] (bf16, row-major) = A[M,K] (row-major) x B,
// fp32 accumulation in TMEM.
//
// Replaces the reference's gemm256_tma_tcgen05_kernel
// (5.GEMM/gemm256_tma_tcgen05_bench.cu:519-736), which computes one 256x256
// tile per CTA with a fresh CTA per tile, waits on each pipe's MMA commit
// every K stage (:680) and sinks C into a checksum (:691-705).  Here:
//
//   * persistent CTAs (one per SM) walk 128x256 output tiles in a grouped
//     order (kGroupM row-blocks share B columns while they are in L2);
//   * warp 0: TMA producer over a kStages-deep ring of (A 128x64, B 256x64)
//     stages; warp 1: single-thread tcgen05.mma issuer (M=128, N=256, K=16,
//     the shape that runs at the full tensor rate); warps 2-5: epilogue;
//   * two TMEM accumulators of 256 columns: the epilogue of tile t (TMEM ->
//     registers -> bf16 -> global) overlaps the main loop of tile t+1;
//   * B is either [N,K] ("column-major B", K-major in shared memory) or
//     [K,N] (row-major, MN-major in shared memory, as the reference's 5.GEMM).
//
// Every wait is bounded (ptx.cuh) and reports a timeout in the status word.
#pragma once

#include "ptx.cuh"

namespace b200 {
namespace gemm {

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 64;
constexpr int kStages = 4;
constexpr int kThreads = 192;
constexpr int kTmaWarp = 0;
constexpr int kMmaWarp = 1;
constexpr int kGroupM = 16;
constexpr uint32_t kTmemCols = 512;
constexpr int kABytes = kBM * kBK * 2;           // 16 KiB
constexpr int kBBytes = kBN * kBK * 2;           // 32 KiB
constexpr int kStageBytes = kABytes + kBBytes;   // 48 KiB
constexpr int kBarOff = kStages * kStageBytes;
// full[S], empty[S], acc_full[2], acc_empty[2], drain
constexpr int kNumBars = 2 * kStages + 5;
constexpr int kTmemSlotOff = kBarOff + kNumBars * 8;
constexpr int kSmemBytes = kTmemSlotOff + 16 + 1024;

enum : uint32_t { kSiteFull = 0x21, kSiteEmpty, kSiteAccFull, kSiteAccEmpty };

struct Params {
  int M, N, K;
  int tiles_m, tiles_n, k_blocks;
  int b_col_major;  // 1: B is [N,K]; 0: B is [K,N]
  uint16_t* C;
};

// Tile t -> (m block, n block) in groups of kGroupM row blocks.
__device__ __forceinline__ void tile_coords(const Params& p, int t, int* mb, int* nb) {
  const int per_group = kGroupM * p.tiles_n;
  const int g = t / per_group;
  const int first_m = g * kGroupM;
  const int gsize = min(kGroupM, p.tiles_m - first_m);
  const int r = t - g * per_group;
  *mb = first_m + r % gsize;
  *nb = r / gsize;
}

__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(addr, parity)) {
    if (globaltimer_ns() - t0 > 50000000ull) break;
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap a_map,
                     const __grid_constant__ CUtensorMap b_map, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBarOff);
  uint64_t* full = bars;
  uint64_t* empty = bars + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kTmemSlotOff);
  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();
  const int num_tiles = p.tiles_m * p.tiles_n;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 128);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  if (warp == kTmaWarp && lane == 0) {
    tma_prefetch_desc(&a_map);
    tma_prefetch_desc(&b_map);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == kTmaWarp) {
    // ================= TMA producer =================
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_last();
      int it = 0, issued_last = -1;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int mb, nb;
        tile_coords(p, t, &mb, &nb);
        for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
          const int s = it % kStages;
          const uint32_t ph = static_cast<uint32_t>(it / kStages) & 1u;
          ok = mbar_wait(&empty[s], ph ^ 1u, kSiteEmpty);
          if (!ok) break;
          uint8_t* sa = smem + s * kStageBytes;
          uint8_t* sb = sa + kABytes;
          mbar_arrive_expect_tx(&full[s], kStageBytes);
          tma_load_2d(sa, &a_map, &full[s], kb * kBK, mb * kBM, pol);
          if (p.b_col_major) {
            tma_load_2d(sb, &b_map, &full[s], kb * kBK, nb * kBN, pol);
          } else {
#pragma unroll
            for (int h = 0; h < kBN / 64; ++h)
              tma_load_2d(sb + h * (kBK * 128), &b_map, &full[s], nb * kBN + h * 64, kb * kBK,
                          pol);
          }
          issued_last = it;
        }
      }
      if (!ok) {
        // Unwinding: let the copies already issued land before the CTA exits.
        for (int i = max(0, issued_last - kStages + 1); i <= issued_last; ++i)
          drain_wait(&full[i % kStages], static_cast<uint32_t>(i / kStages) & 1u);
      }
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ================= MMA issuer =================
    if (lane == 0) {
      constexpr uint32_t idesc_k = idesc_bf16_f32(kBM, kBN, false, false);
      constexpr uint32_t idesc_mn = idesc_bf16_f32(kBM, kBN, false, true);
      const uint32_t idesc = p.b_col_major ? idesc_k : idesc_mn;
      const uint64_t da0 = sdesc_sw128(smem_u32(smem), 16, 1024);
      const uint64_t db0 = p.b_col_major ? sdesc_sw128(smem_u32(smem) + kABytes, 16, 1024)
                                         : sdesc_sw128(smem_u32(smem) + kABytes, kBK * 128, 1024);
      // byte offset >> 4 of one K=16 step inside a stage's B tile
      const uint32_t b_step = p.b_col_major ? 2u : (16u * 128u) >> 4;
      int it = 0, lt = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++lt) {
        const int a = lt & 1;
        ok = mbar_wait(&acc_empty[a], (static_cast<uint32_t>(lt >> 1) & 1u) ^ 1u, kSiteAccEmpty);
        if (!ok) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(a * kBN);
        for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
          const int s = it % kStages;
          ok = mbar_wait(&full[s], static_cast<uint32_t>(it / kStages) & 1u, kSiteFull);
          if (!ok) break;
          tc_fence_after();
          const uint64_t da = da0 + s * (kStageBytes >> 4);
          const uint64_t db = db0 + s * (kStageBytes >> 4);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            mma_ss(d_tmem, da + k * 2, db + k * b_step, idesc, (kb | k) > 0 ? 1u : 0u);
          mma_commit(&empty[s]);
        }
        if (!ok) break;
        mma_commit(&acc_full[a]);
      }
      mma_commit(drain);
      drain_wait(drain, 0);
    }
    __syncwarp();
  } else {
    // ================= epilogue (warps 2-5) =================
    const uint32_t quad = warp & 3u;  // TMEM lane quadrant this warp may access
    const int row = static_cast<int>(quad * 32 + lane);
    const uint32_t lane_addr = (quad * 32u) << 16;
    int lt = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++lt) {
      const int a = lt & 1;
      int mb, nb;
      tile_coords(p, t, &mb, &nb);
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[a],
                                                        static_cast<uint32_t>(lt >> 1) & 1u,
                                                        kSiteAccFull));
      if (!ok) break;
      tc_fence_after();
      const int grow = mb * kBM + row;
      uint16_t* crow = p.C + static_cast<size_t>(grow) * p.N;
#pragma unroll 1
      for (int c0 = 0; c0 < kBN; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(tmem_base + lane_addr + static_cast<uint32_t>(a * kBN + c0), v);
        tmem_wait_ld();
        uint32_t w[16];
#pragma unroll
        for (int e = 0; e < 16; ++e)
          w[e] = pack_bf16x2(__uint_as_float(v[2 * e]), __uint_as_float(v[2 * e + 1]));
        const int gcol = nb * kBN + c0;
        if (grow < p.M) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            if (gcol + q * 8 < p.N)  // N % 8 == 0: an 8-column chunk is all in or all out
              *reinterpret_cast<uint4*>(crow + gcol + q * 8) =
                  make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[a]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace gemm
}  // namespace b200
