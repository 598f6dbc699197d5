// bf16 GEMM for sm_100a: C[M,N] (bf16, row-major) = A[M,K] (row-major) x B,
// fp32 accumulation in TMEM.
//
// Replaces the reference's gemm256_tma_tcgen05_kernel
// (5.GEMM/gemm256_tma_tcgen05_bench.cu:519-736), which computes one 256x256
// tile per CTA with a fresh CTA per tile, waits on each pipe's MMA commit
// every K stage (:680) and sinks C into a checksum (:691-705).  Here a
// cluster of two CTAs computes each 256x256 tile with tcgen05 cta_group::2
// MMAs (M=256, N=256, K=16), persistent over the tiles in a grouped order
// (kGroupM row blocks share B columns while they are in L2), with two TMEM
// accumulators so that the epilogue of tile t overlaps the main loop of
// tile t+1.  B is either [N,K] ("column-major B", K-major in shared memory)
// or [K,N] (row-major, MN-major in shared memory, as the reference's 5.GEMM).
//
// Every wait is bounded (ptx.cuh) and reports a timeout in the status word.
#pragma once

#include "ptx.cuh"

namespace b200 {
namespace gemm {

enum : uint32_t { kSiteFull = 0x21, kSiteEmpty, kSiteAccFull, kSiteAccEmpty };

struct Params {
  int M, N, K;
  int tiles_m, tiles_n, k_blocks;
  int b_col_major;  // 1: B is [N,K]; 0: B is [K,N]
  int group_m;      // row blocks per raster group
};

// Tile t -> (m block, n block) in groups of `group` row blocks: a group's
// tiles walk its row blocks fastest, so the CTAs running at one time share
// a few B column blocks and a few A row blocks while they sit in L2.
__device__ __forceinline__ void tile_coords(const Params& p, int t, int group, int* mb, int* nb) {
  const int per_group = group * p.tiles_n;
  const int g = t / per_group;
  const int first_m = g * group;
  const int gsize = min(group, p.tiles_m - first_m);
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

// ===========================================================================
// 256x256 output tiles per cluster of two CTAs (tcgen05 cta_group::2, the
// reference's 256x256 CTA tile).
//
// Each CTA of the pair loads its 128 rows of A and its 128 rows (N) of B per
// 64-deep K stage; the even CTA issues M=256, N=256, K=16 MMAs that read both
// CTAs' shared memory and leave 128 accumulator rows in each CTA's TMEM.  Per
// SM and per stage that is 32 KiB of TMA traffic for 2 x 128x256x64 MACs,
// half the B bytes of a single-CTA 128x256 tile.  No copy is multicast:
// each CTA fetches its own halves.
//
//   warp 0 (both CTAs): TMA producer; both count their bytes on the even
//                       CTA's full[s] barrier, which the even CTA arms with
//                       the pair's total
//   warp 1 (even CTA):  MMA issuer; commits free the stage (empty[s]) and
//                       publish the accumulator (acc_full[a]) in both CTAs
//   warps 2-5 (both):   epilogue of this CTA's 128 rows; one arrive per warp
//                       on the even CTA's acc_empty[a] (8 per tile)
// ===========================================================================
namespace pair {
constexpr int kBM = 256;  // output rows per pair tile (128 per CTA)
constexpr int kBN = 256;  // output columns per pair tile (128 B rows per CTA)
constexpr int kHalf = 128;
constexpr int kBK = 64;
constexpr int kStages = 6;
constexpr int kThreads = 192;
constexpr int kTmaWarp = 0;
constexpr int kMmaWarp = 1;
constexpr int kGroupM = 8;
constexpr uint32_t kTmemCols = 512;  // two accumulators of 256 fp32 columns
constexpr int kABytes = kHalf * kBK * 2;        // 16 KiB
constexpr int kBBytes = kHalf * kBK * 2;        // 16 KiB
constexpr int kStageBytes = kABytes + kBBytes;  // 32 KiB
// C staging for the TMA stores: two 128-row x 64-column bf16 boxes
// (128-byte swizzled), used in turn.
constexpr int kCBoxCols = 64;
constexpr int kCBoxBytes = kHalf * kCBoxCols * 2;  // 16 KiB
constexpr int kCStageOff = kStages * kStageBytes;
constexpr int kBarOff = kCStageOff + 2 * kCBoxBytes;
constexpr int kNumBars = 2 * kStages + 5;  // full, empty, acc_full[2], acc_empty[2], drain
constexpr int kAbortOff = kBarOff + kNumBars * 8;  // epilogue abort flag
constexpr int kTmemSlotOff = kAbortOff + 16;
constexpr int kSmemBytes = kTmemSlotOff + 16 + 1024;
static_assert(kSmemBytes <= 232448, "exceeds the 227 KiB of shared memory a CTA may use");
constexpr uint32_t kAccEmptyArrivals = 8;  // 4 epilogue warps x 2 CTAs
constexpr int kBarEpilogue = 1;            // named barrier of the four epilogue warps
}  // namespace pair

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(pair::kThreads, 1)
    gemm_bf16_pair_kernel(const __grid_constant__ CUtensorMap a_map,
                          const __grid_constant__ CUtensorMap b_map,
                          const __grid_constant__ CUtensorMap c_map, const Params p) {
  constexpr int kBM = pair::kBM, kBN = pair::kBN, kHalf = pair::kHalf, kBK = pair::kBK;
  constexpr int kStages = pair::kStages, kTmaWarp = pair::kTmaWarp, kMmaWarp = pair::kMmaWarp;
  constexpr int kGroupM = pair::kGroupM, kABytes = pair::kABytes;
  constexpr int kStageBytes = pair::kStageBytes, kBarOff = pair::kBarOff;
  constexpr int kTmemSlotOff = pair::kTmemSlotOff;
  constexpr uint32_t kTmemCols = pair::kTmemCols;
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
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + pair::kAbortOff);
  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int num_tiles = p.tiles_m * p.tiles_n;
  const int cluster_id = static_cast<int>(blockIdx.x >> 1);
  const int num_clusters = static_cast<int>(gridDim.x >> 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], pair::kAccEmptyArrivals);
    }
    mbar_init(drain, 1);
    abort_flag[0] = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  if (warp == kTmaWarp && lane == 0) {
    tma_prefetch_desc(&a_map);
    tma_prefetch_desc(&b_map);
    tma_prefetch_desc(&c_map);
  }
  // Both CTAs' barriers are initialised before either touches the other's.
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == kTmaWarp) {
    // ================= TMA producer (both CTAs) =================
    if (lane == 0) {
      // evict_last on both operands: on B200 evict_normal / evict_first read
      // 8 % / 100 % more from DRAM at 8192^3 and 29 % / 92 % more at 16384^3
      // and ran slower
      const uint64_t pol = l2_policy_evict_last();
      const uint64_t pol_b = pol;
      const int group = p.group_m > 0 ? p.group_m : kGroupM;
      int it = 0, issued_last = -1, lt = 0;
      bool ok = true;
      for (int t = cluster_id; t < num_tiles && ok; t += num_clusters, ++lt) {
        int mb, nb;
        tile_coords(p, t, group, &mb, &nb);
        const int arow = mb * kBM + static_cast<int>(rank) * kHalf;
        const int brow = nb * kBN + static_cast<int>(rank) * kHalf;
        for (int kk = 0; kk < p.k_blocks; ++kk, ++it) {
          // Serpentine K: every other tile walks K downwards, so it starts on
          // the slabs the previous tile (whose row panel the raster usually
          // repeats) loaded last, which are still in L2.  The MMAs sum the
          // slabs in whatever order they arrive.
          const int kb = (lt & 1) ? p.k_blocks - 1 - kk : kk;
          const int s = it % kStages;
          const uint32_t ph = static_cast<uint32_t>(it / kStages) & 1u;
          // Every wait of this kernel suspends in try_wait (20 us hint)
          // instead of polling: 43 % fewer instructions at 8192^3.
          ok = mbar_wait(&empty[s], ph ^ 1u, kSiteEmpty, kDefaultWaitLimitNs, 20000u);
          if (!ok) break;
          uint8_t* sa = smem + s * kStageBytes;
          uint8_t* sb = sa + kABytes;
          if (leader) mbar_arrive_expect_tx(&full[s], 2 * kStageBytes);
          const uint32_t fb = mapa_shared(smem_u32(&full[s]), 0);
          tma_load_2d_pair(sa, &a_map, fb, kb * kBK, arow, pol);
          if (p.b_col_major) {
            tma_load_2d_pair(sb, &b_map, fb, kb * kBK, brow, pol_b);
          } else {
#pragma unroll
            for (int h = 0; h < kHalf / 64; ++h)
              tma_load_2d_pair(sb + h * (kBK * 128), &b_map, fb, brow + h * 64, kb * kBK,
                               pol_b);
          }
          issued_last = it;
        }
      }
      if (!ok) {
        // Unwinding: let the copies already issued land before the pair exits.
        if (leader) {
          for (int i = max(0, issued_last - kStages + 1); i <= issued_last; ++i)
            drain_wait(&full[i % kStages], static_cast<uint32_t>(i / kStages) & 1u);
        } else {
          spin_ns(200000);
        }
      }
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ================= MMA issuer (even CTA) =================
    // The whole warp runs the loop (operands stay warp-uniform); one elected
    // lane issues each MMA and commit.
    if (leader) {
      constexpr uint32_t idesc_k = idesc_bf16_f32(kBM, kBN, false, false);
      constexpr uint32_t idesc_mn = idesc_bf16_f32(kBM, kBN, false, true);
      const uint32_t idesc = p.b_col_major ? idesc_k : idesc_mn;
      const uint64_t da0 = sdesc_sw128(smem_u32(smem), 16, 1024);
      const uint64_t db0 = p.b_col_major ? sdesc_sw128(smem_u32(smem) + kABytes, 16, 1024)
                                         : sdesc_sw128(smem_u32(smem) + kABytes, kBK * 128, 1024);
      const uint32_t b_step = p.b_col_major ? 2u : (16u * 128u) >> 4;
      int it = 0, lt = 0;
      bool ok = true;
      for (int t = cluster_id; t < num_tiles && ok; t += num_clusters, ++lt) {
        const int a = lt & 1;
        ok = __all_sync(0xffffffffu, mbar_wait(&acc_empty[a],
                                               (static_cast<uint32_t>(lt >> 1) & 1u) ^ 1u,
                                               kSiteAccEmpty, kDefaultWaitLimitNs, 20000u));
        if (!ok) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(a * kBN);
        for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
          const int s = it % kStages;
          ok = __all_sync(0xffffffffu,
                          mbar_wait(&full[s], static_cast<uint32_t>(it / kStages) & 1u, kSiteFull,
                                    kDefaultWaitLimitNs, 20000u));
          if (!ok) break;
          tc_fence_after();
          const uint64_t da = da0 + s * (kStageBytes >> 4);
          const uint64_t db = db0 + s * (kStageBytes >> 4);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            mma_ss_pair_warp(d_tmem, da + k * 2, db + k * b_step, idesc, (kb | k) > 0 ? 1u : 0u);
          mma_commit_pair_both_warp(&empty[s], 0x3);
        }
        if (!ok) break;
        mma_commit_pair_both_warp(&acc_full[a], 0x3);
      }
      if (lane == 0) mma_commit_pair_local(drain);
      __syncwarp();
      drain_wait(drain, 0);
    }
    __syncwarp();
  } else {
    // ================= epilogue (warps 2-5, both CTAs) =================
    const uint32_t quad = warp & 3u;
    const int row = static_cast<int>(quad * 32 + lane);
    const uint32_t lane_addr = (quad * 32u) << 16;
    const uint32_t sbase = smem_u32(smem + pair::kCStageOff);
    const bool issuer = warp == 2 && lane == 0;  // issues this CTA's C stores
    // C is never read back: stored evict_first so its lines leave L2 before
    // the A and B panels the next tiles re-read (ncu at 16384^3: DRAM
    // traffic per launch 20.8 GB without the hint, 16.3-16.8 GB with it).
    const uint64_t pol_c = l2_policy_evict_first();
    int lt = 0, box = 0;
    for (int t = cluster_id; t < num_tiles; t += num_clusters, ++lt) {
      const int a = lt & 1;
      int mb, nb;
      tile_coords(p, t, p.group_m > 0 ? p.group_m : kGroupM, &mb, &nb);
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[a],
                                                        static_cast<uint32_t>(lt >> 1) & 1u,
                                                        kSiteAccFull, kDefaultWaitLimitNs, 20000u));
      if (!ok) abort_flag[0] = 1;
      // The four warps leave together: a warp whose wait ran out must not
      // leave the others at a named barrier.
      named_bar_sync(pair::kBarEpilogue, 128);
      if (abort_flag[0] != 0) break;
      tc_fence_after();
      const int grow0 = mb * kBM + static_cast<int>(rank) * kHalf;  // this CTA's first row
      // Row `row` of this CTA's 128 x 256 block, 64 columns at a time: TMEM
      // -> bf16 -> the 128-byte-swizzled staging box -> one TMA store (TMA
      // clips at the edges of C).
#pragma unroll 1
      for (int c0 = 0; c0 < kBN; c0 += pair::kCBoxCols, ++box) {
        const uint32_t sb = sbase + static_cast<uint32_t>((box & 1) * pair::kCBoxBytes);
        if (issuer) bulk_wait_group_read<1>();  // the box's previous store has read it
        named_bar_sync(pair::kBarEpilogue, 128);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t v[32];
          tmem_ld32(tmem_base + lane_addr + static_cast<uint32_t>(a * kBN + c0 + 32 * h), v);
          tmem_wait_ld(v);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e)
              w[e] = pack_bf16x2(__uint_as_float(v[8 * q + 2 * e]),
                                 __uint_as_float(v[8 * q + 2 * e + 1]));
            const int ch = (4 * h + q) ^ (row & 7);
            st_shared_v4(sb + row * 128 + ch * 16, w[0], w[1], w[2], w[3]);
          }
        }
        fence_proxy_async_smem();
        named_bar_sync(pair::kBarEpilogue, 128);
        if (issuer) {
          tma_store_2d_hint(&c_map, smem + pair::kCStageOff + (box & 1) * pair::kCBoxBytes,
                            nb * kBN + c0, grow0, pol_c);
          bulk_commit_group();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&acc_empty[a]), 0));
    }
    if (issuer) bulk_wait_group<0>();  // every store has completed
  }

  // No CTA leaves while its partner may still signal its barriers or read
  // its shared memory.
  tc_fence_before();
  cluster_sync_all();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

}  // namespace gemm
}  // namespace b200
