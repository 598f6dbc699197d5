// Fused attention forward, head_dim 64, non-causal: two Q tiles per work unit.
//
// The same operation as attention_fwd_kernel (attention_kernel.cuh), for the
// shapes where the softmax's exp2 work, not the tensor core, bounds the tile:
// at d=64 the two products of a 128-key tile take about half the tensor time
// of d=128 while the 128 x 128 exponentials stay (the reference's config 4,
// 0.attention: B64 H16 N2048 d64).  A work unit is a pair of adjacent
// 128-row Q tiles A and B of one (batch, q head); both stream the head's K/V
// tiles once, and each has its own softmax pipe:
//
//   warps 0-3   pipe A softmax, warps 4-7 pipe B softmax: thread `lane` of
//               warp w owns query row 32*(w%4) + lane of its pipe's Q tile
//               and all 128 keys of a tile (no cross-thread reduction)
//   warps 8-11  epilogue: O / l -> bf16 -> shared (the pipe's Q buffer) ->
//               TMA store, pipe by pipe
//   warp  12    TMA producer for Q (both pipes) and the K ring; TMEM allocator
//   warp  13    O += P V issuer (both pipes)
//   warp  14    TMA producer for the V ring
//   warp  15    S = Q K^T issuer (both pipes)
//
// The two pipes share no state: each has its own running maxima, row sums and
// O accumulator, so neither ever waits for the other, and their phases drift
// apart.  While one pipe's warps run their exp2 loop, the other pipe's warps on
// the same schedulers work through their control chain (score load, screen,
// publish), which leaves MUFU idle in the one-Q-tile kernel.
//
// TMEM (512 columns): three S buffers [0,128) [128,256) [256,384) rotate over
// the unit's S sequence S(A,0), S(B,0), S(A,1), S(B,1), ... (crossing units);
// O_A at [384,448), O_B at [448,512).  P (bf16 pairs, keys 2c and 2c+1 in
// column c) overwrites the first 64 columns of its S buffer and is consumed
// by a TS-MMA.  S(u+3) reuses the buffer of S(u) once PV(u) has completed
// (p_free), so each pipe can run up to about a tile ahead of the other.
//
// Softmax per tile (one row per thread): an item's first tile and a masked
// tail tile take the exact row max; later tiles compute P against the
// running max and take the max only if the row's P sum exceeds 2^8 (some
// exponent then may have, since every term is at most the sum); O and the
// row sum are rescaled only when the max rises by more than 2^8, exactly as
// in the one-Q-tile kernel.  One exp2 pair in eight runs on the FMA pipe
// (kEmu = 1).
//
// Every wait is bounded (ptx.cuh); a timeout sets the device status word and
// every role unwinds as in the one-Q-tile kernel.
#pragma once

#include "attention_kernel.cuh"

namespace b200 {
namespace attn {
namespace pair {

constexpr int D = 64;
constexpr int kTileBytes = 128 * 128;  // 128 rows x 64 bf16 (one 128-byte-swizzled box)
constexpr int kKStages = 4;
constexpr int kVStages = 4;
constexpr int kQOff = 0;  // Q[pipe][buf], 4 tiles (also the pipe's O staging)
constexpr int kKOff = 4 * kTileBytes;
constexpr int kVOff = kKOff + kKStages * kTileBytes;
constexpr int kLOff = kVOff + kVStages * kTileBytes;  // (m, l) [pipe][128]
constexpr int kFlagOff = kLOff + 2 * 128 * 8;          // abort flag (epilogue)
constexpr int kBarOff = kFlagOff + 16;
// q_full[2][2] q_empty[2][2] k_full[K] k_empty[K] v_full[V] v_empty[V]
// s_ready[3] p_ready[3] p_free[3] pv_done[2] o_full[2] o_empty[2] l_ready[2]
// drain done
constexpr int kNumBars = 8 + 2 * kKStages + 2 * kVStages + 3 * kSBufs + 8 + 2;
constexpr int kTmemSlotOff = kBarOff + kNumBars * 8;
constexpr int kSmemBytes = kTmemSlotOff + 16 + 1024;  // + 1 KiB alignment slack
static_assert(kSmemBytes <= 232448, "exceeds the 227 KiB of shared memory a CTA may use");
constexpr uint32_t kIdescS = idesc_bf16_f32(128, kBN, false, false);
constexpr uint32_t kIdescO = idesc_bf16_f32(128, D, false, true);
constexpr uint32_t kColO = 128 * kSBufs;  // O of pipe p at kColO + 64 p

// Work unit k: Q tiles 2*pr and 2*pr+1 of plane bh; units of one head are
// adjacent, so the CTAs running at one time share its K/V in L2.
struct Unit {
  int zq, zkv, row0;
  int nq;  // Q tiles in the unit: 2, or 1 for the last of an odd count
};

__device__ __forceinline__ Unit decode_unit(const Params& p, int k) {
  const int npairs = (p.n_qtiles + 1) >> 1;
  const int bh = k / npairs;
  const int pr = k - bh * npairs;
  const int b = bh / p.Hq;
  const int hq = bh - b * p.Hq;
  Unit u;
  u.zq = bh;
  u.zkv = b * p.Hkv + hq / p.group;
  u.row0 = pr * 2 * kBM;
  u.nq = (2 * pr + 1 < p.n_qtiles) ? 2 : 1;
  return u;
}

__device__ __forceinline__ int unit_index(int r) {
  return r * static_cast<int>(gridDim.x) + static_cast<int>(blockIdx.x);
}

// P of a 128-key row (s: 128 scores), x = s * sc + nm, stored as bf16 pairs
// over the first 64 columns at tS (this thread's lane); keys at or past
// `valid` get exactly 0.  Accumulates the row sum in two packed pairs.
template <int kEmu, bool kMasked, int kC0 = 0, int kC1 = 8>
__device__ __forceinline__ void p_row(const float* s, float sc, float nm, int valid, uint32_t tS,
                                      uint64_t& ra, uint64_t& rb) {
  const uint64_t sc2 = f2_pack(sc, sc);
  const uint64_t nm2 = f2_pack(nm, nm);
#pragma unroll
  for (int c = kC0; c < kC1; ++c) {
    uint32_t pk[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int key = 16 * c + 2 * i;
      const uint64_t x2 = f2_fma(f2_pack(s[key], s[key + 1]), sc2, nm2);
      float x0, x1, p0, p1;
      f2_unpack(x2, x0, x1);
      if (kMasked) {
        x0 = key < valid ? x0 : -INFINITY;
        x1 = key + 1 < valid ? x1 : -INFINITY;
      }
      if (!kMasked && i < kEmu) {
        exp2_fma_x2(x0, x1, p0, p1);
      } else {
        p0 = ex2_approx(x0);
        p1 = ex2_approx(x1);
      }
      if (i & 1)
        rb = f2_add(rb, f2_pack(p0, p1));
      else
        ra = f2_add(ra, f2_pack(p0, p1));
      pk[i] = pack_bf16x2(p0, p1);
    }
    tmem_st8(tS + 8 * c, pk);
  }
}

// Largest of the row's first `valid` scores (all 128 when valid >= 128).
template <bool kMasked>
__device__ __forceinline__ float row_max(const float* s, int valid) {
  float a[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
  for (int i = 0; i < 128; i += 2) {
    if (kMasked) {
      const float v0 = i < valid ? s[i] : -INFINITY;
      const float v1 = i + 1 < valid ? s[i + 1] : -INFINITY;
      a[(i >> 1) & 3] = fmax3(a[(i >> 1) & 3], v0, v1);
    } else {
      a[(i >> 1) & 3] = fmax3(a[(i >> 1) & 3], s[i], s[i + 1]);
    }
  }
  return fmaxf(fmaxf(a[0], a[1]), fmaxf(a[2], a[3]));
}

template <int kEmu, bool kTrace = false>
__global__ void __launch_bounds__(kThreads, 1)
    attention_pair_kernel(const __grid_constant__ CUtensorMap q_map,
                          const __grid_constant__ CUtensorMap k_map,
                          const __grid_constant__ CUtensorMap v_map,
                          const __grid_constant__ CUtensorMap o_map, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* q_buf = smem + kQOff;  // [pipe][buf]
  uint8_t* k_buf = smem + kKOff;
  uint8_t* v_buf = smem + kVOff;
  float2* stat = reinterpret_cast<float2*>(smem + kLOff);  // [pipe][row] = (m, l)
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kFlagOff);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBarOff);
  uint64_t* q_full = bars;          // [pipe * 2 + buf]
  uint64_t* q_empty = q_full + 4;   // [pipe * 2 + buf]
  uint64_t* k_full = q_empty + 4;
  uint64_t* k_empty = k_full + kKStages;
  uint64_t* v_full = k_empty + kKStages;
  uint64_t* v_empty = v_full + kVStages;
  uint64_t* s_ready = v_empty + kVStages;
  uint64_t* p_ready = s_ready + kSBufs;
  uint64_t* p_free = p_ready + kSBufs;
  uint64_t* pv_done = p_free + kSBufs;  // [pipe]
  uint64_t* o_full = pv_done + 2;       // [pipe]
  uint64_t* o_empty = o_full + 2;       // [pipe]
  uint64_t* l_ready = o_empty + 2;      // [pipe]
  uint64_t* drain = l_ready + 2;
  uint64_t* done = drain + 1;  // phase 0 completes at setup and never changes
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kTmemSlotOff);

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();
  const int rounds = (p.n_items + static_cast<int>(gridDim.x) - 1) / static_cast<int>(gridDim.x);
  const int n = (p.Skv + kBN - 1) / kBN;  // K/V tiles per unit
  const int tail = p.Skv - (n - 1) * kBN;  // valid keys of the last tile (1..128)

  if (threadIdx.x == 0) {
    for (int i = 0; i < 4; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    for (int s = 0; s < kKStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < kVStages; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int i = 0; i < kSBufs; ++i) {
      mbar_init(&s_ready[i], 1);
      mbar_init(&p_ready[i], 4);  // the pipe's four softmax warps
      mbar_init(&p_free[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&pv_done[i], 1);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], 4);  // the four epilogue warps
      mbar_init(&l_ready[i], 4);  // the pipe's four softmax warps
    }
    mbar_init(drain, 2);  // one commit from each MMA issuer
    mbar_init(done, 1);
    mbar_arrive(done);
    abort_flag[0] = 0;
    fence_mbar_init();
  }
  if (warp == kTmaWarp) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
    if (lane == 0) {
      tma_prefetch_desc(&q_map);
      tma_prefetch_desc(&k_map);
      tma_prefetch_desc(&v_map);
      tma_prefetch_desc(&o_map);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Clock trace (kTrace builds): roles as in the one-Q-tile kernel, the
  // softmax roles 2 and 3 being pipe A's warp 0 and pipe B's warp 4; MMA and
  // softmax records carry the S index u as the iteration and the pipe as the
  // tile.
  const bool trace_cta = kTrace && static_cast<int>(blockIdx.x) == p.trace_cta;

  if (warp >= static_cast<uint32_t>(kTmaWarp)) {
    setmaxnreg_dec<kCtlRegs>();
    if (warp == kTmaWarp || warp == kTmaVWarp) {
      // ================= TMA producers (Q + K, and V) =================
      if (lane == 0) {
        const bool is_k = warp == kTmaWarp;
        Tracer<kTrace> tr(p, is_k ? 0 : 5, trace_cta);
        const uint64_t pol_q = l2_policy_evict_first();
        const uint64_t pol_kv = l2_policy_evict_last();
        int t = 0, issued = 0, lq0 = 0, lq1 = 0;
        int q_last[2] = {-1, -1};  // last Q load per pipe (its lq), for the drain
        bool ok = true;
        for (int r = 0; r < rounds && ok; ++r) {
          const int k = unit_index(r);
          if (k >= p.n_items) continue;
          const Unit u = decode_unit(p, k);
          if (is_k) {
            for (int pp = 0; pp < u.nq && ok; ++pp) {
              const int lq = pp ? lq1 : lq0;
              const int qi = 2 * pp + (lq & 1);
              ok = mbar_wait(&q_empty[qi], (static_cast<uint32_t>(lq >> 1) & 1u) ^ 1u,
                             kSiteQEmpty, kDefaultWaitLimitNs, 20000u);
              if (!ok) break;
              mbar_arrive_expect_tx(&q_full[qi], kTileBytes);
              tma_load_3d(q_buf + qi * kTileBytes, &q_map, &q_full[qi], 0, u.row0 + pp * kBM,
                          u.zq, pol_q);
              q_last[pp] = lq;
            }
          }
          if (!ok) break;
          lq0 += 1;
          lq1 += u.nq > 1 ? 1 : 0;
          for (int j = 0; j < n; ++j, ++t) {
            if (is_k) {
              const int ks = t % kKStages;
              ok = mbar_wait(&k_empty[ks], (static_cast<uint32_t>(t / kKStages) & 1u) ^ 1u,
                             kSiteKEmpty, kDefaultWaitLimitNs, 20000u);
              if (!ok) break;
              tr(kEvTmaK, 0, t);
              mbar_arrive_expect_tx(&k_full[ks], kTileBytes);
              tma_load_3d(k_buf + ks * kTileBytes, &k_map, &k_full[ks], 0, j * kBN, u.zkv,
                          pol_kv);
            } else {
              const int vs = t % kVStages;
              ok = mbar_wait(&v_empty[vs], (static_cast<uint32_t>(t / kVStages) & 1u) ^ 1u,
                             kSiteVEmpty, kDefaultWaitLimitNs, 20000u);
              if (!ok) break;
              tr(kEvTmaV, 0, t);
              mbar_arrive_expect_tx(&v_full[vs], kTileBytes);
              tma_load_3d(v_buf + vs * kTileBytes, &v_map, &v_full[vs], 0, j * kBN, u.zkv,
                          pol_kv);
            }
            issued = t + 1;
          }
        }
        if (!ok) {
          // Unwinding: let every copy already issued land before the CTA exits.
          if (is_k) {
            for (int pp = 0; pp < 2; ++pp)
              if (q_last[pp] >= 0)
                drain_wait(&q_full[2 * pp + (q_last[pp] & 1)],
                           static_cast<uint32_t>(q_last[pp] >> 1) & 1u);
            for (int i = max(0, issued - kKStages); i < issued; ++i)
              drain_wait(&k_full[i % kKStages], static_cast<uint32_t>(i / kKStages) & 1u);
          } else {
            for (int i = max(0, issued - kVStages); i < issued; ++i)
              drain_wait(&v_full[i % kVStages], static_cast<uint32_t>(i / kVStages) & 1u);
          }
        }
      }
      __syncwarp();
    } else if (warp == kMmaWarp || warp == kMmaSWarp) {
      // ================= MMA issuers =================
      // Warp 15 issues S, warp 13 PV, for both pipes in the order S(A,j),
      // S(B,j) / PV(A,j), PV(B,j); u counts the S tiles of the CTA.
      const bool is_pv = warp == kMmaWarp;
      Tracer<kTrace> tr(p, is_pv ? 1 : 6, trace_cta && lane == 0);
      const uint64_t dq0 = sdesc_sw128(smem_u32(q_buf), 16, 1024);
      const uint64_t dk0 = sdesc_sw128(smem_u32(k_buf), 16, 1024);
      const uint64_t dv0 = sdesc_sw128(smem_u32(v_buf), kTileBytes, 1024);
      constexpr uint32_t kTile16 = kTileBytes >> 4;
      const uint32_t dn_a = smem_u32(done), dn_p = 0;
      auto bar = [](uint64_t* b_) { return smem_u32(b_); };
      auto wait3 = [&](uint32_t a0, uint32_t p0, uint32_t a1, uint32_t p1, uint32_t a2,
                       uint32_t p2, uint32_t site) -> bool {
        if (!__all_sync(0xffffffffu, mbar_wait3(a0, p0, a1, p1, a2, p2, site))) return false;
        tc_fence_after();
        return true;
      };
      int u = 0, t = 0, lq[2] = {0, 0};
      bool ok = true;
      for (int r = 0; r < rounds && ok; ++r) {
        const int k = unit_index(r);
        if (k >= p.n_items) continue;
        const Unit un = decode_unit(p, k);
        if (!is_pv) {
          for (int pp = 0; pp < un.nq && ok; ++pp)
            ok = wait3(bar(&q_full[2 * pp + (lq[pp] & 1)]), static_cast<uint32_t>(lq[pp] >> 1) & 1u,
                       dn_a, dn_p, dn_a, dn_p, kSiteQFull);
          for (int j = 0; j < n && ok; ++j, ++t) {
            const int ks = t % kKStages;
            ok = wait3(bar(&k_full[ks]), static_cast<uint32_t>(t / kKStages) & 1u, dn_a, dn_p,
                       dn_a, dn_p, kSiteKFull);
            for (int pp = 0; pp < un.nq && ok; ++pp, ++u) {
              const int sb = u % kSBufs;
              ok = wait3(bar(&p_free[sb]), (static_cast<uint32_t>(u / kSBufs) & 1u) ^ 1u, dn_a,
                         dn_p, dn_a, dn_p, kSitePvDone);
              if (!ok) break;
              tr(kEvMmaS, pp, u);
              const uint64_t dq = dq0 + (2 * pp + (lq[pp] & 1)) * kTile16;
              const uint64_t dk = dk0 + ks * kTile16;
              const uint32_t ts = tmem_base + static_cast<uint32_t>(sb * 128);
#pragma unroll
              for (int kk = 0; kk < D / 16; ++kk)
                mma_ss_warp(ts, dq + kk * 2, dk + kk * 2, kIdescS, kk > 0 ? 1u : 0u);
              mma_commit_warp(&s_ready[sb]);
            }
            if (ok) mma_commit_warp(&k_empty[ks]);
          }
        } else {
          for (int j = 0; j < n && ok; ++j, ++t) {
            const int vs = t % kVStages;
            for (int pp = 0; pp < un.nq && ok; ++pp, ++u) {
              const int sb = u % kSBufs;
              // V(j), P(u) and, for the unit's first tile, O of the pipe free
              // (the epilogue has read the pipe's previous unit).
              ok = wait3(bar(&v_full[vs]), static_cast<uint32_t>(t / kVStages) & 1u,
                         bar(&p_ready[sb]), static_cast<uint32_t>(u / kSBufs) & 1u,
                         j == 0 ? bar(&o_empty[pp]) : dn_a,
                         j == 0 ? (static_cast<uint32_t>(lq[pp] & 1) ^ 1u) : dn_p, kSitePReady);
              if (!ok) break;
              tr(kEvMmaPv, pp, u);
              const uint32_t to = tmem_base + kColO + static_cast<uint32_t>(pp * D);
              const uint32_t tp = tmem_base + static_cast<uint32_t>(sb * 128);
              const uint64_t dv = dv0 + vs * kTile16;
#pragma unroll
              for (int kk = 0; kk < kBN / 16; ++kk)
                mma_ts_warp(to, tp + kk * 8, dv + kk * (2048 >> 4), kIdescO,
                            (j > 0 || kk > 0) ? 1u : 0u);
              mma_commit_warp(&p_free[sb]);
              mma_commit_warp(&pv_done[pp]);
            }
            if (ok) mma_commit_warp(&v_empty[vs]);
          }
          if (ok)
            for (int pp = 0; pp < un.nq; ++pp) mma_commit_warp(&o_full[pp]);
        }
        lq[0] += 1;
        lq[1] += un.nq > 1 ? 1 : 0;
      }
      // Every MMA this warp issued has completed once its commit lands.
      mma_commit_warp(drain);
      drain_wait(drain, 0);
      __syncwarp();
    }
  } else if (warp < static_cast<uint32_t>(kEpiWarp0)) {
    setmaxnreg_inc<kSoftmaxRegs>();
    // ================= softmax (warps 0-7) =================
    const int pp = static_cast<int>(warp >> 2);
    const uint32_t quad = warp & 3u;
    const int row = static_cast<int>(quad * 32 + lane);
    const uint32_t lane_addr = (quad * 32u) << 16;
    const uint32_t tO = tmem_base + lane_addr + kColO + static_cast<uint32_t>(pp * D);
    const float c = p.scale_log2;
    Tracer<kTrace> tr(p, 2 + pp, trace_cta && quad == 0 && lane == 0);
    int u = 0, tp = 0, lq = 0;
    bool ok = true;
#pragma unroll 1
    for (int r = 0; r < rounds && ok; ++r) {
      const int k = unit_index(r);
      if (k >= p.n_items) continue;
      const Unit un = decode_unit(p, k);
      if (pp >= un.nq) {  // pipe B has no Q tile in this unit
        u += n * un.nq;
        continue;
      }
      float m = -INFINITY;  // running max of this row (log2 units)
      float l = 0.0f;       // row sum in m
#pragma unroll 1
      for (int j = 0; j < n; ++j, ++tp) {
        const int uu = u + j * un.nq + pp;
        const int sb = uu % kSBufs;
        const uint32_t tS = tmem_base + lane_addr + static_cast<uint32_t>(sb * 128);
        tr(kEvSmWait, pp, uu);
        ok = warp_wait(&s_ready[sb], static_cast<uint32_t>(uu / kSBufs) & 1u, kSiteSReady);
        if (!ok) break;
        tc_fence_after();
        tr(kEvSmReady, pp, uu);
        uint32_t sr[128];
        const bool masked = j == n - 1 && tail < kBN;
        const bool exact = j == 0 || masked;
        tmem_ld_32x32b_x64(tS, *reinterpret_cast<uint32_t(*)[64]>(&sr[0]));
        if (exact) {
          tmem_ld_32x32b_x64(tS + 64, *reinterpret_cast<uint32_t(*)[64]>(&sr[64]));
          tmem_wait_ld(*reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
          reg_written_here(*reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
          reg_written_here(*reinterpret_cast<uint32_t(*)[32]>(&sr[64]));
          reg_written_here(*reinterpret_cast<uint32_t(*)[32]>(&sr[96]));
        } else {
          // First half of the scores, then the second half's load runs
          // under the first half's P.
          tmem_wait_ld(*reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
          reg_written_here(*reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
          tmem_ld_32x32b_x64(tS + 64, *reinterpret_cast<uint32_t(*)[64]>(&sr[64]));
        }
        tr(kEvSmLdDone, pp, uu);
        const float* s = reinterpret_cast<const float*>(sr);
        float f = 1.0f;  // factor on O and l (a rescale)
        bool resc = false;  // some row of the warp rescaled (warp-uniform)
        uint64_t ra = 0ull, rb = 0ull;
        if (exact) {
          // Exact row max first (an item's first tile, or the masked tail).
          const float mx = (masked ? row_max<true>(s, tail) : row_max<false>(s, kBN)) * c;
          tr(kEvSmMaxDone, pp, uu);
          if (m == -INFINITY) {
            m = mx;
          } else if (mx > m + kRescaleLog2) {
            f = ex2_approx(m - mx);
            m = mx;
          }
          if (masked)
            p_row<kEmu, true>(s, c, -m, tail, tS, ra, rb);
          else
            p_row<kEmu, false>(s, c, -m, kBN, tS, ra, rb);
          resc = __any_sync(0xffffffffu, f != 1.0f);
        } else {
          // P against the running max; the row's P sum screens for a jump of
          // the max by more than 2^kRescaleLog2 (then some P exceeds 2^8, and
          // so does the sum).
          p_row<kEmu, false, 0, 4>(s, c, -m, kBN, tS, ra, rb);
          tmem_wait_ld(*reinterpret_cast<uint32_t(*)[32]>(&sr[64]));
          reg_written_here(*reinterpret_cast<uint32_t(*)[32]>(&sr[96]));
          p_row<kEmu, false, 4, 8>(s, c, -m, kBN, tS, ra, rb);
          tr(kEvSmPLoopDone, pp, uu);
          float e0, e1;
          f2_unpack(f2_add(ra, rb), e0, e1);
          const bool big = e0 + e1 > kRescaleP;
          if (__any_sync(0xffffffffu, big)) {
            bool raise = false;
            if (big) {
              const float mx = row_max<false>(s, kBN) * c;
              if (mx > m + kRescaleLog2) {
                f = ex2_approx(m - mx);
                m = mx;
                raise = true;
              }
            }
            resc = __any_sync(0xffffffffu, raise);
            if (resc) {
              // Redo P against the raised maxima (rows that did not move
              // recompute the same values).
              tmem_wait_st();
              ra = 0ull;
              rb = 0ull;
              p_row<kEmu, false>(s, c, -m, kBN, tS, ra, rb);
            }
          }
        }
        tr(kEvSmPComputed, pp, uu);
        // O holds this pipe's tiles before j in the old max: rescale it once
        // PV(j-1) has completed (rare; the tile's PV waits for this P).
        if (resc && j > 0) {
          ok = warp_wait(&pv_done[pp], static_cast<uint32_t>(tp - 1) & 1u, kSitePvDone);
          if (!ok) break;
          tc_fence_after();
#pragma unroll 1
          for (int c0 = 0; c0 < D; c0 += 16) {
            uint32_t o[16];
            tmem_ld16(tO + c0, o);
            tmem_wait_ld();
            reg_written_here16(o);
#pragma unroll
            for (int e = 0; e < 16; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * f);
            tmem_st16(tO + c0, o);
          }
        }
        {
          float e0, e1;
          f2_unpack(f2_add(ra, rb), e0, e1);
          l = l * f + (e0 + e1);
        }
        // Publish P (and any O rescale) to the PV issuer.
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        mbar_arrive_warp(&p_ready[sb]);
        tr(kEvSmPublished, pp, uu);
      }
      if (!ok) break;
      u += n * un.nq;
      // (m, l) of the unit's rows for the epilogue, once it has read the
      // pipe's previous unit.
      ok = warp_wait(&o_empty[pp], (static_cast<uint32_t>(lq) & 1u) ^ 1u, kSiteOEmpty);
      if (!ok) break;
      stat[pp * 128 + row] = make_float2(m, l);
      __syncwarp();
      mbar_arrive_warp(&l_ready[pp]);
      ++lq;
    }
  } else {
    setmaxnreg_dec<kEpiRegs>();
    // ================= epilogue (warps 8-11) =================
    const uint32_t quad = warp & 3u;
    const int row = static_cast<int>(quad * 32 + lane);
    const uint32_t lane_addr = (quad * 32u) << 16;
    const uint64_t pol_o = l2_policy_evict_first();
    int lq[2] = {0, 0};
    bool stop = false;
#pragma unroll 1
    for (int r = 0; r < rounds && !stop; ++r) {
      const int k = unit_index(r);
      if (k >= p.n_items) continue;
      const Unit un = decode_unit(p, k);
#pragma unroll 1
      for (int pp = 0; pp < un.nq; ++pp) {
        const int qi = 2 * pp + (lq[pp] & 1);
        const uint32_t par = static_cast<uint32_t>(lq[pp]) & 1u;
        const bool got = warp_wait(&o_full[pp], par, kSiteOFull) &&
                         warp_wait(&l_ready[pp], par, kSiteLReady);
        if (!got) abort_flag[0] = 1;
        tc_fence_after();
        const float2 ml = stat[pp * 128 + row];
        const float inv = (got && ml.y > 0.0f) ? 1.0f / ml.y : 0.0f;
        const uint32_t obase = smem_u32(q_buf + qi * kTileBytes);
        const uint32_t tO = tmem_base + lane_addr + kColO + static_cast<uint32_t>(pp * D);
#pragma unroll 1
        for (int c0 = 0; c0 < D; c0 += 32) {
          uint32_t o[32];
          if (got) {
            tmem_ld32(tO + c0, o);
            tmem_wait_ld(o);
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = 0u;
          }
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e)
              w[e] = pack_bf16x2(__uint_as_float(o[8 * h + 2 * e]) * inv,
                                 __uint_as_float(o[8 * h + 2 * e + 1]) * inv);
            const int ch = (((c0 + 8 * h) & 63) >> 3) ^ (row & 7);
            st_shared_v4(obase + row * 128 + ch * 16, w[0], w[1], w[2], w[3]);
          }
        }
        tc_fence_before();
        __syncwarp();
        mbar_arrive_warp(&o_empty[pp]);
        fence_proxy_async_smem();
        named_bar_sync(kBarEpilogue, 128);
        if (abort_flag[0] != 0) {
          stop = true;
          break;
        }
        if (quad == 0 && lane == 0) {
          tma_store_3d_hint(&o_map, q_buf + qi * kTileBytes, 0, un.row0 + pp * kBM, un.zq,
                            pol_o);
          bulk_commit_group();
          bulk_wait_group_read<0>();
          mbar_arrive(&q_empty[qi]);
        }
        __syncwarp();
        ++lq[pp];
      }
    }
  }

  // ---- teardown ----
  tc_fence_before();
  __syncthreads();
  if (warp == kTmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace pair
}  // namespace attn
}  // namespace b200
