// Fused attention forward for sm_100a: O = softmax(Q K^T * scale) V.
//
// Replaces the reference's qk_tma_mma_ld_kernel (0.attention/attention.cu:1503-1974)
// and generalises it to the scalar path's semantics
// (real_attention_bf16_d128_kernel, attention.cu:210-274): any B, Hq, Hkv (GQA,
// attention.cu:176-183), Sq != Skv with bottom-right causal masking
// (attention.cu:167-174), ragged tails, head_dim 64 or 128.
//
// One CTA owns two 128-row Q tiles of one (batch, head) and streams that head's
// K/V tiles (128 keys each) once for both:
//
//   warps 0-3  softmax for Q tile 0 (one TMEM lane = one query row per thread)
//   warps 4-7  softmax for Q tile 1
//   warp  8    TMA producer (Q once, then the K/V ring) and TMEM allocator
//   warp  9    tcgen05.mma issuer (one thread)
//
// TMEM (512 columns): S0 [0,128) S1 [128,256) O0 [256,256+D) O1 [256+D,256+2D).
// The softmax overwrites the first 64 columns of S_i with P_i packed as bf16
// pairs, and the PV product reads P straight from TMEM (A operand in TMEM,
// V from shared memory, MN-major).  Issue order per KV tile j:
//   PV0(j), S0(j+1), PV1(j), S1(j+1)
// so each softmax warpgroup works on tile j while the tensor core runs the
// other warpgroup's matrix products.  tcgen05.mma instructions issued by one
// thread execute in order, so S_i(j+1) never overwrites P_i(j) before PV_i(j)
// has read it.
//
// Online softmax keeps a running row maximum m (in log2 units).  O and the row
// sum are rescaled only when a new block raises m by more than kRescaleLog2;
// otherwise P values up to 2^kRescaleLog2 are accumulated unscaled (exact in
// fp32, and the final O / l normalisation is unchanged).
//
// Every wait is bounded (ptx.cuh); a timeout sets the device status word and
// every role unwinds to the common teardown without trapping.
#pragma once

#include "ptx.cuh"

namespace b200 {
namespace attn {

constexpr int kBM = 128;  // query rows per Q tile (= TMEM lanes)
constexpr int kBN = 128;  // keys per K/V tile
constexpr int kThreads = 320;
constexpr int kTmaWarp = 8;
constexpr int kMmaWarp = 9;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleLog2 = 8.0f;

struct Params {
  int B, Hq, Hkv, Sq, Skv;
  int group;       // Hq / Hkv
  int n_qpairs;    // ceil(Sq / 256)
  int causal;      // bottom-right aligned
  int causal_off;  // Skv - Sq
  float scale_log2;  // softmax_scale * log2(e)
};

template <int D>
struct Cfg {
  static_assert(D == 64 || D == 128, "head_dim must be 64 or 128");
  static constexpr int kBoxes = D / 64;            // 64-column (128-byte) TMA boxes per tile
  static constexpr int kBoxBytes = 128 * 64 * 2;   // 16 KiB
  static constexpr int kTileBytes = kBoxes * kBoxBytes;
  static constexpr int kStages = (D == 128) ? 2 : 4;
  static constexpr int kQOff = 0;
  static constexpr int kKOff = 2 * kTileBytes;
  static constexpr int kVOff = kKOff + kStages * kTileBytes;
  static constexpr int kBarOff = kVOff + kStages * kTileBytes;
  // q_full, k_full[S], k_empty[S], v_full[S], v_empty[S], s_ready[2], p_ready[2],
  // o_final[2], drain
  static constexpr int kNumBars = 1 + 4 * kStages + 7;
  static constexpr int kTmemSlotOff = kBarOff + kNumBars * 8;
  static constexpr int kSmemBytes = kTmemSlotOff + 16 + 1024;  // + 1 KiB alignment slack
  static constexpr uint32_t kIdescS = idesc_bf16_f32(128, 128, false, false);
  static constexpr uint32_t kIdescO = idesc_bf16_f32(128, D, false, true);
};

// Wait sites reported in the status word.
enum : uint32_t {
  kSiteQFull = 1, kSiteKFull, kSiteVFull, kSitePReady, kSiteKEmpty, kSiteVEmpty,
  kSiteSReady, kSiteOFinal, kSiteDrain
};

// Number of K/V tiles Q tile `tile_row0` must visit (0 if it has no rows or no
// valid keys) and the smallest per-row key limit inside the tile.
__device__ __forceinline__ void tile_extent(const Params& p, int tile_row0, int* nblk,
                                            int* min_lim) {
  if (tile_row0 >= p.Sq) {
    *nblk = 0;
    *min_lim = 0;
    return;
  }
  const int last_q = min(tile_row0 + kBM - 1, p.Sq - 1);
  int lim = p.Skv;
  int lim0 = p.Skv;
  if (p.causal) {
    lim = min(p.Skv, last_q + p.causal_off + 1);
    lim0 = min(p.Skv, tile_row0 + p.causal_off + 1);
  }
  *nblk = lim <= 0 ? 0 : (lim + kBN - 1) / kBN;
  *min_lim = lim0;
}

// Warp-uniform bounded wait: the warp proceeds only if every lane observed the
// phase, so warp-collective tcgen05.ld/st never run on a partial warp.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, uint32_t site) {
  const bool ok = mbar_wait(bar, parity, site);
  return __all_sync(0xffffffffu, ok);
}

// Wait used only while unwinding after a timeout: ignores the status word and
// gives up after 50 ms (the awaited operations do not depend on other roles).
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(addr, parity)) {
    if (globaltimer_ns() - t0 > 50000000ull) break;
  }
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    attention_fwd_kernel(const __grid_constant__ CUtensorMap q_map,
                         const __grid_constant__ CUtensorMap k_map,
                         const __grid_constant__ CUtensorMap v_map,
                         const __grid_constant__ CUtensorMap o_map, const Params p) {
  using C = Cfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* q_buf = smem + C::kQOff;
  uint8_t* k_buf = smem + C::kKOff;
  uint8_t* v_buf = smem + C::kVOff;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = k_full + C::kStages;
  uint64_t* v_full = k_empty + C::kStages;
  uint64_t* v_empty = v_full + C::kStages;
  uint64_t* s_ready = v_empty + C::kStages;
  uint64_t* p_ready = s_ready + 2;
  uint64_t* o_final = p_ready + 2;
  uint64_t* drain = o_final + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kTmemSlotOff);

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();

  // ---- work item: (batch, q head, pair of Q tiles) ----
  int qpair = static_cast<int>(blockIdx.x % static_cast<uint32_t>(p.n_qpairs));
  const int bh = static_cast<int>(blockIdx.x / static_cast<uint32_t>(p.n_qpairs));
  if (p.causal) qpair = p.n_qpairs - 1 - qpair;  // heaviest tiles launch first
  const int b = bh / p.Hq;
  const int hq = bh - b * p.Hq;
  const int zq = bh;                            // (b * Hq + hq) plane of Q / O
  const int zkv = b * p.Hkv + hq / p.group;     // (b * Hkv + hkv) plane of K / V
  const int row0[2] = {qpair * 2 * kBM, qpair * 2 * kBM + kBM};
  int nblk[2], min_lim[2];
  tile_extent(p, row0[0], &nblk[0], &min_lim[0]);
  tile_extent(p, row0[1], &nblk[1], &min_lim[1]);
  const int nmax = max(nblk[0], nblk[1]);

  // ---- setup ----
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_ready[i], 1);
      mbar_init(&p_ready[i], 128);
      mbar_init(&o_final[i], 1);
    }
    mbar_init(drain, 1);
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

  if (warp == kTmaWarp) {
    // ================= TMA producer =================
    if (lane == 0 && nmax > 0) {
      const uint64_t pol_q = l2_policy_evict_first();
      const uint64_t pol_kv = l2_policy_evict_last();
      uint32_t q_bytes = 0;
      for (int i = 0; i < 2; ++i) q_bytes += nblk[i] > 0 ? C::kTileBytes : 0;
      mbar_arrive_expect_tx(q_full, q_bytes);
      for (int i = 0; i < 2; ++i) {
        if (nblk[i] == 0) continue;
        for (int h = 0; h < C::kBoxes; ++h)
          tma_load_3d(q_buf + i * C::kTileBytes + h * C::kBoxBytes, &q_map, q_full, h * 64,
                      row0[i], zq, pol_q);
      }
      int issued = 0;
      bool ok = true;
      for (int j = 0; j < nmax && ok; ++j) {
        const int s = j % C::kStages;
        const uint32_t ph = static_cast<uint32_t>(j / C::kStages) & 1u;
        ok = mbar_wait(&k_empty[s], ph ^ 1u, kSiteKEmpty);
        if (!ok) break;
        mbar_arrive_expect_tx(&k_full[s], C::kTileBytes);
        for (int h = 0; h < C::kBoxes; ++h)
          tma_load_3d(k_buf + s * C::kTileBytes + h * C::kBoxBytes, &k_map, &k_full[s], h * 64,
                      j * kBN, zkv, pol_kv);
        ok = mbar_wait(&v_empty[s], ph ^ 1u, kSiteVEmpty);
        if (!ok) {
          issued = j;  // K(j) in flight, V(j) not
          drain_wait(&k_full[s], ph);
          break;
        }
        mbar_arrive_expect_tx(&v_full[s], C::kTileBytes);
        for (int h = 0; h < C::kBoxes; ++h)
          tma_load_3d(v_buf + s * C::kTileBytes + h * C::kBoxBytes, &v_map, &v_full[s], h * 64,
                      j * kBN, zkv, pol_kv);
        issued = j + 1;
      }
      if (!ok) {
        // Unwinding: let every copy already issued land before the CTA exits.
        drain_wait(q_full, 0);
        for (int j = max(0, issued - C::kStages); j < issued; ++j) {
          const int s = j % C::kStages;
          const uint32_t ph = static_cast<uint32_t>(j / C::kStages) & 1u;
          drain_wait(&k_full[s], ph);
          drain_wait(&v_full[s], ph);
        }
      }
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ================= MMA issuer =================
    if (lane == 0 && nmax > 0) {
      const uint32_t q_addr = smem_u32(q_buf);
      const uint32_t k_addr = smem_u32(k_buf);
      const uint32_t v_addr = smem_u32(v_buf);
      const uint32_t tS[2] = {tmem_base, tmem_base + 128};
      const uint32_t tO[2] = {tmem_base + 256, tmem_base + 256 + D};

      auto issue_s = [&](int i, int s) {
        const uint32_t qa = q_addr + i * C::kTileBytes;
        const uint32_t ka = k_addr + s * C::kTileBytes;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * C::kBoxBytes + (kk & 3) * 32;
          mma_ss(tS[i], sdesc_sw128(qa + off, 16, 1024), sdesc_sw128(ka + off, 16, 1024),
                 C::kIdescS, kk > 0 ? 1u : 0u);
        }
      };
      auto issue_pv = [&](int i, int s, int j) {
        const uint32_t va = v_addr + s * C::kTileBytes;
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          mma_ts(tO[i], tS[i] + kk * 8, sdesc_sw128(va + kk * 2048, C::kBoxBytes, 1024),
                 C::kIdescO, (j > 0 || kk > 0) ? 1u : 0u);
        }
      };

      bool ok = mbar_wait(q_full, 0, kSiteQFull) && mbar_wait(&k_full[0], 0, kSiteKFull);
      if (ok) {
        tc_fence_after();
        for (int i = 0; i < 2; ++i) {
          if (nblk[i] > 0) {
            issue_s(i, 0);
            mma_commit(&s_ready[i]);
          }
        }
        mma_commit(&k_empty[0]);
      }
      for (int j = 0; j < nmax && ok; ++j) {
        const int s = j % C::kStages;
        const uint32_t ph = static_cast<uint32_t>(j / C::kStages) & 1u;
        const int jn = j + 1;
        const int sn = jn % C::kStages;
        const uint32_t phn = static_cast<uint32_t>(jn / C::kStages) & 1u;
        ok = mbar_wait(&v_full[s], ph, kSiteVFull);
        if (!ok) break;
        if (j < nblk[0]) {
          ok = mbar_wait(&p_ready[0], static_cast<uint32_t>(j) & 1u, kSitePReady);
          if (!ok) break;
          tc_fence_after();
          issue_pv(0, s, j);
          if (j == nblk[0] - 1) mma_commit(&o_final[0]);
        }
        if (jn < nmax) {
          ok = mbar_wait(&k_full[sn], phn, kSiteKFull);
          if (!ok) break;
          tc_fence_after();
          if (jn < nblk[0]) {
            issue_s(0, sn);
            mma_commit(&s_ready[0]);
          }
        }
        if (j < nblk[1]) {
          ok = mbar_wait(&p_ready[1], static_cast<uint32_t>(j) & 1u, kSitePReady);
          if (!ok) break;
          tc_fence_after();
          issue_pv(1, s, j);
          if (j == nblk[1] - 1) mma_commit(&o_final[1]);
        }
        mma_commit(&v_empty[s]);
        if (jn < nmax) {
          if (jn < nblk[1]) {
            issue_s(1, sn);
            mma_commit(&s_ready[1]);
          }
          mma_commit(&k_empty[sn]);
        }
      }
      // Every MMA issued above has completed once this commit lands.
      mma_commit(drain);
      drain_wait(drain, 0);
    }
    __syncwarp();
  } else {
    // ================= softmax + epilogue (warps 0-7) =================
    const int i = static_cast<int>(warp >> 2);  // Q tile
    const uint32_t quad = warp & 3u;
    const int row = static_cast<int>(quad * 32 + lane);
    const uint32_t lane_addr = (quad * 32u) << 16;
    const uint32_t tS = tmem_base + lane_addr + static_cast<uint32_t>(i) * 128u;
    const uint32_t tO = tmem_base + lane_addr + 256u + static_cast<uint32_t>(i * D);
    const int n = nblk[i];
    const int q = row0[i] + row;
    const int lim = p.causal ? min(p.Skv, q + p.causal_off + 1) : p.Skv;
    const float c = p.scale_log2;
    float m = -INFINITY;  // running max of scaled scores (log2 units)
    float l = 0.0f;       // running row sum of P
    bool ok = true;

#pragma unroll 1
    for (int j = 0; j < n; ++j) {
      ok = warp_wait(&s_ready[i], static_cast<uint32_t>(j) & 1u, kSiteSReady);
      if (!ok) break;
      tc_fence_after();
      uint32_t sr[128];
      tmem_ld32(tS + 0, *reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
      tmem_ld32(tS + 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
      tmem_ld32(tS + 64, *reinterpret_cast<uint32_t(*)[32]>(&sr[64]));
      tmem_ld32(tS + 96, *reinterpret_cast<uint32_t(*)[32]>(&sr[96]));
      tmem_wait_ld();
      float* s = reinterpret_cast<float*>(sr);

      const int kbase = j * kBN;
      const bool masked = kbase + kBN > min_lim[i];  // uniform across the tile
      float m_blk;
      if (masked) {
        // Scale first, then mask, so masked keys are exactly -inf for any scale.
        const int valid = lim - kbase;
        float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int e = 0; e < 128; ++e) {
          const float t = e < valid ? s[e] * c : -INFINITY;
          s[e] = t;
          mx[e & 3] = fmaxf(mx[e & 3], t);
        }
        m_blk = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
      } else {
        float mx[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) mx[e] = s[e];
#pragma unroll
        for (int e = 8; e < 128; ++e) mx[e & 7] = fmaxf(mx[e & 7], s[e]);
        m_blk = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                      fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7]))) *
                c;
      }

      // Running-max update with lazy rescaling.
      float factor = 1.0f;
      bool rescale = false;
      if (m == -INFINITY) {
        m = m_blk;  // no probability mass accumulated yet for this row
      } else if (m_blk > m + kRescaleLog2) {
        factor = ex2_approx(m - m_blk);
        m = m_blk;
        rescale = true;
      }
      // P = exp2(score * c - m) as bf16 pairs, written over the first 64
      // columns of S in two halves (S is fully in registers by now).
      const float m_use = (m == -INFINITY) ? 0.0f : m;
      const float sc = masked ? 1.0f : c;  // masked scores are pre-scaled
      const float nm = -m_use;
      float rs[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t pk[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const float p0 = ex2_approx(fmaf(s[64 * half + 2 * e], sc, nm));
          const float p1 = ex2_approx(fmaf(s[64 * half + 2 * e + 1], sc, nm));
          rs[e & 3] += p0 + p1;
          pk[e] = pack_bf16x2(p0, p1);
        }
        tmem_st32(tS + 32 * half, pk);
      }
      l = l * factor + ((rs[0] + rs[1]) + (rs[2] + rs[3]));
      // Rare: rescale the O rows whose maximum jumped.  PV(j-1) has completed
      // (its commit preceded S(j)'s) and PV(j) waits for p_ready below.
      if (__any_sync(0xffffffffu, rescale) && j > 0) {
#pragma unroll 1
        for (int c0 = 0; c0 < D; c0 += 32) {
          uint32_t o[32];
          tmem_ld32(tO + c0, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * factor);
          tmem_st32(tO + c0, o);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_ready[i]);
    }

    // ---- epilogue: O / l -> bf16 -> swizzled smem (reusing Q_i) -> TMA store ----
    if (ok && n > 0) {
      ok = warp_wait(&o_final[i], 0, kSiteOFinal);
      tc_fence_after();
    }
    uint8_t* obuf = q_buf + i * C::kTileBytes;
    const uint32_t obase = smem_u32(obuf);
    const float inv = (ok && n > 0 && l > 0.0f) ? 1.0f / l : 0.0f;
#pragma unroll
    for (int c0 = 0; c0 < D; c0 += 32) {
      uint32_t o[32];
      if (ok && n > 0) {
        tmem_ld32(tO + c0, o);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) o[e] = 0u;
      }
      uint32_t w[16];
#pragma unroll
      for (int e = 0; e < 16; ++e)
        w[e] = pack_bf16x2(__uint_as_float(o[2 * e]) * inv, __uint_as_float(o[2 * e + 1]) * inv);
      const int box = c0 >> 6;
      const int chunk0 = (c0 & 63) >> 3;  // 16-byte chunk index inside the 128-byte row
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int ch = (chunk0 + t) ^ (row & 7);
        st_shared_v4(obase + box * C::kBoxBytes + row * 128 + ch * 16, w[4 * t], w[4 * t + 1],
                     w[4 * t + 2], w[4 * t + 3]);
      }
    }
    fence_proxy_async_smem();
    named_bar_sync(1 + i, 128);
    if (quad == 0 && lane == 0 && row0[i] < p.Sq) {
      for (int h = 0; h < C::kBoxes; ++h)
        tma_store_3d(&o_map, obuf + h * C::kBoxBytes, h * 64, row0[i], zq);
      bulk_commit_group();
      bulk_wait_group_read<0>();
    }
    __syncwarp();
  }

  // ---- teardown ----
  tc_fence_before();
  __syncthreads();
  if (warp == kTmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace attn
}  // namespace b200
