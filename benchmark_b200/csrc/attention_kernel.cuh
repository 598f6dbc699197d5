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
//   warp  8    TMA producer (Q once, then the K and V rings) and TMEM allocator
//   warp  9    tcgen05.mma issuer (one thread)
//
// All matrix products are M=128 x N=128 (S = Q K^T over 128 keys, O += P V over
// 128 head dims, or 64 for D=64): issued back to back, that stream runs at the
// full tensor rate on B200, while N=64 products run ~1.8x below theirs.
//
// TMEM (512 columns):
//   D=128: S0 [0,128) S1 [128,256) O0 [256,384) O1 [384,512); P_i (bf16
//          pairs, 64 columns) overwrites the first half of S_i.
//   D=64:  S0 [0,128) S1 [128,256) O0 [256,320) O1 [320,384) P0 [384,448)
//          P1 [448,512): P has its own columns.
// PV reads P straight from TMEM (A operand in TMEM, V from shared memory,
// MN-major).  P is produced in two 64-key halves with separate ready barriers,
// so the first four PV MMAs run while the softmax computes the second half.
//
// MMA issue order per KV tile j:
//   D=128: PV0(j) S0(j+1) PV1(j) S1(j+1)   (S_i(j+1) overwrites P_i(j); the
//          tensor pipe executes one thread's MMAs in issue order)
//   D=64:  S0(j+1) S1(j+1) PV0(j) PV1(j)   (S_i(j+1) is issued as soon as the
//          softmax has read S_i(j) into registers; the softmax waits for
//          PV_i(j) before writing P_i(j+1) or rescaling O_i)
// The issuer polls every dependency of a step in one instruction group
// (mbar_wait3): a barrier poll whose result is branched on costs a few hundred
// cycles, and the tensor pipe queues only ~4 MMAs.
//
// Softmax: per row, running max m in log2 units; O and the row sum are
// rescaled only when a block raises m by more than kRescaleLog2 (otherwise P
// values up to 2^kRescaleLog2 accumulate unscaled: exact in fp32, and O / l is
// unchanged).  exp2 runs on the MUFU for most elements and on the FMA pipe
// (exp2_fma_x2, ptx.cuh) for kEmu of every 8 element pairs, so the two pipes
// share the load; masked blocks use the MUFU only (exact zeros).
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
  // Clock trace (kTrace instantiations only): per-role record regions of
  // trace_cap records (2 x u64: (event << 32 | tile << 24 | iter), clock64)
  // for CTA trace_cta.  Role r (0 TMA, 1 MMA, 2/3 softmax tile 0/1) starts
  // at trace + r * trace_cap * 2.
  unsigned long long* trace;
  int trace_cap;
  int trace_cta;
};

// Clock-trace events (kTrace); names in benchmark_b200/trace.py.
enum : uint32_t {
  kEvTmaK = 1, kEvTmaV, kEvMmaS, kEvMmaPvLo, kEvMmaPvHi, kEvSmWait, kEvSmReady, kEvSmLdDone,
  kEvSmMaxDone, kEvSmPLo, kEvSmPHi, kEvEpiBegin, kEvEpiEnd, kEvMmaWait, kEvMmaEnd
};

template <bool kTrace>
struct Tracer {
  unsigned long long* base = nullptr;
  int n = 0, cap = 0;
  __device__ __forceinline__ Tracer(const Params& p, int role, bool enable) {
    if (kTrace && enable && p.trace != nullptr) {
      base = p.trace + static_cast<size_t>(role) * p.trace_cap * 2;
      cap = p.trace_cap;
    }
  }
  __device__ __forceinline__ void operator()(uint32_t ev, int tile, int iter) {
    if constexpr (kTrace) {
      if (base != nullptr && n < cap) {
        base[2 * n] = (static_cast<unsigned long long>(ev) << 32) |
                      (static_cast<unsigned long long>(tile & 0xff) << 24) |
                      static_cast<unsigned long long>(iter & 0xffffff);
        base[2 * n + 1] = clock64();
        ++n;
      }
    }
  }
};

template <int D>
struct Cfg {
  static_assert(D == 64 || D == 128, "head_dim must be 64 or 128");
  static constexpr bool kEarlyS = (D == 64);       // S(j+1) before PV(j), own P columns
  static constexpr int kBoxes = D / 64;            // 64-column (128-byte) TMA boxes per tile
  static constexpr int kBoxBytes = 128 * 128;      // 128 rows x 128 B = 16 KiB
  static constexpr int kTileBytes = kBoxes * kBoxBytes;
  static constexpr int kStages = (D == 128) ? 2 : 4;  // K ring and V ring depth
  static constexpr int kQOff = 0;
  static constexpr int kKOff = 2 * kTileBytes;
  static constexpr int kVOff = kKOff + kStages * kTileBytes;
  static constexpr int kBarOff = kVOff + kStages * kTileBytes;
  // q_full, k_full[S], k_empty[S], v_full[S], v_empty[S], s_ready[2], p_lo[2],
  // p_hi[2], o_final[2], s_free[2], pv_done[2], drain
  static constexpr int kNumBars = 1 + 4 * kStages + 2 * 6 + 1;
  static constexpr int kTmemSlotOff = kBarOff + kNumBars * 8;
  static constexpr int kSmemBytes = kTmemSlotOff + 16 + 1024;  // + 1 KiB alignment slack
  static constexpr uint32_t kIdescS = idesc_bf16_f32(128, kBN, false, false);
  static constexpr uint32_t kIdescO = idesc_bf16_f32(128, D, false, true);
  static constexpr uint32_t kColO = 256;
  static constexpr uint32_t kColP = kEarlyS ? 256 + 2 * D : 0;  // D=128: P_i over S_i
};

// Wait sites reported in the status word.
enum : uint32_t {
  kSiteQFull = 1, kSiteKFull, kSiteVFull, kSitePReady, kSiteKEmpty, kSiteVEmpty,
  kSiteSReady, kSiteOFinal, kSiteSFree, kSitePvDone
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

// Warp-uniform bounded wait for the softmax warps: the warp proceeds only if
// every lane observed the phase (warp-collective tcgen05.ld/st never run on a
// partial warp); waiting lanes sleep in the hardware wait so they do not take
// issue slots from the MMA and TMA warps that share their schedulers.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, uint32_t site) {
  const bool ok = mbar_wait(bar, parity, site, kDefaultWaitLimitNs, 20000u);
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

// One 64-key half of P for this thread's row: exp2(x) as 32 bf16 pairs,
// x = s * sc - m (s pre-scaled in masked blocks, sc = 1).  Accumulates the
// fp32 row sum in packed pairs.
template <int kEmu, bool kMasked>
__device__ __forceinline__ void p_half(const float* s, float sc, float nm, uint64_t (&rs)[2],
                                       uint32_t (&pk)[32]) {
  const uint64_t sc2 = f2_pack(sc, sc);
  const uint64_t nm2 = f2_pack(nm, nm);
#pragma unroll
  for (int e = 0; e < 32; ++e) {
    const uint64_t x2 = f2_fma(f2_pack(s[2 * e], s[2 * e + 1]), sc2, nm2);
    float x0, x1, p0, p1;
    f2_unpack(x2, x0, x1);
    if (!kMasked && (e & 7) < kEmu) {
      exp2_fma_x2(x0, x1, p0, p1);
    } else {
      p0 = ex2_approx(x0);
      p1 = ex2_approx(x1);
    }
    rs[e & 1] = f2_add(rs[e & 1], f2_pack(p0, p1));
    pk[e] = pack_bf16x2(p0, p1);
  }
}

template <int D, int kEmu, bool kTrace = false>
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
  uint64_t* p_lo = s_ready + 2;
  uint64_t* p_hi = p_lo + 2;
  uint64_t* o_final = p_hi + 2;
  uint64_t* s_free = o_final + 2;
  uint64_t* pv_done = s_free + 2;
  uint64_t* drain = pv_done + 2;
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
      mbar_init(&p_lo[i], 128);
      mbar_init(&p_hi[i], 128);
      mbar_init(&o_final[i], 1);
      mbar_init(&s_free[i], 128);
      mbar_init(&pv_done[i], 1);
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
  const bool trace_cta = kTrace && static_cast<int>(blockIdx.x) == p.trace_cta;

  if (warp == kTmaWarp) {
    // ================= TMA producer =================
    if (lane == 0 && nmax > 0) {
      Tracer<kTrace> tr(p, 0, trace_cta);
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
        tr(kEvTmaK, 0, j);
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
        tr(kEvTmaV, 0, j);
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
      Tracer<kTrace> tr(p, 1, trace_cta);
      const uint32_t q_addr = smem_u32(q_buf);
      const uint32_t k_addr = smem_u32(k_buf);
      const uint32_t v_addr = smem_u32(v_buf);
      // q_full phase 0 completes once and stays complete: fills unused wait slots.
      const uint32_t dn_a = smem_u32(q_full), dn_p = 0;
      auto bar = [](uint64_t* b_) { return smem_u32(b_); };
      auto par = [](int j) { return static_cast<uint32_t>(j) & 1u; };
      auto kpar = [](int j) { return static_cast<uint32_t>(j / C::kStages) & 1u; };

      // Descriptors are built once; a K step or ring stage only moves the
      // start address, i.e. adds (byte offset >> 4) to the low field (shared
      // addresses stay below 2^18, so the 14-bit field never carries).
      const uint64_t dq0 = sdesc_sw128(q_addr, 16, 1024);
      const uint64_t dk0 = sdesc_sw128(k_addr, 16, 1024);
      const uint64_t dv0 = sdesc_sw128(v_addr, C::kBoxBytes, 1024);
      constexpr uint32_t kTile16 = C::kTileBytes >> 4, kBox16 = C::kBoxBytes >> 4;
      const uint32_t tS[2] = {tmem_base, tmem_base + 128};
      const uint32_t tO[2] = {tmem_base + C::kColO, tmem_base + C::kColO + D};
      const uint32_t tP[2] = {C::kEarlyS ? tmem_base + C::kColP : tS[0],
                              C::kEarlyS ? tmem_base + C::kColP + 64 : tS[1]};

      auto issue_s = [&](int i, int j) {
        tr(kEvMmaS, i, j);
        const uint64_t dq = dq0 + i * kTile16;
        const uint64_t dk = dk0 + (j % C::kStages) * kTile16;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kBox16 + (kk & 3) * 2;
          mma_ss(tS[i], dq + off, dk + off, C::kIdescS, kk > 0 ? 1u : 0u);
        }
        mma_commit(&s_ready[i]);
      };
      // PV for keys [64*half, 64*half + 64) of V tile j.
      auto issue_pv_half = [&](int i, int j, int half) {
        tr(half ? kEvMmaPvHi : kEvMmaPvLo, i, j);
        const uint64_t dv = dv0 + (j % C::kStages) * kTile16;
#pragma unroll
        for (int k4 = 0; k4 < 4; ++k4) {
          const int kk = half * 4 + k4;
          mma_ts(tO[i], tP[i] + kk * 8, dv + kk * (2048 >> 4), C::kIdescO,
                 (j > 0 || kk > 0) ? 1u : 0u);
        }
        if (half) {
          if (C::kEarlyS) mma_commit(&pv_done[i]);
          if (j == nblk[i] - 1) mma_commit(&o_final[i]);
        }
      };
      auto wait3 = [&](uint32_t a0, uint32_t p0, uint32_t a1, uint32_t p1, uint32_t a2,
                       uint32_t p2, uint32_t site) -> bool {
        tr(kEvMmaWait, site, 0);
        if (!mbar_wait3(a0, p0, a1, p1, a2, p2, site)) return false;
        tc_fence_after();
        return true;
      };

      // Prologue: S(0) for both tiles.
      bool ok = wait3(bar(q_full), 0, bar(&k_full[0]), 0, dn_a, dn_p, kSiteKFull);
      if (ok) {
        for (int i = 0; i < 2; ++i)
          if (nblk[i] > 0) issue_s(i, 0);
        mma_commit(&k_empty[0]);
      }
      for (int j = 0; j < nmax && ok; ++j) {
        const int s = j % C::kStages;
        const int jn = j + 1;
        const bool more = jn < nmax;
        const uint32_t kn_a = more ? bar(&k_full[jn % C::kStages]) : dn_a;
        const uint32_t kn_p = more ? kpar(jn) : dn_p;
        if constexpr (C::kEarlyS) {
          // S(j+1) for both tiles as soon as the softmax has S(j) in registers.
          if (more) {
            ok = wait3(kn_a, kn_p, jn < nblk[0] ? bar(&s_free[0]) : dn_a,
                       jn < nblk[0] ? par(j) : dn_p, jn < nblk[1] ? bar(&s_free[1]) : dn_a,
                       jn < nblk[1] ? par(j) : dn_p, kSiteSFree);
            if (!ok) break;
            for (int i = 0; i < 2; ++i)
              if (jn < nblk[i]) issue_s(i, jn);
            mma_commit(&k_empty[jn % C::kStages]);
          }
          for (int i = 0; i < 2 && ok; ++i) {
            if (j >= nblk[i]) continue;
            ok = wait3(bar(&v_full[s]), kpar(j), bar(&p_lo[i]), par(j), dn_a, dn_p,
                       kSitePReady);
            if (!ok) break;
            issue_pv_half(i, j, 0);
            ok = wait3(bar(&p_hi[i]), par(j), dn_a, dn_p, dn_a, dn_p, kSitePReady);
            if (!ok) break;
            issue_pv_half(i, j, 1);
          }
          if (!ok) break;
          mma_commit(&v_empty[s]);
        } else {
          for (int i = 0; i < 2 && ok; ++i) {
            if (j < nblk[i]) {
              ok = wait3(bar(&v_full[s]), kpar(j), bar(&p_lo[i]), par(j), dn_a, dn_p,
                         kSitePReady);
              if (!ok) break;
              issue_pv_half(i, j, 0);
              // S_i(j+1) needs K(j+1) and overwrites P_i(j): after PV_i(j).
              ok = wait3(bar(&p_hi[i]), par(j), jn < nblk[i] ? kn_a : dn_a,
                         jn < nblk[i] ? kn_p : dn_p, dn_a, dn_p, kSitePReady);
              if (!ok) break;
              issue_pv_half(i, j, 1);
            }
            if (jn < nblk[i]) issue_s(i, jn);
          }
          if (!ok) break;
          mma_commit(&v_empty[s]);
          if (more) mma_commit(&k_empty[jn % C::kStages]);
        }
      }
      // Every MMA issued above has completed once this commit lands.
      mma_commit(drain);
      drain_wait(drain, 0);
      tr(kEvMmaEnd, 0, nmax);
    }
    __syncwarp();
  } else {
    // ================= softmax + epilogue (warps 0-7) =================
    const int i = static_cast<int>(warp >> 2);  // Q tile
    const uint32_t quad = warp & 3u;
    const int row = static_cast<int>(quad * 32 + lane);
    const uint32_t lane_addr = (quad * 32u) << 16;
    const uint32_t tS = tmem_base + lane_addr + static_cast<uint32_t>(i) * 128u;
    const uint32_t tO = tmem_base + lane_addr + C::kColO + static_cast<uint32_t>(i * D);
    const uint32_t tP =
        C::kEarlyS ? tmem_base + lane_addr + C::kColP + static_cast<uint32_t>(i) * 64u : tS;
    const int n = nblk[i];
    const int q = row0[i] + row;
    const int lim = p.causal ? min(p.Skv, q + p.causal_off + 1) : p.Skv;
    const float c = p.scale_log2;
    float m = -INFINITY;  // running max of scaled scores (log2 units)
    float l = 0.0f;       // running row sum of P
    bool ok = true;
    Tracer<kTrace> tr(p, 2 + i, trace_cta && quad == 0 && lane == 0);

#pragma unroll 1
    for (int j = 0; j < n; ++j) {
      tr(kEvSmWait, i, j);
      ok = warp_wait(&s_ready[i], static_cast<uint32_t>(j) & 1u, kSiteSReady);
      if (!ok) break;
      tc_fence_after();
      tr(kEvSmReady, i, j);
      uint32_t sr[128];
      tmem_ld32(tS + 0, *reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
      tmem_ld32(tS + 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
      tmem_ld32(tS + 64, *reinterpret_cast<uint32_t(*)[32]>(&sr[64]));
      tmem_ld32(tS + 96, *reinterpret_cast<uint32_t(*)[32]>(&sr[96]));
      tmem_wait_ld();
      tr(kEvSmLdDone, i, j);
      if constexpr (C::kEarlyS) {
        // S_i is in registers: the MMA warp may overwrite it with S_i(j+1).
        tc_fence_before();
        mbar_arrive(&s_free[i]);
      }
      float* s = reinterpret_cast<float*>(sr);

      const int kbase = j * kBN;
      const bool masked = kbase + kBN > min_lim[i];  // uniform across the tile
      float m_blk;
      if (masked) {
        // Scale first, then mask, so masked keys are exactly -inf for any scale.
        const int valid = lim - kbase;
        float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int e = 0; e < kBN; ++e) {
          const float t = e < valid ? s[e] * c : -INFINITY;
          s[e] = t;
          mx[e & 3] = fmaxf(mx[e & 3], t);
        }
        m_blk = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
      } else {
        // 3-input max: 4 independent chains over 124 values + 4 seeds.
        float mx[4] = {s[0], s[1], s[2], s[3]};
#pragma unroll
        for (int e = 4; e < 124; e += 8) {
          mx[0] = fmax3(mx[0], s[e + 0], s[e + 1]);
          mx[1] = fmax3(mx[1], s[e + 2], s[e + 3]);
          mx[2] = fmax3(mx[2], s[e + 4], s[e + 5]);
          mx[3] = fmax3(mx[3], s[e + 6], s[e + 7]);
        }
        mx[0] = fmax3(mx[0], s[124], s[125]);
        mx[1] = fmax3(mx[1], s[126], s[127]);
        m_blk = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * c;
      }
      tr(kEvSmMaxDone, i, j);

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
      if constexpr (C::kEarlyS) {
        // P_i and O_i are still in use by PV_i(j-1) until it completes.
        if (j > 0) {
          ok = warp_wait(&pv_done[i], static_cast<uint32_t>(j - 1) & 1u, kSitePvDone);
          if (!ok) break;
          tc_fence_after();
        }
      }

      const float m_use = (m == -INFINITY) ? 0.0f : m;
      const float sc = masked ? 1.0f : c;  // masked scores are pre-scaled
      uint64_t rs[2] = {0ull, 0ull};
      {
        uint32_t pk[32];
        if (masked)
          p_half<kEmu, true>(s, sc, -m_use, rs, pk);
        else
          p_half<kEmu, false>(s, sc, -m_use, rs, pk);
        tmem_st32(tP, pk);
      }
      // Rare: rescale the O rows whose maximum jumped.  PV_i(j-1) has
      // completed (D=128: its commit preceded S_i(j)'s; D=64: waited above)
      // and PV_i(j) waits for the P barriers below.
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
      mbar_arrive(&p_lo[i]);
      tr(kEvSmPLo, i, j);
      {
        uint32_t pk[32];
        if (masked)
          p_half<kEmu, true>(s + 64, sc, -m_use, rs, pk);
        else
          p_half<kEmu, false>(s + 64, sc, -m_use, rs, pk);
        tmem_st32(tP + 32, pk);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_hi[i]);
      tr(kEvSmPHi, i, j);
      float r0, r1, r2, r3;
      f2_unpack(rs[0], r0, r1);
      f2_unpack(rs[1], r2, r3);
      l = l * factor + ((r0 + r1) + (r2 + r3));
    }

    // ---- epilogue: O / l -> bf16 -> swizzled smem (reusing Q_i) -> TMA store ----
    tr(kEvEpiBegin, i, n);
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
    tr(kEvEpiEnd, i, n);
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
