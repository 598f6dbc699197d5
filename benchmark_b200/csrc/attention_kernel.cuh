// Fused attention forward for sm_100a: O = softmax(Q K^T * scale) V.
//
// Replaces the reference's qk_tma_mma_ld_kernel (0.attention/attention.cu:1503-1974)
// and generalises it to the scalar path's semantics
// (real_attention_bf16_d128_kernel, attention.cu:210-274): any B, Hq, Hkv (GQA,
// attention.cu:176-183), Sq != Skv with bottom-right causal masking
// (attention.cu:167-174), ragged tails, head_dim 64 or 128.
//
// Persistent CTAs (one per SM) walk work items = (batch, q head, 128-row Q
// tile).  Each item streams its head's K/V tiles (128 keys each).  The CTA's
// K/V tiles form one global sequence t (crossing item boundaries); tile t
// belongs to softmax pipe t & 1.  Each pipe keeps its own online-softmax state
// (row max m, row sum l) and its own O accumulator for the item, and the
// epilogue merges the two: O = (O0 2^(m0-m) + O1 2^(m1-m)) / (l0 2^(m0-m) +
// l1 2^(m1-m)), m = max(m0, m1) -- the reference's two-pipe split
// (attention.cu:1715-1947 merges its pipes the same way), here over a
// persistent tile stream.  The two pipes' softmax warps share each scheduler
// and run half a period apart, so one pipe's control latency (score load,
// P publish, barrier waits) overlaps the other pipe's exp2 loop.  Roles:
//
//   warps 0-3   softmax pipe 0, warps 4-7 softmax pipe 1: warp w owns TMEM
//               lanes 32*(w%4) .. +32, one query row per thread, all 128
//               keys of a tile in registers (no cross-thread reduction)
//   warps 8-11  epilogue: merge O0/O1 -> bf16 -> shared -> TMA store
//   warp  12    TMA producer for Q (per item) and the K ring; TMEM allocator
//   warp  13    tcgen05.mma issuer (whole warp, one elected lane issues)
//   warp  14    TMA producer for the V ring
//   warp  15    idle; it completes warpgroup 3, so that each warpgroup can
//               move its register budget with setmaxnreg (softmax 184,
//               epilogue 56, producers/issuer 88 registers per thread)
//
// TMEM (512 columns): S0 [0,128), S1 [128,256), O0 [256, 256+D), O1
// [256+D, 256+2D).  P(t) (bf16 pairs, key pair (2c, 2c+1) in column c)
// overwrites the first 64 columns of its pipe's S buffer and is consumed by a
// TS-MMA (A from TMEM).
//
// MMA issue order over the tile stream: S(0), S(1), then for every t:
// PV(t), S(t+2).  S(t+2) overwrites P(t) of the same pipe after PV(t) in
// issue order (the tensor pipe executes one thread's MMAs in order), and the
// commit that publishes S(t) also covers PV(t-2), so a softmax warp that
// sees S(t) may rescale its pipe's O rows without another wait.
//
// Softmax per tile (one row per thread): the row max is thread-local (64
// three-input max instructions, no shuffles), taken before the exp2 loop.  O
// and the row sums are rescaled only when a tile raises the running max m by
// more than kRescaleLog2 (otherwise P values up to 2^kRescaleLog2 accumulate
// unscaled: exact in fp32, O / l unchanged).  Masked tiles (causal edge,
// ragged tail) put the masked keys at -inf and use MUFU exp2 only (exact
// zeros).
//
// Every wait is bounded (ptx.cuh).  A timeout sets the device status word;
// the epilogue warps, which meet at a named barrier, agree on aborting
// through a shared flag written before the barrier, so no barrier is ever
// left one-sided.
#pragma once

#include "ptx.cuh"

namespace b200 {
namespace attn {

constexpr int kBM = 128;  // query rows per work item (= TMEM lanes)
constexpr int kBN = 128;  // keys per K/V tile
constexpr int kPipes = 2;
constexpr int kEpiWarp0 = 8;
constexpr int kTmaWarp = 12;   // Q and K loads
constexpr int kMmaWarp = 13;
constexpr int kTmaVWarp = 14;  // V loads
constexpr int kThreads = 512;  // warp 15 only completes warpgroup 3
// Registers per thread after the split: softmax warpgroups 0-1 grow, the
// epilogue warpgroup 2 and the producer/issuer warpgroup 3 shrink; the sum is
// the pool the block launches with (512 threads x 128).
constexpr int kLaunchRegs = 65536 / kThreads;
constexpr int kSoftmaxRegs = 184;
constexpr int kEpiRegs = 56;
constexpr int kCtlRegs = 88;
static_assert(8 * 32 * kSoftmaxRegs + 4 * 32 * kEpiRegs + 4 * 32 * kCtlRegs ==
                  kThreads * kLaunchRegs,
              "register split must use exactly the launch pool");
static_assert(kSoftmaxRegs % 8 == 0 && kEpiRegs % 8 == 0 && kCtlRegs % 8 == 0 &&
                  kEpiRegs >= 24 && kCtlRegs >= 24 && kSoftmaxRegs <= 256,
              "setmaxnreg counts");
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleLog2 = 8.0f;
constexpr float kRescaleP = 256.0f;  // 2^kRescaleLog2
constexpr int kBarEpilogue = 1;  // named barrier: warps 8-11

struct Params {
  int B, Hq, Hkv, Sq, Skv;
  int group;     // Hq / Hkv
  int n_qtiles;  // ceil(Sq / 128)
  int n_items;   // B * Hq * n_qtiles
  int causal;      // bottom-right aligned
  int causal_off;  // Skv - Sq
  float scale_log2;  // softmax_scale * log2(e)
  // Clock trace (kTrace instantiations only): per-role record regions of
  // trace_cap records (2 x u64: (event << 32 | tile << 24 | iter), clock64)
  // for CTA trace_cta.  Role r (0 Q/K TMA, 1 MMA, 2/3 softmax pipes 0/1, 4
  // epilogue, 5 V TMA) starts at trace + r * trace_cap * 2.
  unsigned long long* trace;
  int trace_cap;
  int trace_cta;
};

// Clock-trace events (kTrace); names in benchmark_b200/trace.py.
enum : uint32_t {
  kEvTmaK = 1, kEvTmaV, kEvTmaQ, kEvMmaS, kEvMmaPv, kEvMmaWait, kEvMmaGo, kEvMmaEnd, kEvSmWait,
  kEvSmReady, kEvSmLdDone, kEvSmMaxDone, kEvSmPComputed, kEvSmPublished, kEvSmItemEnd,
  kEvEpiBegin, kEvEpiEnd
};
constexpr int kTraceRoles = 6;  // 0 K/Q TMA, 1 MMA, 2/3 softmax pipes 0/1, 4 epilogue, 5 V TMA

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
  static constexpr int kBoxes = D / 64;            // 64-column (128-byte) TMA boxes per tile
  static constexpr int kBoxBytes = 128 * 128;      // 128 rows x 128 B = 16 KiB
  static constexpr int kTileBytes = kBoxes * kBoxBytes;
  static constexpr int kKStages = (D == 128) ? 3 : 4;  // K ring depth
  static constexpr int kVStages = (D == 128) ? 2 : 4;  // V ring depth
  // Small objects first, at the (16-byte aligned) start of dynamic shared
  // memory; the tile region follows at the next 1024-byte boundary (128-byte
  // swizzled TMA boxes need it).  Per-row (m, l) of each pipe for the item
  // the epilogue works on: [pipe][row] float2 (one slot suffices: the softmax
  // writes item li's values only after the epilogue has released item li-1).
  static constexpr int kStatOff = 0;
  static constexpr int kFlagOff = kStatOff + kPipes * 128 * 8;  // abort flag (epilogue)
  static constexpr int kBarOff = kFlagOff + 16;
  // q_full[2] q_empty[2] k_full[K] k_empty[K] v_full[V] v_empty[V]
  // s_ready[2] p_ready[2] o_full o_empty l_ready[2] drain done
  static constexpr int kNumBars = 4 + 2 * kKStages + 2 * kVStages + 2 * kPipes + 2 + 2 + 2;
  static constexpr int kTmemSlotOff = kBarOff + kNumBars * 8;
  static constexpr int kSmallBytes = (kTmemSlotOff + 16 + 15) / 16 * 16;
  // Tile region, relative to its 1024-byte aligned start.
  static constexpr int kQOff = 0;  // Q0, Q1 (also O staging)
  static constexpr int kKOff = 2 * kTileBytes;
  static constexpr int kVOff = kKOff + kKStages * kTileBytes;
  static constexpr int kTileRegion = kVOff + kVStages * kTileBytes;
  // With the d=128 rings the whole budget is needed: the request is the
  // 227 KiB a CTA may use, which holds the layout whenever dynamic shared
  // memory starts at most 1024 - (kSmallBytes % 1024) bytes past a 1024-byte
  // boundary (it starts on one); the kernel checks and reports otherwise.
  static constexpr int kSmemMax = 232448;
  static constexpr int kSmemBytes = kSmallBytes + 1024 + kTileRegion <= kSmemMax
                                        ? kSmallBytes + 1024 + kTileRegion
                                        : kSmemMax;
  static_assert(kSmallBytes + kTileRegion + (1024 - kSmallBytes % 1024) % 1024 <= kSmemMax,
                "exceeds the 227 KiB of shared memory a CTA may use");
  static constexpr uint32_t kIdescS = idesc_bf16_f32(128, kBN, false, false);
  static constexpr uint32_t kIdescO = idesc_bf16_f32(128, D, false, true);
  static constexpr uint32_t kColO = 128 * kPipes;  // O0 at kColO, O1 at kColO + D
  static_assert(kColO + kPipes * D <= kTmemCols, "TMEM budget");
};

// Wait sites reported in the status word.
enum : uint32_t {
  kSiteQFull = 1, kSiteKFull, kSiteVFull, kSitePReady, kSiteKEmpty, kSiteVEmpty,
  kSiteSReady, kSiteOFull, kSiteQEmpty, kSitePvDone, kSiteOEmpty, kSiteLReady,
  kSiteSmemLayout = 0xF0  // the tile region did not fit behind the small objects
};

// Number of K/V tiles the Q tile at `tile_row0` must visit (0 if it has no
// valid keys) and the smallest per-row key limit inside the tile.
__device__ __forceinline__ void tile_extent(const Params& p, int tile_row0, int* nblk,
                                            int* min_lim) {
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

struct Item {
  int zq;    // (b * Hq + hq): plane of Q / O
  int zkv;   // (b * Hkv + hkv): plane of K / V
  int row0;  // first query row
  int n;     // K/V tiles to visit
  int min_lim;
};

// Work item k.  Non-causal: items of one head are adjacent, so the CTAs
// running at one time share a few heads' K/V in L2.  Causal: the heaviest Q
// tiles (last rows) come first.
__device__ __forceinline__ Item decode_item(const Params& p, int k) {
  const int bhs = p.B * p.Hq;
  int bh, qt;
  if (p.causal) {
    qt = p.n_qtiles - 1 - k / bhs;
    bh = k - (k / bhs) * bhs;
  } else {
    bh = k / p.n_qtiles;
    qt = k - bh * p.n_qtiles;
  }
  const int b = bh / p.Hq;
  const int hq = bh - b * p.Hq;
  Item it;
  it.zq = bh;
  it.zkv = b * p.Hkv + hq / p.group;
  it.row0 = qt * kBM;
  tile_extent(p, it.row0, &it.n, &it.min_lim);
  return it;
}

// The r-th item of this CTA: rounds of gridDim.x items; causal rounds
// alternate direction so every CTA gets a similar total of K/V tiles.
__device__ __forceinline__ int item_index(const Params& p, int r) {
  const int g = static_cast<int>(gridDim.x);
  const int c = static_cast<int>(blockIdx.x);
  return r * g + ((p.causal && (r & 1)) ? g - 1 - c : c);
}

// Warp-uniform bounded wait: true only if every lane observed the phase
// (warp-collective tcgen05.ld/st never run on a partial warp).  Waiting lanes
// sleep in the hardware wait so they do not take issue slots from others.
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

// P for keys [16c, 16c+16) of this thread's row (s: those 16 scores):
// exp2(s * sc + nm) as 8 bf16 pairs (pk[i] = keys 2i, 2i+1), accumulating
// the fp32 row sum in two packed pairs.  kEmu of every 8 pairs use the
// FMA-pipe exp2 (exp2_fma_x2).  Masked tiles: keys at or past `va` (counted
// from this chunk's first key) get exactly 0 (MUFU of -inf).
template <int kEmu, bool kMasked>
__device__ __forceinline__ void p_chunk(const float* s, uint64_t sc2, uint64_t nm2, int va,
                                        uint64_t& ra, uint64_t& rb, uint32_t (&pk)[8]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint64_t x2 = f2_fma(f2_pack(s[2 * i], s[2 * i + 1]), sc2, nm2);
    float x0, x1, p0, p1;
    f2_unpack(x2, x0, x1);
    if (kMasked) {
      x0 = 2 * i < va ? x0 : -INFINITY;
      x1 = 2 * i + 1 < va ? x1 : -INFINITY;
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
}

// P of a whole 128-key tile row, stored over the first 64 columns of the
// pipe's S buffer (tS: this thread's lane, column 0).
template <int kEmu, bool kMasked>
__device__ __forceinline__ void p_tile(const float* s, float sc, float nm, int va, uint32_t tS,
                                       uint64_t& ra, uint64_t& rb) {
  const uint64_t sc2 = f2_pack(sc, sc);
  const uint64_t nm2 = f2_pack(nm, nm);
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    uint32_t pk[8];
    p_chunk<kEmu, kMasked>(s + 16 * c, sc2, nm2, va - 16 * c, ra, rb, pk);
    tmem_st8(tS + 8 * c, pk);
  }
}

// Largest of a row's 128 scores (four independent chains).
__device__ __forceinline__ float row_max128(const float* s) {
  float a[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) a[u] = fmaxf(s[2 * u], s[2 * u + 1]);
#pragma unroll
  for (int g = 4; g < 64; ++g) a[g & 3] = fmax3(a[g & 3], s[2 * g], s[2 * g + 1]);
  return fmaxf(fmaxf(a[0], a[1]), fmaxf(a[2], a[3]));
}

template <int D, int kEmu, bool kTrace = false>
__global__ void __launch_bounds__(kThreads, 1)
    attention_fwd_kernel(const __grid_constant__ CUtensorMap q_map,
                         const __grid_constant__ CUtensorMap k_map,
                         const __grid_constant__ CUtensorMap v_map,
                         const __grid_constant__ CUtensorMap o_map, const Params p) {
  using C = Cfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* tiles = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw + C::kSmallBytes) + 1023) &
      ~static_cast<uintptr_t>(1023));
  if (tiles + C::kTileRegion > smem_raw + C::kSmemBytes) {
    // Uniform across the CTA, before any barrier or TMEM use.
    if (threadIdx.x == 0) report_timeout(kSiteSmemLayout);
    return;
  }
  uint8_t* q_buf = tiles + C::kQOff;
  uint8_t* k_buf = tiles + C::kKOff;
  uint8_t* v_buf = tiles + C::kVOff;
  float2* stat = reinterpret_cast<float2*>(smem_raw + C::kStatOff);  // [pipe][row] = (m, l)
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem_raw + C::kFlagOff);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_raw + C::kBarOff);
  uint64_t* q_full = bars;
  uint64_t* q_empty = q_full + 2;
  uint64_t* k_full = q_empty + 2;
  uint64_t* k_empty = k_full + C::kKStages;
  uint64_t* v_full = k_empty + C::kKStages;
  uint64_t* v_empty = v_full + C::kVStages;
  uint64_t* s_ready = v_empty + C::kVStages;
  uint64_t* p_ready = s_ready + kPipes;
  uint64_t* o_full = p_ready + kPipes;
  uint64_t* o_empty = o_full + 1;
  uint64_t* l_ready = o_empty + 1;
  uint64_t* drain = l_ready + 2;
  uint64_t* done = drain + 1;  // phase 0 completes at setup and never changes
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem_raw + C::kTmemSlotOff);

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();
  const int rounds = (p.n_items + static_cast<int>(gridDim.x) - 1) / static_cast<int>(gridDim.x);

  // ---- setup ----
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&l_ready[i], 8);  // all eight softmax warps
    }
    for (int i = 0; i < kPipes; ++i) {
      mbar_init(&s_ready[i], 1);
      mbar_init(&p_ready[i], 4);  // the pipe's four softmax warps
    }
    mbar_init(o_full, 1);
    mbar_init(o_empty, 128);
    for (int s = 0; s < C::kKStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < C::kVStages; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    mbar_init(drain, 1);
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
  const bool trace_cta = kTrace && static_cast<int>(blockIdx.x) == p.trace_cta;
  // Each warpgroup moves its register budget first, inside its own branch,
  // so the compiler sizes each role's code to that role's budget.
  if (warp >= static_cast<uint32_t>(kTmaWarp)) {
    // Warpgroup 3: producers and MMA issuer (warp 15 only completes the group).
    setmaxnreg_dec<kCtlRegs>();
    if (warp == kTmaWarp || warp == kTmaVWarp) {
      // ================= TMA producers (Q + K, and V) =================
      if (lane == 0) {
        const bool is_k = warp == kTmaWarp;
        Tracer<kTrace> tr(p, is_k ? 0 : 5, trace_cta);
        const uint64_t pol_q = l2_policy_evict_first();
        const uint64_t pol_kv = l2_policy_evict_last();
        int t = 0, li = 0, issued = 0, q_issued = -1;
        bool ok = true;
        for (int r = 0; r < rounds && ok; ++r) {
          const int k = item_index(p, r);
          if (k >= p.n_items) continue;
          const Item it = decode_item(p, k);
          const int qb = li & 1;
          const uint32_t qpar = static_cast<uint32_t>(li >> 1) & 1u;
          ++li;
          if (is_k) {
            // Q(li) reuses the buffer the epilogue of item li-2 staged O in.
            ok = mbar_wait(&q_empty[qb], qpar ^ 1u, kSiteQEmpty, kDefaultWaitLimitNs, 20000u);
            if (!ok) break;
            mbar_arrive_expect_tx(&q_full[qb], C::kTileBytes);
            for (int h = 0; h < C::kBoxes; ++h)
              tma_load_3d(q_buf + qb * C::kTileBytes + h * C::kBoxBytes, &q_map, &q_full[qb],
                          h * 64, it.row0, it.zq, pol_q);
            q_issued = li - 1;
            tr(kEvTmaQ, qb, li - 1);
          }
          for (int j = 0; j < it.n; ++j, ++t) {
            if (is_k) {
              const int ks = t % C::kKStages;
              ok = mbar_wait(&k_empty[ks], (static_cast<uint32_t>(t / C::kKStages) & 1u) ^ 1u,
                             kSiteKEmpty, kDefaultWaitLimitNs, 20000u);
              if (!ok) break;
              tr(kEvTmaK, 0, t);
              mbar_arrive_expect_tx(&k_full[ks], C::kTileBytes);
              for (int h = 0; h < C::kBoxes; ++h)
                tma_load_3d(k_buf + ks * C::kTileBytes + h * C::kBoxBytes, &k_map, &k_full[ks],
                            h * 64, j * kBN, it.zkv, pol_kv);
            } else {
              const int vs = t % C::kVStages;
              ok = mbar_wait(&v_empty[vs], (static_cast<uint32_t>(t / C::kVStages) & 1u) ^ 1u,
                             kSiteVEmpty, kDefaultWaitLimitNs, 20000u);
              if (!ok) break;
              tr(kEvTmaV, 0, t);
              mbar_arrive_expect_tx(&v_full[vs], C::kTileBytes);
              for (int h = 0; h < C::kBoxes; ++h)
                tma_load_3d(v_buf + vs * C::kTileBytes + h * C::kBoxBytes, &v_map, &v_full[vs],
                            h * 64, j * kBN, it.zkv, pol_kv);
            }
            issued = t + 1;
          }
        }
        if (!ok) {
          // Unwinding: let every copy already issued land before the CTA exits.
          if (is_k) {
            if (q_issued >= 0)
              drain_wait(&q_full[q_issued & 1], static_cast<uint32_t>(q_issued >> 1) & 1u);
            for (int i = max(0, issued - C::kKStages); i < issued; ++i)
              drain_wait(&k_full[i % C::kKStages], static_cast<uint32_t>(i / C::kKStages) & 1u);
          } else {
            for (int i = max(0, issued - C::kVStages); i < issued; ++i)
              drain_wait(&v_full[i % C::kVStages], static_cast<uint32_t>(i / C::kVStages) & 1u);
          }
        }
      }
      __syncwarp();
    } else if (warp == kMmaWarp) {
      // ================= MMA issuer =================
      // The whole warp runs this loop (operands stay warp-uniform); one elected
      // lane issues each MMA and commit.
      {
        Tracer<kTrace> tr(p, 1, trace_cta && lane == 0);
        const uint32_t q_addr = smem_u32(q_buf);
        const uint32_t k_addr = smem_u32(k_buf);
        const uint32_t v_addr = smem_u32(v_buf);
        // Descriptors are built once; a K step, ring stage or Q buffer only
        // moves the start address, i.e. adds (byte offset >> 4) to the low
        // field (shared addresses stay below 2^18: the 14-bit field never carries).
        const uint64_t dq0 = sdesc_sw128(q_addr, 16, 1024);
        const uint64_t dk0 = sdesc_sw128(k_addr, 16, 1024);
        const uint64_t dv0 = sdesc_sw128(v_addr, C::kBoxBytes, 1024);
        constexpr uint32_t kTile16 = C::kTileBytes >> 4, kBox16 = C::kBoxBytes >> 4;
        // Filler for unused slots of the grouped waits.
        const uint32_t dn_a = smem_u32(done), dn_p = 0;
        auto bar = [](uint64_t* b_) { return smem_u32(b_); };
        auto kpar = [](int t_) { return static_cast<uint32_t>(t_ / C::kKStages) & 1u; };
        auto vpar = [](int t_) { return static_cast<uint32_t>(t_ / C::kVStages) & 1u; };
        auto wait3 = [&](uint32_t a0, uint32_t p0, uint32_t a1, uint32_t p1, uint32_t a2,
                         uint32_t p2, uint32_t site) -> bool {
          tr(kEvMmaWait, site, 0);
          if (!__all_sync(0xffffffffu, mbar_wait3(a0, p0, a1, p1, a2, p2, site))) return false;
          tc_fence_after();
          tr(kEvMmaGo, site, 0);
          return true;
        };
        // S(t) = Q[qb] K(t)^T into pipe (t & 1)'s S buffer.
        auto issue_s = [&](int t_, int qb) {
          tr(kEvMmaS, qb, t_);
          const uint64_t dq = dq0 + qb * kTile16;
          const uint64_t dk = dk0 + (t_ % C::kKStages) * kTile16;
          const uint32_t ts = tmem_base + static_cast<uint32_t>((t_ & 1) * 128);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * kBox16 + (kk & 3) * 2;
            mma_ss_warp(ts, dq + off, dk + off, C::kIdescS, kk > 0 ? 1u : 0u);
          }
          mma_commit_warp(&k_empty[t_ % C::kKStages]);
          mma_commit_warp(&s_ready[t_ & 1]);
        };
        // O[pipe] (+)= P(t) V(t); `first`: the pipe's first tile of the item
        // overwrites O.
        auto issue_pv = [&](int t_, bool first) {
          tr(kEvMmaPv, t_ & 1, t_);
          const uint64_t dv = dv0 + (t_ % C::kVStages) * kTile16;
          const uint32_t tp = tmem_base + static_cast<uint32_t>((t_ & 1) * 128);
          const uint32_t to = tmem_base + C::kColO + static_cast<uint32_t>((t_ & 1) * D);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_ts_warp(to, tp + kk * 8, dv + kk * (2048 >> 4), C::kIdescO,
                        (!first || kk > 0) ? 1u : 0u);
        };
        // Next valid round after r (rounds if none).
        auto next_round = [&](int r) {
          for (++r; r < rounds; ++r)
            if (item_index(p, r) < p.n_items) break;
          return r;
        };

        // S cursor: the next S to issue, at most two tiles ahead of the PV
        // cursor (S(t+2) reuses PV(t)'s P buffer).
        int s_r = next_round(-1), s_li = 0, s_j = 0, s_t = 0;
        Item s_it{};
        auto s_settle = [&]() {  // move past items without K/V tiles
          while (s_r < rounds) {
            s_it = decode_item(p, item_index(p, s_r));
            if (s_it.n > 0) break;
            s_r = next_round(s_r);
            ++s_li;
          }
        };
        s_settle();
        auto issue_s_upto = [&](int limit_t) -> bool {
          while (s_r < rounds && s_t <= limit_t) {
            const int qb = s_li & 1;
            if (s_j == 0 &&
                !wait3(bar(&q_full[qb]), static_cast<uint32_t>(s_li >> 1) & 1u, dn_a, dn_p, dn_a,
                       dn_p, kSiteQFull))
              return false;
            if (!wait3(bar(&k_full[s_t % C::kKStages]), kpar(s_t), dn_a, dn_p, dn_a, dn_p,
                       kSiteKFull))
              return false;
            issue_s(s_t, qb);
            ++s_t;
            if (++s_j == s_it.n) {
              s_j = 0;
              s_r = next_round(s_r);
              ++s_li;
              s_settle();
            }
          }
          return true;
        };

        // PV cursor.
        int t = 0, li = 0;
        bool ok = issue_s_upto(1);
        for (int r = next_round(-1); r < rounds && ok; r = next_round(r), ++li) {
          const Item it = decode_item(p, item_index(p, r));
          const uint32_t oe_par = (static_cast<uint32_t>(li) & 1u) ^ 1u;  // epilogue of li-1
          if (it.n == 0) {
            // No K/V tiles: O stays unwritten (the epilogue stores zeros in Q's
            // buffer, so Q(li) must have landed first).
            ok = wait3(bar(&q_full[li & 1]), static_cast<uint32_t>(li >> 1) & 1u, bar(o_empty),
                       oe_par, dn_a, dn_p, kSiteQFull);
            if (!ok) break;
            mma_commit_warp(o_full);
            continue;
          }
          for (int j = 0; j < it.n && ok; ++j) {
            const int tt = t + j;
            // Both O accumulators are free once the epilogue of item li-1 has
            // read them (the other pipe's first PV comes after this one).
            ok = wait3(bar(&v_full[tt % C::kVStages]), vpar(tt), bar(&p_ready[tt & 1]),
                       static_cast<uint32_t>(tt >> 1) & 1u, j == 0 ? bar(o_empty) : dn_a,
                       j == 0 ? oe_par : dn_p, kSitePReady);
            if (!ok) break;
            issue_pv(tt, j < 2);
            mma_commit_warp(&v_empty[tt % C::kVStages]);
            if (j == it.n - 1) mma_commit_warp(o_full);
            ok = issue_s_upto(tt + 2);
          }
          if (!ok) break;
          t += it.n;
        }
        // Every MMA issued above has completed once this commit lands.
        mma_commit_warp(drain);
        drain_wait(drain, 0);
        tr(kEvMmaEnd, 0, t);
      }
      __syncwarp();
    }
  } else if (warp < static_cast<uint32_t>(kEpiWarp0)) {
    setmaxnreg_inc<kSoftmaxRegs>();
    // ================= softmax (warps 0-7) =================
    // Pipe `pipe` handles the tiles t with (t & 1) == pipe.  Thread `lane`
    // of warp w owns query row 32*(w%4) + lane of the item.
    const int pipe = static_cast<int>(warp >> 2);
    const uint32_t quad = warp & 3u;
    const int row = static_cast<int>(quad * 32 + lane);
    const uint32_t lane_addr = (quad * 32u) << 16;
    const uint32_t tS = tmem_base + lane_addr + static_cast<uint32_t>(pipe * 128);
    const uint32_t tO = tmem_base + lane_addr + C::kColO + static_cast<uint32_t>(pipe * D);
    const float c = p.scale_log2;
    Tracer<kTrace> tr(p, 2 + pipe, trace_cta && quad == 0 && lane == 0);
    int t = 0, li = 0;
    bool ok = true;
    // Multiply this pipe's O rows by f (rare; f = 1 for rows that did not
    // move).  PV(t-2) of this pipe has completed: the commit that published
    // S(t) covers it.
    auto rescale_o = [&](float f) {
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
    };
#pragma unroll 1
    for (int r = 0; r < rounds && ok; ++r) {
      const int k = item_index(p, r);
      if (k >= p.n_items) continue;
      const Item it = decode_item(p, k);
      const int qb = li & 1;
      const int lim = p.causal ? min(p.Skv, it.row0 + row + p.causal_off + 1) : p.Skv;
      // Running max of scaled scores (log2 units) and the row sum (two
      // packed pairs) of this pipe for the item.
      float m = -INFINITY;
      float l = 0.0f;
#pragma unroll 1
      for (int j = ((t & 1) == pipe) ? 0 : 1; j < it.n; j += 2) {
        const int tt = t + j;
        tr(kEvSmWait, pipe, tt);
        ok = warp_wait(&s_ready[pipe], static_cast<uint32_t>(tt >> 1) & 1u, kSiteSReady);
        if (!ok) break;
        tr(kEvSmReady, pipe, tt);
        tc_fence_after();
        uint32_t sr[128];
        tmem_ld_32x32b_x64(tS, *reinterpret_cast<uint32_t(*)[64]>(&sr[0]));
        tmem_ld_32x32b_x64(tS + 64, *reinterpret_cast<uint32_t(*)[64]>(&sr[64]));
        tmem_wait_ld(*reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
        reg_written_here(*reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
        reg_written_here(*reinterpret_cast<uint32_t(*)[32]>(&sr[64]));
        reg_written_here(*reinterpret_cast<uint32_t(*)[32]>(&sr[96]));
        tr(kEvSmLdDone, pipe, tt);
        float* s = reinterpret_cast<float*>(sr);
        const int kbase = j * kBN;
        const bool masked = kbase + kBN > it.min_lim;  // uniform across the CTA
        const bool first = j < 2;  // this pipe's first tile of the item: its PV overwrites O
        // Exact row max (thread-local: the thread holds its whole row), then
        // the running-max update with lazy rescaling.
        // Valid keys of this row in the tile (masked tiles only).
        const int va = lim - kbase;
        float mx;
        if (masked) {
          float a4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
          for (int i = 0; i < 128; ++i) a4[i & 3] = i < va ? fmaxf(a4[i & 3], s[i]) : a4[i & 3];
          const float smax = fmaxf(fmaxf(a4[0], a4[1]), fmaxf(a4[2], a4[3]));
          mx = smax == -INFINITY ? -INFINITY : smax * c;  // no valid key: stays -inf
        } else {
          mx = row_max128(s) * c;  // c >= 0: the max of s*c is c times the max
        }
        tr(kEvSmMaxDone, pipe, tt);
        float f = 1.0f;
        bool rescale = false;
        if (m == -INFINITY) {
          m = mx;  // no probability mass accumulated yet for this row
        } else if (mx > m + kRescaleLog2) {
          f = ex2_approx(m - mx);
          m = mx;
          rescale = true;
        }
        const float nm = (m == -INFINITY) ? 0.0f : -m;
        uint64_t ra = 0ull, rb = 0ull;
        if (masked)
          p_tile<kEmu, true>(s, c, nm, va, tS, ra, rb);
        else
          p_tile<kEmu, false>(s, c, nm, 128, tS, ra, rb);
        // O rows of this pipe follow a raised max (the pipe's first tile of
        // the item needs none: its PV overwrites O).
        if (!first && __any_sync(0xffffffffu, rescale)) rescale_o(f);
        tr(kEvSmPComputed, pipe, tt);
        // Publish P(tt) (and any O rescale) to the MMA issuer.
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        mbar_arrive_warp(&p_ready[pipe]);
        tr(kEvSmPublished, pipe, tt);
        {
          float e0, e1;
          f2_unpack(f2_add(ra, rb), e0, e1);
          l = fmaf(l, f, e0 + e1);
        }
      }
      if (!ok) break;
      // This pipe's (m, l) for the item, handed to the epilogue once it has
      // finished the previous item (li - 1) and read its values.
      ok = warp_wait(o_empty, (static_cast<uint32_t>(li) & 1u) ^ 1u, kSiteOEmpty);
      if (!ok) break;
      stat[pipe * 128 + row] = make_float2(m, l);
      __syncwarp();
      mbar_arrive_warp(&l_ready[qb]);
      tr(kEvSmItemEnd, pipe, li);
      t += it.n;
      ++li;
    }
  } else {
    setmaxnreg_dec<kEpiRegs>();
    // ================= epilogue (warps 8-11) =================
    const uint32_t quad = warp & 3u;
    const int row = static_cast<int>(quad * 32 + lane);
    const uint32_t lane_addr = (quad * 32u) << 16;
    const uint32_t tO0 = tmem_base + lane_addr + C::kColO;
    const uint32_t tO1 = tO0 + D;
    Tracer<kTrace> tr(p, 4, trace_cta && quad == 0 && lane == 0);
    int li = 0;
#pragma unroll 1
    for (int r = 0; r < rounds; ++r) {
      const int k = item_index(p, r);
      if (k >= p.n_items) continue;
      const Item it = decode_item(p, k);
      const int qb = li & 1;
      const uint32_t qpar = static_cast<uint32_t>(li >> 1) & 1u;
      ++li;
      tr(kEvEpiBegin, qb, li - 1);
      const bool got =
          warp_wait(o_full, static_cast<uint32_t>(li - 1) & 1u, kSiteOFull) &&
          warp_wait(&l_ready[qb], qpar, kSiteLReady);
      if (!got) abort_flag[0] = 1;
      tc_fence_after();
      const bool have_o = got && it.n > 0;  // warp-uniform
      // Merge weights: f_p = 2^(m_p - m) / l for pipes with mass, else 0 (a
      // pipe without mass for this row may hold a stale accumulator).
      float f0 = 0.0f, f1 = 0.0f;
      if (have_o) {
        const float2 s0 = stat[row];
        const float2 s1 = stat[128 + row];
        const float mm = fmaxf(s0.x, s1.x);
        const float w0 = s0.y > 0.0f ? ex2_approx(s0.x - mm) : 0.0f;
        const float w1 = s1.y > 0.0f ? ex2_approx(s1.x - mm) : 0.0f;
        const float l = s0.y * w0 + s1.y * w1;
        const float inv = l > 0.0f ? 1.0f / l : 0.0f;
        f0 = w0 * inv;
        f1 = w1 * inv;
      }
      uint8_t* obuf = q_buf + qb * C::kTileBytes;
      const uint32_t obase = smem_u32(obuf);
#pragma unroll 1
      for (int c0 = 0; c0 < D; c0 += 16) {
        uint32_t o[32];  // [0,16) pipe 0, [16,32) pipe 1
        if (have_o) {
          tmem_ld16(tO0 + c0, *reinterpret_cast<uint32_t(*)[16]>(&o[0]));
          tmem_ld16(tO1 + c0, *reinterpret_cast<uint32_t(*)[16]>(&o[16]));
          tmem_wait_ld(o);
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = 0u;
        }
        uint32_t w[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          float v[2];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const float a = __uint_as_float(o[2 * e + h]);
            const float b = __uint_as_float(o[16 + 2 * e + h]);
            v[h] = (f0 != 0.0f ? a * f0 : 0.0f) + (f1 != 0.0f ? b * f1 : 0.0f);
          }
          w[e] = pack_bf16x2(v[0], v[1]);
        }
        const int box = c0 >> 6;
        const int chunk0 = (c0 & 63) >> 3;  // 16-byte chunk index inside the 128-byte row
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int ch = (chunk0 + u) ^ (row & 7);
          st_shared_v4(obase + box * C::kBoxBytes + row * 128 + ch * 16, w[4 * u], w[4 * u + 1],
                       w[4 * u + 2], w[4 * u + 3]);
        }
      }
      tc_fence_before();
      mbar_arrive(o_empty);
      fence_proxy_async_smem();
      named_bar_sync(kBarEpilogue, 128);
      if (abort_flag[0] != 0) break;
      if (quad == 0 && lane == 0) {
        for (int b = 0; b < C::kBoxes; ++b)
          tma_store_3d(&o_map, obuf + b * C::kBoxBytes, b * 64, it.row0, it.zq);
        bulk_commit_group();
        bulk_wait_group_read<0>();
        mbar_arrive(&q_empty[qb]);
      }
      tr(kEvEpiEnd, qb, li - 1);
      __syncwarp();
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

}  // namespace attn
}  // namespace b200
