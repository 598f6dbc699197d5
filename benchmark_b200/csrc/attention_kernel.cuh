// Fused attention forward for sm_100a: O = softmax(Q K^T * scale) V.
//
// Replaces the reference's qk_tma_mma_ld_kernel (0.attention/attention.cu:1503-1974)
// and generalises it to the scalar path's semantics
// (real_attention_bf16_d128_kernel, attention.cu:210-274): any B, Hq, Hkv (GQA,
// attention.cu:176-183), Sq != Skv with bottom-right causal masking
// (attention.cu:167-174), ragged tails, head_dim 64 or 128.
//
// Persistent CTAs (one per SM) walk work items = (batch, q head, 128-row Q
// tile).  Each item streams its head's K/V tiles (128 keys each).  Roles:
//
//   warps 0-7   softmax: warp w owns 16 query rows (TMEM lanes
//               32*(w%4) + 16*(w/4) + [0,16)), four threads per row
//   warps 8-11  epilogue: O / l -> bf16 -> shared -> TMA store
//   warp  12    TMA producer for Q (per item) and the K ring; TMEM allocator
//   warp  13    O += P V issuer (whole warp, one elected lane issues)
//   warp  14    TMA producer for the V ring (its own thread, so K loads run
//               ahead of the V ring's slower turnover)
//   warp  15    S = Q K^T issuer
// Each warpgroup moves its register budget with setmaxnreg (softmax 184,
// epilogue 64, producers/issuers 80 registers per thread).
//
// TMEM (512 columns): three S buffers [0,128) [128,256) [256,384) rotate over
// the global tile sequence; O at [384, 384+D).  P (bf16 pairs) overwrites the
// first 64 columns of its S buffer; keys 0-63 land in columns [0,32), keys
// 64-127 in [32,64).  The epilogue of an item reads O while the softmax
// already works on the next item; the next item's first PV waits for it.
//
// Why this shape: the tensor core runs M=128 products at full rate only for
// N >= 128 with one operand in TMEM or both streams within the 128 B/clk
// shared-memory read budget, and MUFU exp2 (16/clk/SM) costs as many cycles
// per K/V tile as the two 128x128x128 products.  Three S buffers let S(t+1)
// and S(t+2) run while the softmax of tile t runs, so neither the tensor core
// nor the softmax waits on the other's latency and softmax warps may drift a
// tile apart; eight independent softmax warps (16 rows each) put two on
// every scheduler without any cross-warp barrier.
//
// MMA issue over the global tile stream t (crossing item boundaries): warp
// 15 issues S(t) once K(t) has landed and PV(t-3) has completed (p_free: P(t-3)
// lives in the buffer S(t) overwrites); warp 13 issues PV(t) once all eight
// softmax warps have stored P(t) and V(t) has landed.  Two issuers keep the
// tensor pipe fed while one of them waits on a barrier (a single warp issuing
// both streams measured 26 % slower in isolation, peak_probe --probe tile).
//
// Softmax per tile: a thread reads 32 scores of each of its two rows
// (16x256b TMEM loads); where a row max is needed it is completed by two
// shuffles, and the running max m is kept in log2 units.  O and the row sums
// are rescaled only when a block raises m by more than kRescaleLog2
// (otherwise P values up to 2^kRescaleLog2 accumulate unscaled: exact in
// fp32, O / l unchanged), after PV(t-1) has completed.  Unmasked tiles after
// an item's first compute P against the running max directly and take the
// tile max only when the P sums show a jump (rare).  P is stored with
// 16x128b stores, whose column order matches the key pairs each thread
// holds, and published (store wait, fence, one arrive per warp) at the end
// of its own tile, before the next tile's scores are loaded: a TMEM store
// wait or fence behind an outstanding TMEM load waits for that load too.
//
// Short problems (too few Q tiles to fill the SMs) split each Q tile's K/V
// tiles among nsplit work units.  A unit's epilogue writes its unnormalised
// O rows and per-row (m, l) to a workspace in global memory, fences, and
// counts itself in the Q tile's counter; the unit that completes the count
// merges all units (O = sum_u O_u 2^(m_u - m) / sum_u l_u 2^(m_u - m)),
// stores O and resets the counter.  No second launch is needed.
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
constexpr int kEpiWarp0 = 8;
constexpr int kTmaWarp = 12;   // Q and K loads
constexpr int kMmaWarp = 13;   // O += P V issuer
constexpr int kTmaVWarp = 14;  // V loads
constexpr int kMmaSWarp = 15;  // S = Q K^T issuer
constexpr int kThreads = 512;
// Registers per thread after the split: softmax warpgroups 0-1 grow, the
// epilogue warpgroup 2 and the producer/issuer warpgroup 3 shrink; the sum is
// the pool the block launches with (512 threads x 128).
constexpr int kLaunchRegs = 65536 / kThreads;
constexpr int kSoftmaxRegs = 184;
constexpr int kEpiRegs = 64;
constexpr int kCtlRegs = 80;
static_assert(8 * 32 * kSoftmaxRegs + 4 * 32 * kEpiRegs + 4 * 32 * kCtlRegs ==
                  kThreads * kLaunchRegs,
              "register split must use exactly the launch pool");
static_assert(kSoftmaxRegs % 8 == 0 && kEpiRegs % 8 == 0 && kCtlRegs % 8 == 0 &&
                  kEpiRegs >= 24 && kCtlRegs >= 24 && kSoftmaxRegs <= 256,
              "setmaxnreg counts");
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleLog2 = 8.0f;
constexpr float kRescaleP = 256.0f;  // 2^kRescaleLog2
constexpr int kSBufs = 3;  // S buffers in TMEM (P overwrites its S buffer)
constexpr int kBarEpilogue = 1;  // named barrier: warps 8-11

struct Params {
  int B, Hq, Hkv, Sq, Skv;
  int group;     // Hq / Hkv
  int n_qtiles;  // ceil(Sq / 128)
  int n_items;   // work units: B * Hq * n_qtiles * nsplit
  int causal;      // bottom-right aligned
  int causal_off;  // Skv - Sq
  int cgroup;      // causal: Q planes per ordering group (their K/V fit in L2 together)
  // Split K/V ranges (short sequences): each Q tile's K/V tiles are divided
  // among nsplit work units; a unit writes its unnormalised O rows and (m, l)
  // to ws_o / ws_ml, and the last unit of a Q tile to finish (ws_cnt) merges
  // them and stores O.  nsplit = 1: no split, the ws_* are unused.
  int nsplit;
  float* ws_o;          // [units][128][D]
  float2* ws_ml;        // [units][128] (m in log2 units, l)
  unsigned* ws_cnt;     // [Q tiles] arrivals; the merging unit resets it to 0
  float scale_log2;  // softmax_scale * log2(e)
  // Clock trace (kTrace instantiations only): per-role record regions of
  // trace_cap records (2 x u64: (event << 32 | tile << 24 | iter), clock64)
  // for CTA trace_cta.  Role r (0 Q/K TMA, 1 PV issuer, 2/3 softmax warps 0
  // and 4, 4 epilogue, 5 V TMA, 6 S issuer) starts at trace + r * trace_cap * 2.
  unsigned long long* trace;
  int trace_cap;
  int trace_cta;
};

// Clock-trace events (kTrace); names in benchmark_b200/trace.py.
enum : uint32_t {
  kEvTmaK = 1, kEvTmaV, kEvTmaQ, kEvMmaS, kEvMmaPv, kEvMmaWait, kEvMmaGo, kEvMmaEnd, kEvSmWait,
  kEvSmReady, kEvSmLdDone, kEvSmMaxDone, kEvSmPComputed, kEvSmPublished, kEvSmItemEnd,
  kEvEpiBegin, kEvEpiEnd, kEvSmPLoopDone
};
// 0 K/Q TMA, 1 PV issuer, 2/3 softmax warps 0/4, 4 epilogue, 5 V TMA, 6 S issuer
constexpr int kTraceRoles = 7;

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

// kPair: the CTA-pair form (cta_group::2, non-causal d=128).  Each CTA
// of a pair holds half of every K tile (64 keys) and half of every V tile (64
// of its d columns): the pair MMAs take B's N halves from both CTAs, so a
// K/V tile crosses L2 -> shared memory once per pair of Q tiles, and the
// halved stages allow deeper rings in the same shared memory.
template <int D, bool kPair = false>
struct Cfg {
  static_assert(D == 64 || D == 128, "head_dim must be 64 or 128");
  static_assert(!kPair || D == 128, "the CTA-pair form is built for head_dim 128");
  static constexpr int kBoxes = D / 64;            // 64-column (128-byte) TMA boxes per tile
  static constexpr int kBoxBytes = 128 * 128;      // 128 rows x 128 B = 16 KiB
  static constexpr int kTileBytes = kBoxes * kBoxBytes;
  // K stage: kKRows keys x D (kBoxes boxes of kKRows x 128 B); V stage:
  // 128 keys x kVBoxes 64-column boxes.
  static constexpr int kKRows = kPair ? 64 : 128;
  static constexpr int kKBoxBytes = kKRows * 128;
  static constexpr int kKTileBytes = kBoxes * kKBoxBytes;
  static constexpr int kVBoxes = kPair ? kBoxes / 2 : kBoxes;
  static constexpr int kVTileBytes = kVBoxes * kBoxBytes;
  static constexpr int kKStages = kPair ? 6 : (D == 128) ? 3 : 4;  // K ring depth
  static constexpr int kVStages = kPair ? 4 : (D == 128) ? 2 : 4;  // V ring depth
  static constexpr int kQOff = 0;                       // Q0, Q1 (also O staging)
  static constexpr int kKOff = 2 * kTileBytes;
  static constexpr int kVOff = kKOff + kKStages * kKTileBytes;
  // per-row (m, l) of the item the epilogue works on: one slot suffices, the
  // softmax writes item li's values only after the epilogue released li-1
  static constexpr int kLOff = kVOff + kVStages * kVTileBytes;
  static constexpr int kFlagOff = kLOff + 128 * 8;  // abort flag and merge flag (epilogue)
  static constexpr int kBarOff = kFlagOff + 16;
  // q_full[2] q_empty[2] k_full[K] k_empty[K] v_full[V] v_empty[V]
  // s_ready[3] p_ready[3] p_free[3] pv_done o_full o_empty l_ready[2] drain done o_free
  static constexpr int kNumBars = 4 + 2 * kKStages + 2 * kVStages + 3 * kSBufs + 1 + 4 + 3;
  static constexpr int kTmemSlotOff = kBarOff + kNumBars * 8;
  static constexpr int kSmemBytes = kTmemSlotOff + 16 + 1024;  // + 1 KiB alignment slack
  static_assert(kSmemBytes <= 232448, "exceeds the 227 KiB of shared memory a CTA may use");
  static constexpr uint32_t kIdescS = idesc_bf16_f32(kPair ? 256 : 128, kBN, false, false);
  static constexpr uint32_t kIdescO = idesc_bf16_f32(kPair ? 256 : 128, D, false, true);
  static constexpr uint32_t kColO = 128 * kSBufs;
};

// Wait sites reported in the status word.
enum : uint32_t {
  kSiteQFull = 1, kSiteKFull, kSiteVFull, kSitePReady, kSiteKEmpty, kSiteVEmpty,
  kSiteSReady, kSiteOFull, kSiteQEmpty, kSitePvDone, kSiteOEmpty, kSiteLReady,
  kSiteSmemLayout = 0xF0  // reserved: a tile layout that does not fit its shared memory
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
  int j0;    // first K/V tile of this unit (split K/V ranges; else 0)
  int n;     // K/V tiles to visit
  int min_lim;
  int tile;  // Q tile index (unit / nsplit): the merge counter of split units
};

// Work item k.  Non-causal: items of one head are adjacent, so the CTAs
// running at one time share a few heads' K/V in L2.  Causal: planes are taken
// in groups of p.cgroup (sized on the host so that a group's K/V fit in L2
// together); inside a group the heaviest Q tiles (last rows) come first.
__device__ __forceinline__ Item decode_item(const Params& p, int unit) {
  // A Q tile's split units are adjacent, so they run at the same time.
  const int k = unit / p.nsplit;
  const int split = unit - k * p.nsplit;
  const int bhs = p.B * p.Hq;
  int bh, qt;
  if (p.causal) {
    const int per_group = p.cgroup * p.n_qtiles;
    const int g = k / per_group;
    const int kl = k - g * per_group;
    const int gs = min(p.cgroup, bhs - g * p.cgroup);  // planes in this group
    qt = p.n_qtiles - 1 - kl / gs;
    bh = g * p.cgroup + (kl - (kl / gs) * gs);
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
  int n_all;
  tile_extent(p, it.row0, &n_all, &it.min_lim);
  it.j0 = n_all * split / p.nsplit;
  it.n = n_all * (split + 1) / p.nsplit - it.j0;
  it.tile = k;
  return it;
}

// The r-th item of this CTA: rounds of gridDim.x items; causal rounds
// alternate direction so every CTA gets a similar total of K/V tiles.
__device__ __forceinline__ int item_index(const Params& p, int r) {
  const int g = static_cast<int>(gridDim.x);
  const int c = static_cast<int>(blockIdx.x);
  return r * g + ((p.causal && (r & 1)) ? g - 1 - c : c);
}

// CTA-pair form (non-causal): work unit k = (plane, pair of adjacent Q
// tiles); the CTA of cluster rank `rank` takes Q tile 2 * pair + rank (past
// the last tile when n_qtiles is odd: its rows are out of range, TMA reads
// zeros and nothing is stored).  Both CTAs visit all K/V tiles of the plane.
// (Causal problems stay on one CTA per Q tile: pairs there must visit the
// second tile's extent, whose last tile the first tile's rows mask entirely,
// and measured 3-5 % slower on config 3.)
__device__ __forceinline__ Item decode_pair_item(const Params& p, int unit) {
  // Clusters are (2, 1, 1) over a 1-D grid: the cluster rank is blockIdx.x & 1.
  const int rank = static_cast<int>(blockIdx.x & 1u);
  const int npq = (p.n_qtiles + 1) >> 1;
  const int bh = unit / npq;
  const int qt = 2 * (unit - bh * npq) + rank;
  const int b = bh / p.Hq;
  const int hq = bh - b * p.Hq;
  Item it;
  it.zq = bh;
  it.zkv = b * p.Hkv + hq / p.group;
  it.row0 = qt * kBM;
  it.j0 = 0;
  it.n = (p.Skv + kBN - 1) / kBN;
  it.min_lim = p.Skv;
  it.tile = unit;
  return it;
}

// The r-th unit of this CTA pair: rounds of (gridDim.x / 2) units.
__device__ __forceinline__ int pair_item_index(int r) {
  const int g = static_cast<int>(gridDim.x >> 1);
  return r * g + static_cast<int>(blockIdx.x >> 1);
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

// P for 32 keys of each of this thread's two rows (8 repeats of the
// 16x256b layout: s[4g], s[4g+1] row a, s[4g+2], s[4g+3] row b): exp2(x) as
// bf16 pairs, x = s * sc - m (s pre-scaled in masked blocks, sc = 1); pk[2g]
// row a, pk[2g+1] row b (the 16x128b store order).  Accumulates fp32 row
// sums in packed pairs.  kEmu of every 8 pairs use the FMA-pipe exp2
// (exp2_fma_x2), the rest MUFU; masked blocks use MUFU only (exact zeros).
template <int kEmu, bool kMasked>
__device__ __forceinline__ void p_rows(const float* s, float sc, float nm_a, float nm_b,
                                       uint64_t& rs_a, uint64_t& rs_b, uint32_t (&pk)[16]) {
  const uint64_t sc2 = f2_pack(sc, sc);
  const uint64_t na2 = f2_pack(nm_a, nm_a);
  const uint64_t nb2 = f2_pack(nm_b, nm_b);
#pragma unroll
  for (int g = 0; g < 8; ++g) {
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const uint64_t x2 = f2_fma(f2_pack(s[4 * g + 2 * rr], s[4 * g + 2 * rr + 1]), sc2,
                                 rr ? nb2 : na2);
      float x0, x1, p0, p1;
      f2_unpack(x2, x0, x1);
      if (!kMasked && ((2 * g + rr) & 7) < kEmu) {
        exp2_fma_x2(x0, x1, p0, p1);
      } else {
        p0 = ex2_approx(x0);
        p1 = ex2_approx(x1);
      }
      if (rr)
        rs_b = f2_add(rs_b, f2_pack(p0, p1));
      else
        rs_a = f2_add(rs_a, f2_pack(p0, p1));
      pk[2 * g + rr] = pack_bf16x2(p0, p1);
    }
  }
}

template <int D, int kEmu, bool kTrace = false, bool kPair = false>
__global__ void __launch_bounds__(kThreads, 1)
    attention_fwd_kernel(const __grid_constant__ CUtensorMap q_map,
                         const __grid_constant__ CUtensorMap k_map,
                         const __grid_constant__ CUtensorMap v_map,
                         const __grid_constant__ CUtensorMap o_map, const Params p) {
  using C = Cfg<D, kPair>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* q_buf = smem + C::kQOff;
  uint8_t* k_buf = smem + C::kKOff;
  uint8_t* v_buf = smem + C::kVOff;
  float2* stat = reinterpret_cast<float2*>(smem + C::kLOff);  // [row] = (m, l)
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kFlagOff);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* q_full = bars;
  uint64_t* q_empty = q_full + 2;
  uint64_t* k_full = q_empty + 2;
  uint64_t* k_empty = k_full + C::kKStages;
  uint64_t* v_full = k_empty + C::kKStages;
  uint64_t* v_empty = v_full + C::kVStages;
  uint64_t* s_ready = v_empty + C::kVStages;
  uint64_t* p_ready = s_ready + kSBufs;
  uint64_t* p_free = p_ready + kSBufs;  // PV(t) done: S buffer t % kSBufs reusable
  uint64_t* pv_done = p_free + kSBufs;
  uint64_t* o_full = pv_done + 1;
  uint64_t* o_empty = o_full + 1;
  uint64_t* l_ready = o_empty + 1;
  uint64_t* drain = l_ready + 2;
  uint64_t* done = drain + 1;  // phase 0 completes at setup and never changes
  // Pair only, in the leader: both CTAs' epilogues have read O (the PV issuer
  // may overwrite it).  o_empty stays each CTA's own epilogue -> softmax
  // handshake.
  uint64_t* o_free = done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kTmemSlotOff);

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();
  // CTA pair: rank 0 (the leader) issues every MMA for both CTAs and owns
  // the barriers the MMAs wait on (q/k/v_full, p_ready, o_free, p_free);
  // the barriers the MMAs' commits signal exist in both CTAs.
  const uint32_t rank = kPair ? (blockIdx.x & 1u) : 0u;  // = %cluster_ctarank for (2, 1, 1)
  const bool leader = rank == 0;
  const int units_per_round = static_cast<int>(kPair ? gridDim.x >> 1 : gridDim.x);
  const int rounds = (p.n_items + units_per_round - 1) / units_per_round;
  auto item_at = [&](int r) { return kPair ? pair_item_index(r) : item_index(p, r); };
  auto decode_at = [&](int k) {
    return kPair ? decode_pair_item(p, k) : decode_item(p, k);
  };
  // The leader's copy of a barrier of this CTA's layout (shared::cluster).
  auto lead_bar = [&](uint64_t* b_) { return mapa_shared(smem_u32(b_), 0u); };

  // ---- setup ----
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&l_ready[i], 8);
    }
    for (int i = 0; i < kSBufs; ++i) {
      mbar_init(&s_ready[i], 1);
      mbar_init(&p_ready[i], kPair ? 16 : 8);  // softmax warps (of both CTAs)
      mbar_init(&p_free[i], 1);
    }
    mbar_init(o_full, 1);
    mbar_init(o_empty, kPair ? 4 : 128);  // pair: one arrive per epilogue warp
    mbar_init(o_free, 8);                 // pair: every epilogue warp of both CTAs
    for (int s = 0; s < C::kKStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < C::kVStages; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    mbar_init(pv_done, 1);
    mbar_init(drain, 2);  // one commit from each MMA issuer
    mbar_init(done, 1);
    mbar_arrive(done);
    abort_flag[0] = 0;
    abort_flag[1] = 0;
    fence_mbar_init();
  }
  if (warp == kTmaWarp) {
    if constexpr (kPair) {
      tmem_alloc_pair(tmem_slot, kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, kTmemCols);
      tmem_relinquish();
    }
    if (lane == 0) {
      tma_prefetch_desc(&q_map);
      tma_prefetch_desc(&k_map);
      tma_prefetch_desc(&v_map);
      tma_prefetch_desc(&o_map);
    }
  }
  tc_fence_before();
  // A pair's barriers are initialised in both CTAs before either signals the
  // other's.
  if constexpr (kPair)
    cluster_sync_all();
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const bool trace_cta = kTrace && static_cast<int>(blockIdx.x) == p.trace_cta;
  // Each warpgroup moves its register budget first, inside its own branch,
  // so the compiler sizes each role's code to that role's budget.
  if (warp >= static_cast<uint32_t>(kTmaWarp)) {
    // Warpgroup 3: producers and the two MMA issuers.
    setmaxnreg_dec<kCtlRegs>();
    if (warp == kTmaWarp || warp == kTmaVWarp) {
      // ================= TMA producers (Q + K, and V) =================
      if (lane == 0) {
        const bool is_k = warp == kTmaWarp;
        Tracer<kTrace> tr(p, is_k ? 0 : 5, trace_cta);
        // Q is read once; K/V tiles are re-read by every Q tile of their
        // plane while they sit in L2.
        const uint64_t pol_q = l2_policy_evict_first();
        const uint64_t pol_kv = l2_policy_evict_last();
        int t = 0, li = 0, issued = 0, q_issued = -1;
        bool ok = true;
        for (int r = 0; r < rounds && ok; ++r) {
          const int k = item_at(r);
          if (k >= p.n_items) continue;
          const Item it = decode_at(k);
          const int qb = li & 1;
          const uint32_t qpar = static_cast<uint32_t>(li >> 1) & 1u;
          ++li;
          if (is_k) {
            // Q(li) reuses the buffer the epilogue of item li-2 staged O in.
            ok = mbar_wait(&q_empty[qb], qpar ^ 1u, kSiteQEmpty, kDefaultWaitLimitNs, 20000u);
            if (!ok) break;
            if constexpr (kPair) {
              // Both CTAs' Q tiles land on the leader's barrier.
              if (leader) mbar_arrive_expect_tx(&q_full[qb], 2 * C::kTileBytes);
              for (int h = 0; h < C::kBoxes; ++h)
                tma_load_3d_pair(q_buf + qb * C::kTileBytes + h * C::kBoxBytes, &q_map,
                                 lead_bar(&q_full[qb]), h * 64, it.row0, it.zq, pol_q);
            } else {
              mbar_arrive_expect_tx(&q_full[qb], C::kTileBytes);
              for (int h = 0; h < C::kBoxes; ++h)
                tma_load_3d(q_buf + qb * C::kTileBytes + h * C::kBoxBytes, &q_map, &q_full[qb],
                            h * 64, it.row0, it.zq, pol_q);
            }
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
              if constexpr (kPair) {
                // This CTA's 64 keys of the tile; both halves on the leader's barrier.
                if (leader) mbar_arrive_expect_tx(&k_full[ks], 2 * C::kKTileBytes);
                for (int h = 0; h < C::kBoxes; ++h)
                  tma_load_3d_pair(k_buf + ks * C::kKTileBytes + h * C::kKBoxBytes, &k_map,
                                   lead_bar(&k_full[ks]), h * 64,
                                   (it.j0 + j) * kBN + static_cast<int>(rank) * C::kKRows,
                                   it.zkv, pol_kv);
              } else {
                mbar_arrive_expect_tx(&k_full[ks], C::kTileBytes);
                for (int h = 0; h < C::kBoxes; ++h)
                  tma_load_3d(k_buf + ks * C::kTileBytes + h * C::kBoxBytes, &k_map, &k_full[ks],
                              h * 64, (it.j0 + j) * kBN, it.zkv, pol_kv);
              }
            } else {
              const int vs = t % C::kVStages;
              ok = mbar_wait(&v_empty[vs], (static_cast<uint32_t>(t / C::kVStages) & 1u) ^ 1u,
                             kSiteVEmpty, kDefaultWaitLimitNs, 20000u);
              if (!ok) break;
              tr(kEvTmaV, 0, t);
              if constexpr (kPair) {
                // This CTA's 64 columns of d for all 128 keys.
                if (leader) mbar_arrive_expect_tx(&v_full[vs], 2 * C::kVTileBytes);
                for (int h = 0; h < C::kVBoxes; ++h)
                  tma_load_3d_pair(v_buf + vs * C::kVTileBytes + h * C::kBoxBytes, &v_map,
                                   lead_bar(&v_full[vs]),
                                   (static_cast<int>(rank) * C::kVBoxes + h) * 64,
                                   (it.j0 + j) * kBN, it.zkv, pol_kv);
              } else {
                mbar_arrive_expect_tx(&v_full[vs], C::kTileBytes);
                for (int h = 0; h < C::kBoxes; ++h)
                  tma_load_3d(v_buf + vs * C::kTileBytes + h * C::kBoxBytes, &v_map, &v_full[vs],
                              h * 64, (it.j0 + j) * kBN, it.zkv, pol_kv);
              }
            }
            issued = t + 1;
          }
        }
        if (!ok && kPair && !leader) {
          // Unwinding: this CTA's copies count on the leader's barriers; give
          // the ones already issued time to land before the CTA exits.
          spin_ns(200000);
        } else if (!ok) {
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
    } else if (warp == kMmaWarp || warp == kMmaSWarp) {
      // ================= MMA issuers =================
      // Warp 15 issues S = Q K^T, warp 13 issues O += P V.  Each warp runs its
      // loop whole (operands stay warp-uniform) and one elected lane issues
      // each MMA and commit.  Two issuers keep the tensor pipe fed while one
      // of them waits on a barrier: measured with peak_probe --probe tile, a
      // single warp issuing the kernel's per-tile stream (8 SS + 8 TS MMAs,
      // four commits, a grouped barrier test before each group) needs 1,289
      // cycles per tile, two warps 1,024 = the MMAs alone.  A commit tracks
      // only its own thread's MMAs, so each warp signals its own barriers,
      // and the S issuer learns that PV(t) has read P(t) (S buffer t % 3
      // free for S(t+3)) from p_free rather than from issue order.
      // A pair's MMAs are all issued by its leader; the other CTA's issuer
      // warps have nothing to do.
      if (!kPair || leader) {
        const bool is_pv = warp == kMmaWarp;
        // The traced pair's leader records the issuers for either CTA.
        const bool trace_issuer =
            kPair ? (kTrace && static_cast<int>(blockIdx.x >> 1) == (p.trace_cta >> 1))
                  : trace_cta;
        Tracer<kTrace> tr(p, is_pv ? 1 : 6, trace_issuer && lane == 0);
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
        constexpr uint32_t kKTile16 = C::kKTileBytes >> 4, kKBox16 = C::kKBoxBytes >> 4;
        constexpr uint32_t kVTile16 = C::kVTileBytes >> 4;
        // Commits: a pair's go to the barrier in both CTAs (mask 0b11) or to
        // the leader's only.
        auto commit_both = [](uint64_t* b_) {
          if constexpr (kPair)
            mma_commit_pair_both_warp(b_, 3);
          else
            mma_commit_warp(b_);
        };
        auto commit_lead = [](uint64_t* b_) {
          if constexpr (kPair)
            mma_commit_pair_local_warp(b_);
          else
            mma_commit_warp(b_);
        };
        const uint32_t tO = tmem_base + C::kColO;
        // The barrier that says every epilogue reading O is done with it.
        uint64_t* const o_rd = kPair ? o_free : o_empty;
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
        int t = 0, li = 0;
        bool ok = true;
        if (!is_pv) {
          // S(t) = Q[qb] K(t)^T into S buffer t % kSBufs, once K(t) has landed
          // and PV(t - kSBufs) has consumed that buffer's P.
          for (int r = 0; r < rounds && ok; ++r) {
            const int k = item_at(r);
            if (k >= p.n_items) continue;
            const Item it = decode_at(k);
            const int qb = li & 1;
            const uint32_t qpar = static_cast<uint32_t>(li >> 1) & 1u;
            ++li;
            if (it.n == 0) continue;
            ok = wait3(bar(&q_full[qb]), qpar, dn_a, dn_p, dn_a, dn_p, kSiteQFull);
            const uint64_t dq = dq0 + qb * kTile16;
            for (int j = 0; j < it.n && ok; ++j, ++t) {
              const int sb = t % kSBufs;
              ok = wait3(bar(&k_full[t % C::kKStages]), kpar(t), bar(&p_free[sb]),
                         (static_cast<uint32_t>(t / kSBufs) & 1u) ^ 1u, dn_a, dn_p, kSiteKFull);
              if (!ok) break;
              tr(kEvMmaS, qb, t);
              const uint64_t dk = dk0 + (t % C::kKStages) * kKTile16;
              const uint32_t ts = tmem_base + static_cast<uint32_t>(sb * 128);
#pragma unroll
              for (int kk = 0; kk < D / 16; ++kk) {
                const uint32_t off_q = (kk >> 2) * kBox16 + (kk & 3) * 2;
                const uint32_t off_k = (kk >> 2) * kKBox16 + (kk & 3) * 2;
                if constexpr (kPair)
                  mma_ss_pair_warp(ts, dq + off_q, dk + off_k, C::kIdescS, kk > 0 ? 1u : 0u);
                else
                  mma_ss_warp(ts, dq + off_q, dk + off_k, C::kIdescS, kk > 0 ? 1u : 0u);
              }
              commit_both(&k_empty[t % C::kKStages]);
              commit_both(&s_ready[sb]);
            }
          }
        } else {
          for (int r = 0; r < rounds && ok; ++r) {
            const int k = item_at(r);
            if (k >= p.n_items) continue;
            const Item it = decode_at(k);
            const uint32_t oe_par = (static_cast<uint32_t>(li) & 1u) ^ 1u;  // epilogue of li-1
            if (it.n == 0) {
              // No K/V tiles: O stays unwritten (the epilogue stores zeros in Q's
              // buffer, so Q(li) must have landed first).
              ok = wait3(bar(&q_full[li & 1]), static_cast<uint32_t>(li >> 1) & 1u, bar(o_rd),
                         oe_par, dn_a, dn_p, kSiteQFull);
              if (!ok) break;
              commit_both(o_full);
              ++li;
              continue;
            }
            for (int j = 0; j < it.n && ok; ++j, ++t) {
              const int sb = t % kSBufs;
              // V(t), P(t) and, for an item's first tile, O free (the epilogue
              // of item li-1 has read it), in one grouped wait.
              ok = wait3(bar(&v_full[t % C::kVStages]), vpar(t), bar(&p_ready[sb]),
                         static_cast<uint32_t>(t / kSBufs) & 1u, j == 0 ? bar(o_rd) : dn_a,
                         j == 0 ? oe_par : dn_p, kSitePReady);
              if (!ok) break;
              tr(kEvMmaPv, 0, t);
              // O (+)= P(t) V(t): P is read from the S buffer as the A operand.
              const uint64_t dv = dv0 + (t % C::kVStages) * kVTile16;
              const uint32_t tp = tmem_base + static_cast<uint32_t>(sb * 128);
#pragma unroll
              for (int kk = 0; kk < kBN / 16; ++kk) {
                if constexpr (kPair)
                  mma_ts_pair_warp(tO, tp + kk * 8, dv + kk * (2048 >> 4), C::kIdescO,
                                   (j > 0 || kk > 0) ? 1u : 0u);
                else
                  mma_ts_warp(tO, tp + kk * 8, dv + kk * (2048 >> 4), C::kIdescO,
                              (j > 0 || kk > 0) ? 1u : 0u);
              }
              commit_both(&v_empty[t % C::kVStages]);
              commit_lead(&p_free[sb]);
              commit_both(pv_done);
            }
            if (!ok) break;
            commit_both(o_full);
            ++li;
          }
        }
        // Every MMA this warp issued has completed once its commit lands
        // (the barrier counts one commit from each issuer).
        commit_lead(drain);
        drain_wait(drain, 0);
        tr(kEvMmaEnd, 0, t);
      }
      __syncwarp();
    }
  } else if (warp < static_cast<uint32_t>(kEpiWarp0)) {
    setmaxnreg_inc<kSoftmaxRegs>();
    // ================= softmax (warps 0-7) =================
    // Warp w owns 16 rows: TMEM lanes 32*(w%4) + 16*(w/4) + [0,16).  Thread
    // t of the warp holds rows t/4 and t/4+8 and, of every 8 keys, the pair
    // 2*(t%4), 2*(t%4)+1 (16x256b loads); that pair is one packed P column
    // (16x128b stores), and a row's max needs only two shuffles among the
    // four threads that share it.
    const uint32_t quad = warp & 3u;
    const int rbase = static_cast<int>(quad * 32 + (warp >> 2) * 16);
    const int t0 = static_cast<int>(lane & 3u);
    const int ra = rbase + static_cast<int>(lane >> 2);  // rows of this thread
    const int rb = ra + 8;
    const uint32_t lane_addr = static_cast<uint32_t>(rbase) << 16;
    const float c = p.scale_log2;
    Tracer<kTrace> tr(p, 2 + static_cast<int>(warp >> 2), trace_cta && quad == 0 && lane == 0);
    int t = 0, li = 0;
    bool ok = true;
    // K/V tiles this CTA processes in all (the global tile sequence t).
    int g_total = 0;
    for (int r = 0; r < rounds; ++r) {
      const int k = item_at(r);
      if (k < p.n_items) g_total += decode_at(k).n;
    }
    // S(tt) lives in sr once loaded; the load of its successor in the global
    // tile sequence (also across an item boundary) is issued as soon as tile
    // tt's P is computed, so its latency overlaps the P stores and the
    // bookkeeping.
    uint32_t sr[64];
    bool have_s = false;
    // One 16x256b.x16 load of a tile's scores for d=128; two x8 loads (keys
    // 0-63, then 64-127) for d=64 (same registers; measured +3.4 % on d=64
    // and -5 % on d=128).
    auto load_s = [&](uint32_t taddr) {
      if constexpr (D == 64) {
        tmem_ld_16x256b_x8(taddr, *reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
        tmem_ld_16x256b_x8(taddr + 64u, *reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
      } else {
        tmem_ld_16x256b_x16(taddr, sr);
      }
    };
#pragma unroll 1
    for (int r = 0; r < rounds && ok; ++r) {
      const int k = item_at(r);
      if (k >= p.n_items) continue;
      const Item it = decode_at(k);
      const int qb = li & 1;
      const uint32_t tO = tmem_base + lane_addr + C::kColO;
      const int lim_a = p.causal ? min(p.Skv, it.row0 + ra + p.causal_off + 1) : p.Skv;
      const int lim_b = p.causal ? min(p.Skv, it.row0 + rb + p.causal_off + 1) : p.Skv;
      // Running max of scaled scores (log2 units) and this thread's share of
      // the row sums, for rows a and b.
      float m_a = -INFINITY, m_b = -INFINITY;
      uint64_t l2_a = 0ull, l2_b = 0ull;  // packed pairs: even and odd keys
      bool all_finite = false;  // every row of this warp has a finite running max
#pragma unroll 1
      for (int j = 0; j < it.n; ++j) {
        const int tt = t + j;
        const int sb = tt % kSBufs;
        const uint32_t tS = tmem_base + lane_addr + static_cast<uint32_t>(sb * 128);
        tr(kEvSmWait, warp >> 2, tt);
        if (!have_s) {
          ok = warp_wait(&s_ready[sb], static_cast<uint32_t>(tt / kSBufs) & 1u, kSiteSReady);
          if (!ok) break;
          tc_fence_after();
          load_s(tS);
        }
        tr(kEvSmReady, warp >> 2, tt);
        tmem_wait_ld(*reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
        tmem_wait_ld(*reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
        have_s = false;
        tr(kEvSmLdDone, warp >> 2, tt);
        float* s = reinterpret_cast<float*>(sr);
        const int kbase = (it.j0 + j) * kBN;
        const bool masked = kbase + kBN > it.min_lim;  // uniform across the tile
        float f_a = 1.0f, f_b = 1.0f;
        bool rescale = false;    // this thread's rows
        uint64_t rs_a = 0ull, rs_b = 0ull;
        // Readiness of S(tt+1), tested right after this tile's P loop so that
        // the test's latency overlaps the work that follows.
        const int nb = (tt + 1) % kSBufs;
        bool ready = false;      // this lane's test
        bool ready_all = false;  // the warp's vote on it
        // Rescale the O rows whose maximum jumped, once PV(tt-1) has
        // completed (PV(tt) waits for this tile's P barrier); rare.
        auto rescale_o = [&]() {
          if (!warp_wait(pv_done, static_cast<uint32_t>(tt - 1) & 1u, kSitePvDone)) {
            ok = false;
            return;
          }
          tc_fence_after();
#pragma unroll 1
          for (int c0 = 0; c0 < D; c0 += 64) {
            uint32_t o[32];
            tmem_ld_16x256b_x8(tO + c0, o);
            tmem_wait_ld(o);
#pragma unroll
            for (int g = 0; g < 8; ++g) {
              o[4 * g + 0] = __float_as_uint(__uint_as_float(o[4 * g + 0]) * f_a);
              o[4 * g + 1] = __float_as_uint(__uint_as_float(o[4 * g + 1]) * f_a);
              o[4 * g + 2] = __float_as_uint(__uint_as_float(o[4 * g + 2]) * f_b);
              o[4 * g + 3] = __float_as_uint(__uint_as_float(o[4 * g + 3]) * f_b);
            }
            tmem_st_16x256b_x8(tO + c0, o);
          }
        };
        // A later unmasked tile of rows that already have a finite running max
        // computes P against that max at once, without the tile max; only
        // when some row's max rose by more than 2^kRescaleLog2 (rare, screened
        // by the P sums) is the max taken and P recomputed against it.  Same
        // results as taking the max first: m only moves when the block raises
        // it past the threshold, and then to the block max.
        const bool spec = !masked && j > 0 && all_finite;
        if (spec) {
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            uint32_t pk[16];
            p_rows<kEmu, false>(s + 32 * half, c, -m_a, -m_b, rs_a, rs_b, pk);
            tmem_st_16x128b_x8(tS + 32 * half, pk);
          }
          ready = mbar_try_wait(smem_u32(&s_ready[nb]), static_cast<uint32_t>((tt + 1) / kSBufs) & 1u);
          tr(kEvSmPLoopDone, warp >> 2, tt);
          // Some x of the tile exceeds kRescaleLog2 only if some P value
          // exceeds kRescaleP, and then so does the sum of its lane (all terms
          // are non-negative): the partial sums screen for the rare case, and
          // only then are the exact maxima taken.
          float q0, q1, q2, q3;
          f2_unpack(rs_a, q0, q1);
          f2_unpack(rs_b, q2, q3);
          const bool big = __any_sync(0xffffffffu, fmaxf(fmaxf(q0, q1), fmaxf(q2, q3)) > kRescaleP);
          // Both votes in flight before the first branch on either.
          ready_all = __all_sync(0xffffffffu, ready);
          if (big) {
            float ma = -INFINITY, mb = -INFINITY;
#pragma unroll
            for (int g = 0; g < 16; ++g) {
              ma = fmax3(ma, s[4 * g], s[4 * g + 1]);
              mb = fmax3(mb, s[4 * g + 2], s[4 * g + 3]);
            }
            // fma is monotone in s for c >= 0: the max of x is x of the max.
            float xa = fmaf(ma, c, -m_a), xb = fmaf(mb, c, -m_b);
            xa = fmaxf(xa, __shfl_xor_sync(0xffffffffu, xa, 1));
            xb = fmaxf(xb, __shfl_xor_sync(0xffffffffu, xb, 1));
            xa = fmaxf(xa, __shfl_xor_sync(0xffffffffu, xa, 2));
            xb = fmaxf(xb, __shfl_xor_sync(0xffffffffu, xb, 2));
            if (xa > kRescaleLog2) {
              f_a = ex2_approx(-xa);
              m_a += xa;
              rescale = true;
            }
            if (xb > kRescaleLog2) {
              f_b = ex2_approx(-xb);
              m_b += xb;
              rescale = true;
            }
            if (__any_sync(0xffffffffu, rescale)) {
              // Redo P against the raised maxima.
              tmem_wait_st();
              rs_a = 0ull;
              rs_b = 0ull;
#pragma unroll
              for (int half = 0; half < 2; ++half) {
                uint32_t pk[16];
                p_rows<kEmu, false>(s + 32 * half, c, -m_a, -m_b, rs_a, rs_b, pk);
                tmem_st_16x128b_x8(tS + 32 * half, pk);
              }
              rescale_o();
            }
          }
        } else {
          float mx_a, mx_b;
          if (masked) {
            // Scale first, then mask, so masked keys are exactly -inf for any scale.
            const int va = lim_a - kbase - 2 * t0, vb = lim_b - kbase - 2 * t0;
            mx_a = -INFINITY;
            mx_b = -INFINITY;
#pragma unroll
            for (int g = 0; g < 16; ++g) {
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const float xa = 8 * g + e < va ? s[4 * g + e] * c : -INFINITY;
                const float xb = 8 * g + e < vb ? s[4 * g + 2 + e] * c : -INFINITY;
                s[4 * g + e] = xa;
                s[4 * g + 2 + e] = xb;
                mx_a = fmaxf(mx_a, xa);
                mx_b = fmaxf(mx_b, xb);
              }
            }
          } else {
            // Four independent chains per row over the 16 repeats.
            float a[4], b[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              a[u] = fmaxf(s[4 * u], s[4 * u + 1]);
              b[u] = fmaxf(s[4 * u + 2], s[4 * u + 3]);
            }
#pragma unroll
            for (int g = 4; g < 16; ++g) {
              a[g & 3] = fmax3(a[g & 3], s[4 * g], s[4 * g + 1]);
              b[g & 3] = fmax3(b[g & 3], s[4 * g + 2], s[4 * g + 3]);
            }
            mx_a = fmaxf(fmaxf(a[0], a[1]), fmaxf(a[2], a[3])) * c;
            mx_b = fmaxf(fmaxf(b[0], b[1]), fmaxf(b[2], b[3])) * c;
          }
          mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
          mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
          mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
          mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
          tr(kEvSmMaxDone, warp >> 2, tt);
          // Running-max update with lazy rescaling (per row; the four
          // threads of a row hold the same values, so they decide alike).
          if (m_a == -INFINITY) {
            m_a = mx_a;  // no probability mass accumulated yet for this row
          } else if (mx_a > m_a + kRescaleLog2) {
            f_a = ex2_approx(m_a - mx_a);
            m_a = mx_a;
            rescale = true;
          }
          if (m_b == -INFINITY) {
            m_b = mx_b;
          } else if (mx_b > m_b + kRescaleLog2) {
            f_b = ex2_approx(m_b - mx_b);
            m_b = mx_b;
            rescale = true;
          }
          const bool rescale_w = __any_sync(0xffffffffu, rescale);
          all_finite = __all_sync(0xffffffffu, m_a != -INFINITY && m_b != -INFINITY);
          const float nm_a = (m_a == -INFINITY) ? 0.0f : -m_a;
          const float nm_b = (m_b == -INFINITY) ? 0.0f : -m_b;
          const float sc = masked ? 1.0f : c;  // masked scores are pre-scaled
          // P for keys 0-63 (repeats g = 0..7), then 64-127 (g = 8..15).
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            uint32_t pk[16];
            if (masked)
              p_rows<kEmu, true>(s + 32 * half, sc, nm_a, nm_b, rs_a, rs_b, pk);
            else
              p_rows<kEmu, false>(s + 32 * half, sc, nm_a, nm_b, rs_a, rs_b, pk);
            tmem_st_16x128b_x8(tS + 32 * half, pk);
          }
          ready = mbar_try_wait(smem_u32(&s_ready[nb]), static_cast<uint32_t>((tt + 1) / kSBufs) & 1u);
          ready_all = __all_sync(0xffffffffu, ready);
          if (rescale_w && j > 0) rescale_o();
        }
        tr(kEvSmPComputed, warp >> 2, tt);
        // S(tt+1) (the next item's first tile after an item's last), if it is
        // already computed: its load starts once P(tt) is published.
        have_s = ready_all && tt + 1 < g_total && ok;
        if (ok) {
          // Publish P(tt) (and any O rescale) before S(tt+1)'s load is
          // issued: the store wait and fence would otherwise also wait for
          // that load (measured 2 % slower).
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if constexpr (kPair)
            mbar_arrive_cluster_warp(lead_bar(&p_ready[sb]));  // the leader issues PV
          else
            mbar_arrive_warp(&p_ready[sb]);
          tr(kEvSmPublished, warp >> 2, tt);
        }
        if (have_s) {
          tc_fence_after();
          load_s(tmem_base + lane_addr + static_cast<uint32_t>(nb * 128));
        }
        l2_a = f2_fma(l2_a, f2_pack(f_a, f_a), rs_a);
        l2_b = f2_fma(l2_b, f2_pack(f_b, f_b), rs_b);
        if (!ok) break;
      }
      if (!ok) break;
      // Row sums over the four threads of each row, handed to the epilogue
      // once it has finished the previous item (li - 1) and read its sums.
      float l_a, l_b;
      {
        float e0, e1;
        f2_unpack(l2_a, e0, e1);
        l_a = e0 + e1;
        f2_unpack(l2_b, e0, e1);
        l_b = e0 + e1;
      }
      l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
      l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
      l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
      l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
      ok = warp_wait(o_empty, (static_cast<uint32_t>(li) & 1u) ^ 1u, kSiteOEmpty);
      if (!ok) break;
      if (t0 == 0) {
        stat[ra] = make_float2(m_a, l_a);
        stat[rb] = make_float2(m_b, l_b);
      }
      __syncwarp();
      mbar_arrive_warp(&l_ready[qb]);
      tr(kEvSmItemEnd, warp >> 2, li);
      t += it.n;
      ++li;
    }
    if (have_s) {
      // Abandoned prefetch (only after an abort): let the load land.
      tmem_wait_ld(*reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
      tmem_wait_ld(*reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
    }
  } else {
    setmaxnreg_dec<kEpiRegs>();
    // ================= epilogue (warps 8-11) =================
    const uint32_t quad = warp & 3u;
    const int row = static_cast<int>(quad * 32 + lane);
    const uint32_t lane_addr = (quad * 32u) << 16;
    Tracer<kTrace> tr(p, 4, trace_cta && quad == 0 && lane == 0);
    // O is never read back: stored evict_first, its dirty lines do not crowd
    // K/V out of L2.  Measured on config 3 in full (64 causal heads of
    // 16384): without the hint the L2 filled with O lines and K/V came from
    // HBM 6x over (18.9 GB per launch against 3.1 GB with it), and the power
    // that cost lowered the clock under the 1 kW cap.
    const uint64_t pol_o = l2_policy_evict_first();
    int li = 0;
#pragma unroll 1
    for (int r = 0; r < rounds; ++r) {
      const int k = item_at(r);
      if (k >= p.n_items) continue;
      const Item it = decode_at(k);
      const int qb = li & 1;
      const uint32_t qpar = static_cast<uint32_t>(li >> 1) & 1u;
      ++li;
      tr(kEvEpiBegin, qb, li - 1);
      const bool got =
          warp_wait(o_full, static_cast<uint32_t>(li - 1) & 1u, kSiteOFull) &&
          warp_wait(&l_ready[qb], qpar, kSiteLReady);
      if (!got) abort_flag[0] = 1;
      tc_fence_after();
      const uint32_t tO = tmem_base + lane_addr + C::kColO;
      const float2 ml = stat[row];  // (m, l) of this row
      const bool have_o = got && it.n > 0;
      uint8_t* obuf = q_buf + qb * C::kTileBytes;
      const uint32_t obase = smem_u32(obuf);
      // Pack 16 fp32 values of this row (columns c0..c0+15) to bf16 and
      // stage them in the 128-byte-swizzled O tile.
      auto stage16 = [&](int c0, const float* v) {
        uint32_t w[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) w[e] = pack_bf16x2(v[2 * e], v[2 * e + 1]);
        const int box = c0 >> 6;
        const int chunk0 = (c0 & 63) >> 3;  // 16-byte chunk index inside the 128-byte row
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int ch = (chunk0 + u) ^ (row & 7);
          st_shared_v4(obase + box * C::kBoxBytes + row * 128 + ch * 16, w[4 * u], w[4 * u + 1],
                       w[4 * u + 2], w[4 * u + 3]);
        }
      };
      // 8 values (columns c0..c0+7, c0 % 8 == 0): one 16-byte chunk.
      auto stage8 = [&](int c0, const float* v) {
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) w[e] = pack_bf16x2(v[2 * e], v[2 * e + 1]);
        const int ch = ((c0 & 63) >> 3) ^ (row & 7);
        st_shared_v4(obase + (c0 >> 6) * C::kBoxBytes + row * 128 + ch * 16, w[0], w[1], w[2],
                     w[3]);
      };
      bool store = true;  // this unit stores the O tile
      if (kPair || p.nsplit == 1) {
        const float inv = (have_o && ml.y > 0.0f) ? 1.0f / ml.y : 0.0f;
#pragma unroll 1
        for (int c0 = 0; c0 < D; c0 += 32) {
          uint32_t o[32];
          if (have_o) {
            tmem_ld32(tO + c0, o);
            tmem_wait_ld(o);
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = 0u;
          }
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * inv);
          stage16(c0, reinterpret_cast<const float*>(&o[0]));
          stage16(c0 + 16, reinterpret_cast<const float*>(&o[16]));
        }
        tc_fence_before();
        if constexpr (kPair) {
          __syncwarp();
          mbar_arrive_warp(o_empty);
          mbar_arrive_cluster_warp(lead_bar(o_free));  // the leader's PV issuer reuses O
        } else {
          mbar_arrive(o_empty);
        }
      } else {
        // Split unit: this unit's unnormalised O rows and (m, l) go to the
        // workspace; the Q tile's last unit to arrive merges all of them.
        float* my_o = p.ws_o + (static_cast<size_t>(k) * 128 + row) * D;
#pragma unroll 1
        for (int c0 = 0; c0 < D; c0 += 32) {
          uint32_t o[32];
          if (have_o) {
            tmem_ld32(tO + c0, o);
            tmem_wait_ld(o);
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = 0u;
          }
#pragma unroll
          for (int e = 0; e < 8; ++e)
            reinterpret_cast<uint4*>(my_o + c0)[e] =
                make_uint4(o[4 * e], o[4 * e + 1], o[4 * e + 2], o[4 * e + 3]);
        }
        p.ws_ml[static_cast<size_t>(k) * 128 + row] =
            have_o ? ml : make_float2(-INFINITY, 0.0f);
        __threadfence();
        named_bar_sync(kBarEpilogue, 128);  // every row of this unit is written
        if (quad == 0 && lane == 0) {
          int last = 0;
          if (abort_flag[0] == 0) {
            const unsigned prev = atomicAdd(&p.ws_cnt[it.tile], 1u);
            last = prev == static_cast<unsigned>(p.nsplit - 1);
            if (last) p.ws_cnt[it.tile] = 0u;  // every unit has arrived: reset for the next call
          }
          abort_flag[1] = last;
        }
        named_bar_sync(kBarEpilogue, 128);
        store = abort_flag[1] != 0;
        if (store) {
          // Merge: this unit's rows come from TMEM (O is released only
          // afterwards), the other units' from the workspace (L2).
          __threadfence();
          const int u0 = it.tile * p.nsplit;
          float mmax = -INFINITY;
          for (int sp = 0; sp < p.nsplit; ++sp)
            mmax = fmaxf(mmax, __ldcg(&p.ws_ml[static_cast<size_t>(u0 + sp) * 128 + row]).x);
          float lsum = 0.0f;
          for (int sp = 0; sp < p.nsplit; ++sp) {
            const float2 v = __ldcg(&p.ws_ml[static_cast<size_t>(u0 + sp) * 128 + row]);
            if (v.y > 0.0f) lsum += v.y * ex2_approx(v.x - mmax);
          }
          const float inv = lsum > 0.0f ? 1.0f / lsum : 0.0f;
          const float w_own = (have_o && ml.y > 0.0f) ? ex2_approx(ml.x - mmax) * inv : 0.0f;
#pragma unroll 1
          for (int c0 = 0; c0 < D; c0 += 8) {
            // Units are added in unit order (this unit's rows from TMEM at
            // its own place), so the result does not depend on which unit
            // arrived last.
            uint32_t own[8];
            if (have_o) {
              tmem_ld8(tO + c0, own);
              tmem_wait_ld();
              reg_written_here8(own);
            } else {
#pragma unroll
              for (int e = 0; e < 8; ++e) own[e] = 0u;
            }
            float acc[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[e] = 0.0f;
#pragma unroll 1
            for (int sp = 0; sp < p.nsplit; sp += 2) {
              float4 x[2][2];
              float w[2];
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const int uu = u0 + sp + h;
                const bool use = sp + h < p.nsplit && uu != k;
                const float2 v = use ? __ldcg(&p.ws_ml[static_cast<size_t>(uu) * 128 + row])
                                     : make_float2(-INFINITY, 0.0f);
                w[h] = uu == k ? w_own : (v.y > 0.0f ? ex2_approx(v.x - mmax) * inv : 0.0f);
                const float4* src = reinterpret_cast<const float4*>(
                    p.ws_o + (static_cast<size_t>(use ? uu : k) * 128 + row) * D + c0);
                if (uu == k) {
                  x[h][0] = make_float4(__uint_as_float(own[0]), __uint_as_float(own[1]),
                                        __uint_as_float(own[2]), __uint_as_float(own[3]));
                  x[h][1] = make_float4(__uint_as_float(own[4]), __uint_as_float(own[5]),
                                        __uint_as_float(own[6]), __uint_as_float(own[7]));
                } else {
                  x[h][0] = __ldcg(src);
                  x[h][1] = __ldcg(src + 1);
                }
              }
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                if (w[h] == 0.0f) continue;  // no mass: its rows may hold anything
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                  acc[4 * e + 0] = fmaf(x[h][e].x, w[h], acc[4 * e + 0]);
                  acc[4 * e + 1] = fmaf(x[h][e].y, w[h], acc[4 * e + 1]);
                  acc[4 * e + 2] = fmaf(x[h][e].z, w[h], acc[4 * e + 2]);
                  acc[4 * e + 3] = fmaf(x[h][e].w, w[h], acc[4 * e + 3]);
                }
              }
            }
            stage8(c0, acc);
          }
        }
        tc_fence_before();
        mbar_arrive(o_empty);
      }
      fence_proxy_async_smem();
      named_bar_sync(kBarEpilogue, 128);
      if (abort_flag[0] != 0) break;
      if (quad == 0 && lane == 0) {
        // (A pair's second tile past the last Q row has nothing to store.)
        if (store && it.row0 < p.Sq) {
          for (int b = 0; b < C::kBoxes; ++b)
            tma_store_3d_hint(&o_map, obuf + b * C::kBoxBytes, b * 64, it.row0, it.zq, pol_o);
          bulk_commit_group();
          bulk_wait_group_read<0>();
        }
        mbar_arrive(&q_empty[qb]);
      }
      tr(kEvEpiEnd, qb, li - 1);
      __syncwarp();
    }
  }

  // ---- teardown ----
  tc_fence_before();
  // A pair's CTAs leave together: the leader's MMAs read the other CTA's
  // shared memory and TMEM until its drain completes.
  if constexpr (kPair)
    cluster_sync_all();
  else
    __syncthreads();
  if (warp == kTmaWarp) {
    tc_fence_after();
    if constexpr (kPair)
      tmem_dealloc_pair(tmem_base, kTmemCols);
    else
      tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace attn
}  // namespace b200
