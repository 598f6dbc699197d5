// C-ABI entry points (include/b200attn.h).  Single translation unit: the
// kernels are header-only so the device status word is one symbol.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <algorithm>
#include <map>
#include <mutex>
#include <string>

#include "b200attn.h"
#include "ptx.cuh"
#include "attention_kernel.cuh"
#include "attention_pair_kernel.cuh"
#include "reference_kernels.cuh"
#include "gemm_kernel.cuh"

#include <cublas_v2.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace {

thread_local std::string t_last_error;

b200_status fail(b200_status s, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return s;
}

b200_status cuda_fail(cudaError_t e, const char* what) {
  return fail(B200_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---- cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda) ----
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// Encoded tensor maps, cached per (base, shape, box) so repeated calls on the
// same buffers skip the driver encode (a map holds only the address and the
// geometry, so a buffer freed and reallocated at the same address with the
// same shape reuses a valid map).  A fixed direct-mapped table: no host
// allocation, and a collision only costs a fresh encode.
struct MapKey {
  const void* base;
  uint64_t d0, d1, d2;
  uint32_t box0, box1, rank;
  bool operator==(const MapKey& o) const {
    return base == o.base && d0 == o.d0 && d1 == o.d1 && d2 == o.d2 && box0 == o.box0 &&
           box1 == o.box1 && rank == o.rank;
  }
};

class MapCache {
 public:
  bool find(const MapKey& k, CUtensorMap* out) {
    std::lock_guard<std::mutex> lock(mu_);
    const Slot& e = slots_[index(k)];
    if (!e.used || !(e.key == k)) return false;
    *out = e.map;
    return true;
  }
  void put(const MapKey& k, const CUtensorMap& m) {
    std::lock_guard<std::mutex> lock(mu_);
    Slot& e = slots_[index(k)];
    e.key = k;
    e.map = m;
    e.used = true;
  }

 private:
  static constexpr size_t kSlots = 256;
  struct Slot {
    MapKey key{};
    CUtensorMap map{};
    bool used = false;
  };
  static size_t index(const MapKey& k) {
    uint64_t h = reinterpret_cast<uintptr_t>(k.base) * 0x9E3779B97F4A7C15ull;
    for (uint64_t v : {k.d0, k.d1, k.d2, static_cast<uint64_t>(k.box0) << 32 | k.box1,
                       static_cast<uint64_t>(k.rank)})
      h = (h ^ v) * 0x100000001B3ull;
    return static_cast<size_t>(h >> 32) % kSlots;
  }
  std::mutex mu_;
  Slot slots_[kSlots];
};

MapCache& map_cache() {
  static MapCache c;
  return c;
}

b200_status encode_bf16_3d_uncached(CUtensorMap* map, const void* base, uint64_t d0,
                                    uint64_t d1, uint64_t d2, uint32_t box0, uint32_t box1);
b200_status encode_bf16_2d_uncached(CUtensorMap* map, const void* base, uint64_t d0,
                                    uint64_t d1, uint32_t box0, uint32_t box1);

// 3-D bf16 tensor [d2][d1][d0] (d0 contiguous), 128-byte swizzled boxes of
// box0 x box1 x 1 elements.
b200_status encode_bf16_3d(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1,
                           uint64_t d2, uint32_t box0, uint32_t box1) {
  const MapKey key{base, d0, d1, d2, box0, box1, 3};
  if (map_cache().find(key, map)) return B200_OK;
  const b200_status st = encode_bf16_3d_uncached(map, base, d0, d1, d2, box0, box1);
  if (st == B200_OK) map_cache().put(key, *map);
  return st;
}

// 2-D bf16 tensor [d1][d0] (d0 contiguous), 128-byte swizzled boxes.
b200_status encode_bf16_2d(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1,
                           uint32_t box0, uint32_t box1) {
  const MapKey key{base, d0, d1, 1, box0, box1, 2};
  if (map_cache().find(key, map)) return B200_OK;
  const b200_status st = encode_bf16_2d_uncached(map, base, d0, d1, box0, box1);
  if (st == B200_OK) map_cache().put(key, *map);
  return st;
}

b200_status encode_bf16_3d_uncached(CUtensorMap* map, const void* base, uint64_t d0,
                                    uint64_t d1, uint64_t d2, uint32_t box0, uint32_t box1) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(B200_ECUDA, "cuTensorMapEncodeTiled entry point unavailable");
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {d0 * 2, d0 * d1 * 2};
  const cuuint32_t box[3] = {box0, box1, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims,
                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(B200_ECUDA, "cuTensorMapEncodeTiled failed (%d) for dims %llu x %llu x %llu",
                static_cast<int>(r), static_cast<unsigned long long>(d0),
                static_cast<unsigned long long>(d1), static_cast<unsigned long long>(d2));
  return B200_OK;
}

b200_status encode_bf16_2d_uncached(CUtensorMap* map, const void* base, uint64_t d0,
                                    uint64_t d1, uint32_t box0, uint32_t box1) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(B200_ECUDA, "cuTensorMapEncodeTiled entry point unavailable");
  const cuuint64_t dims[2] = {d0, d1};
  const cuuint64_t strides[1] = {d0 * 2};
  const cuuint32_t box[2] = {box0, box1};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(B200_ECUDA, "cuTensorMapEncodeTiled failed (%d) for dims %llu x %llu",
                static_cast<int>(r), static_cast<unsigned long long>(d0),
                static_cast<unsigned long long>(d1));
  return B200_OK;
}

// cudaFuncSetAttribute once per (kernel, device).
template <typename Kernel>
b200_status ensure_smem_attr(Kernel kernel, int bytes, unsigned* done_mask) {
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  std::lock_guard<std::mutex> lock(mu);
  const unsigned bit = 1u << (dev & 31);
  if (*done_mask & bit) return B200_OK;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(MaxDynamicSharedMemorySize)");
  *done_mask |= bit;
  return B200_OK;
}

int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
  return n > 0 ? n : 148;
}

struct AttnShape {
  int B, Hq, Hkv, Sq, Skv, D, causal;
  float scale;
};

b200_status check_attention_args(const void* q, const void* k, const void* v, const void* o,
                                  int B, int Hq, int Hkv, int Sq, int Skv, int D, int causal,
                                  float softmax_scale, AttnShape* out) {
  if (!q || !k || !v || !o) return fail(B200_EINVAL, "attention: null tensor pointer");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o))
    return fail(B200_EINVAL, "attention: tensor pointers must be 16-byte aligned");
  if (B < 1 || Hq < 1 || Hkv < 1 || Sq < 1 || Skv < 1)
    return fail(B200_EINVAL, "attention: invalid shape B=%d Hq=%d Hkv=%d Sq=%d Skv=%d", B, Hq,
                Hkv, Sq, Skv);
  if (Hq % Hkv != 0)
    return fail(B200_EINVAL, "attention: requires Hq %% Hkv == 0; got Hq=%d Hkv=%d", Hq, Hkv);
  if (D != 64 && D != 128)
    return fail(B200_EUNSUPPORTED, "attention: head_dim must be 64 or 128; got D=%d", D);
  const float scale = softmax_scale < 0.0f ? 1.0f / std::sqrt(static_cast<float>(D))
                                           : softmax_scale;
  if (!std::isfinite(scale)) return fail(B200_EINVAL, "attention: softmax_scale is not finite");
  const long long planes_q = static_cast<long long>(B) * Hq;
  const long long planes_kv = static_cast<long long>(B) * Hkv;
  if (planes_q > (1ll << 31) || planes_kv > (1ll << 31))
    return fail(B200_EUNSUPPORTED, "attention: B*H too large");
  *out = AttnShape{B, Hq, Hkv, Sq, Skv, D, causal ? 1 : 0, scale};
  return B200_OK;
}

// FMA-pipe exp2 share (pairs of every 8) per head_dim.  Measured on B200
// (c2: d128, c4: d64 workloads): none for d128, whose softmax tile is bound
// by its control latencies rather than MUFU (one pair in eight lost 1.6 %),
// and one pair in eight for d64, where MUFU is the tighter pipe.
constexpr int kDefaultEmuD128 = 0;
constexpr int kDefaultEmuD64 = 1;

struct TraceArgs {
  unsigned long long* buf = nullptr;
  int cap = 0;
  int cta = -1;
};

// Split K/V ranges for short problems: when the Q tiles cannot fill half the
// SMs and their K/V ranges are long, each Q tile's K/V tiles are divided among
// up to 8 work units (at least 16 K/V tiles each) so that the grid fills the
// GPU; the units' partial results meet in a workspace and the last unit of
// each Q tile merges them.  Measured on B200 (one head, d=128): N=8192 588 ->
// 691 TFLOP/s (causal 295 -> 375) with 2 units per Q tile; with 32 K/V tiles
// per Q tile (2 heads, N=4096) the merge cost more than the split saved
// (519 -> 466), and with 8 (config 1) the units' fixed costs alone did.
int split_count(long long qtiles, int kv_tiles, int sms) {
  if (qtiles * 2 > sms || kv_tiles < 48) return 1;
  const long long n = std::min<long long>({sms / qtiles, kv_tiles / 16, 8});
  return static_cast<int>(std::max<long long>(n, 1));
}

// Workspace of the split units, one per (device, stream) so that calls on
// different streams never share it; grown on demand, never shrunk.
struct SplitWorkspace {
  float* o = nullptr;       // [units][128][128] fp32 (d=64 uses the first 64 columns' worth)
  float2* ml = nullptr;     // [units][128]
  unsigned* cnt = nullptr;  // [Q tiles], zero between calls
  size_t units = 0, tiles = 0;
};

std::mutex& split_mutex() {
  static std::mutex m;
  return m;
}

std::map<std::pair<int, cudaStream_t>, SplitWorkspace>& split_workspaces() {
  static std::map<std::pair<int, cudaStream_t>, SplitWorkspace> w;
  return w;
}

b200_status split_workspace(cudaStream_t stream, size_t units, size_t tiles, SplitWorkspace* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  std::lock_guard<std::mutex> lock(split_mutex());
  SplitWorkspace& w = split_workspaces()[{dev, stream}];
  if (w.units < units || w.tiles < tiles) {
    // Earlier calls on this stream may still use the old buffers.
    if ((e = cudaStreamSynchronize(stream)) != cudaSuccess) return cuda_fail(e, "workspace sync");
    cudaFree(w.o);
    cudaFree(w.ml);
    cudaFree(w.cnt);
    w = SplitWorkspace{};
    const size_t nu = std::max(units, static_cast<size_t>(256));
    const size_t nt = std::max(tiles, static_cast<size_t>(128));
    if ((e = cudaMalloc(&w.o, nu * 128 * 128 * sizeof(float))) != cudaSuccess ||
        (e = cudaMalloc(&w.ml, nu * 128 * sizeof(float2))) != cudaSuccess ||
        (e = cudaMalloc(&w.cnt, nt * sizeof(unsigned))) != cudaSuccess ||
        (e = cudaMemset(w.cnt, 0, nt * sizeof(unsigned))) != cudaSuccess) {
      cudaFree(w.o);
      cudaFree(w.ml);
      cudaFree(w.cnt);
      w = SplitWorkspace{};
      return cuda_fail(e, "attention split workspace");
    }
    w.units = nu;
    w.tiles = nt;
  }
  *out = w;
  return B200_OK;
}

// After a failed call the merge counters may hold partial counts: zero them.
void reset_split_counters(int dev) {
  std::lock_guard<std::mutex> lock(split_mutex());
  for (auto& kv : split_workspaces())
    if (kv.first.first == dev && kv.second.cnt)
      cudaMemset(kv.second.cnt, 0, kv.second.tiles * sizeof(unsigned));
}

// A caller-fixed split count and workspace (attention_fwd_noalloc).
struct FixedScratch {
  int nsplit;            // K/V splits per Q tile; 0: split_count's choice
  float* o;              // [units][128][128] fp32
  float2* ml;            // [units][128]
  unsigned* cnt;         // [Q tiles]
  size_t max_units, max_qtiles;
};

// The two-Q-tile d=64 kernel on already encoded maps (64-column boxes of 128
// rows, as launch_attention encodes them for d=64).
template <int EMU, bool TRACE>
b200_status launch_pair(const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm,
                        const CUtensorMap& om, b200::attn::Params p, long long units,
                        cudaStream_t stream) {
  namespace pa = b200::attn::pair;
  static unsigned attr_done = 0;
  auto kernel = pa::attention_pair_kernel<EMU, TRACE>;
  b200_status st = ensure_smem_attr(kernel, pa::kSmemBytes, &attr_done);
  if (st != B200_OK) return st;
  static const int launch_regs = [kernel] {
    cudaFuncAttributes a{};
    return cudaFuncGetAttributes(&a, kernel) == cudaSuccess ? a.numRegs : -1;
  }();
  if (launch_regs != b200::attn::kLaunchRegs)
    return fail(B200_EUNSUPPORTED,
                "attention (d=64 pairs): kernel has %d registers per thread at launch; its "
                "register split needs exactly %d",
                launch_regs, b200::attn::kLaunchRegs);
  if (units > 0x3fffffffll) return fail(B200_EUNSUPPORTED, "attention: too many work units");
  p.n_items = static_cast<int>(units);
  p.nsplit = 1;
  const int grid = static_cast<int>(std::min<long long>(units, sm_count()));
  kernel<<<grid, b200::attn::kThreads, pa::kSmemBytes, stream>>>(qm, km, vm, om, p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "attention_fwd launch (d=64 pairs)");
  return B200_OK;
}

// Launch `kernel` on clusters of two CTAs (one per SM): as many clusters as
// can be resident at once (cached per device and kernel), or `units`.
template <typename Kernel, typename... Args>
b200_status launch_cluster2(Kernel kernel, int smem_bytes, long long units, cudaStream_t stream,
                            const char* what, Args... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg{};
  cfg.blockDim = dim3(b200::attn::kThreads, 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem_bytes);
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, int> resident;
  int dev = 0, clusters = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    const auto key = std::make_pair(dev, reinterpret_cast<const void*>(kernel));
    auto it = resident.find(key);
    if (it == resident.end()) {
      cfg.gridDim = dim3(2 * (sm_count() / 2), 1, 1);
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess || n < 1) {
        cudaGetLastError();
        n = sm_count() / 2;
      }
      it = resident.emplace(key, n).first;
    }
    clusters = it->second;
  }
  clusters = static_cast<int>(std::min<long long>(units, clusters));
  cfg.gridDim = dim3(2 * static_cast<unsigned>(clusters), 1, 1);
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, args...);
  if (e != cudaSuccess) return cuda_fail(e, what);
  const cudaError_t e2 = cudaGetLastError();
  if (e2 != cudaSuccess) return cuda_fail(e2, what);
  return B200_OK;
}

// The CTA-pair d=128 kernel (cta_group::2): each cluster of two CTAs takes
// two adjacent Q tiles of one plane and splits every K/V tile's shared-memory
// copy between them (K: 64 keys per CTA, V: 64 columns of d per CTA).  `km`
// is encoded with 64-row boxes.
template <int EMU, bool TRACE>
b200_status launch_cpair(const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm,
                         const CUtensorMap& om, b200::attn::Params p, long long units,
                         cudaStream_t stream) {
  using C = b200::attn::Cfg<128, true>;
  static unsigned attr_done = 0;
  auto kernel = b200::attn::attention_fwd_kernel<128, EMU, TRACE, true>;
  b200_status st = ensure_smem_attr(kernel, C::kSmemBytes, &attr_done);
  if (st != B200_OK) return st;
  static const int launch_regs = [kernel] {
    cudaFuncAttributes a{};
    return cudaFuncGetAttributes(&a, kernel) == cudaSuccess ? a.numRegs : -1;
  }();
  if (launch_regs != b200::attn::kLaunchRegs)
    return fail(B200_EUNSUPPORTED,
                "attention (CTA pairs): kernel has %d registers per thread at launch; its "
                "register split needs exactly %d",
                launch_regs, b200::attn::kLaunchRegs);
  if (units > 0x3fffffffll) return fail(B200_EUNSUPPORTED, "attention: too many work units");
  p.n_items = static_cast<int>(units);
  p.nsplit = 1;
  return launch_cluster2(kernel, C::kSmemBytes, units, stream, "attention_fwd launch (CTA pairs)",
                         qm, km, vm, om, p);
}

template <int D, int EMU, bool TRACE = false>
b200_status launch_attention(const void* q, const void* k, const void* v, void* o,
                             const AttnShape& s, cudaStream_t stream,
                             const TraceArgs& tr = TraceArgs{},
                             const FixedScratch* fixed = nullptr) {
  using C = b200::attn::Cfg<D>;
  static unsigned attr_done = 0;
  auto kernel = b200::attn::attention_fwd_kernel<D, EMU, TRACE>;
  b200_status st = ensure_smem_attr(kernel, C::kSmemBytes, &attr_done);
  if (st != B200_OK) return st;
  // The kernel moves registers between warpgroups (setmaxnreg); the split is
  // sized for exactly kLaunchRegs per thread at launch, and an increase that
  // the pool cannot satisfy would never complete.  Refuse any other build.
  static const int launch_regs = [kernel] {
    cudaFuncAttributes a{};
    return cudaFuncGetAttributes(&a, kernel) == cudaSuccess ? a.numRegs : -1;
  }();
  if (launch_regs != b200::attn::kLaunchRegs)
    return fail(B200_EUNSUPPORTED,
                "attention: kernel has %d registers per thread at launch; its register "
                "split needs exactly %d",
                launch_regs, b200::attn::kLaunchRegs);

  CUtensorMap qm, km, vm, om;
  const uint64_t pq = static_cast<uint64_t>(s.B) * s.Hq;
  const uint64_t pkv = static_cast<uint64_t>(s.B) * s.Hkv;
  constexpr uint32_t kRows = b200::attn::kBM, kKvRows = b200::attn::kBN;
  if ((st = encode_bf16_3d(&qm, q, D, s.Sq, pq, 64, kRows)) != B200_OK) return st;
  if ((st = encode_bf16_3d(&km, k, D, s.Skv, pkv, 64, kKvRows)) != B200_OK) return st;
  if ((st = encode_bf16_3d(&vm, v, D, s.Skv, pkv, 64, kKvRows)) != B200_OK) return st;
  if ((st = encode_bf16_3d(&om, o, D, s.Sq, pq, 64, kRows)) != B200_OK) return st;

  b200::attn::Params p{};
  p.B = s.B;
  p.Hq = s.Hq;
  p.Hkv = s.Hkv;
  p.Sq = s.Sq;
  p.Skv = s.Skv;
  p.group = s.Hq / s.Hkv;
  p.n_qtiles = (s.Sq + b200::attn::kBM - 1) / b200::attn::kBM;
  const long long qtiles = static_cast<long long>(pq) * p.n_qtiles;
  const int kv_tiles = (s.Skv + b200::attn::kBN - 1) / b200::attn::kBN;
  p.nsplit = (fixed && fixed->nsplit > 0) ? fixed->nsplit : split_count(qtiles, kv_tiles, sm_count());
  const long long items = qtiles * p.nsplit;
  if (items > 0x3fffffffll) return fail(B200_EUNSUPPORTED, "attention: too many work items");
  p.n_items = static_cast<int>(items);
  if (p.nsplit > 1 && fixed) {
    if (static_cast<unsigned long long>(items) > fixed->max_units ||
        static_cast<unsigned long long>(qtiles) > fixed->max_qtiles)
      return fail(B200_EUNSUPPORTED,
                  "attention_fwd_noalloc: %lld split units (%lld Q tiles x %d splits) exceed its "
                  "fixed scratch of %zu units and %zu Q tiles; pass fewer splits (1 needs no "
                  "scratch) or use attention_fwd",
                  items, qtiles, p.nsplit, fixed->max_units, fixed->max_qtiles);
    // The merge counters must start at zero; a call that failed part-way
    // may have left counts behind.
    const cudaError_t e = cudaMemsetAsync(fixed->cnt, 0, static_cast<size_t>(qtiles) *
                                                             sizeof(unsigned), stream);
    if (e != cudaSuccess) return cuda_fail(e, "attention_fwd_noalloc: clear merge counters");
    p.ws_o = fixed->o;
    p.ws_ml = fixed->ml;
    p.ws_cnt = fixed->cnt;
  } else if (p.nsplit > 1) {
    SplitWorkspace w;
    if ((st = split_workspace(stream, static_cast<size_t>(items), static_cast<size_t>(qtiles),
                              &w)) != B200_OK)
      return st;
    p.ws_o = w.o;
    p.ws_ml = w.ml;
    p.ws_cnt = w.cnt;
  }
  p.causal = s.causal;
  p.causal_off = s.Skv - s.Sq;
  p.scale_log2 = s.scale * 1.4426950408889634f;
  p.trace = tr.buf;
  p.trace_cap = tr.cap;
  p.trace_cta = tr.cta;
  // Causal items are ordered in groups of planes whose K/V (shared by the
  // group's query heads under GQA) fit in about half of the 126 MB L2, so the
  // CTAs running at one time share their K/V there.  Measured on B200 at
  // interleaved, equal clocks (with evict_first K/V loads and O stores
  // without a hint, the policies of the time): config 3 in full (64 heads,
  // N=16384) ~25 % faster than one heaviest-first order over all heads.
  {
    const double kv_bytes = 4.0 * static_cast<double>(s.Skv) * D;  // K + V of one kv plane
    const double budget = 64.0 * (1 << 20);
    const long long g = static_cast<long long>(budget / kv_bytes) * p.group;
    p.cgroup = static_cast<int>(std::max<long long>(1, std::min<long long>(g, pq)));
  }
  if constexpr (D == 64) {
    // Non-causal d=64 problems that fill the GPU without a K/V split run two
    // Q tiles per work unit (attention_pair_kernel.cuh).
    const long long units = static_cast<long long>(pq) * ((p.n_qtiles + 1) / 2);
    if (!s.causal && p.nsplit == 1 && units >= sm_count())
      return launch_pair<EMU, TRACE>(qm, km, vm, om, p, units, stream);
  } else {
    // Non-causal d=128 problems with a pair of Q tiles for every two SMs
    // and no K/V split run on CTA pairs (cta_group::2).
    const long long units = static_cast<long long>(pq) * ((p.n_qtiles + 1) / 2);
    if (!s.causal && p.nsplit == 1 && 2 * units >= sm_count()) {
      CUtensorMap km_pair;
      if ((st = encode_bf16_3d(&km_pair, k, D, s.Skv, pkv, 64,
                               b200::attn::Cfg<128, true>::kKRows)) != B200_OK)
        return st;
      return launch_cpair<EMU, TRACE>(qm, km_pair, vm, om, p, units, stream);
    }
  }
  // Persistent: one CTA per SM (shared memory admits one), or fewer items.
  const int grid = static_cast<int>(std::min<long long>(items, sm_count()));
  kernel<<<grid, b200::attn::kThreads, C::kSmemBytes, stream>>>(qm, km, vm, om, p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "attention_fwd launch");
  return B200_OK;
}

b200_status check_gemm_args(const void* A, const void* Bm, const void* C, int M, int N, int K,
                            const char* who) {
  if (!A || !Bm || !C) return fail(B200_EINVAL, "%s: null matrix pointer", who);
  if (!aligned16(A) || !aligned16(Bm) || !aligned16(C))
    return fail(B200_EINVAL, "%s: matrix pointers must be 16-byte aligned", who);
  if (M < 1 || N < 1 || K < 1)
    return fail(B200_EINVAL, "%s: invalid shape M=%d N=%d K=%d", who, M, N, K);
  if (K % 8 != 0 || N % 8 != 0)
    return fail(B200_EUNSUPPORTED, "%s: K and N must be multiples of 8 (16-byte rows); got "
                "N=%d K=%d", who, N, K);
  return B200_OK;
}


// One cuBLAS handle per (thread, device) for the comparator.
cublasHandle_t cublas_handle(b200_status* st) {
  thread_local std::map<int, cublasHandle_t> handles;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    *st = fail(B200_ECUDA, "cudaGetDevice");
    return nullptr;
  }
  auto it = handles.find(dev);
  if (it != handles.end()) return it->second;
  cublasHandle_t h = nullptr;
  if (cublasCreate(&h) != CUBLAS_STATUS_SUCCESS) {
    *st = fail(B200_ECUDA, "cublasCreate failed");
    return nullptr;
  }
  handles[dev] = h;
  return h;
}

}  // namespace

extern "C" {

const char* b200_last_error(void) { return t_last_error.c_str(); }

int b200_version(void) { return 100; }

b200_status attention_fwd(const void* q, const void* k, const void* v, void* o, int B, int Hq,
                          int Hkv, int Sq, int Skv, int D, int causal, float softmax_scale,
                          b200_stream_t stream) {
  AttnShape s;
  b200_status st = check_attention_args(q, k, v, o, B, Hq, Hkv, Sq, Skv, D, causal,
                                        softmax_scale, &s);
  if (st != B200_OK) return st;
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  return D == 128 ? launch_attention<128, kDefaultEmuD128>(q, k, v, o, s, cs)
                  : launch_attention<64, kDefaultEmuD64>(q, k, v, o, s, cs);
}

}  // extern "C"

// Scratch of attention_fwd_noalloc: the split units' unnormalised O rows
// (fp32), their per-row (m, l) and the Q tiles' merge counters, in one fixed
// device array so that the entry point allocates nothing.  Every GPU that
// loads this library holds it (about 8.1 MiB) until the process exits, and
// every call shares it: calls that overlap on the GPU (other streams, other
// host threads) race on it.
constexpr size_t kNoAllocUnits = 128;   // split units per call (Q tiles x splits)
constexpr size_t kNoAllocQTiles = 1024; // Q tiles per call when splitting
constexpr size_t kNoAllocOBytes = kNoAllocUnits * 128 * 128 * sizeof(float);
constexpr size_t kNoAllocMlBytes = kNoAllocUnits * 128 * sizeof(float2);
constexpr size_t kNoAllocCntBytes = kNoAllocQTiles * sizeof(unsigned);
static __device__ __align__(256) unsigned char
    g_noalloc_scratch[kNoAllocOBytes + kNoAllocMlBytes + kNoAllocCntBytes];

namespace {
// The array's device address on the current device.  In host code its name
// is only a host-side stand-in, so the address is looked up once per device
// (with that device current) and cached.
b200_status noalloc_scratch(unsigned char** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  constexpr int kMaxDevices = 64;
  if (dev < 0 || dev >= kMaxDevices)
    return fail(B200_EUNSUPPORTED, "attention_fwd_noalloc: device %d out of range", dev);
  static std::mutex mu;
  static void* addr[kMaxDevices] = {};
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || ptr == nullptr)
      return cuda_fail(e != cudaSuccess ? e : cudaErrorInvalidSymbol,
                       "attention_fwd_noalloc: cudaGetSymbolAddress(scratch)");
    addr[dev] = ptr;
  }
  *out = static_cast<unsigned char*>(addr[dev]);
  return B200_OK;
}
}  // namespace

extern "C" {

b200_status attention_fwd_noalloc(const void* q, const void* k, const void* v, void* o, int B,
                                  int Hq, int Hkv, int Sq, int Skv, int D, int causal,
                                  float softmax_scale, int nsplit, b200_stream_t stream) {
  AttnShape s;
  b200_status st = check_attention_args(q, k, v, o, B, Hq, Hkv, Sq, Skv, D, causal,
                                        softmax_scale, &s);
  if (st != B200_OK) return st;
  if (nsplit < 0 || nsplit > 8)
    return fail(B200_EINVAL, "attention_fwd_noalloc: nsplit must be 0..8; got %d", nsplit);
  unsigned char* base = nullptr;
  if ((st = noalloc_scratch(&base)) != B200_OK) return st;
  const FixedScratch f{nsplit, reinterpret_cast<float*>(base),
                       reinterpret_cast<float2*>(base + kNoAllocOBytes),
                       reinterpret_cast<unsigned*>(base + kNoAllocOBytes + kNoAllocMlBytes),
                       kNoAllocUnits, kNoAllocQTiles};
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  return D == 128 ? launch_attention<128, kDefaultEmuD128>(q, k, v, o, s, cs, TraceArgs{}, &f)
                  : launch_attention<64, kDefaultEmuD64>(q, k, v, o, s, cs, TraceArgs{}, &f);
}

b200_status attention_fwd_trace(const void* q, const void* k, const void* v, void* o, int B,
                                int Hq, int Hkv, int Sq, int Skv, int D, int causal,
                                float softmax_scale, unsigned long long* trace, int trace_cap,
                                int trace_cta, b200_stream_t stream) {
  AttnShape s;
  b200_status st = check_attention_args(q, k, v, o, B, Hq, Hkv, Sq, Skv, D, causal,
                                        softmax_scale, &s);
  if (st != B200_OK) return st;
  if (!trace || trace_cap < 1 || trace_cta < 0)
    return fail(B200_EINVAL, "attention_fwd_trace: need a trace buffer, cap >= 1, cta >= 0");
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  const TraceArgs tr{trace, trace_cap, trace_cta};
  return D == 128 ? launch_attention<128, kDefaultEmuD128, true>(q, k, v, o, s, cs, tr)
                  : launch_attention<64, kDefaultEmuD64, true>(q, k, v, o, s, cs, tr);
}

b200_status attention_fwd_scalar(const void* q, const void* k, const void* v, void* o, int B,
                                 int Hq, int Hkv, int Sq, int Skv, int D, int causal,
                                 float softmax_scale, b200_stream_t stream) {
  AttnShape s;
  b200_status st = check_attention_args(q, k, v, o, B, Hq, Hkv, Sq, Skv, D, causal,
                                        softmax_scale, &s);
  if (st != B200_OK) return st;
  if (static_cast<long long>(B) * Hq > 65535)
    return fail(B200_EUNSUPPORTED, "attention_fwd_scalar: B*Hq must be <= 65535");
  b200::ref::ScalarParams p{};
  p.q = static_cast<const uint16_t*>(q);
  p.k = static_cast<const uint16_t*>(k);
  p.v = static_cast<const uint16_t*>(v);
  p.o = static_cast<uint16_t*>(o);
  p.B = B;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.Sq = Sq;
  p.Skv = Skv;
  p.group = Hq / Hkv;
  p.causal = s.causal;
  p.scale = s.scale;
  const dim3 grid((Sq + 3) / 4, B * Hq);
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  if (D == 128)
    b200::ref::attention_scalar_kernel<128><<<grid, 128, 0, cs>>>(p);
  else
    b200::ref::attention_scalar_kernel<64><<<grid, 128, 0, cs>>>(p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "attention_fwd_scalar launch");
  return B200_OK;
}

b200_status b200_fill_normal_bf16(void* dst, uint64_t n, uint64_t seed, uint32_t tensor_id,
                                  uint64_t index_base, float mean, float sigma,
                                  b200_stream_t stream) {
  if (n == 0) return B200_OK;
  if (!dst) return fail(B200_EINVAL, "fill: null pointer");
  const uint64_t key = b200::ref::stream_key(seed, tensor_id);
  const unsigned blocks = static_cast<unsigned>(std::min<uint64_t>((n + 255) / 256, 148 * 32));
  b200::ref::fill_normal_bf16_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<uint16_t*>(dst), n, key, index_base, mean, sigma);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "fill_normal launch");
  return B200_OK;
}

b200_status b200_fill_uniform_bf16(void* dst, uint64_t n, uint64_t seed, uint32_t tensor_id,
                                   uint64_t index_base, float lo, float hi,
                                   b200_stream_t stream) {
  if (n == 0) return B200_OK;
  if (!dst) return fail(B200_EINVAL, "fill: null pointer");
  const uint64_t key = b200::ref::stream_key(seed, tensor_id);
  const unsigned blocks = static_cast<unsigned>(std::min<uint64_t>((n + 255) / 256, 148 * 32));
  b200::ref::fill_uniform_bf16_kernel<<<blocks, 256, 0,
                                        reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<uint16_t*>(dst), n, key, index_base, lo, hi);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "fill_uniform launch");
  return B200_OK;
}

b200_status b200_check(b200_stream_t stream) {
  cudaError_t e = cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  uint32_t status = 0;
  e = cudaMemcpyFromSymbol(&status, b200::g_status, sizeof(status));
  if (e != cudaSuccess) return cuda_fail(e, "read status word");
  if (status != 0) {
    const uint32_t zero = 0;
    e = cudaMemcpyToSymbol(b200::g_status, &zero, sizeof(zero));
    if (e != cudaSuccess) return cuda_fail(e, "clear status word");
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) reset_split_counters(dev);
    const uint32_t site = (status >> 8) & 0xffu;
    if (site == b200::attn::kSiteSmemLayout)
      return fail(B200_ECUDA, "attention kernel: dynamic shared memory starts too far past a "
                  "1024-byte boundary for its tile layout (status 0x%08x)", status);
    return fail(B200_ETIMEOUT, "device wait timed out (status 0x%08x, site %u)", status, site);
  }
  return B200_OK;
}

}  // extern "C"

namespace {
__global__ void selftest_wait_kernel(uint64_t limit_ns) {
  __shared__ uint64_t bar;
  b200::mbar_init(&bar, 1);
  b200::fence_mbar_init();
  // Nothing ever arrives: the bounded wait must give up and report.
  (void)b200::mbar_wait(&bar, 0, 0xEE, limit_ns);
}
}  // namespace

namespace {
// Evaluates the softmax's two exp2 paths elementwise: the FMA-pipe polynomial
// (exp2_fma_x2, in pairs) and MUFU ex2.approx.ftz.
__global__ void selftest_exp2_kernel(const float* x, float* y_fma, float* y_mufu, uint64_t n) {
  const uint64_t i = 2 * (blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x);
  if (i >= n) return;
  const float x0 = x[i];
  const float x1 = i + 1 < n ? x[i + 1] : 0.0f;
  float y0, y1;
  b200::exp2_fma_x2(x0, x1, y0, y1);
  y_fma[i] = y0;
  y_mufu[i] = b200::ex2_approx(x0);
  if (i + 1 < n) {
    y_fma[i + 1] = y1;
    y_mufu[i + 1] = b200::ex2_approx(x1);
  }
}
}  // namespace

extern "C" b200_status b200_selftest_exp2(const float* x, float* y_fma, float* y_mufu,
                                          uint64_t n, b200_stream_t stream) {
  if (n == 0) return B200_OK;
  if (!x || !y_fma || !y_mufu) return fail(B200_EINVAL, "b200_selftest_exp2: null pointer");
  const uint64_t blocks = (n + 511) / 512;
  if (blocks > 0x7fffffffull) return fail(B200_EUNSUPPORTED, "b200_selftest_exp2: n too large");
  selftest_exp2_kernel<<<static_cast<unsigned>(blocks), 256, 0,
                         reinterpret_cast<cudaStream_t>(stream)>>>(x, y_fma, y_mufu, n);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "b200_selftest_exp2 launch");
  return B200_OK;
}

extern "C" b200_status b200_selftest_wait_timeout(uint64_t limit_ns, b200_stream_t stream) {
  if (limit_ns < 1000) limit_ns = 1000;
  if (limit_ns > 100000000ull) limit_ns = 100000000ull;
  selftest_wait_kernel<<<1, 1, 0, reinterpret_cast<cudaStream_t>(stream)>>>(limit_ns);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "selftest launch");
  return B200_OK;
}

namespace {

b200::gemm::Params gemm_params(int M, int N, int K, int b_col_major, int bm, int bn, int bk) {
  b200::gemm::Params p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.tiles_m = (M + bm - 1) / bm;
  p.tiles_n = (N + bn - 1) / bn;
  p.k_blocks = (K + bk - 1) / bk;
  p.b_col_major = b_col_major ? 1 : 0;
  return p;
}

// Raster group (256-row blocks per group), measured on B200 (B [K,N]): groups
// of 8 are best at 8192^3 (16 costs 0.4 %), groups of 16 at 16384^3 (+2 %
// over 8; groups of 4 or 32 read 30-50 % more from DRAM).
int gemm_default_group(int K) { return K >= 12288 ? 16 : 8; }

// Clusters of two that can be resident at once on the current device.
int pair_clusters_resident() {
  static std::mutex mu;
  static std::map<int, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(dev);
  if (it != cache.end()) return it->second;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(2 * (sm_count() / 2), 1, 1);
  cfg.blockDim = dim3(b200::gemm::pair::kThreads, 1, 1);
  cfg.dynamicSmemBytes = b200::gemm::pair::kSmemBytes;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, b200::gemm::gemm_bf16_pair_kernel, &cfg) !=
          cudaSuccess ||
      n < 1) {
    cudaGetLastError();
    n = sm_count() / 2;
  }
  cache[dev] = n;
  return n;
}

b200_status launch_gemm_pair(const void* A, const void* Bm, void* C, int M, int N, int K,
                             int b_col_major, cudaStream_t stream) {
  namespace g = b200::gemm;
  static unsigned attr_done = 0;
  b200_status st = ensure_smem_attr(g::gemm_bf16_pair_kernel, g::pair::kSmemBytes, &attr_done);
  if (st != B200_OK) return st;
  CUtensorMap am, bm;
  // Each CTA of a pair loads 128-row halves of the 256-row A and B tiles.
  if ((st = encode_bf16_2d(&am, A, K, M, g::pair::kBK, g::pair::kHalf)) != B200_OK) return st;
  if (b_col_major)
    st = encode_bf16_2d(&bm, Bm, K, N, g::pair::kBK, g::pair::kHalf);
  else
    st = encode_bf16_2d(&bm, Bm, N, K, 64, g::pair::kBK);
  if (st != B200_OK) return st;
  CUtensorMap cm;  // C [M, N]: 64-column x 128-row boxes, the epilogue's staging unit
  if ((st = encode_bf16_2d(&cm, C, N, M, g::pair::kCBoxCols, g::pair::kHalf)) != B200_OK)
    return st;
  g::Params p = gemm_params(M, N, K, b_col_major, g::pair::kBM, g::pair::kBN, g::pair::kBK);
  p.group_m = gemm_default_group(K);
  const long long tiles = static_cast<long long>(p.tiles_m) * p.tiles_n;
  if (tiles > 0x3fffffffll) return fail(B200_EUNSUPPORTED, "gemm_bf16: too many tiles");
  const long long clusters = std::min<long long>(tiles, pair_clusters_resident());
  g::gemm_bf16_pair_kernel<<<static_cast<unsigned>(2 * clusters), g::pair::kThreads,
                             g::pair::kSmemBytes, stream>>>(am, bm, cm, p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "gemm_bf16 (pair) launch");
  return B200_OK;
}

}  // namespace

extern "C" b200_status gemm_bf16(const void* A, const void* Bm, void* C, int M, int N, int K,
                                 int b_col_major, b200_stream_t stream) {
  const b200_status st = check_gemm_args(A, Bm, C, M, N, K, "gemm_bf16");
  if (st != B200_OK) return st;
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  return launch_gemm_pair(A, Bm, C, M, N, K, b_col_major, s);
}

extern "C" b200_status gemm_bf16_cublas(const void* A, const void* Bm, void* C, int M, int N,
                                        int K, int b_col_major, b200_stream_t stream) {
  b200_status st = check_gemm_args(A, Bm, C, M, N, K, "gemm_bf16_cublas");
  if (st != B200_OK) return st;
  cublasHandle_t h = cublas_handle(&st);
  if (!h) return st;
  if (cublasSetStream(h, reinterpret_cast<cudaStream_t>(stream)) != CUBLAS_STATUS_SUCCESS)
    return fail(B200_ECUDA, "cublasSetStream failed");
  // Row-major C = A B is column-major C^T = B^T A^T: cuBLAS sees A as a
  // column-major K x M matrix (op N) and B as K x N column-major if it is
  // stored [N,K] (op T), or N x K column-major if stored [K,N] (op N).
  const float alpha = 1.0f, beta = 0.0f;
  const cublasStatus_t r = cublasGemmEx(
      h, b_col_major ? CUBLAS_OP_T : CUBLAS_OP_N, CUBLAS_OP_N, N, M, K, &alpha, Bm, CUDA_R_16BF,
      b_col_major ? K : N, A, CUDA_R_16BF, K, &beta, C, CUDA_R_16BF, N, CUBLAS_COMPUTE_32F,
      CUBLAS_GEMM_DEFAULT);
  if (r != CUBLAS_STATUS_SUCCESS) return fail(B200_ECUDA, "cublasGemmEx failed (%d)", (int)r);
  return B200_OK;
}

namespace {
__global__ void fill_cublas_pattern_kernel(void* dst, uint64_t n, int mode, float scale) {
  const uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x;
  if (i >= n) return;
  const float v = (static_cast<float>(i % 251) - 125.0f) * scale;
  if (mode == B200_CUBLAS_FP16)
    static_cast<__half*>(dst)[i] = __float2half_rn(v);
  else if (mode == B200_CUBLAS_BF16)
    static_cast<__nv_bfloat16*>(dst)[i] = __float2bfloat16_rn(v);
  else
    static_cast<float*>(dst)[i] = v;
}
}  // namespace

extern "C" b200_status b200_fill_cublas_pattern(void* dst, uint64_t n, int mode, float scale,
                                                b200_stream_t stream) {
  if (mode < B200_CUBLAS_FP16 || mode > B200_CUBLAS_FP32)
    return fail(B200_EINVAL, "b200_fill_cublas_pattern: unknown mode %d", mode);
  if (n == 0) return B200_OK;
  if (!dst) return fail(B200_EINVAL, "b200_fill_cublas_pattern: null pointer");
  const uint64_t blocks = (n + 255) / 256;
  if (blocks > 0x7fffffffull) return fail(B200_EUNSUPPORTED, "b200_fill_cublas_pattern: too big");
  fill_cublas_pattern_kernel<<<static_cast<unsigned>(blocks), 256, 0,
                               reinterpret_cast<cudaStream_t>(stream)>>>(dst, n, mode, scale);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "b200_fill_cublas_pattern launch");
  return B200_OK;
}

extern "C" b200_status gemm_cublas_mode(const void* A, const void* Bm, void* C, int M, int N,
                                        int K, int mode, b200_stream_t stream) {
  if (!A || !Bm || !C) return fail(B200_EINVAL, "gemm_cublas_mode: null matrix pointer");
  if (M < 1 || N < 1 || K < 1) return fail(B200_EINVAL, "gemm_cublas_mode: invalid shape");
  cudaDataType_t type;
  cublasComputeType_t compute;
  cublasGemmAlgo_t algo = CUBLAS_GEMM_DEFAULT_TENSOR_OP;
  switch (mode) {
    case B200_CUBLAS_FP16: type = CUDA_R_16F; compute = CUBLAS_COMPUTE_32F; break;
    case B200_CUBLAS_BF16: type = CUDA_R_16BF; compute = CUBLAS_COMPUTE_32F; break;
    case B200_CUBLAS_TF32: type = CUDA_R_32F; compute = CUBLAS_COMPUTE_32F_FAST_TF32; break;
    case B200_CUBLAS_FP32:
      type = CUDA_R_32F;
      compute = CUBLAS_COMPUTE_32F_PEDANTIC;
      algo = CUBLAS_GEMM_DEFAULT;
      break;
    default: return fail(B200_EINVAL, "gemm_cublas_mode: unknown mode %d", mode);
  }
  b200_status st = B200_OK;
  cublasHandle_t h = cublas_handle(&st);
  if (!h) return st;
  if (cublasSetStream(h, reinterpret_cast<cudaStream_t>(stream)) != CUBLAS_STATUS_SUCCESS)
    return fail(B200_ECUDA, "cublasSetStream failed");
  const float alpha = 1.0f, beta = 0.0f;
  const cublasStatus_t r = cublasGemmEx(h, CUBLAS_OP_N, CUBLAS_OP_N, M, N, K, &alpha, A, type, M,
                                        Bm, type, K, &beta, C, type, M, compute, algo);
  if (r != CUBLAS_STATUS_SUCCESS) return fail(B200_ECUDA, "cublasGemmEx failed (%d)", (int)r);
  return B200_OK;
}

extern "C" b200_status gemm_f32_reference(const void* A, const void* Bm, void* C, int M, int N,
                                          int K, int b_col_major, b200_stream_t stream) {
  if (!A || !Bm || !C) return fail(B200_EINVAL, "gemm_f32_reference: null matrix pointer");
  if (M < 1 || N < 1 || K < 1) return fail(B200_EINVAL, "gemm_f32_reference: invalid shape");
  const dim3 grid((N + 63) / 64, (M + 63) / 64);
  b200::ref::gemm_f32_reference_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(A), static_cast<const uint16_t*>(Bm), static_cast<float*>(C),
      M, N, K, b_col_major);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "gemm_f32_reference launch");
  return B200_OK;
}
