// CPU oracle -- TEST INFRASTRUCTURE ONLY (see oracle.h).  Never part of the
// product path.
//
// Restates, operation for operation, the reference harness's CPU attention
// build_real_attention_reference (0.attention/main.cu:1333-1388) and its input
// patterns (0.attention/main.cu:1266-1325).  Two changes that cannot alter a
// single bit of the result, only its speed:
//   * exp(score - max) is evaluated once per key and reused for the
//     denominator and for every head dim (the reference re-evaluates the same
//     expression inside its d loop; std::exp is a pure function);
//   * the PV loop runs keys outer / dims inner; each output element still
//     accumulates its terms in ascending key order.
// Heads are processed in parallel; each row's arithmetic is independent of
// the thread count.  Compile without -ffast-math and without FMA contraction
// into wider targets (plain -O2 on x86-64), as the reference's host code is.
#include "oracle.h"

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <limits>
#include <string>
#include <thread>
#include <vector>

namespace {

float bf16_to_f32(uint16_t bits) {
  const uint32_t w = static_cast<uint32_t>(bits) << 16;
  float f;
  std::memcpy(&f, &w, sizeof(f));
  return f;
}

// Bottom-right aligned causal visibility (0.attention/attention.cu:167-174).
bool key_visible(int q_idx, int k_idx, int sq, int skv, int causal) {
  if (!causal) return true;
  return k_idx <= q_idx + (skv - sq);
}

// GQA head map (0.attention/attention.cu:176-183).
int kv_head_for(int hq, int hq_count, int hkv_count) {
  if (hkv_count <= 1) return 0;
  if (hkv_count == hq_count) return hq;
  const int group = hq_count / hkv_count;
  const int mapped = group > 0 ? hq / group : 0;
  return mapped < hkv_count ? mapped : hkv_count - 1;
}

int resolve_threads(int threads) {
  if (threads > 0) return threads;
  const unsigned hc = std::thread::hardware_concurrency();
  return hc == 0 ? 1 : static_cast<int>(hc);
}

template <typename Fn>
void parallel_for(int count, int threads, Fn fn) {
  threads = std::max(1, std::min(resolve_threads(threads), count));
  if (threads == 1) {
    for (int i = 0; i < count; ++i) fn(i);
    return;
  }
  std::atomic<int> next{0};
  std::vector<std::thread> pool;
  pool.reserve(threads);
  for (int t = 0; t < threads; ++t) {
    pool.emplace_back([&] {
      for (int i = next.fetch_add(1); i < count; i = next.fetch_add(1)) fn(i);
    });
  }
  for (auto& th : pool) th.join();
}

// One (b, hq) head, query rows [q_begin, q_end).  Output rows are written to
// out[(q - q_begin) * D + d].
void attention_head_rows(const uint16_t* q, const uint16_t* k, const uint16_t* v, int Hq,
                         int Hkv, int Sq, int Skv, int D, float scale, int causal, int b, int hq,
                         int q_begin, int q_end, float* out) {
  const int hkv = kv_head_for(hq, Hq, Hkv);
  const size_t kv_base = (static_cast<size_t>(b) * Hkv + hkv) * static_cast<size_t>(Skv) * D;
  std::vector<float> kf(static_cast<size_t>(Skv) * D), vf(static_cast<size_t>(Skv) * D);
  for (size_t i = 0; i < kf.size(); ++i) {
    kf[i] = bf16_to_f32(k[kv_base + i]);
    vf[i] = bf16_to_f32(v[kv_base + i]);
  }
  std::vector<float> qf(D), scores(Skv), w(Skv), acc(D);
  const float neg_inf = -std::numeric_limits<float>::infinity();
  for (int q_idx = q_begin; q_idx < q_end; ++q_idx) {
    float* orow = out + static_cast<size_t>(q_idx - q_begin) * D;
    std::fill(orow, orow + D, 0.0f);
    const size_t q_base = ((static_cast<size_t>(b) * Hq + hq) * Sq + q_idx) * D;
    for (int d = 0; d < D; ++d) qf[d] = bf16_to_f32(q[q_base + d]);
    float row_max = neg_inf;
    for (int k_idx = 0; k_idx < Skv; ++k_idx) {
      if (!key_visible(q_idx, k_idx, Sq, Skv, causal)) {
        scores[k_idx] = neg_inf;
        continue;
      }
      const float* kr = &kf[static_cast<size_t>(k_idx) * D];
      float dot = 0.0f;
      for (int d = 0; d < D; ++d) dot += qf[d] * kr[d];
      const float score = dot * scale;
      scores[k_idx] = score;
      row_max = std::max(row_max, score);
    }
    if (!std::isfinite(row_max)) continue;
    float denom = 0.0f;
    for (int k_idx = 0; k_idx < Skv; ++k_idx) {
      if (!std::isfinite(scores[k_idx])) continue;
      w[k_idx] = std::exp(scores[k_idx] - row_max);
      denom += w[k_idx];
    }
    std::fill(acc.begin(), acc.end(), 0.0f);
    for (int k_idx = 0; k_idx < Skv; ++k_idx) {
      if (!std::isfinite(scores[k_idx])) continue;
      const float wk = w[k_idx];
      const float* vr = &vf[static_cast<size_t>(k_idx) * D];
      for (int d = 0; d < D; ++d) acc[d] += wk * vr[d];
    }
    for (int d = 0; d < D; ++d) orow[d] = denom > 0.0f ? acc[d] / denom : 0.0f;
  }
}

uint32_t mix_hash_u32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return x;
}

float centered_hash_value(uint32_t x) {
  const uint32_t h = mix_hash_u32(x);
  const float u = static_cast<float>(h & 0xffffu) * (1.0f / 65535.0f);
  return u * 2.0f - 1.0f;
}

float pattern_value(const std::string& pattern, char matrix, int b, int h, int s, int d) {
  if (pattern == "constant") return matrix == 'v' ? 0.125f : 0.0625f;
  if (pattern == "onehot") {
    if (matrix == 'q' || matrix == 'k') return d == (s & 127) ? 1.0f : 0.0f;
    return d == ((s + h) & 127) ? 0.5f : 0.0f;
  }
  if (pattern == "rank1") {
    const float s_scale = static_cast<float>((s % 17) + 1) * 0.0078125f;
    const float d_scale = static_cast<float>((d % 19) + 1) * 0.00390625f;
    const float h_scale = static_cast<float>((h % 7) + 1) * 0.0009765625f;
    if (matrix == 'v') return 0.5f * s_scale + d_scale + h_scale;
    return s_scale + d_scale + h_scale;
  }
  const uint32_t tag = matrix == 'q' ? 0x1234u : (matrix == 'k' ? 0x5678u : 0x9abcu);
  const uint32_t idx = static_cast<uint32_t>(b) * 131071u + static_cast<uint32_t>(h) * 8191u +
                       static_cast<uint32_t>(s) * 257u + static_cast<uint32_t>(d);
  const float amp = matrix == 'v' ? 0.5f : 0.25f;
  return amp * centered_hash_value(tag ^ idx);
}

}  // namespace

extern "C" {

uint16_t oracle_f32_to_bf16(float value) {
  uint32_t bits;
  std::memcpy(&bits, &value, sizeof(bits));
  const uint32_t lsb = (bits >> 16) & 1u;
  bits += 0x7fffu + lsb;
  return static_cast<uint16_t>(bits >> 16);
}

void oracle_attention_f32(const uint16_t* q, const uint16_t* k, const uint16_t* v, int B, int Hq,
                          int Hkv, int Sq, int Skv, int D, float softmax_scale, int causal,
                          float* out, int threads) {
  parallel_for(B * Hq, threads, [&](int bh) {
    const int b = bh / Hq, hq = bh % Hq;
    attention_head_rows(q, k, v, Hq, Hkv, Sq, Skv, D, softmax_scale, causal, b, hq, 0, Sq,
                        out + static_cast<size_t>(bh) * Sq * D);
  });
}

void oracle_attention_rows_f32(const uint16_t* q, const uint16_t* k, const uint16_t* v, int B,
                               int Hq, int Hkv, int Sq, int Skv, int D, float softmax_scale,
                               int causal, int b, int h_begin, int h_end, int q_begin, int q_end,
                               float* out, int threads) {
  (void)B;
  const int heads = h_end - h_begin;
  const int rows = q_end - q_begin;
  if (heads <= 0 || rows <= 0) return;
  // Split each head's rows into chunks so a few heads still use every core.
  const int chunk = std::max(1, rows / std::max(1, resolve_threads(threads) / heads + 1));
  const int chunks = (rows + chunk - 1) / chunk;
  parallel_for(heads * chunks, threads, [&](int task) {
    const int hh = task / chunks, c = task % chunks;
    const int r0 = q_begin + c * chunk, r1 = std::min(q_end, r0 + chunk);
    attention_head_rows(q, k, v, Hq, Hkv, Sq, Skv, D, softmax_scale, causal, b, h_begin + hh,
                        r0, r1,
                        out + (static_cast<size_t>(hh) * rows + (r0 - q_begin)) * D);
  });
}

void oracle_fill_pattern_bf16(uint16_t* dst, const char* pattern, char matrix, int B, int H, int S,
                              int D) {
  const std::string pat(pattern);
  for (int b = 0; b < B; ++b)
    for (int h = 0; h < H; ++h)
      for (int s = 0; s < S; ++s)
        for (int d = 0; d < D; ++d) {
          const size_t idx = ((static_cast<size_t>(b) * H + h) * S + s) * D + d;
          dst[idx] = oracle_f32_to_bf16(pattern_value(pat, matrix, b, h, s, d));
        }
}

uint64_t oracle_fnv1a64(const void* data, size_t bytes) {
  const uint8_t* p = static_cast<const uint8_t*>(data);
  uint64_t hash = 1469598103934665603ull;
  for (size_t i = 0; i < bytes; ++i) {
    hash ^= static_cast<uint64_t>(p[i]);
    hash *= 1099511628211ull;
  }
  return hash;
}

}  // extern "C"
