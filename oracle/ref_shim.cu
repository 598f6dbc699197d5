// Builds the REFERENCE's own CPU attention into oracle/_ref/libref_attention.so
// -- TEST INFRASTRUCTURE ONLY.
//
// The reference keeps its CPU reference attention, bf16 helpers and pattern
// fillers as host functions inside 0.attention/main.cu (anonymous namespace,
// same translation unit as its main()).  This file compiles that source where
// it lies (the Makefile passes the reference root with -I) with main renamed,
// and exports thin C wrappers so the restatement in attention_ref.cpp can be
// checked bit for bit against the reference's own code.  Nothing here is
// copied from the reference; no reference kernel is launched.
#define main b200_reference_attention_main
#include "0.attention/main.cu"
#undef main

#include <cstring>

extern "C" {

// build_real_attention_reference (0.attention/main.cu:1333-1388).
void ref_attention_f32(const uint16_t* q, const uint16_t* k, const uint16_t* v, int B, int Hq,
                       int Hkv, int Sq, int Skv, int D, float softmax_scale, int causal,
                       float* out) {
  const size_t nq = static_cast<size_t>(B) * Hq * Sq * D;
  const size_t nkv = static_cast<size_t>(B) * Hkv * Skv * D;
  std::vector<uint16_t> hq(q, q + nq), hk(k, k + nkv), hv(v, v + nkv);
  std::vector<float> ref;
  build_real_attention_reference(hq, hk, hv, B, Hq, Hkv, Sq, Skv, D, softmax_scale, causal != 0,
                                 &ref);
  std::memcpy(out, ref.data(), ref.size() * sizeof(float));
}

// fill_real_bf16_matrix (0.attention/main.cu:1308-1325).
void ref_fill_pattern_bf16(uint16_t* dst, const char* pattern, char matrix, int B, int H, int S,
                           int D) {
  std::vector<uint16_t> buf(static_cast<size_t>(B) * H * S * D);
  fill_real_bf16_matrix(buf, std::string(pattern), matrix, B, H, S, D);
  std::memcpy(dst, buf.data(), buf.size() * sizeof(uint16_t));
}

// validation_checksum_bytes (0.attention/main.cu:1511-1519).
uint64_t ref_fnv1a64(const void* data, size_t bytes) {
  return validation_checksum_bytes(data, bytes);
}

}  // extern "C"
