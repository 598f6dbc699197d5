/*
 * CPU oracle -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain C++ restatement of the reference's CPU arithmetic for the hot path.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may call
 * it, and only as the checker or the timed CPU baseline.  The product path
 * (libb200attn.so) never links or calls it.
 *
 * Pinned against the reference itself: oracle/ref_shim.cu compiles the
 * reference's own build_real_attention_reference (0.attention/main.cu:1333-1388)
 * into oracle/_ref/, tests/golden/make_golden.py records its outputs as
 * FNV-1a fingerprints, and tests/test_oracle.py requires this restatement to
 * reproduce them bit for bit.
 */
#ifndef B200_ORACLE_H
#define B200_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* fp32 attention, restating 0.attention/main.cu:1333-1388.
 * q: [B,Hq,Sq,D] bf16 bits, k/v: [B,Hkv,Skv,D], out: [B,Hq,Sq,D] fp32.
 * Work is split over (b, hq) heads on `threads` threads (<= 0: all cores);
 * the arithmetic of each row is identical for every thread count. */
void oracle_attention_f32(const uint16_t* q, const uint16_t* k, const uint16_t* v, int B, int Hq,
                          int Hkv, int Sq, int Skv, int D, float softmax_scale, int causal,
                          float* out, int threads);

/* Same, for query rows [q_begin, q_end) of heads [h_begin, h_end) of batch b
 * only; out receives (h_end-h_begin) * (q_end-q_begin) * D floats.  Used to
 * check full-size tensors on a sample. */
void oracle_attention_rows_f32(const uint16_t* q, const uint16_t* k, const uint16_t* v, int B,
                               int Hq, int Hkv, int Sq, int Skv, int D, float softmax_scale,
                               int causal, int b, int h_begin, int h_end, int q_begin, int q_end,
                               float* out, int threads);

/* Deterministic validation patterns of the harness, restating
 * 0.attention/main.cu:1266-1325: "constant", "onehot", "rank1", else hash
 * "random".  matrix is 'q', 'k' or 'v'.  dst: [B,H,S,D] bf16 bits (RNE). */
void oracle_fill_pattern_bf16(uint16_t* dst, const char* pattern, char matrix, int B, int H, int S,
                              int D);

/* fp32 -> bf16 bits, round to nearest even (0.attention/main.cu:1159-1165). */
uint16_t oracle_f32_to_bf16(float x);

/* GEMM reference restating 5.GEMM/gemm256_tma_tcgen05_bench.cu:1115-1137:
 * double accumulation of bf16 inputs in k order.  A: [M,K] row-major;
 * B: [N,K] if b_col_major else [K,N].  Rows [row_begin, row_end) of C are
 * written to out ((row_end-row_begin) x N doubles). */
void oracle_gemm_f64(const uint16_t* A, const uint16_t* Bm, int M, int N, int K, int b_col_major,
                     int row_begin, int row_end, double* out, int threads);

/* GEMM validation fills, restating 5.GEMM/gemm256_tma_tcgen05_bench.cu:1013-1023
 * ("pattern" or "ones"); which = 'a' ([rows,cols] = [M,K]) or 'b' ([K,N]). */
void oracle_gemm_fill_bf16(uint16_t* dst, char which, const char* pattern, int rows, int cols);

/* FNV-1a 64-bit over raw bytes (0.attention/main.cu:1511-1519). */
uint64_t oracle_fnv1a64(const void* data, size_t bytes);

#ifdef __cplusplus
}
#endif

#endif /* B200_ORACLE_H */
