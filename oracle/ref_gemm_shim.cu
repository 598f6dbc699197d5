// Builds the REFERENCE's own GEMM validation fills into
// oracle/_ref/libref_gemm.so -- TEST INFRASTRUCTURE ONLY.
//
// validation_a_value / validation_b_value and the bf16 rounding live as host
// functions inside 5.GEMM/gemm256_tma_tcgen05_bench.cu (anonymous namespace,
// same translation unit as its main()).  This file compiles that source where
// it lies (reference root passed with -I) with main renamed and exports a C
// wrapper, so oracle_gemm_fill_bf16 can be checked bit for bit.
#define main b200_reference_gemm_main
#include "5.GEMM/gemm256_tma_tcgen05_bench.cu"
#undef main

extern "C" void ref_gemm_fill_bf16(uint16_t* dst, char which, const char* pattern, int rows,
                                   int cols) {
  const bool ones = std::strcmp(pattern, "ones") == 0;
  for (int r = 0; r < rows; ++r)
    for (int c = 0; c < cols; ++c) {
      const float value =
          which == 'a' ? validation_a_value(ones, r, c) : validation_b_value(ones, r, c);
      dst[static_cast<size_t>(r) * cols + c] = float_to_bf16_bits_host(value);
    }
}
