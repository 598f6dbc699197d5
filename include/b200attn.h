/*
 * b200attn -- C ABI of the sm_100a fused attention forward and bf16 GEMM.
 *
 * The reference (rhrnald/benchmark) has no library boundary: its harness
 * launches kernels directly.  Each entry point below replaces one such launch
 * site; the citation after it names the reference code it stands in for
 * (paths relative to the reference project root).
 *
 * Conventions
 *   - All tensor pointers are device pointers owned by the caller, 16-byte
 *     aligned, contiguous.
 *   - attention_fwd splits the K/V range of short problems (too few 128-row
 *     Q tiles to fill the GPU, K/V ranges of 48 or more 128-key tiles) among
 *     several CTAs that merge through a workspace.  The workspace belongs to
 *     the library, one per (device, stream); the first such call on a
 *     (device, stream) allocates it (cudaMalloc, which synchronises the
 *     device) and later calls reuse it, growing it when a larger problem
 *     needs more.  Nothing else allocates.
 *   - bf16 tensors are passed as raw 16-bit words (uint16_t storage).
 *   - Calls are asynchronous on `stream` (NULL = legacy default stream) and
 *     use the calling thread's current CUDA device.
 *   - TMA tensor maps are encoded on the first call for a (pointer, shape)
 *     and kept in a fixed-size table, so repeated calls on the same buffers
 *     skip the driver encode.
 *   - Errors are returned as b200_status, never by exit(); a message for the
 *     most recent failure on the calling thread is in b200_last_error().
 *   - Device-side waits are bounded.  A kernel whose pipeline wait runs out
 *     records it in a per-device status word; b200_check() synchronises the
 *     stream, reports B200_ETIMEOUT and clears the word.  While the word is
 *     set, later kernels on that device abandon their work early.
 */
#ifndef B200ATTN_H
#define B200ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same object as cudaStream_t; spelled out so C callers need no CUDA headers. */
typedef struct CUstream_st* b200_stream_t;

typedef enum {
  B200_OK = 0,
  B200_EINVAL = 1,       /* bad argument: null/misaligned pointer, bad shape */
  B200_EUNSUPPORTED = 2, /* valid request this build does not implement */
  B200_ECUDA = 3,        /* CUDA runtime / driver error */
  B200_ETIMEOUT = 4      /* a device-side bounded wait ran out */
} b200_status;

/*
 * Fused attention forward: O = softmax(Q K^T * scale) V, bf16 in / bf16 out,
 * fp32 accumulation and softmax.
 *   q, o : [B, Hq,  Sq,  D]      k, v : [B, Hkv, Skv, D]
 *   D in {64, 128}; Hq % Hkv == 0 (query head h reads kv head h / (Hq/Hkv));
 *   causal != 0: key j is visible to query i iff j <= i + (Skv - Sq)
 *   (bottom-right aligned); rows with no visible key produce zeros.
 *   softmax_scale < 0 selects 1/sqrt(D).
 * Replaces the launch of qk_tma_mma_ld_kernel in 0.attention/main.cu:521-569
 * (benchmark) and 0.attention/main.cu:1901-1911 (fused validation); accepts
 * every shape the scalar path accepts (0.attention/main.cu:1706-1721) plus D=64.
 * Non-causal D=128 problems with a pair of Q tiles per two SMs run on
 * clusters of two CTAs (tcgen05 cta_group::2); the results are the same bits.
 */
b200_status attention_fwd(const void* q, const void* k, const void* v, void* o, int B, int Hq,
                          int Hkv, int Sq, int Skv, int D, int causal, float softmax_scale,
                          b200_stream_t stream);

/*
 * attention_fwd for callers that cannot allocate device memory: it runs the
 * same kernel, but when it splits a short problem's K/V range among several
 * CTAs their partial results meet in a fixed scratch array compiled into
 * this library instead of a workspace allocated with cudaMalloc.  Meant for
 * plugin hosts that own all device memory through their own pool and
 * forbid other allocations, and for latency-bound callers that cannot take
 * cudaMalloc's device-wide synchronisation.  The caller still passes every
 * input and output; nothing is allocated.
 *   nsplit: K/V splits per 128-row Q tile, 1..8; 1 uses no scratch (any
 *   size); 0 picks the same split as attention_fwd.
 *   Limit: when splitting, at most 128 split units (Q tiles x nsplit) and
 *   1024 Q tiles per call; larger requests return B200_EUNSUPPORTED with a
 *   message naming the limit.
 *   The scratch (about 8.1 MiB) is held by every GPU that loads the library
 *   until the process exits, and is shared by all calls: calls that overlap
 *   on the GPU (other streams or threads) race and must be serialised by the
 *   caller.  Each call clears the merge counters it uses before its kernel.
 *   The first call on a device looks up the array's device address there
 *   (cudaGetSymbolAddress) and caches it; make that first call before any
 *   stream capture.
 * This entry point has no counterpart in the reference.
 */
b200_status attention_fwd_noalloc(const void* q, const void* k, const void* v, void* o, int B,
                                  int Hq, int Hkv, int Sq, int Skv, int D, int causal,
                                  float softmax_scale, int nsplit, b200_stream_t stream);

/*
 * attention_fwd with clock-cycle tracing of one CTA (diagnostics; runs the
 * default exp2 split).  trace: device buffer of 7 * trace_cap * 2 uint64
 * (zero it first).  Role r (0 Q/K TMA producer, 1 PV MMA issuer, 2 and 3
 * softmax warps 0 and 4, 4 epilogue, 5 V TMA producer, 6 S MMA issuer)
 * writes up to trace_cap records at trace + r*trace_cap*2, each
 * {(event << 32) | (tile << 24) | iteration, clock64()}; the iteration of
 * TMA, MMA and softmax records is the CTA's global K/V tile index (for
 * non-causal d=64 problems, traced on the two-Q-tile kernel that runs them:
 * the S index, with the pipe as the tile field; for problems that run on CTA
 * pairs the MMA issuers of the traced CTA's pair are recorded, which live in
 * its even CTA).  Events
 * are listed in benchmark_b200/trace.py, which also writes the reference's
 * per-iteration trace CSV.  Stands in for the reference's
 * ATTENTION_CLOCK_TRACE build and its per-stage CSV
 * (0.attention/main.cu:175-272, 0.attention/main.cu:808-1157).
 */
b200_status attention_fwd_trace(const void* q, const void* k, const void* v, void* o, int B,
                                int Hq, int Hkv, int Sq, int Skv, int D, int causal,
                                float softmax_scale, unsigned long long* trace, int trace_cap,
                                int trace_cta, b200_stream_t stream);

/*
 * Validation-only CUDA-core attention with the same arguments and semantics
 * (exact two-pass softmax with expf, fp32).  Replaces the launch of
 * real_attention_bf16_d128_kernel in 0.attention/main.cu:1776-1779; also
 * accepts D=64.  Requires B*Hq <= 65535.
 */
b200_status attention_fwd_scalar(const void* q, const void* k, const void* v, void* o, int B,
                                 int Hq, int Hkv, int Sq, int Skv, int D, int causal,
                                 float softmax_scale, b200_stream_t stream);

/*
 * bf16 GEMM: C[M,N] (bf16, row-major) = A[M,K] (row-major) x B, fp32
 * accumulation.  b_col_major = 1: B stored [N,K] (column-major B);
 * b_col_major = 0: B stored [K,N] (row-major, the reference 5.GEMM layout).
 * Requires K % 8 == 0 and N % 8 == 0 (16-byte rows); any M, N, K >= 1.
 * Replaces the launch of gemm256_tma_tcgen05_kernel in
 * 5.GEMM/gemm256_tma_tcgen05_bench.cu:937-956 (benchmark) and :1101-1104
 * (validation), which take only multiples of 256 and write C as fp32 or not
 * at all.
 */
b200_status gemm_bf16(const void* A, const void* B, void* C, int M, int N, int K,
                      int b_col_major, b200_stream_t stream);

/*
 * Comparator: the same product through cublasGemmEx (bf16 in/out, fp32
 * compute).  Stands in for 6.cuBLAS/cublas_gemm_bench.cu:226-231.
 */
b200_status gemm_bf16_cublas(const void* A, const void* B, void* C, int M, int N, int K,
                             int b_col_major, b200_stream_t stream);

/*
 * The reference's cuBLAS benchmark in each of its modes
 * (6.cuBLAS/cublas_gemm_bench.cu:145-166, call :226-231): column-major
 * C[M,N] = A[M,K] B[K,N] with lda = M, ldb = K, ldc = M, no transposes.
 * Element type of A, B and C by mode: fp16 / bf16 (2 bytes, fp32
 * accumulate), tf32 (fp32 storage, TF32 tensor cores), fp32 (CUDA cores,
 * pedantic).  Comparator only: timed, never used on the product path.
 */
typedef enum {
  B200_CUBLAS_FP16 = 0,
  B200_CUBLAS_BF16 = 1,
  B200_CUBLAS_TF32 = 2,
  B200_CUBLAS_FP32 = 3
} b200_cublas_mode;

b200_status gemm_cublas_mode(const void* A, const void* B, void* C, int M, int N, int K,
                             int mode, b200_stream_t stream);

/*
 * The cuBLAS benchmark's input pattern, value i = ((i % 251) - 125) * scale
 * in the mode's element type (6.cuBLAS/cublas_gemm_bench.cu:28-58).
 */
b200_status b200_fill_cublas_pattern(void* dst, uint64_t n, int mode, float scale,
                                     b200_stream_t stream);

/*
 * Validation-only fp32 CUDA-core GEMM: C[M,N] fp32 row-major.  GPU analogue
 * of the reference's double-precision CPU loop
 * (5.GEMM/gemm256_tma_tcgen05_bench.cu:1115-1137) for full-size checks.
 */
b200_status gemm_f32_reference(const void* A, const void* B, void* C, int M, int N, int K,
                               int b_col_major, b200_stream_t stream);

/*
 * Seeded bf16 generators (counter-based: value = f(seed, tensor_id,
 * index_base + i)), so any shard of a tensor can be generated independently.
 * Stand in for the benchmark fill fill_packed_bf16 (0.attention/attention.cu:142-147,
 * launched at 0.attention/main.cu:2068-2075), which has no seed or distribution.
 */
b200_status b200_fill_normal_bf16(void* dst, uint64_t n, uint64_t seed, uint32_t tensor_id,
                                  uint64_t index_base, float mean, float sigma,
                                  b200_stream_t stream);
b200_status b200_fill_uniform_bf16(void* dst, uint64_t n, uint64_t seed, uint32_t tensor_id,
                                   uint64_t index_base, float lo, float hi,
                                   b200_stream_t stream);

/* Synchronise `stream`, then read and clear the device status word.
 * Stands in for the RunResult.status checks of 0.attention/main.cu:541-592. */
b200_status b200_check(b200_stream_t stream);

/* Message for the most recent failure on this thread ("" if none). */
const char* b200_last_error(void);

/* ABI version: major * 10000 + minor * 100 + patch. */
int b200_version(void);

/*
 * Self-test of the bounded-wait machinery: launches one thread that waits on
 * an mbarrier nothing ever arrives at, with the given limit (clamped to
 * [1 us, 100 ms]).  After b200_check() the caller must see B200_ETIMEOUT.
 * No reference counterpart (the reference's waits are unbounded,
 * 0.attention/ptx_wrappers.cuh:195-211).
 */
b200_status b200_selftest_wait_timeout(uint64_t limit_ns, b200_stream_t stream);

/*
 * Self-test of the softmax's two exp2 implementations: for each of the n fp32
 * inputs x[i] (device buffers), y_fma[i] = the FMA-pipe polynomial exp2 and
 * y_mufu[i] = ex2.approx.ftz (MUFU).  The polynomial clamps x to [-126, 126],
 * so it returns 2^-126 below that range and 2^126 above it; inside it its
 * relative error is below 7.5e-5 (degree-3 minimax fit).  Stands in for the
 * reference's software exp2 emulation (0.attention/ptx_wrappers.cuh:711-741),
 * which has no test of its own.
 */
b200_status b200_selftest_exp2(const float* x, float* y_fma, float* y_mufu, uint64_t n,
                               b200_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* B200ATTN_H */
