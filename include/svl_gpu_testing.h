/*
 * svl_gpu_testing.h -- kernel-level entry points of libsvl_gpu.so used by the
 * parity tests to check one kernel at a time against the CPU oracle.
 *
 * NOT part of the drop-in boundary (svl_gpu.h): the reference has no
 * counterpart for these; they exist so a failing end-to-end parity test can be
 * narrowed to one kernel.  All pointers are device pointers; each call
 * synchronises `stream` (a cudaStream_t, NULL = legacy default stream) and
 * returns an svl_status.
 */
#ifndef SVL_GPU_TESTING_H
#define SVL_GPU_TESTING_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* C[M, N] = A[M, K] . B[N, K]^T on the tcgen05 TF32 tensor-core GEMM
 * (the kernel behind every linear of the encoder, kernels.rs:655-685).
 * epilogue 0 = alpha * acc, 1 = GeGLU over 128-row interleaved gate/up
 * blocks (n_out = output width), 2 = gelu(acc) * aux.  tf32_tma is a flag
 * word: bit 0 selects the TFLOAT32 TMA data type for the operand copies,
 * bit 1 forces the one-CTA kernel instead of the CTA-pair kernel that
 * M >= 256 and N >= 256 would otherwise use, bit 2 runs the products on
 * FP16 operands the way the encoder does (A rows and all of B scaled by
 * powers of two, converted on the device). */
int svl_test_gemm_tf32(const float* A, int lda, const float* B, int ldb, float* C, int ldc, int M, int N, int K,
                       int epilogue, float alpha, const float* aux, int ld_aux, int round_out, int n_out,
                       int tf32_tma, void* stream);

/* The same product on FP16 operands (as bit 2 above) stored the way the
 * encoder stores its per-layer table and full-attention q/k/v: C16 FP16 with
 * one power-of-two scale per (row, 128-column group), group_inv[row *
 * group_stride + col / 128] = the inverse scale (value = C16 * group_inv) and
 * row_ss[...] = the group's sum of squares of the unrounded values.  Needs
 * N % 128 == 0 and N > 128; single_cta forces the one-CTA kernel. */
int svl_test_gemm_grouped(const float* A, int lda, const float* B, int ldb, uint16_t* C16, int ldc, int M, int N,
                          int K, float alpha, float* group_inv, float* row_ss, int group_stride, int single_cta,
                          void* stream);

/* Bidirectional GQA attention (kernels.rs:1037-1135, scale 1.0) over the
 * fused [T, ld] qkv rows of a packed batch; window < 0 = full attention.
 * d_cu / h_cu: the batch + 1 offsets on the device and on the host.
 * impl 0 = FP32 SIMT kernel (any head dim), 1 = tcgen05 TF32 kernels
 * (head dim a multiple of 32, at most 512; the CTA-pair kernel when the head
 * dim is a multiple of 64 up to 256 and each KV head serves an even number
 * of query heads, else the one-CTA kernel), 2 = the one-CTA kernel always. */
int svl_test_attention(const float* qkv, int ld, int T, int nh, int kvh, int hd, const uint64_t* d_cu,
                       const uint64_t* h_cu, int batch, int window, int impl, float* out, int ld_out, void* stream);

/* Per-kernel-category CUDA-event timing of a model's / an index's launches
 * (bench.py puts these live kernel times beside the roofline).  Categories:
 * 0 tensor-core GEMMs, 1 attention, 2 norms / residual / RoPE, 3 other,
 * 4 search screen, 5 search rescoring.  *_read synchronises, fills ms[6] and
 * launches[6] (launch counts are kept even while timing is off) and resets. */
typedef struct svl_model svl_model;
typedef struct svl_index svl_index;
int svl_model_profile(svl_model* model, int enable);
int svl_model_profile_read(svl_model* model, double* ms, uint64_t* launches);
int svl_index_profile(svl_index* index, int enable);
int svl_index_profile_read(svl_index* index, double* ms, uint64_t* launches);

#ifdef __cplusplus
}
#endif
#endif
