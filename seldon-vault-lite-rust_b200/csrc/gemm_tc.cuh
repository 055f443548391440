// gemm_tc.cuh -- host interface of the tcgen05 TF32 GEMM (gemm_tc.cu).
//
// C[M, N] = A[M, K] . B[N, K]^T with A, B row-major FP32 (both K-major), the
// layout of every linear layer in the reference (kernels.rs:655-685:
// out[r, c] = sum_k in[r, k] * W[c, k]).  Products run on the tensor cores in
// TF32 with FP32 accumulation in TMEM.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace svl {

enum GemmEpilogue : int {
  kEpiStore = 0,    // C = alpha * acc
  kEpiGeglu = 1,    // B rows interleaved in 128-row blocks [gate | up]; C[:, f] = gelu(g) * u
  kEpiPleGate = 2,  // C = gelu(acc) * aux[row, aux_col0 + col]
  kEpiQkv = 3,      // fused q/k/v projection with 256-wide heads: per-head RMSNorm
                    // (q_norm / k_norm weights, v unscaled) and rotate-half RoPE
  kEpiQkv16 = 4,    // internal: kEpiQkv writing FP16 (selected by GemmParams::out_f16)
  kEpiGeglu16 = 5,  // internal: kEpiGeglu writing FP16 scaled by 1 / out_inv[row]
  kEpiPleGate16 = 6,  // internal: kEpiPleGate writing FP16 scaled by 1 / out_inv[row]
  kEpiStore16 = 7,    // internal: kEpiStore writing FP16 with one power-of-two scale per
                      // (row, 128-column group) (selected by GemmParams::group_inv)
};

struct GemmParams {
  const void* A;  // FP32 (or FP16 with f16)
  int lda;        // elements
  const void* B;
  int ldb;
  float* C;
  int ldc;
  int M, N, K;  // N = rows of B
  int n_out;    // kEpiGeglu: true output width F (B holds F padded to 128-row gate/up blocks)
  int epilogue;
  float alpha;
  const float* aux;  // kEpiPleGate
  int ld_aux;
  int round_out;     // round outputs to the TF32 grid (they feed another GEMM)
  uint32_t* err;     // device error word (nullable)
  int tf32_tma;      // TMA data type TFLOAT32 instead of FLOAT32 (operand rounding by the copy engine)
  int single_cta;    // force the one-CTA kernel (tests compare it with the CTA-pair kernel)
  // kEpiQkv: heads of 256 columns, [nh q heads | kvh k heads | kvh v heads]
  int nh, kvh;
  const float* q_norm;       // [256]
  const float* k_norm;       // [256]
  const float2* rope;        // [128][rope_stride] (cos, sin), position fastest
  int rope_stride;           // positions in the table
  const uint32_t* pos_of;    // [M] position of each row in its sequence
  float eps;
  int out_f16;               // kEpiQkv / kEpiGeglu / kEpiPleGate: C is FP16 (uint16_t, ldc in elements)
  const float* out_inv;      // FP16 GeGLU / PLE-gate outputs: stored = value / out_inv[row] (powers of two)
  // FP16 operands (A and B uint16_t, lda / ldb in elements, multiples of 8):
  // the true operands are A[r, :] * a_inv[r] and B * b_scale (exact powers
  // of two from the producers; NULL = 1), applied to the accumulator.
  int f16;
  const float* a_inv;
  const float* b_scale;  // one inverse scale for all of B (a device scalar; NULL = 1)
  // FP16 PLE gate: the aux slice is the un-normalised per-layer input; the
  // epilogue applies its RMSNorm: aux * aux_row_inv[row * aux_row_stride] *
  // aux_col_w[col] (NULL aux_col_w: aux used as is)
  const float* aux_row_inv;
  int aux_row_stride;
  const float* aux_col_w;
  // kEpiStore: per (row, 128-column group) sum of squares of the stored
  // values, row_ss[row * row_ss_stride + col / 128] (NULL: none; needs
  // N % 128 == 0 and N > 128, so each epilogue warp owns whole groups)
  float* row_ss;
  int row_ss_stride;
  // kEpiStore with FP16 output: C is FP16 (ldc in elements), each (row,
  // 128-column group) stored times a power of two whose inverse goes to
  // group_inv[row * row_ss_stride + col / 128] (the value = stored *
  // group_inv); row_ss then holds the unscaled values' sums of squares
  float* group_inv;
};

// Validates and launches on `stream`.  Returns cudaSuccess or an error code.
// Requirements: K % 4 == 0, lda/ldb/ldc % 4 == 0, A/B 16-byte aligned (FP16
// operands: K, lda, ldb multiples of 8).
cudaError_t gemm_tf32(const GemmParams& p, cudaStream_t stream);

// Number of SMs of the current device (cached).
int sm_count();

}  // namespace svl
