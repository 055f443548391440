// row_fused.cuh -- encoder steps fused per 128-row block (row_fused.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace svl {

// Operands of the fused per-layer-input block (src/model/text.rs:474-513)
// for a hidden and per-layer width of 512: PLE-gate GEMM, GELU x the
// RMS-normalised per-layer slice, PLE-projection GEMM, post norm, residual,
// layer scalar and the next block's pre-norm, in one kernel.
struct PleBlockParams {
  int T;                         // rows (tokens)
  const uint16_t* xn16;          // [T, 512] FP16 copy of the residual stream (the gate GEMM's A), row scale xn_inv
  const float* xn_inv;           // [T]
  const uint16_t* w_gate16;      // [512, 512] FP16 per_layer_input_gate, scale *w_gate_inv
  const float* w_gate_inv;
  const uint16_t* w_proj16;      // [512, 512] FP16 per_layer_projection, scale *w_proj_inv
  const float* w_proj_inv;
  const uint16_t* per_layer16;   // this layer's raw per-layer slice in FP16: row t at per_layer16 + t * ld_pl,
  int ld_pl;                     //   128-column part g scaled by 1 / pgi[t * pss_stride + g]
  const float* pss;              // its rows' sums of squares in four 128-column parts (the PLE
  const float* pgi;              //   projection's row_ss) and the parts' inverse scales
  int pss_stride;                //   (group_inv): pss / pgi[t * pss_stride + 0..3]
  const float* ple_norm;         // [512] per_layer_projection_norm weight
  float* hidden;                 // [T, 512] residual stream, updated in place
  const float* w_post;           // [512] post_per_layer_input_norm weight
  float layer_scalar;
  const float* w_next;           // [512] the next block's pre-norm weight
  float eps;
  uint16_t* xn16_out;            // [T, 512] next GEMM's FP16 operand (may alias xn16)
  float* xn_inv_out;             // [T] its row scales (may alias xn_inv)
  uint32_t* err;
};

// An N = 512 projection fused with the residual step after it (the attention
// output projection, the FFN down projection):
//   hidden = hidden + rmsnorm(a16 @ w16^T * scales) * w_post
// then out16 / xn_inv_out: the next GEMM's FP16 operand (out = 0: the
// next block's pre-norm rmsnorm(hidden) * w_next; 1: the same plus
// bound_inv, the GeGLU output's row scale from |xn| (bound_a, bound_b: the
// gate and up weight row-norm maxima); 2: a copy of hidden).
enum RowOut : int { kOutNormNext = 0, kOutNormNextBound = 1, kOutCopy = 2 };

struct ResidualArgs {
  int T;
  float* hidden;           // [T, 512]
  const float* w_post;     // [512]
  float layer_scalar;      // applied when apply_scalar
  int apply_scalar;
  const float* w_next;     // [512] (out 0 and 1)
  float eps;
  float* xn_inv_out;       // [T]
  float* bound_inv;        // [T] (out 1)
  float bound_a, bound_b;
  uint32_t* err;
};

struct GemmResidualLaunch {
  int K;                   // reduction width, a multiple of 64
  const uint16_t* a16;     // [T, K] FP16 (row pitch lda), row scales a_inv (NULL: 1)
  int lda;
  const float* a_inv;
  const uint16_t* w16;     // [512, K] FP16 weight, inverse scale *w_inv
  const float* w_inv;
  uint16_t* out16;         // [T, 512]
  int out;                 // a RowOut
  ResidualArgs res;
};
bool gemm_residual_supported(int hidden, int k);
cudaError_t launch_gemm_residual(const GemmResidualLaunch& g, cudaStream_t st);

// True when the fused block applies (hidden and per-layer widths of 512).
bool ple_block_supported(int hidden, int per_layer);
cudaError_t launch_ple_block(const PleBlockParams& p, cudaStream_t st);

}  // namespace svl
