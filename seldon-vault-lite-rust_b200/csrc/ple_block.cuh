// ple_block.cuh -- the fused per-layer-input block of an encoder layer.
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
  const float* per_layer;        // this layer's raw per-layer slice: row t at per_layer + t * ld_pl
  int ld_pl;
  const float* pinv;             // its RMSNorm inverse per row: pinv[t * pinv_stride]
  int pinv_stride;
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

// True when the fused block applies (hidden and per-layer widths of 512).
bool ple_block_supported(int hidden, int per_layer);
cudaError_t launch_ple_block(const PleBlockParams& p, cudaStream_t st);

}  // namespace svl
