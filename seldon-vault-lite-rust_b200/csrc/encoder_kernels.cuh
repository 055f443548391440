// encoder_kernels.cuh -- launchers of the bandwidth-bound encoder kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace svl {

void launch_positions(const uint64_t* cu, uint32_t batch, uint32_t* seq_of, uint32_t* pos_of, cudaStream_t st);
void launch_embed(const uint32_t* ids, int T, const float* table, int H, uint32_t vocab, float scale, float* hidden,
                  uint32_t* err, cudaStream_t st);
// out16 / inv16 (optional): the normalised rows as FP16 GEMM operand rows
// with power-of-two row scales instead of FP32 `out` (width a multiple of 128
// up to 1024, else returns false without launching).
// row_absmax (optional): each output row's largest magnitude.
// row_inv (optional): each row's 1 / rms.  out = NULL with no out16 writes
// only these statistics (vectorised widths).
bool launch_rmsnorm_rows(const float* in, int ld_in, float* out, int ld_out, int rows, int width, const float* w,
                         float pre, float eps, int round_out, uint32_t* err, cudaStream_t st,
                         uint16_t* out16 = nullptr, float* inv16 = nullptr, float* row_absmax = nullptr,
                         float* row_inv = nullptr);
// rope: optional [positions][hd / 2] (cos, sin) table from launch_rope_table
// (NULL: angles computed in the kernel).  out16: optional FP16 destination
// with qkv's layout (the attention operands; qkv is then left as it was);
// needs the rope table and hd 128, 256 or 512, else returns false.
bool launch_qkv_post(float* qkv, int ld, int T, int nh, int kvh, int hd, const float* q_norm, const float* k_norm,
                     const float* inv_freq, const float2* rope, const uint32_t* pos_of, float eps, int round_qk,
                     uint16_t* out16, uint32_t* err, cudaStream_t st);
// The same from an FP16 projection stored with per-(row, 128-column group)
// power-of-two scales gi and partial sums of squares pss (the GEMM's
// kEpiStore16 outputs, row stride gstride); FP16 output only.
bool launch_qkv_post16(const uint16_t* in16, const float* gi, const float* pss, int gstride, int ld, int T, int nh,
                       int kvh, int hd, const float* q_norm, const float* k_norm, const float2* rope,
                       const uint32_t* pos_of, float eps, uint16_t* out16, uint32_t* err, cudaStream_t st);
void launch_rope_table(const float* inv_freq, int half, int n_pos, int position_major, float2* out, cudaStream_t st);
// kResExact may be or'ed into a mode: xn is then written exact (not
// TF32-rounded), for the split-precision GEMMs that expand it themselves.
enum ResNormMode : int { kResNone = 0, kResNormNext = 1, kResRoundedCopy = 2, kResExact = 4 };
// Per-row FP16 scale of the output of the GEMM that xn feeds, from a bound
// (bound_scale_row in encoder_kernels.cu): inv[row] = its inverse (2^e).
struct BoundScale {
  float* inv = nullptr;
  float a_max = 0.0f, b_max = 0.0f;
  const float* row_max = nullptr;  // optional x_max per row (stride apart)
  int stride = 1;
};
// xn16 / xn_inv (optional): xn as FP16 GEMM operand rows with power-of-two
// row scales instead of FP32 (H a multiple of 128 up to 1024, else returns
// false without launching).
// bound (optional, with xn16): also the FP16 row scales of the next GEMM's
// output (see BoundScale).
bool launch_residual_norm(float* hidden, const float* delta, int T, int H, const float* w_post, float layer_scalar,
                          int apply_scalar, const float* w_next, float* xn, int mode, float eps, uint32_t* err,
                          cudaStream_t st, uint16_t* xn16 = nullptr, float* xn_inv = nullptr,
                          const BoundScale* bound = nullptr);
bool launch_attention_simt(const float* qkv, int ld, int T, int nh, int kvh, int hd, const uint64_t* cu,
                           const uint32_t* seq_of, const uint32_t* pos_of, int window, float* out, int ld_out,
                           int round_out, uint32_t* err, cudaStream_t st);
// mean: [batch, E] scratch (the pooled rows before normalisation).
void launch_pool_normalize(const float* projected, int E, const uint64_t* cu, int batch, int dim, float* mean,
                           float* pooled, float* normalized, float* out, uint32_t* err, cudaStream_t st);
void launch_round_tf32(float* x, size_t n, cudaStream_t st);
// Split-precision operand expansion: in [rows, K] (row pitch ld_in) ->
// out [rows, 3K] as [hi | hi | lo] (activations) or [hi | lo | hi]
// (weights = 1), hi = TF32(x), lo = TF32(x - hi).
void launch_split3(const float* in, int ld_in, float* out, int rows, int K, int weights, cudaStream_t st);
// out2[0] / out2[1] (device words, zeroed by the caller) = the largest row L2
// norm over rows with (row / period) even / odd (period 0: all rows in out2[0]),
// as float bits.
void launch_row_norm_max(const float* w, int rows, int cols, int period, uint32_t* out2, cudaStream_t st);
// n values -> FP16 with one power-of-two scale (largest magnitude in
// [2^14, 2^15)); *inv_out (device) = the inverse scale; scratch: one device word.
void launch_matrix_to_f16(const float* in, size_t n, uint16_t* out, float* inv_out, uint32_t* scratch, cudaStream_t st);
// FP32 rows -> FP16 GEMM operand rows, each scaled by a power of two 2^-e
// (largest magnitude in [2^14, 2^15)); inv_scale[row] = 2^e.
void launch_rows_to_f16(const float* in, int ld_in, uint16_t* out, int ld_out, int rows, int width, float* inv_scale,
                        uint32_t* err, cudaStream_t st);
void launch_bf16_widen(const uint16_t* in, float* out, size_t n, cudaStream_t st);
void launch_finite_check(const float* x, size_t n, uint32_t* err, cudaStream_t st);

}  // namespace svl
