// attention_f16.cuh -- CTA-pair attention with FP16 tensor-core operands
// (attention_f16.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace svl {

struct AttnF16Params {
  const uint16_t* qkv;  // [T, ld] FP16: q heads, k heads, v heads (normalised, RoPE applied)
  int ld, T, nh, kvh, hd;
  int window;           // inclusive two-sided radius, < 0 for full attention
  float* out;           // [T, ld_out] FP32, head h at column h * hd
  int ld_out;
  int round_out;        // round outputs to the TF32 grid (they feed the o projection)
  uint32_t* err;
};

// Head dims 128, 256 and 512 with an even number of query heads per KV head.
bool attention_f16_supported(int hd, int nh, int kvh);
// Bytes of device workspace the launcher needs for its work list.
size_t attention_f16_items_bytes(const uint64_t* cu_host, int batch, int nh, int hd);
// cu_host: batch + 1 sequence offsets on the host (the work list is built from it).
cudaError_t launch_attention_f16(const AttnF16Params& p, const uint64_t* cu_host, int batch, void* d_items_ws,
                                 size_t ws_bytes, cudaStream_t st);
// Round-to-nearest-even FP32 -> FP16 copy (test inputs).
void launch_f32_to_f16(const float* in, uint16_t* out, size_t n, cudaStream_t st);

}  // namespace svl
