// attention_f16.cuh -- CTA-pair attention with FP16 tensor-core operands
// (attention_f16.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

namespace svl {

struct AttnF16Params {
  const uint16_t* qkv;  // [T, ld] FP16: q heads, k heads, v heads (normalised, RoPE applied)
  int ld, T, nh, kvh, hd;
  int window;           // inclusive two-sided radius, < 0 for full attention
  float* out;           // [T, ld_out] FP32, head h at column h * hd
  int ld_out;
  int round_out;        // round outputs to the TF32 grid (they feed the o projection)
  uint16_t* out16;      // optional: O in FP16 instead (|O| <= max |v| <= sqrt(hd)), same layout as out
  uint32_t* err;
};

// Head dims 128, 256 and 512 with an even number of query heads per KV head.
bool attention_f16_supported(int hd, int nh, int kvh);
// Builds the work schedule of one attention shape for the current device:
// 128-query blocks x head pairs (x head-dim halves for hd 512) spread over as
// many CTA pairs as the GPU holds at once.  `out` receives the words to upload
// (16-byte aligned on the device).  Returns the number of CTA pairs (0: no
// work, < 0: error).  cu_host: batch + 1 sequence offsets on the host.
int attention_f16_schedule(const uint64_t* cu_host, int batch, int nh, int hd, int window, std::vector<uint32_t>* out);
// Launches with a schedule from attention_f16_schedule (same nh, hd, window,
// batch) already on the device.
cudaError_t launch_attention_f16(const AttnF16Params& p, const uint32_t* d_schedule, int pairs, cudaStream_t st);
// Round-to-nearest-even FP32 -> FP16 copy (test inputs).
void launch_f32_to_f16(const float* in, uint16_t* out, size_t n, cudaStream_t st);

}  // namespace svl
