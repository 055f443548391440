// attention_tc.cuh -- tcgen05 flash-style attention (attention_tc.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace svl {

struct AttnParams {
  const float* qkv;  // [T, ld]: q heads, k heads, v heads (TF32-rounded)
  int ld, T, nh, kvh, hd;
  int dsplit;        // set by the launcher: 2 when hd > 256
  int window;        // inclusive two-sided radius, < 0 for full attention
  float* out;        // [T, ld_out], head h at column h * hd
  int ld_out;
  int round_out;     // round outputs to the TF32 grid (they feed the o projection)
  int single_cta;    // force the one-CTA kernel (tests compare it with the CTA-pair kernel)
  uint32_t* err;
};

bool attention_tc_supported(int hd);
// Bytes of device workspace the launcher needs for its work list.
size_t attention_tc_items_bytes(const uint64_t* cu_host, int batch, int nh);
// cu_host: batch + 1 sequence offsets on the host (the work list is built from it).
cudaError_t launch_attention_tc(const AttnParams& p, const uint64_t* cu_host, int batch, void* d_items_ws,
                                size_t ws_bytes, cudaStream_t st);

}  // namespace svl
