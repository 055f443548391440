// gemm_tc.cu -- persistent, warp-specialised tcgen05 TF32 GEMM for sm_100a.
//
// Roles per CTA (192 threads, one CTA per SM):
//   warp 0      TMA producer: A and B K-slices (32 FP32 = 128 B, SWIZZLE_128B)
//               into a STAGES-deep shared-memory ring;
//   warp 1      TMEM allocator and single-thread tcgen05.mma issuer
//               (M = 128, N = BN, K = 8 per instruction);
//   warps 2..9  epilogue: tcgen05.ld of the FP32 accumulator (warp w owns TMEM
//               lanes 32 * (w % 4) .. and half of the tile's columns, so each
//               SM sub-partition runs two epilogue warps), fused epilogue,
//               vectorised stores.
// Two TMEM accumulators (2 * BN columns) let the epilogue of tile i overlap
// the MMAs of tile i + 1.  Tiles are walked n-fastest so CTAs running at the
// same time share the A rows in L2.
//
// Replaces kernels::linear (src/tensor/kernels.rs:577-685) for every
// projection of the encoder (src/model/text.rs:287-528).

#include <cuda.h>

#include <mutex>

#include "common.cuh"
#include "gemm_tc.cuh"

namespace svl {

namespace {

constexpr int BM = 128;
constexpr int BK = 32;  // FP32 elements per 128-byte swizzle row
constexpr int kThreads = 320;  // warp 0 TMA, warp 1 MMA, warps 2..9 epilogue

template <int BN>
struct Cfg {
  static constexpr int STAGES = BN == 256 ? 4 : 6;
  static constexpr int A_BYTES = BM * BK * 4;
  static constexpr int B_BYTES = BN * BK * 4;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
  static constexpr uint32_t TMEM_COLS = 2 * BN;
  static_assert(SMEM <= 232448, "shared memory");
};

template <int BN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tf32_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                     GemmParams p) {
  using C = Cfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* full = (uint64_t*)(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tmem_full = empty + C::STAGES;
  uint64_t* tmem_empty = tmem_full + 2;
  uint32_t* tmem_slot = (uint32_t*)(tmem_empty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (p.M + BM - 1) / BM;
  const int num_n = (p.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_k = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], 256);
    }
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        const int m0 = (tile / num_n) * BM;
        const int n0 = (tile % num_n) * BN;
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.err)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * C::STAGE_BYTES;
          mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
          tma_load_2d(sa, &map_a, &full[stage], kb * BK, m0);
          tma_load_2d(sa + C::A_BYTES, &map_b, &full[stage], kb * BK, n0);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_tf32(BM, BN, 0);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1, p.err)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * C::STAGE_BYTES);
          const uint32_t b_addr = a_addr + C::A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 8; ++k) {
            const uint64_t ad = sdesc(a_addr + k * 32, 16, 1024, kLayoutSW128);
            const uint64_t bd = sdesc(b_addr + k * 32, 16, 1024, kLayoutSW128);
            mma_tf32(d, ad, bd, idesc, (kb | k) != 0);
          }
          mma_commit(&empty[stage]);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        mma_commit(&tmem_full[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else {
    // epilogue warps 2..5
    const int lane_grp = warp & 3;
    const int half = (warp - 2) >> 2;  // warps 2..5 take the first half of the columns, 6..9 the second
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const int m0 = (tile / num_n) * BM;
      const int n0 = (tile % num_n) * BN;
      const bool ready = mbar_wait(&tmem_full[acc], acc_phase, p.err);
      __syncwarp();
      if (!__all_sync(0xffffffffu, ready)) break;
      tc_fence_after();
      const int row = m0 + lane_grp * 32 + lane;
      const uint32_t taddr = tmem_base + ((uint32_t)(lane_grp * 32) << 16) + (uint32_t)(acc * BN);
      float v[32];
      if constexpr (EPI == kEpiGeglu) {
        // columns [0, BN/2) hold gate rows, [BN/2, BN) the matching up rows
        float u[32];
        const int f0 = n0 / 2;
#pragma unroll 1
        for (int c = half * (BN / 128); c < (half + 1) * (BN / 128); ++c) {
          tmem_ld32(taddr + c * 32, v);
          tmem_ld32(taddr + BN / 2 + c * 32, u);
          const int col0 = f0 + c * 32;
          if (row < p.M && col0 < p.n_out) {
            float* out = p.C + (size_t)row * p.ldc + col0;
            const int ncols = p.n_out - col0;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              float r = gelu_tanh(v[j]) * u[j];
              v[j] = p.round_out ? round_tf32(r) : r;
            }
            if (ncols >= 32) {
#pragma unroll
              for (int j = 0; j < 32; j += 4) *(float4*)(out + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
            } else {
              for (int j = 0; j < ncols; ++j) out[j] = v[j];
            }
          }
        }
      } else {
#pragma unroll 1
        for (int c = half * (BN / 64); c < (half + 1) * (BN / 64); ++c) {
          tmem_ld32(taddr + c * 32, v);
          const int col0 = n0 + c * 32;
          if (row < p.M && col0 < p.N) {
            float* out = p.C + (size_t)row * p.ldc + col0;
            const int ncols = p.N - col0;
            if constexpr (EPI == kEpiPleGate) {
              const float* aux = p.aux + (size_t)row * p.ld_aux + col0;
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                float r = j < ncols ? gelu_tanh(v[j]) * aux[j] : 0.0f;
                v[j] = p.round_out ? round_tf32(r) : r;
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                float r = v[j] * p.alpha;
                v[j] = p.round_out ? round_tf32(r) : r;
              }
            }
            if (ncols >= 32) {
#pragma unroll
              for (int j = 0; j < 32; j += 4) *(float4*)(out + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
            } else {
              for (int j = 0; j < ncols; ++j) out[j] = v[j];
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tmem_empty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host --
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)ptr;
  });
  return fn;
}

// rows x cols FP32 matrix with row pitch ld (elements); box = 32 x box_rows.
bool make_map(CUtensorMap* map, const float* base, int rows, int cols, int ld, int box_rows, bool tf32) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t elem[2] = {1, 1};
  CUresult r = enc(map, tf32 ? CU_TENSOR_MAP_DATA_TYPE_TFLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                   (void*)base, dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int BN, int EPI>
cudaError_t launch(const GemmParams& p, cudaStream_t stream) {
  using C = Cfg<BN>;
  static bool attr_set = false;  // per (BN, EPI) instantiation
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(gemm_tf32_kernel<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  CUtensorMap ma, mb;
  if (!make_map(&ma, p.A, p.M, p.K, p.lda, BM, p.tf32_tma) || !make_map(&mb, p.B, p.N, p.K, p.ldb, BN, p.tf32_tma))
    return cudaErrorInvalidValue;
  const int tiles = ((p.M + BM - 1) / BM) * ((p.N + BN - 1) / BN);
  const int grid = tiles < sm_count() ? tiles : sm_count();
  gemm_tf32_kernel<BN, EPI><<<grid, kThreads, C::SMEM, stream>>>(ma, mb, p);
  return cudaGetLastError();
}

}  // namespace

int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 1;
  }
  return n;
}

cudaError_t gemm_tf32(const GemmParams& p, cudaStream_t stream) {
  if (p.M <= 0 || p.N <= 0) return cudaSuccess;
  if (p.K <= 0 || p.K % 4 || p.lda % 4 || p.ldb % 4 || p.ldc % 4 || ((uintptr_t)p.A & 15) || ((uintptr_t)p.B & 15))
    return cudaErrorInvalidValue;
  if (p.lda < p.K || p.ldb < p.K) return cudaErrorInvalidValue;
  switch (p.epilogue) {
    case kEpiStore:
      if (p.N <= 128) return launch<128, kEpiStore>(p, stream);
      return launch<256, kEpiStore>(p, stream);
    case kEpiGeglu:
      if (p.N % 256 || p.n_out <= 0 || p.n_out > p.N / 2) return cudaErrorInvalidValue;  // 128-row gate/up blocks
      return launch<256, kEpiGeglu>(p, stream);
    case kEpiPleGate:
      if (!p.aux) return cudaErrorInvalidValue;
      if (p.N <= 128) return launch<128, kEpiPleGate>(p, stream);
      return launch<256, kEpiPleGate>(p, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace svl
