// row_fused.cu -- encoder steps whose output rows are normalised as a whole,
// each as ONE kernel per 128-row block that owns its rows' full 512 columns.
//
// ple_block_kernel: the per-layer-input block of one encoder layer
// (src/model/text.rs:474-513):
//
//   gate   = gelu(xn @ W_gate^T) * rmsnorm(per_layer[:, l])     (text.rs:474-497)
//   delta  = gate @ W_proj^T                                     (text.rs:498-501)
//   hidden = (hidden + rmsnorm(delta) * w_post) * layer_scalar   (text.rs:502-513)
//   xn     = rmsnorm(hidden) * w_next  (the next block's pre-norm, FP16 operand)
//
// Unfused, this is two N = 512 GEMMs and a residual kernel per half batch:
// 76 tiles of 256 x 256 for 74 CTA pairs each (one tile per pair, nothing to
// overlap its fill and epilogue with), the gated rows written to and read
// back from memory, and a latency-bound residual step.  Here a CTA owns 128
// full rows: both GEMMs' 128 x 512 accumulators take the SM's 512 TMEM
// columns in turn, the gated row never leaves the SM (the first epilogue
// writes it in FP16 -- with its exact row scale, the whole row being on chip
// -- into shared memory as the second GEMM's A operand), and the residual
// arithmetic runs one thread per (row, column half) with no warp reductions.
//
// Warp 0 issues the TMA loads (the A tile once, the weights through a 3-stage
// ring of 256 x 64 FP16 slices), warp 1 the tcgen05 MMAs (M = 128, N = 256,
// kind::f16, two per K slice for the row's two column halves), warps 2..9
// the epilogues (warp w: TMEM lanes 32 (w % 4).., columns 256 ((w - 2) / 4)..).
// Every wait is bounded (mbar_wait); an epilogue thread never leaves early, so
// the named barriers and the gated-rows barrier always complete.

#include <mutex>

#include "common.cuh"
#include "row_fused.cuh"

namespace svl {

namespace {

constexpr int kRows = 128;                       // rows per CTA (the MMA's M)
constexpr int kWidth = 512;                      // H = P: both GEMMs' N and K
constexpr int kChunkK = 64;                      // FP16 elements per 128-byte operand row
constexpr int kNumKChunks = kWidth / kChunkK;    // 8
constexpr int kABytes = kRows * 128;             // one K chunk of A: 16 KB
constexpr int kARegion = kNumKChunks * kABytes;  // the whole A tile: 128 KB
constexpr int kHalfN = 256;                      // one MMA's N
constexpr int kBBytes = kHalfN * 128;            // one (K chunk, N half) weight slice: 32 KB
constexpr int kStages = 3;
constexpr int kEntries = 2 * kNumKChunks;        // weight slices per GEMM
constexpr int kThreads = 320;                    // PLE block: warp 0 TMA, warp 1 MMA, warps 2..9 epilogue
constexpr int kEpiThreads = 256;
constexpr int kXchgBytes = 2 * kRows * 4;        // per-row partials of the two column halves
constexpr int kBarBytes = 256;
constexpr int kSmem = kARegion + kStages * kBBytes + kXchgBytes + kBarBytes + 1024;
static_assert(kSmem <= 232448, "shared memory");
static_assert((1 + 2 * kStages + 2 + 16) * 8 + 4 <= kBarBytes, "barrier area");

// Named barrier 1 over the epilogue warps: 8 of them (each row in two column
// halves) or 16 (the residual projections' epilogue: four column quarters).
template <int kParts>
SVL_DEV void epi_sync() {
  static_assert(kParts == 2 || kParts == 4, "epilogue parts");
  if constexpr (kParts == 2)
    asm volatile("bar.sync 1, 256;" ::: "memory");
  else
    asm volatile("bar.sync 1, 512;" ::: "memory");
}

// The residual epilogue's row exchange: four per-row quantities, one partial
// per column part (2 KB per part); the per-warp column weights follow it.
template <int kParts>
constexpr int xchg_bytes() {
  return 4 * kParts * kRows * 4;
}
// PLE block: its 8 warps' column weights (8 x 2 KB) sit in the weight ring
// after the row exchange; the ring is idle once the last GEMM is done.
constexpr int kWeightsOff = xchg_bytes<2>();


// What a row-fused kernel does with its 128 x 512 delta (the projection's
// output, in TMEM) after the GEMM:
//   hidden = (hidden + rmsnorm(delta) * w_post) [* layer_scalar]
// then the next GEMM's FP16 operand rows with power-of-two row scales:
//   kOutNormNext       rmsnorm(hidden) * w_next      (text.rs:345-352, 435-441)
//   kOutNormNextBound  the same, plus the row scale of the GeGLU output that
//                      operand produces (the bound of the residual kernel's
//                      BoundScale: 2 max(n a_max, 0.17) n b_max, n = |xn|)
//   kOutCopy           hidden itself (the PLE block's copy of the stream)

// A warp's kSpan columns (256 or 128) of the residual epilogue's per-column
// weights (w_post, then w_next or w_post again), kSpan / 128 float4 of each
// per lane: loaded before the accumulator wait, parked in the warp's
// 8 * kSpan bytes of shared memory during the first pass (park_col_weights),
// then read as broadcasts.  Each chunk loading its weights from global memory
// would put an L2 round trip on every chunk.
template <int kSpan>
struct ColWeights {
  static constexpr int V = kSpan / 128;  // float4 per lane and weight
  float4 r[2 * V];
};

template <int kSpan>
SVL_DEV ColWeights<kSpan> load_col_weights(const float* w_post, const float* w_next, int c0, int lane) {
  constexpr int V = ColWeights<kSpan>::V;
  const float4* wp = (const float4*)(w_post + c0) + V * lane;
  const float4* wn = (const float4*)(w_next + c0) + V * lane;
  ColWeights<kSpan> w;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    w.r[i] = wp[i];
    w.r[V + i] = wn[i];
  }
  return w;
}

template <int kSpan>
SVL_DEV void park_col_weights(const ColWeights<kSpan>& w, float* wsm, int lane) {
  constexpr int V = ColWeights<kSpan>::V;
  float4* s = (float4*)wsm;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    s[V * lane + i] = w.r[i];
    s[kSpan / 4 + V * lane + i] = w.r[V + i];
  }
}

// Loads TMEM chunk q + 1 (32 columns) into nxt without waiting, when it exists
// (q is warp-uniform); the caller waits (tmem_ld_wait, tmem_regs_after_wait)
// after working on chunk q, so the load's latency overlaps that work.
template <int kChunks>
SVL_DEV void tmem_prefetch_chunk(uint32_t taddr, int q, uint32_t* nxt) {
  if (q + 1 < kChunks) tmem_ld32_nowait(taddr + (q + 1) * 32, nxt);
}

SVL_DEV void tmem_take_chunk(uint32_t* cur, uint32_t* nxt) {
  tmem_ld_wait();
  tmem_regs_after_wait(nxt);
#pragma unroll
  for (int j = 0; j < 32; ++j) cur[j] = nxt[j];
}

// A pass over a warp's kChunks TMEM chunks of 32 columns.  With kAhead the
// next chunk's load is in flight while the current one is worked on (two
// 32-register buffers); without it (the 16-warp epilogue, 96 registers a
// thread) each chunk is loaded when it is needed and the other warps of the
// sub-partition cover the wait.
template <int kChunks, bool kAhead>
struct TmemPass {
  uint32_t cur[32];
  uint32_t nxt[kAhead ? 32 : 1];
  SVL_DEV void begin(uint32_t taddr) {
    if constexpr (kAhead) {
      tmem_ld32_nowait(taddr, nxt);
      tmem_take_chunk(cur, nxt);
    }
  }
  // chunk q into cur (and, ahead, chunk q + 1 on its way)
  SVL_DEV void at(uint32_t taddr, int q) {
    if constexpr (kAhead) {
      tmem_prefetch_chunk<kChunks>(taddr, q, nxt);
    } else {
      tmem_ld32_nowait(taddr + q * 32, cur);
      tmem_ld_wait();
      tmem_regs_after_wait(cur);
    }
  }
  SVL_DEV void done() {
    if constexpr (kAhead) tmem_take_chunk(cur, nxt);
  }
};

// A row's total of its kParts per-part partials x[part * 128 + rl].
template <int kParts>
SVL_DEV float part_sum(const float* x, int rl) {
  if constexpr (kParts == 2)
    return __fadd_rn(x[rl], x[kRows + rl]);
  else
    return __fadd_rn(__fadd_rn(x[rl], x[kRows + rl]), __fadd_rn(x[2 * kRows + rl], x[3 * kRows + rl]));
}

template <int kParts>
SVL_DEV float part_max(const float* x, int rl) {
  float m = fmax_abs_nan(x[rl], x[kRows + rl]);
  if constexpr (kParts == 4) m = fmax_abs_nan(m, fmax_abs_nan(x[2 * kRows + rl], x[3 * kRows + rl]));
  return m;
}

// The residual epilogue of one epilogue thread (row rl of the block, columns
// c0 .. c0 + 512 / kParts - 1: its part of the row), with the delta scaled by
// dsc.  st2: the warp's two 4 KB staging buffers; xch: the row exchange
// (xchg_bytes<kParts>()); wsm: the warp's 8 * 512 / kParts bytes for its
// column weights (cw); lb / lphase: the warp's two staging-load barriers and
// their phases.  Every TMEM access is made by the whole warp (`ok` is
// warp-uniform); rows past T load as zeros and are clipped from the stores.
// Each pass keeps the next chunk's TMEM load in flight while it works on the
// current one, and sums with four partial accumulators.
template <int OUT, int kParts>
SVL_DEV void residual_epilogue(const ResidualArgs& a, const CUtensorMap* map_h, const CUtensorMap* map_y, float dsc,
                               bool ok, uint32_t taddr, uint8_t* st2, float* xch,
                               const ColWeights<kWidth / kParts>& cw, float* wsm, uint64_t* lb, uint32_t& lphase,
                               int lane, int part, int rl, int row, int y0, int c0, bool& bad) {
  constexpr int kSpan = kWidth / kParts;
  constexpr int kChunks = kSpan / 32;
  const bool live = row < a.T;
  float* xss = xch;                         // [kParts][128] sum of squares of delta
  float* xss2 = xch + kParts * kRows;       // [kParts][128] sum of squares of the new residual
  float* xmax = xch + 2 * kParts * kRows;   // [kParts][128] largest |output before scaling|
  float* xnss = xch + 3 * kParts * kRows;   // [kParts][128] sum of squares of the normalised output
  const float* wps = wsm;          // w_post of this part's columns
  const float* wns = wsm + kSpan;  // w_next (kOutCopy: w_post)
  auto issue = [&](uint8_t* buf, int b, int x) {
    fence_async_smem();
    mbar_arrive_expect_tx(&lb[b], 32 * 32 * 4);
    tma_load_2d(buf, map_h, &lb[b], x, y0);
  };
  float ss = 0.0f;
  if (ok) {
    if (lane == 0) {  // the first residual boxes load during the first pass
      issue(st2, 0, c0);
      issue(st2 + 4096, 1, c0 + 32);
    }
    float s4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 1
    for (int q = 0; q < kChunks; q += 2) {
      uint32_t r0[32], r1[32];
      tmem_ld32_nowait(taddr + q * 32, r0);
      tmem_ld32_nowait(taddr + q * 32 + 32, r1);
      tmem_ld_wait();
      tmem_regs_after_wait(r0);
      tmem_regs_after_wait(r1);
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float a0 = __uint_as_float(r0[j]), a1 = __uint_as_float(r1[j]);
        s4[j & 3] = fmaf(a0, a0, s4[j & 3]);
        s4[j & 3] = fmaf(a1, a1, s4[j & 3]);
      }
    }
    ss = ((s4[0] + s4[1]) + (s4[2] + s4[3])) * (dsc * dsc);
  }
  park_col_weights<kSpan>(cw, wsm, lane);  // read after the exchange barrier below
  xss[part * kRows + rl] = ss;
  epi_sync<kParts>();
  const float ss_row = part_sum<kParts>(xss, rl);
  bad |= live && !isfinite(ss_row);
  const float inv = 1.0f / sqrtf(__fadd_rn(ss_row / (float)kWidth, a.eps));
  const float kd = dsc * inv;  // accumulator -> normalised delta
  float ss2 = 0.0f, mvw = 0.0f;
  if (ok) {
    float p4[4] = {0.0f, 0.0f, 0.0f, 0.0f}, m4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    TmemPass<kChunks, kParts == 2> tp;
    const uint32_t* cur = tp.cur;
    tp.begin(taddr);
#pragma unroll 1
    for (int q = 0; q < kChunks; ++q) {
      tp.at(taddr, q);
      const int b = q & 1;
      uint8_t* buf = st2 + b * 4096;
      const bool got = __all_sync(0xffffffffu, mbar_wait(&lb[b], (lphase >> b) & 1u, a.err));
      lphase ^= 1u << b;
      ok = ok && got;
      float h[32];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float4 v = *(const float4*)(buf + lane * 128 + ((u ^ (lane & 7)) * 16));
        h[4 * u] = v.x, h[4 * u + 1] = v.y, h[4 * u + 2] = v.z, h[4 * u + 3] = v.w;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float4 wp = *(const float4*)(wps + q * 32 + 4 * u);
        const float4 wn = *(const float4*)(wns + q * 32 + 4 * u);
        const float wpv[4] = {wp.x, wp.y, wp.z, wp.w};
        const float wnv[4] = {wn.x, wn.y, wn.z, wn.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int j = 4 * u + k;
          float v = fmaf(__uint_as_float(cur[j]) * kd, wpv[k], h[j]);
          if (a.apply_scalar) v *= a.layer_scalar;
          h[j] = v;
          p4[k] = fmaf(v, v, p4[k]);
          m4[k] = fmax_abs_nan(m4[k], OUT == kOutCopy ? v : v * wnv[k]);
        }
      }
      tmem_st32(taddr + q * 32, h);
      store_chunk_tma(map_h, (float*)buf, h, lane, c0 + q * 32, y0);  // committed bulk group
      if (lane == 0 && q + 2 < kChunks) {
        tma_store_wait_read();  // that store has read buffer b
        issue(buf, b, c0 + (q + 2) * 32);
      }
      __syncwarp();
      tp.done();
    }
    tmem_st_wait();
    ss2 = (p4[0] + p4[1]) + (p4[2] + p4[3]);
    mvw = fmax_abs_nan(fmax_abs_nan(m4[0], m4[1]), fmax_abs_nan(m4[2], m4[3]));
  }
  if (!live) ss2 = mvw = 0.0f;
  xss2[part * kRows + rl] = ss2;
  xmax[part * kRows + rl] = mvw;
  epi_sync<kParts>();
  const float ss2_row = part_sum<kParts>(xss2, rl);
  bad |= live && !isfinite(ss2_row);
  const float inv2 = OUT == kOutCopy ? 1.0f : 1.0f / sqrtf(__fadd_rn(ss2_row / (float)kWidth, a.eps));
  const float xmx = part_max<kParts>(xmax, rl) * inv2;
  bad |= live && !(xmx <= 3.0e38f);
  float xs, xinv;
  pow2_row_scale(xmx, xs, xinv);
  const float kx = inv2 * xs;
  float nsq = 0.0f;
  if (ok) {
    Staging sg{(float*)st2, 2};
    float n4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    TmemPass<kChunks, kParts == 2> tp;
    const uint32_t* cur = tp.cur;
    tp.begin(taddr);
#pragma unroll 1
    for (int q = 0; q < kChunks; ++q) {
      tp.at(taddr, q);
      // the FP16 values: h * inv2 * w_next * xs (xs a power of two); the
      // bound's sum of squares is taken of them and unscaled once at the end
      float h[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) h[j] = __uint_as_float(cur[j]) * kx;
      if (OUT != kOutCopy) {
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const float4 wn = *(const float4*)(wns + q * 32 + 4 * u);
          h[4 * u] *= wn.x;
          h[4 * u + 1] *= wn.y;
          h[4 * u + 2] *= wn.z;
          h[4 * u + 3] *= wn.w;
        }
      }
      uint32_t w[16];
#pragma unroll
      for (int m = 0; m < 16; ++m) {
        if (OUT == kOutNormNextBound) n4[m & 3] = fmaf(h[2 * m + 1], h[2 * m + 1], fmaf(h[2 * m], h[2 * m], n4[m & 3]));
        w[m] = pack_half2(h[2 * m], h[2 * m + 1]);
      }
      store_row64_f16(map_y, sg, w, lane, c0 + q * 32, y0);
      tp.done();
    }
    nsq = ((n4[0] + n4[1]) + (n4[2] + n4[3])) * (xinv * xinv);
    if (live && part == 0) a.xn_inv_out[row] = xinv;
  }
  if (OUT == kOutNormNextBound) {
    xnss[part * kRows + rl] = live ? nsq : 0.0f;
    epi_sync<kParts>();
    if (ok && live && part == 0) {
      const float n = sqrtf(part_sum<kParts>(xnss, rl));
      float scale, binv;
      pow2_row_scale(2.0f * fmaxf(n * a.bound_a, 0.17f) * (n * a.bound_b), scale, binv);
      a.bound_inv[row] = binv;
    }
  }
  if (lane == 0) tma_store_wait_all();
}

__global__ void __launch_bounds__(kThreads, 1)
    ple_block_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_wg,
                     const __grid_constant__ CUtensorMap map_wp, const __grid_constant__ CUtensorMap map_pl,
                     const __grid_constant__ CUtensorMap map_h, const __grid_constant__ CUtensorMap map_y,
                     PleBlockParams p) {
  extern __shared__ uint8_t smem_raw[];
  pdl_trigger();
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* a_region = smem;
  uint8_t* b_ring = smem + kARegion;
  float* xchg = (float*)(b_ring + kStages * kBBytes);
  uint64_t* bars = (uint64_t*)((uint8_t*)xchg + kXchgBytes);
  uint64_t* a_full = bars;
  uint64_t* b_full = bars + 1;
  uint64_t* b_empty = b_full + kStages;
  uint64_t* d_full = b_empty + kStages;  // phase 0: gate GEMM done, phase 1: projection GEMM done
  uint64_t* g_ready = d_full + 1;        // gated rows in shared memory, first accumulator drained
  uint64_t* ld_bar = g_ready + 1;        // [16]: two staging loads per epilogue warp
  uint32_t* tmem_slot = (uint32_t*)(ld_bar + 16);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * kRows;
  if (threadIdx.x == 0) {
    mbar_init(a_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&b_full[s], 1);
      mbar_init(&b_empty[s], 1);
    }
    mbar_init(d_full, 1);
    mbar_init(g_ready, kEpiThreads);
    for (int b = 0; b < 16; ++b) mbar_init(&ld_bar[b], 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_wg);
    tma_prefetch_desc(&map_wp);
    tma_prefetch_desc(&map_pl);
    tma_prefetch_desc(&map_h);
    tma_prefetch_desc(&map_y);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // xn16, hidden and the per-layer statistics are complete from here

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(a_full, kARegion);
      for (int j = 0; j < kNumKChunks; ++j) tma_load_2d(a_region + j * kABytes, &map_a, a_full, j * kChunkK, row0);
      int stage = 0;
      uint32_t phase = 0;
      for (int e = 0; e < 2 * kEntries; ++e) {
        // the ring is the first epilogue's staging until the gated rows are written
        if (e == kEntries && !mbar_wait(g_ready, 0, p.err)) break;
        if (!mbar_wait(&b_empty[stage], phase ^ 1, p.err)) break;
        const int g = e / kEntries, j = (e % kEntries) >> 1, h = e & 1;
        mbar_arrive_expect_tx(&b_full[stage], kBBytes);
        tma_load_2d(b_ring + stage * kBBytes, g ? &map_wp : &map_wg, &b_full[stage], j * kChunkK, h * kHalfN);
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(kRows, kHalfN, 0);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = mbar_wait(a_full, 0, p.err);
      for (int g = 0; ok && g < 2; ++g) {
        if (g == 1 && !mbar_wait(g_ready, 0, p.err)) break;
        tc_fence_after();
        for (int e = 0; e < kEntries; ++e) {
          if (!mbar_wait(&b_full[stage], phase, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int j = e >> 1, h = e & 1;
          const uint32_t a_addr = smem_u32(a_region + j * kABytes);
          const uint32_t b_addr = smem_u32(b_ring + stage * kBBytes);
          const uint32_t d = tmem_base + (uint32_t)(h * kHalfN);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_f16(d, sdesc(a_addr + k * 32, 16, 1024, kLayoutSW128), sdesc(b_addr + k * 32, 16, 1024, kLayoutSW128),
                    idesc, (j | k) != 0);
          mma_commit(&b_empty[stage]);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) mma_commit(d_full);
      }
    }
  } else {
    // Epilogue warp ew: TMEM lanes (rows) 32 (warp % 4).., columns c0.. (its
    // half).  Global traffic goes through two 4 KB staging buffers per warp
    // as 32 x 32 TMA boxes -- the FP16 per-layer slice (a lane reads its
    // row's 64 bytes, 16-byte units XOR-swizzled by (row / 2) % 4), the FP32
    // residual rows (128 bytes, by row % 8): the weight ring holds them in
    // the first epilogue (the producer holds the projection weights back
    // until the gated rows are written), the A tile in the second (the
    // projection GEMM is done with it).  Rows past T load
    // as zeros and are clipped from the stores, so no lane branches around
    // the warp-collective TMEM accesses; `ok` is kept warp-uniform.
    const int ew = warp - 2;
    const int lane_grp = warp & 3;
    const int half = ew >> 2;
    const int rl = lane_grp * 32 + lane;  // row within the block = TMEM lane
    const int row = row0 + rl;
    const int y0 = row0 + lane_grp * 32;  // first row of this warp's boxes
    const bool live = row < p.T;
    const uint32_t taddr = tmem_base + ((uint32_t)(lane_grp * 32) << 16) + (uint32_t)(half * kHalfN);
    const int c0 = half * kHalfN;  // first column of this warp's half
    uint64_t* lb = ld_bar + 2 * ew;
    uint32_t lphase = 0;  // bit b: phase of lb[b]
    constexpr int kChunks = kHalfN / 32;
    // per-row inputs, read before the accumulator wait
    const float ai = (live ? p.xn_inv[row] : 1.0f) * *p.w_gate_inv;
    // the slice's RMSNorm inverse from the projection's four partial sums
    float ar = 0.0f, gi0 = 0.0f, gi1 = 0.0f;  // gi: the inverse scales of this half's two FP16 parts
    if (live) {
      const float* ps = p.pss + (size_t)row * p.pss_stride;
      const float ss = (ps[0] + ps[1]) + (ps[2] + ps[3]);
      ar = 1.0f / sqrtf(__fadd_rn(ss / (float)kWidth, p.eps));
      const float* pg = p.pgi + (size_t)row * p.pss_stride + c0 / 128;
      gi0 = pg[0];
      gi1 = pg[1];
    }
    const ColWeights<kHalfN> cw = load_col_weights<kHalfN>(p.w_post, p.w_next, c0, lane);
    const float4* gnp = (const float4*)(p.ple_norm + c0) + 2 * lane;  // this lane's 8 norm weights
    const float4 gn0 = gnp[0], gn1 = gnp[1];
    bool bad = false;
    // a staged box: issue (lane 0), wait (all lanes), read / write this lane's row
    auto issue = [&](const CUtensorMap* map, uint8_t* buf, int b, int x) {
      fence_async_smem();  // earlier generic accesses of the buffer come first
      mbar_arrive_expect_tx(&lb[b], 32 * 32 * 2);  // a 32 x 32 FP16 box
      tma_load_2d(buf, map, &lb[b], x, y0);
    };
    auto arrived = [&](int b) {
      const bool got = mbar_wait(&lb[b], (lphase >> b) & 1u, p.err);
      lphase ^= 1u << b;
      return got;
    };
    // this lane's row of a 32 x 32 FP16 box (64-byte rows, 16-byte units
    // XOR-swizzled by (row / 2) % 4), times the part's inverse scale (exact)
    auto read_row = [&](const uint8_t* buf, float gi, float* x) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint4 v = *(const uint4*)(buf + lane * 64 + ((k ^ ((lane >> 1) & 3)) * 16));
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const float2 f = unpack_half2(w[m]);
          x[8 * k + 2 * m] = f.x * gi;
          x[8 * k + 2 * m + 1] = f.y * gi;
        }
      }
    };

    // ---- epilogue 1: gated = gelu(acc * ai) * ((aux * ar) * gamma), kept in
    // TMEM, then FP16 with the row's exact scale into the A tile
    bool ok = mbar_wait(d_full, 0, p.err);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    uint8_t* st1 = b_ring + ew * 8192;  // two 4 KB buffers
    // this half's per-layer norm weights, 1 KB per warp in the ring's third
    // slot (idle until the projection weights load)
    float* gns = (float*)(b_ring + 2 * kBBytes + ew * 1024);
    ((float4*)gns)[2 * lane] = gn0;
    ((float4*)gns)[2 * lane + 1] = gn1;
    __syncwarp();
    float gmax = 0.0f;
    if (ok) {
      if (lane == 0) {
        issue(&map_pl, st1, 0, c0);
        issue(&map_pl, st1 + 4096, 1, c0 + 32);
      }
      float m4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      uint32_t cur[32], nxt[32];
      tmem_ld32_nowait(taddr, nxt);
      tmem_take_chunk(cur, nxt);
#pragma unroll 1
      for (int q = 0; q < kChunks; ++q) {
        tmem_prefetch_chunk<kChunks>(taddr, q, nxt);
        const int b = q & 1;
        const bool got = __all_sync(0xffffffffu, arrived(b));
        ok = ok && got;
        float x[32], g[32];
        read_row(st1 + b * 4096, q < 4 ? gi0 : gi1, x);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const float4 w = *(const float4*)(gns + q * 32 + 4 * u);
          const float ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int j = 4 * u + k;
            g[j] = gelu_tanh(__uint_as_float(cur[j]) * ai) * __fmul_rn(__fmul_rn(x[j], ar), ws[k]);
            m4[k] = fmax_abs_nan(m4[k], g[j]);
          }
        }
        tmem_st32(taddr + q * 32, g);
        fence_async_smem();
        __syncwarp();  // every lane has read buffer b
        if (lane == 0 && q + 2 < kChunks) issue(&map_pl, st1 + b * 4096, b, c0 + (q + 2) * 32);
        tmem_take_chunk(cur, nxt);
      }
      tmem_st_wait();
      gmax = fmax_abs_nan(fmax_abs_nan(m4[0], m4[1]), fmax_abs_nan(m4[2], m4[3]));
    }
    if (!live) gmax = 0.0f;
    xchg[half * kRows + rl] = gmax;
    epi_sync<2>();
    const float rmax = fmax_abs_nan(xchg[rl], xchg[kRows + rl]);
    bad |= live && !(rmax <= 3.0e38f);
    float gs, ginv;
    pow2_row_scale(rmax, gs, ginv);
    if (ok) {
      uint32_t cur[32], nxt[32];
      tmem_ld32_nowait(taddr, nxt);
      tmem_take_chunk(cur, nxt);
#pragma unroll 1
      for (int q = 0; q < kChunks; ++q) {
        tmem_prefetch_chunk<kChunks>(taddr, q, nxt);
        uint32_t w[16];
#pragma unroll
        for (int m = 0; m < 16; ++m)
          w[m] = pack_half2(__uint_as_float(cur[2 * m]) * gs, __uint_as_float(cur[2 * m + 1]) * gs);
        // column c0 + 32q of the gated row is K element c0 + 32q of the
        // projection: K chunk (c0 + 32q) / 64, 16-byte units from
        // ((c0 + 32q) % 64) / 8 on, XOR-swizzled by row % 8 (the SW128
        // K-major layout the MMA reads)
        const int kcol = c0 + q * 32;
        uint8_t* rowp = a_region + (kcol / kChunkK) * kABytes + rl * 128;
        const int u0 = (kcol % kChunkK) / 8;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          *(uint4*)(rowp + (((u0 + k) ^ (rl & 7)) * 16)) = make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
        tmem_take_chunk(cur, nxt);
      }
    }
    tc_fence_before();    // this thread's accumulator reads are done
    fence_async_smem();   // its gated rows and staging reads precede the async proxy's
    mbar_arrive(g_ready);

    // ---- epilogue 2: delta = acc * ginv * w_proj scale; residual, layer
    // scalar, next pre-norm (the A tile is free: its staging; the weight ring
    // is idle: its row exchanges)
    ok = mbar_wait(d_full, 1, p.err) && ok;
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    ResidualArgs ra{};
    ra.T = p.T;
    ra.hidden = p.hidden;
    ra.w_post = p.w_post;
    ra.layer_scalar = p.layer_scalar;
    ra.apply_scalar = 1;
    ra.w_next = p.w_next;
    ra.eps = p.eps;
    ra.xn_inv_out = p.xn_inv_out;
    ra.err = p.err;
    residual_epilogue<kOutNormNext, 2>(ra, &map_h, &map_y, ginv * *p.w_proj_inv, ok, taddr, a_region + ew * 8192,
                                    (float*)b_ring, cw, (float*)(b_ring + kWeightsOff + ew * 2048), lb, lphase,
                                    lane, half, rl, row, y0, c0, bad);
    if (bad) atomicOr(p.err, SVL_DEVERR_NONFINITE);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

// gemm_residual_kernel: an N = 512 projection fused with the residual step
// that follows it -- the attention output projection (text.rs:424-433, then
// the pre-FF norm) and the FFN down projection (text.rs:458-472, then the
// PLE block's copy of the stream).  A ([T, K] FP16, K = 1024..) streams
// through a 4-slot ring of 128 x 64 slices beside a 4-slot ring of 256 x 64
// weight slices; per K slice two MMAs (N = 256 each) fill the row's two
// accumulator halves; after the last one the residual epilogue runs.  Its
// 4 x kParts warps split each row into kParts column parts: with 8 warps the
// A ring is their staging and the weight ring their row exchange, with 16
// the weight ring (128 KB) their staging and the A ring their row exchange.
constexpr int kRingA = 4, kRingB = 4;
constexpr int kGrBarBytes = 512;  // up to 49 mbarriers and the TMEM address
constexpr int kGrSmem = kRingA * kABytes + kRingB * kBBytes + kGrBarBytes + 1024;
static_assert((2 * kRingA + 2 * kRingB + 1 + 32) * 8 + 4 <= kGrBarBytes, "barrier area");
static_assert(kGrSmem <= 232448, "shared memory");
static_assert(16 * 8192 <= kRingB * kBBytes && 8 * 8192 <= kRingA * kABytes, "epilogue staging");
static_assert(xchg_bytes<4>() + 16 * 1024 <= kRingA * kABytes && xchg_bytes<2>() + 8 * 2048 <= kRingB * kBBytes,
              "row exchange and column weights");

template <int kParts>
constexpr int gr_threads() {
  return 64 + 128 * kParts;  // warp 0 TMA, warp 1 MMA, 4 kParts epilogue warps
}

struct GemmResidualParams {
  int K;
  const float* a_inv;     // [T] A row scales (NULL: 1)
  const float* w_inv;     // device scalar: the weight's inverse scale
  ResidualArgs res;
};

template <int OUT, int kParts>
__global__ void __launch_bounds__(gr_threads<kParts>(), 1)
    gemm_residual_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_w,
                         const __grid_constant__ CUtensorMap map_h, const __grid_constant__ CUtensorMap map_y,
                         GemmResidualParams p) {
  extern __shared__ uint8_t smem_raw[];
  pdl_trigger();
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* a_ring = smem;
  uint8_t* b_ring = smem + kRingA * kABytes;
  uint64_t* bars = (uint64_t*)(b_ring + kRingB * kBBytes);
  uint64_t* a_full = bars;
  uint64_t* a_empty = a_full + kRingA;
  uint64_t* b_full = a_empty + kRingA;
  uint64_t* b_empty = b_full + kRingB;
  uint64_t* d_full = b_empty + kRingB;
  uint64_t* ld_bar = d_full + 1;  // [8 kParts]: two staging loads per epilogue warp
  uint32_t* tmem_slot = (uint32_t*)(ld_bar + 8 * kParts);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * kRows;
  const int nk = p.K / kChunkK;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kRingA; ++i) {
      mbar_init(&a_full[i], 1);
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < kRingB; ++i) {
      mbar_init(&b_full[i], 1);
      mbar_init(&b_empty[i], 1);
    }
    mbar_init(d_full, 1);
    for (int b = 0; b < 8 * kParts; ++b) mbar_init(&ld_bar[b], 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_w);
    tma_prefetch_desc(&map_h);
    tma_prefetch_desc(&map_y);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // A, the residual rows and the row scales are complete from here

  if (warp == 0) {
    if (lane == 0) {
      int sa = 0, sb = 0;
      uint32_t pa = 0, pb = 0;
      bool ok = true;
      for (int j = 0; ok && j < nk; ++j) {
        if (!mbar_wait(&a_empty[sa], pa ^ 1, p.res.err)) break;
        mbar_arrive_expect_tx(&a_full[sa], kABytes);
        tma_load_2d(a_ring + sa * kABytes, &map_a, &a_full[sa], j * kChunkK, row0);
        if (++sa == kRingA) {
          sa = 0;
          pa ^= 1;
        }
        for (int h = 0; h < 2; ++h) {
          if (!mbar_wait(&b_empty[sb], pb ^ 1, p.res.err)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&b_full[sb], kBBytes);
          tma_load_2d(b_ring + sb * kBBytes, &map_w, &b_full[sb], j * kChunkK, h * kHalfN);
          if (++sb == kRingB) {
            sb = 0;
            pb ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(kRows, kHalfN, 0);
      int sa = 0, sb = 0;
      uint32_t pa = 0, pb = 0;
      bool ok = true;
      for (int j = 0; ok && j < nk; ++j) {
        if (!mbar_wait(&a_full[sa], pa, p.res.err)) break;
        tc_fence_after();
        const uint32_t a_addr = smem_u32(a_ring + sa * kABytes);
        for (int h = 0; h < 2; ++h) {
          if (!mbar_wait(&b_full[sb], pb, p.res.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t b_addr = smem_u32(b_ring + sb * kBBytes);
          const uint32_t d = tmem_base + (uint32_t)(h * kHalfN);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_f16(d, sdesc(a_addr + k * 32, 16, 1024, kLayoutSW128), sdesc(b_addr + k * 32, 16, 1024, kLayoutSW128),
                    idesc, (j | k) != 0);
          mma_commit(&b_empty[sb]);
          if (++sb == kRingB) {
            sb = 0;
            pb ^= 1;
          }
        }
        mma_commit(&a_empty[sa]);
        if (++sa == kRingA) {
          sa = 0;
          pa ^= 1;
        }
      }
      if (ok) mma_commit(d_full);
    }
  } else {
    // epilogue warp ew: TMEM lanes (rows) 32 (warp % 4).., columns c0.. (its
    // part: every part has one warp of each lane group)
    constexpr int kSpan = kWidth / kParts;
    const int ew = warp - 2;
    const int lane_grp = warp & 3;
    const int part = ew >> 2;
    const int rl = lane_grp * 32 + lane;
    const int row = row0 + rl;
    const int y0 = row0 + lane_grp * 32;
    const int c0 = part * kSpan;
    const bool live = row < p.res.T;
    const uint32_t taddr = tmem_base + ((uint32_t)(lane_grp * 32) << 16) + (uint32_t)c0;
    const float dsc = (p.a_inv && live ? p.a_inv[row] : 1.0f) * *p.w_inv;  // before the accumulator wait
    const ColWeights<kSpan> cw =
        load_col_weights<kSpan>(p.res.w_post, OUT == kOutCopy ? p.res.w_post : p.res.w_next, c0, lane);
    // staging, row exchange and column weights in the rings the GEMM is done with
    uint8_t* stage_area = kParts == 2 ? a_ring : b_ring;
    uint8_t* xchg_area = kParts == 2 ? b_ring : a_ring;
    uint32_t lphase = 0;
    bool bad = false;
    bool ok = mbar_wait(d_full, 0, p.res.err);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    residual_epilogue<OUT, kParts>(p.res, &map_h, &map_y, dsc, ok, taddr, stage_area + ew * 8192, (float*)xchg_area,
                                   cw, (float*)(xchg_area + xchg_bytes<kParts>() + ew * 8 * kSpan), ld_bar + 2 * ew,
                                   lphase, lane, part, rl, row, y0, c0, bad);
    if (bad) atomicOr(p.res.err, SVL_DEVERR_NONFINITE);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

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

// A 2-D row-major tensor map: rows x cols elements of `bytes` (2: FP16,
// 4: FP32) with a row pitch of ld elements, boxes of box_cols x box_rows.
bool make_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld, int bytes,
              uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swz) {
  EncodeTiledFn enc = encode_fn();
  if (!enc || ((uintptr_t)base & 15) || (ld * bytes) % 16) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * bytes)};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t elem[2] = {1, 1};
  return enc(map, bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void*)base,
             dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

template <int kParts>
cudaError_t launch_residual_parts(int out, const CUtensorMap& ma, const CUtensorMap& mw, const CUtensorMap& mh,
                                  const CUtensorMap& my, const GemmResidualParams& p, unsigned blocks,
                                  cudaStream_t st) {
  const dim3 grid(blocks), block(gr_threads<kParts>());
  cudaError_t e;
  if (out == kOutNormNextBound) {
    static std::atomic<uint64_t> opted{0};
    if ((e = smem_opt_in(gemm_residual_kernel<kOutNormNextBound, kParts>, kGrSmem, &opted)) != cudaSuccess) return e;
    launch_pdl(gemm_residual_kernel<kOutNormNextBound, kParts>, grid, block, kGrSmem, st, ma, mw, mh, my, p);
  } else if (out == kOutCopy) {
    static std::atomic<uint64_t> opted{0};
    if ((e = smem_opt_in(gemm_residual_kernel<kOutCopy, kParts>, kGrSmem, &opted)) != cudaSuccess) return e;
    launch_pdl(gemm_residual_kernel<kOutCopy, kParts>, grid, block, kGrSmem, st, ma, mw, mh, my, p);
  } else {
    static std::atomic<uint64_t> opted{0};
    if ((e = smem_opt_in(gemm_residual_kernel<kOutNormNext, kParts>, kGrSmem, &opted)) != cudaSuccess) return e;
    launch_pdl(gemm_residual_kernel<kOutNormNext, kParts>, grid, block, kGrSmem, st, ma, mw, mh, my, p);
  }
  return cudaGetLastError();
}

}  // namespace

bool ple_block_supported(int hidden, int per_layer) { return hidden == kWidth && per_layer == kWidth; }

bool gemm_residual_supported(int hidden, int k) { return hidden == kWidth && k >= kChunkK && k % kChunkK == 0; }

cudaError_t launch_gemm_residual(const GemmResidualLaunch& g, cudaStream_t st) {
  const ResidualArgs& r = g.res;
  if (r.T <= 0) return cudaSuccess;
  if (!gemm_residual_supported(kWidth, g.K) || !aligned16(r.hidden) || !aligned16(r.w_post) ||
      (g.out != kOutCopy && !aligned16(r.w_next)) || !aligned16(g.out16) || (g.out == kOutNormNextBound && !r.bound_inv))
    return cudaErrorInvalidValue;
  CUtensorMap ma, mw, mh, my;
  const uint64_t T = (uint64_t)r.T;
  if (!make_map(&ma, g.a16, T, (uint64_t)g.K, (uint64_t)g.lda, 2, kChunkK, kRows, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map(&mw, g.w16, kWidth, (uint64_t)g.K, (uint64_t)g.K, 2, kChunkK, kHalfN, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map(&mh, r.hidden, T, kWidth, kWidth, 4, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map(&my, g.out16, T, kWidth, kWidth, 2, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B))
    return cudaErrorInvalidValue;
  GemmResidualParams p{};
  p.K = g.K;
  p.a_inv = g.a_inv;
  p.w_inv = g.w_inv;
  p.res = r;
  return launch_residual_parts<4>(g.out, ma, mw, mh, my, p, (unsigned)((r.T + kRows - 1) / kRows), st);
}

cudaError_t launch_ple_block(const PleBlockParams& p, cudaStream_t st) {
  if (p.T <= 0) return cudaSuccess;
  // the per-layer slice's FP16 boxes (16-byte row pitch), float4 weights and
  // residual rows, FP16 output rows
  if (p.ld_pl % 8 || !aligned16(p.per_layer16) || !p.pss || !p.pgi || !aligned16(p.hidden) || !aligned16(p.ple_norm) ||
      !aligned16(p.w_post) || !aligned16(p.w_next) || !aligned16(p.xn16_out))
    return cudaErrorInvalidValue;
  // operands: FP16 boxes of 64 elements (128 bytes) x rows, SWIZZLE_128B;
  // staged epilogue traffic: 32 x 32 boxes (the FP16 per-layer slice and
  // output rows: 64-byte rows, SWIZZLE_64B; FP32 residual rows: 128-byte
  // rows, SWIZZLE_128B)
  CUtensorMap ma, mg, mp, mpl, mh, my;
  const uint64_t T = (uint64_t)p.T;
  if (!make_map(&ma, p.xn16, T, kWidth, kWidth, 2, kChunkK, kRows, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map(&mg, p.w_gate16, kWidth, kWidth, kWidth, 2, kChunkK, kHalfN, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map(&mp, p.w_proj16, kWidth, kWidth, kWidth, 2, kChunkK, kHalfN, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map(&mpl, p.per_layer16, T, kWidth, (uint64_t)p.ld_pl, 2, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B) ||
      !make_map(&mh, p.hidden, T, kWidth, kWidth, 4, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map(&my, p.xn16_out, T, kWidth, kWidth, 2, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B))
    return cudaErrorInvalidValue;
  static std::atomic<uint64_t> opted{0};
  cudaError_t e = smem_opt_in(ple_block_kernel, kSmem, &opted);
  if (e != cudaSuccess) return e;
  launch_pdl(ple_block_kernel, dim3((unsigned)((p.T + kRows - 1) / kRows)), dim3(kThreads), kSmem, st, ma, mg, mp, mpl,
             mh, my, p);
  return cudaGetLastError();
}

}  // namespace svl

