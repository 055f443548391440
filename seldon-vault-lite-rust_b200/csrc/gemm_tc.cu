// gemm_tc.cu -- persistent, warp-specialised tcgen05 TF32 GEMMs for sm_100a.
//
// Two kernels share one structure (320 threads, one CTA per SM):
//   warp 0      TMA producer: A and B K-slices (32 FP32 = 128 B, SWIZZLE_128B)
//               into a shared-memory ring;
//   warp 1      TMEM allocator and single-thread tcgen05.mma issuer;
//   warps 2..9  epilogue: tcgen05.ld of the FP32 accumulator (warp w owns TMEM
//               lanes 32 * (w % 4) .. and half of the tile's columns, so each
//               SM sub-partition runs two epilogue warps), the fused epilogue
//               math, and a TMA store of every 32 x 32 chunk out of a
//               per-warp swizzled staging buffer (coalesced, edge-clipped).
// Two TMEM accumulators let the epilogue of tile i overlap the MMAs of tile
// i + 1; tiles are walked n-fastest so concurrent CTAs share A rows in L2.
//   * gemm_tf32_kernel<BN>: one CTA per 128 x BN tile (M = 128 MMAs);
//   * gemm_pair_tf32_kernel: a CTA pair per 256 x 256 tile (cta_group::2,
//     M = 256 MMAs), used whenever M >= 256 and N >= 256.
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
// Epilogue staging: one 32 x 32 FP32 chunk (4 KB) per epilogue warp (a second
// buffer per warp measured no faster and costs a pipeline stage).
template <int BN>
struct Cfg {
  static constexpr int STAGES = BN == 256 ? 4 : 6;
  static constexpr int STAGING_BUFS = 1;
  static constexpr int STAGING_BYTES = 8 * 4096 * STAGING_BUFS;
  static constexpr int A_BYTES = BM * BK * 4;
  static constexpr int B_BYTES = BN * BK * 4;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int SMEM = STAGES * STAGE_BYTES + STAGING_BYTES + 1024 /*align*/ + 512 /*barriers*/;
  static constexpr uint32_t TMEM_COLS = 2 * BN;
  static_assert(SMEM <= 232448, "shared memory");
};

// Epilogue of one accumulator tile for one warp: its 32 rows (lane = row,
// first row `row0`), column chunks [c_begin, c_end) of 32 starting at tile
// column n0 (for GeGLU, the tile's first B row; its gate chunks c pair with
// up chunks c + tile_n / 64).  taddr = TMEM address of this warp's lanes,
// column 0 of the accumulator.

// Per-row factors of an epilogue, read before the accumulator is waited on
// (global loads issued after the wait cost ~1000 cycles per tile):
//   ai  the A row's inverse operand scale times B's (1 for FP32 operands);
//   os  1 / out_inv[row] of FP16 GeGLU / PLE-gate outputs.
//   ar  the PLE aux row's RMSNorm inverse (aux_row_inv), 1 without.
struct RowScales {
  float ai, os, ar;
};
SVL_DEV RowScales row_scales(const GemmParams& p, int row) {
  RowScales r;
  r.ai = ((p.a_inv && row < p.M) ? p.a_inv[row] : 1.0f) * (p.b_scale ? *p.b_scale : 1.0f);
  r.os = (p.out_inv && row < p.M) ? 1.0f / p.out_inv[row] : 1.0f;
  r.ar = (p.aux_row_inv && row < p.M) ? p.aux_row_inv[(size_t)row * p.aux_row_stride] : 1.0f;
  return r;
}

// An accumulator value (raw TMEM word w) with the operand scales undone
// exactly: FP16 operands carry power-of-two scales (ai = 1 for FP32
// operands, a multiplication by one).
SVL_DEV float unscale1(const GemmParams&, float ai, uint32_t w, int) { return __uint_as_float(w) * ai; }
SVL_DEV void unscale32(const GemmParams& p, float ai, const uint32_t* r, int brow0, float* x) {
#pragma unroll
  for (int j = 0; j < 32; ++j) x[j] = unscale1(p, ai, r[j], brow0 + j);
}

// Issues up to four 32-column TMEM loads (cols[q] < 0: none), waits once and
// ties the registers to the wait: one TMEM round trip for a warp's whole
// share of the tile (each load alone waits ~900 cycles while the tensor core
// is writing the other accumulator).
SVL_DEV void tmem_ld_group(uint32_t taddr, const int (&cols)[4], uint32_t* r) {
#pragma unroll
  for (int q = 0; q < 4; ++q)
    if (cols[q] >= 0) tmem_ld32_nowait(taddr + cols[q], r + q * 32);
  tmem_ld_wait();
#pragma unroll
  for (int q = 0; q < 4; ++q) tmem_regs_after_wait(r + q * 32);
}

// PLE-gate epilogue: TMA load of one 32 x 32 FP32 aux chunk (x, y) into a
// 4 KB staging buffer, completing on `bar` (lane 0).
SVL_DEV void ple_issue_aux(const CUtensorMap* map_aux, uint64_t* bar, float* buf, int32_t x, int32_t y) {
  mbar_arrive_expect_tx(bar, 32 * 32 * 4);
  tma_load_2d(buf, map_aux, bar, x, y);
}

// Issues the FP16 PLE-gate epilogue's first aux chunk (and, with two staging
// buffers, the second) of the warp's share [c_begin, c_end) before the
// accumulator wait, once earlier stores have read the buffers (lane 0).
SVL_DEV void ple_first_aux(const GemmParams& p, const CUtensorMap* map_aux, uint64_t* abar, const Staging& sg, int n0,
                           int row0, int c_begin, int c_end, int lane) {
  const int c_last = (p.N - n0 + 31) / 32 < c_end ? (p.N - n0 + 31) / 32 : c_end;
  if (lane == 0 && c_begin < c_last) {
    tma_store_wait_read();
    ple_issue_aux(map_aux, &abar[0], sg.base, n0 + c_begin * 32, row0);
    if (sg.nbufs > 1 && c_begin + 1 < c_last)
      ple_issue_aux(map_aux, &abar[1], sg.base + 1024, n0 + (c_begin + 1) * 32, row0);
  }
}

// Epilogue of one accumulator tile for one warp (see above).  `release()`
// hands the accumulator back to the MMA warp; the epilogues that hold their
// whole share in registers call it before storing, the others when done.
template <int EPI, class Release>
SVL_DEV void epilogue_chunks(const GemmParams& p, const CUtensorMap* map_c, const CUtensorMap* map_aux, uint64_t* abar,
                             uint32_t& aphase, Staging& sg, uint32_t taddr, int row0, int n0, int tile_n, int c_begin,
                             int c_end, int lane, RowScales rs, Release&& release) {
  float v[32];
  const float ai = rs.ai;
  // Accumulator columns [col, col + 32) of this lane's row, B rows brow0..
  auto ld = [&](int col, int brow0, float* x) {
    uint32_t r[32];
    tmem_ld32_nowait(taddr + col, r);
    tmem_ld_wait();
    tmem_regs_after_wait(r);
    unscale32(p, ai, r, brow0, x);
  };
  if constexpr (EPI == kEpiQkv || EPI == kEpiQkv16) {
    // The tile is one 256-wide head (text.rs:353-405): pass 1 sums the squares
    // of the row's 256 values, pass 2 normalises the rotate-half pairs
    // (p, p + 128) held in chunks (c, c + 4) and applies RoPE to q and k.
    const int head = n0 / 256;
    const bool is_q = head < p.nh, is_k = !is_q && head < p.nh + p.kvh;
    const float* w = is_q ? p.q_norm : (is_k ? p.k_norm : nullptr);
    float ss = 0.0f;
    if constexpr (EPI == kEpiQkv16) {
      // four chunks per TMEM round trip; four interleaved partial sums (a
      // 256-long dependent add chain cost ~1,000 cycles per tile), combined
      // in a fixed order so both warps of a row agree
      float sp[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 1
      for (int c4 = 0; c4 < 8; c4 += 4) {
        uint32_t o[128];
        const int cols[4] = {c4 * 32, (c4 + 1) * 32, (c4 + 2) * 32, (c4 + 3) * 32};
        tmem_ld_group(taddr, cols, o);
        // one FMA per value: the raw accumulator's squares, scaled once below
        // by ai^2 (ai a power of two)
#pragma unroll
        for (int j = 0; j < 128; ++j) {
          const float x = __uint_as_float(o[j]);
          sp[j & 3] = fmaf(x, x, sp[j & 3]);
        }
      }
      ss = ((sp[0] + sp[1]) + (sp[2] + sp[3])) * (ai * ai);
    } else {
#pragma unroll 1
      for (int c = 0; c < 8; ++c) {
        ld(c * 32, n0 + c * 32, v);
#pragma unroll
        for (int j = 0; j < 32; ++j) ss = __fadd_rn(ss, __fmul_rn(v[j], v[j]));
      }
    }
    const float inv = 1.0f / sqrtf(__fadd_rn(ss / 256.0f, p.eps));
    const int row = row0 + lane;
    // rope is [pair][position]: the warp's lanes (consecutive tokens) read adjacent entries
    const float2* cs = p.rope + (row < p.M ? p.pos_of[row] : 0);
    const size_t stride = (size_t)p.rope_stride;
    bool bad = !isfinite(ss);
    // normalised (and rotated) pair (a, b) of rotate-half partners p, p + 128
    auto finish = [&](int pi, float& a, float& b) {
      a = __fmul_rn(a, inv);
      b = __fmul_rn(b, inv);
      if (w) {
        a = __fmul_rn(a, w[pi]);
        b = __fmul_rn(b, w[128 + pi]);
        const float2 t = cs[pi * stride];  // (cos, sin)
        const float r0 = __fsub_rn(__fmul_rn(a, t.x), __fmul_rn(b, t.y));
        const float r1 = __fadd_rn(__fmul_rn(a, t.y), __fmul_rn(b, t.x));
        a = r0;
        b = r1;
      }
    };
    if constexpr (EPI == kEpiQkv16) {
      // per chunk: 32 FP16 columns = one 64-byte row per lane, q/k/v values in
      // the first 2 KB of the staging buffer, their rotate-half partners in
      // the second (SWIZZLE_64B: 16-byte unit ^= (row / 2) % 4)
#pragma unroll 1
      for (int c = c_begin; c < c_end; ++c) {
        // (cos, sin) of the chunk's 32 pairs for this row, issued before the
        // TMEM load so their L2 latency overlaps it (one load per pair inside
        // the loop below left ~80 cycles per pair waiting on L2)
        float2 t[32];
        if (w) {
#pragma unroll
          for (int j = 0; j < 32; ++j) t[j] = cs[(size_t)(c * 32 + j) * stride];
        }
        uint32_t o[64];  // chunks c and c + 4 in one TMEM round trip
        tmem_ld32_nowait(taddr + c * 32, o);
        tmem_ld32_nowait(taddr + (c + 4) * 32, o + 32);
        tmem_ld_wait();
        tmem_regs_after_wait(o);
        tmem_regs_after_wait(o + 32);
        // ai is a power of two: (acc * ai) * inv == acc * (ai * inv) exactly
        const float sc = ai * inv;
        float amax = 0.0f;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int pi = c * 32 + j;
          float a = __fmul_rn(__uint_as_float(o[j]), sc);
          float b = __fmul_rn(__uint_as_float(o[32 + j]), sc);
          if (w) {
            a = __fmul_rn(a, w[pi]);
            b = __fmul_rn(b, w[128 + pi]);
            // the rotation with one rounding per output (FMA): the FP16
            // store that follows rounds 13 bits more
            const float r0 = fmaf(a, t[j].x, -(b * t[j].y));
            const float r1 = fmaf(a, t[j].y, b * t[j].x);
            a = r0;
            b = r1;
          }
          amax = fmax_abs_nan(fmax_abs_nan(amax, a), b);
          o[j] = __float_as_uint(a);
          o[32 + j] = __float_as_uint(b);
        }
        // FP16 holds |x| <= 65504: anything larger is reported, not stored as inf
        bad |= !(amax <= 65504.0f);
        // packed pairs over the words just read (j <= 2j)
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          o[j] = pack_half2(__uint_as_float(o[2 * j]), __uint_as_float(o[2 * j + 1]));
          o[32 + j] = pack_half2(__uint_as_float(o[32 + 2 * j]), __uint_as_float(o[32 + 2 * j + 1]));
        }
        const uint32_t* pv = o;
        const uint32_t* pu = o + 32;
        float* stage = sg.acquire(lane);
        uint8_t* ra = (uint8_t*)stage + lane * 64;
        uint8_t* rb = ra + 2048;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int off = (k ^ ((lane >> 1) & 3)) * 16;
          *(uint4*)(ra + off) = make_uint4(pv[4 * k], pv[4 * k + 1], pv[4 * k + 2], pv[4 * k + 3]);
          *(uint4*)(rb + off) = make_uint4(pu[4 * k], pu[4 * k + 1], pu[4 * k + 2], pu[4 * k + 3]);
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(map_c, stage, n0 + c * 32, row0);
          tma_store_2d(map_c, (uint8_t*)stage + 2048, n0 + 128 + c * 32, row0);
          tma_store_commit();
        }
        sg.release();
      }
      if (bad && row < p.M) atomicOr(p.err, SVL_DEVERR_NONFINITE);
      return;
    } else {
    float u[32];
#pragma unroll 1
    for (int c = c_begin; c < c_end; ++c) {
      ld(c * 32, n0 + c * 32, v);
      ld((c + 4) * 32, n0 + (c + 4) * 32, u);
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        finish(c * 32 + j, v[j], u[j]);
        bad |= !isfinite(v[j]) || !isfinite(u[j]);
        v[j] = round_tf32(v[j]);
        u[j] = round_tf32(u[j]);
      }
      store_chunk_tma(map_c, sg.acquire(lane), v, lane, n0 + c * 32, row0);
      sg.release();
      store_chunk_tma(map_c, sg.acquire(lane), u, lane, n0 + 128 + c * 32, row0);
      sg.release();
    }
    if (bad && row < p.M) atomicOr(p.err, SVL_DEVERR_NONFINITE);
    }
  } else if constexpr (EPI == kEpiGeglu16) {
    // FP16 rows of 64 bytes (SWIZZLE_64B: 16-byte unit ^= (row / 2) % 4), the
    // value scaled by the row's power of two (a bound on the whole row).  The
    // warp's (at most two) gate / up chunk pairs are read in one TMEM round
    // trip and the accumulator is released before any store.
    const int f0 = n0 / 2;
    const int row = row0 + lane;
    const float os = rs.os;
    float amax = 0.0f;  // largest |output| (NaN if any)
    const int nch = c_end - c_begin;  // <= 2
    uint32_t r[128];
    const int cols[4] = {nch > 0 ? c_begin * 32 : -1, nch > 0 ? tile_n / 2 + c_begin * 32 : -1,
                         nch > 1 ? (c_begin + 1) * 32 : -1, nch > 1 ? tile_n / 2 + (c_begin + 1) * 32 : -1};
    tmem_ld_group(taddr, cols, r);
    release();
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int c = c_begin + q;
      const int col0 = f0 + c * 32;
      if (q < nch && col0 < p.n_out) {
        // the packed FP16 pairs overwrite gate words already read (j / 2 <= j)
        uint32_t* g = r + q * 64;
        const uint32_t* up = g + 32;
        const float aos = ai * os;  // powers of two: (u * ai) * os == u * (ai * os)
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const float r0 = gelu_tanh(__uint_as_float(g[j]) * ai) * (__uint_as_float(up[j]) * aos);
          const float r1 = gelu_tanh(__uint_as_float(g[j + 1]) * ai) * (__uint_as_float(up[j + 1]) * aos);
          amax = fmax_abs_nan(fmax_abs_nan(amax, r0), r1);
          g[j / 2] = pack_half2(r0, r1);
        }
        store_row64_f16(map_c, sg, g, lane, col0, row0);
      }
    }
    // FP16 holds |x| <= 65504: anything larger is reported, not stored as inf
    if (!(amax <= 65504.0f) && row < p.M) atomicOr(p.err, SVL_DEVERR_NONFINITE);
  } else if constexpr (EPI == kEpiGeglu) {
    float u[32];
    const int f0 = n0 / 2;
#pragma unroll 1
    for (int c = c_begin; c < c_end; ++c) {
      ld(c * 32, n0 + c * 32, v);
      ld(tile_n / 2 + c * 32, n0 + tile_n / 2 + c * 32, u);
      const int col0 = f0 + c * 32;
      if (col0 < p.n_out) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float r = gelu_tanh(v[j]) * u[j];
          v[j] = p.round_out ? round_tf32(r) : r;
        }
        store_chunk_tma(map_c, sg.acquire(lane), v, lane, col0, row0);
        sg.release();
      }
    }
  } else if constexpr (EPI == kEpiPleGate16) {
    // gelu(acc) * aux in FP16 (64-byte rows, SWIZZLE_64B, scaled by the row's
    // power of two) over the warp's (at most four) 32 x 32 chunks.  Each aux
    // chunk comes by TMA straight into a staging buffer (128-byte swizzled
    // FP32 rows): the caller issued the first one (two, with two buffers)
    // before waiting for the accumulator, so they load during the MMAs; a
    // buffer's next aux chunk is issued once its FP16 store has read it.
    // abar[b] is buffer b's barrier, aphase bit b its phase.
    const int row = row0 + lane;
    const bool two = sg.nbufs > 1;
    const int c_last = (p.N - n0 + 31) / 32 < c_end ? (p.N - n0 + 31) / 32 : c_end;  // chunks inside N
    const int nch = c_last - c_begin;  // <= 4
    const float os = rs.os;
    float amax = 0.0f;  // largest |output| (NaN if any)
#pragma unroll 1
    for (int q = 0; q < nch; ++q) {
      {
        const int c = c_begin + q;
        uint32_t w[32];
        tmem_ld32_nowait(taddr + c * 32, w);
        tmem_ld_wait();
        tmem_regs_after_wait(w);
        const int b = two ? (q & 1) : 0;
        uint8_t* stage = (uint8_t*)(sg.base + b * 1024);
        if (!two && q > 0 && lane == 0) {
          tma_store_wait_read();  // the previous chunk's store has read the buffer
          ple_issue_aux(map_aux, &abar[0], sg.base, n0 + c * 32, row0);
        }
        const bool got = mbar_wait(&abar[b], (aphase >> b) & 1u, p.err);
        aphase ^= 1u << b;
        __syncwarp();
        if (!__all_sync(0xffffffffu, got)) return;
        // read the row's aux values (RMS-normalised here when the producer
        // left them raw: (x * inv) * w, the norm kernel's own order), then
        // write the FP16 row over the first half of the same buffer (packed
        // pairs reuse the chunk's words)
        const uint8_t* srow = stage + lane * 128;
        const float4* cw = p.aux_col_w ? (const float4*)(p.aux_col_w + n0 + c * 32) : nullptr;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          float4 x = *(const float4*)(srow + ((u ^ (lane & 7)) * 16));
          if (cw) {
            const float4 g = cw[u];
            x = make_float4(__fmul_rn(__fmul_rn(x.x, rs.ar), g.x), __fmul_rn(__fmul_rn(x.y, rs.ar), g.y),
                            __fmul_rn(__fmul_rn(x.z, rs.ar), g.z), __fmul_rn(__fmul_rn(x.w, rs.ar), g.w));
          }
          const float r0 = gelu_tanh(__uint_as_float(w[4 * u]) * ai) * (x.x * os);
          const float r1 = gelu_tanh(__uint_as_float(w[4 * u + 1]) * ai) * (x.y * os);
          const float r2 = gelu_tanh(__uint_as_float(w[4 * u + 2]) * ai) * (x.z * os);
          const float r3 = gelu_tanh(__uint_as_float(w[4 * u + 3]) * ai) * (x.w * os);
          amax = fmax_abs_nan(fmax_abs_nan(fmax_abs_nan(fmax_abs_nan(amax, r0), r1), r2), r3);
          w[2 * u] = row < p.M ? pack_half2(r0, r1) : 0u;
          w[2 * u + 1] = row < p.M ? pack_half2(r2, r3) : 0u;
        }
        __syncwarp();  // every lane has read its aux row before the buffer is overwritten
#pragma unroll
        for (int k = 0; k < 4; ++k)
          *(uint4*)(stage + lane * 64 + ((k ^ ((lane >> 1) & 3)) * 16)) =
              make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(map_c, stage, n0 + c * 32, row0);
          tma_store_commit();
          if (two && q + 2 < nch) {
            tma_store_wait_read();  // that store has read the buffer
            ple_issue_aux(map_aux, &abar[b], sg.base + b * 1024, n0 + (c + 2) * 32, row0);
          }
        }
      }
    }
    if (!(amax <= 65504.0f) && row < p.M) atomicOr(p.err, SVL_DEVERR_NONFINITE);
  } else if constexpr (EPI == kEpiPleGate) {
    // gelu(acc) * aux over the warp's 32 x 32 chunks: each aux chunk comes by
    // TMA straight into a staging buffer (the same 128-byte swizzled rows the
    // output store uses); with two buffers the next chunk's load is in flight
    // while this one is computed and stored.  abar[b] (buffer b's barrier),
    // aphase bit b its phase.
    const int row = row0 + lane;
    const bool two = sg.nbufs > 1;
    auto issue_aux = [&](int c, int b) {  // lane 0
      mbar_arrive_expect_tx(&abar[b], 32 * 32 * 4);
      tma_load_2d(sg.base + b * 1024, map_aux, &abar[b], n0 + c * 32, row0);
    };
    const int c_last = (p.N - n0 + 31) / 32 < c_end ? (p.N - n0 + 31) / 32 : c_end;  // chunks inside N
    if (two && c_begin < c_last) {
      if (lane == 0) {
        tma_store_wait_read();  // earlier stores are done with both buffers
        issue_aux(c_begin, 0);
      }
      __syncwarp();
    }
#pragma unroll 1
    for (int c = c_begin; c < c_last; ++c) {
      const int col0 = n0 + c * 32;
      const int b = two ? (c - c_begin) & 1 : 0;
      float* stage;
      if (two) {
        stage = sg.base + b * 1024;
        if (c + 1 < c_last && lane == 0) {
          tma_store_wait_read();  // the other buffer's store (previous chunk) has read it
          issue_aux(c + 1, b ^ 1);
        }
      } else {
        stage = sg.acquire(lane);
        if (lane == 0) issue_aux(c, 0);
      }
      ld(c * 32, col0, v);
      const bool got = mbar_wait(&abar[b], (aphase >> b) & 1u, p.err);
      aphase ^= 1u << b;
      __syncwarp();
      if (!__all_sync(0xffffffffu, got)) return;
      uint8_t* srow = (uint8_t*)stage + lane * 128;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        float4* q = (float4*)(srow + ((u ^ (lane & 7)) * 16));
        const float4 x = *q;
        const float xs[4] = {x.x, x.y, x.z, x.w};
        float o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float r = row < p.M ? gelu_tanh(v[4 * u + k]) * xs[k] : 0.0f;
          o[k] = p.round_out ? round_tf32(r) : r;
        }
        *q = make_float4(o[0], o[1], o[2], o[3]);
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(map_c, stage, col0, row0);
        tma_store_commit();
      }
      if (!two) sg.release();
    }
  } else if constexpr (EPI == kEpiStore16) {
    // FP16 rows with one power-of-two scale per (row, 128-column group): the
    // warp's share is exactly one group (N % 128 == 0); its inverse scale
    // goes to group_inv and, with row_ss, the unscaled values' sum of squares
    const int nch = c_end - c_begin;  // <= 4
    uint32_t r[128];
    const int cols[4] = {nch > 0 ? c_begin * 32 : -1, nch > 1 ? (c_begin + 1) * 32 : -1,
                         nch > 2 ? (c_begin + 2) * 32 : -1, nch > 3 ? (c_begin + 3) * 32 : -1};
    tmem_ld_group(taddr, cols, r);
    release();
    const int row = row0 + lane;
    float ss = 0.0f, mx = 0.0f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int col0 = n0 + (c_begin + q) * 32;
      const bool in = q < nch && col0 < p.N;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float x = in ? unscale1(p, ai, r[q * 32 + j], col0 + j) * p.alpha : 0.0f;
        ss = fmaf(x, x, ss);
        mx = fmax_abs_nan(mx, x);
        r[q * 32 + j] = __float_as_uint(x);
      }
    }
    float sc, inv;
    pow2_row_scale(mx, sc, inv);
    if (!(mx <= 3.0e38f) && row < p.M) atomicOr(p.err, SVL_DEVERR_NONFINITE);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int col0 = n0 + (c_begin + q) * 32;
      if (q < nch && col0 < p.N) {
        uint32_t w[16];
#pragma unroll
        for (int m = 0; m < 16; ++m)
          w[m] = pack_half2(__uint_as_float(r[q * 32 + 2 * m]) * sc, __uint_as_float(r[q * 32 + 2 * m + 1]) * sc);
        store_row64_f16(map_c, sg, w, lane, col0, row0);
      }
    }
    if (nch > 0 && row < p.M && n0 + c_begin * 32 < p.N) {
      const size_t g = (size_t)row * p.row_ss_stride + (n0 + c_begin * 32) / 128;
      p.group_inv[g] = inv;
      if (p.row_ss) p.row_ss[g] = ss;
    }
  } else {
    // the warp's (at most four) chunks in one TMEM round trip; the
    // accumulator is released before any store
    const int nch = c_end - c_begin;  // <= 4
    uint32_t r[128];
    const int cols[4] = {nch > 0 ? c_begin * 32 : -1, nch > 1 ? (c_begin + 1) * 32 : -1,
                         nch > 2 ? (c_begin + 2) * 32 : -1, nch > 3 ? (c_begin + 3) * 32 : -1};
    tmem_ld_group(taddr, cols, r);
    release();
    float ss = 0.0f;  // the stored values' sum of squares (row_ss)
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int col0 = n0 + (c_begin + q) * 32;
      if (q < nch && col0 < p.N) {
        uint32_t* w = r + q * 32;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          float x = unscale1(p, ai, w[j], col0 + j) * p.alpha;
          x = p.round_out ? round_tf32(x) : x;
          ss = fmaf(x, x, ss);
          w[j] = __float_as_uint(x);
        }
        store_chunk_tma(map_c, sg.acquire(lane), w, lane, col0, row0);
        sg.release();
      }
    }
    if (p.row_ss && nch > 0 && row0 + lane < p.M && n0 + c_begin * 32 < p.N)
      p.row_ss[(size_t)(row0 + lane) * p.row_ss_stride + (n0 + c_begin * 32) / 128] = ss;
  }
}

// F16: FP16 operands (kind::f16, K = 64 elements per stage) instead of FP32
// (kind::tf32, 32 per stage); a compile-time choice, since a runtime branch
// in the single-thread MMA and TMA loops cost ~25% of the GEMM's time.
template <int BN, int EPI, bool F16>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tf32_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                     const __grid_constant__ CUtensorMap map_c, const __grid_constant__ CUtensorMap map_aux,
                     GemmParams p) {
  using C = Cfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  pdl_trigger();
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  float* staging = (float*)(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* full = (uint64_t*)(smem + C::STAGES * C::STAGE_BYTES + C::STAGING_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tmem_full = empty + C::STAGES;
  uint64_t* tmem_empty = tmem_full + 2;
  uint64_t* aux_full = tmem_empty + 2;  // [16]: two per epilogue warp (PLE gate aux loads)
  uint32_t* tmem_slot = (uint32_t*)(aux_full + 16);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (p.M + BM - 1) / BM;
  const int num_n = (p.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  constexpr int bk = F16 ? 64 : BK;  // elements per 128-byte swizzle row
  const int num_k = (p.K + bk - 1) / bk;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], 8);  // one arrival per epilogue warp
    }
    for (int w = 0; w < 16; ++w) mbar_init(&aux_full[w], 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
    tma_prefetch_desc(&map_c);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // the previous kernel's outputs (A, row scales) are complete from here

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
          tma_load_2d(sa, &map_a, &full[stage], kb * bk, m0);
          tma_load_2d(sa + C::A_BYTES, &map_b, &full[stage], kb * bk, n0);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = F16 ? idesc_f16(BM, BN, 0) : idesc_tf32(BM, BN, 0);
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
          // four MMAs of 32 bytes of K each: K = 8 TF32 or 16 FP16 elements
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t ad = sdesc(a_addr + k * 32, 16, 1024, kLayoutSW128);
            const uint64_t bd = sdesc(b_addr + k * 32, 16, 1024, kLayoutSW128);
            if constexpr (F16)
              mma_f16(d, ad, bd, idesc, (kb | k) != 0);
            else
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
    const int lane_grp = warp & 3;
    const int half = (warp - 2) >> 2;  // warps 2..5: first half of the columns, 6..9: second
    Staging sg{staging + (warp - 2) * 1024 * C::STAGING_BUFS, C::STAGING_BUFS};
    uint32_t aphase = 0;
    const int chunks = (EPI == kEpiGeglu || EPI == kEpiGeglu16 || EPI == kEpiQkv || EPI == kEpiQkv16) ? BN / 64 : BN / 32;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const int m0 = (tile / num_n) * BM;
      const int n0 = (tile % num_n) * BN;
      if constexpr (EPI == kEpiPleGate || EPI == kEpiPleGate16) {
        // pull this warp's aux chunks into L2 while the tile's MMAs run
        if (lane == 0)
          for (int c = half * chunks / 2; c < (half + 1) * chunks / 2; ++c)
            if (n0 + c * 32 < p.N) tma_prefetch_l2_2d(&map_aux, n0 + c * 32, m0 + lane_grp * 32);
      }
      if constexpr (EPI == kEpiPleGate16)
        ple_first_aux(p, &map_aux, &aux_full[2 * (warp - 2)], sg, n0, m0 + lane_grp * 32, half * chunks / 2,
                      (half + 1) * chunks / 2, lane);
      const RowScales rs = row_scales(p, m0 + lane_grp * 32 + lane);
      const bool ready = mbar_wait(&tmem_full[acc], acc_phase, p.err);
      __syncwarp();
      if (!__all_sync(0xffffffffu, ready)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(lane_grp * 32) << 16) + (uint32_t)(acc * BN);
      bool released = false;
      auto release = [&]() {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tmem_empty[acc]);
        released = true;
      };
      epilogue_chunks<EPI>(p, &map_c, &map_aux, &aux_full[2 * (warp - 2)], aphase, sg, taddr, m0 + lane_grp * 32, n0, BN,
                           half * chunks / 2, (half + 1) * chunks / 2, lane, rs, release);
      if (!released) release();
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    if (lane == 0) tma_store_wait_all();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ------------------------------------------------------- CTA-pair GEMM --
// The same GEMM with 256 x 256 output tiles computed by a CTA pair
// (cta_group::2): each CTA of the pair loads its 128 rows of A and its 128 of
// the tile's 256 B rows, so a CTA moves 32 KB of operands per 2.1 MFLOP
// instead of 48 KB; the pair leader issues tcgen05.mma with M = 256, N = 256,
// and each CTA's TMEM receives the accumulator rows of its own A half.
//   * both CTAs' TMA loads complete on the leader's full barrier, which the
//     leader's producer arms with the bytes of both halves;
//   * the leader's commits are multicast to the matching barrier of both CTAs
//     (stage free, accumulator ready);
//   * every epilogue warp of both CTAs arrives on the leader's
//     accumulator-free barrier (the follower's through its cluster address).
constexpr int PR_ROWS = 128;  // rows of A and of B per CTA of the pair
constexpr int PR_TILE = 256;  // pair tile, M and N
// The PLE-gate epilogue streams a second operand (the per-layer slice) by
// TMA one chunk ahead, and the FP16 GeGLU epilogue's two stores per tile no
// longer wait for each other, so their kernels get two staging buffers per
// epilogue warp and one pipeline stage less (K = 512 needs only 8 stages;
// measured: GeGLU 35.5 -> 33.7 us per half batch, the FP32 stores slower).
template <int EPI>
struct PairCfg {
  static constexpr bool kTwoBufs = EPI == kEpiPleGate || EPI == kEpiPleGate16 || EPI == kEpiGeglu16;
  static constexpr int STAGES = kTwoBufs ? 5 : 6;
  static constexpr int STAGING_BUFS = kTwoBufs ? 2 : 1;
};
constexpr int PR_HALF_BYTES = PR_ROWS * BK * 4;  // 16 KB
constexpr int PR_STAGE_BYTES = 2 * PR_HALF_BYTES;
constexpr int kBarrierBytes = 512;  // ring, accumulator and aux (2 per epilogue warp) barriers
template <int EPI>
constexpr int pr_smem() {
  return PairCfg<EPI>::STAGES * PR_STAGE_BYTES + 8 * 4096 * PairCfg<EPI>::STAGING_BUFS + 1024 + kBarrierBytes;
}
static_assert(pr_smem<kEpiStore>() <= 232448 && pr_smem<kEpiPleGate>() <= 232448, "shared memory");

template <int EPI, bool F16>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_pair_tf32_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                          const __grid_constant__ CUtensorMap map_c, const __grid_constant__ CUtensorMap map_aux,
                          GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  pdl_trigger();
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  constexpr int PR_STAGES = PairCfg<EPI>::STAGES;
  constexpr int PR_STAGING_BUFS = PairCfg<EPI>::STAGING_BUFS;
  float* staging = (float*)(smem + PR_STAGES * PR_STAGE_BYTES);
  uint64_t* full = (uint64_t*)(smem + PR_STAGES * PR_STAGE_BYTES + 8 * 4096 * PR_STAGING_BUFS);
  uint64_t* empty = full + PR_STAGES;
  uint64_t* tmem_full = empty + PR_STAGES;
  uint64_t* tmem_empty = tmem_full + 2;
  uint64_t* aux_full = tmem_empty + 2;  // [16]: two per epilogue warp (PLE gate aux loads)
  uint32_t* tmem_slot = (uint32_t*)(aux_full + 16);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank() & 1u;  // 0 = leader of the pair
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1;
  const int n_pairs = gridDim.x >> 1;
  const int num_m = (p.M + PR_TILE - 1) / PR_TILE;
  const int num_n = (p.N + PR_TILE - 1) / PR_TILE;
  const int num_tiles = num_m * num_n;
  constexpr int bk = F16 ? 64 : BK;  // elements per 128-byte swizzle row
  const int num_k = (p.K + bk - 1) / bk;

  if (threadIdx.x == 0) {
    for (int s = 0; s < PR_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], 16);  // 8 epilogue warps x 2 CTAs
    }
    for (int w = 0; w < 16; ++w) mbar_init(&aux_full[w], 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
    tma_prefetch_desc(&map_c);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncwarp();
  cluster_sync();  // barrier inits and TMEM allocation visible to the pair
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // the previous kernel's outputs (A, row scales) are complete from here

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < num_tiles; tile += n_pairs) {
        const int m0 = (tile / num_n) * PR_TILE + (int)rank * PR_ROWS;
        const int n0 = (tile % num_n) * PR_TILE + (int)rank * PR_ROWS;
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.err)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * PR_STAGE_BYTES;
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * PR_STAGE_BYTES);
          const uint32_t bar = map_to_rank(smem_u32(&full[stage]), 0);
          tma_load_2d_pair(sa, &map_a, bar, kb * bk, m0);
          tma_load_2d_pair(sa + PR_HALF_BYTES, &map_b, bar, kb * bk, n0);
          if (++stage == PR_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      constexpr uint32_t idesc = F16 ? idesc_f16(PR_TILE, PR_TILE, 0) : idesc_tf32(PR_TILE, PR_TILE, 0);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < num_tiles; tile += n_pairs) {
        if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1, p.err)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * PR_TILE);
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * PR_STAGE_BYTES);
          const uint32_t b_addr = a_addr + PR_HALF_BYTES;
          // four MMAs of 32 bytes of K each: K = 8 TF32 or 16 FP16 elements
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t ad = sdesc(a_addr + k * 32, 16, 1024, kLayoutSW128);
            const uint64_t bd = sdesc(b_addr + k * 32, 16, 1024, kLayoutSW128);
            if constexpr (F16)
              mma_f16_pair(d, ad, bd, idesc, (kb | k) != 0);
            else
              mma_tf32_pair(d, ad, bd, idesc, (kb | k) != 0);
          }
          mma_commit_pair(&empty[stage], 0x3);
          if (++stage == PR_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        mma_commit_pair(&tmem_full[acc], 0x3);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else {
    // epilogue warps 2..9 of both CTAs: this CTA's 128 accumulator rows
    const int lane_grp = warp & 3;
    const int half = (warp - 2) >> 2;
    Staging sg{staging + (warp - 2) * 1024 * PR_STAGING_BUFS, PR_STAGING_BUFS};
    uint32_t aphase = 0;
    const int chunks = (EPI == kEpiGeglu || EPI == kEpiGeglu16 || EPI == kEpiQkv || EPI == kEpiQkv16) ? PR_TILE / 64 : PR_TILE / 32;
    const uint32_t empty_leader0 = map_to_rank(smem_u32(&tmem_empty[0]), 0);
    const uint32_t empty_leader1 = map_to_rank(smem_u32(&tmem_empty[1]), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = pair; tile < num_tiles; tile += n_pairs) {
      const int m0 = (tile / num_n) * PR_TILE + (int)rank * PR_ROWS;
      const int n0 = (tile % num_n) * PR_TILE;
      if constexpr (EPI == kEpiPleGate || EPI == kEpiPleGate16) {
        // pull this warp's aux chunks into L2 while the tile's MMAs run
        if (lane == 0)
          for (int c = half * chunks / 2; c < (half + 1) * chunks / 2; ++c)
            if (n0 + c * 32 < p.N) tma_prefetch_l2_2d(&map_aux, n0 + c * 32, m0 + lane_grp * 32);
      }
      if constexpr (EPI == kEpiPleGate16)
        ple_first_aux(p, &map_aux, &aux_full[2 * (warp - 2)], sg, n0, m0 + lane_grp * 32, half * chunks / 2,
                      (half + 1) * chunks / 2, lane);
      if constexpr (EPI == kEpiQkv16) {
        // pull the (cos, sin) entries of this warp's rotate-half pairs into L2
        // while the tile's MMAs run (a q / k tile's epilogue otherwise waited
        // ~1 us per chunk pair on them)
        if (n0 / 256 < p.nh + p.kvh) {
          const int r = m0 + lane_grp * 32 + lane;
          const float2* cs = p.rope + (r < p.M ? p.pos_of[r] : 0);
          for (int pi = half * chunks / 2 * 32; pi < (half + 1) * chunks / 2 * 32; ++pi)
            asm volatile("prefetch.global.L2 [%0];" ::"l"(cs + (size_t)pi * p.rope_stride));
        }
      }
      const RowScales rs = row_scales(p, m0 + lane_grp * 32 + lane);
      const bool ready = mbar_wait(&tmem_full[acc], acc_phase, p.err);
      __syncwarp();
      if (!__all_sync(0xffffffffu, ready)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(lane_grp * 32) << 16) + (uint32_t)(acc * PR_TILE);
      bool released = false;
      auto release = [&]() {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (leader)
            mbar_arrive(&tmem_empty[acc]);
          else
            mbar_arrive_cluster(acc ? empty_leader1 : empty_leader0);
        }
        released = true;
      };
      epilogue_chunks<EPI>(p, &map_c, &map_aux, &aux_full[2 * (warp - 2)], aphase, sg, taddr, m0 + lane_grp * 32, n0,
                           PR_TILE, half * chunks / 2, (half + 1) * chunks / 2, lane, rs, release);
      if (!released) release();
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    if (lane == 0) tma_store_wait_all();
  }
  tc_fence_before();
  __syncwarp();
  cluster_sync();  // no CTA of the pair leaves while the other may still signal it
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 512);
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

// rows x cols matrix with row pitch ld (elements); boxes of 128 bytes x
// box_rows, SWIZZLE_128B (operand loads and the epilogue's staged stores).
// FP32 (optionally typed TFLOAT32, the copy engine then rounds) or FP16.
enum class Elem { f32, tf32, f16 };

bool make_map(CUtensorMap* map, const void* base, int rows, int cols, int ld, int box_rows, Elem e) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  const int bytes = e == Elem::f16 ? 2 : 4;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * bytes};
  cuuint32_t box[2] = {(cuuint32_t)(128 / bytes), (cuuint32_t)box_rows};
  cuuint32_t elem[2] = {1, 1};
  const CUtensorMapDataType type = e == Elem::f16    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                   : e == Elem::tf32 ? CU_TENSOR_MAP_DATA_TYPE_TFLOAT32
                                                     : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  CUresult r = enc(map, type, 2, (void*)base, dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

Elem operand_elem(const GemmParams& p) { return p.f16 ? Elem::f16 : (p.tf32_tma ? Elem::tf32 : Elem::f32); }

// PLE gate: the aux slice [M, N] (row pitch ld_aux) in 32 x 32 FP32 boxes;
// other epilogues get a copy of the output map (never read).
bool make_aux_map(CUtensorMap* map, const GemmParams& p, const CUtensorMap& out) {
  if (p.epilogue != kEpiPleGate) {  // (the FP16 form shares the aux map)
    *map = out;
    return true;
  }
  if (p.ld_aux % 4 || ((uintptr_t)p.aux & 15)) return false;
  return make_map(map, p.aux, p.M, p.N, p.ld_aux, 32, Elem::f32);
}

// The output map: M rows x (n_out or N) columns, 32 x 32 boxes (FP32 with
// 128-byte swizzled rows, or FP16 with 64-byte swizzled rows).
bool make_out_map(CUtensorMap* map, const GemmParams& p) {
  const int cols = p.epilogue == kEpiGeglu ? p.n_out : p.N;
  if (p.out_f16) {
    EncodeTiledFn enc = encode_fn();
    if (!enc || p.ldc % 8) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)p.M};
    cuuint64_t strides[1] = {(cuuint64_t)p.ldc * 2};
    cuuint32_t box[2] = {32, 32};
    cuuint32_t elem[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void*)p.C, dims, strides, box, elem,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
  }
  return make_map(map, p.C, p.M, cols, p.ldc, 32, Elem::f32);
}

template <int BN, int EPI, bool F16>
cudaError_t launch_t(const GemmParams& p, cudaStream_t stream) {
  using C = Cfg<BN>;
  static std::atomic<uint64_t> opted{0};  // per instantiation, one bit per device
  cudaError_t e = smem_opt_in(gemm_tf32_kernel<BN, EPI, F16>, C::SMEM, &opted);
  if (e != cudaSuccess) return e;
  CUtensorMap ma, mb, mc;
  CUtensorMap mx;
  if (!make_map(&ma, p.A, p.M, p.K, p.lda, BM, operand_elem(p)) ||
      !make_map(&mb, p.B, p.N, p.K, p.ldb, BN, operand_elem(p)) || !make_out_map(&mc, p) ||
      !make_aux_map(&mx, p, mc))
    return cudaErrorInvalidValue;
  const int tiles = ((p.M + BM - 1) / BM) * ((p.N + BN - 1) / BN);
  const int grid = tiles < sm_count() ? tiles : sm_count();
  launch_pdl(gemm_tf32_kernel<BN, EPI, F16>, dim3(grid), dim3(kThreads), C::SMEM, stream, ma, mb, mc, mx, p);
  return cudaGetLastError();
}

template <int BN, int EPI>
cudaError_t launch(const GemmParams& p, cudaStream_t stream) {
  return p.f16 ? launch_t<BN, EPI, true>(p, stream) : launch_t<BN, EPI, false>(p, stream);
}

template <int EPI, bool F16>
cudaError_t launch_pair_t(const GemmParams& p, cudaStream_t stream) {
  static std::atomic<uint64_t> opted{0};
  cudaError_t e = smem_opt_in(gemm_pair_tf32_kernel<EPI, F16>, pr_smem<EPI>(), &opted);
  if (e != cudaSuccess) return e;
  CUtensorMap ma, mb, mc;
  CUtensorMap mx;
  if (!make_map(&ma, p.A, p.M, p.K, p.lda, PR_ROWS, operand_elem(p)) ||
      !make_map(&mb, p.B, p.N, p.K, p.ldb, PR_ROWS, operand_elem(p)) || !make_out_map(&mc, p) ||
      !make_aux_map(&mx, p, mc))
    return cudaErrorInvalidValue;
  const int tiles = ((p.M + PR_TILE - 1) / PR_TILE) * ((p.N + PR_TILE - 1) / PR_TILE);
  int pairs = sm_count() / 2;
  if (tiles < pairs) pairs = tiles;
  launch_pdl(gemm_pair_tf32_kernel<EPI, F16>, dim3(2 * pairs), dim3(kThreads), pr_smem<EPI>(), stream, ma, mb, mc, mx,
             p);
  return cudaGetLastError();
}

template <int EPI>
cudaError_t launch_pair(const GemmParams& p, cudaStream_t stream) {
  return p.f16 ? launch_pair_t<EPI, true>(p, stream) : launch_pair_t<EPI, false>(p, stream);
}

// The pair kernel needs at least one full 256-row tile of A and of B.
bool use_pair(const GemmParams& p) { return p.M >= PR_TILE && p.N >= PR_TILE && !p.single_cta; }

}  // namespace

// SM count of the current device (cached per device ordinal).
int sm_count() {
  static std::atomic<int> cache[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  int n = dev >= 0 && dev < 64 ? cache[dev].load(std::memory_order_relaxed) : 0;
  if (!n) {
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 1;
    if (dev >= 0 && dev < 64) cache[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

cudaError_t gemm_tf32(const GemmParams& p, cudaStream_t stream) {
  if (p.M <= 0 || p.N <= 0) return cudaSuccess;
  if (p.K <= 0 || p.K % 4 || p.lda % 4 || p.ldb % 4 || p.ldc % 4 || ((uintptr_t)p.A & 15) || ((uintptr_t)p.B & 15) ||
      ((uintptr_t)p.C & 15))
    return cudaErrorInvalidValue;
  if (p.lda < p.K || p.ldb < p.K) return cudaErrorInvalidValue;
  if (p.f16 && (p.K % 8 || p.lda % 8 || p.ldb % 8)) return cudaErrorInvalidValue;
  const bool grouped = p.epilogue == kEpiStore && p.group_inv;  // FP16 with per-group scales
  if (p.out_f16 && p.epilogue != kEpiQkv && p.epilogue != kEpiGeglu && p.epilogue != kEpiPleGate && !grouped)
    return cudaErrorInvalidValue;
  if (p.out_f16 && p.epilogue != kEpiQkv && !grouped && !p.out_inv) return cudaErrorInvalidValue;
  if (grouped && (!p.out_f16 || p.ldc % 8)) return cudaErrorInvalidValue;
  if ((p.row_ss || p.group_inv) &&
      (p.epilogue != kEpiStore || p.N % 128 || p.N <= 128 || p.row_ss_stride < p.N / 128))
    return cudaErrorInvalidValue;
  switch (p.epilogue) {
    case kEpiStore:
      if (grouped) {
        if (use_pair(p)) return launch_pair<kEpiStore16>(p, stream);
        return launch<256, kEpiStore16>(p, stream);
      }
      if (use_pair(p)) return launch_pair<kEpiStore>(p, stream);
      if (p.N <= 128) return launch<128, kEpiStore>(p, stream);
      return launch<256, kEpiStore>(p, stream);
    case kEpiGeglu:
      if (p.N % 256 || p.n_out <= 0 || p.n_out > p.N / 2 || p.n_out % 4) return cudaErrorInvalidValue;
      if (p.out_f16) {
        if (use_pair(p)) return launch_pair<kEpiGeglu16>(p, stream);
        return launch<256, kEpiGeglu16>(p, stream);
      }
      if (use_pair(p)) return launch_pair<kEpiGeglu>(p, stream);
      return launch<256, kEpiGeglu>(p, stream);
    case kEpiPleGate:
      if (!p.aux) return cudaErrorInvalidValue;
      if (p.out_f16) {
        if (use_pair(p)) return launch_pair<kEpiPleGate16>(p, stream);
        if (p.N <= 128) return launch<128, kEpiPleGate16>(p, stream);
        return launch<256, kEpiPleGate16>(p, stream);
      }
      if (use_pair(p)) return launch_pair<kEpiPleGate>(p, stream);
      if (p.N <= 128) return launch<128, kEpiPleGate>(p, stream);
      return launch<256, kEpiPleGate>(p, stream);
    case kEpiQkv:  // one 256-column tile per head
      if (p.N % 256 || !p.q_norm || !p.k_norm || !p.rope || !p.pos_of || p.N != 256 * (p.nh + 2 * p.kvh))
        return cudaErrorInvalidValue;
      if (p.out_f16) {
        if (use_pair(p)) return launch_pair<kEpiQkv16>(p, stream);
        return launch<256, kEpiQkv16>(p, stream);
      }
      if (use_pair(p)) return launch_pair<kEpiQkv>(p, stream);
      return launch<256, kEpiQkv>(p, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace svl
