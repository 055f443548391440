// search.cu -- exact cosine top-k over a device-resident corpus
// (src/index/vector.rs:17-97, Index::search src/index/mod.rs:325-388).
//
// Fast path (k <= kMaxFastK, dim % 4 == 0), three kernels:
//   1. query_prep: per query the reference's f64 norm (sequential sum,
//      vector.rs:34-46; zero / non-finite -> Usage) and a unit-norm copy for
//      the screen, rounded to FP16 (or to TF32);
//   2. screen_topk: a persistent tcgen05 GEMM (queries x corpus^T, TMA-fed,
//      TMEM accumulators) whose epilogue keeps, per query and per corpus
//      range, the KC best screen scores.  CTA c works on query block
//      c % n_qb and corpus range c / n_qb, so the n_qb CTAs of one range
//      stream the same corpus tiles together and the corpus leaves HBM once.
//      An index screens an FP16 copy of its unit-norm rows (kind::f16: twice
//      the TF32 tensor rate, half the bytes, the same 11-bit significand);
//      the allocation-free entry point screens the caller's FP32 rows in TF32;
//   3. rescore_select: per query, the k-th best screen score s_k; every
//      candidate with screen >= s_k - 2*delta is rescored EXACTLY as the
//      reference does (f64, sequential over the dimension, no fused
//      multiply-add), then ranked by (score desc, chunk id asc).
// delta bounds |screen - cosine| (FP16 or TF32 operands, FP32 accumulation), so any
// row left out of a range's list -- its screen score is at most that list's
// KC-th score tau -- cannot reach the exact top-k when tau < s_k - 2*delta.
// A query failing that check is answered by the full path.
//
// Full path (any k, any dim, and fallback): exact f64 scores of every row,
// then a stable radix sort by score over rows pre-ordered by chunk id, so
// ties come out by ascending chunk id -- the reference's complete ordering.

#include <cub/cub.cuh>
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "gemm_tc.cuh"
#include "model.cuh"
#include "search.cuh"

namespace svl {

namespace {

constexpr int BM = 128, BN = 256, BK = 32;
constexpr int kThreads = 320;  // warp 0 TMA, warp 1 MMA, warps 2..9 epilogue
constexpr int kEpiThreads = 256;
constexpr int kSlotBytes = kEpiThreads * 32 * 4;  // the epilogue's insertion slots
constexpr int A_BYTES = BM * BK * 4, B_BYTES = BN * BK * 4, STAGE_BYTES = A_BYTES + B_BYTES;
constexpr uint32_t kNoRow = 0xFFFFFFFFu;
// |screen score - f64 cosine| <= kDelta.  TF32: operands carry at most 2^-10
// (corpus, truncated by the tensor core) + 2^-11 (query, rounded) relative
// error each; FP16: 2^-11 + 2^-11 (both rounded to nearest), plus at most
// 2^-25 absolute per component below the FP16 normal range (2^-14), i.e.
// <= 2 * sqrt(dim) * 2^-25 <= 5.4e-6 in all.  Either way times
// sum |q_i||v_i| <= 1 (unit vectors), plus FP32 accumulation over <= 8192
// terms of magnitude <= 1 (<= 2^-24 * dim * max partial).  1.6e-3 for dim
// 768 (TF32); 2e-3 leaves margin.
constexpr double kDelta = 2.0e-3;

template <int KC>
struct ScreenCfg {
  static constexpr int STAGES = 4;
  static constexpr int SMEM = STAGES * STAGE_BYTES + kSlotBytes + 1024 + 256;
  static_assert(SMEM <= 232448, "shared memory");
};

}  // namespace

// ------------------------------------------------------------- kernels --

// vector.rs:34-46: f64 sum of squares in order; qnorm = sqrt.  Also writes
// the unit query for the screen: TF32-rounded (qhat) and / or FP16 (qhat16,
// round to nearest).  One thread per query.
__global__ void query_prep_kernel(const float* __restrict__ q, int nq, int dim, double* __restrict__ qnorm,
                                  float* __restrict__ qhat, uint16_t* __restrict__ qhat16, uint32_t* err) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nq) return;
  const float* x = q + (size_t)i * dim;
  double sum = 0.0;
  bool finite = true;
  for (int d = 0; d < dim; ++d) {
    const double v = (double)x[d];
    finite &= isfinite(x[d]);
    sum = __dadd_rn(sum, __dmul_rn(v, v));
  }
  const bool ok = finite && isfinite(sum) && sum > 0.0;
  const double n = ok ? __dsqrt_rn(sum) : 0.0;
  qnorm[i] = n;
  if (!ok) atomicOr(err, SVL_DEVERR_BAD_QUERY);
  if (qhat)
    for (int d = 0; d < dim; ++d) qhat[(size_t)i * dim + d] = ok ? round_tf32((float)((double)x[d] / n)) : 0.0f;
  if (qhat16)
    for (int d = 0; d < dim; ++d)
      qhat16[(size_t)i * dim + d] = ok ? __half_as_ushort(__float2half_rn((float)((double)x[d] / n))) : (uint16_t)0;
}

// Chunk::new normalisation (storage/model.rs:546-581) of appended rows, in
// place: f64 sequential sum of squares, value = (f32)(v / norm); rows16 (if
// set) receives the FP16 copy the screen reads (round to nearest).
__global__ void append_normalize_kernel(float* __restrict__ rows, uint16_t* __restrict__ rows16, uint64_t n, int dim,
                                        uint32_t* err) {
  const uint64_t r = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (r >= n) return;
  float* x = rows + r * dim;
  double sum = 0.0;
  bool finite = true;
  for (int d = 0; d < dim; ++d) {
    const double v = (double)x[d];
    finite &= isfinite(x[d]);
    sum = __dadd_rn(sum, __dmul_rn(v, v));
  }
  if (!finite || !isfinite(sum) || sum <= 0.0) {
    atomicOr(err, SVL_DEVERR_BAD_ROW);
    return;
  }
  const double norm = __dsqrt_rn(sum);
  for (int d = 0; d < dim; ++d) {
    const float u = (float)__ddiv_rn((double)x[d], norm);
    x[d] = u;
    if (rows16) rows16[r * dim + d] = __half_as_ushort(__float2half_rn(u));
  }
}

// vector.rs:72-86 for one (query, row): exact f64 dot and row norm, summed
// in dimension order without contraction; score = dot / (|q| * sqrt(vsum)).
SVL_DEV double exact_cosine(const float* __restrict__ q, double qn, const float* __restrict__ v, int dim,
                            bool* bad_row) {
  double dot = 0.0, vsum = 0.0;
  for (int d = 0; d < dim; ++d) {
    const double a = (double)q[d], b = (double)v[d];
    dot = __dadd_rn(dot, __dmul_rn(a, b));
    vsum = __dadd_rn(vsum, __dmul_rn(b, b));
  }
  if (!isfinite(vsum) || vsum <= 0.0) *bad_row = true;
  return __ddiv_rn(dot, __dmul_rn(qn, __dsqrt_rn(vsum)));
}

// One accumulator tile of the screen for one epilogue thread: its query's
// scores against corpus rows t * BN + [half * BN / 2, (half + 1) * BN / 2)
// (TMEM columns; taddr = this warp's lanes, column 0 of the accumulator)
// folded into its sorted KC best (cs, cr); `seen` counts the valid rows.
// A chunk holding a score above the current KC-th goes through `slot` (this
// thread's 32 floats of shared memory, 256 floats apart so a warp's accesses
// are conflict free) and one rolled loop, so the insertion code exists once:
// unrolled per column it ran to thousands of instructions and the epilogue
// stalled on instruction fetch.
template <int KC>
SVL_DEV void screen_tile(const ScreenParams& p, uint32_t taddr, int t, int half, float (&cs)[KC], uint32_t (&cr)[KC],
                         uint64_t& seen, float* slot) {
  float v[32];
#pragma unroll 1
  for (int c = half * (BN / 64); c < (half + 1) * (BN / 64); ++c) {
    tmem_ld32(taddr + c * 32, v);
    const uint64_t row0 = (uint64_t)t * BN + c * 32;
    const int nvalid = row0 >= p.n_rows ? 0 : (p.n_rows - row0 < 32 ? (int)(p.n_rows - row0) : 32);
    if (nvalid < 32 || p.mask) {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        bool valid = j < nvalid;
        if (valid && p.mask) valid = p.mask[row0 + j] != 0;
        seen += valid;
        if (!valid) v[j] = -INFINITY;
      }
    } else {
      seen += 32;
    }
    // common case: nothing in this chunk beats the current KC-th score
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < 32; j += 4) mx = fmaxf(mx, fmaxf(fmaxf(v[j], v[j + 1]), fmaxf(v[j + 2], v[j + 3])));
    if (mx > cs[KC - 1]) {
      const float th = cs[KC - 1];
      uint32_t cand = 0;  // columns above the KC-th score as the chunk starts
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        slot[j * kEpiThreads] = v[j];
        cand |= (v[j] > th ? 1u : 0u) << j;
      }
      while (cand) {
        const int j = __ffs(cand) - 1;
        cand &= cand - 1;
        const float x = slot[j * kEpiThreads];
        if (x > cs[KC - 1]) {
          cs[KC - 1] = x;
          cr[KC - 1] = (uint32_t)(row0 + j);
#pragma unroll
          for (int i = KC - 1; i > 0; --i) {  // one insertion step, static indices
            if (cs[i] > cs[i - 1]) {
              const float ts = cs[i];
              cs[i] = cs[i - 1];
              cs[i - 1] = ts;
              const uint32_t tr = cr[i];
              cr[i] = cr[i - 1];
              cr[i - 1] = tr;
            }
          }
        }
      }
    }
  }
}

// Writes a thread's KC candidates and its list's tau.
template <int KC>
SVL_DEV void screen_emit(const ScreenParams& p, int query, int list, const float (&cs)[KC], const uint32_t (&cr)[KC],
                         uint64_t seen) {
  if (query < p.n_queries) {
    const size_t base = ((size_t)query * p.n_lists + list) * KC;
#pragma unroll
    for (int i = 0; i < KC; ++i) {
      p.cand_score[base + i] = cs[i];
      p.cand_row[base + i] = cr[i];
    }
    // every valid row not kept scores at most the KC-th kept screen score
    p.tau[(size_t)query * p.n_lists + list] = seen > (uint64_t)KC ? cs[KC - 1] : -INFINITY;
  }
}

// F16: FP16 queries and corpus (kind::f16, 64 elements per 128-byte stage
// row) instead of TF32 (32), a compile-time choice like the GEMMs'.
template <int KC, bool F16>
__global__ void __launch_bounds__(kThreads, 1)
    screen_topk_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_c,
                       ScreenParams p) {
  using C = ScreenCfg<KC>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  float* slots = (float*)(smem + C::STAGES * STAGE_BYTES);
  uint64_t* full = (uint64_t*)(smem + C::STAGES * STAGE_BYTES + kSlotBytes);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tmem_full = empty + C::STAGES;
  uint64_t* tmem_empty = tmem_full + 2;
  uint32_t* tmem_slot = (uint32_t*)(tmem_empty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qb = blockIdx.x % p.n_qb;
  const int range = blockIdx.x / p.n_qb;
  const int n_tiles = (int)((p.n_rows + BN - 1) / BN);
  const int t_begin = (int)((int64_t)n_tiles * range / p.n_ranges);
  const int t_end = (int)((int64_t)n_tiles * (range + 1) / p.n_ranges);
  constexpr int bk = F16 ? 64 : BK;  // elements per 128-byte stage row
  const int num_k = (p.dim + bk - 1) / bk;

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
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&map_q);
      tma_prefetch_desc(&map_c);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = t_begin; ok && t < t_end; ++t) {
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.err)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * STAGE_BYTES;
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          tma_load_2d(sa, &map_q, &full[stage], kb * bk, qb * BM);
          tma_load_2d(sa + A_BYTES, &map_c, &full[stage], kb * bk, t * BN);
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
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int t = t_begin; ok && t < t_end; ++t) {
        if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1, p.err)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t b_addr = a_addr + A_BYTES;
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
    // epilogue: thread owns query qb*128 + (w % 4)*32 + lane and one half of the
    // tile's columns; its best KC (score, row) pairs stay sorted in registers
    const int lane_grp = warp & 3;
    const int half = (warp - 2) >> 2;
    const int et = lane_grp * 32 + lane;
    float* slot = slots + (threadIdx.x - 64);
    const int query = qb * BM + et;
    const int list = range * 2 + half;  // one candidate list per (range, column half)
    float cs[KC];
    uint32_t cr[KC];
#pragma unroll
    for (int i = 0; i < KC; ++i) {
      cs[i] = -INFINITY;
      cr[i] = kNoRow;
    }
    uint64_t seen = 0;  // valid rows offered to this list
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = t_begin; t < t_end; ++t) {
      const bool ready = mbar_wait(&tmem_full[acc], acc_phase, p.err);
      __syncwarp();
      if (!__all_sync(0xffffffffu, ready)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(lane_grp * 32) << 16) + (uint32_t)(acc * BN);
      screen_tile<KC>(p, taddr, t, half, cs, cr, seen, slot);
      tc_fence_before();
      mbar_arrive(&tmem_empty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    screen_emit<KC>(p, query, list, cs, cr, seen);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
  }
}

// The FP16 screen on CTA pairs (cta_group::2): a pair tile is 256 queries
// (128 per CTA, its own A rows) x 256 corpus rows (128 loaded by each CTA,
// the B halves of one M = 256, N = 256 MMA), so a CTA moves 32 KB of
// operands per 128-byte K slice for the work the one-CTA screen needs 48 KB
// for.  Pair c works on 256-query block c % n_qb and corpus range c / n_qb;
// each CTA's TMEM holds its 128 queries x 256 rows, and its epilogue is the
// one-CTA screen's.  Loads complete on the leader's barriers; the leader's
// commits reach both CTAs; epilogue warps of both CTAs arrive on the
// leader's accumulator-free barrier.
constexpr int PBM = 128;                        // query rows per CTA
constexpr int PAIR_A_BYTES = PBM * 128;         // 64 FP16 x 128 rows
constexpr int PAIR_B_BYTES = (BN / 2) * 128;    // this CTA's 128 corpus rows
constexpr int PAIR_STAGE_BYTES = PAIR_A_BYTES + PAIR_B_BYTES;
constexpr int PAIR_STAGES = 6;
constexpr int PAIR_SMEM = PAIR_STAGES * PAIR_STAGE_BYTES + kSlotBytes + 1024 + 256;
static_assert(PAIR_SMEM <= 232448, "shared memory");

template <int KC>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    screen_pair_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_c,
                       ScreenParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  float* slots = (float*)(smem + PAIR_STAGES * PAIR_STAGE_BYTES);
  uint64_t* full = (uint64_t*)(smem + PAIR_STAGES * PAIR_STAGE_BYTES + kSlotBytes);
  uint64_t* empty = full + PAIR_STAGES;
  uint64_t* tmem_full = empty + PAIR_STAGES;
  uint64_t* tmem_empty = tmem_full + 2;
  uint32_t* tmem_slot = (uint32_t*)(tmem_empty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank() & 1u;
  const bool leader = rank == 0;
  const int pair = (int)(blockIdx.x >> 1);
  const int qb = pair % p.n_qb;  // 256-query block
  const int range = pair / p.n_qb;
  const int n_tiles = (int)((p.n_rows + BN - 1) / BN);
  const int t_begin = (int)((int64_t)n_tiles * range / p.n_ranges);
  const int t_end = (int)((int64_t)n_tiles * (range + 1) / p.n_ranges);
  const int num_k = (p.dim + 63) / 64;

  if (threadIdx.x == 0) {
    for (int s = 0; s < PAIR_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], 16);  // 8 epilogue warps x 2 CTAs
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 2 * BN);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncwarp();
  cluster_sync();  // barrier inits and TMEM allocation visible to the pair
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&map_q);
      tma_prefetch_desc(&map_c);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = t_begin; ok && t < t_end; ++t) {
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.err)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * PAIR_STAGE_BYTES;
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * PAIR_STAGE_BYTES);
          const uint32_t bar = map_to_rank(smem_u32(&full[stage]), 0);
          tma_load_2d_pair(sa, &map_q, bar, kb * 64, qb * 2 * PBM + (int)rank * PBM);
          tma_load_2d_pair(sa + PAIR_A_BYTES, &map_c, bar, kb * 64, t * BN + (int)rank * (BN / 2));
          if (++stage == PAIR_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      constexpr uint32_t idesc = idesc_f16(2 * PBM, BN, 0);
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int t = t_begin; ok && t < t_end; ++t) {
        if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1, p.err)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * PAIR_STAGE_BYTES);
          const uint32_t b_addr = a_addr + PAIR_A_BYTES;
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_f16_pair(d, sdesc(a_addr + k * 32, 16, 1024, kLayoutSW128), sdesc(b_addr + k * 32, 16, 1024, kLayoutSW128),
                         idesc, (kb | k) != 0);
          mma_commit_pair(&empty[stage], 0x3);
          if (++stage == PAIR_STAGES) {
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
    // epilogue: thread owns query qb*256 + rank*128 + (w % 4)*32 + lane and one
    // half of the tile's columns (the one-CTA screen's epilogue)
    const int lane_grp = warp & 3;
    const int half = (warp - 2) >> 2;
    const int et = lane_grp * 32 + lane;
    float* slot = slots + (threadIdx.x - 64);
    const int query = qb * 2 * PBM + (int)rank * PBM + et;
    const int list = range * 2 + half;
    const uint32_t empty_leader0 = map_to_rank(smem_u32(&tmem_empty[0]), 0);
    const uint32_t empty_leader1 = map_to_rank(smem_u32(&tmem_empty[1]), 0);
    float cs[KC];
    uint32_t cr[KC];
#pragma unroll
    for (int i = 0; i < KC; ++i) {
      cs[i] = -INFINITY;
      cr[i] = kNoRow;
    }
    uint64_t seen = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = t_begin; t < t_end; ++t) {
      const bool ready = mbar_wait(&tmem_full[acc], acc_phase, p.err);
      __syncwarp();
      if (!__all_sync(0xffffffffu, ready)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(lane_grp * 32) << 16) + (uint32_t)(acc * BN);
      screen_tile<KC>(p, taddr, t, half, cs, cr, seen, slot);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (leader)
          mbar_arrive(&tmem_empty[acc]);
        else
          mbar_arrive_cluster(acc ? empty_leader1 : empty_leader0);
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    screen_emit<KC>(p, query, list, cs, cr, seen);
  }
  tc_fence_before();
  __syncwarp();
  cluster_sync();  // no CTA of the pair leaves while the other may still signal it
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 2 * BN);
  }
}

// (score desc, chunk id asc, row asc) -- vector.rs:90-95.
SVL_DEV bool beats(double sa, uint64_t ca, uint64_t ra, double sb, uint64_t cb, uint64_t rb) {
  if (sa != sb) return sa > sb;
  if (ca != cb) return ca < cb;
  return ra < rb;
}

constexpr int kRescoreThreads = 256;
constexpr int kMaxCand = 148 * 32;  // n_lists * kc
constexpr int kMaxSel = 1024;       // rescored candidates per query (more -> full path)
constexpr int kRescoreSmem = kMaxCand * 8 + kMaxSel * 12;

// One CTA per query.  See the file comment for the selection rule.
__global__ void __launch_bounds__(kRescoreThreads)
    rescore_select_kernel(RescoreParams p) {
  extern __shared__ uint8_t rescore_smem[];
  double* s_exact = (double*)rescore_smem;                    // [kMaxSel]
  float* s_screen = (float*)(s_exact + kMaxSel);              // [kMaxCand]
  uint32_t* s_row = (uint32_t*)(s_screen + kMaxCand);         // [kMaxCand]
  uint32_t* s_sel = s_row + kMaxCand;                         // [kMaxSel]
  __shared__ int s_nsel, s_nvalid;
  __shared__ float s_red[32];
  __shared__ int s_cnt[32];
  __shared__ int s_fallback;
  __shared__ int s_badrow;
  const int q = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int ncand = p.n_lists * p.kc;
  if (tid == 0) {
    s_nsel = 0;
    s_nvalid = 0;
    s_fallback = 0;
    s_badrow = 0;
  }
  __syncthreads();
  if (p.qnorm[q] <= 0.0) {  // invalid query: already flagged by query_prep
    if (tid == 0) p.out_count[q] = 0;
    return;
  }
  // load candidates and the largest tau
  float tau = -INFINITY;
  int nvalid_local = 0;
  for (int i = tid; i < ncand; i += kRescoreThreads) {
    s_screen[i] = p.cand_score[(size_t)q * ncand + i];
    s_row[i] = p.cand_row[(size_t)q * ncand + i];
    nvalid_local += s_row[i] != kNoRow;
  }
  for (int r = tid; r < p.n_lists; r += kRescoreThreads) tau = fmaxf(tau, p.tau[(size_t)q * p.n_lists + r]);
  tau = warp_max(tau);
  if (lane == 0) s_red[wid] = tau;
  atomicAdd(&s_nvalid, nvalid_local);
  __syncthreads();
  if (tid < 32) {
    float v = tid < kRescoreThreads / 32 ? s_red[tid] : -INFINITY;
    v = warp_max(v);
    if (tid == 0) s_red[0] = v;
  }
  __syncthreads();
  const float max_tau = s_red[0];
  const int nvalid = s_nvalid;
  const int k = p.k;
  // k-th largest screen score by bisection on the order-preserving integer image
  float lower = -INFINITY;
  if (nvalid >= k) {
    // find the largest x with count(screen >= x) >= k, over the float bit patterns
    auto key = [](float f) -> uint32_t {
      const uint32_t u = __float_as_uint(f);
      return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    };
    uint32_t lo = 0, hi = 0xFFFFFFFFu;  // invariant: count(key >= lo) >= k
    while (lo < hi) {
      const uint32_t mid = lo + (uint32_t)(((uint64_t)hi - lo + 1) / 2);
      int c = 0;
      for (int i = tid; i < ncand; i += kRescoreThreads) c += (s_row[i] != kNoRow && key(s_screen[i]) >= mid);
#pragma unroll
      for (int o = 16; o; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
      __syncthreads();
      if (lane == 0) s_cnt[wid] = c;
      __syncthreads();
      int tot = 0;
      for (int w = 0; w < kRescoreThreads / 32; ++w) tot += s_cnt[w];
      if (tot >= k)
        lo = mid;
      else
        hi = mid - 1;
    }
    const uint32_t u = (lo & 0x80000000u) ? (lo & 0x7FFFFFFFu) : ~lo;
    const float kth = __uint_as_float(u);
    lower = (float)((double)kth - 2.0 * kDelta);
    if (max_tau >= lower) s_fallback = 1;
  }
  __syncthreads();
  if (s_fallback) {
    if (tid == 0) {
      p.fallback[q] = 1;
      p.out_count[q] = 0;
    }
    return;
  }
  for (int i = tid; i < ncand; i += kRescoreThreads)
    if (s_row[i] != kNoRow && s_screen[i] >= lower) {
      const int slot = atomicAdd(&s_nsel, 1);
      if (slot < kMaxSel) s_sel[slot] = i;
    }
  __syncthreads();
  const int nsel = s_nsel;
  if (nsel > kMaxSel) {  // too many near-ties for the fast path
    if (tid == 0) {
      p.fallback[q] = 1;
      p.out_count[q] = 0;
    }
    return;
  }
  const float* qv = p.queries + (size_t)q * p.dim;
  const double qn = p.qnorm[q];
  bool bad = false;
  for (int i = tid; i < nsel; i += kRescoreThreads) {
    const uint32_t row = s_row[s_sel[i]];
    s_exact[i] = exact_cosine(qv, qn, p.rows + (size_t)row * p.dim, p.dim, &bad);
  }
  if (bad) s_badrow = 1;
  __syncthreads();
  if (s_badrow) {
    if (tid == 0) {
      atomicOr(p.err, SVL_DEVERR_BAD_ROW);
      p.out_count[q] = 0;
    }
    return;
  }
  const int kout = nsel < k ? nsel : k;
  for (int i = tid; i < nsel; i += kRescoreThreads) {
    const uint32_t ri = s_row[s_sel[i]];
    const uint64_t ci = p.chunk_ids[ri];
    int rank = 0;
    for (int j = 0; j < nsel; ++j) {
      const uint32_t rj = s_row[s_sel[j]];
      rank += beats(s_exact[j], p.chunk_ids[rj], rj, s_exact[i], ci, ri);
    }
    if (rank < kout) {
      const size_t o = (size_t)q * p.k + rank;
      p.out_rows[o] = ri;
      p.out_scores[o] = s_exact[i];
      if (p.out_chunk_ids) p.out_chunk_ids[o] = ci;
    }
  }
  if (tid == 0) p.out_count[q] = (uint32_t)kout;
}

// Asynchronous global -> shared copies (cp.async; 16 bytes bypass L1).
SVL_DEV void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
SVL_DEV void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
SVL_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
SVL_DEV void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Full path: exact f64 score of every row for one query, in chunk-id order
// (position i scores row order[i]), written as sortable keys (ascending key
// = descending score) for the complete ranking.  Each thread keeps one row's
// sequential f64 sums (exact_cosine's order, so scores are bit-identical to
// the reference's); the block stages its 128 rows 32 dimensions at a time in
// shared memory with cp.async copies that are coalesced per row (8 threads
// copy one row's 128 bytes), double-buffered so that step s + 1 loads while
// step s is summed -- a single buffer left the warps waiting on global loads
// (long-scoreboard stalls) with the FP64 pipe ~9% busy.  Rows are padded to
// 36 floats: 16-byte aligned copies, and float4 reads of 8 consecutive rows
// fall in distinct banks.
constexpr int kFullRows = 128;   // rows (threads) per block
constexpr int kFullStep = 32;    // dimensions staged per step
constexpr int kFullStride = 36;  // floats per staged row
template <int VEC>  // floats per copy: 4 when dim % 4 == 0 (16-byte aligned rows), else 1
__global__ void __launch_bounds__(kFullRows)
    full_scores_kernel(const float* __restrict__ query, double qn, const float* __restrict__ rows,
                       const uint64_t* __restrict__ order, uint64_t n, int dim, const uint8_t* __restrict__ mask,
                       uint64_t* __restrict__ keys, double* __restrict__ scores, uint32_t* err) {
  __shared__ __align__(16) float tile[2][kFullRows * kFullStride];
  __shared__ double qd[2][kFullStep];
  __shared__ uint64_t row_of[kFullRows];
  const int tid = threadIdx.x;
  const uint64_t i0 = blockIdx.x * (uint64_t)kFullRows;
  const uint64_t i = i0 + tid;
  row_of[tid] = i < n ? order[i] : 0;
  const bool live = i < n && !(mask && !mask[row_of[tid]]);
  __syncthreads();
  const int rows_here = n - i0 < (uint64_t)kFullRows ? (int)(n - i0) : kFullRows;
  const int steps = (dim + kFullStep - 1) / kFullStep;
  constexpr int kSegs = kFullStep / VEC;  // copies per row per step
  auto stage = [&](int s) {
    const int d0 = s * kFullStep;
    const int w = dim - d0 < kFullStep ? dim - d0 : kFullStep;
    const int segs = (w + VEC - 1) / VEC;  // w is a multiple of VEC
    float* t = tile[s & 1];
    for (int c = tid; c < kFullRows * kSegs; c += kFullRows) {
      const int r = c / kSegs, g = c % kSegs;
      if (r < rows_here && g < segs) {
        const float* src = rows + row_of[r] * (uint64_t)dim + d0 + g * VEC;
        float* dst = t + r * kFullStride + g * VEC;
        if constexpr (VEC == 4)
          cp_async16(dst, src);
        else
          cp_async4(dst, src);
      }
    }
    if (tid < w) qd[s & 1][tid] = (double)query[d0 + tid];
    cp_async_commit();
  };
  double dot = 0.0, vsum = 0.0;
  stage(0);
  for (int s = 0; s < steps; ++s) {
    if (s + 1 < steps) {
      stage(s + 1);
      cp_async_wait<1>();  // this thread's copies of step s are in
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();  // everyone's copies of step s are in
    if (live) {
      const int w = dim - s * kFullStep < kFullStep ? dim - s * kFullStep : kFullStep;
      const float* t = tile[s & 1] + tid * kFullStride;
      const double* qq = qd[s & 1];
      if (w == kFullStep) {
#pragma unroll
        for (int u = 0; u < kFullStep / 4; ++u) {
          const float4 b4 = *(const float4*)(t + 4 * u);
          const float bs[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const double a = qq[4 * u + k], b = (double)bs[k];
            dot = __dadd_rn(dot, __dmul_rn(a, b));
            vsum = __dadd_rn(vsum, __dmul_rn(b, b));
          }
        }
      } else {
        for (int d = 0; d < w; ++d) {
          const double a = qq[d], b = (double)t[d];
          dot = __dadd_rn(dot, __dmul_rn(a, b));
          vsum = __dadd_rn(vsum, __dmul_rn(b, b));
        }
      }
    }
    __syncthreads();  // buffer s & 1 is free for step s + 2
  }
  if (i >= n) return;
  const uint64_t r = row_of[tid];
  if (!live) {
    keys[i] = ~0ull;  // filtered rows sort last and are not reported
    scores[r] = 0.0;
    return;
  }
  if (!isfinite(vsum) || vsum <= 0.0) atomicOr(err, SVL_DEVERR_BAD_ROW);
  const double sc = __ddiv_rn(dot, __dmul_rn(qn, __dsqrt_rn(vsum)));
  scores[r] = sc;
  // f64 total order image, inverted so that larger scores get smaller keys
  uint64_t u = (uint64_t)__double_as_longlong(sc);
  u = (u & 0x8000000000000000ull) ? ~u : (u | 0x8000000000000000ull);
  keys[i] = ~u == ~0ull ? ~0ull - 1 : ~u;
}

// The first k entries of the sorted ranking (out_count zeroed by the
// caller; filtered rows carry the largest key and are not reported).
__global__ void full_emit_kernel(const uint64_t* __restrict__ sorted_rows, const uint64_t* __restrict__ sorted_keys,
                                 const double* __restrict__ scores, const uint64_t* __restrict__ chunk_ids, int k,
                                 uint64_t* out_rows, uint64_t* out_chunk_ids, double* out_scores, uint32_t* out_count) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  bool hit = false;
  if (i < k && sorted_keys[i] != ~0ull) {
    const uint64_t r = sorted_rows[i];
    out_rows[i] = r;
    out_scores[i] = scores[r];
    if (out_chunk_ids) out_chunk_ids[i] = chunk_ids[r];
    hit = true;
  }
  const int c = __syncthreads_count(hit);
  if (threadIdx.x == 0 && c) atomicAdd(out_count, (uint32_t)c);
}

// k-way merge of per-shard sorted top-k lists; one thread per query.
__global__ void merge_topk_kernel(const double* __restrict__ scores, const uint64_t* __restrict__ chunk_ids,
                                  const uint64_t* __restrict__ rows, const uint32_t* __restrict__ counts,
                                  uint32_t n_shards, uint32_t nq, uint32_t k, double* out_scores,
                                  uint64_t* out_chunk_ids, uint64_t* out_rows, uint32_t* out_shard,
                                  uint32_t* out_counts) {
  const uint32_t q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= nq) return;
  uint32_t head[64];
  for (uint32_t s = 0; s < n_shards && s < 64; ++s) head[s] = 0;
  uint32_t n = 0;
  for (; n < k; ++n) {
    int best = -1;
    double bs = 0.0;
    uint64_t bc = 0;
    for (uint32_t s = 0; s < n_shards && s < 64; ++s) {
      const uint32_t c = counts[(size_t)s * nq + q];
      if (head[s] >= c) continue;
      const size_t idx = ((size_t)s * nq + q) * k + head[s];
      const double sc = scores[idx];
      const uint64_t ch = chunk_ids[idx];
      if (best < 0 || sc > bs || (sc == bs && ch < bc)) {
        best = (int)s;
        bs = sc;
        bc = ch;
      }
    }
    if (best < 0) break;
    const size_t idx = ((size_t)best * nq + q) * k + head[best];
    out_scores[(size_t)q * k + n] = bs;
    out_chunk_ids[(size_t)q * k + n] = bc;
    if (out_rows) out_rows[(size_t)q * k + n] = rows ? rows[idx] : 0;
    if (out_shard) out_shard[(size_t)q * k + n] = (uint32_t)best;
    ++head[best];
  }
  out_counts[q] = n;
}

__global__ void iota_kernel(uint64_t* x, uint64_t n) {
  const uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (i < n) x[i] = i;
}

// ------------------------------------------------------------------ host --

namespace {

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

// rows x cols row-major matrix (FP32, or FP16 with f16) in boxes of 128
// bytes x box_rows, SWIZZLE_128B; columns past `cols` read as zeros.
bool make_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows, bool f16 = false) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  const uint64_t eb = f16 ? 2 : 4;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * eb};
  cuuint32_t box[2] = {(cuuint32_t)(128 / eb), box_rows};
  cuuint32_t elem[2] = {1, 1};
  return enc(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void*)base, dims,
             strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

// The screen for one (KC, operand type), opting in to its shared memory once
// per instantiation and device (a failed opt-in leaves the launch undone,
// which the caller's cudaGetLastError check reports).
template <int KC, bool F16>
void launch_screen(int grid, const CUtensorMap& mq, const CUtensorMap& mc, const ScreenParams& sp, cudaStream_t st) {
  static std::atomic<uint64_t> opted{0};
  if (smem_opt_in(screen_topk_kernel<KC, F16>, ScreenCfg<KC>::SMEM, &opted) != cudaSuccess) return;
  screen_topk_kernel<KC, F16><<<grid, kThreads, ScreenCfg<KC>::SMEM, st>>>(mq, mc, sp);
}

template <int KC>
void launch_screen_pair(int grid, const CUtensorMap& mq, const CUtensorMap& mc, const ScreenParams& sp,
                        cudaStream_t st) {
  static std::atomic<uint64_t> opted{0};
  if (smem_opt_in(screen_pair_kernel<KC>, PAIR_SMEM, &opted) != cudaSuccess) return;
  screen_pair_kernel<KC><<<grid, kThreads, PAIR_SMEM, st>>>(mq, mc, sp);
}

Index::~Index() {
  if (device >= 0) cudaSetDevice(device);
  if (rows) cudaFree(rows);
  if (rows16) cudaFree(rows16);
  if (chunk_ids) cudaFree(chunk_ids);
  for (auto& kv : ws) cudaFree(kv.second.ptr);
  if (err_d) cudaFree(err_d);
  if (err_h) cudaFreeHost(err_h);
  if (stream) cudaStreamDestroy(stream);
}

void* Index::workspace(const char* name, size_t bytes) {
  Buf& b = ws[name];
  if (b.bytes >= bytes) return b.ptr;
  if (b.ptr) cudaFree(b.ptr);
  b.ptr = nullptr;
  b.bytes = 0;
  const size_t rounded = (bytes + (size_t(1) << 20) - 1) & ~((size_t(1) << 20) - 1);
  if (cudaMalloc(&b.ptr, rounded) != cudaSuccess) return nullptr;
  b.bytes = rounded;
  return b.ptr;
}

int Index::create(int dev, uint32_t d, uint64_t cap, std::string* msg) {
  device = dev;
  dim = d;
  capacity = cap;
  if (d == 0) {
    *msg = "embedding must have at least one dimension";
    return SVL_USAGE;
  }
  if (d > kMaxEmbeddingDimension) {
    *msg = "embedding dimension above the 8192-dimension cap";
    return SVL_LIMIT_EXCEEDED;
  }
  if (cap > ((uint64_t)1 << 32) - 2) {
    *msg = "index capacity above 2^32 - 2 rows";
    return SVL_LIMIT_EXCEEDED;
  }
  if (cudaSetDevice(dev) != cudaSuccess) {
    *msg = "cannot select CUDA device";
    return SVL_INTERNAL;
  }
  if (cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMalloc(&err_d, 4) != cudaSuccess || cudaMallocHost(&err_h, 4) != cudaSuccess) {
    *msg = "CUDA initialisation failed";
    return SVL_INTERNAL;
  }
  cudaMemset(err_d, 0, 4);
  // FP16 screening copy for dimensions whose FP16 rows are whole 16-byte
  // units (TMA row pitch); SVL_SEARCH_TF32=1 at creation screens the FP32
  // rows in TF32 instead and saves the copy's cap * dim * 2 bytes
  const char* t = std::getenv("SVL_SEARCH_TF32");
  const bool f16 = d % 8 == 0 && !(t && t[0] == '1');
  if (cap) {
    if (cudaMalloc(&rows, cap * d * 4) != cudaSuccess || cudaMalloc(&chunk_ids, cap * 8) != cudaSuccess ||
        (f16 && cudaMalloc(&rows16, cap * d * 2) != cudaSuccess)) {
      *msg = "out of device memory for the index";
      return SVL_LIMIT_EXCEEDED;
    }
  }
  return SVL_OK;
}

int Index::append_device(const float* d_rows, const uint64_t* d_ids, uint64_t n, cudaStream_t st, bool ids_on_host,
                         const uint64_t* h_ids, std::string* msg) {
  if (n == 0) return SVL_OK;
  if (len + n > capacity) {
    *msg = "index capacity exceeded";
    return SVL_LIMIT_EXCEEDED;
  }
  float* dst = rows + len * dim;
  cudaMemcpyAsync(dst, d_rows, n * dim * 4, cudaMemcpyDefault, st);
  if (ids_on_host)
    cudaMemcpyAsync(chunk_ids + len, h_ids, n * 8, cudaMemcpyHostToDevice, st);
  else
    cudaMemcpyAsync(chunk_ids + len, d_ids, n * 8, cudaMemcpyDeviceToDevice, st);
  append_normalize_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(dst, rows16 ? rows16 + len * dim : nullptr, n,
                                                                        (int)dim, err_d);
  len += n;
  order_valid = false;
  return cudaGetLastError() == cudaSuccess ? SVL_OK : SVL_INTERNAL;
}

// Rows in ascending chunk-id order (stable), rebuilt after appends.
int Index::ensure_order(cudaStream_t st) {
  if (order_valid) return SVL_OK;
  uint64_t* iota = (uint64_t*)workspace("iota", len * 8);
  uint64_t* ord = (uint64_t*)workspace("order", len * 8);
  uint64_t* keys_out = (uint64_t*)workspace("order_keys", len * 8);
  if (!iota || !ord || !keys_out) return SVL_LIMIT_EXCEEDED;
  iota_kernel<<<(unsigned)((len + 255) / 256), 256, 0, st>>>(iota, len);
  size_t temp = 0;
  cub::DeviceRadixSort::SortPairs(nullptr, temp, chunk_ids, keys_out, iota, ord, (int64_t)len, 0, 64, st);
  void* t = workspace("cub_order", temp);
  if (!t) return SVL_LIMIT_EXCEEDED;
  cub::DeviceRadixSort::SortPairs(t, temp, chunk_ids, keys_out, iota, ord, (int64_t)len, 0, 64, st);
  order = ord;
  order_valid = true;
  return SVL_OK;
}

int Index::search_full_one(const float* d_query, double qn, const uint8_t* d_mask, uint32_t k, uint64_t* d_rows,
                           uint64_t* d_chunk, double* d_scores, uint32_t* d_count, cudaStream_t st) {
  int rc = ensure_order(st);
  if (rc) return rc;
  uint64_t* keys = (uint64_t*)workspace("full_keys", len * 8);
  uint64_t* keys_sorted = (uint64_t*)workspace("full_keys_sorted", len * 8);
  uint64_t* rows_sorted = (uint64_t*)workspace("full_rows_sorted", len * 8);
  double* scores = (double*)workspace("full_scores", len * 8);
  if (!keys || !keys_sorted || !rows_sorted || !scores) return SVL_LIMIT_EXCEEDED;
  const unsigned blocks = (unsigned)((len + kFullRows - 1) / kFullRows);
  if (dim % 4 == 0)
    full_scores_kernel<4><<<blocks, kFullRows, 0, st>>>(d_query, qn, rows, order, len, (int)dim, d_mask, keys, scores,
                                                         err_d);
  else
    full_scores_kernel<1><<<blocks, kFullRows, 0, st>>>(d_query, qn, rows, order, len, (int)dim, d_mask, keys, scores,
                                                         err_d);
  size_t temp = 0;
  cub::DeviceRadixSort::SortPairs(nullptr, temp, keys, keys_sorted, order, rows_sorted, (int64_t)len, 0, 64, st);
  void* t = workspace("cub_full", temp);
  if (!t) return SVL_LIMIT_EXCEEDED;
  cub::DeviceRadixSort::SortPairs(t, temp, keys, keys_sorted, order, rows_sorted, (int64_t)len, 0, 64, st);
  const int kk = (int)std::min<uint64_t>(k, len);
  cudaMemsetAsync(d_count, 0, 4, st);
  if (kk > 0)
    full_emit_kernel<<<(unsigned)((kk + 255) / 256), 256, 0, st>>>(rows_sorted, keys_sorted, scores, chunk_ids, kk,
                                                                   d_rows, d_chunk, d_scores, d_count);
  return cudaGetLastError() == cudaSuccess ? SVL_OK : SVL_INTERNAL;
}

// Device-resident search.  When `fallback_h` is non-null the fast path's
// per-query fallback flags are copied there (stream must be synchronised by
// the caller before reading them); with a null pointer a needed fallback
// raises SVL_DEVERR_OVERFLOW instead.
int Index::search_device(const float* d_queries, uint32_t nq, const uint8_t* d_mask, uint32_t k, uint64_t* d_rows,
                         uint64_t* d_chunk, double* d_scores, uint32_t* d_counts, cudaStream_t st,
                         uint8_t* fallback_h, std::string* msg) {
  if (nq == 0) return SVL_OK;
  if (k == 0) {
    *msg = "k must be at least 1";
    return SVL_USAGE;
  }
  const bool f16 = rows16 != nullptr;
  double* qnorm = (double*)workspace("qnorm", (size_t)nq * 8);
  // the screen's query operand, padded with zero rows to a whole query block
  // (256 rows covers both screens): a block that ran past the last query
  // would be zero-filled by the TMA on every K slice of every corpus tile,
  // which at a few queries made the screen slower than at 128
  const size_t eb = f16 ? 2 : 4;
  const size_t nq_pad = ((size_t)nq + 255) / 256 * 256;
  void* qhat = workspace("qhat", nq_pad * dim * eb);
  uint8_t* fb = (uint8_t*)workspace("fallback", nq);
  if (!qnorm || !qhat || !fb) {
    *msg = "out of device memory for the search";
    return SVL_LIMIT_EXCEEDED;
  }
  {
    Profiler::Scope sp0(&prof, kProfOther, st);
    query_prep_kernel<<<(nq + 127) / 128, 128, 0, st>>>(d_queries, (int)nq, (int)dim, qnorm,
                                                        f16 ? nullptr : (float*)qhat, f16 ? (uint16_t*)qhat : nullptr,
                                                        err_d);
  }
  cudaMemsetAsync(fb, 0, nq, st);
  cudaMemsetAsync(d_counts, 0, (size_t)nq * 4, st);
  if (nq_pad > nq) cudaMemsetAsync((uint8_t*)qhat + (size_t)nq * dim * eb, 0, (nq_pad - nq) * dim * eb, st);
  if (len == 0) return SVL_OK;
  const bool fast = k <= (uint32_t)kMaxFastK && dim % 4 == 0;
  if (fast) {
    const int kc = k <= 16 ? 16 : 32;
    // more than one 128-query block: the CTA-pair screen (256 queries per pair)
    const bool pair = f16 && nq > (uint32_t)BM;
    const int qrows = pair ? 2 * BM : BM;
    const int n_qb = (int)((nq + qrows - 1) / qrows);
    const int sms = pair ? sm_count() / 2 : sm_count();
    int n_ranges = sms / n_qb;
    if (n_ranges < 1) n_ranges = 1;
    if (2 * n_ranges * kc > kMaxCand) n_ranges = kMaxCand / (2 * kc);
    const int n_tiles = (int)((len + BN - 1) / BN);
    if (n_ranges > n_tiles) n_ranges = n_tiles;
    const int n_lists = 2 * n_ranges;
    float* cs = (float*)workspace("cand_score", (size_t)nq * n_lists * kc * 4);
    uint32_t* cr = (uint32_t*)workspace("cand_row", (size_t)nq * n_lists * kc * 4);
    float* tau = (float*)workspace("tau", (size_t)nq * n_lists * 4);
    if (!cs || !cr || !tau) {
      *msg = "out of device memory for the search";
      return SVL_LIMIT_EXCEEDED;
    }
    CUtensorMap mq, mc;
    if (!make_map(&mq, qhat, nq_pad, dim, BM, f16) ||
        !make_map(&mc, f16 ? (const void*)rows16 : rows, len, dim, pair ? BN / 2 : BN, f16)) {
      *msg = "tensor map creation failed";
      return SVL_INTERNAL;
    }
    ScreenParams sp{};
    sp.n_queries = (int)nq;
    sp.n_rows = len;
    sp.dim = (int)dim;
    sp.mask = d_mask;
    sp.n_qb = n_qb;
    sp.n_ranges = n_ranges;
    sp.n_lists = n_lists;
    sp.cand_score = cs;
    sp.cand_row = cr;
    sp.tau = tau;
    sp.err = err_d;
    const int grid = n_qb * n_ranges;
    Profiler::Scope* ss = new Profiler::Scope(&prof, kProfScreen, st);
    if (pair && kc == 16)
      launch_screen_pair<16>(2 * grid, mq, mc, sp, st);
    else if (pair)
      launch_screen_pair<32>(2 * grid, mq, mc, sp, st);
    else if (kc == 16 && f16)
      launch_screen<16, true>(grid, mq, mc, sp, st);
    else if (kc == 16)
      launch_screen<16, false>(grid, mq, mc, sp, st);
    else if (f16)
      launch_screen<32, true>(grid, mq, mc, sp, st);
    else
      launch_screen<32, false>(grid, mq, mc, sp, st);
    delete ss;
    if (n_lists * kc > kMaxCand) {
      *msg = "candidate list too long";
      return SVL_INTERNAL;
    }
    RescoreParams rp{};
    rp.queries = d_queries;
    rp.qnorm = qnorm;
    rp.rows = rows;
    rp.chunk_ids = chunk_ids;
    rp.dim = (int)dim;
    rp.n_lists = n_lists;
    rp.kc = kc;
    rp.k = (int)k;
    rp.cand_score = cs;
    rp.cand_row = cr;
    rp.tau = tau;
    rp.out_rows = d_rows;
    rp.out_chunk_ids = d_chunk;
    rp.out_scores = d_scores;
    rp.out_count = d_counts;
    rp.fallback = fb;
    rp.err = err_d;
    static std::atomic<uint64_t> rescore_opted{0};
    smem_opt_in(rescore_select_kernel, kRescoreSmem, &rescore_opted);  // a failure shows as a launch error
    {
      Profiler::Scope sp1(&prof, kProfRescore, st);
      rescore_select_kernel<<<nq, kRescoreThreads, kRescoreSmem, st>>>(rp);
    }
    if (fallback_h) cudaMemcpyAsync(fallback_h, fb, nq, cudaMemcpyDeviceToHost, st);
  } else {
    // full path for every query (host-driven loop; qnorm is needed on the host)
    std::vector<double> qn(nq);
    cudaMemcpyAsync(qn.data(), qnorm, (size_t)nq * 8, cudaMemcpyDeviceToHost, st);
    cudaStreamSynchronize(st);
    for (uint32_t q = 0; q < nq; ++q) {
      if (qn[q] <= 0.0) continue;
      int rc = search_full_one(d_queries + (size_t)q * dim, qn[q], d_mask, k, d_rows + (size_t)q * k,
                               d_chunk ? d_chunk + (size_t)q * k : nullptr, d_scores + (size_t)q * k, d_counts + q, st);
      if (rc) {
        *msg = "full-ranking search failed";
        return rc;
      }
    }
  }
  if (cudaGetLastError() != cudaSuccess) {
    *msg = "search kernel launch failed";
    return SVL_INTERNAL;
  }
  return SVL_OK;
}

// Runs the full path for the queries whose fast-path check failed.
int Index::resolve_fallbacks(const float* d_queries, uint32_t nq, const uint8_t* fallback_h, const uint8_t* d_mask,
                             uint32_t k, uint64_t* d_rows, uint64_t* d_chunk, double* d_scores, uint32_t* d_counts,
                             cudaStream_t st, std::string* msg) {
  double* qnorm = (double*)workspace("qnorm", (size_t)nq * 8);
  std::vector<double> qn;
  for (uint32_t q = 0; q < nq; ++q) {
    if (!fallback_h[q]) continue;
    if (qn.empty()) {
      qn.resize(nq);
      cudaMemcpyAsync(qn.data(), qnorm, (size_t)nq * 8, cudaMemcpyDeviceToHost, st);
      cudaStreamSynchronize(st);
    }
    ++fallbacks;
    int rc = search_full_one(d_queries + (size_t)q * dim, qn[q], d_mask, k, d_rows + (size_t)q * k,
                             d_chunk ? d_chunk + (size_t)q * k : nullptr, d_scores + (size_t)q * k, d_counts + q, st);
    if (rc) {
      *msg = "full-ranking fallback failed";
      return rc;
    }
  }
  return SVL_OK;
}

int merge_topk_device(const double* scores, const uint64_t* chunk_ids, const uint64_t* rows, const uint32_t* counts,
                      uint32_t n_shards, uint32_t nq, uint32_t k, double* out_scores, uint64_t* out_chunk_ids,
                      uint64_t* out_rows, uint32_t* out_shard, uint32_t* out_counts, cudaStream_t st) {
  if (n_shards > 64) return SVL_LIMIT_EXCEEDED;
  if (nq == 0) return SVL_OK;
  merge_topk_kernel<<<(nq + 127) / 128, 128, 0, st>>>(scores, chunk_ids, rows, counts, n_shards, nq, k, out_scores,
                                                      out_chunk_ids, out_rows, out_shard, out_counts);
  return cudaGetLastError() == cudaSuccess ? SVL_OK : SVL_INTERNAL;
}

}  // namespace svl

// --------------------------------------------------- allocation-free search --
//
// svl_search_noalloc runs the same three search kernels as svl_index_search
// (query_prep, screen_topk, rescore_select) over a corpus the caller already
// holds in device memory, without allocating anything.  It exists for callers
// that must not call cudaMalloc: a host whose device memory is carved up ahead
// of time by a pool the library must not bypass, a serving loop with a fixed
// memory budget, or a call made from a thread that may not take the driver's
// allocation lock.  All of its scratch lives in the file-scope array below:
// kNoAllocScratchBytes of device memory that every GPU loading the library
// holds until the process exits, shared by every call on that GPU.

namespace {

constexpr uint32_t kNoAllocMaxQueries = 128;  // one query block of the screen
constexpr uint32_t kNoAllocMaxDim = 1024;
constexpr uint32_t kNoAllocMaxK = 32;         // the fast path's largest k
constexpr int kNoAllocMaxRanges = 64;         // corpus ranges of the screen
constexpr size_t kNoAllocErrOff = 0;          // device error word
constexpr size_t kNoAllocQnormOff = 256;      // f64 query norms
constexpr size_t kNoAllocFallbackOff = kNoAllocQnormOff + kNoAllocMaxQueries * 8;
constexpr size_t kNoAllocQhatOff = kNoAllocFallbackOff + 256;
constexpr size_t kNoAllocTauOff = kNoAllocQhatOff + (size_t)kNoAllocMaxQueries * kNoAllocMaxDim * 4;
constexpr size_t kNoAllocCandScoreOff = kNoAllocTauOff + (size_t)kNoAllocMaxQueries * kNoAllocMaxRanges * 4;
constexpr size_t kNoAllocCandRowOff =
    kNoAllocCandScoreOff + (size_t)kNoAllocMaxQueries * kNoAllocMaxRanges * kNoAllocMaxK * 4;
constexpr size_t kNoAllocScratchBytes =
    kNoAllocCandRowOff + (size_t)kNoAllocMaxQueries * kNoAllocMaxRanges * kNoAllocMaxK * 4;  // ~2.6 MiB

// The scratch itself.  Host code must not take its address directly: on the
// host `noalloc_scratch` names a host-side stand-in, so the device address is
// looked up once per device with cudaGetSymbolAddress.
static __device__ __align__(256) uint8_t noalloc_scratch[kNoAllocScratchBytes];

constexpr int kNoAllocMaxDevices = 64;
std::mutex noalloc_mu;
uint8_t* noalloc_base[kNoAllocMaxDevices] = {};

// One-time set-up on the current device: the scratch address and the
// shared-memory opt-in of the kernels this entry point launches.
int noalloc_setup(int dev, uint8_t** base, std::string* msg) {
  std::lock_guard<std::mutex> lock(noalloc_mu);
  if (noalloc_base[dev]) {
    *base = noalloc_base[dev];
    return SVL_OK;
  }
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, noalloc_scratch);
  if (e != cudaSuccess || !p) {
    *msg = std::string("cudaGetSymbolAddress of the search scratch failed: ") + cudaGetErrorString(e);
    return SVL_INTERNAL;
  }
  if (cudaFuncSetAttribute(svl::screen_topk_kernel<16, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           svl::ScreenCfg<16>::SMEM) != cudaSuccess ||
      cudaFuncSetAttribute(svl::screen_topk_kernel<32, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           svl::ScreenCfg<32>::SMEM) != cudaSuccess ||
      cudaFuncSetAttribute(svl::rescore_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           svl::kRescoreSmem) != cudaSuccess) {
    *msg = "kernel attribute set-up failed";
    return SVL_INTERNAL;
  }
  noalloc_base[dev] = (uint8_t*)p;
  *base = (uint8_t*)p;
  return SVL_OK;
}

}  // namespace

extern "C" int svl_search_noalloc(const float* d_rows, const uint64_t* d_chunk_ids, uint64_t n_rows, uint32_t dim,
                                  const float* d_queries, uint32_t n_queries, const uint8_t* d_row_mask, uint32_t k,
                                  uint64_t* d_out_rows, uint64_t* d_out_chunk_ids, double* d_out_scores,
                                  uint32_t* d_out_counts, void* stream, char* err, size_t err_len) {
  using namespace svl;
  // d_out_chunk_ids may be NULL (the chunk ids are then not written)
  if (!d_rows || !d_chunk_ids || !d_queries || !d_out_rows || !d_out_scores || !d_out_counts) {
    set_err(err, err_len, "null argument");
    return SVL_USAGE;
  }
  if (((uintptr_t)d_rows & 15) || ((uintptr_t)d_queries & 15)) {
    set_err(err, err_len, "d_rows and d_queries must be 16-byte aligned");
    return SVL_USAGE;
  }
  if (n_queries == 0 || n_queries > kNoAllocMaxQueries) {
    set_err(err, err_len, "svl_search_noalloc takes 1.." + std::to_string(kNoAllocMaxQueries) + " queries, got " +
                              std::to_string(n_queries));
    return SVL_LIMIT_EXCEEDED;
  }
  if (dim == 0 || dim > kNoAllocMaxDim || dim % 4) {
    set_err(err, err_len, "svl_search_noalloc takes a dimension in 4.." + std::to_string(kNoAllocMaxDim) +
                              " that is a multiple of 4, got " + std::to_string(dim));
    return SVL_LIMIT_EXCEEDED;
  }
  if (k == 0 || k > kNoAllocMaxK) {
    set_err(err, err_len, "svl_search_noalloc takes k in 1.." + std::to_string(kNoAllocMaxK) + ", got " +
                              std::to_string(k));
    return SVL_LIMIT_EXCEEDED;
  }
  if (n_rows > ((uint64_t)1 << 32) - 2) {
    set_err(err, err_len, "svl_search_noalloc takes at most 2^32 - 2 rows");
    return SVL_LIMIT_EXCEEDED;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) {
    set_err(err, err_len, "no usable current CUDA device");
    return SVL_INTERNAL;
  }
  std::string msg;
  uint8_t* base = nullptr;
  int rc = noalloc_setup(dev, &base, &msg);
  if (rc) {
    set_err(err, err_len, msg);
    return rc;
  }
  cudaStream_t st = (cudaStream_t)stream;
  // an error left by earlier, unrelated launches must not be blamed on this call
  (void)cudaGetLastError();
  uint32_t* err_d = (uint32_t*)(base + kNoAllocErrOff);
  double* qnorm = (double*)(base + kNoAllocQnormOff);
  uint8_t* fallback = base + kNoAllocFallbackOff;
  float* qhat = (float*)(base + kNoAllocQhatOff);
  float* tau = (float*)(base + kNoAllocTauOff);
  float* cand_score = (float*)(base + kNoAllocCandScoreOff);
  uint32_t* cand_row = (uint32_t*)(base + kNoAllocCandRowOff);
  // the scratch keeps the previous call's contents: reset what must start at zero
  cudaMemsetAsync(err_d, 0, 4, st);
  cudaMemsetAsync(fallback, 0, n_queries, st);
  cudaMemsetAsync(d_out_counts, 0, (size_t)n_queries * 4, st);
  query_prep_kernel<<<(n_queries + 127) / 128, 128, 0, st>>>(d_queries, (int)n_queries, (int)dim, qnorm, qhat,
                                                             nullptr, err_d);
  if (n_rows > 0) {
    const int kc = k <= 16 ? 16 : 32;
    const int n_tiles = (int)((n_rows + BN - 1) / BN);
    int n_ranges = sm_count();
    if (n_ranges > kNoAllocMaxRanges / 2) n_ranges = kNoAllocMaxRanges / 2;  // two lists per range
    if (n_ranges > n_tiles) n_ranges = n_tiles;
    CUtensorMap mq, mc;
    if (!make_map(&mq, qhat, n_queries, dim, BM) || !make_map(&mc, d_rows, n_rows, dim, BN)) {
      set_err(err, err_len, "tensor map creation failed (rows must be 16-byte aligned)");
      return SVL_INTERNAL;
    }
    ScreenParams sp{};
    sp.n_queries = (int)n_queries;
    sp.n_rows = n_rows;
    sp.dim = (int)dim;
    sp.mask = d_row_mask;
    sp.n_qb = 1;
    sp.n_ranges = n_ranges;
    sp.n_lists = 2 * n_ranges;
    sp.cand_score = cand_score;
    sp.cand_row = cand_row;
    sp.tau = tau;
    sp.err = err_d;
    if (kc == 16)
      screen_topk_kernel<16, false><<<n_ranges, kThreads, ScreenCfg<16>::SMEM, st>>>(mq, mc, sp);
    else
      screen_topk_kernel<32, false><<<n_ranges, kThreads, ScreenCfg<32>::SMEM, st>>>(mq, mc, sp);
    RescoreParams rp{};
    rp.queries = d_queries;
    rp.qnorm = qnorm;
    rp.rows = d_rows;
    rp.chunk_ids = d_chunk_ids;
    rp.dim = (int)dim;
    rp.n_lists = 2 * n_ranges;
    rp.kc = kc;
    rp.k = (int)k;
    rp.cand_score = cand_score;
    rp.cand_row = cand_row;
    rp.tau = tau;
    rp.out_rows = d_out_rows;
    rp.out_chunk_ids = d_out_chunk_ids;
    rp.out_scores = d_out_scores;
    rp.out_count = d_out_counts;
    rp.fallback = fallback;
    rp.err = err_d;
    rescore_select_kernel<<<n_queries, kRescoreThreads, kRescoreSmem, st>>>(rp);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_err(err, err_len, std::string("search launch failed: ") + cudaGetErrorString(e));
    return SVL_INTERNAL;
  }
  // synchronous: the status covers the device-side checks of this call
  uint32_t word = 0;
  uint8_t flags[kNoAllocMaxQueries];
  if (cudaMemcpyAsync(&word, err_d, 4, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaMemcpyAsync(flags, fallback, n_queries, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess) {
    set_err(err, err_len, "CUDA error while finishing the search");
    return SVL_INTERNAL;
  }
  rc = status_from_device(word, &msg);
  if (rc) {
    set_err(err, err_len, msg);
    return rc;
  }
  for (uint32_t q = 0; q < n_queries; ++q)
    if (flags[q]) {
      set_err(err, err_len, "query " + std::to_string(q) +
                                " has too many near-ties for the allocation-free path; use svl_index_search");
      return SVL_UNSUPPORTED;
    }
  return SVL_OK;
}
