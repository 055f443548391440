// attention_tc.cu -- bidirectional GQA attention on the tcgen05 tensor cores
// (TF32 operands, FP32 accumulation), replacing
// kernels::bidirectional_attention (src/tensor/kernels.rs:1037-1135) for
// head dims that are multiples of 32.
//
// One CTA = one block of 128 query rows of one sequence, one query head and
// one half of the head dimension when hd > 256 (the O accumulator of a
// 128 x 512 tile would not fit TMEM next to S, so the two halves recompute S).
//   warp 0      TMA producer over the fused qkv rows: per key block, the
//               Q and K slices of 32 head dims (K-major, SWIZZLE_128B), then
//               the V slices of 32 keys x (hd / dsplit) dims (MN-major);
//   warp 1      TMEM allocator and single-thread MMA issuer:
//               S[b] = Q K^T (M 128, N 128, K 8) into one of two TMEM buffers,
//               O += P V (M 128, N hd/dsplit, K 8) with P from shared memory;
//   warps 2..5  softmax and epilogue, one query row per thread (TMEM lane):
//               masks the sequence end and the sliding window |i - j| <= W,
//               keeps a running max m and sum l, writes P = exp(S - m) to
//               shared memory in the layout the MMA reads, and rescales O only
//               when the row max grows by more than kRescale nats (otherwise
//               the stale max is kept: exp(S - m) <= e^kRescale stays finite).
// TMEM columns: S0 [0, 128), S1 [128, 256), O [256, 256 + hd/dsplit).
// Key blocks that lie entirely outside a query block's window are skipped.
// Scale 1.0 (text.rs:421).  Every wait is bounded (common.cuh).

#include <algorithm>
#include <vector>

#include "attention_tc.cuh"
#include "common.cuh"

namespace svl {

namespace {

constexpr int BQ = 128;    // query rows per CTA
constexpr int BKV = 128;   // keys per block
constexpr int DC = 32;     // head dims per Q/K slice (128 bytes)
constexpr int VK = 32;     // keys per V slice
constexpr int STAGES = 4;
constexpr int STAGE_BYTES = 32768;
constexpr int P_BYTES = BQ * BKV * 4;  // 64 KB, 4 K-major SW128 chunks of 32 keys
constexpr int SMEM = STAGES * STAGE_BYTES + P_BYTES + 1024 + 256;
constexpr int kThreads = 192;
constexpr float kRescale = 8.0f;
constexpr float kLog2e = 1.4426950408889634f;
static_assert(SMEM <= 232448, "shared memory");

struct WorkItem {
  uint32_t seq_start, len, q0, pad;
};


__global__ void __launch_bounds__(kThreads, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap map_qk, const __grid_constant__ CUtensorMap map_v,
                        const WorkItem* __restrict__ items, AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* ring = smem;
  uint8_t* pbuf = smem + STAGES * STAGE_BYTES;
  uint64_t* full = (uint64_t*)(pbuf + P_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* s_full = empty + STAGES;  // [2]
  uint64_t* s_free = s_full + 2;      // [2]
  uint64_t* p_full = s_free + 2;
  uint64_t* pv_done = p_full + 1;
  uint32_t* tmem_slot = (uint32_t*)(pv_done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const WorkItem it = items[blockIdx.x];
  const int h = blockIdx.y;
  const int dh = blockIdx.z;                 // which half of the head dim
  const int dn = p.hd / p.dsplit;            // output dims of this CTA (MMA N of P V)
  const int kvh = h / (p.nh / p.kvh);
  const int L = (int)it.len;
  const int q0 = (int)it.q0;
  // key blocks that can hold a key of some query row of this block
  int kb_lo = 0, kb_hi = (L - 1) / BKV;
  if (p.window >= 0) {
    const int lo = q0 - p.window, hi = q0 + BQ - 1 + p.window;
    kb_lo = lo > 0 ? lo / BKV : 0;
    kb_hi = (hi < L - 1 ? hi : L - 1) / BKV;
  }
  const int nblk = kb_hi - kb_lo + 1;
  const int n_dc = p.hd / DC;  // Q/K slices per key block
  const int n_vs = BKV / VK;   // V slices per key block
  const int q_col = h * p.hd;
  const int k_col = (p.nh + kvh) * p.hd;
  const int v_col = (p.nh + p.kvh + kvh) * p.hd + dh * dn;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_free[b], 128);
    }
    mbar_init(p_full, 128);
    mbar_init(pv_done, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&map_qk);
      tma_prefetch_desc(&map_v);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      auto next = [&]() {
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      };
      auto load_s = [&](int j) {
        const int krow = (int)it.seq_start + (kb_lo + j) * BKV;
        for (int c = 0; ok && c < n_dc; ++c) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.err)) {
            ok = false;
            return;
          }
          uint8_t* dst = ring + stage * STAGE_BYTES;
          mbar_arrive_expect_tx(&full[stage], 2 * BQ * DC * 4);
          tma_load_2d(dst, &map_qk, &full[stage], q_col + c * DC, (int)it.seq_start + q0);
          tma_load_2d(dst + BQ * DC * 4, &map_qk, &full[stage], k_col + c * DC, krow);
          next();
        }
      };
      auto load_v = [&](int j) {
        const int krow = (int)it.seq_start + (kb_lo + j) * BKV;
        for (int s = 0; ok && s < n_vs; ++s) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.err)) {
            ok = false;
            return;
          }
          uint8_t* dst = ring + stage * STAGE_BYTES;
          mbar_arrive_expect_tx(&full[stage], VK * dn * 4);
          for (int c = 0; c < dn / DC; ++c)
            tma_load_2d(dst + c * (VK * DC * 4), &map_v, &full[stage], v_col + c * DC, krow + s * VK);
          next();
        }
      };
      for (int j = 0; ok && j < nblk; ++j) {
        load_s(j);
        if (j >= 1) load_v(j - 1);
      }
      if (ok) load_v(nblk - 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc_s = idesc_tf32(BQ, BKV, 0);
      const uint32_t idesc_o = idesc_tf32(BQ, (uint32_t)dn, 1);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      auto next = [&]() {
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      };
      auto issue_s = [&](int j) {
        const int b = j & 1;
        if (!mbar_wait(&s_free[b], ((j >> 1) & 1) ^ 1, p.err)) {
          ok = false;
          return;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(b * BKV);
        for (int c = 0; c < n_dc; ++c) {
          if (!mbar_wait(&full[stage], phase, p.err)) {
            ok = false;
            return;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(ring + stage * STAGE_BYTES);
          const uint32_t bb = a + BQ * DC * 4;
#pragma unroll
          for (int k = 0; k < DC / 8; ++k)
            mma_tf32(d, sdesc(a + k * 32, 16, 1024, kLayoutSW128), sdesc(bb + k * 32, 16, 1024, kLayoutSW128),
                     idesc_s, (c | k) != 0);
          mma_commit(&empty[stage]);
          next();
        }
        mma_commit(&s_full[b]);
      };
      auto issue_pv = [&](int j) {
        if (!mbar_wait(p_full, j & 1, p.err)) {
          ok = false;
          return;
        }
        tc_fence_after();
        const uint32_t d = tmem + 256;
        const uint32_t pa = smem_u32(pbuf);
        for (int s = 0; s < n_vs; ++s) {
          if (!mbar_wait(&full[stage], phase, p.err)) {
            ok = false;
            return;
          }
          tc_fence_after();
          const uint32_t v = smem_u32(ring + stage * STAGE_BYTES);
#pragma unroll
          for (int k = 0; k < VK / 8; ++k)
            // B = V slice, MN-major SWIZZLE_128B_BASE32B: atoms of 4 key rows x
            // 128 bytes (SBO 512), 32-dim chunks 4 KB apart (LBO), 8 keys per MMA
            mma_tf32(d, sdesc(pa + s * (BQ * 128) + k * 32, 16, 1024, kLayoutSW128),
                     sdesc(v + k * 1024, VK * DC * 4, 512, kLayoutSW128Base32B), idesc_o, (j | s | k) != 0);
          mma_commit(&empty[stage]);
          next();
        }
        mma_commit(pv_done);
      };
      for (int j = 0; ok && j < nblk; ++j) {
        issue_s(j);
        if (ok && j >= 1) issue_pv(j - 1);
      }
      if (ok) issue_pv(nblk - 1);
    }
  } else {
    // softmax / epilogue warps: thread owns query row r of the block
    const int lg = warp & 3;
    const int r = lg * 32 + lane;
    const int qi = q0 + r;
    const bool q_valid = qi < L;
    const uint32_t lane_addr = (uint32_t)(lg * 32) << 16;
    // keys this row attends: [key_lo, key_hi] (empty for rows past the sequence end)
    int key_lo = 0, key_hi = L - 1;
    if (p.window >= 0) {
      key_lo = qi - p.window > 0 ? qi - p.window : 0;
      key_hi = qi + p.window < L - 1 ? qi + p.window : L - 1;
    }
    if (!q_valid) {
      key_lo = 1 << 30;
      key_hi = -1;
    }
    float m = -INFINITY, l = 0.0f;
    bool bad = false, ok = true;
    for (int j = 0; j < nblk; ++j) {
      const int b = j & 1;
      const bool got = mbar_wait(&s_full[b], (j >> 1) & 1, p.err);
      __syncwarp();
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[BKV];
#pragma unroll
      for (int c = 0; c < BKV / 32; ++c) tmem_ld32(tmem + lane_addr + b * BKV + c * 32, s + c * 32);
      tc_fence_before();
      mbar_arrive(&s_free[b]);
      const int k0 = (kb_lo + j) * BKV;
      if (k0 < key_lo || k0 + BKV - 1 > key_hi) {  // block straddles this row's key range
#pragma unroll
        for (int c = 0; c < BKV; ++c)
          if (k0 + c < key_lo || k0 + c > key_hi) s[c] = -INFINITY;
      }
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < BKV; c += 4) mx = fmaxf(mx, fmaxf(fmaxf(s[c], s[c + 1]), fmaxf(s[c + 2], s[c + 3])));
      bad |= mx == INFINITY;
      float m_new = m;
      bool rescale = false;
      if (mx > m + kRescale || (m == -INFINITY && mx > -INFINITY)) {
        m_new = mx;
        rescale = m != -INFINITY;  // O and l are still zero while m is -inf
      }
      // exp(s - m) = exp2(s * log2(e) - m * log2(e)); masked scores are -inf -> 0
      const float ml = m_new == -INFINITY ? 0.0f : m_new * kLog2e;
      float rowsum = 0.0f;
#pragma unroll
      for (int c = 0; c < BKV; ++c) {
        const float e = exp2f(fmaf(s[c], kLog2e, -ml));
        s[c] = round_tf32(e);
        rowsum += e;
      }
      // P buffer and O are touched only after P V of the previous block finished
      if (j >= 1) {
        const bool pv = mbar_wait(pv_done, (j - 1) & 1, p.err);
        __syncwarp();
        if (!__all_sync(0xffffffffu, pv)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      const float factor = rescale ? expf(m - m_new) : 1.0f;
      if (__any_sync(0xffffffffu, rescale)) {
        float o[32];
        for (int c = 0; c < dn / 32; ++c) {
          const uint32_t addr = tmem + lane_addr + 256 + c * 32;
          tmem_ld32(addr, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= factor;
          tmem_st32(addr, o);
        }
        tmem_st_wait();
      }
      l = l * factor + rowsum;
      m = m_new;
      // P row r into the four K-major SWIZZLE_128B chunks (32 keys each)
#pragma unroll
      for (int c = 0; c < BKV / 32; ++c) {
        uint8_t* row = pbuf + c * (BQ * 128) + r * 128;
#pragma unroll
        for (int u = 0; u < 8; ++u)
          *(float4*)(row + ((u ^ (r & 7)) * 16)) =
              make_float4(s[c * 32 + 4 * u], s[c * 32 + 4 * u + 1], s[c * 32 + 4 * u + 2], s[c * 32 + 4 * u + 3]);
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok) {
      const bool fin = mbar_wait(pv_done, (nblk - 1) & 1, p.err);
      __syncwarp();
      if (__all_sync(0xffffffffu, fin)) {
        tc_fence_after();
        bad |= q_valid && !isfinite(l);
        const float inv = 1.0f / l;
        float* out = p.out + (size_t)(it.seq_start + (uint32_t)qi) * p.ld_out + h * p.hd + dh * dn;
        float o[32];
        for (int c = 0; c < dn / 32; ++c) {
          tmem_ld32(tmem + lane_addr + 256 + c * 32, o);
          if (q_valid) {
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
              float4 v4 = make_float4(o[i] * inv, o[i + 1] * inv, o[i + 2] * inv, o[i + 3] * inv);
              if (p.round_out) {
                v4.x = round_tf32(v4.x);
                v4.y = round_tf32(v4.y);
                v4.z = round_tf32(v4.z);
                v4.w = round_tf32(v4.w);
              }
              bad |= !isfinite(v4.x) || !isfinite(v4.y) || !isfinite(v4.z) || !isfinite(v4.w);
              *(float4*)(out + c * 32 + i) = v4;
            }
          }
        }
      }
    }
    if (bad) atomicOr(p.err, SVL_DEVERR_NONFINITE);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------ CTA-pair kernel --
// attention_pair_kernel: the two query heads 2 hp and 2 hp + 1 that share a
// KV head (even GQA group), over the same 128-query block, run as one M = 256
// tile on a CTA pair (cta_group::2): CTA `rank` owns head 2 hp + rank.  Per
// 128-key block j:
//   S[j & 1] = Q K^T   M 256, N 128: A = this CTA's resident Q (loaded once),
//                      B = 64 keys from each CTA (K-major, 64 dims per stage);
//   P = softmax rows, written back over S[j & 1] in TMEM (tcgen05.st);
//   O += P V           M 256, N hd: A = P read from TMEM, B = hd / 2 value
//                      dims from each CTA (MN-major, 32 keys per stage).
// Each CTA therefore streams half of K and half of V per block, Q is read
// from memory once, and P never touches shared memory.  For hd = 256 a CTA's
// shared memory moves ~384 KB per block (128 KB of TMA writes, 192 KB of S
// operands, 64 KB of V) for 16.8 MFLOP, against ~900 KB in the one-CTA
// kernel: shared-memory bandwidth is what bounds an M = 128 TF32 MMA.
//
// Warps: 0 loads Q and K (K ring), 6 loads V (V ring), 1 issues the MMAs
// (leader CTA), 2..5 run the softmax and the epilogue.  The issuer follows
// the dependencies rather than a fixed order: S(j) may start once PV(j - 2)
// has finished reading P from the same TMEM columns, PV(j) once both CTAs'
// softmax wrote P(j); when both are ready S goes first, so the softmax warps
// (the scarcer resource at TF32 rates) never wait behind a P V product.
// K and V have separate FIFO rings because that order is data dependent.
// TMEM columns (per CTA): S0 [0, 128), S1 [128, 256), O [256, 256 + hd).
constexpr int PQ_BYTES = BQ * 256 * 4;  // resident Q for hd <= 256 (128 KB)
constexpr int PSTAGE_BYTES = 16384;
constexpr int PK_STAGES = 3;
constexpr int PV_STAGES = 3;
constexpr int PKEYS = BKV / 2;  // keys per CTA per block (B rows of S)
constexpr int PSMEM = PQ_BYTES + (PK_STAGES + PV_STAGES) * PSTAGE_BYTES + 1024 + 256;
constexpr int kPairThreads = 224;
constexpr int kPrefetchBlocks = 4;  // key blocks of K / V pulled into L2 ahead
static_assert(PSMEM <= 232448, "shared memory");

struct PairItem {
  uint32_t seq_start, len, q0, hp;
};

// One FIFO ring of shared-memory stages: the producer's and the consumer's
// position.
struct Ring {
  uint8_t* base;
  uint64_t* full;
  uint64_t* empty;
  int n;
  int stage = 0;
  uint32_t phase = 0;
  SVL_DEV uint8_t* at() const { return base + stage * PSTAGE_BYTES; }
  SVL_DEV void next() {
    if (++stage == n) {
      stage = 0;
      phase ^= 1;
    }
  }
};

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPairThreads, 1)
    attention_pair_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                          const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_o,
                          const PairItem* __restrict__ items, AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* qbuf = smem;  // hd / 32 chunks of 128 rows x 128 B (K-major SW128)
  uint8_t* kring = smem + PQ_BYTES;
  uint8_t* vring = kring + PK_STAGES * PSTAGE_BYTES;
  uint64_t* bars = (uint64_t*)(vring + PV_STAGES * PSTAGE_BYTES);
  uint64_t* k_full = bars;
  uint64_t* k_empty = k_full + PK_STAGES;
  uint64_t* v_full = k_empty + PK_STAGES;
  uint64_t* v_empty = v_full + PV_STAGES;
  uint64_t* q_full = v_empty + PV_STAGES;
  uint64_t* s_full = q_full + 1;   // [2]
  uint64_t* p_full = s_full + 2;   // [2], leader only
  uint64_t* pv_done = p_full + 2;  // [2]
  uint32_t* tmem_slot = (uint32_t*)(pv_done + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank() & 1u;
  const bool leader = rank == 0;
  const PairItem it = items[blockIdx.x >> 1];
  const int hd = p.hd, hd2 = p.hd / 2;
  const int h = 2 * (int)it.hp + (int)rank;
  const int kvh = h / (p.nh / p.kvh);
  const int L = (int)it.len;
  const int q0 = (int)it.q0;
  const int row0 = (int)it.seq_start;
  int kb_lo = 0, kb_hi = (L - 1) / BKV;
  if (p.window >= 0) {
    const int lo = q0 - p.window, hi = q0 + BQ - 1 + p.window;
    kb_lo = lo > 0 ? lo / BKV : 0;
    kb_hi = (hi < L - 1 ? hi : L - 1) / BKV;
  }
  const int nblk = kb_hi - kb_lo + 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < PK_STAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < PV_STAGES; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    mbar_init(q_full, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], 8);  // 4 softmax warps x 2 CTAs
      mbar_init(&pv_done[b], 1);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncwarp();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 || warp == 6) {
    if (lane == 0) {
      // producers of both CTAs; every load completes on the leader's barrier
      const bool is_k = warp == 0;
      Ring ring{is_k ? kring : vring, is_k ? k_full : v_full, is_k ? k_empty : v_empty,
                is_k ? PK_STAGES : PV_STAGES};
      if (is_k) {
        tma_prefetch_desc(&map_q);
        tma_prefetch_desc(&map_k);
        if (leader) mbar_arrive_expect_tx(q_full, 2 * BQ * hd * 4);
        const uint32_t qbar = map_to_rank(smem_u32(q_full), 0);
        for (int c = 0; c < hd / DC; ++c)
          tma_load_2d_pair(qbuf + c * (BQ * DC * 4), &map_q, qbar, h * hd + c * DC, row0 + q0);
      } else {
        tma_prefetch_desc(&map_v);
      }
      const int k_col = (p.nh + kvh) * hd;
      const int v_col = (p.nh + p.kvh + kvh) * hd + (int)rank * hd2;
      const int per_block = is_k ? hd / 64 : BKV / VK;
      const uint32_t bytes = is_k ? 2 * 2 * PKEYS * DC * 4 : 2 * VK * hd2 * 4;
      // Pull this CTA's K (or V) tiles of the next kPrefetchBlocks key blocks
      // into L2 ahead of the ring: the ring then waits on L2, not on DRAM.
      auto prefetch = [&](int j) {
        const int krow = row0 + (kb_lo + j) * BKV;
        if (is_k) {
          for (int c = 0; c < hd / DC; ++c) tma_prefetch_l2_2d(&map_k, k_col + c * DC, krow + (int)rank * PKEYS);
        } else {
          for (int s = 0; s < BKV / VK; ++s)
            for (int c = 0; c < hd2 / DC; ++c) tma_prefetch_l2_2d(&map_v, v_col + c * DC, krow + s * VK);
        }
      };
      for (int j = 0; j < nblk && j < kPrefetchBlocks; ++j) prefetch(j);
      bool ok = true;
      for (int j = 0; ok && j < nblk; ++j) {
        const int krow = row0 + (kb_lo + j) * BKV;
        if (j + kPrefetchBlocks < nblk) prefetch(j + kPrefetchBlocks);
        for (int s = 0; s < per_block; ++s) {
          if (!mbar_wait(&ring.empty[ring.stage], ring.phase ^ 1, p.err)) {
            ok = false;
            break;
          }
          uint8_t* dst = ring.at();
          if (leader) mbar_arrive_expect_tx(&ring.full[ring.stage], bytes);
          const uint32_t bar = map_to_rank(smem_u32(&ring.full[ring.stage]), 0);
          if (is_k) {
            tma_load_2d_pair(dst, &map_k, bar, k_col + s * 64, krow + (int)rank * PKEYS);
            tma_load_2d_pair(dst + PKEYS * DC * 4, &map_k, bar, k_col + s * 64 + DC, krow + (int)rank * PKEYS);
          } else {
            for (int c = 0; c < hd2 / DC; ++c)
              tma_load_2d_pair(dst + c * (VK * DC * 4), &map_v, bar, v_col + c * DC, krow + s * VK);
          }
          ring.next();
        }
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      const uint32_t idesc_s = idesc_tf32(2 * BQ, BKV, 0);
      const uint32_t idesc_o = idesc_tf32(2 * BQ, (uint32_t)hd, 1);
      Ring kr{kring, k_full, k_empty, PK_STAGES};
      Ring vr{vring, v_full, v_empty, PV_STAGES};
      bool ok = mbar_wait(q_full, 0, p.err);
      tc_fence_after();
      const uint32_t qa = smem_u32(qbuf);
      auto issue_s = [&](int j) {
        const uint32_t d = tmem + (uint32_t)((j & 1) * BKV);
        for (int c = 0; ok && c < hd / 64; ++c) {
          if (!mbar_wait(&kr.full[kr.stage], kr.phase, p.err)) {
            ok = false;
            return;
          }
          tc_fence_after();
          const uint32_t kb = smem_u32(kr.at());
#pragma unroll
          for (int hh = 0; hh < 2; ++hh)
#pragma unroll
            for (int k = 0; k < DC / 8; ++k)
              mma_tf32_pair(d, sdesc(qa + (2 * c + hh) * (BQ * DC * 4) + k * 32, 16, 1024, kLayoutSW128),
                            sdesc(kb + hh * (PKEYS * DC * 4) + k * 32, 16, 1024, kLayoutSW128), idesc_s,
                            (c | hh | k) != 0);
          mma_commit_pair(&kr.empty[kr.stage], 0x3);
          kr.next();
        }
        mma_commit_pair(&s_full[j & 1], 0x3);
      };
      auto issue_pv = [&](int j) {
        const uint32_t d = tmem + 256;
        const uint32_t pa = tmem + (uint32_t)((j & 1) * BKV);
        for (int s = 0; ok && s < BKV / VK; ++s) {
          if (!mbar_wait(&vr.full[vr.stage], vr.phase, p.err)) {
            ok = false;
            return;
          }
          tc_fence_after();
          const uint32_t v = smem_u32(vr.at());
#pragma unroll
          for (int k = 0; k < VK / 8; ++k)
            mma_tf32_pair_ts(d, pa + (uint32_t)(s * VK + k * 8),
                             sdesc(v + k * 1024, VK * DC * 4, 512, kLayoutSW128Base32B), idesc_o, (j | s | k) != 0);
          mma_commit_pair(&vr.empty[vr.stage], 0x3);
          vr.next();
        }
        mma_commit_pair(&pv_done[j & 1], 0x3);
      };
      // ns: next S to issue, np: next PV.  S(ns) needs its TMEM buffer back
      // (PV(ns - 2) issued and finished); PV(np) needs P(np) from both CTAs.
      int ns = 0, np = 0;
      uint64_t idle_since = 0;
      while (ok && np < nblk) {
        if (ns < nblk && ns < np + 2 && (ns < 2 || mbar_test(&pv_done[ns & 1], ((ns - 2) >> 1) & 1))) {
          tc_fence_after();
          issue_s(ns++);
          idle_since = 0;
        } else if (np < ns && mbar_test_cluster(&p_full[np & 1], (np >> 1) & 1)) {
          tc_fence_after();
          issue_pv(np++);
          idle_since = 0;
        } else if (idle_since == 0) {
          idle_since = global_ns();
        } else if (global_ns() - idle_since > kWaitDeadlineNs) {
          atomicOr(p.err, SVL_DEVERR_TIMEOUT);
          ok = false;
        }
      }
    }
  } else {
    // softmax / epilogue warps of both CTAs: thread owns query row r of its head
    const int lg = warp & 3;
    const int r = lg * 32 + lane;
    const int qi = q0 + r;
    const bool q_valid = qi < L;
    const uint32_t lane_addr = (uint32_t)(lg * 32) << 16;
    int key_lo = 0, key_hi = L - 1;
    if (p.window >= 0) {
      key_lo = qi - p.window > 0 ? qi - p.window : 0;
      key_hi = qi + p.window < L - 1 ? qi + p.window : L - 1;
    }
    if (!q_valid) {
      key_lo = 1 << 30;
      key_hi = -1;
    }
    const uint32_t p_full_leader0 = map_to_rank(smem_u32(&p_full[0]), 0);
    const uint32_t p_full_leader1 = map_to_rank(smem_u32(&p_full[1]), 0);
    float m = -INFINITY, l = 0.0f;
    bool bad = false, ok = true;
    for (int j = 0; j < nblk; ++j) {
      const int b = j & 1;
      const bool got = mbar_wait(&s_full[b], (j >> 1) & 1, p.err);
      __syncwarp();
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sr[BKV];
#pragma unroll
      for (int c = 0; c < BKV / 32; ++c) tmem_ld32_nowait(tmem + lane_addr + b * BKV + c * 32, sr + c * 32);
      tmem_ld_wait();
#pragma unroll
      for (int c = 0; c < BKV / 32; ++c) tmem_regs_after_wait(sr + c * 32);
      auto sv = [&](int c) { return __uint_as_float(sr[c]); };
      const int k0 = (kb_lo + j) * BKV;
      if (k0 < key_lo || k0 + BKV - 1 > key_hi) {
#pragma unroll
        for (int c = 0; c < BKV; ++c)
          if (k0 + c < key_lo || k0 + c > key_hi) sr[c] = __float_as_uint(-INFINITY);
      }
      // row max over four independent chains
      float mq[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        mq[q] = fmax3(sv(q * 32), sv(q * 32 + 1), sv(q * 32 + 2));
#pragma unroll
        for (int c = 3; c < 31; c += 2) mq[q] = fmax3(mq[q], sv(q * 32 + c), sv(q * 32 + c + 1));
        mq[q] = fmaxf(mq[q], sv(q * 32 + 31));
      }
      const float mx = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3]));
      bad |= mx == INFINITY;
      float m_new = m;
      bool rescale = false;
      if (mx > m + kRescale || (m == -INFINITY && mx > -INFINITY)) {
        m_new = mx;
        rescale = m != -INFINITY;
      }
      const float factor = rescale ? expf(m - m_new) : 1.0f;
      if (__any_sync(0xffffffffu, rescale)) {
        // O may be rescaled only once PV(j - 1) has finished accumulating
        const bool pv = mbar_wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, p.err);
        __syncwarp();
        if (!__all_sync(0xffffffffu, pv)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float o[32];
        for (int c = 0; c < hd / 32; ++c) {
          const uint32_t addr = tmem + lane_addr + 256 + c * 32;
          tmem_ld32(addr, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= factor;
          tmem_st32(addr, o);
        }
      }
      // P = 2^(s log2(e) - m log2(e)) rounded to the TF32 grid (nearest, ties
      // away: add half a TF32 unit, clear the 13 low bits), stored over S one
      // 32-column chunk at a time; l sums exactly the weights the tensor core
      // multiplies
      const float ml = m_new == -INFINITY ? 0.0f : m_new * kLog2e;
      float rs[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int q = 0; q < BKV / 32; ++q) {
#pragma unroll
        for (int c = q * 32; c < q * 32 + 32; ++c) {
          const float e = ex2_approx(fmaf(sv(c), kLog2e, -ml));
          sr[c] = (__float_as_uint(e) + 0x1000u) & 0xFFFFE000u;
          rs[c & 3] += __uint_as_float(sr[c]);
        }
        tmem_st32(tmem + lane_addr + b * BKV + q * 32, sr + q * 32);
      }
      l = l * factor + ((rs[0] + rs[1]) + (rs[2] + rs[3]));
      m = m_new;
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (leader)
          mbar_arrive(&p_full[b]);
        else
          mbar_arrive_cluster(b ? p_full_leader1 : p_full_leader0);
      }
    }
    if (ok) {
      const int jl = nblk - 1;
      const bool fin = mbar_wait(&pv_done[jl & 1], (jl >> 1) & 1, p.err);
      __syncwarp();
      if (__all_sync(0xffffffffu, fin)) {
        tc_fence_after();
        bad |= q_valid && !isfinite(l);
        const float inv = 1.0f / l;
        // every MMA has completed: the Q buffer is free for the store staging
        float* stage_buf = (float*)(qbuf + (warp - 2) * (PQ_BYTES / 4));  // 32 KB per warp
        const bool whole = q0 + lg * 32 + 32 <= L;  // the warp's 32 rows are all in the sequence
        float* out = p.out + (size_t)(row0 + qi) * p.ld_out + h * hd;
        float o[32];
        for (int c = 0; c < hd / 32; ++c) {
          tmem_ld32(tmem + lane_addr + 256 + c * 32, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            float v = o[i] * inv;
            if (p.round_out) v = round_tf32(v);
            bad |= q_valid && !isfinite(v);
            o[i] = v;
          }
          if (whole) {
            // a staging chunk of its own per column block: no store waits on another
            float* st = stage_buf + c * 1024;
            uint8_t* row = (uint8_t*)st + lane * 128;
#pragma unroll
            for (int u = 0; u < 8; ++u)
              *(float4*)(row + ((u ^ (lane & 7)) * 16)) =
                  make_float4(o[4 * u], o[4 * u + 1], o[4 * u + 2], o[4 * u + 3]);
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&map_o, st, h * hd + c * 32, row0 + q0 + lg * 32);
              tma_store_commit();
            }
          } else if (q_valid) {
#pragma unroll
            for (int i = 0; i < 32; i += 4)
              *(float4*)(out + c * 32 + i) = make_float4(o[i], o[i + 1], o[i + 2], o[i + 3]);
          }
        }
        if (lane == 0) tma_store_wait_all();
      }
    }
    if (bad) atomicOr(p.err, SVL_DEVERR_NONFINITE);
  }
  tc_fence_before();
  __syncwarp();
  cluster_sync();  // no CTA of the pair leaves while the other may still read or signal it
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)ptr;
  }
  return fn;
}

// Q / K slices use the 128-byte swizzle (K-major operands); V slices use the
// 128-byte swizzle with 32-byte atomicity, the only shared-memory layout the
// tensor core accepts for an MN-major 32-bit operand.
bool make_map(CUtensorMap* map, const float* base, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows,
              bool mn_major) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 4};
  cuuint32_t box[2] = {(cuuint32_t)DC, box_rows};
  cuuint32_t elem[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void*)base, dims, strides, box, elem,
             CU_TENSOR_MAP_INTERLEAVE_NONE, mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool attention_tc_supported(int hd) { return hd % 32 == 0 && hd >= 32 && hd <= 512; }

namespace {

bool pair_eligible(const AttnParams& p) {
  return !p.single_cta && p.hd % 64 == 0 && p.hd <= 256 && p.kvh > 0 && p.nh % p.kvh == 0 &&
         (p.nh / p.kvh) % 2 == 0 && p.ld_out % 4 == 0 && ((uintptr_t)p.out & 15) == 0;
}

int key_blocks(uint32_t len, uint32_t q0, int window) {
  int lo = 0, hi = ((int)len - 1) / BKV;
  if (window >= 0) {
    const int a = (int)q0 - window, b = (int)q0 + BQ - 1 + window;
    lo = a > 0 ? a / BKV : 0;
    hi = (b < (int)len - 1 ? b : (int)len - 1) / BKV;
  }
  return hi - lo + 1;
}

cudaError_t launch_pair(const AttnParams& p, const uint64_t* cu_host, int batch, void* d_items_ws, size_t ws_bytes,
                        cudaStream_t st) {
  // one work item per (128-query block, head pair), longest first so the
  // block scheduler hands out the heavy pairs before the light ones
  std::vector<PairItem> items;
  std::vector<int> cost;
  for (int b = 0; b < batch; ++b) {
    const uint32_t s = (uint32_t)cu_host[b], n = (uint32_t)(cu_host[b + 1] - cu_host[b]);
    for (uint32_t q0 = 0; q0 < n; q0 += BQ)
      for (int hp = 0; hp < p.nh / 2; ++hp) items.push_back({s, n, q0, (uint32_t)hp});
  }
  if (items.empty()) return cudaSuccess;
  if (items.size() * sizeof(PairItem) > ws_bytes) return cudaErrorInvalidValue;
  std::stable_sort(items.begin(), items.end(), [&](const PairItem& a, const PairItem& b) {
    return key_blocks(a.len, a.q0, p.window) > key_blocks(b.len, b.q0, p.window);
  });
  cudaError_t e = cudaMemcpyAsync(d_items_ws, items.data(), items.size() * sizeof(PairItem), cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) return e;
  CUtensorMap mq, mk, mv, mo;
  const uint64_t width = (uint64_t)(p.nh + 2 * p.kvh) * p.hd;
  if (!make_map(&mq, p.qkv, (uint64_t)p.T, width, (uint64_t)p.ld, BQ, false) ||
      !make_map(&mk, p.qkv, (uint64_t)p.T, width, (uint64_t)p.ld, PKEYS, false) ||
      !make_map(&mv, p.qkv, (uint64_t)p.T, width, (uint64_t)p.ld, VK, true) ||
      !make_map(&mo, p.out, (uint64_t)p.T, (uint64_t)p.nh * p.hd, (uint64_t)p.ld_out, 32, false))
    return cudaErrorInvalidValue;
  static std::atomic<uint64_t> opted{0};
  e = smem_opt_in(attention_pair_kernel, PSMEM, &opted);
  if (e != cudaSuccess) return e;
  attention_pair_kernel<<<(unsigned)(2 * items.size()), kPairThreads, PSMEM, st>>>(mq, mk, mv, mo,
                                                                             (const PairItem*)d_items_ws, p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_attention_tc(const AttnParams& prm, const uint64_t* cu_host, int batch, void* d_items_ws,
                                size_t ws_bytes, cudaStream_t st) {
  if (!attention_tc_supported(prm.hd)) return cudaErrorInvalidValue;
  AttnParams p = prm;
  if (pair_eligible(p)) {
    p.dsplit = 1;
    return launch_pair(p, cu_host, batch, d_items_ws, ws_bytes, st);
  }
  p.dsplit = p.hd > 256 ? 2 : 1;
  // one work item per 128-row query block of every sequence
  std::vector<WorkItem> items;
  for (int b = 0; b < batch; ++b) {
    const uint32_t s = (uint32_t)cu_host[b], n = (uint32_t)(cu_host[b + 1] - cu_host[b]);
    for (uint32_t q0 = 0; q0 < n; q0 += BQ) items.push_back({s, n, q0, 0});
  }
  if (items.empty()) return cudaSuccess;
  if (items.size() * sizeof(WorkItem) > ws_bytes) return cudaErrorInvalidValue;
  cudaError_t e = cudaMemcpyAsync(d_items_ws, items.data(), items.size() * sizeof(WorkItem), cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) return e;
  CUtensorMap mqk, mv;
  const uint64_t width = (uint64_t)(p.nh + 2 * p.kvh) * p.hd;
  if (!make_map(&mqk, p.qkv, (uint64_t)p.T, width, (uint64_t)p.ld, BQ, false) ||
      !make_map(&mv, p.qkv, (uint64_t)p.T, width, (uint64_t)p.ld, VK, true))
    return cudaErrorInvalidValue;
  static std::atomic<uint64_t> opted{0};
  e = smem_opt_in(attention_tc_kernel, SMEM, &opted);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)items.size(), (unsigned)p.nh, (unsigned)p.dsplit);
  attention_tc_kernel<<<grid, kThreads, SMEM, st>>>(mqk, mv, (const WorkItem*)d_items_ws, p);
  return cudaGetLastError();
}

size_t attention_tc_items_bytes(const uint64_t* cu_host, int batch, int nh) {
  size_t n = 0;
  for (int b = 0; b < batch; ++b) n += (size_t)((cu_host[b + 1] - cu_host[b] + BQ - 1) / BQ);
  // the CTA-pair kernel has one item per query block and head pair
  const size_t per = nh > 2 ? (size_t)(nh / 2) : 1;
  return n * per * sizeof(PairItem);
}

}  // namespace svl
