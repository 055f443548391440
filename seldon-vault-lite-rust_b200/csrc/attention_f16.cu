// attention_f16.cu -- bidirectional GQA attention on a CTA pair with FP16
// tensor-core operands (kind::f16, FP32 accumulation), replacing
// kernels::bidirectional_attention (src/tensor/kernels.rs:1037-1135) for head
// dims 128, 256 and 512 when every KV head serves an even number of query
// heads (all EmbeddingGemma layers).
//
// Precision: q and k are RMS-normalised with their weights and v without
// (text.rs:370-405), so |q|, |k|, |v| stay within sqrt(hd) times the norm
// weights; P = exp(S - m) stays below e^8 under the lazy rescale below.  FP16
// holds all of these with an 11-bit significand -- the same as TF32 -- so the
// products carry exactly the TF32 rounding of the other tensor-core paths,
// while the operands take half the bytes and the MMA runs at twice the TF32
// rate.  A value beyond the FP16 range would become infinite and is reported
// as a non-finite activation by the producer's check.
//
// Work item = (128-query block of one sequence, pair of query heads 2 hp,
// 2 hp + 1 that share a KV head, half dh of the head dim when hd = 512).  A
// persistent CTA pair (cta_group::2) works through its list of items, each as
// one M = 256 tile; CTA `rank` owns head 2 hp + rank.  Per 128-key block:
//   S[g & 1] = Q K^T   M 256, N 128, K 16: A = this CTA's resident Q,
//                      B = 64 keys from each CTA (K-major, 64 dims per stage);
//   P = softmax rows, FP16, written over the first 64 columns of S[g & 1];
//   O += P V           M 256, N dn = hd / dsplit: A = P from TMEM, B = dn / 2
//                      value dims from each CTA (MN-major, 32 keys per stage);
// g counts key blocks over the pair's whole list, so the barrier phases and
// the two S buffers run on across items and item i + 1's Q and K loads and
// first S products overlap item i's softmax tail and epilogue.
// Warps: 0 loads Q and K, 2 loads V, 1 issues the MMAs (leader CTA) in
// dependency order (S(g) once PV(g - 2) has read the TMEM it overwrites and
// the item's Q is in; PV(g) once both CTAs wrote P(g) and, for an item's
// first block, the previous epilogue has read O; S first when both are
// ready), 4..7 run the softmax (one query row per thread) and hand each
// item's row sums through shared memory to 8..11, which run the epilogue
// (O / l from TMEM, FP16 or FP32 stores) while 4..7 start the next item.
// TMEM columns (per CTA): S0 [0, 128), S1 [128, 256), O [256, 256 + dn).
// The host assigns items to pairs longest first, each to the least loaded
// pair, with one pair per cluster slot the GPU can hold at once.
// Every wait is bounded (common.cuh).

#include <algorithm>
#include <vector>

#include "attention_f16.cuh"
#include "common.cuh"

namespace svl {

namespace {

constexpr int BQ = 128;          // query rows per CTA
constexpr int BKV = 128;         // keys per block
constexpr int DC = 64;           // FP16 elements per 128-byte swizzle row
constexpr int KEYS = BKV / 2;    // keys per CTA per block (B rows of S)
constexpr int VK = 32;           // keys per V stage
constexpr int STAGE = 8192;      // bytes per ring stage
// Warps: 0 Q/K loads, 1 MMA issue (and TMEM), 2 V loads, 3 idle (warpgroup
// 0); 4..7 softmax (warpgroup 1); 8..11 epilogue (warpgroup 2).
constexpr int kThreads = 384;
// Registers per thread after setmaxnreg: the loaders' warpgroup gives up
// registers, the softmax warpgroup (a 128-column row of S in registers)
// takes them; the epilogue warpgroup keeps the launch count.  The sum must
// fit the launch's pool (kThreads x launch count): checked on the host
// against the compiled count before the first launch.
constexpr int kRegsLoad = 64, kRegsSoftmax = 232;
constexpr int kLsumBytes = 2 * 128 * 4;  // row sums handed from softmax to epilogue, per item parity
constexpr int kSmemLimit = 232448;
constexpr int kBarrierBytes = 512;
constexpr int kStagingBytes = 4 * 2 * 4096;  // epilogue: 4 warps x 2 chunk buffers
constexpr float kRescale = 8.0f;
constexpr float kLog2e = 1.4426950408889634f;

// Shared-memory plan for a head dim: resident Q, epilogue staging, then the
// K and V rings.
struct Plan {
  int q_bytes, k_stages, v_stages, smem;
};

__host__ __device__ constexpr Plan plan_for(int hd) {
  const int q_bytes = BQ * hd * 2;
  const int stages = (kSmemLimit - 1024 - kBarrierBytes - kLsumBytes - kStagingBytes - q_bytes) / STAGE;
  return Plan{q_bytes, stages / 2, stages - stages / 2,
              1024 + q_bytes + kStagingBytes + stages * STAGE + kLsumBytes + kBarrierBytes};
}
static_assert(plan_for(512).k_stages >= 4 && plan_for(512).smem <= kSmemLimit, "shared memory");
static_assert(2 * (plan_for(128).k_stages + plan_for(128).v_stages) * 8 + 14 * 8 + 4 <= kBarrierBytes, "barriers");

struct Item {
  uint32_t seq_start, len, q0, hp_dh;  // hp_dh = head pair | (dim half << 16)
};

struct Span {
  int kb_lo, nblk;
};

__host__ __device__ inline Span span_of(uint32_t len, uint32_t q0, int window) {
  int lo = 0, hi = ((int)len - 1) / BKV;
  if (window >= 0) {
    const int a = (int)q0 - window, b = (int)q0 + BQ - 1 + window;
    lo = a > 0 ? a / BKV : 0;
    hi = (b < (int)len - 1 ? b : (int)len - 1) / BKV;
  }
  return Span{lo, hi - lo + 1};
}

struct Ring {
  uint8_t* base;
  uint64_t* full;
  uint64_t* empty;
  int n;
  int stage = 0;
  uint32_t phase = 0;
  SVL_DEV uint8_t* at() const { return base + stage * STAGE; }
  SVL_DEV void next() {
    if (++stage == n) {
      stage = 0;
      phase ^= 1;
    }
  }
};

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    attention_f16_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                         const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_o,
                         const uint32_t* __restrict__ offsets, const Item* __restrict__ items, AttnF16Params p) {
  extern __shared__ uint8_t smem_raw[];
  pdl_trigger();
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int hd = p.hd;
  const Plan plan = plan_for(hd);
  const int dsplit = hd > 256 ? 2 : 1;
  const int dn = hd / dsplit;  // O dims of this pair
  const int dv = dn / 2;       // V dims loaded by each CTA
  uint8_t* qbuf = smem;        // hd / 64 chunks of 128 rows x 128 B (K-major SW128)
  uint8_t* staging = smem + plan.q_bytes;
  uint8_t* kring = staging + kStagingBytes;
  uint8_t* vring = kring + plan.k_stages * STAGE;
  float* lsum = (float*)(vring + plan.v_stages * STAGE);  // [2][BQ]
  uint64_t* bars = (uint64_t*)((uint8_t*)lsum + kLsumBytes);
  uint64_t* k_full = bars;
  uint64_t* k_empty = k_full + plan.k_stages;
  uint64_t* v_full = k_empty + plan.k_stages;
  uint64_t* v_empty = v_full + plan.v_stages;
  uint64_t* q_full = v_empty + plan.v_stages;
  uint64_t* q_empty = q_full + 1;
  uint64_t* o_empty = q_empty + 1;  // leader only
  uint64_t* s_full = o_empty + 1;   // [2]
  uint64_t* p_full = s_full + 2;    // [2], leader only
  uint64_t* pv_done = p_full + 2;   // [2]
  uint64_t* l_full = pv_done + 2;   // [2] row sums of an item written (softmax -> epilogue)
  uint64_t* l_empty = l_full + 2;   // [2] and read
  uint32_t* tmem_slot = (uint32_t*)(l_empty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank() & 1u;
  const bool leader = rank == 0;
  const int pair = (int)(blockIdx.x >> 1);
  const int it_lo = (int)offsets[pair], it_hi = (int)offsets[pair + 1];
  auto head_of = [&](const Item& it) { return 2 * (int)(it.hp_dh & 0xFFFFu) + (int)rank; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < plan.k_stages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < plan.v_stages; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    mbar_init(o_empty, 8);  // 4 epilogue warps x 2 CTAs
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], 8);  // 4 softmax warps x 2 CTAs
      mbar_init(&pv_done[b], 1);
      mbar_init(&l_full[b], 128);   // softmax threads of this CTA
      mbar_init(&l_empty[b], 128);  // epilogue threads of this CTA
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
  // The work list (offsets, items) was copied in before the previous kernel
  // ran; q/k/v and the outputs are touched only after this wait.
  pdl_wait();

  if (warp < 4) {
  setmaxnreg_dec<kRegsLoad>();
  if (warp == 0 || warp == 2) {
    if (lane == 0) {
      // producers of both CTAs; every load completes on the leader's barrier
      const bool is_k = warp == 0;
      Ring ring{is_k ? kring : vring, is_k ? k_full : v_full, is_k ? k_empty : v_empty,
                is_k ? plan.k_stages : plan.v_stages};
      if (is_k) {
        tma_prefetch_desc(&map_q);
        tma_prefetch_desc(&map_k);
      } else {
        tma_prefetch_desc(&map_v);
      }
      const int per_block = is_k ? hd / DC : BKV / VK;
      const uint32_t bytes = is_k ? 2 * KEYS * 128 : 2 * VK * dv * 2;
      bool ok = true;
      for (int i = it_lo; ok && i < it_hi; ++i) {
        const Item it = items[i];
        const Span sp = span_of(it.len, it.q0, p.window);
        const int h = head_of(it);
        const int kvh = h / (p.nh / p.kvh);
        const int row0 = (int)it.seq_start;
        if (is_k) {
          // Q of this item once every S product of the previous one is done
          if (i > it_lo && !mbar_wait(q_empty, (uint32_t)(i - it_lo - 1) & 1u, p.err)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(q_full, 2 * BQ * hd * 2);
          const uint32_t qbar = map_to_rank(smem_u32(q_full), 0);
          for (int c = 0; c < hd / DC; ++c)
            tma_load_2d_pair(qbuf + c * (BQ * 128), &map_q, qbar, h * hd + c * DC, row0 + (int)it.q0);
        }
        const int k_col = (p.nh + kvh) * hd;
        const int v_col = (p.nh + p.kvh + kvh) * hd + (int)(it.hp_dh >> 16) * dn + (int)rank * dv;
        for (int j = 0; ok && j < sp.nblk; ++j) {
          const int krow = row0 + (sp.kb_lo + j) * BKV;
          for (int s = 0; s < per_block; ++s) {
            if (!mbar_wait(&ring.empty[ring.stage], ring.phase ^ 1, p.err)) {
              ok = false;
              break;
            }
            uint8_t* dst = ring.at();
            if (leader) mbar_arrive_expect_tx(&ring.full[ring.stage], bytes);
            const uint32_t bar = map_to_rank(smem_u32(&ring.full[ring.stage]), 0);
            if (is_k) {
              tma_load_2d_pair(dst, &map_k, bar, k_col + s * DC, krow + (int)rank * KEYS);
            } else {
              for (int c = 0; c < dv / DC; ++c)
                tma_load_2d_pair(dst + c * (VK * 128), &map_v, bar, v_col + c * DC, krow + s * VK);
            }
            ring.next();
          }
        }
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      const uint32_t idesc_s = idesc_f16(2 * BQ, BKV, 0);
      const uint32_t idesc_o = idesc_f16(2 * BQ, (uint32_t)dn, 1);
      Ring kr{kring, k_full, k_empty, plan.k_stages};
      Ring vr{vring, v_full, v_empty, plan.v_stages};
      const uint32_t qa = smem_u32(qbuf);
      bool ok = true;
      auto issue_s = [&](int g) {
        const uint32_t d = tmem + (uint32_t)((g & 1) * BKV);
        for (int c = 0; ok && c < hd / DC; ++c) {
          if (!mbar_wait(&kr.full[kr.stage], kr.phase, p.err)) {
            ok = false;
            return;
          }
          tc_fence_after();
          const uint32_t kb = smem_u32(kr.at());
#pragma unroll
          for (int k = 0; k < DC / 16; ++k)
            mma_f16_pair(d, sdesc(qa + c * (BQ * 128) + k * 32, 16, 1024, kLayoutSW128),
                         sdesc(kb + k * 32, 16, 1024, kLayoutSW128), idesc_s, (c | k) != 0);
          mma_commit_pair(&kr.empty[kr.stage], 0x3);
          kr.next();
        }
        mma_commit_pair(&s_full[g & 1], 0x3);
      };
      auto issue_pv = [&](int g, int j) {
        const uint32_t d = tmem + 256;
        const uint32_t pa = tmem + (uint32_t)((g & 1) * BKV);  // P: 64 packed columns
        for (int s = 0; ok && s < BKV / VK; ++s) {
          if (!mbar_wait(&vr.full[vr.stage], vr.phase, p.err)) {
            ok = false;
            return;
          }
          tc_fence_after();
          const uint32_t v = smem_u32(vr.at());
#pragma unroll
          for (int k = 0; k < VK / 16; ++k)
            // B = V, MN-major SWIZZLE_128B: 8-key atoms of 128-byte rows (SBO
            // 1024), 64-dim chunks VK x 128 bytes apart (LBO), 16 keys per MMA
            mma_f16_pair_ts(d, pa + (uint32_t)((s * VK + k * 16) / 2), sdesc(v + k * 2048, VK * 128, 1024, kLayoutSW128),
                            idesc_o, (j | s | k) != 0);
          mma_commit_pair(&vr.empty[vr.stage], 0x3);
          vr.next();
        }
        mma_commit_pair(&pv_done[g & 1], 0x3);
      };
      // S cursor (item si, block sj, global block sg) and PV cursor (pi, pj, pg)
      int si = it_lo, sj = 0, sg = 0, pi = it_lo, pj = 0, pg = 0;
      int s_nblk = si < it_hi ? span_of(items[si].len, items[si].q0, p.window).nblk : 0;
      int p_nblk = s_nblk;
      bool q_in = false;
      uint64_t idle_since = 0;
      while (ok && pi < it_hi) {
        bool did = false;
        if (si < it_hi && sg < pg + 2 && (sg < 2 || mbar_test(&pv_done[sg & 1], (uint32_t)((sg - 2) >> 1) & 1u))) {
          if (sj == 0 && !q_in) q_in = mbar_test(q_full, (uint32_t)(si - it_lo) & 1u);
          if (sj > 0 || q_in) {
            tc_fence_after();
            issue_s(sg);
            ++sg;
            if (++sj == s_nblk) {
              mma_commit_pair(q_empty, 0x3);  // Q may be replaced once these products are done
              sj = 0;
              q_in = false;
              if (++si < it_hi) s_nblk = span_of(items[si].len, items[si].q0, p.window).nblk;
            }
            did = true;
          }
        }
        if (!did && pg < sg && mbar_test_cluster(&p_full[pg & 1], (uint32_t)(pg >> 1) & 1u) &&
            (pj > 0 || pi == it_lo || mbar_test_cluster(o_empty, (uint32_t)(pi - it_lo - 1) & 1u))) {
          tc_fence_after();
          issue_pv(pg, pj);
          ++pg;
          if (++pj == p_nblk) {
            pj = 0;
            if (++pi < it_hi) p_nblk = span_of(items[pi].len, items[pi].q0, p.window).nblk;
          }
          did = true;
        }
        if (did) {
          idle_since = 0;
        } else if (idle_since == 0) {
          idle_since = global_ns();
        } else if (global_ns() - idle_since > kWaitDeadlineNs) {
          atomicOr(p.err, SVL_DEVERR_TIMEOUT);
          ok = false;
        }
      }
    }
  }
  } else if (warp < 8) {
    setmaxnreg_inc<kRegsSoftmax>();
    // softmax warps of both CTAs: thread owns query row r of its head
    const int lg = warp & 3;
    const int r = lg * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(lg * 32) << 16;
    const uint32_t p_full_leader0 = map_to_rank(smem_u32(&p_full[0]), 0);
    const uint32_t p_full_leader1 = map_to_rank(smem_u32(&p_full[1]), 0);
    int g = 0;  // global key block
    bool bad = false, ok = true;
    for (int i = it_lo; ok && i < it_hi; ++i) {
      const Item it = items[i];
      const Span sp = span_of(it.len, it.q0, p.window);
      const int L = (int)it.len, q0 = (int)it.q0;
      const int qi = q0 + r;
      const bool q_valid = qi < L;
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
      for (int j = 0; j < sp.nblk; ++j, ++g) {
        const int b = g & 1;
        const bool got = mbar_wait(&s_full[b], (uint32_t)(g >> 1) & 1u, p.err);
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
        const int k0 = (sp.kb_lo + j) * BKV;
        if (k0 < key_lo || k0 + BKV - 1 > key_hi) {
#pragma unroll
          for (int c = 0; c < BKV; ++c)
            if (k0 + c < key_lo || k0 + c > key_hi) sr[c] = __float_as_uint(-INFINITY);
        }
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
          rescale = m != -INFINITY;  // only from the item's second block on
        }
        const float factor = rescale ? expf(m - m_new) : 1.0f;
        if (__any_sync(0xffffffffu, rescale)) {
          // O may be rescaled only once PV(g - 1) has finished accumulating
          const bool pv = mbar_wait(&pv_done[(g - 1) & 1], (uint32_t)((g - 1) >> 1) & 1u, p.err);
          __syncwarp();
          if (!__all_sync(0xffffffffu, pv)) {
            ok = false;
            break;
          }
          tc_fence_after();
          float o[32];
          for (int c = 0; c < dn / 32; ++c) {
            const uint32_t addr = tmem + lane_addr + 256 + c * 32;
            tmem_ld32(addr, o);
#pragma unroll
            for (int u = 0; u < 32; ++u) o[u] *= factor;
            tmem_st32(addr, o);
          }
        }
        // P = 2^(s log2(e) - m log2(e)) in FP16 (nearest even), two keys per
        // TMEM column, written over the first half of S's columns
        const float ml = m_new == -INFINITY ? 0.0f : m_new * kLog2e;
        float rs[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int q = 0; q < BKV / 32; ++q) {
          uint32_t pk[16];
#pragma unroll
          for (int u = 0; u < 16; ++u) {
            const float e0 = ex2_approx(fmaf(sv(q * 32 + 2 * u), kLog2e, -ml));
            const float e1 = ex2_approx(fmaf(sv(q * 32 + 2 * u + 1), kLog2e, -ml));
            pk[u] = pack_half2(e0, e1);
            rs[u & 3] += e0 + e1;
          }
          tmem_st16(tmem + lane_addr + b * BKV + q * 16, pk);
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
      if (!ok) break;
      // hand the row sum to the epilogue warps (slot = item parity)
      const int slot = (i - it_lo) & 1;
      if (i - it_lo >= 2 && !mbar_wait(&l_empty[slot], (uint32_t)((i - it_lo - 2) >> 1) & 1u, p.err)) break;
      lsum[slot * BQ + r] = l;
      mbar_arrive(&l_full[slot]);
    }
    if (bad) atomicOr(p.err, SVL_DEVERR_NONFINITE);
  } else {
    // epilogue warps of both CTAs: O / l of row r of each item once its last
    // P V has finished, while the softmax warps run the next item
    const int lg = warp & 3;
    const int r = lg * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(lg * 32) << 16;
    const uint32_t o_empty_leader = map_to_rank(smem_u32(o_empty), 0);
    uint8_t* stage_base = staging + (warp - 8) * 8192;
    int g = 0;         // global key block
    uint32_t nst = 0;  // TMA stores issued by this warp (staging buffer = nst & 1)
    bool bad = false, ok = true;
    for (int i = it_lo; ok && i < it_hi; ++i) {
      const Item it = items[i];
      const Span sp = span_of(it.len, it.q0, p.window);
      const int L = (int)it.len, q0 = (int)it.q0, row0 = (int)it.seq_start;
      const int h = head_of(it);
      const int qi = q0 + r;
      const bool q_valid = qi < L;
      g += sp.nblk;
      const int slot = (i - it_lo) & 1;
      const bool got_l = mbar_wait(&l_full[slot], (uint32_t)((i - it_lo) >> 1) & 1u, p.err);
      __syncwarp();
      if (!__all_sync(0xffffffffu, got_l)) break;
      const float l = lsum[slot * BQ + r];
      mbar_arrive(&l_empty[slot]);
      // O / l once the item's last P V has finished
      const int gl = g - 1;
      const bool fin = mbar_wait(&pv_done[gl & 1], (uint32_t)(gl >> 1) & 1u, p.err);
      __syncwarp();
      if (!__all_sync(0xffffffffu, fin)) {
        ok = false;
        break;
      }
      tc_fence_after();
      bad |= q_valid && !isfinite(l);
      const float inv = 1.0f / l;
      const bool whole = q0 + lg * 32 + 32 <= L;  // the warp's 32 rows are all in the sequence
      const int ocol = h * hd + (int)(it.hp_dh >> 16) * dn;
      float* out = p.out16 ? nullptr : p.out + (size_t)(row0 + qi) * p.ld_out + ocol;
      // O in four-chunk (128-column) groups: four TMEM loads per wait.  No
      // per-element range checks: O is a convex combination of the (finite,
      // FP16-range) v rows, so a finite positive l is all that is checked.
      uint32_t oraw[128];
      for (int c4 = 0; c4 < dn / 32; c4 += 4) {
#pragma unroll
        for (int q = 0; q < 4; ++q) tmem_ld32_nowait(tmem + lane_addr + 256 + (c4 + q) * 32, oraw + q * 32);
        tmem_ld_wait();
#pragma unroll
        for (int q = 0; q < 4; ++q) tmem_regs_after_wait(oraw + q * 32);
        if (c4 + 4 == dn / 32) {
          // O is read: the next item's first P V may overwrite it
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if (leader)
              mbar_arrive(o_empty);
            else
              mbar_arrive_cluster(o_empty_leader);
          }
        }
        if (p.out16) {
          // FP16 rows of 64 bytes (SWIZZLE_64B: 16-byte unit ^= (row / 2) % 4),
          // two chunks per staging buffer, proxy fence and bulk group
#pragma unroll
          for (int q = 0; q < 4; q += 2) {
            const int c = c4 + q;
            uint32_t pk[32];
#pragma unroll
            for (int u = 0; u < 32; ++u)
              pk[u] = pack_half2(__uint_as_float(oraw[q * 32 + 2 * u]) * inv, __uint_as_float(oraw[q * 32 + 2 * u + 1]) * inv);
            if (whole) {
              // double-buffered staging: the group two back has read this buffer
              if (lane == 0 && nst >= 2) tma_store_wait_read1();
              __syncwarp();
              uint8_t* st = stage_base + (nst & 1) * 4096;
#pragma unroll
              for (int hh = 0; hh < 2; ++hh)
#pragma unroll
                for (int k = 0; k < 4; ++k)
                  *(uint4*)(st + hh * 2048 + lane * 64 + ((k ^ ((lane >> 1) & 3)) * 16)) =
                      make_uint4(pk[hh * 16 + 4 * k], pk[hh * 16 + 4 * k + 1], pk[hh * 16 + 4 * k + 2],
                                 pk[hh * 16 + 4 * k + 3]);
              fence_async_smem();
              __syncwarp();
              if (lane == 0) {
                tma_store_2d(&map_o, st, ocol + c * 32, row0 + q0 + lg * 32);
                tma_store_2d(&map_o, st + 2048, ocol + (c + 1) * 32, row0 + q0 + lg * 32);
                tma_store_commit();
              }
              ++nst;
            } else if (q_valid) {
              uint4* o16 = (uint4*)(p.out16 + (size_t)(row0 + qi) * p.ld_out + ocol + c * 32);
#pragma unroll
              for (int k = 0; k < 8; ++k) o16[k] = make_uint4(pk[4 * k], pk[4 * k + 1], pk[4 * k + 2], pk[4 * k + 3]);
            }
          }
          continue;
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int c = c4 + q;
          float o[32];
#pragma unroll
          for (int u = 0; u < 32; ++u) {
            const float v = __uint_as_float(oraw[q * 32 + u]) * inv;
            o[u] = p.round_out ? round_tf32(v) : v;
          }
          if (whole) {
            // double-buffered staging: the store two chunks back has read this buffer
            if (lane == 0 && nst >= 2) tma_store_wait_read1();
            __syncwarp();
            float* st = (float*)(stage_base + (nst & 1) * 4096);
            uint8_t* row = (uint8_t*)st + lane * 128;
#pragma unroll
            for (int u = 0; u < 8; ++u)
              *(float4*)(row + ((u ^ (lane & 7)) * 16)) = make_float4(o[4 * u], o[4 * u + 1], o[4 * u + 2], o[4 * u + 3]);
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&map_o, st, ocol + c * 32, row0 + q0 + lg * 32);
              tma_store_commit();
            }
            ++nst;
          } else if (q_valid) {
#pragma unroll
            for (int u = 0; u < 32; u += 4)
              *(float4*)(out + c * 32 + u) = make_float4(o[u], o[u + 1], o[u + 2], o[u + 3]);
          }
        }
      }
    }
    if (lane == 0) tma_store_wait_read();  // the staging must outlive the stores' reads
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

__global__ void f32_to_f16_kernel(const float* __restrict__ in, uint16_t* __restrict__ out, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; 2 * i < n; i += (size_t)gridDim.x * blockDim.x) {
    const float a = in[2 * i], b = 2 * i + 1 < n ? in[2 * i + 1] : 0.0f;
    const uint32_t h = pack_half2(a, b);
    out[2 * i] = (uint16_t)(h & 0xFFFFu);
    if (2 * i + 1 < n) out[2 * i + 1] = (uint16_t)(h >> 16);
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

// Row-major 2-D map with 128-byte swizzled boxes of 128 bytes x box_rows.
bool make_map(CUtensorMap* map, const void* base, CUtensorMapDataType type, int elem_bytes, uint64_t rows,
              uint64_t cols, uint64_t ld, uint32_t box_rows) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * (uint64_t)elem_bytes};
  cuuint32_t box[2] = {(cuuint32_t)(128 / elem_bytes), box_rows};
  cuuint32_t elem[2] = {1, 1};
  return enc(map, type, 2, (void*)base, dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// FP16 output map: 32 x 32 boxes of 64-byte rows, SWIZZLE_64B.
bool make_map_f16_64(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t elem[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void*)base, dims, strides, box, elem,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Sets the kernel's shared-memory limit and returns how many CTA pairs of a
// head dim the current device holds at once (cached per device and plan).
int resident_pairs(int hd) {
  static std::atomic<int> cache[64][3] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return 0;
  const int slot = hd == 128 ? 0 : (hd == 256 ? 1 : 2);
  // devices past 63 repeat the (idempotent) set-up on every call
  std::atomic<int>* cached = dev < 64 ? &cache[dev][slot] : nullptr;
  if (cached) {
    const int have = cached->load(std::memory_order_acquire);
    if (have) return have;
  }
  // setmaxnreg moves registers between warpgroups within the launch's pool
  // (kThreads x the compiled count): an increase the pool cannot cover would
  // wait forever, so the split is checked against the compiled count here
  cudaFuncAttributes fa{};
  if (cudaFuncGetAttributes(&fa, attention_f16_kernel) != cudaSuccess || fa.numRegs < kRegsLoad ||
      fa.numRegs > kRegsSoftmax || (kRegsLoad + kRegsSoftmax + fa.numRegs) > 3 * fa.numRegs)
    return 0;
  if (cudaFuncSetAttribute(attention_f16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit) !=
      cudaSuccess)
    return 0;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(2 * 64, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = (size_t)plan_for(hd).smem;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, (void*)attention_f16_kernel, &cfg) != cudaSuccess || clusters <= 0) {
    cudaGetLastError();
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    clusters = sms / 2;  // one CTA per SM
  }
  const int n = clusters > 0 ? clusters : 1;
  if (cached) cached->store(n, std::memory_order_release);
  return n;
}

}  // namespace

bool attention_f16_supported(int hd, int nh, int kvh) {
  return (hd == 128 || hd == 256 || hd == 512) && kvh > 0 && nh % kvh == 0 && (nh / kvh) % 2 == 0;
}

int attention_f16_schedule(const uint64_t* cu_host, int batch, int nh, int hd, int window, std::vector<uint32_t>* out) {
  out->clear();
  if ((hd != 128 && hd != 256 && hd != 512) || nh < 2) return 0;
  const int dsplit = hd > 256 ? 2 : 1;
  // Built on every forward before its first launch (the host time of a
  // synchronous call), so with flat per-thread buffers and a counting sort:
  // items in sequence order, then stably by cost (key blocks + 1, at most
  // 65 for 8,192 tokens) in descending order, each assigned longest first to
  // the least loaded pair.
  thread_local std::vector<Item> items, sorted;
  thread_local std::vector<int> cost, sorted_cost, owner, count, at_pair;
  items.clear();
  for (int b = 0; b < batch; ++b) {
    const uint32_t s = (uint32_t)cu_host[b], n = (uint32_t)(cu_host[b + 1] - cu_host[b]);
    for (uint32_t q0 = 0; q0 < n; q0 += BQ)
      for (int hp = 0; hp < nh / 2; ++hp)
        for (int dh = 0; dh < dsplit; ++dh) items.push_back({s, n, q0, (uint32_t)hp | ((uint32_t)dh << 16)});
  }
  if (items.empty()) return 0;
  int pairs = resident_pairs(hd);
  if (pairs <= 0) return -1;
  const size_t n_items = items.size();
  if ((size_t)pairs > n_items) pairs = (int)n_items;
  cost.resize(n_items);
  int max_cost = 0;
  for (size_t i = 0; i < n_items; ++i) {
    cost[i] = span_of(items[i].len, items[i].q0, window).nblk + 1;
    max_cost = cost[i] > max_cost ? cost[i] : max_cost;
  }
  // counting sort, descending cost, stable
  count.assign((size_t)max_cost + 2, 0);
  for (size_t i = 0; i < n_items; ++i) ++count[(size_t)(max_cost - cost[i])];
  for (int c = 0, sum = 0; c <= max_cost + 1; ++c) {
    const int k = count[(size_t)c];
    count[(size_t)c] = sum;
    sum += k;
  }
  sorted.resize(n_items);
  owner.resize(n_items);
  sorted_cost.resize(n_items);
  for (size_t i = 0; i < n_items; ++i) {
    const int slot = count[(size_t)(max_cost - cost[i])]++;
    sorted[(size_t)slot] = items[i];
    sorted_cost[(size_t)slot] = cost[i];
  }
  // longest first, each to the least loaded pair
  std::vector<std::pair<long, int>> heap;
  heap.reserve((size_t)pairs);
  for (int i = 0; i < pairs; ++i) heap.push_back({0L, i});
  auto cmp = [](const std::pair<long, int>& a, const std::pair<long, int>& b) {
    return a.first != b.first ? a.first > b.first : a.second > b.second;
  };
  std::make_heap(heap.begin(), heap.end(), cmp);
  at_pair.assign((size_t)pairs + 1, 0);
  for (size_t i = 0; i < n_items; ++i) {
    std::pop_heap(heap.begin(), heap.end(), cmp);
    owner[i] = heap.back().second;
    ++at_pair[(size_t)owner[i] + 1];
    heap.back().first += sorted_cost[i];
    std::push_heap(heap.begin(), heap.end(), cmp);
  }
  for (int i = 0; i < pairs; ++i) at_pair[(size_t)i + 1] += at_pair[(size_t)i];
  // [pairs + 1 offsets, padded to 4 words][items, each pair's in assignment order]
  const size_t head = ((size_t)pairs + 1 + 3) / 4 * 4;
  out->assign(head + n_items * 4, 0u);
  for (int i = 0; i <= pairs; ++i) (*out)[(size_t)i] = (uint32_t)at_pair[(size_t)i];
  for (size_t i = 0; i < n_items; ++i) {
    uint32_t* w = out->data() + head + (size_t)at_pair[(size_t)owner[i]]++ * 4;
    const Item& it = sorted[i];
    w[0] = it.seq_start;
    w[1] = it.len;
    w[2] = it.q0;
    w[3] = it.hp_dh;
  }
  return pairs;
}

cudaError_t launch_attention_f16(const AttnF16Params& p, const uint32_t* d_schedule, int pairs, cudaStream_t st) {
  if (pairs == 0) return cudaSuccess;
  if (pairs < 0 || !attention_f16_supported(p.hd, p.nh, p.kvh) || p.ld % 8 != 0 || p.ld_out % 4 != 0 ||
      ((uintptr_t)p.qkv & 15) != 0 || ((uintptr_t)(p.out16 ? (void*)p.out16 : (void*)p.out) & 15) != 0 ||
      (p.out16 && p.ld_out % 8 != 0) || ((uintptr_t)d_schedule & 15) != 0)
    return cudaErrorInvalidValue;
  CUtensorMap mq, mk, mv, mo;
  const uint64_t width = (uint64_t)(p.nh + 2 * p.kvh) * p.hd;
  if (!make_map(&mq, p.qkv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)p.T, width, (uint64_t)p.ld, BQ) ||
      !make_map(&mk, p.qkv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)p.T, width, (uint64_t)p.ld, KEYS) ||
      !make_map(&mv, p.qkv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)p.T, width, (uint64_t)p.ld, VK) ||
      !(p.out16 ? make_map_f16_64(&mo, p.out16, (uint64_t)p.T, (uint64_t)p.nh * p.hd, (uint64_t)p.ld_out)
                : make_map(&mo, p.out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)p.T, (uint64_t)p.nh * p.hd,
                           (uint64_t)p.ld_out, 32)))
    return cudaErrorInvalidValue;
  if (resident_pairs(p.hd) <= 0) return cudaErrorInvalidValue;  // also sets the shared-memory limit
  const size_t head = ((size_t)pairs + 1 + 3) / 4 * 4;
  launch_pdl(attention_f16_kernel, dim3((unsigned)(2 * pairs)), dim3(kThreads), (size_t)plan_for(p.hd).smem, st, mq, mk,
             mv, mo, d_schedule, (const Item*)(d_schedule + head), p);
  return cudaGetLastError();
}

void launch_f32_to_f16(const float* in, uint16_t* out, size_t n, cudaStream_t st) {
  f32_to_f16_kernel<<<1184, 256, 0, st>>>(in, out, n);
}

}  // namespace svl
