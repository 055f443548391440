// common.cuh -- shared device helpers for the sm_100a kernels of libsvl_gpu.
//
// Hand-written PTX wrappers for mbarriers, TMA (cp.async.bulk.tensor, never
// with .multicast::cluster: every kernel here also runs in multi-GPU jobs),
// and the tcgen05 tensor-core / TMEM instructions.  Every spin-wait is
// bounded by a wall-clock deadline; on expiry the kernel records
// SVL_DEVERR_TIMEOUT in the device error word and unwinds instead of hanging.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdlib>

#include "../../include/svl_gpu.h"

// Bits of the per-handle device error word (read back by the host).
enum : uint32_t {
  SVL_DEVERR_NONFINITE = 1u << 0,   // a non-finite activation (-> SVL_INTERNAL)
  SVL_DEVERR_BAD_TOKEN = 1u << 1,   // token id >= vocab (-> SVL_CORRUPT)
  SVL_DEVERR_TIMEOUT = 1u << 2,     // a bounded wait expired (-> SVL_INTERNAL)
  SVL_DEVERR_BAD_QUERY = 1u << 3,   // zero / non-finite query (-> SVL_USAGE)
  SVL_DEVERR_BAD_ROW = 1u << 4,     // zero / non-finite stored row (-> SVL_USAGE/INTERNAL)
  SVL_DEVERR_OVERFLOW = 1u << 5,    // a candidate list overflowed (-> SVL_INTERNAL)
  SVL_DEVERR_PEER = 1u << 6,        // another rank's shard search failed (-> SVL_INTERNAL)
};

#define SVL_DEV __device__ __forceinline__

// Wait deadline for any spin loop: 4 s of global time.
constexpr uint64_t kWaitDeadlineNs = 4000000000ull;

SVL_DEV uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

SVL_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// ------------------------------------------------------------- mbarrier --
SVL_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

SVL_DEV void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

SVL_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

SVL_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

SVL_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase.  Returns false (and flags the error
// word) once the deadline passes; callers then unwind.
SVL_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0 && global_ns() - start > kWaitDeadlineNs) {
      if (err) atomicOr(err, SVL_DEVERR_TIMEOUT);
      return false;
    }
  }
}

// ------------------------------------------------------------------ TMA --
SVL_DEV void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// 2-D tiled load, coordinates (x = innermost element index, y = row).  x must
// be a multiple of 4 for 32-bit elements (16-byte rule); callers only pass
// multiples of the 32-element box width.
SVL_DEV void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// Prefetch of a 2-D tile into L2 (no shared memory, no completion to wait for).
SVL_DEV void tma_prefetch_l2_2d(const CUtensorMap* map, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(map), "r"(x), "r"(y)
               : "memory");
}

// 3-D tiled load (x innermost).
SVL_DEV void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int32_t x, int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// Two FP32 values rounded to FP16 (nearest even) and packed: `lo` in bits
// 0..15, `hi` in bits 16..31 (element order of a 16-bit operand in memory).
SVL_DEV uint32_t pack_half2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// The two FP16 halves of a packed word as floats (low half first), exact.
SVL_DEV float2 unpack_half2(uint32_t w) {
  float lo, hi;
  asm("{\n.reg .b16 l, h;\nmov.b32 {l, h}, %2;\ncvt.f32.f16 %0, l;\ncvt.f32.f16 %1, h;\n}" : "=f"(lo), "=f"(hi) : "r"(w));
  return make_float2(lo, hi);
}

// Power-of-two operand scale for a row whose largest magnitude is `maxabs`:
// scale = 2^-e with maxabs * scale in [2^14, 2^15), so the row stored in FP16
// keeps every value in the normal range (11-bit significand, the TF32
// precision) down to 2^-29 of its maximum; inv = 2^e undoes it exactly.
// Zero or non-finite maxima get scale 1 (non-finite values are reported by
// the producer's own check).
SVL_DEV void pow2_row_scale(float maxabs, float& scale, float& inv) {
  int e = 0;
  if (maxabs > 0.0f && maxabs <= 3.0e38f) {
    const int E = (int)((__float_as_uint(maxabs) >> 23) & 0xFFu);  // biased exponent (0 for subnormals)
    e = (E > 0 ? E : 1) - 141;
    e = e < -100 ? -100 : (e > 100 ? 100 : e);
  }
  scale = __uint_as_float((uint32_t)(127 - e) << 23);
  inv = __uint_as_float((uint32_t)(127 + e) << 23);
}

// fence making generic-proxy shared-memory writes visible to the async proxy
// (TMA stores, tensor-core operand reads)
SVL_DEV void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 2-D tiled store from shared memory (bulk-group completion).  Coordinates
// are never negative here; rows / columns past the tensor are clipped.
SVL_DEV void tma_store_2d(const CUtensorMap* map, const void* src, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(map), "r"(x), "r"(y),
               "r"(smem_u32(src))
               : "memory");
}

// Closes the bulk group of the stores issued since the last commit.
SVL_DEV void tma_store_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

SVL_DEV void tma_store_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// All but the most recent bulk store group have finished reading shared memory.
SVL_DEV void tma_store_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
SVL_DEV void tma_store_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Writes a warp's 32 x 32 FP32 output chunk (lane = row, v = its 32 columns)
// at global (x, y) through `buf`, a 4 KB, 1024-byte aligned staging buffer the
// warp has acquired: rows of 128 bytes with the 16-byte units XOR-swizzled by
// row % 8 (the SWIZZLE_128B layout of the store's tensor map), so the shared
// writes are bank-conflict free and the global write is one TMA operation,
// committed as one bulk group.
SVL_DEV void store_chunk_tma(const CUtensorMap* map, float* buf, const float* v, int lane, int32_t x, int32_t y) {
  uint8_t* row = (uint8_t*)buf + lane * 128;
#pragma unroll
  for (int u = 0; u < 8; ++u)
    *(float4*)(row + ((u ^ (lane & 7)) * 16)) = make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
  fence_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(map, buf, x, y);
    tma_store_commit();
  }
}

// The same from the FP32 values' bit patterns.
SVL_DEV void store_chunk_tma(const CUtensorMap* map, float* buf, const uint32_t* w, int lane, int32_t x, int32_t y) {
  uint8_t* row = (uint8_t*)buf + lane * 128;
#pragma unroll
  for (int u = 0; u < 8; ++u)
    *(uint4*)(row + ((u ^ (lane & 7)) * 16)) = make_uint4(w[4 * u], w[4 * u + 1], w[4 * u + 2], w[4 * u + 3]);
  fence_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(map, buf, x, y);
    tma_store_commit();
  }
}

// A warp's epilogue staging: `nbufs` (1 or 2) 4 KB buffers used in turn; each
// use ends with exactly one committed bulk-store group, so a buffer may be
// rewritten once all but the last nbufs - 1 groups have read shared memory.
struct Staging {
  float* base;
  int nbufs;
  uint32_t uses = 0;
  SVL_DEV float* acquire(int lane) {
    if (lane == 0) {
      if (nbufs > 1)
        tma_store_wait_read1();
      else
        tma_store_wait_read();
    }
    __syncwarp();
    return base + (nbufs > 1 ? (uses & 1u) * 1024 : 0);
  }
  SVL_DEV void release() { ++uses; }
};

// Stores a warp's 32 x 32 FP16 chunk (lane = row, 16 packed words) through
// its staging: 64-byte rows, 16-byte units XOR-swizzled by (row / 2) % 4 (the
// SWIZZLE_64B layout of an FP16 output map), one committed bulk group.
SVL_DEV void store_row64_f16(const CUtensorMap* map, Staging& sg, const uint32_t* pk, int lane, int32_t x, int32_t y) {
  uint8_t* buf = (uint8_t*)sg.acquire(lane);
#pragma unroll
  for (int k = 0; k < 4; ++k)
    *(uint4*)(buf + lane * 64 + ((k ^ ((lane >> 1) & 3)) * 16)) = make_uint4(pk[4 * k], pk[4 * k + 1], pk[4 * k + 2],
                                                                            pk[4 * k + 3]);
  fence_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(map, buf, x, y);
    tma_store_commit();
  }
  sg.release();
}

// ------------------------------------------------------------- tcgen05 --
// Shared-memory matrix descriptor (tcgen05 "version 1" format):
//   [0,14) start >> 4, [16,30) LBO >> 4, [32,46) SBO >> 4, [46,48) = 1,
//   [49,52) base offset (0: atoms are 1024-byte aligned), [61,64) layout.
enum : uint32_t { kLayoutSW128Base32B = 1, kLayoutSW128 = 2 };

SVL_DEV uint64_t sdesc(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes, uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)(layout & 7u) << 61;
  return d;
}

// Instruction descriptor for kind::tf32 with an FP32 accumulator:
//   [4,6) D format = 1 (F32), [7,10) A = 2 (TF32), [10,13) B = 2 (TF32),
//   [15] A major (0 = K), [16] B major (0 = K, 1 = MN), [17,23) N >> 3,
//   [24,29) M >> 4.
__host__ __device__ constexpr uint32_t idesc_tf32(uint32_t m, uint32_t n, uint32_t b_mn_major) {
  return (1u << 4) | (2u << 7) | (2u << 10) | (b_mn_major << 16) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

// Instruction descriptor for kind::f16 with FP16 A and B and an FP32
// accumulator: [4,6) D format = 1 (F32), [7,10) A = 0 (F16), [10,13) B = 0
// (F16), [16] B major, [17,23) N >> 3, [24,29) M >> 4.
__host__ __device__ constexpr uint32_t idesc_f16(uint32_t m, uint32_t n, uint32_t b_mn_major) {
  return (1u << 4) | (b_mn_major << 16) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

SVL_DEV void tmem_alloc(uint32_t* slot_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot_smem)),
               "r"(ncols)
               : "memory");
}

SVL_DEV void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

SVL_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

SVL_DEV void mma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// kind::f16 (FP16 A and B, K = 16 per instruction), one CTA.
SVL_DEV void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives on `bar` once every previously issued tcgen05.mma of this thread
// has completed (and its smem operands may be overwritten).
SVL_DEV void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// ---------------------------------------------- CTA pairs (cta_group::2) --
SVL_DEV uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

SVL_DEV void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// shared::cluster address of the same shared variable in CTA `rank`.
SVL_DEV uint32_t map_to_rank(uint32_t smem_addr, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_addr), "r"(rank));
  return out;
}

// Arrive on an mbarrier of another CTA of the cluster (address from map_to_rank).
// Default semantics (release at CTA scope): the signals sent this way publish
// completed tensor-memory work (after tcgen05.wait + fence::before_thread_sync)
// or the end of reads, never generic-memory data, and a cluster-scope release
// costs ~1,400 cycles under load.
SVL_DEV void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// 2-D tiled load into this CTA's shared memory whose completion is counted on
// the pair leader's mbarrier (`bar_cluster`, a shared::cluster address).
SVL_DEV void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}

SVL_DEV void tmem_alloc_pair(uint32_t* slot_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot_smem)),
               "r"(ncols)
               : "memory");
}

SVL_DEV void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

SVL_DEV void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// M = 256 MMA over a CTA pair: A rows 0..127 and B columns 0..N/2-1 come from
// the leader's shared memory, the other halves from the peer's, at the same
// offsets; D rows 0..127 land in the leader's TMEM, 128..255 in the peer's.
SVL_DEV void mma_tf32_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// As mma_tf32_pair with A read from tensor memory: each CTA's 128 lanes of
// `a_tmem` (row = lane, K = 8 consecutive 32-bit columns) hold its A rows.
SVL_DEV void mma_tf32_pair_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// kind::f16 forms of the pair MMAs (K = 16 per instruction).
SVL_DEV void mma_f16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// A from tensor memory: 16-bit elements packed two per 32-bit column (lower
// index in the low half), K = 16 elements = 8 columns per instruction.
SVL_DEV void mma_f16_pair_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Bounded wait with cluster-scope acquire: for barriers that the peer CTA
// of a pair arrives on (its writes before the arrive become visible).
SVL_DEV bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, uint32_t* err) {
  auto try_once = [&]() {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
  };
  if (try_once()) return true;
  const uint64_t start = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (try_once()) return true;
    if ((i & 255u) == 0 && global_ns() - start > kWaitDeadlineNs) {
      if (err) atomicOr(err, SVL_DEVERR_TIMEOUT);
      return false;
    }
  }
}

// Arrives on the mbarrier at this shared offset in every CTA of `cta_mask`
// once all prior tcgen05.mma of the pair have completed.
SVL_DEV void mma_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}

SVL_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
SVL_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Loads 32 consecutive FP32 columns of this thread's TMEM lane:
// taddr = base | (lane_base << 16) | column.
SVL_DEV void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Loads 16 consecutive FP32 columns of this thread's TMEM lane.
SVL_DEV void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Stores 32 consecutive FP32 columns into this thread's TMEM lane.
SVL_DEV void tmem_st32(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
      "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
      "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])),
      "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
      "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])),
      "r"(__float_as_uint(v[23])), "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])),
      "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])),
      "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

SVL_DEV void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Stores 16 consecutive 32-bit columns into this thread's TMEM lane.
SVL_DEV void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}


SVL_DEV void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// tmem_ld32 without the wait: issue several, then tmem_ld_wait_regs on each
// destination array (the wait must precede every use of the registers).
SVL_DEV void tmem_ld32_nowait(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

SVL_DEV void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Ties 32 registers written by tmem_ld32_nowait to a preceding tmem_ld_wait:
// the empty volatile statement stays after the wait and every later use of
// the registers depends on it.
SVL_DEV void tmem_regs_after_wait(uint32_t* r) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31]));
}

// Hardware base-2 exponential (PTX ex2.approx.ftz.f32): -inf -> +0, results
// below the normal range flush to zero.
SVL_DEV float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

SVL_DEV float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Non-blocking mbarrier phase tests (test_wait never suspends the thread,
// unlike try_wait): for a thread that polls several barriers.
SVL_DEV bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

SVL_DEV bool mbar_test_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

SVL_DEV bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .b32 r;\n\t.reg .pred p;\n\t"
      "elect.sync r|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(pred));
  return pred != 0;
}

// Round-to-nearest (ties away) conversion of an FP32 value to the TF32 grid
// (10 explicit mantissa bits), kept in an FP32 container.  Tensor cores read
// only the top 19 bits of a tf32 operand; producers of GEMM operands round
// with this so the tensor core sees a rounded, not a truncated, value.
SVL_DEV float round_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// GELU with the tanh approximation (src/tensor/kernels.rs:380-383):
//   0.5 * v * (1 + tanh(u)),  u = 0.7978846 * (v + 0.044715 * v^3).
// Since 0.5 * (1 + tanh(u)) = 1 / (1 + exp(-2u)), this is v / (1 + exp(-2u)),
// and exp(-2u) = 2^z with z = v * (c0 + c1 * v^2), c0 = -2 * 0.7978846 *
// log2(e), c1 = c0 * 0.044715: three multiply-adds, the hardware ex2 and a
// fast divide (relative error ~1e-6, far below the FP16 / TF32 operand
// rounding of the GEMM that produced v).  Large |v| saturate correctly:
// 2^z -> inf gives 0, 2^z -> 0 gives v (v^2 overflowing to inf included).
SVL_DEV float gelu_tanh(float v) {
  constexpr float c0 = -2.0f * 0.7978846f * 1.4426950408889634f;
  constexpr float c1 = c0 * 0.044715f;
  const float z = v * fmaf(v * v, c1, c0);
  return __fdividef(v, 1.0f + ex2_approx(z));
}

// Programmatic dependent launch: a kernel launched with launch_pdl may start
// while the previous kernel of its stream is still running.  pdl_trigger()
// lets the next kernel launch (once every CTA of this grid has called it or
// exited); pdl_wait() blocks until the previous grid has completed and its
// memory is visible -- every kernel launched that way calls it before it
// touches any buffer an earlier kernel writes or reads.  Both are no-ops for
// an ordinary launch.
SVL_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
SVL_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Per-warpgroup register reallocation (all four warps of a warpgroup execute
// it): inc takes registers from the block's pool, dec returns them.
template <int N>
SVL_DEV void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
SVL_DEV void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// max(m, |x|) that propagates NaN (PTX max.NaN), for range checks that must
// also catch non-finite values.
SVL_DEV float fmax_abs_nan(float m, float x) {
  float y;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(y) : "f"(m), "f"(fabsf(x)));
  return y;
}

SVL_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

SVL_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Launches `kern` with programmatic dependent launch allowed (the kernel must
// follow the pdl_wait() rule above); SVL_PDL=0 in the environment launches
// ordinarily instead.
inline bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("SVL_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

// Opts `kern` in to `bytes` of dynamic shared memory on the CURRENT device.
// cudaFuncSetAttribute applies to the current device only, and models and
// indexes of one process may live on different devices, so the opt-in is
// remembered per (kernel, device) in `done` (one bit per device ordinal,
// set atomically: concurrent first calls may both set the attribute, which
// is harmless).  Devices past 63 are opted in on every call.
template <typename... KArgs>
inline cudaError_t smem_opt_in(void (*kern)(KArgs...), int bytes, std::atomic<uint64_t>* done) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = dev < 64 ? 1ull << dev : 0;
  if (bit && (done->load(std::memory_order_acquire) & bit)) return cudaSuccess;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && bit) done->fetch_or(bit, std::memory_order_acq_rel);
  return e;
}
