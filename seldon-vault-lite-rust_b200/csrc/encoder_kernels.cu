// encoder_kernels.cu -- the bandwidth-bound steps of the encoder forward
// (src/model/text.rs:182-538) as coalesced warp-per-row kernels.
//
// Packed-batch layout: the B sequences of a call are concatenated into T
// token rows; every activation is a row-major [T, width] FP32 matrix.  A
// token's sequence and position come from `seq_of` / `pos_of`.
//
// Arithmetic follows the reference kernels (kernels.rs) element by element;
// sums of squares are warp-tree reductions instead of the reference's
// sequential loop, which changes only the last bits (within the parity
// tolerance).  Multiplications are written with __fmul_rn / __fadd_rn where
// the reference rounds each operation, so the compiler does not fuse them.

#include "common.cuh"
#include "encoder_kernels.cuh"

namespace svl {

// --------------------------------------------------------------- indices --
__global__ void positions_kernel(const uint64_t* __restrict__ cu, uint32_t batch, uint32_t* __restrict__ seq_of,
                                 uint32_t* __restrict__ pos_of) {
  pdl_trigger();
  pdl_wait();
  const uint32_t b = blockIdx.x;
  if (b >= batch) return;
  const uint64_t s = cu[b], e = cu[b + 1];
  for (uint64_t t = s + threadIdx.x; t < e; t += blockDim.x) {
    seq_of[t] = b;
    pos_of[t] = (uint32_t)(t - s);
  }
}

// text.rs:211-224: hidden[t] = E[id_t] * embedding_scale.
__global__ void embed_kernel(const uint32_t* __restrict__ ids, int T, const float* __restrict__ table, int H,
                             uint32_t vocab, float scale, float* __restrict__ hidden, uint32_t* err) {
  pdl_trigger();
  pdl_wait();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= T) return;
  const uint32_t id = ids[warp];
  float* dst = hidden + (size_t)warp * H;
  if (id >= vocab) {
    if (lane == 0) atomicOr(err, SVL_DEVERR_BAD_TOKEN);
    for (int i = lane; i < H; i += 32) dst[i] = 0.0f;
    return;
  }
  const float* src = table + (size_t)id * H;
  for (int i = lane; i < H; i += 32) dst[i] = __fmul_rn(src[i], scale);
}

// kernels.rs:743-776 / 825-857 over `rows` rows of `width`, in place allowed:
// out = (x * pre) * inverse * w, inverse = 1 / sqrt(sum((x*pre)^2) / width + eps).
// `pre` is the PLE scale folded in before the norm (text.rs:294-306).
__global__ void rmsnorm_rows_kernel(const float* __restrict__ in, int ld_in, float* out, int ld_out, int rows,
                                    int width, const float* __restrict__ w, float pre, float eps, int round_out,
                                    uint32_t* err) {
  pdl_trigger();
  pdl_wait();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const float* x = in + (size_t)warp * ld_in;
  float* y = out + (size_t)warp * ld_out;
  float ss = 0.0f;
  for (int i = lane; i < width; i += 32) {
    const float v = __fmul_rn(x[i], pre);
    ss = __fadd_rn(ss, __fmul_rn(v, v));
  }
  ss = warp_sum(ss);
  const float inv = 1.0f / sqrtf(__fadd_rn(ss / (float)width, eps));
  bool bad = !isfinite(ss);
  for (int i = lane; i < width; i += 32) {
    float v = __fmul_rn(__fmul_rn(x[i], pre), inv);
    if (w) v = __fmul_rn(v, w[i]);
    bad |= !isfinite(v);
    y[i] = round_out ? round_tf32(v) : v;
  }
  if (bad) atomicOr(err, SVL_DEVERR_NONFINITE);
}

// text.rs:370-405: per-head q_norm / k_norm (weighted) and unscaled v norm,
// then rotate-half RoPE of q and k at the token's position (position offset 0).
// One warp per (token, head slot); slots [0, nh) are q, [nh, nh+kvh) k,
// [nh+kvh, nh+2kvh) v.  In place on the fused qkv row.
__global__ void qkv_post_kernel(float* __restrict__ qkv, int ld, int T, int nh, int kvh, int hd,
                                const float* __restrict__ q_norm, const float* __restrict__ k_norm,
                                const float* __restrict__ inv_freq, const uint32_t* __restrict__ pos_of,
                                float eps, int round_qk, uint32_t* err) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ float qkv_post_smem[];
  const int warp_in_block = threadIdx.x >> 5;
  const int gwarp = blockIdx.x * (blockDim.x >> 5) + warp_in_block;
  const int lane = threadIdx.x & 31;
  const int slots = nh + 2 * kvh;
  if (gwarp >= T * slots) return;
  const int t = gwarp / slots;
  const int slot = gwarp % slots;
  float* x = qkv + (size_t)t * ld + (size_t)slot * hd;
  float* buf = qkv_post_smem + warp_in_block * hd;
  const bool is_q = slot < nh, is_k = !is_q && slot < nh + kvh;
  const float* w = is_q ? q_norm : (is_k ? k_norm : nullptr);
  float ss = 0.0f;
  for (int i = lane; i < hd; i += 32) ss = __fadd_rn(ss, __fmul_rn(x[i], x[i]));
  ss = warp_sum(ss);
  const float inv = 1.0f / sqrtf(__fadd_rn(ss / (float)hd, eps));
  bool bad = !isfinite(ss);
  for (int i = lane; i < hd; i += 32) {
    float v = __fmul_rn(x[i], inv);
    if (w) v = __fmul_rn(v, w[i]);
    buf[i] = v;
  }
  __syncwarp();
  if (!is_q && !is_k) {
    for (int i = lane; i < hd; i += 32) {
      bad |= !isfinite(buf[i]);
      x[i] = round_qk ? round_tf32(buf[i]) : buf[i];
    }
  } else {
    const int half = hd / 2;
    const float position = (float)pos_of[t];
    for (int p = lane; p < half; p += 32) {
      const float angle = __fmul_rn(position, inv_freq[p]);
      float s, c;
      sincosf(angle, &s, &c);
      const float first = buf[p], second = buf[p + half];
      float a = __fsub_rn(__fmul_rn(first, c), __fmul_rn(second, s));
      float b = __fadd_rn(__fmul_rn(first, s), __fmul_rn(second, c));
      bad |= !isfinite(a) || !isfinite(b);
      x[p] = round_qk ? round_tf32(a) : a;
      x[p + half] = round_qk ? round_tf32(b) : b;
    }
  }
  if (bad) atomicOr(err, SVL_DEVERR_NONFINITE);
}

// Residual update shared by the three blocks of a layer (text.rs:424-433,
// 465-472, 502-513):
//   hidden = (hidden + rmsnorm(delta, w_post)) [* layer_scalar]
// then xn = rmsnorm(hidden, w_next) -- the next block's pre-norm -- for
// mode kResNormNext, or xn = hidden for kResRoundedCopy; xn only feeds a GEMM,
// so it is written TF32-rounded, or exact with kResExact or'ed into the mode
// (the split-precision GEMMs expand it themselves).  One warp per token row.
__global__ void residual_norm_kernel(float* __restrict__ hidden, const float* __restrict__ delta, int T, int H,
                                     const float* __restrict__ w_post, float layer_scalar, int apply_scalar,
                                     const float* __restrict__ w_next, float* __restrict__ xn, int mode, float eps,
                                     uint32_t* err) {
  pdl_trigger();
  pdl_wait();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= T) return;
  float* h = hidden + (size_t)warp * H;
  const float* d = delta + (size_t)warp * H;
  float ss = 0.0f;
  for (int i = lane; i < H; i += 32) ss = __fadd_rn(ss, __fmul_rn(d[i], d[i]));
  ss = warp_sum(ss);
  const float inv = 1.0f / sqrtf(__fadd_rn(ss / (float)H, eps));
  bool bad = !isfinite(ss);
  float ss2 = 0.0f;
  for (int i = lane; i < H; i += 32) {
    float v = __fadd_rn(h[i], __fmul_rn(__fmul_rn(d[i], inv), w_post[i]));
    if (apply_scalar) v = __fmul_rn(v, layer_scalar);
    bad |= !isfinite(v);
    h[i] = v;
    ss2 = __fadd_rn(ss2, __fmul_rn(v, v));
  }
  const bool rnd = !(mode & kResExact);
  mode &= ~kResExact;
  if (mode == kResRoundedCopy) {
    float* y = xn + (size_t)warp * H;
    for (int i = lane; i < H; i += 32) y[i] = rnd ? round_tf32(h[i]) : h[i];
  } else if (mode == kResNormNext) {
    ss2 = warp_sum(ss2);
    const float inv2 = 1.0f / sqrtf(__fadd_rn(ss2 / (float)H, eps));
    float* y = xn + (size_t)warp * H;
    for (int i = lane; i < H; i += 32) {
      const float v = __fmul_rn(__fmul_rn(h[i], inv2), w_next[i]);
      y[i] = rnd ? round_tf32(v) : v;
    }
  }
  if (bad) atomicOr(err, SVL_DEVERR_NONFINITE);
}

// kernels.rs:1037-1135 bidirectional GQA attention, scale 1.0, window radius
// `window` (< 0: full).  Online softmax; one warp per (query token, head),
// four keys per step for ILP.  Reads q/k/v from the fused qkv rows.
template <int R>  // R = ceil(hd / 32) elements per lane
__global__ void attention_simt_kernel(const float* __restrict__ qkv, int ld, int T, int nh, int kvh, int hd,
                                      const uint64_t* __restrict__ cu, const uint32_t* __restrict__ seq_of,
                                      const uint32_t* __restrict__ pos_of, int window, float* __restrict__ out,
                                      int ld_out, int round_out, uint32_t* err) {
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int h = blockIdx.y;
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  const int groups = nh / kvh;
  const int kv = h / groups;
  const uint32_t s = seq_of[t];
  const int64_t start = (int64_t)cu[s];
  const int L = (int)(cu[s + 1] - cu[s]);
  const int p = (int)pos_of[t];
  int j0 = 0, j1 = L - 1;
  if (window >= 0) {
    j0 = p - window > 0 ? p - window : 0;
    j1 = p + window < L - 1 ? p + window : L - 1;
  }
  float q[R], o[R];
  const float* qrow = qkv + (size_t)t * ld + (size_t)h * hd;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int i = lane + 32 * r;
    q[r] = i < hd ? qrow[i] : 0.0f;
    o[r] = 0.0f;
  }
  const size_t koff = (size_t)nh * hd + (size_t)kv * hd;
  const size_t voff = (size_t)(nh + kvh) * hd + (size_t)kv * hd;
  float m = -INFINITY, l = 0.0f;
  bool bad = false;
  for (int j = j0; j <= j1; j += 4) {
    float sc[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int jj = j + u <= j1 ? j + u : j1;
      const float* krow = qkv + (size_t)(start + jj) * ld + koff;
      float acc = 0.0f;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int i = lane + 32 * r;
        if (i < hd) acc = fmaf(q[r], krow[i], acc);
      }
      sc[u] = acc;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) sc[u] = warp_sum(sc[u]);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (j + u > j1) break;
      const float score = sc[u];
      bad |= !isfinite(score);
      const float m_new = fmaxf(m, score);
      const float corr = expf(m - m_new);
      const float pe = expf(score - m_new);
      l = l * corr + pe;
      const float* vrow = qkv + (size_t)(start + j + u) * ld + voff;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int i = lane + 32 * r;
        const float vv = i < hd ? vrow[i] : 0.0f;
        o[r] = fmaf(pe, vv, o[r] * corr);
      }
      m = m_new;
    }
  }
  const float inv_l = 1.0f / l;
  float* orow = out + (size_t)t * ld_out + (size_t)h * hd;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int i = lane + 32 * r;
    if (i < hd) {
      const float v = o[r] * inv_l;
      bad |= !isfinite(v);
      orow[i] = round_out ? round_tf32(v) : v;
    }
  }
  if (bad && lane == 0) atomicOr(err, SVL_DEVERR_NONFINITE);
}

// text.rs:529-531 + kernels.rs:916-927: per sequence, pooled = mean of the
// projected rows (column sums in row order, then * (1 / rows), exactly the
// reference's loop), normalized = l2(pooled), out = l2(normalized[:dim]).
// Mean pool, one thread per (sequence, column): the column's rows summed in
// the reference's order, then scaled by 1 / length (kernels.rs:916-927).
__global__ void pool_mean_kernel(const float* __restrict__ projected, int E, const uint64_t* __restrict__ cu,
                                 float* __restrict__ mean) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= E) return;
  const uint64_t r0 = cu[b], r1 = cu[b + 1], L = r1 - r0;
  const float* x = projected + r0 * E + c;
  // One thread per column of a sequence is bound by load latency: rows are
  // loaded 32 at a time, the next group in flight while the current one is
  // added (the adds stay in row order).
  constexpr int G = 32;
  float cur[G], nxt[G];
#pragma unroll
  for (int j = 0; j < G; ++j) cur[j] = (uint64_t)j < L ? x[(uint64_t)j * E] : 0.0f;
  float acc = 0.0f;
  for (uint64_t r = 0; r < L; r += G) {
#pragma unroll
    for (int j = 0; j < G; ++j) nxt[j] = r + G + j < L ? x[(r + G + j) * E] : 0.0f;
#pragma unroll
    for (int j = 0; j < G; ++j)
      if (r + j < L) acc = __fadd_rn(acc, cur[j]);
#pragma unroll
    for (int j = 0; j < G; ++j) cur[j] = nxt[j];
  }
  mean[(size_t)b * E + c] = __fmul_rn(acc, 1.0f / (float)L);
}

// L2 normalisation and Matryoshka truncation of the pooled rows (one block
// per sequence).
__global__ void pool_normalize_kernel(const float* __restrict__ mean, int E, int dim, float* __restrict__ pooled_out,
                                      float* __restrict__ normalized_out, float* __restrict__ out, uint32_t* err) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ float pool_smem[];  // E floats + 32 partials
  float* red = pool_smem + E;
  const int b = blockIdx.x;
  float ss = 0.0f, ss_dim = 0.0f;
  for (int c = threadIdx.x; c < E; c += blockDim.x) {
    const float acc = mean[(size_t)b * E + c];
    pool_smem[c] = acc;
    if (pooled_out) pooled_out[(size_t)b * E + c] = acc;
    ss = __fadd_rn(ss, __fmul_rn(acc, acc));
  }
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  ss = warp_sum(ss);
  if (lane == 0) red[wid] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < nw ? red[threadIdx.x] : 0.0f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float total = red[0];
  __syncthreads();
  const bool bad = !isfinite(total) || total <= 0.0f;
  const float inv = 1.0f / sqrtf(total);
  for (int c = threadIdx.x; c < E; c += blockDim.x) {
    const float v = __fmul_rn(pool_smem[c], inv);
    pool_smem[c] = v;
    if (normalized_out) normalized_out[(size_t)b * E + c] = v;
    if (c < dim) ss_dim = __fadd_rn(ss_dim, __fmul_rn(v, v));
  }
  ss_dim = warp_sum(ss_dim);
  if (lane == 0) red[wid] = ss_dim;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < nw ? red[threadIdx.x] : 0.0f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float inv_dim = 1.0f / sqrtf(red[0]);
  if (out)
    for (int c = threadIdx.x; c < dim; c += blockDim.x) out[(size_t)b * dim + c] = __fmul_rn(pool_smem[c], inv_dim);
  if (threadIdx.x == 0 && (bad || !isfinite(red[0]) || red[0] <= 0.0f)) atomicOr(err, SVL_DEVERR_NONFINITE);
}

// Rounds a buffer to the TF32 grid in place (weights at upload).
__global__ void round_tf32_kernel(float* x, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    x[i] = round_tf32(x[i]);
}

// Widens BF16 bits to FP32 (src/binary/bf16.rs:40: bits << 16).
__global__ void bf16_widen_kernel(const uint16_t* __restrict__ in, float* __restrict__ out, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    out[i] = __uint_as_float((uint32_t)in[i] << 16);
}

// Operand expansion for the split-precision GEMMs: x = hi + lo with hi the
// TF32 rounding of x (round to nearest, ties away) and lo the TF32 rounding
// of the exact remainder x - hi.  Activation rows [rows, K] become
// [hi | hi | lo] and weight rows [hi | lo | hi] (weights = 1), so one
// TF32 product over K' = 3K accumulates hi*hi + hi*lo + lo*hi: every product
// then carries ~22 significant bits instead of 11 (the dropped lo*lo term
// and the rounding of lo are ~2^-22 relative).
__global__ void split3_kernel(const float* __restrict__ in, int ld_in, float* __restrict__ out, int rows, int K,
                              int weights) {
  pdl_trigger();
  pdl_wait();
  const size_t n = (size_t)rows * K;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / K, c = i - r * K;
    const float x = in[r * ld_in + c];
    const float hi = round_tf32(x);
    const float lo = round_tf32(__fsub_rn(x, hi));
    float* o = out + r * 3 * (size_t)K + c;
    o[0] = hi;
    o[K] = weights ? lo : hi;
    o[2 * (size_t)K] = weights ? hi : lo;
  }
}

// Flags a non-finite value anywhere in x (weight validation at upload).
__global__ void finite_check_kernel(const float* __restrict__ x, size_t n, uint32_t* err) {
  bool bad = false;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    bad |= !isfinite(x[i]);
  if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) atomicOr(err, SVL_DEVERR_NONFINITE);
}

// ------------------------------------------- register-resident row kernels --
// The same three row operations for widths that are multiples of 128 (the
// production model: hidden 512, per-layer input 512, head dims 256 / 512).
// A warp holds its whole row in registers (V float4 per lane), so every load
// of the row is in flight at once and nothing is read twice.

// The FP16 row scale of a GEMM output that no single kernel sees whole (the
// GeGLU and PLE-gate outputs, written tile by tile) from a bound that holds
// for every element: with n = ||a|| the norm of the row `a` that feeds the
// producing GEMM, |gelu(a . w_g) * x| <= max(n * a_max, 0.17) * x_max, where
// a_max = the largest row norm of that GEMM's weight (Cauchy-Schwarz; gelu(t)
// >= -0.17) and x_max = n * b_max (GeGLU: x = a . w_u) or row_max[r * stride]
// (PLE gate: x = the per-layer input).  A loose bound only moves the row
// down inside FP16's normal range; twice the bound keeps clear of overflow.
template <int V>
SVL_DEV void bound_scale_row(const BoundScale& bs, const float4* a, int row, int lane) {
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < V; ++i) ss += a[i].x * a[i].x + a[i].y * a[i].y + a[i].z * a[i].z + a[i].w * a[i].w;
  const float n = sqrtf(warp_sum(ss));
  const float x_max = bs.row_max ? bs.row_max[(size_t)row * bs.stride] : n * bs.b_max;
  float scale, inv;
  pow2_row_scale(2.0f * fmaxf(n * bs.a_max, 0.17f) * x_max, scale, inv);
  if (lane == 0) bs.inv[row] = inv;
}

// A warp's row (V float4 per lane, lane-interleaved) as an FP16 GEMM operand
// row: power-of-two scaled so the largest magnitude lies in [2^14, 2^15)
// (pow2_row_scale), *inv_out = the inverse scale.
template <int V>
SVL_DEV void store_row_f16(const float4* v, uint16_t* y, float* inv_out, int lane) {
  float mx = 0.0f;
#pragma unroll
  for (int i = 0; i < V; ++i) mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
  mx = warp_max(mx);
  float scale, inv;
  pow2_row_scale(mx, scale, inv);
  uint2* y2 = (uint2*)y;
#pragma unroll
  for (int i = 0; i < V; ++i)
    y2[lane + 32 * i] = make_uint2(pack_half2(v[i].x * scale, v[i].y * scale), pack_half2(v[i].z * scale, v[i].w * scale));
  if (lane == 0) *inv_out = inv;
}

template <int V>  // row width = 128 * V
__global__ void residual_norm_vec_kernel(float* __restrict__ hidden, const float* __restrict__ delta, int T,
                                         const float* __restrict__ w_post, float layer_scalar, int apply_scalar,
                                         const float* __restrict__ w_next, float* __restrict__ xn, int mode,
                                         float eps, uint16_t* __restrict__ xn16, float* __restrict__ xn_inv,
                                         BoundScale bs, uint32_t* err) {
  pdl_trigger();
  pdl_wait();
  constexpr int H = 128 * V;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= T) return;
  const bool rnd = !(mode & kResExact);
  mode &= ~kResExact;
  float4* h4 = (float4*)(hidden + (size_t)warp * H);
  const float4* d4 = (const float4*)(delta + (size_t)warp * H);
  float4 d[V], h[V];
#pragma unroll
  for (int i = 0; i < V; ++i) {
    d[i] = d4[lane + 32 * i];
    h[i] = h4[lane + 32 * i];
  }
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < V; ++i)
    ss = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(ss, __fmul_rn(d[i].x, d[i].x)), __fmul_rn(d[i].y, d[i].y)),
                             __fmul_rn(d[i].z, d[i].z)),
                   __fmul_rn(d[i].w, d[i].w));
  ss = warp_sum(ss);
  const float inv = 1.0f / sqrtf(__fadd_rn(ss / (float)H, eps));
  bool bad = !isfinite(ss);
  float ss2 = 0.0f;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const float4 w = ((const float4*)w_post)[lane + 32 * i];
    float4 v;
    v.x = __fadd_rn(h[i].x, __fmul_rn(__fmul_rn(d[i].x, inv), w.x));
    v.y = __fadd_rn(h[i].y, __fmul_rn(__fmul_rn(d[i].y, inv), w.y));
    v.z = __fadd_rn(h[i].z, __fmul_rn(__fmul_rn(d[i].z, inv), w.z));
    v.w = __fadd_rn(h[i].w, __fmul_rn(__fmul_rn(d[i].w, inv), w.w));
    if (apply_scalar) {
      v.x = __fmul_rn(v.x, layer_scalar);
      v.y = __fmul_rn(v.y, layer_scalar);
      v.z = __fmul_rn(v.z, layer_scalar);
      v.w = __fmul_rn(v.w, layer_scalar);
    }
    bad |= !isfinite(v.x) || !isfinite(v.y) || !isfinite(v.z) || !isfinite(v.w);
    h[i] = v;
    h4[lane + 32 * i] = v;
    ss2 = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(ss2, __fmul_rn(v.x, v.x)), __fmul_rn(v.y, v.y)), __fmul_rn(v.z, v.z)),
                    __fmul_rn(v.w, v.w));
  }
  if (xn16) {
    // FP16 operand rows for the next GEMM (row-scaled)
    if (mode == kResRoundedCopy) {
      store_row_f16<V>(h, xn16 + (size_t)warp * H, xn_inv + warp, lane);
      if (bs.inv) bound_scale_row<V>(bs, h, warp, lane);
    } else if (mode == kResNormNext) {
      ss2 = warp_sum(ss2);
      const float inv2 = 1.0f / sqrtf(__fadd_rn(ss2 / (float)H, eps));
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const float4 w = ((const float4*)w_next)[lane + 32 * i];
        h[i] = make_float4(__fmul_rn(__fmul_rn(h[i].x, inv2), w.x), __fmul_rn(__fmul_rn(h[i].y, inv2), w.y),
                           __fmul_rn(__fmul_rn(h[i].z, inv2), w.z), __fmul_rn(__fmul_rn(h[i].w, inv2), w.w));
      }
      store_row_f16<V>(h, xn16 + (size_t)warp * H, xn_inv + warp, lane);
      if (bs.inv) bound_scale_row<V>(bs, h, warp, lane);
    }
    if (bad) atomicOr(err, SVL_DEVERR_NONFINITE);
    return;
  }
  float4* y4 = (float4*)(xn + (size_t)warp * H);
  auto r4 = [rnd](float4 v) {
    return rnd ? make_float4(round_tf32(v.x), round_tf32(v.y), round_tf32(v.z), round_tf32(v.w)) : v;
  };
  if (mode == kResRoundedCopy) {
#pragma unroll
    for (int i = 0; i < V; ++i) y4[lane + 32 * i] = r4(h[i]);
  } else if (mode == kResNormNext) {
    ss2 = warp_sum(ss2);
    const float inv2 = 1.0f / sqrtf(__fadd_rn(ss2 / (float)H, eps));
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const float4 w = ((const float4*)w_next)[lane + 32 * i];
      y4[lane + 32 * i] = r4(make_float4(__fmul_rn(__fmul_rn(h[i].x, inv2), w.x), __fmul_rn(__fmul_rn(h[i].y, inv2), w.y),
                                         __fmul_rn(__fmul_rn(h[i].z, inv2), w.z), __fmul_rn(__fmul_rn(h[i].w, inv2), w.w)));
    }
  }
  if (bad) atomicOr(err, SVL_DEVERR_NONFINITE);
}

template <int V>  // row width = 128 * V
__global__ void rmsnorm_rows_vec_kernel(const float* __restrict__ in, int ld_in, float* out, int ld_out, int rows,
                                        const float* __restrict__ w, float pre, float eps, int round_out,
                                        uint16_t* __restrict__ out16, float* __restrict__ inv16,
                                        float* __restrict__ row_absmax, float* __restrict__ row_inv, uint32_t* err) {
  pdl_trigger();
  pdl_wait();
  constexpr int W = 128 * V;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const float4* x4 = (const float4*)(in + (size_t)warp * ld_in);
  float4 x[V];
#pragma unroll
  for (int i = 0; i < V; ++i) {
    x[i] = x4[lane + 32 * i];
    x[i].x = __fmul_rn(x[i].x, pre);
    x[i].y = __fmul_rn(x[i].y, pre);
    x[i].z = __fmul_rn(x[i].z, pre);
    x[i].w = __fmul_rn(x[i].w, pre);
  }
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < V; ++i)
    ss = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(ss, __fmul_rn(x[i].x, x[i].x)), __fmul_rn(x[i].y, x[i].y)),
                             __fmul_rn(x[i].z, x[i].z)),
                   __fmul_rn(x[i].w, x[i].w));
  ss = warp_sum(ss);
  const float inv = 1.0f / sqrtf(__fadd_rn(ss / (float)W, eps));
  if (row_inv && lane == 0) row_inv[warp] = inv;
  bool bad = !isfinite(ss);
#pragma unroll
  for (int i = 0; i < V; ++i) {
    float4 v = make_float4(__fmul_rn(x[i].x, inv), __fmul_rn(x[i].y, inv), __fmul_rn(x[i].z, inv), __fmul_rn(x[i].w, inv));
    if (w) {
      const float4 g = ((const float4*)w)[lane + 32 * i];
      v = make_float4(__fmul_rn(v.x, g.x), __fmul_rn(v.y, g.y), __fmul_rn(v.z, g.z), __fmul_rn(v.w, g.w));
    }
    bad |= !isfinite(v.x) || !isfinite(v.y) || !isfinite(v.z) || !isfinite(v.w);
    x[i] = v;
  }
  if (row_absmax) {
    float mx = 0.0f;
#pragma unroll
    for (int i = 0; i < V; ++i)
      mx = fmaxf(mx, fmaxf(fmaxf(fabsf(x[i].x), fabsf(x[i].y)), fmaxf(fabsf(x[i].z), fabsf(x[i].w))));
    mx = warp_max(mx);
    if (lane == 0) row_absmax[warp] = mx;
  }
  if (out16) {
    store_row_f16<V>(x, out16 + (size_t)warp * ld_out, inv16 + warp, lane);
  } else if (out) {  // (statistics only without an output)
    float4* y4 = (float4*)(out + (size_t)warp * ld_out);
#pragma unroll
    for (int i = 0; i < V; ++i) {
      float4 v = x[i];
      if (round_out) v = make_float4(round_tf32(v.x), round_tf32(v.y), round_tf32(v.z), round_tf32(v.w));
      y4[lane + 32 * i] = v;
    }
  }
  if (bad) atomicOr(err, SVL_DEVERR_NONFINITE);
}

// Per-head norms and RoPE (text.rs:370-405) with a head of hd = 32 * E values
// held as E / 4 chunks of 128: lane l holds elements 128 c + 4 l .. 128 c +
// 4 l + 3 of chunk c, so each warp access covers 512 contiguous bytes.  For
// hd >= 256 the rotate-half partner of element e < hd / 2 (e + hd / 2) sits in
// chunk c + E / 8 of the same lane; for hd = 128 it is 16 lanes away.
// cos / sin come from `rope` = [position][hd / 2] (cos, sin) pairs computed
// once per model with the same sincosf of (position * inv_freq).
// IN16: the projection was stored in FP16 by the GEMM's grouped epilogue
// (kEpiStore16): chunk c of the head is one 128-column group, its values
// in16 * gi[group], and the head's sum of squares is the sum of its groups'
// partial sums pss[group] (of the unrounded values), added in order.
template <int E, bool IN16>
__global__ void qkv_post_vec_kernel(float* __restrict__ qkv, int ld, int T, int nh, int kvh,
                                    const float* __restrict__ q_norm, const float* __restrict__ k_norm,
                                    const float2* __restrict__ rope, const uint32_t* __restrict__ pos_of, float eps,
                                    int round_qkv, uint16_t* __restrict__ out16, uint32_t* err,
                                    const uint16_t* __restrict__ in16, const float* __restrict__ gi,
                                    const float* __restrict__ pss, int gstride) {
  pdl_trigger();
  pdl_wait();
  constexpr int HD = 32 * E, HALF = HD / 2, C = E / 4;
  const int gwarp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int slots = nh + 2 * kvh;
  if (gwarp >= T * slots) return;
  const int t = gwarp / slots;
  const int slot = gwarp % slots;
  float4* x = IN16 ? nullptr : (float4*)(qkv + (size_t)t * ld + (size_t)slot * HD);
  const bool is_q = slot < nh, is_k = !is_q && slot < nh + kvh;
  float4 v[C];
  float ss = 0.0f;
  if constexpr (IN16) {
    const uint2* x16 = (const uint2*)(in16 + (size_t)t * ld + (size_t)slot * HD);
    const size_t g0 = (size_t)t * gstride + (size_t)slot * HD / 128;
#pragma unroll
    for (int c = 0; c < C; ++c) {
      const uint2 w = x16[lane + 32 * c];
      const float s = gi[g0 + c];
      const float2 a = unpack_half2(w.x), b = unpack_half2(w.y);
      v[c] = make_float4(a.x * s, a.y * s, b.x * s, b.y * s);
      ss += pss[g0 + c];
    }
  } else {
#pragma unroll
    for (int c = 0; c < C; ++c) v[c] = x[lane + 32 * c];
#pragma unroll
    for (int c = 0; c < C; ++c) {
      ss = __fadd_rn(ss, __fmul_rn(v[c].x, v[c].x));
      ss = __fadd_rn(ss, __fmul_rn(v[c].y, v[c].y));
      ss = __fadd_rn(ss, __fmul_rn(v[c].z, v[c].z));
      ss = __fadd_rn(ss, __fmul_rn(v[c].w, v[c].w));
    }
    ss = warp_sum(ss);
  }
  const float inv = 1.0f / sqrtf(__fadd_rn(ss / (float)HD, eps));
  bool bad = !isfinite(ss);
  const float* w = is_q ? q_norm : (is_k ? k_norm : nullptr);
#pragma unroll
  for (int c = 0; c < C; ++c)
    v[c] = make_float4(__fmul_rn(v[c].x, inv), __fmul_rn(v[c].y, inv), __fmul_rn(v[c].z, inv), __fmul_rn(v[c].w, inv));
  if (w) {
#pragma unroll
    for (int c = 0; c < C; ++c) {
      const float4 g = ((const float4*)w)[lane + 32 * c];
      v[c] = make_float4(__fmul_rn(v[c].x, g.x), __fmul_rn(v[c].y, g.y), __fmul_rn(v[c].z, g.z),
                         __fmul_rn(v[c].w, g.w));
    }
    // two (cos, sin) pairs per float4: pairs 2 k and 2 k + 1
    const float4* cs = (const float4*)(rope + (size_t)pos_of[t] * HALF);
    auto rot = [](float a, float b, float co, float si, float& ra, float& rb) {
      ra = __fsub_rn(__fmul_rn(a, co), __fmul_rn(b, si));
      rb = __fadd_rn(__fmul_rn(a, si), __fmul_rn(b, co));
    };
    if constexpr (C >= 2) {
#pragma unroll
      for (int c = 0; c < C / 2; ++c) {
        const float4 t0 = cs[64 * c + 2 * lane], t1 = cs[64 * c + 2 * lane + 1];
        float4 a = v[c], b = v[c + C / 2];
        rot(a.x, b.x, t0.x, t0.y, v[c].x, v[c + C / 2].x);
        rot(a.y, b.y, t0.z, t0.w, v[c].y, v[c + C / 2].y);
        rot(a.z, b.z, t1.x, t1.y, v[c].z, v[c + C / 2].z);
        rot(a.w, b.w, t1.z, t1.w, v[c].w, v[c + C / 2].w);
      }
    } else {
      // hd = 128: lanes 0..15 hold the first half, lane l + 16 the partners
      const bool first = lane < 16;
      const int q = lane & 15;
      const float4 t0 = cs[2 * q], t1 = cs[2 * q + 1];
      float4 o = v[0];
      const float4 pt = make_float4(__shfl_xor_sync(0xffffffffu, o.x, 16), __shfl_xor_sync(0xffffffffu, o.y, 16),
                                    __shfl_xor_sync(0xffffffffu, o.z, 16), __shfl_xor_sync(0xffffffffu, o.w, 16));
      const float4 a = first ? o : pt, b = first ? pt : o;
      float4 ra, rb;
      rot(a.x, b.x, t0.x, t0.y, ra.x, rb.x);
      rot(a.y, b.y, t0.z, t0.w, ra.y, rb.y);
      rot(a.z, b.z, t1.x, t1.y, ra.z, rb.z);
      rot(a.w, b.w, t1.z, t1.w, ra.w, rb.w);
      v[0] = first ? ra : rb;
    }
  }
  if (IN16 || out16) {
    // FP16 copy for the attention kernel (same [t][slot * HD] layout); FP16
    // holds |x| <= 65504, anything larger is reported
    uint2* y = (uint2*)(out16 + (size_t)t * ld + (size_t)slot * HD);
#pragma unroll
    for (int c = 0; c < C; ++c) {
      const float4 o = v[c];
      bad |= !(fmaxf(fmaxf(fabsf(o.x), fabsf(o.y)), fmaxf(fabsf(o.z), fabsf(o.w))) <= 65504.0f);
      y[lane + 32 * c] = make_uint2(pack_half2(o.x, o.y), pack_half2(o.z, o.w));
    }
  } else {
#pragma unroll
    for (int c = 0; c < C; ++c) {
      float4 o = v[c];
      bad |= !isfinite(o.x) || !isfinite(o.y) || !isfinite(o.z) || !isfinite(o.w);
      if (round_qkv) o = make_float4(round_tf32(o.x), round_tf32(o.y), round_tf32(o.z), round_tf32(o.w));
      x[lane + 32 * c] = o;
    }
  }
  if (bad) atomicOr(err, SVL_DEVERR_NONFINITE);
}

// (cos, sin) of (position * inv_freq[p]) for positions [0, n_pos), the angle
// and the functions exactly as qkv_post_kernel evaluates them.  Layout
// [position][p] (position_major) or [p][position] (pair-major: consecutive
// positions adjacent, for a warp whose lanes are consecutive tokens).
__global__ void rope_table_kernel(const float* __restrict__ inv_freq, int half, int n_pos, int position_major,
                                  float2* __restrict__ out) {
  const size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= (size_t)n_pos * half) return;
  const int pos = (int)(i / half), p = (int)(i % half);
  float s, c;
  sincosf(__fmul_rn((float)pos, inv_freq[p]), &s, &c);
  out[position_major ? i : (size_t)p * n_pos + pos] = make_float2(c, s);
}

// FP32 rows -> FP16 GEMM operand rows with a power-of-two scale per row (one
// warp per row): out = fp16(in * 2^-e), inv_scale[row] = 2^e.
__global__ void rows_to_f16_kernel(const float* __restrict__ in, int ld_in, uint16_t* __restrict__ out, int ld_out,
                                   int rows, int width, float* __restrict__ inv_scale, uint32_t* err) {
  pdl_trigger();
  pdl_wait();
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* x = in + (size_t)row * ld_in;
  float mx = 0.0f;
  bool bad = false;
  for (int i = lane; i < width; i += 32) {
    const float v = x[i];
    bad |= !isfinite(v);
    mx = fmaxf(mx, fabsf(v));
  }
  mx = warp_max(mx);
  float scale, inv;
  pow2_row_scale(mx, scale, inv);
  uint16_t* y = out + (size_t)row * ld_out;
  for (int i = 2 * lane; i < width; i += 64) {
    const uint32_t h = pack_half2(x[i] * scale, i + 1 < width ? x[i + 1] * scale : 0.0f);
    y[i] = (uint16_t)(h & 0xFFFFu);
    if (i + 1 < width) y[i + 1] = (uint16_t)(h >> 16);
  }
  if (lane == 0) inv_scale[row] = inv;
  if (bad && err) atomicOr(err, SVL_DEVERR_NONFINITE);
}

// A whole matrix -> FP16 with one power-of-two scale (weights: their rows
// span far fewer binades than FP16's normal range).  Pass 1 reduces the
// largest magnitude into *maxbits (non-negative floats order like their bit
// patterns); pass 2 converts and writes the inverse scale.
__global__ void matrix_absmax_kernel(const float* __restrict__ in, size_t n, uint32_t* maxbits) {
  float mx = 0.0f;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    mx = fmaxf(mx, fabsf(in[i]));
  mx = warp_max(mx);
  if ((threadIdx.x & 31) == 0) atomicMax(maxbits, __float_as_uint(mx));
}

__global__ void matrix_to_f16_kernel(const float* __restrict__ in, size_t n, const uint32_t* maxbits,
                                     uint16_t* __restrict__ out, float* inv_out) {
  float scale, inv;
  pow2_row_scale(__uint_as_float(*maxbits), scale, inv);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; 2 * i < n; i += (size_t)gridDim.x * blockDim.x) {
    const uint32_t h = pack_half2(in[2 * i] * scale, 2 * i + 1 < n ? in[2 * i + 1] * scale : 0.0f);
    out[2 * i] = (uint16_t)(h & 0xFFFFu);
    if (2 * i + 1 < n) out[2 * i + 1] = (uint16_t)(h >> 16);
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) *inv_out = inv;
}

// Largest row L2 norm of a [rows, cols] matrix, split by row class: rows with
// (row / period) even go to out[0], the others to out[1] (period 0: all to
// out[0]); out[] must start at zero (non-negative floats order like their
// bits).  One warp per row.
__global__ void row_norm_max_kernel(const float* __restrict__ w, int rows, int cols, int period, uint32_t* out) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* x = w + (size_t)row * cols;
  float ss = 0.0f;
  for (int i = lane; i < cols; i += 32) ss = fmaf(x[i], x[i], ss);
  ss = warp_sum(ss);
  if (lane == 0) atomicMax(out + (period > 0 && (row / period) % 2 == 1 ? 1 : 0), __float_as_uint(sqrtf(ss)));
}

// ------------------------------------------------------------ launchers --
static inline int blocks_for(size_t warps, int warps_per_block) {
  return (int)((warps + warps_per_block - 1) / warps_per_block);
}

void launch_positions(const uint64_t* cu, uint32_t batch, uint32_t* seq_of, uint32_t* pos_of, cudaStream_t st) {
  launch_pdl(positions_kernel, dim3(batch), dim3(256), 0, st, cu, batch, seq_of, pos_of);
}

void launch_embed(const uint32_t* ids, int T, const float* table, int H, uint32_t vocab, float scale, float* hidden,
                  uint32_t* err, cudaStream_t st) {
  launch_pdl(embed_kernel, dim3(blocks_for(T, 8)), dim3(256), 0, st, ids, T, table, H, vocab, scale, hidden, err);
}

static inline bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

bool launch_rmsnorm_rows(const float* in, int ld_in, float* out, int ld_out, int rows, int width, const float* w,
                         float pre, float eps, int round_out, uint32_t* err, cudaStream_t st, uint16_t* out16,
                         float* inv16, float* row_absmax, float* row_inv) {
  const bool vec = width % 128 == 0 && ld_in % 4 == 0 && ld_out % 4 == 0 && aligned16(in) &&
                   (out16 ? aligned16(out16) && aligned16(inv16) : aligned16(out)) && (!w || aligned16(w));
#define SVL_RMS(V)                                                                                              \
  launch_pdl(rmsnorm_rows_vec_kernel<V>, dim3(blocks_for(rows, 8)), dim3(256), 0, st, in, ld_in, out, ld_out, rows, w, pre, eps, \
                                                                  round_out, out16, inv16, row_absmax, row_inv, err)
  if (vec && width == 512) SVL_RMS(4);
  else if (vec && width == 256) SVL_RMS(2);
  else if (vec && width == 1024) SVL_RMS(8);
  else if (vec && width == 128) SVL_RMS(1);
  else if (out16 || row_absmax || row_inv || !out)
    return false;  // FP16 operands, row statistics and no-output runs only from the vectorised kernel
  else
    launch_pdl(rmsnorm_rows_kernel, dim3(blocks_for(rows, 8)), dim3(256), 0, st, in, ld_in, out, ld_out, rows, width, w, pre, eps,
                                                             round_out, err);
#undef SVL_RMS
  return true;
}

void launch_rope_table(const float* inv_freq, int half, int n_pos, int position_major, float2* out, cudaStream_t st) {
  const size_t n = (size_t)n_pos * half;
  rope_table_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(inv_freq, half, n_pos, position_major, out);
}

bool launch_qkv_post(float* qkv, int ld, int T, int nh, int kvh, int hd, const float* q_norm, const float* k_norm,
                     const float* inv_freq, const float2* rope, const uint32_t* pos_of, float eps, int round_qk,
                     uint16_t* out16, uint32_t* err, cudaStream_t st) {
  const size_t warps = (size_t)T * (nh + 2 * kvh);
  const bool vec = rope && ld % 4 == 0 && aligned16(qkv) && aligned16(q_norm) && aligned16(k_norm) &&
                   aligned16(rope) && (!out16 || aligned16(out16));
#define SVL_QP(EE)                                                                                                   \
  launch_pdl(qkv_post_vec_kernel<EE, false>, dim3(blocks_for(warps, 8)), dim3(256), 0, st, qkv, ld, T, nh, kvh, q_norm, k_norm, rope, pos_of, \
                                                                eps, round_qk, out16, err, (const uint16_t*)nullptr, (const float*)nullptr, (const float*)nullptr, 0)
  if (vec && hd == 256)
    SVL_QP(8);
  else if (vec && hd == 512)
    SVL_QP(16);
  else if (vec && hd == 128)
    SVL_QP(4);
  else if (out16)
    return false;  // FP16 output only from the vectorised kernel
  else
    launch_pdl(qkv_post_kernel, dim3(blocks_for(warps, 8)), dim3(256), 8 * hd * sizeof(float), st, qkv, ld, T, nh, kvh, hd, q_norm, k_norm,
                                                                               inv_freq, pos_of, eps, round_qk, err);
#undef SVL_QP
  return true;
}

bool launch_qkv_post16(const uint16_t* in16, const float* gi, const float* pss, int gstride, int ld, int T, int nh,
                       int kvh, int hd, const float* q_norm, const float* k_norm, const float2* rope,
                       const uint32_t* pos_of, float eps, uint16_t* out16, uint32_t* err, cudaStream_t st) {
  const size_t warps = (size_t)T * (nh + 2 * kvh);
  if (!rope || !out16 || ld % 128 || gstride < ld / 128 || !aligned16(in16) || !aligned16(q_norm) ||
      !aligned16(k_norm) || !aligned16(rope) || !aligned16(out16) || (hd != 128 && hd != 256 && hd != 512))
    return false;
#define SVL_QP16(EE)                                                                                          \
  launch_pdl(qkv_post_vec_kernel<EE, true>, dim3(blocks_for(warps, 8)), dim3(256), 0, st, (float*)nullptr, ld, T, nh, \
             kvh, q_norm, k_norm, rope, pos_of, eps, 0, out16, err, in16, gi, pss, gstride)
  if (hd == 512)
    SVL_QP16(16);
  else if (hd == 256)
    SVL_QP16(8);
  else
    SVL_QP16(4);
#undef SVL_QP16
  return true;
}

bool launch_residual_norm(float* hidden, const float* delta, int T, int H, const float* w_post, float layer_scalar,
                          int apply_scalar, const float* w_next, float* xn, int mode, float eps, uint32_t* err,
                          cudaStream_t st, uint16_t* xn16, float* xn_inv, const BoundScale* bound) {
  const bool vec = H % 128 == 0 && aligned16(hidden) && aligned16(delta) && aligned16(w_post) &&
                   (xn16 ? aligned16(xn16) && aligned16(xn_inv) : aligned16(xn)) && (!w_next || aligned16(w_next));
  const BoundScale bs = bound ? *bound : BoundScale{};
#define SVL_RES(V)                                                                                               \
  launch_pdl(residual_norm_vec_kernel<V>, dim3(blocks_for(T, 8)), dim3(256), 0, st, hidden, delta, T, w_post, layer_scalar,          \
                                                                apply_scalar, w_next, xn, mode, eps, xn16, xn_inv, \
                                                                bs, err)
  if (vec && H == 512) SVL_RES(4);
  else if (vec && H == 256) SVL_RES(2);
  else if (vec && H == 1024) SVL_RES(8);
  else if (vec && H == 128) SVL_RES(1);
  else if (xn16 || bound)
    return false;  // FP16 operands only from the vectorised kernel
  else
    launch_pdl(residual_norm_kernel, dim3(blocks_for(T, 8)), dim3(256), 0, st, hidden, delta, T, H, w_post, layer_scalar, apply_scalar,
                                                           w_next, xn, mode, eps, err);
#undef SVL_RES
  return true;
}

bool launch_attention_simt(const float* qkv, int ld, int T, int nh, int kvh, int hd, const uint64_t* cu,
                           const uint32_t* seq_of, const uint32_t* pos_of, int window, float* out, int ld_out,
                           int round_out, uint32_t* err, cudaStream_t st) {
  dim3 grid(blocks_for(T, 4), nh);
  const int R = (hd + 31) / 32;
#define SVL_ATT(RR) \
  attention_simt_kernel<RR><<<grid, 128, 0, st>>>(qkv, ld, T, nh, kvh, hd, cu, seq_of, pos_of, window, out, ld_out, round_out, err)
  if (R <= 1) SVL_ATT(1);
  else if (R <= 2) SVL_ATT(2);
  else if (R <= 4) SVL_ATT(4);
  else if (R <= 8) SVL_ATT(8);
  else if (R <= 16) SVL_ATT(16);
  else if (R <= 32) SVL_ATT(32);
  else return false;
#undef SVL_ATT
  return true;
}

void launch_pool_normalize(const float* projected, int E, const uint64_t* cu, int batch, int dim, float* mean,
                           float* pooled, float* normalized, float* out, uint32_t* err, cudaStream_t st) {
  launch_pdl(pool_mean_kernel, dim3(dim3((unsigned)((E + 127) / 128), (unsigned)batch)), dim3(128), 0, st, projected, E, cu, mean);
  launch_pdl(pool_normalize_kernel, dim3(batch), dim3(256), (E + 32) * sizeof(float), st, mean, E, dim, pooled, normalized, out, err);
}

void launch_rows_to_f16(const float* in, int ld_in, uint16_t* out, int ld_out, int rows, int width, float* inv_scale,
                        uint32_t* err, cudaStream_t st) {
  launch_pdl(rows_to_f16_kernel, dim3(blocks_for(rows, 8)), dim3(256), 0, st, in, ld_in, out, ld_out, rows, width, inv_scale, err);
}

void launch_matrix_to_f16(const float* in, size_t n, uint16_t* out, float* inv_out, uint32_t* scratch, cudaStream_t st) {
  cudaMemsetAsync(scratch, 0, sizeof(uint32_t), st);
  matrix_absmax_kernel<<<1184, 256, 0, st>>>(in, n, scratch);
  matrix_to_f16_kernel<<<1184, 256, 0, st>>>(in, n, scratch, out, inv_out);
}

void launch_row_norm_max(const float* w, int rows, int cols, int period, uint32_t* out2, cudaStream_t st) {
  row_norm_max_kernel<<<blocks_for(rows, 8), 256, 0, st>>>(w, rows, cols, period, out2);
}

void launch_split3(const float* in, int ld_in, float* out, int rows, int K, int weights, cudaStream_t st) {
  const size_t n = (size_t)rows * K;
  const unsigned blocks = (unsigned)(n / 256 + 1 < 2368 ? n / 256 + 1 : 2368);
  launch_pdl(split3_kernel, dim3(blocks), dim3(256), 0, st, in, ld_in, out, rows, K, weights);
}

void launch_round_tf32(float* x, size_t n, cudaStream_t st) {
  round_tf32_kernel<<<1184, 256, 0, st>>>(x, n);
}

void launch_bf16_widen(const uint16_t* in, float* out, size_t n, cudaStream_t st) {
  bf16_widen_kernel<<<1184, 256, 0, st>>>(in, out, n);
}

void launch_finite_check(const float* x, size_t n, uint32_t* err, cudaStream_t st) {
  finite_check_kernel<<<1184, 256, 0, st>>>(x, n, err);
}

}  // namespace svl
