// prep.cuh -- the element-wise pre-ops of the attention block, fused into one
// pass over the active rows: per-head QK RMSNorm, optional unweighted V norm,
// NeoX RoPE at each row's sequence position, and the store of post-RoPE K/V
// into the position-indexed cache. Mirrors src/model/forward.rs:296-320:
//   norm_heads          src/model/ops.rs:385-389 (rms_norm_inplace :107-114)
//   rms_norm_noscale    src/model/ops.rs:117-124 (Gemma V, forward.rs:304-308)
//   rotate_rows         src/model/ops.rs:432-452
//   StepCache::store    src/model/cache.rs:62-70
// One warp handles one (token, head) row of Q, K or V. HBM-bound: each row is
// read once and written once.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>

#include "sm100.cuh"

namespace ca {

struct PrepParams {
  const __nv_bfloat16* q;  // [batch, na, H, hd]
  const __nv_bfloat16* k;  // [batch, na, Hkv, hd]
  const __nv_bfloat16* v;
  const int* pos;          // [batch, na]
  const float* q_norm_w;   // [hd] or null
  const float* k_norm_w;
  int v_norm;
  float eps;
  const float* rope;       // [rope_len, rope_dim/2, 2]
  int rope_len, rope_dim;
  __nv_bfloat16* q_out;    // [batch, na, H, hd]
  __nv_bfloat16* cache_k;  // [batch, n_total, Hkv, hd]
  __nv_bfloat16* cache_v;
  int batch, na, n_total, H, Hkv, hd;
  // Rows of one token per warp job in the vectorised kernels (a multiple of
  // the rows a warp covers per step): 16 for large batches; small batches
  // use one step per job so that more warps share the short pass.
  int rows_per_job;
  // Variable-length batches (cu_active != null): sequence b owns active rows
  // cu_active[b] .. cu_active[b+1]-1 and cache rows cu_total[b] ..; the
  // cache row of a token is cu_total[b] + its position.
  const int* cu_active;
  const int* cu_total;
  long long total_active;
  int* err;  // status word of the call (null: the device-wide word)
};

// Active tokens of the whole call.
__device__ __forceinline__ long long prep_tokens(const PrepParams& p) {
  return p.cu_active ? p.total_active : static_cast<long long>(p.batch) * p.na;
}

// Cache row (sequence base + position) of active token `tok`.
__device__ __forceinline__ long long cache_row(const PrepParams& p, long long tok, int pos) {
  if (!p.cu_active) return static_cast<long long>(tok / p.na) * p.n_total + pos;
  int lo = 0, hi = p.batch - 1;  // last b with cu_active[b] <= tok
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(p.cu_active + mid) <= tok) lo = mid;
    else hi = mid - 1;
  }
  return static_cast<long long>(__ldg(p.cu_total + lo)) + pos;
}

__device__ __forceinline__ uint32_t pack2_bf16(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// Sum of squares as the reference forms it: f32 products accumulated in f64.
__device__ __forceinline__ float rms_scale(const float* x, int hd, int lane, float eps) {
  double ss = 0.0;
  for (int e = lane; e < hd; e += 32) ss += static_cast<double>(__fmul_rn(x[e], x[e]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  return __fdiv_rn(1.f, static_cast<float>(sqrt(ss / hd + static_cast<double>(eps))));
}

__global__ void __launch_bounds__(256) prep_block_kernel(const PrepParams p) {
  extern __shared__ float prep_smem[];  // 8 warps x hd floats
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* buf = prep_smem + warp * p.hd;
  const int rows_q = p.H, rows_kv = p.Hkv;
  const int per_tok = rows_q + 2 * rows_kv;
  const long long jobs = prep_tokens(p) * per_tok;
  for (long long job = static_cast<long long>(blockIdx.x) * 8 + warp; job < jobs;
       job += static_cast<long long>(gridDim.x) * 8) {
    const long long tok = job / per_tok;  // b * na + t
    const int r = static_cast<int>(job % per_tok);
    const int pos = p.pos[tok];
    const long long crow = cache_row(p, tok, pos);
    const __nv_bfloat16* src;
    __nv_bfloat16* dst;
    const float* w = nullptr;
    bool norm = false, rope = true;
    if (r < rows_q) {
      src = p.q + (tok * p.H + r) * p.hd;
      dst = p.q_out + (tok * p.H + r) * p.hd;
      w = p.q_norm_w;
      norm = w != nullptr;
    } else if (r < rows_q + rows_kv) {
      const int h = r - rows_q;
      src = p.k + (tok * p.Hkv + h) * p.hd;
      dst = p.cache_k + (crow * p.Hkv + h) * p.hd;
      w = p.k_norm_w;
      norm = w != nullptr;
    } else {
      const int h = r - rows_q - rows_kv;
      src = p.v + (tok * p.Hkv + h) * p.hd;
      dst = p.cache_v + (crow * p.Hkv + h) * p.hd;
      norm = p.v_norm != 0;
      rope = false;  // V is not rotated (forward.rs:310 rotates Q and K only)
    }
    for (int e = lane; e < p.hd; e += 32) buf[e] = __bfloat162float(src[e]);
    __syncwarp();
    if (norm) {
      const float sc = rms_scale(buf, p.hd, lane, p.eps);
      for (int e = lane; e < p.hd; e += 32)
        buf[e] = w ? __fmul_rn(__fmul_rn(buf[e], sc), w[e]) : __fmul_rn(buf[e], sc);
      __syncwarp();
    }
    const int half = rope ? p.rope_dim / 2 : 0;
    for (int i = lane; i < half; i += 32) {
      const float sn = p.rope[2 * (static_cast<long long>(pos) * half + i)];
      const float cs = p.rope[2 * (static_cast<long long>(pos) * half + i) + 1];
      const float a = buf[i], bb = buf[i + half];
      dst[i] = __float2bfloat16_rn(__fsub_rn(__fmul_rn(a, cs), __fmul_rn(bb, sn)));
      dst[i + half] = __float2bfloat16_rn(__fadd_rn(__fmul_rn(a, sn), __fmul_rn(bb, cs)));
    }
    for (int e = 2 * half + lane; e < p.hd; e += 32) dst[e] = __float2bfloat16_rn(buf[e]);
    __syncwarp();
  }
}

// Vectorised form for head_dim in {64, 128, 256} with rope_dim % 16 == 0:
// one warp per (token, group of up to 16 rows). Each lane owns 8 consecutive elements of a row (one
// 16-byte load and store); a row spans LPR = head_dim / 8 lanes, so a warp
// covers 32 / LPR rows at a time and walks the token's H + 2 Hkv rows. The
// token's RoPE (sin, cos) entries are loaded once and reused for all its Q
// and K rows (they share the position). The partner element of the NeoX
// rotation (i <-> i + rope_dim/2) comes from a per-warp staging row.
template <int LPR>
__global__ void __launch_bounds__(256) prep_token_kernel(const PrepParams p) {
  constexpr int RPW = 32 / LPR;  // rows per warp per step
  constexpr int HD = LPR * 8;
  __shared__ __align__(16) float stage[8][RPW][HD];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane / LPR, sl = lane % LPR;
  const int e0 = sl * 8;
  const int half = p.rope_dim / 2;
  const long long n_tok = prep_tokens(p);
  const int per_tok = p.H + 2 * p.Hkv;
  // A job is up to rows_per_job rows of one token.
  const int kRowsPerJob = p.rows_per_job;
  const int chunks = (per_tok + kRowsPerJob - 1) / kRowsPerJob;
  const long long n_jobs = n_tok * chunks;
  float* buf = stage[warp][sub];
  for (long long job = static_cast<long long>(blockIdx.x) * 8 + warp; job < n_jobs;
       job += static_cast<long long>(gridDim.x) * 8) {
    const long long tok = job / chunks;
    const int row_beg = static_cast<int>(job % chunks) * kRowsPerJob;
    const int row_end = min(per_tok, row_beg + kRowsPerJob);
    const int pos = __ldg(p.pos + tok);
    const long long crow = cache_row(p, tok, pos);
    // This lane's 8 (sin, cos) pairs: entries e0..e0+7 of the lower or upper
    // half map to table entries (e0 mod half)..+7; rope_dim % 16 == 0 keeps
    // them inside one half.
    float sn[8], cs[8];
    const bool rot = e0 < 2 * half;
    {
      const int idx = e0 < half ? e0 : e0 - half;
      const float4* t4 = reinterpret_cast<const float4*>(p.rope + 2 * (static_cast<long long>(pos) * half + idx));
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 v = rot ? __ldg(t4 + i) : make_float4(0.f, 1.f, 0.f, 1.f);
        sn[2 * i] = v.x;
        cs[2 * i] = v.y;
        sn[2 * i + 1] = v.z;
        cs[2 * i + 1] = v.w;
      }
    }
    for (int r0 = row_beg; r0 < row_end; r0 += RPW) {
      const int r = r0 + sub;
      const bool active = r < row_end;
      const int rr = active ? r : r0;
      const __nv_bfloat16* src;
      __nv_bfloat16* dst;
      const float* w = nullptr;
      bool norm, rope = true;
      if (rr < p.H) {
        src = p.q + (tok * p.H + rr) * HD;
        dst = p.q_out + (tok * p.H + rr) * HD;
        w = p.q_norm_w;
        norm = w != nullptr;
      } else if (rr < p.H + p.Hkv) {
        const int h = rr - p.H;
        src = p.k + (tok * p.Hkv + h) * HD;
        dst = p.cache_k + (crow * p.Hkv + h) * HD;
        w = p.k_norm_w;
        norm = w != nullptr;
      } else {
        const int h = rr - p.H - p.Hkv;
        src = p.v + (tok * p.Hkv + h) * HD;
        dst = p.cache_v + (crow * p.Hkv + h) * HD;
        norm = p.v_norm != 0;
        rope = false;  // V is not rotated (forward.rs:310 rotates Q and K only)
      }
      float x[8];
      {
        const uint4 raw = __ldg(reinterpret_cast<const uint4*>(src + e0));
        const uint32_t wv[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          x[2 * i] = __uint_as_float(wv[i] << 16);
          x[2 * i + 1] = __uint_as_float(wv[i] & 0xffff0000u);
        }
      }
      // Every lane joins the reduction; `norm` may differ between the rows.
      double ss = 0.0;
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += static_cast<double>(__fmul_rn(x[i], x[i]));
#pragma unroll
      for (int o = LPR / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (norm) {
        const float sc =
            __fdiv_rn(1.f, static_cast<float>(sqrt(ss / HD + static_cast<double>(p.eps))));
        if (w) {
          const float4 w0 = __ldg(reinterpret_cast<const float4*>(w + e0));
          const float4 w1 = __ldg(reinterpret_cast<const float4*>(w + e0) + 1);
          const float wf[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
          for (int i = 0; i < 8; ++i) x[i] = __fmul_rn(__fmul_rn(x[i], sc), wf[i]);
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) x[i] = __fmul_rn(x[i], sc);
        }
      }
      reinterpret_cast<float4*>(buf + e0)[0] = make_float4(x[0], x[1], x[2], x[3]);
      reinterpret_cast<float4*>(buf + e0)[1] = make_float4(x[4], x[5], x[6], x[7]);
      __syncwarp();
      float y[8];
      if (rope && rot) {
        const int pe = e0 < half ? e0 + half : e0 - half;  // partner elements
        const float4 q0 = reinterpret_cast<const float4*>(buf + pe)[0];
        const float4 q1 = reinterpret_cast<const float4*>(buf + pe)[1];
        const float pr[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        if (e0 < half) {
#pragma unroll
          for (int i = 0; i < 8; ++i)
            y[i] = __fsub_rn(__fmul_rn(x[i], cs[i]), __fmul_rn(pr[i], sn[i]));
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i)
            y[i] = __fadd_rn(__fmul_rn(pr[i], sn[i]), __fmul_rn(x[i], cs[i]));
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) y[i] = x[i];
      }
      __syncwarp();
      if (active) {
        uint4 o;
        o.x = pack2_bf16(y[0], y[1]);
        o.y = pack2_bf16(y[2], y[3]);
        o.z = pack2_bf16(y[4], y[5]);
        o.w = pack2_bf16(y[6], y[7]);
        *reinterpret_cast<uint4*>(dst + e0) = o;
      }
    }
  }
}

// Full-rotation form (rope_dim == head_dim; dispatched for 256): lane sl of a
// row owns elements 4 sl .. 4 sl + 3 and their NeoX partners half + 4 sl ..
// half + 4 sl + 3 (half = head_dim / 2), loaded and stored as two 8-byte
// pieces. Every rotation pair is then inside one lane: no exchange through
// shared memory or shuffles, which leaves the row's f64 sum-of-squares
// reduction as the only cross-lane traffic (the kernel is bound by the
// shared-memory / shuffle pipe, not by HBM, when partners are exchanged;
// at head_dim 256 this form measured 10% faster, at 128 slower).
// Norm gains and the token's (sin, cos) entries are held in registers.
template <int LPR>
__global__ void __launch_bounds__(256) prep_pair_kernel(const PrepParams p) {
  constexpr int RPW = 32 / LPR;  // rows per warp per step
  constexpr int HD = LPR * 8;
  constexpr int HALF = HD / 2;
  const int kRowsPerJob = p.rows_per_job;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane / LPR, sl = lane % LPR;
  const int e0 = sl * 4;  // lower element block; the upper is e0 + HALF
  // Gains of the lane's 8 elements: [0..3] lower block, [4..7] upper block.
  float wq[8], wk[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) wq[i] = wk[i] = 1.f;
  if (p.q_norm_w) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      wq[i] = __ldg(p.q_norm_w + e0 + i);
      wq[4 + i] = __ldg(p.q_norm_w + HALF + e0 + i);
    }
  }
  if (p.k_norm_w) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      wk[i] = __ldg(p.k_norm_w + e0 + i);
      wk[4 + i] = __ldg(p.k_norm_w + HALF + e0 + i);
    }
  }
  const long long n_tok = prep_tokens(p);
  const int per_tok = p.H + 2 * p.Hkv;
  const int chunks = (per_tok + kRowsPerJob - 1) / kRowsPerJob;
  const long long n_jobs = n_tok * chunks;
  for (long long job = static_cast<long long>(blockIdx.x) * 8 + warp; job < n_jobs;
       job += static_cast<long long>(gridDim.x) * 8) {
    const long long tok = job / chunks;
    const int row_beg = static_cast<int>(job % chunks) * kRowsPerJob;
    const int row_end = min(per_tok, row_beg + kRowsPerJob);
    const int pos = __ldg(p.pos + tok);
    const long long crow = cache_row(p, tok, pos);
    float sn[4], cs[4];
    {
      const float4* t4 =
          reinterpret_cast<const float4*>(p.rope + 2 * (static_cast<long long>(pos) * HALF + e0));
      const float4 a = __ldg(t4), c = __ldg(t4 + 1);
      sn[0] = a.x; cs[0] = a.y; sn[1] = a.z; cs[1] = a.w;
      sn[2] = c.x; cs[2] = c.y; sn[3] = c.z; cs[3] = c.w;
    }
    for (int r0 = row_beg; r0 < row_end; r0 += RPW) {
      const int r = r0 + sub;
      const bool active = r < row_end;
      const int rr = active ? r : r0;
      const __nv_bfloat16* src;
      __nv_bfloat16* dst;
      int kind;  // 0 Q, 1 K, 2 V
      if (rr < p.H) {
        src = p.q + (tok * p.H + rr) * HD;
        dst = p.q_out + (tok * p.H + rr) * HD;
        kind = 0;
      } else if (rr < p.H + p.Hkv) {
        const int h = rr - p.H;
        src = p.k + (tok * p.Hkv + h) * HD;
        dst = p.cache_k + (crow * p.Hkv + h) * HD;
        kind = 1;
      } else {
        const int h = rr - p.H - p.Hkv;
        src = p.v + (tok * p.Hkv + h) * HD;
        dst = p.cache_v + (crow * p.Hkv + h) * HD;
        kind = 2;
      }
      const uint2 lo = __ldg(reinterpret_cast<const uint2*>(src + e0));
      const uint2 hi = __ldg(reinterpret_cast<const uint2*>(src + HALF + e0));
      float x[8];
      x[0] = __uint_as_float(lo.x << 16); x[1] = __uint_as_float(lo.x & 0xffff0000u);
      x[2] = __uint_as_float(lo.y << 16); x[3] = __uint_as_float(lo.y & 0xffff0000u);
      x[4] = __uint_as_float(hi.x << 16); x[5] = __uint_as_float(hi.x & 0xffff0000u);
      x[6] = __uint_as_float(hi.y << 16); x[7] = __uint_as_float(hi.y & 0xffff0000u);
      // Sum of squares as the reference forms it: f32 products summed in f64.
      double ss = 0.0;
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += static_cast<double>(__fmul_rn(x[i], x[i]));
#pragma unroll
      for (int o = LPR / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const bool weighted = kind == 0 ? p.q_norm_w != nullptr
                                      : kind == 1 ? p.k_norm_w != nullptr : false;
      const bool norm = kind == 2 ? p.v_norm != 0 : weighted;
      if (norm) {
        const float sc =
            __fdiv_rn(1.f, static_cast<float>(sqrt(ss / HD + static_cast<double>(p.eps))));
        if (weighted) {
#pragma unroll
          for (int i = 0; i < 8; ++i)
            x[i] = __fmul_rn(__fmul_rn(x[i], sc), kind == 0 ? wq[i] : wk[i]);
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) x[i] = __fmul_rn(x[i], sc);
        }
      }
      float y[8];
      if (kind != 2) {  // V is not rotated (forward.rs:310 rotates Q and K only)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float a = x[i], c = x[4 + i];
          y[i] = __fsub_rn(__fmul_rn(a, cs[i]), __fmul_rn(c, sn[i]));
          y[4 + i] = __fadd_rn(__fmul_rn(a, sn[i]), __fmul_rn(c, cs[i]));
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) y[i] = x[i];
      }
      if (active) {
        *reinterpret_cast<uint2*>(dst + e0) = make_uint2(pack2_bf16(y[0], y[1]), pack2_bf16(y[2], y[3]));
        *reinterpret_cast<uint2*>(dst + HALF + e0) =
            make_uint2(pack2_bf16(y[4], y[5]), pack2_bf16(y[6], y[7]));
      }
    }
  }
}

// Bulk-copy form (dispatched at head_dim 256; rope_dim % 16 == 0, 16-byte
// aligned Q/K/V): one producer lane per CTA streams each token's Q, K and V
// rows (contiguous in the inputs: H, Hkv and Hkv rows of head_dim) into a
// ring of kPrepStages shared-memory stages with cp.async.bulk, so many
// bytes are in flight per SM without holding registers; eight consumer warps
// normalise and rotate the rows out of shared memory (a NeoX partner element
// sits in the same staged row, so no exchange is needed) and store them to
// q_work and the cache. Arithmetic identical to prep_token_kernel.
constexpr int kPrepStages = 4;
constexpr int kPrepConsumers = 8;  // warps
constexpr int kPrepThreads = 32 * (kPrepConsumers + 1);

template <int LPR>
__global__ void __launch_bounds__(kPrepThreads) prep_bulk_kernel(const PrepParams p) {
  constexpr int RPW = 32 / LPR;  // rows per warp per step
  constexpr int HD = LPR * 8;
  extern __shared__ __align__(128) uint8_t prep_ring[];
  const int rows = p.H + 2 * p.Hkv;
  const uint32_t stage_bytes = static_cast<uint32_t>(rows) * HD * 2;
  const uint32_t ring = smem_u32(prep_ring);
  const uint32_t bars = ring + kPrepStages * stage_bytes;  // full[S], empty[S]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long n_tok = prep_tokens(p);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kPrepStages; ++s) {
      mbar_init(bars + 8 * s, 1);
      mbar_init(bars + 8 * (kPrepStages + s), kPrepConsumers);
    }
    fence_barrier_init();
  }
  __syncthreads();
  bool dead = false;
  if (warp == kPrepConsumers) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      int it = 0;
      for (long long tok = blockIdx.x; tok < n_tok; tok += gridDim.x, ++it) {
        const int s = it % kPrepStages;
        if (it >= kPrepStages &&
            !mbar_wait(bars + 8 * (kPrepStages + s), ((it / kPrepStages) - 1) & 1, dead, p.err))
          break;
        const uint32_t dst = ring + s * stage_bytes;
        mbar_arrive_expect_tx(bars + 8 * s, stage_bytes);
        if (p.H > 0) bulk_load(dst, p.q + tok * p.H * HD, p.H * HD * 2, bars + 8 * s);
        bulk_load(dst + p.H * HD * 2, p.k + tok * p.Hkv * HD, p.Hkv * HD * 2, bars + 8 * s);
        bulk_load(dst + (p.H + p.Hkv) * HD * 2, p.v + tok * p.Hkv * HD, p.Hkv * HD * 2,
                  bars + 8 * s);
      }
      // Leave no bulk copy in flight: wait (bounded) for the last stages.
      bool d2 = false;
      for (int j = it > kPrepStages ? it - kPrepStages : 0; j < it; ++j)
        mbar_wait(bars + 8 * (j % kPrepStages), (j / kPrepStages) & 1, d2, p.err);
    }
    return;
  }
  // ------------------------------------------------------------ consumers
  const int sub = lane / LPR, sl = lane % LPR;
  const int e0 = sl * 8;
  const int half = p.rope_dim / 2;
  const bool rot = e0 < 2 * half;
  const int pe = e0 < half ? e0 + half : e0 - half;  // NeoX partner elements
  int it = 0;
  for (long long tok = blockIdx.x; tok < n_tok; tok += gridDim.x, ++it) {
    const int s = it % kPrepStages;
    if (!mbar_wait(bars + 8 * s, (it / kPrepStages) & 1, dead, p.err)) break;
    const uint8_t* stage = prep_ring + s * stage_bytes;
    const int pos = __ldg(p.pos + tok);
    const long long crow = cache_row(p, tok, pos);
    float sn[8], cs[8];
    {
      const int idx = e0 < half ? e0 : e0 - half;
      const float4* t4 =
          reinterpret_cast<const float4*>(p.rope + 2 * (static_cast<long long>(pos) * half + idx));
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 v = rot ? __ldg(t4 + i) : make_float4(0.f, 1.f, 0.f, 1.f);
        sn[2 * i] = v.x;
        cs[2 * i] = v.y;
        sn[2 * i + 1] = v.z;
        cs[2 * i + 1] = v.w;
      }
    }
    for (int r0 = warp * RPW; r0 < rows; r0 += kPrepConsumers * RPW) {
      const int r = r0 + sub;
      const bool active = r < rows;
      const int rr = active ? r : r0;
      __nv_bfloat16* dst;
      const float* w = nullptr;
      bool norm, rope = true;
      if (rr < p.H) {
        dst = p.q_out + (tok * p.H + rr) * HD;
        w = p.q_norm_w;
        norm = w != nullptr;
      } else if (rr < p.H + p.Hkv) {
        dst = p.cache_k + (crow * p.Hkv + (rr - p.H)) * HD;
        w = p.k_norm_w;
        norm = w != nullptr;
      } else {
        dst = p.cache_v + (crow * p.Hkv + (rr - p.H - p.Hkv)) * HD;
        norm = p.v_norm != 0;
        rope = false;  // V is not rotated (forward.rs:310 rotates Q and K only)
      }
      const uint8_t* src = stage + static_cast<size_t>(rr) * HD * 2;
      float x[8], xp[8];
      {
        const uint4 raw = *reinterpret_cast<const uint4*>(src + e0 * 2);
        const uint32_t wv[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          x[2 * i] = __uint_as_float(wv[i] << 16);
          x[2 * i + 1] = __uint_as_float(wv[i] & 0xffff0000u);
        }
      }
      const bool do_rot = rope && rot;
      if (do_rot) {
        const uint4 raw = *reinterpret_cast<const uint4*>(src + pe * 2);
        const uint32_t wv[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          xp[2 * i] = __uint_as_float(wv[i] << 16);
          xp[2 * i + 1] = __uint_as_float(wv[i] & 0xffff0000u);
        }
      }
      // Every lane joins the reduction; `norm` may differ between the rows.
      double ss = 0.0;
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += static_cast<double>(__fmul_rn(x[i], x[i]));
#pragma unroll
      for (int o = LPR / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (norm) {
        const float sc =
            __fdiv_rn(1.f, static_cast<float>(sqrt(ss / HD + static_cast<double>(p.eps))));
        if (w) {
          const float4 w0 = __ldg(reinterpret_cast<const float4*>(w + e0));
          const float4 w1 = __ldg(reinterpret_cast<const float4*>(w + e0) + 1);
          const float wf[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
          for (int i = 0; i < 8; ++i) x[i] = __fmul_rn(__fmul_rn(x[i], sc), wf[i]);
          if (do_rot) {
            const float4 q0 = __ldg(reinterpret_cast<const float4*>(w + pe));
            const float4 q1 = __ldg(reinterpret_cast<const float4*>(w + pe) + 1);
            const float wp[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
            for (int i = 0; i < 8; ++i) xp[i] = __fmul_rn(__fmul_rn(xp[i], sc), wp[i]);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) x[i] = __fmul_rn(x[i], sc);
          if (do_rot) {
#pragma unroll
            for (int i = 0; i < 8; ++i) xp[i] = __fmul_rn(xp[i], sc);
          }
        }
      }
      float y[8];
      if (do_rot) {
        if (e0 < half) {
#pragma unroll
          for (int i = 0; i < 8; ++i)
            y[i] = __fsub_rn(__fmul_rn(x[i], cs[i]), __fmul_rn(xp[i], sn[i]));
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i)
            y[i] = __fadd_rn(__fmul_rn(xp[i], sn[i]), __fmul_rn(x[i], cs[i]));
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) y[i] = x[i];
      }
      if (active) {
        uint4 o;
        o.x = pack2_bf16(y[0], y[1]);
        o.y = pack2_bf16(y[2], y[3]);
        o.z = pack2_bf16(y[4], y[5]);
        o.w = pack2_bf16(y[6], y[7]);
        *reinterpret_cast<uint4*>(dst + e0) = o;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(bars + 8 * (kPrepStages + s));
  }
}


// Ring form for full rotation (rope_dim == head_dim, head_dim 64 / 128 / 256,
// 16-byte aligned rows). One producer lane per CTA streams T tokens per
// stage into a ring of kRingStages shared-memory stages: their Q rows, K rows
// and V rows (three cp.async.bulk copies: tokens are contiguous in each
// input), their positions (read by the producer and written beside the rows)
// and each token's row of the (sin, cos) table (one bulk copy per token), so
// no consumer waits on a dependent global load. kRingConsumers warps take the
// staged row groups round-robin across stages. A row spans LPR = head_dim / 32
// lanes and each lane owns four 16-byte chunks of it, chunk c * LPR + sl (c =
// 0..3, sl = lane within the row): chunks c and c + 2 are NeoX partners
// (element i and i + head_dim / 2), so every rotation pair is inside one lane
// and the only cross-lane step is the row's sum of squares (log2 LPR
// shuffles). Rows a multiple of 128 bytes apart would read the same banks, so
// each row of a bank phase walks its chunks in an order XOR-ed with its row
// index and the loaded registers are put back in order with selects.
// Arithmetic is the reference's, as in the other forms: f32 squares summed in
// f64 (exact for bf16 inputs), scale = 1 / (float) sqrt(ss / head_dim + eps),
// x * scale * w, then (a cos - b sin, a sin + b cos) with separately rounded
// products.
constexpr int kRingStages = 4;
constexpr int kRingConsumers = 16;  // warps
constexpr int kRingThreads = 32 * (kRingConsumers + 1);

// Shared memory of one stage: rows, then T positions (16-byte padded), then T
// table rows of head_dim floats.
__host__ __device__ inline uint32_t ring_stage_bytes(int T, int rows_tok, int hd) {
  return static_cast<uint32_t>(T) * rows_tok * hd * 2 + ((T * 4 + 15) / 16) * 16 +
         static_cast<uint32_t>(T) * hd * 4;
}
__host__ __device__ inline uint32_t ring_smem_bytes(int T, int rows_tok, int hd) {
  return kRingStages * ring_stage_bytes(T, rows_tok, hd) + 2 * hd * 4 + 16 * kRingStages;
}

template <int HD>
__global__ void __launch_bounds__(kRingThreads) prep_ring_kernel(const PrepParams p, int T) {
  constexpr int LPR = HD / 32;   // lanes per row
  constexpr int RPW = 32 / LPR;  // rows per warp step (one row group)
  constexpr int SWZ = 8 / LPR;   // rows sharing one 8-lane bank phase
  constexpr int Q4 = HD / 4;     // elements between a lane's consecutive chunks
  extern __shared__ __align__(128) uint8_t prep_ring[];
  const int rows_tok = p.H + 2 * p.Hkv;
  const int stage_rows = T * rows_tok;
  const uint32_t row_bytes = static_cast<uint32_t>(stage_rows) * HD * 2;
  const uint32_t pos_off = row_bytes, tab_off = row_bytes + ((T * 4 + 15) / 16) * 16;
  const uint32_t stage_bytes = ring_stage_bytes(T, rows_tok, HD);
  float* w_s = reinterpret_cast<float*>(prep_ring + kRingStages * stage_bytes);  // [2][HD]
  const uint32_t ring = smem_u32(prep_ring);
  const uint32_t bars = ring + kRingStages * stage_bytes + 2 * HD * 4;  // full[S], empty[S]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long n_tok = prep_tokens(p);
  const long long n_stage = (n_tok + T - 1) / T;
  const int groups = (stage_rows + RPW - 1) / RPW;  // row groups per stage
  if (threadIdx.x == 0) {
    for (int s = 0; s < kRingStages; ++s) {
      mbar_init(bars + 8 * s, 1);
      mbar_init(bars + 8 * (kRingStages + s), kRingConsumers);
    }
    fence_barrier_init();
  }
  for (int e = threadIdx.x; e < HD; e += blockDim.x) {
    w_s[e] = p.q_norm_w ? p.q_norm_w[e] : 1.f;
    w_s[HD + e] = p.k_norm_w ? p.k_norm_w[e] : 1.f;
  }
  __syncthreads();
  bool dead = false;
  if (warp == kRingConsumers) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      int it = 0;
      for (long long g = blockIdx.x; g < n_stage; g += gridDim.x, ++it) {
        const int s = it % kRingStages;
        if (it >= kRingStages &&
            !mbar_wait(bars + 8 * (kRingStages + s), ((it / kRingStages) - 1) & 1, dead, p.err))
          break;
        const long long tok0 = g * T;
        const int nt = static_cast<int>(min(static_cast<long long>(T), n_tok - tok0));
        const uint32_t dst = ring + s * stage_bytes;
        int* pos_s = reinterpret_cast<int*>(prep_ring + s * stage_bytes + pos_off);
        mbar_arrive_expect_tx(bars + 8 * s, static_cast<uint32_t>(nt) * (rows_tok * HD * 2 + HD * 4));
        if (p.H > 0)
          bulk_load(dst, p.q + tok0 * p.H * HD, nt * p.H * HD * 2, bars + 8 * s);
        bulk_load(dst + T * p.H * HD * 2, p.k + tok0 * p.Hkv * HD, nt * p.Hkv * HD * 2,
                  bars + 8 * s);
        bulk_load(dst + T * (p.H + p.Hkv) * HD * 2, p.v + tok0 * p.Hkv * HD,
                  nt * p.Hkv * HD * 2, bars + 8 * s);
        for (int t = 0; t < nt; ++t) {
          const int pos = __ldg(p.pos + tok0 + t);
          pos_s[t] = pos;  // ordered before the consumers' reads by the stage barrier
          bulk_load(dst + tab_off + t * HD * 4, p.rope + static_cast<long long>(pos) * HD,
                    HD * 4, bars + 8 * s);
        }
      }
      // Leave no bulk copy in flight: wait (bounded) for the last stages.
      bool d2 = false;
      for (int j = it > kRingStages ? it - kRingStages : 0; j < it; ++j)
        mbar_wait(bars + 8 * (j % kRingStages), (j / kRingStages) & 1, d2, p.err);
    }
    return;
  }
  // ------------------------------------------------------------ consumers
  const int sub = lane / LPR, sl = lane % LPR;
  const int sw = sub % SWZ;  // chunk-order XOR of this lane's row
  int it = 0;
  long long gbase = 0;  // this CTA's row groups before the current stage
  for (long long g = blockIdx.x; g < n_stage; g += gridDim.x, ++it, gbase += groups) {
    const int s = it % kRingStages;
    if (!mbar_wait(bars + 8 * s, (it / kRingStages) & 1, dead, p.err)) break;
    const long long tok0 = g * T;
    const int nt = static_cast<int>(min(static_cast<long long>(T), n_tok - tok0));
    const uint8_t* stage = prep_ring + s * stage_bytes;
    const int* pos_s = reinterpret_cast<const int*>(stage + pos_off);
    // Row groups k of this stage with (gbase + k) % consumers == warp.
    const int k0 = static_cast<int>((warp - gbase % kRingConsumers + kRingConsumers) %
                                    kRingConsumers);
    for (int k = k0; k < groups; k += kRingConsumers) {
      const int i = k * RPW + sub;  // row of the stage
      int kind, t, h;               // 0 Q, 1 K, 2 V; token in the stage; head
      if (i < T * p.H) {
        kind = 0; t = i / p.H; h = i - t * p.H;
      } else if (i < T * (p.H + p.Hkv)) {
        const int j = i - T * p.H;
        kind = 1; t = j / p.Hkv; h = j - t * p.Hkv;
      } else {
        const int j = i - T * (p.H + p.Hkv);
        kind = 2; t = j / p.Hkv; h = j - t * p.Hkv;
      }
      const bool valid = i < stage_rows && t < nt;
      // Chunks in bank-spread order, then back in logical order.
      const uint8_t* src = stage + static_cast<size_t>(valid ? i : 0) * HD * 2;
      uint4 raw[4];
#pragma unroll
      for (int c = 0; c < 4; ++c)
        raw[c] = *reinterpret_cast<const uint4*>(src + ((c ^ sw) * LPR + sl) * 16);
      if (sw & 1) {
        const uint4 t0 = raw[0], t2 = raw[2];
        raw[0] = raw[1]; raw[1] = t0; raw[2] = raw[3]; raw[3] = t2;
      }
      if (SWZ > 2 && (sw & 2)) {
        const uint4 t0 = raw[0], t1 = raw[1];
        raw[0] = raw[2]; raw[1] = raw[3]; raw[2] = t0; raw[3] = t1;
      }
      float x[32];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint32_t wv[4] = {raw[c].x, raw[c].y, raw[c].z, raw[c].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          x[c * 8 + 2 * e] = __uint_as_float(wv[e] << 16);
          x[c * 8 + 2 * e + 1] = __uint_as_float(wv[e] & 0xffff0000u);
        }
      }
      const bool weighted = kind == 0 ? p.q_norm_w != nullptr
                                      : kind == 1 ? p.k_norm_w != nullptr : false;
      const bool norm = valid && (kind == 2 ? p.v_norm != 0 : weighted);
      // Four independent chains; each term is an exact f32 square, so the
      // f64 sums are exact for the rows bf16 inputs form and the order is free.
      double ss = 0.0;
      if (norm) {
        double s4[4] = {0.0, 0.0, 0.0, 0.0};
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const double d = static_cast<double>(x[e]);
          s4[e & 3] = fma(d, d, s4[e & 3]);  // == s + (double)(x * x)
        }
        ss = (s4[0] + s4[1]) + (s4[2] + s4[3]);
      }
#pragma unroll
      for (int o = LPR / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (!valid) continue;
      const long long tok = tok0 + t;
      const int pos = pos_s[t];
      if (norm) {
        const float sc =
            __fdiv_rn(1.f, static_cast<float>(sqrt(ss / HD + static_cast<double>(p.eps))));
        if (weighted) {
          const float* w = w_s + (kind == 0 ? 0 : HD);
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const float4 w0 = *reinterpret_cast<const float4*>(w + c * Q4 + sl * 8);
            const float4 w1 = *reinterpret_cast<const float4*>(w + c * Q4 + sl * 8 + 4);
            const float wf[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
            for (int e = 0; e < 8; ++e) x[c * 8 + e] = __fmul_rn(__fmul_rn(x[c * 8 + e], sc), wf[e]);
          }
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) x[e] = __fmul_rn(x[e], sc);
        }
      }
      __nv_bfloat16* dst;
      if (kind == 0) {
        dst = p.q_out + (tok * p.H + h) * HD;
      } else {
        const long long crow = cache_row(p, tok, pos);
        dst = (kind == 1 ? p.cache_k : p.cache_v) + (crow * p.Hkv + h) * HD;
      }
      if (kind != 2) {  // V is not rotated (forward.rs:310 rotates Q and K only)
        // Chunks c and c + 2 (c = 0, 1) pair up; chunk c's elements use table
        // entries c * Q4 + sl * 8 .. + 7 of the token's staged row.
        const float* tab = reinterpret_cast<const float*>(stage + tab_off) + t * HD;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const float4* t4 = reinterpret_cast<const float4*>(tab + 2 * (c * Q4 + sl * 8));
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float4 v = t4[q];  // (sin, cos) of elements 2q, 2q + 1
            const float sn[2] = {v.x, v.z}, cs[2] = {v.y, v.w};
#pragma unroll
            for (int e2 = 0; e2 < 2; ++e2) {
              const int ia = c * 8 + 2 * q + e2, ib = ia + 16;
              const float a = x[ia], b = x[ib];
              x[ia] = __fsub_rn(__fmul_rn(a, cs[e2]), __fmul_rn(b, sn[e2]));
              x[ib] = __fadd_rn(__fmul_rn(a, sn[e2]), __fmul_rn(b, cs[e2]));
            }
          }
        }
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint4 o;
        o.x = pack2_bf16(x[c * 8 + 0], x[c * 8 + 1]);
        o.y = pack2_bf16(x[c * 8 + 2], x[c * 8 + 3]);
        o.z = pack2_bf16(x[c * 8 + 4], x[c * 8 + 5]);
        o.w = pack2_bf16(x[c * 8 + 6], x[c * 8 + 7]);
        *reinterpret_cast<uint4*>(dst + (c * LPR + sl) * 8) = o;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(bars + 8 * (kRingStages + s));
  }
}


// fp32 -> bf16 (round to nearest even), used by the host-buffer entry point.
__global__ void f32_to_bf16_kernel(const float* __restrict__ in, __nv_bfloat16* __restrict__ out,
                                   long long n) {
  const long long n4 = n / 4;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float4 x = reinterpret_cast<const float4*>(in)[i];
    __nv_bfloat162 a = __floats2bfloat162_rn(x.x, x.y);
    __nv_bfloat162 c = __floats2bfloat162_rn(x.z, x.w);
    reinterpret_cast<__nv_bfloat162*>(out)[2 * i] = a;
    reinterpret_cast<__nv_bfloat162*>(out)[2 * i + 1] = c;
  }
  for (long long i = n4 * 4 + blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
       i < n; i += static_cast<long long>(gridDim.x) * blockDim.x)
    out[i] = __float2bfloat16_rn(in[i]);
}

// fp32 [rows, hd] -> bf16 [rows, hd_p] with zero columns hd..hd_p-1, for
// head dims that are not a multiple of 8 (TMA rows must be 16-byte multiples).
__global__ void f32_to_bf16_pad_kernel(const float* __restrict__ in,
                                       __nv_bfloat16* __restrict__ out, long long rows, int hd,
                                       int hd_p) {
  const long long n = rows * hd_p;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / hd_p;
    const int c = static_cast<int>(i - r * hd_p);
    out[i] = __float2bfloat16_rn(c < hd ? in[r * hd + c] : 0.f);
  }
}

}  // namespace ca
