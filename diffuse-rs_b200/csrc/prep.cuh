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
};

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
  const long long jobs = static_cast<long long>(p.batch) * p.na * per_tok;
  for (long long job = static_cast<long long>(blockIdx.x) * 8 + warp; job < jobs;
       job += static_cast<long long>(gridDim.x) * 8) {
    const long long tok = job / per_tok;  // b * na + t
    const int r = static_cast<int>(job % per_tok);
    const int b = static_cast<int>(tok / p.na);
    const int pos = p.pos[tok];
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
      dst = p.cache_k + ((static_cast<long long>(b) * p.n_total + pos) * p.Hkv + h) * p.hd;
      w = p.k_norm_w;
      norm = w != nullptr;
    } else {
      const int h = r - rows_q - rows_kv;
      src = p.v + (tok * p.Hkv + h) * p.hd;
      dst = p.cache_v + ((static_cast<long long>(b) * p.n_total + pos) * p.Hkv + h) * p.hd;
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

// Vectorised form for head_dim in {64, 128, 256}: each lane owns 8
// consecutive elements (one 16-byte load and store), a row spans LPR =
// head_dim / 8 lanes and a warp handles 32 / LPR rows at once. The RoPE
// partner element (i <-> i + rope_dim/2) is read back from a per-warp staging
// row in shared memory.
template <int LPR>
__global__ void __launch_bounds__(256) prep_block_vec_kernel(const PrepParams p) {
  constexpr int RPW = 32 / LPR;   // rows per warp
  constexpr int HD = LPR * 8;
  __shared__ float stage[8][RPW][HD];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane / LPR, sl = lane % LPR;
  float* buf = stage[warp][sub];
  const int per_tok = p.H + 2 * p.Hkv;
  const long long jobs = static_cast<long long>(p.batch) * p.na * per_tok;
  const long long wstride = static_cast<long long>(gridDim.x) * 8 * RPW;
  for (long long base = (static_cast<long long>(blockIdx.x) * 8 + warp) * RPW; base < jobs;
       base += wstride) {
    const long long job = base + sub;
    const bool active = job < jobs;
    const long long jj = active ? job : base;
    const long long tok = jj / per_tok;
    const int r = static_cast<int>(jj % per_tok);
    const int b = static_cast<int>(tok / p.na);
    const int pos = p.pos[tok];
    const __nv_bfloat16* src;
    __nv_bfloat16* dst;
    const float* w = nullptr;
    bool norm = false, rope = true;
    if (r < p.H) {
      src = p.q + (tok * p.H + r) * HD;
      dst = p.q_out + (tok * p.H + r) * HD;
      w = p.q_norm_w;
      norm = w != nullptr;
    } else if (r < p.H + p.Hkv) {
      const int h = r - p.H;
      src = p.k + (tok * p.Hkv + h) * HD;
      dst = p.cache_k + ((static_cast<long long>(b) * p.n_total + pos) * p.Hkv + h) * HD;
      w = p.k_norm_w;
      norm = w != nullptr;
    } else {
      const int h = r - p.H - p.Hkv;
      src = p.v + (tok * p.Hkv + h) * HD;
      dst = p.cache_v + ((static_cast<long long>(b) * p.n_total + pos) * p.Hkv + h) * HD;
      norm = p.v_norm != 0;
      rope = false;
    }
    const int e0 = sl * 8;
    float x[8];
    {
      const uint4 raw = *reinterpret_cast<const uint4*>(src + e0);
      const uint32_t wv[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        x[2 * i] = __uint_as_float(wv[i] << 16);
        x[2 * i + 1] = __uint_as_float(wv[i] & 0xffff0000u);
      }
    }
    // Every lane of the warp joins the reductions; `norm` may differ per row.
    double ss = 0.0;
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += static_cast<double>(__fmul_rn(x[i], x[i]));
#pragma unroll
    for (int o = LPR / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (norm) {
      const float sc =
          __fdiv_rn(1.f, static_cast<float>(sqrt(ss / HD + static_cast<double>(p.eps))));
#pragma unroll
      for (int i = 0; i < 8; ++i) x[i] = w ? __fmul_rn(__fmul_rn(x[i], sc), w[e0 + i])
                                           : __fmul_rn(x[i], sc);
    }
    const int half = rope ? p.rope_dim / 2 : 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) buf[e0 + i] = x[i];
    __syncwarp();
    float y[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = e0 + i;
      if (e < half) {
        const float2 sc2 = reinterpret_cast<const float2*>(p.rope)[static_cast<long long>(pos) * half + e];
        y[i] = __fsub_rn(__fmul_rn(x[i], sc2.y), __fmul_rn(buf[e + half], sc2.x));
      } else if (e < 2 * half) {
        const int j = e - half;
        const float2 sc2 = reinterpret_cast<const float2*>(p.rope)[static_cast<long long>(pos) * half + j];
        y[i] = __fadd_rn(__fmul_rn(buf[j], sc2.x), __fmul_rn(x[i], sc2.y));
      } else {
        y[i] = x[i];
      }
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
