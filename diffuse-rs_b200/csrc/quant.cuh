// quant.cuh -- GGUF block formats of the reference's weights, dequantised on
// the GPU: Q4_K, Q6_K, Q4_0, Q8_0 and F16 rows to bf16 or fp32
// (dequantize_q4k_row / _q6k_row / _q4_0_row / _q8_0_row and f16_to_f32,
// src/kernels.rs:46-217). Used once at load for projection weights (the
// projections then run as bf16 GEMMs with fp32 accumulation) and per step
// for the token-embedding gather (embed_tokens, src/model/forward.rs:
// 175-246). Byte/integer work, HBM-bound: one warp per 256 weights, each
// lane producing 8 consecutive outputs with one 16- or 32-byte store. The
// f32 arithmetic is the reference's, operation for operation (no
// contraction), so fp32 outputs are bit-identical to it.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace ca {

enum QType { kQF16 = 1, kQ4_0 = 2, kQ8_0 = 8, kQ4_K = 12, kQ6_K = 14 };

__host__ __device__ constexpr long long qrow_bytes(int qtype, long long cols) {
  return qtype == kQF16   ? 2 * cols
         : qtype == kQ4_0 ? cols / 32 * 18
         : qtype == kQ8_0 ? cols / 32 * 34
         : qtype == kQ4_K ? cols / 256 * 144
         : qtype == kQ6_K ? cols / 256 * 210
                          : 0;
}

struct DequantParams {
  const uint8_t* src;   // rows of qrow_bytes(qtype, cols) bytes
  long long rows, cols;
  const int* row_ids;   // output row i <- source row row_ids[i] (null: i)
  long long n_out;
  void* dst;            // [n_out, dst_stride]
  int dst_f32;
  long long dst_stride;
  float scale;          // applied after dequantisation (1: none)
  int qtype;
  int* err;             // set when a row id is out of range
};

__device__ __forceinline__ float h2f(const uint8_t* p) {
  const unsigned short h = static_cast<unsigned short>(p[0] | (p[1] << 8));
  return __half2float(__ushort_as_half(h));  // exact, subnormals included
}

// Exact float of a small integer (|v| < 2^22) without the XU pipe's
// int-to-float conversion: v is added to the mantissa of 1.5 * 2^23 and that
// constant subtracted again (both steps exact).
__device__ __forceinline__ float small_i2f(int v) {
  return __fsub_rn(__int_as_float(0x4B400000 + v), 12582912.0f);
}

// The 6-bit scale (which = 0) or min (which = 1) of sub-block j of a Q4_K
// block, from its 12 packed bytes (the utmp unpacking of the reference).
__device__ __forceinline__ int q4k_scale(const uint8_t* s, int j, int which) {
  if (j < 4) return which ? (s[j + 4] & 63) : (s[j] & 63);
  return which ? ((s[j + 4] >> 4) | ((s[j] >> 6) << 4)) : ((s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4));
}

// Eight consecutive weights idx .. idx + 7 (idx % 8 == 0) of one row.
__device__ __forceinline__ void dequant8(int qtype, const uint8_t* row, int idx, float (&o)[8]) {
  if (qtype == kQ4_K) {
    // Blocks of 144 bytes keep 8-byte alignment: the header (d, dmin) and
    // the 12 scale bytes load as 32-bit words, the lane's 8 quant bytes as
    // one 64-bit word.
    const uint8_t* b = row + (idx >> 8) * 144;
    const int v = idx & 255;
    const int pair = v >> 6, w = v & 63;  // 64 weights share one byte range
    const int sub = 2 * pair + (w >= 32 ? 1 : 0);
    const uint32_t hdr = __ldg(reinterpret_cast<const uint32_t*>(b));
    const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(hdr & 0xffffu)));
    const float dmin = __half2float(__ushort_as_half(static_cast<unsigned short>(hdr >> 16)));
    uint8_t s12[12];
    *reinterpret_cast<uint32_t*>(s12) = __ldg(reinterpret_cast<const uint32_t*>(b + 4));
    *reinterpret_cast<uint32_t*>(s12 + 4) = __ldg(reinterpret_cast<const uint32_t*>(b + 8));
    *reinterpret_cast<uint32_t*>(s12 + 8) = __ldg(reinterpret_cast<const uint32_t*>(b + 12));
    const float sc = small_i2f(q4k_scale(s12, sub, 0));
    const float mn = small_i2f(q4k_scale(s12, sub, 1));
    const uint2 qv = __ldg(reinterpret_cast<const uint2*>(b + 16 + pair * 32 + (w & 31)));
    const uint8_t qs[8] = {static_cast<uint8_t>(qv.x), static_cast<uint8_t>(qv.x >> 8),
                           static_cast<uint8_t>(qv.x >> 16), static_cast<uint8_t>(qv.x >> 24),
                           static_cast<uint8_t>(qv.y), static_cast<uint8_t>(qv.y >> 8),
                           static_cast<uint8_t>(qv.y >> 16), static_cast<uint8_t>(qv.y >> 24)};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int q = w >= 32 ? (qs[k] >> 4) : (qs[k] & 0xF);
      // d * sc * q - dmin * mn, left to right, no contraction
      o[k] = __fsub_rn(__fmul_rn(__fmul_rn(d, sc), small_i2f(q)), __fmul_rn(dmin, mn));
    }
  } else if (qtype == kQ6_K) {
    const uint8_t* b = row + (idx >> 8) * 210;
    const int v = idx & 255;
    const int h = v >> 7, g = (v & 127) >> 5, l0 = v & 31;
    const uint8_t* ql = b + h * 64 + (g & 1) * 32 + l0;
    const uint8_t* qh = b + 128 + h * 32 + l0;
    const float sc = __fmul_rn(h2f(b + 208), small_i2f(static_cast<int8_t>(b[192 + (v >> 4)])));
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int lo = g < 2 ? (ql[k] & 0xF) : (ql[k] >> 4);
      const int hi = (qh[k] >> (2 * g)) & 3;
      o[k] = __fmul_rn(sc, small_i2f((lo | (hi << 4)) - 32));
    }
  } else if (qtype == kQ4_0) {
    const uint8_t* b = row + (idx >> 5) * 18;
    const int w = idx & 31;
    const float d = h2f(b);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int q = w < 16 ? (b[2 + w + k] & 0xF) : (b[2 + w - 16 + k] >> 4);
      o[k] = __fmul_rn(d, __fsub_rn(small_i2f(q), 8.0f));
    }
  } else if (qtype == kQ8_0) {
    const uint8_t* b = row + (idx >> 5) * 34;
    const float d = h2f(b);
#pragma unroll
    for (int k = 0; k < 8; ++k)
      o[k] = __fmul_rn(d, small_i2f(static_cast<int8_t>(b[2 + (idx & 31) + k])));
  } else {  // F16
#pragma unroll
    for (int k = 0; k < 8; ++k) o[k] = h2f(row + 2 * (idx + k));
  }
}

// A work item is kUnits consecutive 256-weight units of one output row; one
// warp per item (grid-stride), all loads of the item issued before any is
// consumed. Item indices are 32-bit: one unsigned division per item.
constexpr int kUnits = 4;

__device__ __forceinline__ void dequant_store(const DequantParams& p, long long i, int idx,
                                              const float (&o)[8]) {
  const long long off = i * p.dst_stride + idx;
  if (p.dst_f32) {
    float4* d = reinterpret_cast<float4*>(static_cast<float*>(p.dst) + off);
    d[0] = make_float4(o[0], o[1], o[2], o[3]);
    d[1] = make_float4(o[4], o[5], o[6], o[7]);
  } else {
    uint4 w;
    w.x = pack_bf16(o[0], o[1]);
    w.y = pack_bf16(o[2], o[3]);
    w.z = pack_bf16(o[4], o[5]);
    w.w = pack_bf16(o[6], o[7]);
    *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.dst) + off) = w;
  }
}

__global__ void __launch_bounds__(256) dequant_kernel(const DequantParams p) {
  const int lane = threadIdx.x & 31;
  const unsigned units_per_row = static_cast<unsigned>((p.cols + 255) / 256);
  const unsigned items_per_row = (units_per_row + kUnits - 1) / kUnits;
  const unsigned items = static_cast<unsigned>(p.n_out) * items_per_row;
  const long long rb = qrow_bytes(p.qtype, p.cols);
  const unsigned nwarps = (gridDim.x * blockDim.x) >> 5;
  for (unsigned it = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; it < items; it += nwarps) {
    const unsigned i = it / items_per_row;
    const unsigned u0 = (it - i * items_per_row) * kUnits;
    const long long r = p.row_ids ? p.row_ids[i] : i;
    if (r < 0 || r >= p.rows) {
      if (lane == 0 && p.err) atomicExch(p.err, 1);
      continue;
    }
    const uint8_t* row = p.src + r * rb;
    float o[kUnits][8];
#pragma unroll
    for (int k = 0; k < kUnits; ++k) {
      const int idx = static_cast<int>((u0 + k) * 256 + lane * 8);
      if (idx < p.cols) dequant8(p.qtype, row, idx, o[k]);
    }
#pragma unroll
    for (int k = 0; k < kUnits; ++k) {
      const int idx = static_cast<int>((u0 + k) * 256 + lane * 8);
      if (idx >= p.cols) break;
      if (p.scale != 1.f) {
#pragma unroll
        for (int e = 0; e < 8; ++e) o[k][e] = __fmul_rn(o[k][e], p.scale);
      }
      dequant_store(p, i, idx, o[k]);
    }
  }
}

}  // namespace ca
