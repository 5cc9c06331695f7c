// sampler.cuh -- per-candidate statistics of one denoising step on the GPU.
//
// Mirrors collect_candidates (src/model/sampler.rs:720-749) for the greedy
// pick (temperature 0, pick_token :754-764) after suppress_mask_token and
// suppress_tokens (:90-113): for each masked candidate, over its logit row,
//   token    first index of the row maximum
//   margin   top1 - top2 of the row's values (top2_logits :75-87; equal
//            maxima give margin 0)
//   entropy  compute_entropy (:7-20): sum of -p * lp over entries with
//            p > 1e-10, lp = (l - max) - ln(sum exp(l - max))
//   prob     exp(top1 - log_sum_exp(row)) (:22-25)
// Exponentials use the fast exp (ex2.approx; relative error ~1e-6 for the
// arguments here), well inside the step's tolerance on entropy and prob.
// The logits are read from HBM once per row for the first four reductions
// (an online max / sum of exponentials) and a second time, mostly from L2
// (the resident CTAs' rows, 0.5 MB each at a 126k vocabulary), for the
// entropy's thresholded sum. HBM-bound.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace ca {

constexpr int kCandThreads = 1024;

struct CandParams {
  float* logits;         // [rows, row_stride]; suppressed entries are set to -inf in place
  long long n_vocab;
  long long row_stride;
  const int* rows;       // [n_cand] logit row of each candidate
  int n_cand;
  int mask_id;           // < 0: none
  const int* suppress;   // [n_suppress] or null
  int n_suppress;
  int want_entropy;
  int want_prob;
  int* token;
  float* entropy;
  float* margin;
  float* prob;
};

// Running statistics of a stretch of one row.
struct CandAcc {
  float t1, t2;  // the two largest values (with multiplicity)
  int idx;       // first index holding t1
  float s;       // sum of exp(l - t1) over the stretch
};

__device__ __forceinline__ void cand_push(CandAcc& a, float x, int j) {
  if (x > a.t1) {
    a.s = (a.t1 == -INFINITY ? 0.f : a.s * __expf(a.t1 - x)) + 1.f;
    a.t2 = a.t1;
    a.t1 = x;
    a.idx = j;
  } else {
    if (x > a.t2) a.t2 = x;
    if (x != -INFINITY) a.s += __expf(x - a.t1);
  }
}

__device__ __forceinline__ CandAcc cand_merge(const CandAcc& a, const CandAcc& b) {
  CandAcc r;
  const bool a_hi = a.t1 > b.t1 || (a.t1 == b.t1 && a.idx < b.idx);
  const CandAcc& hi = a_hi ? a : b;
  const CandAcc& lo = a_hi ? b : a;
  r.t1 = hi.t1;
  r.idx = hi.idx;
  r.t2 = fmaxf(lo.t1, fmaxf(hi.t2, lo.t2));
  if (hi.t1 == -INFINITY) {
    r.s = 0.f;
  } else {
    r.s = hi.s + (lo.t1 == -INFINITY ? 0.f : lo.s * expf(lo.t1 - hi.t1));
  }
  return r;
}

__device__ __forceinline__ CandAcc cand_shfl(const CandAcc& a, int o) {
  CandAcc b;
  b.t1 = __shfl_xor_sync(0xffffffffu, a.t1, o);
  b.t2 = __shfl_xor_sync(0xffffffffu, a.t2, o);
  b.idx = __shfl_xor_sync(0xffffffffu, a.idx, o);
  b.s = __shfl_xor_sync(0xffffffffu, a.s, o);
  return b;
}

__device__ void cand_row(const CandParams& p, int c, CandAcc* red, float* red_h, int tid,
                         int lane, int warp);

// One row per CTA iteration; CTAs are persistent (at most one per SM), so
// the rows being reduced at any time (one per SM) stay resident in L2 for
// the entropy pass: 148 rows of a 126k vocabulary are 74 MB.
__global__ void __launch_bounds__(kCandThreads) cand_stats_kernel(const CandParams p) {
  __shared__ CandAcc red[kCandThreads / 32];
  __shared__ float red_h[kCandThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int c = blockIdx.x; c < p.n_cand; c += gridDim.x) {
    cand_row(p, c, red, red_h, tid, lane, warp);
    __syncthreads();  // red / red_h are reused by the next row
  }
}

__device__ void cand_row(const CandParams& p, int c, CandAcc* red, float* red_h, int tid,
                         int lane, int warp) {
  float* row = p.logits + static_cast<long long>(p.rows[c]) * p.row_stride;
  // Suppression writes first (the reference sets these logits to -inf).
  if (tid == 0 && p.mask_id >= 0 && p.mask_id < p.n_vocab) row[p.mask_id] = -INFINITY;
  for (int i = tid; i < p.n_suppress; i += kCandThreads) {
    const int id = p.suppress[i];
    if (id >= 0 && id < p.n_vocab) row[id] = -INFINITY;
  }
  __syncthreads();

  CandAcc a{-INFINITY, -INFINITY, 0x7fffffff, 0.f};
  const long long n = p.n_vocab;
  const bool vec = (reinterpret_cast<uintptr_t>(row) & 15u) == 0;
  long long done = 0;
  if (vec) {
    // Four 16-byte loads in flight per thread before any is consumed: one
    // CTA per row leaves few warps per SM, so each must keep HBM busy.
    const long long n4 = n / 4;
    const float4* r4 = reinterpret_cast<const float4*>(row);
    constexpr int U = 4;
    long long i = tid;
    for (; i + (U - 1) * kCandThreads < n4; i += U * kCandThreads) {
      float4 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) v[u] = __ldg(r4 + i + u * kCandThreads);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int j = static_cast<int>(4 * (i + u * kCandThreads));
        cand_push(a, v[u].x, j);
        cand_push(a, v[u].y, j + 1);
        cand_push(a, v[u].z, j + 2);
        cand_push(a, v[u].w, j + 3);
      }
    }
    for (; i < n4; i += kCandThreads) {
      const float4 v = __ldg(r4 + i);
      const int j = static_cast<int>(4 * i);
      cand_push(a, v.x, j);
      cand_push(a, v.y, j + 1);
      cand_push(a, v.z, j + 2);
      cand_push(a, v.w, j + 3);
    }
    done = 4 * n4;
  }
  for (long long i = done + tid; i < n; i += kCandThreads) cand_push(a, row[i], static_cast<int>(i));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) a = cand_merge(a, cand_shfl(a, o));
  if (lane == 0) red[warp] = a;
  __syncthreads();
  if (warp == 0) {
    a = lane < kCandThreads / 32 ? red[lane] : CandAcc{-INFINITY, -INFINITY, 0x7fffffff, 0.f};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a = cand_merge(a, cand_shfl(a, o));
    if (lane == 0) red[0] = a;
  }
  __syncthreads();
  a = red[0];
  const float mx = a.t1;
  const float log_sum = logf(a.s);  // sum_exp.ln()

  float h = 0.f;
  if (p.want_entropy) {
    // acc - p * lp over entries with p = exp(lp) > 1e-10 (compute_entropy).
    auto term = [&](float x) {
      const float lp = (x - mx) - log_sum;
      const float pr = __expf(lp);
      if (pr > 1e-10f) h -= pr * lp;
    };
    if (vec) {
      const long long n4 = n / 4;
      const float4* r4 = reinterpret_cast<const float4*>(row);
      constexpr int U = 4;
      long long i = tid;
      for (; i + (U - 1) * kCandThreads < n4; i += U * kCandThreads) {
        float4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) v[u] = __ldg(r4 + i + u * kCandThreads);
#pragma unroll
        for (int u = 0; u < U; ++u) {
          term(v[u].x);
          term(v[u].y);
          term(v[u].z);
          term(v[u].w);
        }
      }
      for (; i < n4; i += kCandThreads) {
        const float4 v = __ldg(r4 + i);
        term(v.x);
        term(v.y);
        term(v.z);
        term(v.w);
      }
    }
    for (long long i = done + tid; i < n; i += kCandThreads) term(row[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) h += __shfl_xor_sync(0xffffffffu, h, o);
    if (lane == 0) red_h[warp] = h;
    __syncthreads();
    if (tid == 0) {
      h = 0.f;
      for (int w = 0; w < kCandThreads / 32; ++w) h += red_h[w];
    }
  }
  if (tid == 0) {
    // pick_token starts from (0, -inf) with a strict >: a row with no finite
    // maximum picks token 0.
    p.token[c] = mx == -INFINITY ? 0 : a.idx;
    if (p.margin) p.margin[c] = a.t1 - a.t2;
    if (p.entropy) p.entropy[c] = p.want_entropy ? h : 0.f;
    if (p.prob) p.prob[c] = p.want_prob ? expf(a.t1 - (mx + log_sum)) : 0.f;
  }
}

}  // namespace ca
