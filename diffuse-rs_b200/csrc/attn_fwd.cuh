// attn_fwd.cuh -- bidirectional canvas attention forward for sm_100a.
//
// One CTA computes one Q tile of 128 TMEM lanes for one (sequence, kv head).
// The 128 rows are (query token, head-in-GQA-group) pairs, token-major, so a
// kv head's whole group shares one K/V stream (src/model/attention.rs:149 maps
// head h to kv head h / G). Semantics follow attention() and visible()
// (src/model/attention.rs:35-57, :106-186): per query row, softmax over every
// visible key of scale * q.k, times V; rows with no visible key give NaN.
//
// Warp roles (384 threads):
//   warp 0      TMA producer: Q once, then K tiles through an ST-stage ring
//   warp 1      TMEM allocator + tcgen05.mma issuer (one elected lane)
//   warps 2-3   prologue: build the list of key tiles that have any visible
//               (query, key) pair, flagging tiles that need per-element masks;
//               afterwards warp 3 streams V tiles through their own ring
//   warps 4-11  softmax + O correction + epilogue; TMEM lane r (= row r) is
//               shared by warps 4 + r/32 and 8 + r/32, each owning half of the
//               tile's key columns and half of O's columns
//
// Pipeline per visible key tile j (S double-buffered in TMEM, P in smem):
//   S[j&1] = Q K_j^T           (tcgen05.mma, SS, fp32 accumulate in TMEM)
//   P_j    = exp2(S*c - m)     (softmax warps, bf16 into swizzled smem)
//   O     += P_j V_j           (tcgen05.mma, SS, V read MN-major)
// The MMA warp issues S[j+1] before PV[j], so the tensor core works on the
// next tile while the softmax warps exponentiate this one. Running maxima are
// rescaled lazily: O is corrected only when a row max grows by more than 2^8,
// which is exact (the final 1/l uses the same stale max).
#pragma once

#include <climits>
#include <cstdint>

#include "sm100.cuh"

namespace ca {

constexpr int kNoWindow = INT_MAX;
constexpr int kFwdThreads = 384;  // 4 control warps + 8 softmax warps

struct FwdParams {
  void* out;
  int out_f32;
  int64_t out_row_stride;  // elements between query tokens in `out`
  int batch, sq, sk;       // uniform batch (cu_q == nullptr)
  const int* cu_q;
  const int* cu_k;
  int n_head, n_head_kv, G, hd;
  int QT;  // query tokens per tile = 128 / G
  int R;   // rows per tile = QT * G (<= 128)
  const int* q_pos;
  const int* k_pos;
  const int* q_seq;
  const int* k_seq;
  const int* q_prefix;
  int window;         // kNoWindow = None
  int causal_prefix;  // -1 = None
  float scale;
  float scale_log2;   // scale * log2(e)
  float softcap;      // 0 = off
  int any_mask;       // any of: positions, seq ids, prefixes, window, causal prefix
};

template <int HDP_, int BN_, int ST_, bool PRECISE_ = false>
struct FwdCfg {
  static constexpr int HDP = HDP_;  // head_dim padded to a multiple of 64
  static constexpr int BN = BN_;    // keys per tile
  static constexpr int ST = ST_;    // stages of each of the K and V rings
  // PRECISE: P is split into bf16 hi + lo terms (two PV MMAs), so the softmax
  // weights reach the tensor core with ~16 significant bits instead of 8.
  static constexpr bool PRECISE = PRECISE_;
  static constexpr int kPTerms = PRECISE ? 2 : 1;
  static constexpr int kChunks = HDP / 64;  // 128-byte swizzle atoms along head_dim
  static constexpr int kQChunk = 128 * 128;
  static constexpr int kKChunk = BN * 128;
  static constexpr int kPChunk = 128 * 128;
  static constexpr int kQBytes = kChunks * kQChunk;
  static constexpr int kKVBytes = kChunks * kKChunk;
  static constexpr int kPBytes = kPTerms * (BN / 64) * kPChunk;
  static constexpr int kPTermBytes = (BN / 64) * kPChunk;
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + kQBytes;
  static constexpr int kOffV = kOffK + ST * kKVBytes;
  static constexpr int kOffP = kOffV + ST * kKVBytes;
  static constexpr int kOffBar = kOffP + kPBytes;
  // Barriers. K and V stages are released separately: a K stage as soon as
  // its Q K^T MMA completes, a V stage when its P V MMA completes, so the
  // next key tile's load overlaps the current tile's softmax.
  static constexpr int kBarQ = 0;
  static constexpr int kBarK = 1;             // [ST] K tile landed
  static constexpr int kBarV = kBarK + ST;    // [ST] V tile landed
  static constexpr int kBarKE = kBarV + ST;   // [ST] K stage free
  static constexpr int kBarVE = kBarKE + ST;  // [ST] V stage free
  static constexpr int kBarS = kBarVE + ST;   // [2] S buffer holds Q K^T
  static constexpr int kBarP = kBarS + 2;     // P written (8 softmax warps)
  static constexpr int kBarO = kBarP + 1;     // P V of the latest tile done
  static constexpr int kBarF = kBarO + 1;     // all MMAs done
  static constexpr int kBarX = kBarF + 1;     // [4] softmax warp-pair exchange
  static constexpr int kNumBars = kBarX + 4;
  // Largest key-tile count per sequence (keys <= kMaxTiles * BN).
  static constexpr int kMaxTiles = (PRECISE && HDP == 256) ? 256 : 1024;
  static constexpr int kOffList = kOffBar + kNumBars * 8;
  static constexpr int kOffXch = kOffList + kMaxTiles * 2;  // float [parity][half][128]
  static constexpr int kOffMisc = kOffXch + 2 * 2 * 128 * 4;
  static constexpr int kMiscBytes = 64;
  static constexpr int kSmemBytes = kOffMisc + kMiscBytes;
  static constexpr int kTmemCols = 512;
  static constexpr int kOCol = 2 * BN;  // O accumulator columns [2BN, 2BN + HDP)
  static constexpr uint32_t kIdescS = umma_idesc_bf16(128, BN, 0, 0);
  static constexpr uint32_t kIdescO = umma_idesc_bf16(128, HDP, 0, 1);
  static_assert(kOCol + HDP <= kTmemCols, "TMEM budget");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
  static_assert(BN % 64 == 0 && BN <= 256 && HDP % 64 == 0 && HDP <= 256, "tile shape");
};

// visible(): src/model/attention.rs:35-57 on int32 positions.
__device__ __forceinline__ bool visible_dev(int qpos, int kpos, int qseq, int kseq, int window,
                                            int prefix) {
  if (qseq != kseq) return false;
  if (window != kNoWindow) {
    const long long d = static_cast<long long>(qpos) - kpos;
    if ((d < 0 ? -d : d) >= window) return false;
  }
  if (prefix >= 0 && qpos < prefix) return kpos <= qpos;
  return true;
}

__device__ __forceinline__ float u2f(uint32_t x) { return __uint_as_float(x); }
__device__ __forceinline__ uint32_t f2u(float x) { return __float_as_uint(x); }

// tanh(x) = 1 - 2 / (e^{2x} + 1), with e^{2x} = 2^{2x log2 e}; |x| clamped at
// 15 where tanh is 1 to fp32 precision. Used only by the soft-cap extension.
__device__ __forceinline__ float tanh_via_exp2(float x) {
  x = fminf(fmaxf(x, -15.f), 15.f);
  const float e = ex2_approx(x * 2.8853900817779268f);  // 2 * log2(e)
  return 1.f - __fdividef(2.f, e + 1.f);
}

}  // namespace ca

namespace ca {

// Sequence extents of batch entry b.
__device__ __forceinline__ void seq_range(const FwdParams& p, int b, int& q_beg, int& q_len,
                                          int& k_beg, int& k_len) {
  if (p.cu_q) {
    q_beg = p.cu_q[b];
    q_len = p.cu_q[b + 1] - q_beg;
  } else {
    q_beg = b * p.sq;
    q_len = p.sq;
  }
  if (p.cu_k) {
    k_beg = p.cu_k[b];
    k_len = p.cu_k[b + 1] - k_beg;
  } else {
    k_beg = b * p.sk;
    k_len = p.sk;
  }
}

// Prologue of warps 2-3: classify every key tile of the sequence against this
// CTA's query tile (0 = no visible pair, 1 = every pair visible, 2 = needs
// per-element masks) and compact the visible ones into `list` (bit 15 marks
// partial tiles). The per-tile flags are first written in place into `list`
// and then compacted; misc[1] receives the count.
template <class C>
__device__ void build_tile_list(const FwdParams& p, int q_beg, int q_len, int k_beg, int k_len,
                                int qtile, uint16_t* list, int* misc, int tid64) {
  uint16_t* flags = list;
  const int lane = tid64 & 31;
  const int w = tid64 >> 5;  // 0..1
  const int n_kt = (k_len + C::BN - 1) / C::BN;
  if (!p.any_mask) {
    for (int kt = tid64; kt < n_kt; kt += 64)
      flags[kt] = ((kt + 1) * C::BN <= k_len) ? 1 : 2;
  } else {
    // Query-tile summary over valid tokens.
    int* qs = misc + 4;  // [pos_min, pos_max, seq_min, seq_max, causal_min, n_causal, n_tok]
    if (tid64 == 0) {
      qs[0] = INT_MAX; qs[1] = INT_MIN; qs[2] = INT_MAX; qs[3] = INT_MIN;
      qs[4] = INT_MAX; qs[5] = 0; qs[6] = 0;
    }
    named_bar_sync(1, 64);
    const int t0 = qtile * p.QT;
    const int nt = min(p.QT, q_len - t0);
    for (int t = tid64; t < nt; t += 64) {
      const int tl = t0 + t;
      const int g = q_beg + tl;
      const int qp = p.q_pos ? p.q_pos[g] : tl;
      const int qsq = p.q_seq ? p.q_seq[g] : 0;
      const int pre = p.q_prefix ? p.q_prefix[g] : p.causal_prefix;
      atomicMin(&qs[0], qp); atomicMax(&qs[1], qp);
      atomicMin(&qs[2], qsq); atomicMax(&qs[3], qsq);
      if (pre >= 0 && qp < pre) { atomicMin(&qs[4], qp); atomicAdd(&qs[5], 1); }
    }
    named_bar_sync(1, 64);
    const long long qpmin = qs[0], qpmax = qs[1];
    const int qsmin = qs[2], qsmax = qs[3], cmin = qs[4];
    const bool any_causal = qs[5] > 0, all_causal = qs[5] == nt;
    for (int kt = w; kt < n_kt; kt += 2) {
      int kpmin = INT_MAX, kpmax = INT_MIN, ksmin = INT_MAX, ksmax = INT_MIN;
#pragma unroll
      for (int e = 0; e < C::BN / 32; ++e) {
        const int kl = kt * C::BN + e * 32 + lane;
        if (kl < k_len) {
          const int g = k_beg + kl;
          const int kp = p.k_pos ? p.k_pos[g] : kl;
          const int ksq = p.k_seq ? p.k_seq[g] : 0;
          kpmin = min(kpmin, kp); kpmax = max(kpmax, kp);
          ksmin = min(ksmin, ksq); ksmax = max(ksmax, ksq);
        }
      }
      kpmin = __reduce_min_sync(0xffffffffu, kpmin);
      kpmax = __reduce_max_sync(0xffffffffu, kpmax);
      ksmin = __reduce_min_sync(0xffffffffu, ksmin);
      ksmax = __reduce_max_sync(0xffffffffu, ksmax);
      if (lane == 0) {
        uint16_t f = 2;
        const bool ragged = (kt + 1) * C::BN > k_len;
        if (nt <= 0 || qsmax < ksmin || ksmax < qsmin) {
          f = 0;
        } else if (p.window != kNoWindow &&
                   (kpmin - qpmax >= p.window || qpmin - kpmax >= p.window)) {
          f = 0;
        } else if (all_causal && kpmin > qpmax) {
          f = 0;
        } else if (!ragged && qsmin == qsmax && ksmin == ksmax && qsmin == ksmin &&
                   (p.window == kNoWindow ||
                    max(qpmax - kpmin, (long long)kpmax - qpmin) < p.window) &&
                   (!any_causal || kpmax <= cmin)) {
          f = 1;
        }
        flags[kt] = f;
      }
    }
  }
  named_bar_sync(1, 64);
  if (w == 0) {
    int count = 0;
    for (int base = 0; base < n_kt; base += 32) {
      const int kt = base + lane;
      const uint16_t f = kt < n_kt ? flags[kt] : 0;
      const unsigned ball = __ballot_sync(0xffffffffu, f != 0);  // all reads precede writes
      if (f) {
        const int pos = count + __popc(ball & ((1u << lane) - 1u));
        list[pos] = static_cast<uint16_t>(kt | (f == 2 ? 0x8000 : 0));
      }
      count += __popc(ball);
    }
    if (lane == 0) misc[1] = count;
  }
}

}  // namespace ca

namespace ca {

template <class C>
__global__ void __launch_bounds__(kFwdThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                    const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const FwdParams p) {
  constexpr int BN = C::BN, HDP = C::HDP, ST = C::ST;
  // 128-byte swizzled tiles need 1024-byte aligned bases. The kernel has no
  // static shared memory, so the dynamic window starts 1024-aligned; if it
  // ever did not, report it instead of computing garbage.
  extern __shared__ __align__(1024) uint8_t smem[];
  if ((smem_u32(smem) & 1023u) != 0) {
    if (threadIdx.x == 0) atomicExch(&g_device_error, kErrLayout);
    return;
  }
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int qtile = blockIdx.x;
  const int kvh = blockIdx.y;
  const int b = blockIdx.z;

  int q_beg, q_len, k_beg, k_len;
  seq_range(p, b, q_beg, q_len, k_beg, k_len);
  if (qtile * p.QT >= q_len) return;  // uniform across the CTA

  const uint32_t sQ = smem_u32(smem + C::kOffQ);
  const uint32_t sK = smem_u32(smem + C::kOffK);
  const uint32_t sV = smem_u32(smem + C::kOffV);
  const uint32_t sP = smem_u32(smem + C::kOffP);
  const uint32_t bar0 = smem_u32(smem + C::kOffBar);
  auto bar = [&](int i) -> uint32_t { return bar0 + 8u * i; };
  uint16_t* list = reinterpret_cast<uint16_t*>(smem + C::kOffList);
  int* misc = reinterpret_cast<int*>(smem + C::kOffMisc);  // [0]=tmem base [1]=n_tiles

  if (tid == 0) {
    mbar_init(bar(C::kBarQ), 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(bar(C::kBarK + s), 1);
      mbar_init(bar(C::kBarV + s), 1);
      mbar_init(bar(C::kBarKE + s), 1);
      mbar_init(bar(C::kBarVE + s), 1);
    }
    mbar_init(bar(C::kBarS), 1);
    mbar_init(bar(C::kBarS + 1), 1);
    mbar_init(bar(C::kBarP), 8);
    mbar_init(bar(C::kBarO), 1);
    mbar_init(bar(C::kBarF), 1);
    for (int i = 0; i < 4; ++i) mbar_init(bar(C::kBarX + i), 2);
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(misc), C::kTmemCols);
    tmem_relinquish();
  }
  if (warp == 2 || warp == 3) {
    build_tile_list<C>(p, q_beg, q_len, k_beg, k_len, qtile, list, misc, tid - 64);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = static_cast<uint32_t>(misc[0]);
  const int n = misc[1];
  bool dead = false;

  if (warp == 0 || warp == 3) {
    // ------------------------------------------------------------ producers
    // Warp 0 streams Q and the K tiles, warp 3 the V tiles: the two rings
    // drain at different times (K after Q K^T, V after P V).
    if (lane == 0) {
      const bool is_k = warp == 0;
      const CUtensorMap* tm = is_k ? &tm_k : &tm_v;
      const uint32_t ring = is_k ? sK : sV;
      const int full = is_k ? C::kBarK : C::kBarV;
      const int empty = is_k ? C::kBarKE : C::kBarVE;
      if (is_k) {
        const int q_tok0 = q_beg + qtile * p.QT;
        mbar_arrive_expect_tx(bar(C::kBarQ), C::kChunks * 128u * p.R);
#pragma unroll
        for (int c = 0; c < C::kChunks; ++c)
          tma_load_3d(sQ + c * C::kQChunk, &tm_q, bar(C::kBarQ), c * 64, kvh * p.G, q_tok0);
      }
      for (int j = 0; j < n; ++j) {
        const int s = j % ST;
        if (j >= ST && !mbar_wait(bar(empty + s), ((j / ST) - 1) & 1, dead)) break;
        const int krow = k_beg + (list[j] & 0x7fff) * BN;
        mbar_arrive_expect_tx(bar(full + s), C::kKVBytes);
#pragma unroll
        for (int c = 0; c < C::kChunks; ++c)
          tma_load_3d(ring + s * C::kKVBytes + c * C::kKChunk, tm, bar(full + s), c * 64, kvh,
                      krow);
      }
      // Leave no bulk copy in flight: wait (bounded) for the last loads.
      bool d2 = false;
      if (is_k) mbar_wait(bar(C::kBarQ), 0, d2);
      for (int j = max(0, n - ST); j < n; ++j) mbar_wait(bar(full + j % ST), (j / ST) & 1, d2);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      auto issue_pv = [&](int i) -> bool {
        if (!mbar_wait(bar(C::kBarP), i & 1, dead)) return false;
        const int s = i % ST;
        if (!mbar_wait(bar(C::kBarV + s), (i / ST) & 1, dead)) return false;
        tc_fence_after();
        const uint32_t vbase = sV + s * C::kKVBytes;
#pragma unroll
        for (int term = 0; term < C::kPTerms; ++term) {
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            const uint64_t a = umma_desc_sw128(
                sP + term * C::kPTermBytes + (kk >> 2) * C::kPChunk + (kk & 3) * 32, 16, 1024);
            const uint64_t bd = umma_desc_sw128(vbase + kk * 2048, C::kKChunk, 1024);
            umma_ss(tmem + C::kOCol, a, bd, C::kIdescO, (i > 0 || kk > 0 || term > 0) ? 1u : 0u);
          }
        }
        umma_commit(bar(C::kBarO));
        umma_commit(bar(C::kBarVE + s));
        return true;
      };
      if (n > 0 && mbar_wait(bar(C::kBarQ), 0, dead)) {
        for (int j = 0; j < n; ++j) {
          const int s = j % ST;
          if (!mbar_wait(bar(C::kBarK + s), (j / ST) & 1, dead)) break;
          tc_fence_after();
          const uint32_t kbase = sK + s * C::kKVBytes;
          const uint32_t sdst = tmem + (j & 1) * BN;
#pragma unroll
          for (int kk = 0; kk < HDP / 16; ++kk) {
            const uint64_t a = umma_desc_sw128(sQ + (kk >> 2) * C::kQChunk + (kk & 3) * 32, 16, 1024);
            const uint64_t bd = umma_desc_sw128(kbase + (kk >> 2) * C::kKChunk + (kk & 3) * 32, 16, 1024);
            umma_ss(sdst, a, bd, C::kIdescS, kk > 0 ? 1u : 0u);
          }
          umma_commit(bar(C::kBarS + (j & 1)));
          umma_commit(bar(C::kBarKE + s));
          if (j >= 1 && !issue_pv(j - 1)) break;
        }
        if (!dead) issue_pv(n - 1);
      }
      // Every MMA this thread issued completes before the role ends.
      umma_commit(bar(C::kBarF));
      bool d2 = false;
      mbar_wait(bar(C::kBarF), 0, d2);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax
    // Warps w and w+4 share TMEM lane quarter wq (rows 32wq..32wq+31); `half`
    // picks which half of each tile's key columns (and of O's columns) the
    // warp owns. Row maxima and sums are combined through shared memory.
    constexpr int BH = BN / 2;   // S columns per warp
    constexpr int OH = HDP / 2;  // O columns per warp
    const int sw = warp - 4;
    const int wq = sw & 3;
    const int half = sw >> 2;
    const int r = wq * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    float* xch = reinterpret_cast<float*>(smem + C::kOffXch);  // [parity][half][128]
    const uint32_t xbar = bar(C::kBarX + wq);
    const int t_local = qtile * p.QT + r / p.G;
    const bool row_valid = r < p.R && t_local < q_len;
    const int gq = q_beg + (row_valid ? t_local : 0);
    int qpos = 0, qseq = 0, qpre = -1;
    if (row_valid && p.any_mask) {
      qpos = p.q_pos ? p.q_pos[gq] : t_local;
      qseq = p.q_seq ? p.q_seq[gq] : 0;
      qpre = p.q_prefix ? p.q_prefix[gq] : p.causal_prefix;
    }
    const float sl2 = p.scale_log2;
    const bool fast_ok = p.softcap == 0.f && sl2 >= 0.f;
    float m = -INFINITY, l = 0.f;

    for (int j = 0; j < n; ++j) {
      const int entry = list[j];
      const int kt = entry & 0x7fff;
      const bool partial = (entry & 0x8000) != 0;
      mbar_wait(bar(C::kBarS + (j & 1)), (j >> 1) & 1, dead);
      dead = __any_sync(0xffffffffu, dead);
      if (dead) break;
      tc_fence_after();
      uint32_t sr[BH];
#pragma unroll
      for (int c = 0; c < BH / 32; ++c)
        tmem_ld32(tmem + lane_off + (j & 1) * BN + half * BH + c * 32,
                  *reinterpret_cast<uint32_t(*)[32]>(&sr[c * 32]));
      tmem_wait_ld();

      // Partial row max over this warp's columns (8 independent chains: one
      // warp per SM sub-partition cannot hide a long dependent chain).
      float pmax;
      const bool fast = fast_ok && !partial;
      {
        float mx8[8];
#pragma unroll
        for (int a = 0; a < 8; ++a) mx8[a] = -INFINITY;
        if (fast) {
#pragma unroll
          for (int i = 0; i < BH; ++i) mx8[i & 7] = fmaxf(mx8[i & 7], u2f(sr[i]));
        } else {
#pragma unroll
          for (int i = 0; i < BH; ++i) {
            float t;
            if (p.softcap != 0.f) {
              const float x = u2f(sr[i]) * p.scale;
              t = p.softcap * tanh_via_exp2(x / p.softcap) * 1.4426950408889634f;
            } else {
              t = u2f(sr[i]) * sl2;
            }
            if (partial) {
              const int kl = kt * BN + half * BH + i;
              bool ok = kl < k_len;
              if (ok && p.any_mask) {
                const int g = k_beg + kl;
                const int kp = p.k_pos ? p.k_pos[g] : kl;
                const int ks = p.k_seq ? p.k_seq[g] : 0;
                ok = visible_dev(qpos, kp, qseq, ks, p.window, qpre);
              }
              if (!ok) t = -INFINITY;
            }
            sr[i] = f2u(t);
            mx8[i & 7] = fmaxf(mx8[i & 7], t);
          }
        }
        pmax = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                     fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      }
      // Exchange with the partner warp (same rows, other columns).
      xch[((j & 1) * 2 + half) * 128 + r] = pmax;
      __syncwarp();
      if (lane == 0) mbar_arrive(xbar);
      mbar_wait(xbar, j & 1, dead);
      dead = __any_sync(0xffffffffu, dead);
      if (dead) break;
      const float rmax = fmaxf(pmax, xch[((j & 1) * 2 + (half ^ 1)) * 128 + r]);
      const float mcand = fast ? rmax * sl2 : rmax;

      const bool resc = mcand > m + 8.f;
      float corr = 1.f;
      if (resc) {
        corr = ex2_approx(m - mcand);
        m = mcand;
      }
      const float mu = (m == -INFINITY) ? 0.f : m;
      float sum4[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t pk[BH / 2];
      uint32_t pl[C::PRECISE ? BH / 2 : 1];
#pragma unroll
      for (int i = 0; i < BH; i += 2) {
        float p0, p1;
        if (fast) {
          p0 = ex2_approx(fmaf(u2f(sr[i]), sl2, -mu));
          p1 = ex2_approx(fmaf(u2f(sr[i + 1]), sl2, -mu));
        } else {
          p0 = ex2_approx(u2f(sr[i]) - mu);
          p1 = ex2_approx(u2f(sr[i + 1]) - mu);
        }
        sum4[(i >> 1) & 3] += p0 + p1;
        pk[i / 2] = pack_bf16(p0, p1);
        if constexpr (C::PRECISE) {
          const float h0 = __uint_as_float(pk[i / 2] << 16);
          const float h1 = __uint_as_float(pk[i / 2] & 0xffff0000u);
          pl[i / 2] = pack_bf16(p0 - h0, p1 - h1);
        }
      }
      l = l * corr + ((sum4[0] + sum4[1]) + (sum4[2] + sum4[3]));

      // P's buffer and O are free once P V of the previous tile completed.
      if (j > 0) {
        mbar_wait(bar(C::kBarO), (j - 1) & 1, dead);
        dead = __any_sync(0xffffffffu, dead);
        if (dead) break;
        tc_fence_after();
        if (__any_sync(0xffffffffu, resc)) {
#pragma unroll 1
          for (int c = 0; c < OH / 32; ++c) {
            uint32_t o[32];
            const uint32_t ta = tmem + lane_off + C::kOCol + half * OH + c * 32;
            tmem_ld32(ta, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = f2u(u2f(o[i]) * corr);
            tmem_st32(ta, o);
          }
          tmem_wait_st();
        }
      }
      // P row r: 128-byte rows of 64 keys, 16-byte units XOR-swizzled by (r & 7).
#pragma unroll
      for (int u = 0; u < BH / 8; ++u) {
        const int key0 = half * BH + u * 8;
        const uint32_t addr =
            sP + (key0 >> 6) * C::kPChunk + r * 128 + ((((key0 & 63) >> 3) ^ (r & 7)) << 4);
        st_shared_v4(addr, pk[u * 4], pk[u * 4 + 1], pk[u * 4 + 2], pk[u * 4 + 3]);
        if constexpr (C::PRECISE)
          st_shared_v4(addr + C::kPTermBytes, pl[u * 4], pl[u * 4 + 1], pl[u * 4 + 2],
                       pl[u * 4 + 3]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(C::kBarP));
    }

    // ------------------------------------------------------------ epilogue
    bool have_o = n > 0 && !dead;
    if (have_o) {
      mbar_wait(bar(C::kBarO), (n - 1) & 1, dead);
      dead = __any_sync(0xffffffffu, dead);
      have_o = !dead;
      tc_fence_after();
    }
    if (have_o) {  // row sum = both halves' partial sums (same running max)
      xch[((n & 1) * 2 + half) * 128 + r] = l;
      __syncwarp();
      if (lane == 0) mbar_arrive(xbar);
      mbar_wait(xbar, n & 1, dead);
      dead = __any_sync(0xffffffffu, dead);
      have_o = !dead;
      l += xch[((n & 1) * 2 + (half ^ 1)) * 128 + r];
    }
    const float inv = have_o ? 1.f / l : __int_as_float(0x7fc00000);
    const int head = kvh * p.G + (r % p.G);
#pragma unroll 1
    for (int c = 0; c < OH / 32; ++c) {
      uint32_t o[32];
      if (have_o) {
        tmem_ld32(tmem + lane_off + C::kOCol + half * OH + c * 32, o);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = 0u;
      }
      if (row_valid) {
        const int64_t obase = static_cast<int64_t>(gq) * p.out_row_stride +
                              static_cast<int64_t>(head) * p.hd;
#pragma unroll
        for (int g8 = 0; g8 < 4; ++g8) {
          const int col = half * OH + c * 32 + g8 * 8;
          if (col < p.hd) {
            float v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = have_o ? u2f(o[g8 * 8 + i]) * inv : inv;
            if (p.out_f32) {
              float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + obase + col);
              dst[0] = make_float4(v[0], v[1], v[2], v[3]);
              dst[1] = make_float4(v[4], v[5], v[6], v[7]);
            } else {
              uint4 w;
              w.x = pack_bf16(v[0], v[1]);
              w.y = pack_bf16(v[2], v[3]);
              w.z = pack_bf16(v[4], v[5]);
              w.w = pack_bf16(v[6], v[7]);
              *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.out) + obase + col) = w;
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

}  // namespace ca
