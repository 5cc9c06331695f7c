// attn_fwd.cuh -- bidirectional canvas attention forward for sm_100a.
//
// One CTA computes one Q tile of 128 TMEM lanes for one (sequence, kv head).
// The 128 rows are (query token, head-in-GQA-group) pairs, token-major, so a
// kv head's whole group shares one K/V stream (src/model/attention.rs:149 maps
// head h to kv head h / G). Semantics follow attention() and visible()
// (src/model/attention.rs:35-57, :106-186): per query row, softmax over every
// visible key of scale * q.k, times V; rows with no visible key give NaN.
//
// Warp roles (352 threads, one CTA per SM):
//   warp 0      TMA producer of Q and the K ring (lane 0)
//   warp 1      TMEM allocator + tcgen05.mma issuer (lane 0)
//   warp 2      TMA producer of the V ring (lane 0)
//   warps 0-1   prologue: build the list of key tiles that have any visible
//               (query, key) pair, flagging tiles that need per-element masks
//   warps 3-10  softmax, O correction and epilogue in two groups of four
//               warps (3-6 and 7-10); warp w reaches TMEM lanes 32 (w % 4)..+31
//
// Pipeline per visible key tile j (S double-buffered in TMEM; P in TMEM too):
//   S[j&1] = Q K_j^T           (tcgen05.mma, SS, fp32 accumulate in TMEM)
//   P_j    = exp2(S*c - m)     (softmax warps, bf16 written over S[j&1])
//   O     += P_j V_j           (tcgen05.mma, TS: P from TMEM, V MN-major smem)
// Keeping P out of shared memory matters: while SS MMAs stream their operands
// at N = 128, ordinary shared-memory stores from other warps barely progress.
// Two softmax groups take alternate key tiles (or, head_dim 256, halves of
// each tile), so one group exponentiates while the tensor core runs the other
// group's MMAs. Running maxima are rescaled lazily: O is corrected only when a
// row max grows by more than 2^8, which is exact (the final 1/l uses the same
// stale max).
#pragma once

#include <climits>
#include <cstdint>
#include <type_traits>

#include "sm100.cuh"

namespace ca {

constexpr int kNoWindow = INT_MAX;

constexpr int kMaxPeers = 7;  // other GPUs of one 8-GPU box

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
  const int* seq_prefix;  // per-sequence causal prefix [batch] (when q_prefix is null)
  int window;         // kNoWindow = None
  int causal_prefix;  // -1 = None
  float scale;
  float scale_log2;   // scale * log2(e)
  float softcap;      // 0 = off
  int tma_out;        // uniform batch: the epilogue stores O through tm_o
  // Fused Q pre-ops (head_dim 128, rotation over the full head): the Q tile
  // is loaded pre-norm, pre-RoPE and the softmax warps apply the per-head
  // RMSNorm (gains fq_w, may be null) and NeoX RoPE (table fq_rope, entry
  // (pos, i) at 2 (pos * 64 + i)) in shared memory before the first Q K^T.
  int fuse_q;
  const float* fq_w;
  const float* fq_rope;
  float fq_eps;
  int any_mask;       // any of: seq ids, prefixes, window, causal prefix (positions
                      // alone mask nothing: they matter only to those masks)
  int* err;           // device status word of this launch (null: g_device_error)
  // Other GPUs' output buffers mapped into this process (same layout and
  // strides as `out`): the epilogue stores every output row there as well,
  // over NVLink, so a head-sharded layer's rows reach each rank's full
  // [tokens, n_head, head_dim] buffer as the tiles finish.
  void* peer_out[kMaxPeers];
  int n_peer;
  // NVLink multicast address bound to `out` on every rank (same offsets):
  // the uniform-batch epilogue writes the staged tile through it with
  // multimem stores instead of storing to `out` (the switch delivers each
  // row to every rank's buffer, this one's included).
  void* mc_out;
};

// Softmax organisation of a CTA (see the file comment):
//   kSplit  both warp groups see every key tile, each on half of its key
//           columns and half of O (head_dim 256: TMEM holds one O)
//   kAlt    group g takes key tiles g, g+2, ... with its own S/P buffer and
//           O, merged at the end (head_dim <= 192)
//   kOne    one softmax group (four warps) taking every key tile, S double-
//           buffered, one O; half the TMEM and about half the shared memory
//           of kAlt, so two CTAs share an SM and one's prologue and epilogue
//           overlap the other's main loop (head_dim 128, 64-key tiles)
enum FwdMode { kSplit = 0, kAlt = 1, kOne = 3 };


template <int HDP_, int BN_, int ST_, bool PRECISE_, int MODE_, int STK_ = ST_, int KSUB_ = 1,
          int VSUB_ = 1, int OS_ = 1>
struct FwdCfg {
  static constexpr int HDP = HDP_;  // head_dim padded to a multiple of 64
  static constexpr int BN = BN_;    // keys per tile
  static constexpr int ST = ST_;    // stages of the V ring
  static constexpr int STK = STK_;  // stages of the K ring (Q K^T waits on K first)
  // PRECISE: P is split into bf16 hi + lo terms (two P V MMAs), so the
  // softmax weights reach the tensor core with ~16 significant bits, not 8.
  static constexpr bool PRECISE = PRECISE_;
  static constexpr int MODE = MODE_;
  static constexpr bool ALT = MODE == kAlt;
  static constexpr bool SPLIT = MODE == kSplit;
  static constexpr bool ONE = MODE == kOne;
  static constexpr int kGroups = ONE ? 1 : 2;                // softmax groups of four warps
  static constexpr int kSoftThreads = 128 * kGroups;
  static constexpr int kThreads = 96 + kSoftThreads;         // + 3 control warps
  static constexpr int kMinBlocks = ONE ? 2 : 1;             // CTAs per SM
  static constexpr int kPTerms = PRECISE ? 2 : 1;
  // Wide heads (head_dim > 256): OS CTAs share one Q tile, each computing
  // S = Q K^T over the whole head and owning HDO = HDP / OS columns of O
  // (an fp32 O of 512 columns would fill TMEM). K tiles then stream as KSUB
  // units of HDP / KSUB dims and V tiles as VSUB units of BN / VSUB keys, so
  // that the whole Q tile stays resident beside rings of several units.
  static constexpr int OS = OS_;
  static constexpr int HDO = HDP / OS;  // O columns of this CTA
  static constexpr int KSUB = KSUB_;
  static constexpr int VSUB = VSUB_;
  // S buffers in TMEM (P overwrites S in place). kSplit keeps one O, which
  // leaves room for a third buffer: S runs two tiles ahead of the softmax.
  static constexpr int SB = SPLIT ? 3 : 2;
  static constexpr int kChunks = HDP / 64;  // 128-byte swizzle atoms along head_dim
  static constexpr int kQChunk = 128 * 128;
  static constexpr int kKChunk = BN * 128;
  static constexpr int kQBytes = kChunks * kQChunk;
  static constexpr int kKUnitChunks = kChunks / KSUB;   // atoms per K unit
  static constexpr int kKUnitBytes = kKUnitChunks * kKChunk;
  static constexpr int kVRows = BN / VSUB;              // keys per V unit
  static constexpr int kVChunk = kVRows * 128;
  static constexpr int kOChunks = HDO / 64;             // V atoms this CTA reads
  static constexpr int kVUnitBytes = kOChunks * kVChunk;
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + kQBytes;
  static constexpr int kOffV = kOffK + STK * kKUnitBytes;
  static constexpr int kOffBar = kOffV + ST * kVUnitBytes;
  // Barriers. K and V stages are released separately: a K stage as soon as
  // its Q K^T MMA completes, a V stage when its P V MMA(s) complete.
  static constexpr int kBarQ = 0;
  static constexpr int kBarK = 1;             // [STK] K unit landed
  static constexpr int kBarV = kBarK + STK;   // [ST] V unit landed
  static constexpr int kBarKE = kBarV + ST;   // [STK] K stage free
  static constexpr int kBarVE = kBarKE + STK; // [ST] V stage free
  static constexpr int kBarS = kBarVE + ST;   // [SB] S buffer holds Q K^T
  static constexpr int kBarP = kBarS + SB;    // [2] P written over S (per group)
  static constexpr int kBarO = kBarP + 2;     // [2] P V done (per O accumulator)
  static constexpr int kBarF = kBarO + 2;     // all MMAs done
  static constexpr int kBarX = kBarF + 1;     // [4] softmax warp-pair exchange
  static constexpr int kBarQR = kBarX + 4;    // fused Q pre-ops done
  static constexpr int kNumBars = kBarQR + 1;
  // Largest key-tile count per sequence (keys <= kMaxTiles * BN).
  static constexpr int kMaxTiles = 1024;
  static constexpr int kOffList = kOffBar + kNumBars * 8;
  // Warp-pair exchange, float [parity][half][128]: kSplit's per-tile row
  // maxima and the epilogue's partial (max, sum) of each group.
  static constexpr int kXchBytes = 2 * 2 * 128 * 4;
  static constexpr int kOffXch = kOffList + kMaxTiles * 2;
  static constexpr int kOffMisc = kOffXch + kXchBytes;
  static constexpr int kMiscBytes = 64;
  static constexpr int kSmemBytes = kOffMisc + kMiscBytes;
  static constexpr int kTmemCols = ONE ? 256 : 512;
  static constexpr int kOCol = SB * BN;  // O accumulator(s) after the S buffers
  static constexpr uint32_t kIdescS = umma_idesc_bf16(128, BN, 0, 0);
  static constexpr uint32_t kIdescO = umma_idesc_bf16(128, HDO, 0, 1);
  static_assert(kOCol + (ALT ? 2 : 1) * HDO <= kTmemCols, "TMEM budget");
  static_assert(!ONE || (OS == 1 && KSUB == 1 && VSUB == 1), "one group: whole-tile units");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
  static_assert(BN % 64 == 0 && BN <= 256 && HDP % 64 == 0 && HDP <= 512, "tile shape");
  static_assert(HDO % 64 == 0 && HDO <= 256 && kChunks % KSUB == 0 && BN % (16 * VSUB) == 0,
                "unit shape");
  static_assert(OS == 1 || SPLIT, "wide heads use the split softmax");
  // The epilogue stages the output tile (up to fp32) in shared memory that
  // is idle by then: the K/V rings, or for wide heads the Q tile.
  static constexpr int kStageChunk = 128 * 128;  // one 128-byte column chunk, 128 rows
  static constexpr int kOffStage = OS > 1 ? kOffQ : kOffK;
  static constexpr int kStageBytes = OS > 1 ? kQBytes : STK * kKUnitBytes + ST * kVUnitBytes;
  static_assert(128 * HDO * 4 <= kStageBytes, "output staging fits in idle shared memory");
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

// Blackwell packed / three-input forms for the softmax inner loops
// (sm_100: fma.rn.f32x2 / add.f32x2 through __ffma2_rn / __fadd2_rn, and the
// three-operand max.f32 of PTX 8.8).
#ifndef CA_F32X2
#define CA_F32X2 1
#endif
#ifndef CA_MAX3
#define CA_MAX3 1
#endif
#ifndef CA_TANH2
#define CA_TANH2 1
#endif
// In the head_dim <= 192 (kAlt) kernel, every CA_POLY_EVERY-th key pair of
// unmasked, uncapped tiles takes its exponentials on the FMA pipe
// (ex2_poly3x2) instead of MUFU; 0 = never. Measured on B200: 1 in 8 pairs
// c3 +0.4%, c2 +1.2%; 1 in 4 c3 -4.5%; the kSplit kernel loses 1.7% at 1 in 8.
#ifndef CA_POLY_EVERY
#define CA_POLY_EVERY 8
#endif
constexpr int kPolyEvery = CA_POLY_EVERY > 0 ? CA_POLY_EVERY : 1;
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ float u2f(uint32_t x) { return __uint_as_float(x); }
__device__ __forceinline__ uint32_t f2u(float x) { return __float_as_uint(x); }

// tanh(x) = 1 - 2 / (e^{2x} + 1), with e^{2x} = 2^{2x log2 e}; |x| clamped at
// 15 where tanh is 1 to fp32 precision. Used only by the soft-cap extension;
// the exponential runs on the FMA pipe (ex2_poly) to spare the MUFU unit.
__device__ __forceinline__ float tanh_via_exp2(float x) {
  x = fminf(fmaxf(x, -15.f), 15.f);
  const float e = ex2_poly(x * 2.8853900817779268f);  // 2 * log2(e)
  return 1.f - __fdividef(2.f, e + 1.f);
}

// tanh(u) = u * P(u^2) for |u| <= kTanhPolyMax: P of degree 5 in u^2,
// weighted least squares (relative error) on Chebyshev nodes in u^2, fitted
// for this kernel; max abs error 5.3e-8 and max relative error 1.0e-7 in
// float32 Horner evaluation. No MUFU op. Used for soft-cap tiles whose
// scaled scores all lie in range (with QK-norm, nearly every tile).
constexpr float kTanhPolyMax = 0.625f;
constexpr float kTanhC1 = -0.3333325982093811f;
constexpr float kTanhC2 = 0.13331091403961182f;
constexpr float kTanhC3 = -0.053718484938144684f;
constexpr float kTanhC4 = 0.020583488047122955f;
constexpr float kTanhC5 = -0.005652355030179024f;
__device__ __forceinline__ float tanh_poly(float u) {
  const float w = u * u;
  float p = fmaf(kTanhC5, w, kTanhC4);
  p = fmaf(p, w, kTanhC3);
  p = fmaf(p, w, kTanhC2);
  p = fmaf(p, w, kTanhC1);
  p = fmaf(p, w, 1.f);
  return u * p;
}

// tanh_poly on two values at once with packed f32x2 FMAs (same operations
// in the same order, so the same results as two tanh_poly calls).
__device__ __forceinline__ float2 tanh_poly2(float2 u) {
  const float2 w = __fmul2_rn(u, u);
  float2 p = __ffma2_rn(make_float2(kTanhC5, kTanhC5), w, make_float2(kTanhC4, kTanhC4));
  p = __ffma2_rn(p, w, make_float2(kTanhC3, kTanhC3));
  p = __ffma2_rn(p, w, make_float2(kTanhC2, kTanhC2));
  p = __ffma2_rn(p, w, make_float2(kTanhC1, kTanhC1));
  p = __ffma2_rn(p, w, make_float2(1.f, 1.f));
  return __fmul2_rn(u, p);
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

// Prologue of warps 0-1: classify every key tile of the sequence against this
// CTA's query rows (0 = no visible pair, 1 = every pair visible, 2 = needs
// per-element masks, 3 = ragged end only: every pair of its valid keys
// visible) and compact the visible ones into `list` (kind in bits 14-15). The per-tile flags are first written in place into `list`
// and then compacted; misc[1] receives the count.
template <class C>
__device__ void build_tile_list(const FwdParams& p, int b, int q_beg, int q_len, int k_beg,
                                int k_len, int t0, int span, uint16_t* list, int* misc,
                                int tid64) {
  uint16_t* flags = list;
  const int lane = tid64 & 31;
  const int w = tid64 >> 5;  // 0..1
  const int n_kt = (k_len + C::BN - 1) / C::BN;
  if (!p.any_mask) {
    for (int kt = tid64; kt < n_kt; kt += 64)
      flags[kt] = ((kt + 1) * C::BN <= k_len) ? 1 : 3;
  } else {
    // Query-tile summary over valid tokens.
    int* qs = misc + 4;  // [pos_min, pos_max, seq_min, seq_max, causal_min, n_causal, n_tok]
    if (tid64 == 0) {
      qs[0] = INT_MAX; qs[1] = INT_MIN; qs[2] = INT_MAX; qs[3] = INT_MIN;
      qs[4] = INT_MAX; qs[5] = 0; qs[6] = 0;
    }
    named_bar_sync(1, 64);
    const int nt = min(span, q_len - t0);  // query tokens of this CTA
    // Per-thread partials, one warp reduction each, one shared atomic per
    // warp (the loads of all tokens are independent and overlap).
    int pmin = INT_MAX, pmax = INT_MIN, smin = INT_MAX, smax = INT_MIN, cpmin = INT_MAX, ncaus = 0;
    for (int t = tid64; t < nt; t += 64) {
      const int tl = t0 + t;
      const int g = q_beg + tl;
      const int qp = p.q_pos ? p.q_pos[g] : tl;
      const int qsq = p.q_seq ? p.q_seq[g] : 0;
      const int pre = p.q_prefix ? p.q_prefix[g]
                                 : p.seq_prefix ? p.seq_prefix[b] : p.causal_prefix;
      pmin = min(pmin, qp); pmax = max(pmax, qp);
      smin = min(smin, qsq); smax = max(smax, qsq);
      if (pre >= 0 && qp < pre) { cpmin = min(cpmin, qp); ++ncaus; }
    }
    pmin = __reduce_min_sync(0xffffffffu, pmin);
    pmax = __reduce_max_sync(0xffffffffu, pmax);
    smin = __reduce_min_sync(0xffffffffu, smin);
    smax = __reduce_max_sync(0xffffffffu, smax);
    cpmin = __reduce_min_sync(0xffffffffu, cpmin);
    ncaus = __reduce_add_sync(0xffffffffu, ncaus);
    if (lane == 0) {
      atomicMin(&qs[0], pmin); atomicMax(&qs[1], pmax);
      atomicMin(&qs[2], smin); atomicMax(&qs[3], smax);
      atomicMin(&qs[4], cpmin); atomicAdd(&qs[5], ncaus);
    }
    named_bar_sync(1, 64);
    const long long qpmin = qs[0], qpmax = qs[1];
    const int qsmin = qs[2], qsmax = qs[3], cmin = qs[4];
    const bool any_causal = qs[5] > 0, all_causal = qs[5] == nt;
    // Keys with implicit positions (index = position) and no sequence ids:
    // a tile's position range is arithmetic, so each thread classifies whole
    // tiles with no loads or warp reductions (the sliding-window case).
    const bool implicit_k = !p.k_pos && !p.k_seq;
    for (int kt = implicit_k ? tid64 : n_kt; kt < n_kt; kt += 64) {
      const int kpmin = kt * C::BN, kpmax = min(k_len, (kt + 1) * C::BN) - 1;
      const bool ragged = (kt + 1) * C::BN > k_len;
      uint16_t f = 2;
      if (nt <= 0 || qsmax < 0 || 0 < qsmin) {
        f = 0;
      } else if (p.window != kNoWindow &&
                 (kpmin - qpmax >= p.window || qpmin - kpmax >= p.window)) {
        f = 0;
      } else if (all_causal && kpmin > qpmax) {
        f = 0;
      } else if (qsmin == qsmax && qsmin == 0 &&
                 (p.window == kNoWindow ||
                  max(qpmax - kpmin, (long long)kpmax - qpmin) < p.window) &&
                 (!any_causal || kpmax <= cmin)) {
        f = ragged ? 3 : 1;
      }
      flags[kt] = f;
    }
    for (int kt = implicit_k ? n_kt : w; kt < n_kt; kt += 2) {
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
        } else if (qsmin == qsmax && ksmin == ksmax && qsmin == ksmin &&
                   (p.window == kNoWindow ||
                    max(qpmax - kpmin, (long long)kpmax - qpmin) < p.window) &&
                   (!any_causal || kpmax <= cmin)) {
          f = ragged ? 3 : 1;  // every pair visible among the tile's valid keys
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
        // Bits 14-15: 0 every pair visible, 1 only the first (k_len - kt*BN)
        // keys valid (ragged end, all visible), 2 per-element masks needed.
        list[pos] = static_cast<uint16_t>(kt | (f == 2 ? 2 << 14 : f == 3 ? 1 << 14 : 0));
      }
      count += __popc(ball);
    }
    if (lane == 0) misc[1] = count;
  }
}

}  // namespace ca

namespace ca {

// Fused Q pre-ops, run by the softmax threads once the raw Q tile has
// landed. With two softmax groups (256 threads) thread tt owns row tt / 2 and
// the NeoX pairs (i, i + 64) for i in 32 (tt & 1) .. +31; with one group (128
// threads) thread tt owns the whole row tt. A thread's columns are 16-byte
// units of both 64-column chunks of the 128-byte-swizzled tile (unit u of row
// r sits at u ^ (r & 7)). Arithmetic is that of the pre-ops kernel
// (norm_heads / rms_norm_inplace, src/model/ops.rs:107-114, 385-389;
// rotate_rows :432-452): f32 squares summed in f64 (exact for bf16 inputs;
// the two 32-column halves' sums are added last in both forms, so both give
// the same bits), scale = 1 / (float)sqrt(ss / 128 + eps), x * scale * w,
// then (a, b) -> (a cos - b sin, a sin + b cos), rounded to bf16 in place.
// The writes are fenced for the tensor core's (async) proxy, the softmax
// threads meet at a named barrier and one arrival releases the first Q K^T.
template <class C>
__device__ __forceinline__ void fuse_q_prep(const FwdParams& p, uint32_t sQ, uint32_t bar_q,
                                            uint32_t bar_qr, int t0, int q_beg, int q_len,
                                            int tt, bool& dead) {
  constexpr int TPR = C::ONE ? 1 : 2;  // threads per Q row
  constexpr int NH = 2 / TPR;          // 32-column halves per thread
  mbar_wait(bar_q, 0, dead, p.err);
  const int r = tt / TPR, h0 = tt % TPR;
  const int t_local = t0 + r / p.G;
  const bool valid = !dead && r < p.R && t_local < q_len;
  // Four 16-byte units per chunk and half: units 4h .. 4h + 3 (columns
  // 32h .. 32h + 31).
  uint32_t lo[NH][16], hi[NH][16];
  const uint32_t row_lo = sQ + r * 128, row_hi = sQ + C::kQChunk + r * 128;
#pragma unroll
  for (int hh = 0; hh < NH; ++hh)
#pragma unroll
    for (int i = 0; i < 16; ++i) lo[hh][i] = hi[hh][i] = 0u;
  if (valid) {
#pragma unroll
    for (int hh = 0; hh < NH; ++hh) {
      const int h = h0 + hh;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint32_t off = static_cast<uint32_t>(((4 * h + u) ^ (r & 7)) << 4);
        asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(lo[hh][4 * u]), "=r"(lo[hh][4 * u + 1]), "=r"(lo[hh][4 * u + 2]),
                       "=r"(lo[hh][4 * u + 3])
                     : "r"(row_lo + off));
        asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(hi[hh][4 * u]), "=r"(hi[hh][4 * u + 1]), "=r"(hi[hh][4 * u + 2]),
                       "=r"(hi[hh][4 * u + 3])
                     : "r"(row_hi + off));
      }
    }
  }
  double sh[NH];
#pragma unroll
  for (int hh = 0; hh < NH; ++hh) {
    double ss = 0.0;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float a0 = __uint_as_float(lo[hh][i] << 16);
      const float a1 = __uint_as_float(lo[hh][i] & 0xffff0000u);
      const float b0 = __uint_as_float(hi[hh][i] << 16);
      const float b1 = __uint_as_float(hi[hh][i] & 0xffff0000u);
      ss += static_cast<double>(__fmul_rn(a0, a0));
      ss += static_cast<double>(__fmul_rn(a1, a1));
      ss += static_cast<double>(__fmul_rn(b0, b0));
      ss += static_cast<double>(__fmul_rn(b1, b1));
    }
    sh[hh] = ss;
  }
  double ss;
  if constexpr (TPR == 2) ss = sh[0] + __shfl_xor_sync(0xffffffffu, sh[0], 1);  // other half
  else ss = sh[0] + sh[NH - 1];
  if (valid) {
    const int pos = p.q_pos ? p.q_pos[q_beg + t_local] : t_local;
    const bool norm = p.fq_w != nullptr;
    const float sc =
        __fdiv_rn(1.f, static_cast<float>(sqrt(ss / 128.0 + static_cast<double>(p.fq_eps))));
#pragma unroll
    for (int hh = 0; hh < NH; ++hh) {
      const int h = h0 + hh;
      const float* cs_row = p.fq_rope + 2 * (static_cast<long long>(pos) * 64 + 32 * h);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        float a[2] = {__uint_as_float(lo[hh][i] << 16), __uint_as_float(lo[hh][i] & 0xffff0000u)};
        float b[2] = {__uint_as_float(hi[hh][i] << 16), __uint_as_float(hi[hh][i] & 0xffff0000u)};
        const float4 t = __ldg(reinterpret_cast<const float4*>(cs_row) + i);  // (sin, cos) x 2
        const float sn[2] = {t.x, t.z}, cs[2] = {t.y, t.w};
        float ya[2], yb[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int col = 32 * h + 2 * i + e;
          if (norm) {
            a[e] = __fmul_rn(__fmul_rn(a[e], sc), __ldg(p.fq_w + col));
            b[e] = __fmul_rn(__fmul_rn(b[e], sc), __ldg(p.fq_w + 64 + col));
          }
          ya[e] = __fsub_rn(__fmul_rn(a[e], cs[e]), __fmul_rn(b[e], sn[e]));
          yb[e] = __fadd_rn(__fmul_rn(a[e], sn[e]), __fmul_rn(b[e], cs[e]));
        }
        lo[hh][i] = pack_bf16(ya[0], ya[1]);
        hi[hh][i] = pack_bf16(yb[0], yb[1]);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint32_t off = static_cast<uint32_t>(((4 * h + u) ^ (r & 7)) << 4);
        st_shared_v4(row_lo + off, lo[hh][4 * u], lo[hh][4 * u + 1], lo[hh][4 * u + 2],
                     lo[hh][4 * u + 3]);
        st_shared_v4(row_hi + off, hi[hh][4 * u], hi[hh][4 * u + 1], hi[hh][4 * u + 2],
                     hi[hh][4 * u + 3]);
      }
    }
  }
  fence_proxy_async_smem();
  named_bar_sync(3, C::kSoftThreads);
  if (tt == 0) mbar_arrive(bar_qr);
}

// Output tensor maps of the peer buffers (same shape as tm_o), used when the
// epilogue stores through TMA: the bulk copies to other GPUs run on the TMA
// engine after the tile is staged, so the CTA does not wait on NVLink.
struct PeerMaps {
  CUtensorMap m[kMaxPeers];
};

// Stores one 16-byte unit of an output row at element offset `off` of every
// peer buffer (plain st.global over NVLink; peers are never read here). Used
// by the row-store epilogue (variable-length batches).
__device__ __forceinline__ void store_peers(const FwdParams& p, int64_t off, uint4 w) {
#pragma unroll 1
  for (int i = 0; i < p.n_peer; ++i) {
    char* base = static_cast<char*>(p.peer_out[i]);
    *reinterpret_cast<uint4*>(base + off * (p.out_f32 ? 4 : 2)) = w;
  }
}

template <class C>
__global__ void __launch_bounds__(C::kThreads, C::kMinBlocks)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                    const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v,
                    const __grid_constant__ CUtensorMap tm_o, const FwdParams p,
                    const __grid_constant__ PeerMaps pm) {
  constexpr int BN = C::BN, HDP = C::HDP, ST = C::ST, STK = C::STK;
  constexpr bool ALT = C::ALT, SPLIT = C::SPLIT, ONE = C::ONE;
  // 128-byte swizzled tiles need 1024-byte aligned bases. The kernel has no
  // static shared memory, so the dynamic window starts 1024-aligned; if it
  // ever did not, report it instead of computing garbage.
  extern __shared__ __align__(1024) uint8_t smem[];
  if ((smem_u32(smem) & 1023u) != 0) {
    if (threadIdx.x == 0) atomicExch(p.err ? p.err : &g_device_error, kErrLayout);
    return;
  }
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int qtile = blockIdx.x / C::OS;  // query tile
  const int ohalf = blockIdx.x % C::OS;  // which HDO columns of O (wide heads)
  const int kvh = blockIdx.y;
  const int b = blockIdx.z;

  int q_beg, q_len, k_beg, k_len;
  seq_range(p, b, q_beg, q_len, k_beg, k_len);
  const int t0 = qtile * p.QT;  // first query token of this CTA
  if (t0 >= q_len) return;           // uniform across the CTA

  const uint32_t sQ = smem_u32(smem + C::kOffQ);
  const uint32_t sK = smem_u32(smem + C::kOffK);
  const uint32_t sV = smem_u32(smem + C::kOffV);
  const uint32_t bar0 = smem_u32(smem + C::kOffBar);
  auto bar = [&](int i) -> uint32_t { return bar0 + 8u * i; };
  uint16_t* list = reinterpret_cast<uint16_t*>(smem + C::kOffList);
  int* misc = reinterpret_cast<int*>(smem + C::kOffMisc);  // [0]=tmem base [1]=n_tiles
  // K unit u (tile u / KSUB, head_dim atoms of part u % KSUB) of the tile at
  // key row `row`, into K stage s; V unit u (keys (u % VSUB) * kVRows.. of
  // the tile, this CTA's HDO columns) into V stage s.
  auto load_k_unit = [&](int u, int s, int row) {
    const int part = u % C::KSUB;
    mbar_arrive_expect_tx(bar(C::kBarK + s), C::kKUnitBytes);
#pragma unroll
    for (int c = 0; c < C::kKUnitChunks; ++c)
      tma_load_3d(sK + s * C::kKUnitBytes + c * C::kKChunk, &tm_k, bar(C::kBarK + s),
                  (part * C::kKUnitChunks + c) * 64, kvh, row);
  };
  auto load_v_unit = [&](int u, int s, int row) {
    const int part = u % C::VSUB;
    mbar_arrive_expect_tx(bar(C::kBarV + s), C::kVUnitBytes);
#pragma unroll
    for (int c = 0; c < C::kOChunks; ++c)
      tma_load_3d(sV + s * C::kVUnitBytes + c * C::kVChunk, &tm_v, bar(C::kBarV + s),
                  ohalf * C::HDO + c * 64, kvh, row + part * C::kVRows);
  };

  if (tid == 0) {
    mbar_init(bar(C::kBarQ), 1);
    for (int s = 0; s < STK; ++s) {
      mbar_init(bar(C::kBarK + s), 1);
      mbar_init(bar(C::kBarKE + s), 1);
    }
    for (int s = 0; s < ST; ++s) {
      mbar_init(bar(C::kBarV + s), 1);
      mbar_init(bar(C::kBarVE + s), 1);
    }
    for (int i = 0; i < C::SB; ++i) mbar_init(bar(C::kBarS + i), 1);
    for (int g = 0; g < 2; ++g) {
      mbar_init(bar(C::kBarP + g), SPLIT ? 8 : 4);
      mbar_init(bar(C::kBarO + g), 1);
    }
    mbar_init(bar(C::kBarF), 1);
    for (int i = 0; i < 4; ++i) mbar_init(bar(C::kBarX + i), 2);
    mbar_init(bar(C::kBarQR), 1);
    fence_barrier_init();
    fence_proxy_async_smem();
    // Q does not depend on the tile list: start its load right away.
    mbar_arrive_expect_tx(bar(C::kBarQ), C::kChunks * 128u * p.R);
#pragma unroll
    for (int c = 0; c < C::kChunks; ++c)
      tma_load_3d(sQ + c * C::kQChunk, &tm_q, bar(C::kBarQ), c * 64, kvh * p.G, q_beg + t0);
    // Without masks the visible tiles are 0, 1, 2, ...: the first ring
    // stages of K and V load now too, overlapping the tile list and the
    // TMEM allocation (the producers continue from stage STK / ST).
    if (!p.any_mask) {
      const int n_kt = (k_len + BN - 1) / BN;
      const int ek = min(STK, n_kt * C::KSUB), ev = min(ST, n_kt * C::VSUB);
      for (int u = 0; u < ek || u < ev; ++u) {
        if (u < ek) load_k_unit(u, u, k_beg + (u / C::KSUB) * BN);
        if (u < ev) load_v_unit(u, u, k_beg + (u / C::VSUB) * BN);
      }
    }
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(misc), C::kTmemCols);
    tmem_relinquish();
  }
  if (warp <= 1)
    build_tile_list<C>(p, b, q_beg, q_len, k_beg, k_len, t0, p.QT, list, misc, tid);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = static_cast<uint32_t>(misc[0]);
  const int n = misc[1];
  bool dead = false;

  if (warp == 0 || warp == 2) {
    // ------------------------------------------------------------ producers
    // Warp 0 streams Q and the K tiles, warp 2 the V tiles. The two rings
    // drain at different times (K after Q K^T, V after P V); as two lanes of
    // one warp their diverged waits delayed each other's loads.
    if (lane == 0) {
      const bool is_k = warp == 0;
      const int full = is_k ? C::kBarK : C::kBarV;
      const int empty = is_k ? C::kBarKE : C::kBarVE;
      const int NS = is_k ? STK : ST;              // stages of this ring
      const int SUB = is_k ? C::KSUB : C::VSUB;    // units per key tile
      const int U = n * SUB;
      for (int u = p.any_mask ? 0 : min(NS, U); u < U; ++u) {
        const int s = u % NS;
        if (u >= NS && !mbar_wait(bar(empty + s), ((u / NS) - 1) & 1, dead, p.err)) break;
        const int row = k_beg + (list[u / SUB] & 0x3fff) * BN;
        if (is_k) load_k_unit(u, s, row);
        else load_v_unit(u, s, row);
      }
      // Leave no bulk copy in flight: wait (bounded) for the last loads.
      bool d2 = false;
      if (is_k) mbar_wait(bar(C::kBarQ), 0, d2, p.err);
      for (int u = max(0, U - NS); u < U; ++u)
        mbar_wait(bar(full + u % NS), (u / NS) & 1, d2, p.err);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      // The P V accumulator tile i goes into, and its use count.
      auto og = [&](int i) -> int { return ALT ? (i & 1) : 0; };
      auto ouse = [&](int i) -> int { return ALT ? (i >> 1) : i; };
      // S[j] = Q K_j^T into S buffer j % SB. That buffer last held P[j - SB],
      // so P V[j - SB] must have completed (it reads P from there). kAlt
      // and kOne wait for it here (no later P V on that barrier is issued
      // yet);
      // kSplit issues S[j] after P V[j - 2], whose issue already waited for
      // P V[j - 3].
      // K arrives in KSUB units per tile (one unit for head_dim <= 256), each
      // released as soon as its share of the Q K^T MMAs completes.
      auto issue_s = [&](int j) -> bool {
        const int sb = j % C::SB;
        constexpr int KK = HDP / 16 / C::KSUB;  // 16-wide k-steps per K unit
#pragma unroll
        for (int part = 0; part < C::KSUB; ++part) {
          const int u = j * C::KSUB + part;
          const int s = u % STK;
          if (!mbar_wait(bar(C::kBarK + s), (u / STK) & 1, dead, p.err)) return false;
          if (part == 0 && !SPLIT && j >= C::SB &&
              !mbar_wait(bar(C::kBarO + og(j - C::SB)), ouse(j - C::SB) & 1, dead, p.err))
            return false;
          tc_fence_after();
          const uint32_t kbase = sK + s * C::kKUnitBytes;
#pragma unroll
          for (int k2 = 0; k2 < KK; ++k2) {
            const int kk = part * KK + k2;
            const uint64_t a =
                umma_desc_sw128(sQ + (kk >> 2) * C::kQChunk + (kk & 3) * 32, 16, 1024);
            const uint64_t bd =
                umma_desc_sw128(kbase + (k2 >> 2) * C::kKChunk + (k2 & 3) * 32, 16, 1024);
            umma_ss(tmem + sb * BN, a, bd, C::kIdescS, kk > 0 ? 1u : 0u);
          }
          if (part == C::KSUB - 1) umma_commit(bar(C::kBarS + sb));
          umma_commit(bar(C::kBarKE + s));
        }
        return true;
      };
      // O[g] += P[i] V_i, P read from TMEM (S buffer i % SB, 16 columns per
      // 16 keys: hi terms in the first 8, lo terms in the last 8). V arrives
      // in VSUB units of kVRows keys per tile.
      auto issue_pv = [&](int i) -> bool {
        const int g = og(i), use = ouse(i);
        constexpr int KK = BN / 16 / C::VSUB;  // 16-key steps per V unit
        const uint32_t pcol = tmem + (i % C::SB) * BN;
        const uint32_t dst = tmem + C::kOCol + g * C::HDO;
#pragma unroll
        for (int part = 0; part < C::VSUB; ++part) {
          const int u = i * C::VSUB + part;
          const int s = u % ST;
          if (!mbar_wait(bar(C::kBarV + s), (u / ST) & 1, dead, p.err)) return false;
          if (part == 0) {
            if (!mbar_wait(bar(C::kBarP + g), use & 1, dead, p.err)) return false;
            // kSplit: P V[i - 1] done (frees the buffer S[i + 2] takes).
            // Checked before P V[i] is issued, so the O barrier is at most
            // one phase on.
            if (SPLIT && i > 0 && !mbar_wait(bar(C::kBarO), (i - 1) & 1, dead, p.err))
              return false;
          }
          tc_fence_after();
          const uint32_t vbase = sV + s * C::kVUnitBytes;
#pragma unroll
          for (int term = 0; term < C::kPTerms; ++term) {
#pragma unroll
            for (int k2 = 0; k2 < KK; ++k2) {
              const int kk = part * KK + k2;
              const uint64_t bd = umma_desc_sw128(vbase + k2 * 2048, C::kVChunk, 1024);
              umma_ts(dst, pcol + kk * 16 + term * 8, bd, C::kIdescO,
                      (use > 0 || kk > 0 || term > 0) ? 1u : 0u);
            }
          }
          if (part == C::VSUB - 1) umma_commit(bar(C::kBarO + g));
          umma_commit(bar(C::kBarVE + s));
        }
        return true;
      };
      // Order: S[0], S[1], then per tile j: P V[j] once P[j] is written,
      // then S[j+2]. kAlt: S[j+2] reuses P[j]'s buffer and waits for P V[j];
      // the other group's softmax covers the gap. kSplit: S[j+2] takes the
      // buffer of P[j-1], so the tensor core runs P V[j] and S[j+2] back to
      // back while the softmax works on S[j+1].
      if (n > 0 && mbar_wait(bar(C::kBarQ), 0, dead, p.err) &&
          (!p.fuse_q || mbar_wait(bar(C::kBarQR), 0, dead, p.err))) {
        bool ok = issue_s(0) && (n < 2 || issue_s(1));
        for (int j = 0; ok && j < n; ++j) ok = issue_pv(j) && (j + 2 >= n || issue_s(j + 2));
      }
      // Every MMA this thread issued completes before the role ends.
      umma_commit(bar(C::kBarF));
      bool d2 = false;
      mbar_wait(bar(C::kBarF), 0, d2, p.err);
    }
  } else {
    // ------------------------------------------------------------ softmax
    // Warps 3..10: warp w reaches TMEM lanes 32 (w % 4) .. +31, so each lane
    // quarter q has two warps, one per group (grp 0: warps 3-6, 1: 7-10).
    constexpr int SC = SPLIT ? BN / 2 : BN;    // S columns per thread per tile
    constexpr int OC = SPLIT ? C::HDO / 2 : C::HDO;  // O columns this group owns
    const int wq = warp & 3;
    const int grp = (warp - 3) >> 2;
    const int r = wq * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const int s_col0 = SPLIT ? grp * SC : 0;
    const uint32_t o_own = C::kOCol + grp * OC;
    const int pg = SPLIT ? 0 : grp;  // P barrier and O accumulator of this group
    const uint32_t xbar = bar(C::kBarX + wq);
    const int t_local = t0 + r / p.G;
    const bool row_valid = r < p.R && t_local < q_len;
    const int gq = q_beg + (row_valid ? t_local : 0);
    int qpos = 0, qseq = 0, qpre = -1;
    if (row_valid && p.any_mask) {
      qpos = p.q_pos ? p.q_pos[gq] : t_local;
      qseq = p.q_seq ? p.q_seq[gq] : 0;
      qpre = p.q_prefix ? p.q_prefix[gq] : p.seq_prefix ? p.seq_prefix[b] : p.causal_prefix;
    }
    const float sl2 = p.scale_log2;
    const bool fast_ok = p.softcap == 0.f && sl2 >= 0.f;
    // The sliding window is the only mask and positions are contiguous:
    // visibility within a tile is a band test on the key index.
    // (window 0 makes every key invisible: left to the generic form.)
    const bool band_ok = p.window != kNoWindow && p.window > 0 && !p.k_pos && !p.k_seq &&
                         !p.q_seq && !p.q_prefix && !p.seq_prefix && p.causal_prefix < 0;
    // Soft-cap: logit = cap * tanh(score * scale / cap), in log2 units.
    const float scale_cap = p.softcap != 0.f ? p.scale / p.softcap : 0.f;
    const float cap_l2 = p.softcap * 1.4426950408889634f;
    float m = -INFINITY, l = 0.f;
    int used = 0;  // tiles this thread has processed

    if constexpr (HDP == 128) {
      if (p.fuse_q) fuse_q_prep<C>(p, sQ, bar(C::kBarQ), bar(C::kBarQR), t0, q_beg, q_len,
                                   (warp - 3) * 32 + lane, dead);
    }

    for (int j = ALT ? grp : 0; j < n; j += ALT ? 2 : 1) {
      const int entry = list[j];
      const int kt = entry & 0x3fff;
      const int kind = entry >> 14;  // 0 full, 1 ragged end, 2 masked
      const int sb = j % C::SB;
      mbar_wait(bar(C::kBarS + sb), (j / C::SB) & 1, dead, p.err);
      dead = __any_sync(0xffffffffu, dead);
      if (dead) break;
      tc_fence_after();
      // Each thread reads its row of S from TMEM once (32-column loads, one
      // wait) and keeps it in registers: pass 1 forms the row max, pass 2
      // exponentiates and writes P back over the columns of S. The masked
      // form instead streams 8- and 16-column pieces twice (cold path).
      constexpr int LB = 32;
      const uint32_t s_addr = tmem + lane_off + sb * BN + s_col0;
      // The arithmetic is picked per tile (uniform) as a value transform and
      // a mask, each loop unrolled with both as template constants:
      //   value  kPlain    s * scale (scale >= 0, no soft-cap): FFMA + ex2
      //          kCap      soft-cap (or negative scale): exact tanh
      //          kCapPoly  kCap whose scaled scores all lie where tanh_poly
      //                    is exact (decided after pass 1): no MUFU op
      //   mask   kNone     every key of the tile visible
      //          kRagged   keys at or past `nvalid` masked (sequence end)
      //          kBand     |q pos - key| < window, positions contiguous (the
      //                    sliding window is the only mask): integer test
      // Other masks (seq ids, prefixes, explicit key positions) take the
      // generic form: compact rolled loops over 8- and 16-column TMEM loads
      // with per-element visible() (cold: a few tiles per CTA).
      enum { kPlain, kCap, kCapPoly };
      enum { kNone, kRagged, kBand, kGenericMask };
      int val = fast_ok ? kPlain : kCap;
      const int msk = kind == 0 ? kNone : kind == 1 ? kRagged : band_ok ? kBand : kGenericMask;
      const bool generic = msk == kGenericMask;
      const int nvalid = k_len - kt * BN - s_col0;  // keys of this thread's columns
      // kBand: key i of the thread's columns is visible iff
      // (unsigned)(band0 - i) <= band2, i.e. |qpos - key| < window.
      const int band0 = qpos - (kt * BN + s_col0) + p.window - 1;
      const uint32_t band2 = 2u * static_cast<uint32_t>(p.window) - 2u;
      const float sgn = p.scale < 0.f ? -1.f : 1.f;
      // Scaled log2-domain logit without masks (soft-cap, any scale sign).
      auto logit_nm = [&](uint32_t bits) -> float {
        if (p.softcap != 0.f) return cap_l2 * tanh_via_exp2(u2f(bits) * scale_cap);
        return u2f(bits) * sl2;
      };
      // With per-element visibility (masked keys -> -inf).
      auto logit = [&](uint32_t bits, int i) -> float {
        float t = logit_nm(bits);
        const int kl = kt * BN + s_col0 + i;
        bool ok = kl < k_len;
        if (ok && p.any_mask) {
          const int g = k_beg + kl;
          const int kp = p.k_pos ? p.k_pos[g] : kl;
          const int ks = p.k_seq ? p.k_seq[g] : 0;
          ok = visible_dev(qpos, kp, qseq, ks, p.window, qpre);
        }
        return ok ? t : -INFINITY;
      };
      // Visibility of column i under mask M (compile-time M, constant i).
      auto vis = [&](auto msk_c, int i) -> bool {
        constexpr int M = decltype(msk_c)::value;
        if constexpr (M == kNone) return true;
        else if constexpr (M == kRagged) return i < nvalid;
        else return i < nvalid && static_cast<uint32_t>(band0 - i) <= band2;
      };
      // Calls f(value, mask) with the tile's forms as template constants.
      auto dispatch = [&](auto f) {
        using P0 = std::integral_constant<int, kPlain>;
        using P1 = std::integral_constant<int, kCap>;
        using P2 = std::integral_constant<int, kCapPoly>;
        using M0 = std::integral_constant<int, kNone>;
        using M1 = std::integral_constant<int, kRagged>;
        using M2 = std::integral_constant<int, kBand>;
        if (val == kPlain) {
          if (msk == kNone) f(P0{}, M0{});
          else if (msk == kRagged) f(P0{}, M1{});
          else f(P0{}, M2{});
        } else if (val == kCap) {
          if (msk == kNone) f(P1{}, M0{});
          else if (msk == kRagged) f(P1{}, M1{});
          else f(P1{}, M2{});
        } else {
          if (msk == kNone) f(P2{}, M0{});
          else if (msk == kRagged) f(P2{}, M1{});
          else f(P2{}, M2{});
        }
      };

      // Pass 1: row max over this thread's columns (8 independent chains).
      uint32_t srow[SC];
      float rmax;
      float amax = 0.f;  // kCap: largest |raw score| among visible keys
      {
        float mx8[8];
#pragma unroll
        for (int a = 0; a < 8; ++a) mx8[a] = -INFINITY;
        auto pass1 = [&](auto val_c, auto msk_c) {
          constexpr int V = decltype(val_c)::value;
#pragma unroll
          for (int cb = 0; cb < SC / LB; ++cb)
            tmem_ld32(s_addr + cb * LB, *reinterpret_cast<uint32_t(*)[LB]>(&srow[cb * LB]));
          tmem_wait_ld();
#pragma unroll
          for (int cb = 0; cb < SC / LB; ++cb) {
            const uint32_t* sr = &srow[cb * LB];
            float v[LB];
#pragma unroll
            for (int i = 0; i < LB; ++i) {
              // kCap: the logit is monotonic in sgn * raw score.
              const float x = V == kPlain ? u2f(sr[i]) : sgn * u2f(sr[i]);
              v[i] = vis(msk_c, cb * LB + i) ? x : -INFINITY;
            }
#if CA_MAX3
#pragma unroll
            for (int i = 0; i < LB; i += 2) mx8[(i >> 1) & 7] = fmax3(mx8[(i >> 1) & 7], v[i], v[i + 1]);
#else
#pragma unroll
            for (int i = 0; i < LB; ++i) mx8[i & 7] = fmaxf(mx8[i & 7], v[i]);
#endif
            if constexpr (V == kCap) {
#pragma unroll
              for (int i = 0; i < LB; ++i)
                amax = fmaxf(amax, vis(msk_c, cb * LB + i) ? fabsf(v[i]) : 0.f);
            }
          }
        };
        if (generic) {
#pragma unroll 1
          for (int c8 = 0; c8 < SC / 8; ++c8) {
            uint32_t sr[8];
            tmem_ld8(s_addr + c8 * 8, sr);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 8; ++i) mx8[i] = fmaxf(mx8[i], logit(sr[i], c8 * 8 + i));
          }
        } else {
          dispatch(pass1);
        }
        rmax = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                     fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      }
      if constexpr (SPLIT) {
        // Combine with the partner warp (same rows, other key columns).
        float* xch = reinterpret_cast<float*>(smem + C::kOffXch);
        xch[((j & 1) * 2 + grp) * 128 + r] = rmax;
        __syncwarp();
        if (lane == 0) mbar_arrive(xbar);
        mbar_wait(xbar, j & 1, dead, p.err);
        dead = __any_sync(0xffffffffu, dead);
        if (dead) break;
        rmax = fmaxf(rmax, xch[((j & 1) * 2 + (grp ^ 1)) * 128 + r]);
      }
      // Plain maxima are raw scores; kCap's is sgn * raw score (the soft-
      // capped logit is monotonic in it); the generic form's is a logit.
      float mcand;
      if (generic) mcand = rmax;
      else if (val == kPlain) mcand = rmax * sl2;
      else mcand = rmax == -INFINITY ? rmax : logit_nm(f2u(sgn * rmax));
      // Soft-cap tiles whose scaled scores all lie in tanh_poly's range (per
      // warp; the two warps of a kSplit pair may choose differently, both
      // forms give the same logits to ~1e-7).
      if (!generic && val == kCap && p.softcap != 0.f &&
          __all_sync(0xffffffffu, amax * fabsf(scale_cap) <= kTanhPolyMax))
        val = kCapPoly;
      const bool resc = mcand > m + 8.f;
      float corr = 1.f;
      if (resc) {
        corr = ex2_approx(m - mcand);
        m = mcand;
      }
      const float mu = (m == -INFINITY) ? 0.f : m;

      // Pass 2: exponentiate and write P into the S buffer, in the layout the
      // P V MMA reads as its TMEM A operand: the 16 keys of block kk take
      // columns 16 kk .. 16 kk + 15, bf16 pairs of the hi terms in the first 8
      // and (PRECISE) of the lo terms in the last 8. Every block lands inside
      // the columns it was read from, so no unread S is overwritten.
      float sum4[4] = {0.f, 0.f, 0.f, 0.f};
#if CA_F32X2
      float2 sum2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#endif
      auto emit = [&](float p0, float p1, int q2, uint32_t& hi, uint32_t& lo) {
#if CA_F32X2
        sum2[q2 & 1] = __fadd2_rn(sum2[q2 & 1], make_float2(p0, p1));
#else
        sum4[q2 & 3] += p0 + p1;
#endif
        hi = pack_bf16(p0, p1);
        if constexpr (C::PRECISE) {
          const float h0 = __uint_as_float(hi << 16);
          const float h1 = __uint_as_float(hi & 0xffff0000u);
          lo = pack_bf16(p0 - h0, p1 - h1);
        }
      };
      if (generic) {
#pragma unroll 1
        for (int c16 = 0; c16 < SC / 16; ++c16) {
          uint32_t sr[16], hi[8], lo[8];
          tmem_ld16(s_addr + c16 * 16, sr);
          tmem_wait_ld();
#pragma unroll
          for (int q2 = 0; q2 < 8; ++q2)
            emit(ex2_approx(logit(sr[2 * q2], c16 * 16 + 2 * q2) - mu),
                 ex2_approx(logit(sr[2 * q2 + 1], c16 * 16 + 2 * q2 + 1) - mu), q2, hi[q2],
                 lo[q2]);
          tmem_st8(s_addr + c16 * 16, hi);
          if constexpr (C::PRECISE) tmem_st8(s_addr + c16 * 16 + 8, lo);
        }
      } else {
        auto pass2 = [&](auto val_c, auto msk_c) {
          constexpr int V = decltype(val_c)::value;
          constexpr int M = decltype(msk_c)::value;
#pragma unroll
          for (int cb = 0; cb < SC / LB; ++cb) {
            const uint32_t* sr = &srow[cb * LB];
#pragma unroll
            for (int blk = 0; blk < LB / 16; ++blk) {
              uint32_t hi[8], lo[8];
#pragma unroll
              for (int q2 = 0; q2 < 8; ++q2) {
                const int i = blk * 16 + q2 * 2;
                float x0, x1;
                if constexpr (V == kCap) {
                  x0 = logit_nm(sr[i]) - mu;
                  x1 = logit_nm(sr[i + 1]) - mu;
                } else if constexpr (V == kCapPoly) {
                  // Packed form only in the head_dim 256 (kSplit) kernel: it
                  // measured +4% on soft-capped layers there, but -1.3% on
                  // the head_dim 128 kernel's uncapped tiles (code layout).
                  if constexpr (SPLIT && CA_TANH2) {
                    const float2 t = tanh_poly2(__fmul2_rn(
                        make_float2(u2f(sr[i]), u2f(sr[i + 1])), make_float2(scale_cap, scale_cap)));
                    const float2 x01 = __ffma2_rn(make_float2(cap_l2, cap_l2), t,
                                                  make_float2(-mu, -mu));
                    x0 = x01.x;
                    x1 = x01.y;
                  } else {
                    x0 = fmaf(cap_l2, tanh_poly(u2f(sr[i]) * scale_cap), -mu);
                    x1 = fmaf(cap_l2, tanh_poly(u2f(sr[i + 1]) * scale_cap), -mu);
                  }
                } else {
#if CA_F32X2
                  const float2 x01 = __ffma2_rn(make_float2(u2f(sr[i]), u2f(sr[i + 1])),
                                                make_float2(sl2, sl2), make_float2(-mu, -mu));
                  x0 = x01.x;
                  x1 = x01.y;
#else
                  x0 = fmaf(u2f(sr[i]), sl2, -mu);
                  x1 = fmaf(u2f(sr[i + 1]), sl2, -mu);
#endif
                }
                if constexpr (M != kNone) {
                  x0 = vis(msk_c, cb * LB + i) ? x0 : -INFINITY;
                  x1 = vis(msk_c, cb * LB + i + 1) ? x1 : -INFINITY;
                }
                if constexpr ((ALT || ONE) && V == kPlain && M == kNone && !C::PRECISE &&
                              CA_POLY_EVERY > 0) {
                  if (q2 % kPolyEvery == kPolyEvery - 1) {
                    const float2 e = ex2_poly3x2(x0, x1);
                    emit(e.x, e.y, q2, hi[q2], lo[q2]);
                    continue;
                  }
                }
                emit(ex2_approx(x0), ex2_approx(x1), q2, hi[q2], lo[q2]);
              }
              tmem_st8(s_addr + cb * LB + blk * 16, hi);
              if constexpr (C::PRECISE) tmem_st8(s_addr + cb * LB + blk * 16 + 8, lo);
            }
          }
        };
        dispatch(pass2);
      }
#if CA_F32X2
      sum4[0] += sum2[0].x;
      sum4[1] += sum2[0].y;
      sum4[2] += sum2[1].x;
      sum4[3] += sum2[1].y;
#endif
      l = l * corr + ((sum4[0] + sum4[1]) + (sum4[2] + sum4[3]));
      // kAlt: this group's previous P V completed before S[j] was computed.
      // kSplit: the previous P V (tile j - 1) may still run; wait for it. The
      // wait also keeps the O barrier from running two phases ahead of any
      // waiter (P V[j] cannot start before this warp's P arrival below).
      if constexpr (SPLIT) {
        if (used > 0) {
          mbar_wait(bar(C::kBarO), (j - 1) & 1, dead, p.err);
          dead = __any_sync(0xffffffffu, dead);
          if (dead) break;
          tc_fence_after();
        }
      }
      // kOne: wait for the previous tile's P V. It may still accumulate into
      // O (which a correction rescales), and its completion shows that the
      // MMA issuer has taken P[j - 1]: S[j] was issued before P V[j - 1], so
      // without this wait the group could arrive for P[j] while the issuer
      // still waits (on V[j - 1]) for P[j - 1], and the P barrier would run
      // two phases ahead of that parity wait.
      if constexpr (ONE) {
        if (used > 0) {
          mbar_wait(bar(C::kBarO), (j - 1) & 1, dead, p.err);
          dead = __any_sync(0xffffffffu, dead);
          if (dead) break;
          tc_fence_after();
        }
      }
      // Lazy correction of O (rare after the first tiles).
      if (used > 0 && __any_sync(0xffffffffu, resc)) {
#pragma unroll 1
        for (int c = 0; c < OC / 32; ++c) {
          uint32_t o[32];
          const uint32_t ta = tmem + lane_off + o_own + c * 32;
          tmem_ld32(ta, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = f2u(u2f(o[i]) * corr);
          tmem_st32(ta, o);
        }
      }
      // P (and any corrected O) must be in TMEM before the P V MMA is issued.
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(C::kBarP + pg));
      ++used;
    }

    // ------------------------------------------------------------ epilogue
    // Wait for this group's last P V. kAlt: merge the two groups' (max, sum, O) partials. kSplit: add the two
    // halves' row sums (same running max).
    // kAlt: wait until every MMA is done (the output is staged in the K/V
    // rings; this also covers a group that had no tile of its own).
    if (ALT && n > 0 && !dead) {
      mbar_wait(bar(C::kBarF), 0, dead, p.err);
      dead = __any_sync(0xffffffffu, dead);
      tc_fence_after();
    } else if (used > 0 && !dead) {
      mbar_wait(bar(C::kBarO + pg), (used - 1) & 1, dead, p.err);
      dead = __any_sync(0xffffffffu, dead);
      tc_fence_after();
    }
    // Wide heads stage the output in the Q tile: its load must have landed
    // (a tile with no visible key issues no MMA that would have waited).
    if constexpr (C::kOffStage == C::kOffQ) {
      if (p.tma_out && n == 0) mbar_wait(bar(C::kBarQ), 0, dead, p.err);
    }
    bool have = n > 0 && !dead;
    float s_me = 1.f, s_ot = 0.f, inv = __int_as_float(0x7fc00000);
    const int n_me = ALT ? (grp == 0 ? (n + 1) / 2 : n / 2) : n;
    const int n_ot = ALT ? (grp == 0 ? n / 2 : (n + 1) / 2) : 0;
    if (have && ONE) {
      inv = 1.f / l;  // a single group owns every row and column
    } else if (have) {
      // kAlt: [group][l, m][128].
      float* xch = reinterpret_cast<float*>(smem + C::kOffXch);
      float* xo = ALT ? xch + grp * 256 : xch + ((n & 1) * 2 + grp) * 128;
      float* xp = ALT ? xch + (grp ^ 1) * 256 : xch + ((n & 1) * 2 + (grp ^ 1)) * 128;
      xo[r] = l;
      if (ALT) xo[128 + r] = m;
      __syncwarp();
      if (lane == 0) mbar_arrive(xbar);
      mbar_wait(xbar, ALT ? 0 : (n & 1), dead, p.err);
      dead = __any_sync(0xffffffffu, dead);
      have = !dead;
      tc_fence_after();
      const float l_ot = xp[r];
      if (ALT) {
        const float m_ot = xp[128 + r];
        const float mt = fmaxf(n_me > 0 ? m : -INFINITY, n_ot > 0 ? m_ot : -INFINITY);
        const float mref = mt == -INFINITY ? 0.f : mt;
        s_me = n_me > 0 ? ex2_approx(m - mref) : 0.f;
        s_ot = n_ot > 0 ? ex2_approx(m_ot - mref) : 0.f;
        inv = 1.f / (s_me * (n_me > 0 ? l : 0.f) + s_ot * (n_ot > 0 ? l_ot : 0.f));
      } else {
        inv = 1.f / (l + l_ot);
      }
    }
    const int head = kvh * p.G + (r % p.G);
    // Columns this warp writes: kAlt half of the columns from both
    // accumulators; kSplit its own half.
    constexpr int WC = ONE ? C::HDO : C::HDO / 2;
    const int col0 = ONE ? 0 : grp * WC;
    const uint32_t o_me = ALT ? C::kOCol + grp * C::HDO + col0 : o_own;
    const uint32_t o_ot = C::kOCol + (grp ^ 1) * C::HDO + col0;
    const int ocol = ohalf * C::HDO;  // this CTA's first output column
#pragma unroll 1
    for (int c = 0; c < WC / 32; ++c) {
      const int col_base = col0 + c * 32;
      uint32_t o[32];
      float v[32];
      if (have && n_me > 0) {
        tmem_ld32(tmem + lane_off + o_me + c * 32, o);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = u2f(o[i]) * s_me;
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = 0.f;
      }
      if (ALT && have && n_ot > 0) {
        tmem_ld32(tmem + lane_off + o_ot + c * 32, o);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = fmaf(u2f(o[i]), s_ot, v[i]);
      }
      if (p.tma_out) {
        // Stage row r in 128-byte column chunks, 16-byte units XOR-swizzled
        // by r & 7 (the tensor map's 128-byte swizzle); rows past the
        // sequence end and columns past head_dim are clipped by the store.
        uint8_t* stg = smem + C::kOffStage;
        if (p.out_f32) {
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int col = col_base + u * 4;
            const int ci = col >> 5, uu = (col & 31) >> 2;
            float4 w;
            w.x = have ? v[u * 4] * inv : inv;
            w.y = have ? v[u * 4 + 1] * inv : inv;
            w.z = have ? v[u * 4 + 2] * inv : inv;
            w.w = have ? v[u * 4 + 3] * inv : inv;
            *reinterpret_cast<float4*>(stg + ci * C::kStageChunk + r * 128 +
                                       ((uu ^ (r & 7)) << 4)) = w;
          }
        } else {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int col = col_base + u * 8;
            const int ci = col >> 6, uu = (col & 63) >> 3;
            float w8[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) w8[i] = have ? v[u * 8 + i] * inv : inv;
            uint4 w;
            w.x = pack_bf16(w8[0], w8[1]);
            w.y = pack_bf16(w8[2], w8[3]);
            w.z = pack_bf16(w8[4], w8[5]);
            w.w = pack_bf16(w8[6], w8[7]);
            *reinterpret_cast<uint4*>(stg + ci * C::kStageChunk + r * 128 +
                                      ((uu ^ (r & 7)) << 4)) = w;
          }
        }
      } else if (row_valid) {
        const int64_t obase = static_cast<int64_t>(gq) * p.out_row_stride +
                              static_cast<int64_t>(head) * p.hd;
#pragma unroll
        for (int g8 = 0; g8 < 4; ++g8) {
          const int col = ocol + col_base + g8 * 8;
          if (col < p.hd) {
            float w8[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) w8[i] = have ? v[g8 * 8 + i] * inv : inv;
            if (p.out_f32) {
              float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + obase + col);
              const float4 a = make_float4(w8[0], w8[1], w8[2], w8[3]);
              const float4 b4 = make_float4(w8[4], w8[5], w8[6], w8[7]);
              dst[0] = a;
              dst[1] = b4;
              if (p.n_peer) {
                store_peers(p, obase + col, *reinterpret_cast<const uint4*>(&a));
                store_peers(p, obase + col + 4, *reinterpret_cast<const uint4*>(&b4));
              }
            } else {
              uint4 w;
              w.x = pack_bf16(w8[0], w8[1]);
              w.y = pack_bf16(w8[2], w8[3]);
              w.z = pack_bf16(w8[4], w8[5]);
              w.w = pack_bf16(w8[6], w8[7]);
              *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.out) + obase + col) = w;
              if (p.n_peer) store_peers(p, obase + col, w);
            }
          }
        }
      }
    }
    if (p.tma_out && p.mc_out) {
      // Multicast output: every softmax thread copies 16-byte units of the
      // staged tile to the multicast address, consecutive threads along a
      // row (a row of the tile is contiguous in `out`), so each warp writes
      // whole 128-byte lines. The switch replicates each store to every
      // rank's buffer: one crossing of this GPU's NVLink per row.
      named_bar_sync(2, C::kSoftThreads);
      const int es = p.out_f32 ? 4 : 2;
      const int inner = 128 / es;                 // elements per staged chunk
      const int upr = (C::HDO * es) / 16;         // 16-byte units per row
      const int q_beg_u = b * p.sq;
      const int tid_s = (warp - 3) * 32 + lane;
      for (int u = tid_s; u < p.R * upr; u += C::kSoftThreads) {
        const int rr = u / upr, cu = u % upr;     // tile row, unit within the row
        const int ci = cu >> 3, uu = cu & 7;      // staged chunk, unit within it
        const int tl = t0 + rr / p.G;
        const int col = ocol + ci * inner + uu * (16 / es);
        if (tl >= q_len || col >= p.hd) continue;
        const uint4 w = *reinterpret_cast<const uint4*>(
            smem + C::kOffStage + ci * C::kStageChunk + rr * 128 + ((uu ^ (rr & 7)) << 4));
        const int64_t off = (static_cast<int64_t>(q_beg_u + tl) * p.out_row_stride +
                             static_cast<int64_t>(kvh * p.G + rr % p.G) * p.hd + col) * es;
        multimem_st_v4(static_cast<uint8_t*>(p.mc_out) + off, w);
      }
    } else if (p.tma_out) {
      // All softmax warps have staged their rows: one thread stores the tile.
      fence_proxy_async_smem();
      named_bar_sync(2, C::kSoftThreads);
      if (warp == 3 && lane == 0) {
        const int inner = p.out_f32 ? 32 : 64;  // elements per 128-byte chunk
        for (int ci = 0; ci * inner < C::HDO && ocol + ci * inner < p.hd; ++ci) {
          const uint32_t src = smem_u32(smem + C::kOffStage + ci * C::kStageChunk);
          tma_store_4d(&tm_o, src, ocol + ci * inner, kvh * p.G, t0, b);
          // The same tile into every peer's buffer (head-sharded layers).
          for (int i = 0; i < p.n_peer; ++i)
            tma_store_4d(&pm.m[i], src, ocol + ci * inner, kvh * p.G, t0, b);
        }
        bulk_commit_group();
        bulk_wait_group_read0();
      }
    }
  }

  // Peer stores need no fence here: a CTA that waited for them would hold
  // its SM idle, and the grid's completion already orders them before any
  // stream-ordered barrier the host issues afterwards.
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

}  // namespace ca
