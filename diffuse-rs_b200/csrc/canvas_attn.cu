// canvas_attn.cu -- the single translation unit of libcanvas_attn.so: the
// sm_100a kernels (attn_fwd.cuh, prep.cuh) and the C ABI declared in
// include/canvas_attn.h.
#include <cuda.h>
#include <cuda_runtime.h>

#include <climits>
#include <cmath>
#include <cstdint>
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <vector>

#include "host_round.h"

#include "canvas_attn.h"
#include "attn_fwd.cuh"
#include "prep.cuh"
#include "sampler.cuh"
#include "quant.cuh"
#include <cublasLt.h>

namespace ca {
namespace {

constexpr int kMaxDevices = 64;

// ---------------------------------------------------------------- driver entry
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 3-D bf16 view [tokens][heads][hd] (innermost first in TMA order), boxes of
// 64 x box_heads x box_tokens with 128-byte swizzle; out-of-range reads fill 0.
int make_tmap(CUtensorMap* m, const void* base, int64_t hd, int64_t heads, int64_t tokens,
              int64_t row_stride_elems, uint32_t box_heads, uint32_t box_tokens) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return CA_ERR_CUDA;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(hd), static_cast<cuuint64_t>(heads),
                        static_cast<cuuint64_t>(tokens)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(hd) * 2,
                           static_cast<cuuint64_t>(row_stride_elems) * 2};
  cuuint32_t box[3] = {64, box_heads, box_tokens};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides,
                  box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? CA_OK : CA_ERR_INVALID;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// 4-D view of the output [batch][tokens][heads][hd] (uniform batch), bf16 or
// fp32, boxes of one 128-byte column chunk x box_heads x box_tokens, 128-byte
// swizzle. Stores clip at each sequence's end and at head_dim.
int make_tmap_out(CUtensorMap* m, void* base, int64_t hd, int64_t heads, int64_t sq,
                  int64_t batch, int64_t row_stride_elems, bool f32, uint32_t box_heads,
                  uint32_t box_tokens) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return CA_ERR_CUDA;
  const uint64_t es = f32 ? 4 : 2;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(hd), static_cast<cuuint64_t>(heads),
                        static_cast<cuuint64_t>(sq), static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(hd) * es,
                           static_cast<cuuint64_t>(row_stride_elems) * es,
                           static_cast<cuuint64_t>(row_stride_elems * sq) * es};
  cuuint32_t box[4] = {static_cast<cuuint32_t>(128 / es), box_heads, box_tokens, 1};
  cuuint32_t elem[4] = {1, 1, 1, 1};
  CUresult r = fn(m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4,
                  base, dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? CA_OK : CA_ERR_INVALID;
}

// ---------------------------------------------------------------- launch
// Builds the tensor maps for one tile configuration and launches it.
struct Launch {
  const ca_dev_args* a;
  const FwdParams* p;
  int64_t total_q, total_k;
  int max_sq;
  int64_t max_sk;
  int64_t qrs, krs;
  cudaStream_t st;

  template <class C>
  int run() const {
    static bool attr_done[kMaxDevices] = {};
    const int64_t n_kt = (max_sk + C::BN - 1) / C::BN;
    if (n_kt > C::kMaxTiles) return CA_ERR_UNSUPPORTED;
    CUtensorMap tq, tk, tv, to;
    const int hd = p->hd;
    const int64_t tk_rows = total_k == 0 ? 1 : total_k;
    int rc;
    if ((rc = make_tmap(&tq, a->q, hd, p->n_head, total_q, qrs, p->G, p->QT)) != CA_OK) return rc;
    if ((rc = make_tmap(&tk, a->k, hd, p->n_head_kv, tk_rows, krs, 1, C::BN)) != CA_OK) return rc;
    if ((rc = make_tmap(&tv, a->v, hd, p->n_head_kv, tk_rows, krs, 1, C::kVRows)) != CA_OK)
      return rc;
    // Uniform batches store O through a tensor map (the map clips at each
    // sequence's end); otherwise the kernel stores rows itself.
    FwdParams pl = *p;
    const int64_t es = p->out_f32 ? 4 : 2;
    pl.tma_out = !a->cu_q && p->batch > 0 && p->sq > 0 && aligned16(a->out) &&
                 (p->out_row_stride * es) % 16 == 0 && (p->hd * es) % 16 == 0;
    if (pl.tma_out &&
        make_tmap_out(&to, a->out, hd, p->n_head, p->sq, p->batch, p->out_row_stride,
                      p->out_f32 != 0, p->G, p->QT) != CA_OK)
      pl.tma_out = 0;
    if (!pl.tma_out) to = tq;  // unused
    if (pl.mc_out && !pl.tma_out) return CA_ERR_UNSUPPORTED;
    // Peer buffers: tensor maps of the same shape for the TMA epilogue;
    // the row-store epilogue writes them with plain stores instead.
    PeerMaps pm;
    std::memset(&pm, 0, sizeof(pm));
    for (int i = 0; pl.tma_out && i < pl.n_peer; ++i)
      if (make_tmap_out(&pm.m[i], pl.peer_out[i], hd, p->n_head, p->sq, p->batch,
                        p->out_row_stride, p->out_f32 != 0, p->G, p->QT) != CA_OK)
        return CA_ERR_INVALID;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return CA_ERR_CUDA;
    if (!attr_done[dev]) {
      if (cudaFuncSetAttribute(attn_fwd_kernel<C>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               C::kSmemBytes) != cudaSuccess)
        return CA_ERR_CUDA;
      // Configurations meant to share an SM ask for the whole carve-out.
      if (C::kMinBlocks > 1 &&
          cudaFuncSetAttribute(attn_fwd_kernel<C>, cudaFuncAttributePreferredSharedMemoryCarveout,
                               100) != cudaSuccess)
        return CA_ERR_CUDA;
      attr_done[dev] = true;
    }
    const int n_qtiles = (max_sq + p->QT - 1) / p->QT;
    dim3 grid(n_qtiles * C::OS, p->n_head_kv, p->batch);
    attn_fwd_kernel<C><<<grid, C::kThreads, C::kSmemBytes, st>>>(tq, tk, tv, to, pl, pm);
    return cudaGetLastError() == cudaSuccess ? CA_OK : CA_ERR_CUDA;
  }
};


int clamp_opt(int64_t v) {  // Option<usize> as int32 (None = -1)
  if (v < 0) return -1;
  return v > INT_MAX ? INT_MAX : static_cast<int>(v);
}

}  // namespace

// Validates a device-args struct and launches the attention kernel.
// Fused Q pre-ops for the block path (see FwdParams::fuse_q).
#ifndef CA_FUSE_Q
#define CA_FUSE_Q 1
#endif
#ifndef CA_PREP_RING
#define CA_PREP_RING 1
#endif
#ifndef CA_PREP_BULK
#define CA_PREP_BULK 1
#endif
struct QFuse {
  const float* w;     // q norm gains [128] or null
  const float* rope;  // [rope_len, 64, 2] (sin, cos)
  float eps;
};

int attention_dev_impl(const ca_dev_args* a, cudaStream_t st, const QFuse* fq = nullptr) {
  if (!a || !a->q || !a->k || !a->v || !a->out) return CA_ERR_INVALID;
  const int H = a->n_head, Hkv = a->n_head_kv, hd = a->head_dim;
  if (H <= 0 || Hkv <= 0 || hd <= 0 || a->batch < 0) return CA_ERR_INVALID;
  if (H % Hkv != 0) return CA_ERR_INVALID;
  if (hd % 8 != 0 || hd > 512) return CA_ERR_UNSUPPORTED;
  const int G = H / Hkv;
  if (G > 128) return CA_ERR_UNSUPPORTED;
  if (a->batch == 0) return CA_OK;
  const bool varlen = a->cu_q != nullptr || a->cu_k != nullptr;
  if (varlen && (!a->cu_q || !a->cu_k || a->total_q < 0 || a->total_k < 0 || a->max_sq < 0))
    return CA_ERR_INVALID;
  if (!varlen && (a->sq < 0 || a->sk < 0)) return CA_ERR_INVALID;
  const int64_t total_q = varlen ? a->total_q : static_cast<int64_t>(a->batch) * a->sq;
  const int64_t total_k = varlen ? a->total_k : static_cast<int64_t>(a->batch) * a->sk;
  const int max_sq = varlen ? a->max_sq : a->sq;
  const int64_t max_sk = varlen ? total_k : a->sk;
  if (total_q == 0 || max_sq == 0) return CA_OK;
  if (total_q > INT_MAX || total_k > INT_MAX) return CA_ERR_UNSUPPORTED;
  const int64_t qrs = a->q_row_stride ? a->q_row_stride : static_cast<int64_t>(H) * hd;
  const int64_t krs = a->kv_row_stride ? a->kv_row_stride : static_cast<int64_t>(Hkv) * hd;
  const int64_t ors = a->out_row_stride ? a->out_row_stride : static_cast<int64_t>(H) * hd;
  if (qrs < static_cast<int64_t>(H) * hd || krs < static_cast<int64_t>(Hkv) * hd ||
      ors < static_cast<int64_t>(H) * hd)
    return CA_ERR_INVALID;
  // TMA: 16-byte aligned bases and strides; epilogue: 16-byte output vectors.
  if (!aligned16(a->q) || !aligned16(a->k) || !aligned16(a->v) || !aligned16(a->out) ||
      qrs % 8 || krs % 8 || ors % (a->out_f32 ? 4 : 8))
    return CA_ERR_INVALID;

  const int hdp = (hd + 63) / 64 * 64;

  FwdParams p{};
  p.out = a->out;
  p.out_f32 = a->out_f32 ? 1 : 0;
  p.out_row_stride = ors;
  p.batch = a->batch;
  p.sq = a->sq;
  p.sk = a->sk;
  p.cu_q = a->cu_q;
  p.cu_k = a->cu_k;
  p.n_head = H;
  p.n_head_kv = Hkv;
  p.G = G;
  p.hd = hd;
  p.QT = 128 / G;
  p.R = p.QT * G;
  p.q_pos = a->q_pos;
  p.k_pos = a->k_pos;
  p.q_seq = a->q_seq;
  p.k_seq = a->k_seq;
  p.q_prefix = a->q_prefix;
  p.seq_prefix = a->seq_prefix;
  p.window = a->sliding_window < 0 ? kNoWindow
                                   : static_cast<int>(a->sliding_window >= INT_MAX
                                                          ? INT_MAX - 1
                                                          : a->sliding_window);
  p.causal_prefix = clamp_opt(a->causal_prefix);
  p.scale = a->scale;
  p.scale_log2 = a->scale * 1.4426950408889634f;
  p.softcap = a->softcap > 0.f ? a->softcap : 0.f;
  // Positions alone mask nothing (visible() reads them only for the window
  // and the causal prefix), so they do not make a mask by themselves.
  p.any_mask = (a->q_seq || a->k_seq || a->q_prefix || a->seq_prefix ||
                p.window != kNoWindow || p.causal_prefix >= 0)
                   ? 1
                   : 0;

  p.err = a->status;
  if (a->n_peer_out < 0 || a->n_peer_out > kMaxPeers || (a->n_peer_out > 0 && !a->peer_out))
    return CA_ERR_INVALID;
  p.n_peer = a->n_peer_out;
  for (int i = 0; i < p.n_peer; ++i) {
    if (!a->peer_out[i] || !aligned16(a->peer_out[i])) return CA_ERR_INVALID;
    p.peer_out[i] = a->peer_out[i];
  }
  // Multicast output: one multimem store per row reaches every rank's
  // buffer (uniform batches, which stage the tile for the store pass).
  p.mc_out = a->out_multicast;
  if (p.mc_out && (a->cu_q || p.n_peer > 0 || !aligned16(p.mc_out))) return CA_ERR_INVALID;
  p.fuse_q = fq != nullptr;
  p.fq_w = fq ? fq->w : nullptr;
  p.fq_rope = fq ? fq->rope : nullptr;
  p.fq_eps = fq ? fq->eps : 0.f;

  Launch L{a, &p, total_q, total_k, max_sq, max_sk, qrs, krs, st};
  // One Q tile per CTA. head_dim <= 192: the two softmax groups alternate
  // key tiles (kAlt). head_dim 256: they split every tile's key columns
  // around one O, with three S buffers (kSplit). P lives in TMEM, so shared
  // memory holds only Q and the K/V rings. Two stages measured faster than
  // three at head_dim 128 (970 vs 949 TFLOP/s at B8 S4096 H16; the smaller
  // shared-memory carve-out leaves more L1), and at head_dim 64 and 192. (kSplit with three S buffers
  // at head_dim 128 measured 746 vs 823 TFLOP/s for kAlt.)
  // head_dim 257..512: two CTAs per Q tile, each owning half of O's columns
  // (TMEM cannot hold a 512-column fp32 O beside the S buffers); K streams in
  // units of 128 head_dim columns and V in units of 32 keys, so the whole
  // Q tile (up to 128 KB) stays resident.
  if (hdp > 256) {
    if (hdp <= 384)
      return a->precise ? L.run<FwdCfg<384, 64, 2, true, kSplit, 3, 3, 2, 2>>()
                        : L.run<FwdCfg<384, 64, 2, false, kSplit, 3, 3, 2, 2>>();
    return a->precise ? L.run<FwdCfg<512, 64, 2, true, kSplit, 3, 4, 2, 2>>()
                      : L.run<FwdCfg<512, 64, 2, false, kSplit, 3, 4, 2, 2>>();
  }
  // One softmax group per CTA and two CTAs per SM (head_dim 128) for grids
  // of at least two CTAs per SM whose CTAs see few keys: one CTA's prologue
  // and epilogue then overlap the other's main loop. Measured on B200: c2
  // (16 key tiles of 64 per CTA) 556 -> 616 TFLOP/s; with 32+ tiles of 128
  // (c3) the two-group kernel is 2% faster, and with one CTA per SM (c4)
  // the half-size rings keep too few bytes in flight (5.0 -> 3.5 TB/s).
  const int64_t ctas = static_cast<int64_t>((max_sq + p.QT - 1) / p.QT) * Hkv * a->batch;
  const int64_t keys_seen =
      p.window != kNoWindow ? std::min<int64_t>(max_sk, 2LL * p.window + p.QT) : max_sk;
  const bool one = hdp == 128 && ctas >= 2 * 148 && keys_seen <= 2048;
  if (one)
    return a->precise ? L.run<FwdCfg<128, 64, 2, true, kOne>>()
                      : L.run<FwdCfg<128, 64, 2, false, kOne>>();
  if (a->precise) {
    if (hdp == 64) return L.run<FwdCfg<64, 128, 2, true, kAlt>>();
    if (hdp == 128) return L.run<FwdCfg<128, 128, 2, true, kAlt>>();
    if (hdp == 192) return L.run<FwdCfg<192, 64, 2, true, kAlt>>();
    return L.run<FwdCfg<256, 64, 2, true, kSplit>>();
  }
  if (hdp == 64) return L.run<FwdCfg<64, 128, 2, false, kAlt>>();
  if (hdp == 128) return L.run<FwdCfg<128, 128, 2, false, kAlt>>();
  if (hdp == 192) return L.run<FwdCfg<192, 64, 2, false, kAlt>>();
  return L.run<FwdCfg<256, 64, 2, false, kSplit>>();
}

}  // namespace ca

namespace ca {
namespace {

// Whether the block path rotates Q inside the attention kernel (head_dim 128
// with rotation over the whole head, grids of at most 8 waves, at least 512
// keys); q_work is then neither written nor read. `vec`: every pointer is
// 16-byte aligned and rope_dim % 16 == 0.
bool block_fuses_q(const ca_block_args* a, bool vec) {
  const int H = a->n_head, Hkv = a->n_head_kv;
  if (!CA_FUSE_Q || !vec || a->head_dim != 128 || a->rope_dim != 128 || H / Hkv > 128 ||
      a->cu_active)
    return false;
  const long long fq_ctas = static_cast<long long>(a->batch) * Hkv *
                            ((a->n_active + 128 / (H / Hkv) - 1) / (128 / (H / Hkv)));
  return fq_ctas <= 148LL * 8 && a->n_total >= 512;
}

bool block_vec(const ca_block_args* a) {
  return aligned16(a->q) && aligned16(a->k) && aligned16(a->v) && aligned16(a->q_work) &&
         aligned16(a->cache_k) && aligned16(a->cache_v) && aligned16(a->rope) &&
         (!a->q_norm_w || aligned16(a->q_norm_w)) && (!a->k_norm_w || aligned16(a->k_norm_w)) &&
         a->rope_dim % 16 == 0;
}

int block_impl(const ca_block_args* a, cudaStream_t st) {
  if (!a || !a->q || !a->k || !a->v || !a->active_pos || !a->rope || !a->cache_k ||
      !a->cache_v || !a->q_work || !a->out)
    return CA_ERR_INVALID;
  const int H = a->n_head, Hkv = a->n_head_kv, hd = a->head_dim;
  const bool varlen = a->cu_active != nullptr;
  if (a->batch < 0 || H <= 0 || Hkv <= 0 || hd <= 0 || H % Hkv) return CA_ERR_INVALID;
  if (varlen ? (!a->cu_total || a->total_active < 0 || a->total_cache < 0 || a->max_active < 0)
             : (a->n_active < 0 || a->n_total < a->n_active))
    return CA_ERR_INVALID;
  if (a->rope_dim < 0 || a->rope_dim > hd || a->rope_dim % 2 || a->rope_len <= 0)
    return CA_ERR_INVALID;
  if (a->batch == 0 || (varlen ? a->total_active == 0 : a->n_active == 0)) return CA_OK;
  if (varlen && (a->total_active > INT_MAX || a->total_cache > INT_MAX)) return CA_ERR_UNSUPPORTED;
  PrepParams pp{};
  pp.q = static_cast<const __nv_bfloat16*>(a->q);
  pp.k = static_cast<const __nv_bfloat16*>(a->k);
  pp.v = static_cast<const __nv_bfloat16*>(a->v);
  pp.pos = a->active_pos;
  pp.q_norm_w = a->q_norm_w;
  pp.k_norm_w = a->k_norm_w;
  pp.v_norm = a->v_norm;
  pp.eps = a->rms_eps;
  pp.rope = a->rope;
  pp.rope_len = a->rope_len;
  pp.rope_dim = a->rope_dim;
  pp.q_out = static_cast<__nv_bfloat16*>(a->q_work);
  pp.cache_k = static_cast<__nv_bfloat16*>(a->cache_k);
  pp.cache_v = static_cast<__nv_bfloat16*>(a->cache_v);
  pp.batch = a->batch;
  pp.na = a->n_active;
  pp.n_total = a->n_total;
  pp.cu_active = a->cu_active;
  pp.cu_total = a->cu_total;
  pp.total_active = varlen ? a->total_active : 0;
  const bool vec = block_vec(a);
  // head_dim 128 with rotation over the whole head: the attention kernel
  // normalises and rotates its own Q tile (each Q row belongs to exactly one
  // CTA), so the pre-ops pass covers K and V only and Q never round-trips
  // through HBM; q_work is then unused.
  // The in-kernel pass lengthens every CTA's prologue, paid once per wave of
  // CTAs and not amortised over few key tiles: measured on B200 (bench.py
  // steps, same box) c2 (7 waves, 8 key tiles) -2.7%, c4 (1 wave, 33 tiles)
  // -1%, c1 (1 key tile) +7%, c3 (28 waves) +3%.
  const bool fuse_q = block_fuses_q(a, vec);
  const int Hp = fuse_q ? 0 : H;  // Q rows handled by the pre-ops pass
  pp.H = Hp;
  pp.Hkv = Hkv;
  pp.hd = hd;
  const long long toks =
      varlen ? a->total_active : static_cast<long long>(a->batch) * a->n_active;
  const long long jobs = toks * (Hp + 2 * Hkv);
  pp.err = a->status;
  const long long stage = static_cast<long long>(Hp + 2 * Hkv) * hd * 2;
  const size_t bulk_smem = kPrepStages * stage + 16 * kPrepStages;
  // Bulk-copy pre-ops (a shared-memory ring per CTA) at head_dim 256: c5's
  // layer block 4.59 ms against 4.75 with prep_pair_kernel. At head_dim 128
  // both forms are bound by the per-row arithmetic (f64 sum of squares,
  // shuffles), not by bytes in flight, and the token kernel measured 1.6%
  // faster (c3 block 1.345 vs 1.366 ms).
  // Ring form for full rotation on passes of at least 256K rows (c3: 1.6M
  // rows 0.245 -> 0.155 ms; c5: 1.0M rows per layer, 11.77 -> 11.32 ms per
  // step): as many tokens per stage as fit in 48 KB of rows (at most 16).
  // Short passes (c2's 32K and c4's 8K rows of K and V) measured 3-5 us
  // faster on the token kernel, whose many small jobs start at once.
  int ring_t = 0;
  if (vec && a->rope_dim == hd && (hd == 64 || hd == 128 || hd == 256) &&
      jobs >= 256LL * 1024) {
    const long long tok_bytes = static_cast<long long>(Hp + 2 * Hkv) * hd * 2;
    ring_t = static_cast<int>(std::min<long long>(16, 48 * 1024 / tok_bytes));
    while (ring_t > 0 && ring_smem_bytes(ring_t, Hp + 2 * Hkv, hd) > 227 * 1024) --ring_t;
  }
  if (CA_PREP_RING && ring_t > 0) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return CA_ERR_CUDA;
    const void* fn = hd == 64    ? reinterpret_cast<const void*>(prep_ring_kernel<64>)
                     : hd == 128 ? reinterpret_cast<const void*>(prep_ring_kernel<128>)
                                 : reinterpret_cast<const void*>(prep_ring_kernel<256>);
    const int fi = hd == 64 ? 0 : hd == 128 ? 1 : 2;
    static bool ring_attr[kMaxDevices][3] = {};
    const size_t smem = ring_smem_bytes(ring_t, Hp + 2 * Hkv, hd);
    if (!ring_attr[dev][fi]) {
      if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) !=
          cudaSuccess)
        return CA_ERR_CUDA;
      ring_attr[dev][fi] = true;
    }
    int per_sm = 1, n_sm = 148;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kRingThreads, smem) !=
            cudaSuccess ||
        per_sm < 1)
      per_sm = 1;
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
    const long long n_stage = (toks + ring_t - 1) / ring_t;
    const int blocks = static_cast<int>(std::min<long long>(n_stage, 1LL * n_sm * per_sm));
    if (hd == 64) prep_ring_kernel<64><<<blocks, kRingThreads, smem, st>>>(pp, ring_t);
    else if (hd == 128) prep_ring_kernel<128><<<blocks, kRingThreads, smem, st>>>(pp, ring_t);
    else prep_ring_kernel<256><<<blocks, kRingThreads, smem, st>>>(pp, ring_t);
  } else if (CA_PREP_BULK && vec && hd == 256 && bulk_smem <= 112 * 1024) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return CA_ERR_CUDA;
    static bool attr_done[kMaxDevices] = {};
    const void* fn = reinterpret_cast<const void*>(prep_bulk_kernel<32>);
    if (!attr_done[dev]) {
      if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 112 * 1024) !=
          cudaSuccess)
        return CA_ERR_CUDA;
      attr_done[dev] = true;
    }
    // Exactly one wave of resident CTAs (they stride over the tokens).
    int per_sm = 1, n_sm = 148;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kPrepThreads, bulk_smem) !=
            cudaSuccess ||
        per_sm < 1)
      per_sm = 1;
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
    const int blocks = static_cast<int>(std::min<long long>(toks, 1LL * n_sm * per_sm));
    prep_bulk_kernel<32><<<blocks, kPrepThreads, bulk_smem, st>>>(pp);
  } else if (vec && (hd == 64 || hd == 128 || hd == 256)) {
    // 16-row jobs unless that leaves fewer jobs than 64 warps per SM; then
    // one warp step per job (256 / head_dim rows).
    pp.rows_per_job = 16;
    if (toks * ((Hp + 2 * Hkv + 15) / 16) < 148LL * 64) pp.rows_per_job = 256 / hd;
    const long long pjobs =
        toks * ((Hp + 2 * Hkv + pp.rows_per_job - 1) / pp.rows_per_job);
    const int blocks = static_cast<int>(std::min<long long>((pjobs + 7) / 8, 148LL * 8));
    // head_dim 256 with full rotation: every NeoX pair inside one lane
    // (measured faster there; at 64 / 128 the partner-exchange form is).
    if (hd == 256 && a->rope_dim == hd) prep_pair_kernel<32><<<blocks, 256, 0, st>>>(pp);
    else if (hd == 64) prep_token_kernel<8><<<blocks, 256, 0, st>>>(pp);
    else if (hd == 128) prep_token_kernel<16><<<blocks, 256, 0, st>>>(pp);
    else prep_token_kernel<32><<<blocks, 256, 0, st>>>(pp);
  } else {
    const int blocks = static_cast<int>(std::min<long long>((jobs + 7) / 8, 148LL * 16));
    prep_block_kernel<<<blocks, 256, 8 * hd * sizeof(float), st>>>(pp);
  }
  if (cudaGetLastError() != cudaSuccess) return CA_ERR_CUDA;

  ca_dev_args d{};
  d.q = fuse_q ? a->q : a->q_work;
  d.k = a->cache_k;
  d.v = a->cache_v;
  d.out = a->out;
  d.out_f32 = a->out_f32;
  d.out_row_stride = a->out_row_stride;
  d.peer_out = a->peer_out;
  d.n_peer_out = a->n_peer_out;
  d.out_multicast = a->out_multicast;
  d.batch = a->batch;
  d.sq = a->n_active;
  d.sk = a->n_total;
  d.n_head = H;
  d.n_head_kv = Hkv;
  d.head_dim = hd;
  d.q_pos = a->active_pos;  // keys are positions 0..n_total-1 in order: k_pos = identity
  d.sliding_window = a->sliding_window;
  d.causal_prefix = a->causal_prefix;
  d.seq_prefix = a->seq_prefix;
  d.scale = a->scale;
  d.softcap = a->softcap;
  d.precise = a->precise;
  d.status = a->status;
  if (varlen) {  // keys of sequence b: its cache rows, positions 0.. in order
    d.cu_q = a->cu_active;
    d.cu_k = a->cu_total;
    d.total_q = a->total_active;
    d.total_k = a->total_cache;
    d.max_sq = a->max_active;
  }
  if (fuse_q) {
    const QFuse fq{a->q_norm_w, a->rope, a->rms_eps};
    return attention_dev_impl(&d, st, &fq);
  }
  return attention_dev_impl(&d, st);
}

// Library-owned device buffers of the host-buffer entry point, one set per
// device, grown on demand and kept for the process lifetime.
constexpr int kMaxChunks = 8;
struct HostCtx {
  std::mutex mu;
  cudaStream_t stream = nullptr;  // copies in
  cudaStream_t comp = nullptr;    // conversions + attention (pipelined calls)
  cudaStream_t outs = nullptr;    // copies out (pipelined calls)
  cudaEvent_t ev[2 * kMaxChunks + 1] = {};
  void* buf = nullptr;
  size_t cap = 0;
  uint16_t* pin = nullptr;  // pinned host staging of bf16-rounded Q/K/V
  size_t pin_cap = 0;
};
HostCtx g_host[kMaxDevices];

// Host rounding of the pipelined host-buffer calls (CA_HOST_ROUND=0 keeps
// fp32 over PCIe and rounds on the GPU).
bool host_round_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("CA_HOST_ROUND");
    return !(e && e[0] == '0');
  }();
  return on;
}

size_t align_up(size_t x) { return (x + 255) / 256 * 256; }

int host_f32_impl(float* out, const float* q, const float* k, const float* v, const ca_shape* s,
                  const ca_rows* qr, const ca_rows* kr) {
  if (!out || !q || !k || !v || !s || !qr || !kr) return CA_ERR_INVALID;
  if (s->nq < 0 || s->nk < 0 || s->n_head <= 0 || s->n_head_kv <= 0 || s->head_dim <= 0 ||
      s->n_head % s->n_head_kv)
    return CA_ERR_INVALID;
  if (s->nq == 0) return CA_OK;
  if ((s->nq > 0 && !qr->pos) || (s->nk > 0 && !kr->pos)) return CA_ERR_INVALID;
  if (s->nq > INT_MAX || s->nk > INT_MAX) return CA_ERR_UNSUPPORTED;
  const bool qseq = qr->seq && qr->n_seq > 0, kseq = kr->seq && kr->n_seq > 0;
  const bool qpre = qr->prefix && qr->n_prefix > 0;
  if ((qseq && qr->n_seq < static_cast<size_t>(s->nq)) ||
      (kseq && kr->n_seq < static_cast<size_t>(s->nk)) ||
      (qpre && qr->n_prefix < static_cast<size_t>(s->nq)))
    return CA_ERR_INVALID;
  // Row metadata to int32 on the host; positions and ids must fit.
  const int64_t nq = s->nq, nk = s->nk;
  std::vector<int32_t> meta;
  meta.reserve(3 * nq + 2 * nk);
  auto push = [&](const int64_t* src, int64_t n, bool is_prefix) -> bool {
    for (int64_t i = 0; i < n; ++i) {
      int64_t x = src[i];
      if (x < 0) return false;
      if (x > INT_MAX) {
        if (!is_prefix) return false;
        x = INT_MAX;
      }
      meta.push_back(static_cast<int32_t>(x));
    }
    return true;
  };
  // Positions are usize: they must fit int32 here.
  if (!push(qr->pos, nq, false) || !push(kr->pos, nk, false)) return CA_ERR_UNSUPPORTED;
  const size_t off_qseq = meta.size();
  if (qseq && !push(qr->seq, nq, false)) return CA_ERR_UNSUPPORTED;
  const size_t off_kseq = meta.size();
  if (kseq && !push(kr->seq, nk, false)) return CA_ERR_UNSUPPORTED;
  const size_t off_qpre = meta.size();
  if (qpre && !push(qr->prefix, nq, true)) return CA_ERR_UNSUPPORTED;
  // A single non-empty seq side compares against id 0 on the other side.
  std::vector<int32_t> zeros;

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev >= kMaxDevices) return CA_ERR_CUDA;
  HostCtx& c = g_host[dev];
  std::lock_guard<std::mutex> lock(c.mu);
  if (!c.stream && cudaStreamCreateWithFlags(&c.stream, cudaStreamNonBlocking) != cudaSuccess)
    return CA_ERR_CUDA;
  if (s->head_dim > 4096) return CA_ERR_UNSUPPORTED;
  const int hd = static_cast<int>(s->head_dim);
  const int hd_p = (hd + 7) / 8 * 8;  // TMA rows must be 16-byte multiples
  const int64_t qe = nq * s->n_head * hd, ke = nk * s->n_head_kv * hd;
  const int64_t qe_p = nq * s->n_head * hd_p, ke_p = nk * s->n_head_kv * hd_p;
  const size_t b_qf = align_up(qe * 4), b_kf = align_up(ke * 4);
  const size_t b_qh = align_up(qe_p * 2), b_kh = align_up(ke_p * 2);
  const size_t b_out = hd_p == hd ? 0 : align_up(qe_p * 4);
  // Metadata, the zero ids of a one-sided seq test, and this call's status word.
  const size_t b_meta = align_up(meta.size() * 4 + 4 * (nq + nk) + 4);
  // Layout: [q f32 | k f32 | v f32 | q bf16 | k bf16 | v bf16 | out f32 | meta].
  // With no padding the fp32 output overwrites the fp32 Q staging copy.
  const size_t need = b_qf + 2 * b_kf + b_qh + 2 * b_kh + b_out + b_meta;
  if (need > c.cap) {
    if (c.buf) cudaFree(c.buf);
    c.buf = nullptr;
    c.cap = 0;
    if (cudaMalloc(&c.buf, need) != cudaSuccess) return CA_ERR_NOMEM;
    c.cap = need;
  }
  char* base = static_cast<char*>(c.buf);
  size_t off = 0;
  auto carve = [&](size_t bytes) { char* r = base + off; off += bytes; return r; };
  float* dq = reinterpret_cast<float*>(carve(b_qf));
  float* dk = reinterpret_cast<float*>(carve(b_kf));
  float* dv = reinterpret_cast<float*>(carve(b_kf));
  __nv_bfloat16* hq = reinterpret_cast<__nv_bfloat16*>(carve(b_qh));
  __nv_bfloat16* hk = reinterpret_cast<__nv_bfloat16*>(carve(b_kh));
  __nv_bfloat16* hv = reinterpret_cast<__nv_bfloat16*>(carve(b_kh));
  float* dout = b_out ? reinterpret_cast<float*>(carve(b_out)) : dq;
  int32_t* dmeta = reinterpret_cast<int32_t*>(carve(b_meta));
  int32_t* dzero = dmeta + meta.size();
  int32_t* dstatus = dzero + nq + nk;
  // Reads this call's status word after the stream work is done.
  auto call_status = [&]() -> int {
    int32_t derr = 0;
    if (cudaMemcpy(&derr, dstatus, sizeof(derr), cudaMemcpyDeviceToHost) != cudaSuccess)
      return CA_ERR_CUDA;
    return derr == 0 ? CA_OK : CA_ERR_TIMEOUT;
  };
  cudaStream_t st = c.stream;
  // Large calls without head_dim padding run as a pipeline over chunks of
  // query rows on three streams: K, V and the row metadata are copied in
  // first; then per chunk the Q rows are copied in (stream `stream`),
  // converted and attended over all keys (`comp`), and the output rows are
  // copied out (`outs`) while later chunks are still arriving. Rows are
  // independent (attention.rs:116), so the results equal the one-shot form.
  const int64_t q_bytes = qe * 4;
  const int n_chunks =
      (hd_p == hd && nk > 0 && q_bytes >= (16ll << 20))
          ? static_cast<int>(std::min<int64_t>(kMaxChunks, std::max<int64_t>(2, q_bytes >> 22)))
          : 1;
  if (n_chunks > 1) {
    // On an error, drain what was queued so the next call cannot overlap it.
    auto fail = [&](int rc) {
      cudaStreamSynchronize(st);
      if (c.comp) cudaStreamSynchronize(c.comp);
      if (c.outs) cudaStreamSynchronize(c.outs);
      return rc;
    };
    if (!c.comp && cudaStreamCreateWithFlags(&c.comp, cudaStreamNonBlocking) != cudaSuccess)
      return CA_ERR_CUDA;
    if (!c.outs && cudaStreamCreateWithFlags(&c.outs, cudaStreamNonBlocking) != cudaSuccess)
      return CA_ERR_CUDA;
    for (auto& e : c.ev)
      if (!e && cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess)
        return CA_ERR_CUDA;
    const int64_t row_e = s->n_head * hd;  // elements per query row
    const int64_t rows_per = (nq + n_chunks - 1) / n_chunks;
    // Q, K and V are rounded to bf16 by host threads into pinned staging
    // and cross PCIe as bf16 (half the bytes; the copy engine then reads
    // pinned memory directly), the next chunk being rounded while the
    // current one is in flight. The rounding equals the GPU's, so the
    // kernels see the same operands as with fp32 copies.
    const size_t pin_need = static_cast<size_t>(2 * ke + qe) * 2;
    bool hr = host_round_enabled();
    if (hr && pin_need > c.pin_cap) {
      if (c.pin) cudaFreeHost(c.pin);
      c.pin = nullptr;
      c.pin_cap = 0;
      if (cudaHostAlloc(reinterpret_cast<void**>(&c.pin), pin_need, cudaHostAllocDefault) ==
          cudaSuccess)
        c.pin_cap = pin_need;
      else
        cudaGetLastError();  // fall back to fp32 copies
    }
    hr = hr && c.pin_cap >= pin_need;
    uint16_t* pk = hr ? c.pin : nullptr;
    uint16_t* pv = hr ? c.pin + ke : nullptr;
    uint16_t* pq = hr ? c.pin + 2 * ke : nullptr;
    // One rounding job for the whole call: K and V in pieces of at most 2M
    // elements, then each Q chunk; a piece is copied as soon as it is rounded.
    std::vector<RoundSeg> segs;
    std::vector<__nv_bfloat16*> seg_dev;
    int kv_segs = 0;
    if (hr) {
      constexpr int64_t kPiece = 1 << 20;
      for (int t = 0; t < 2; ++t)
        for (int64_t o = 0; o < ke; o += kPiece) {
          segs.push_back({(t ? v : k) + o, (t ? pv : pk) + o,
                          static_cast<size_t>(std::min(kPiece, ke - o))});
          seg_dev.push_back((t ? hv : hk) + o);
        }
      kv_segs = static_cast<int>(segs.size());
      for (int ch = 0; ch < n_chunks; ++ch) {
        const int64_t r0 = ch * rows_per, rows = std::min<int64_t>(rows_per, nq - r0);
        if (rows <= 0) break;
        segs.push_back({q + r0 * row_e, pq + r0 * row_e, static_cast<size_t>(rows * row_e)});
        seg_dev.push_back(hq + r0 * row_e);
      }
    }
    std::unique_ptr<RoundBatch> rb(hr ? new RoundBatch(segs.data(), static_cast<int>(segs.size()))
                                      : nullptr);
    bool okp = cudaMemcpyAsync(dmeta, meta.data(), meta.size() * 4, cudaMemcpyHostToDevice,
                               st) == cudaSuccess;
    if (hr) {
      for (int i = 0; i < kv_segs; ++i) {
        rb->wait(i);
        okp = okp && cudaMemcpyAsync(seg_dev[i], segs[i].dst, segs[i].n * 2,
                                     cudaMemcpyHostToDevice, st) == cudaSuccess;
      }
    } else {
      okp = okp && cudaMemcpyAsync(dk, k, ke * 4, cudaMemcpyHostToDevice, st) == cudaSuccess &&
            cudaMemcpyAsync(dv, v, ke * 4, cudaMemcpyHostToDevice, st) == cudaSuccess;
    }
    if (okp && qseq != kseq) okp = cudaMemsetAsync(dzero, 0, 4 * (nq + nk), st) == cudaSuccess;
    okp = okp && cudaMemsetAsync(dstatus, 0, 4, st) == cudaSuccess;
    okp = okp && cudaEventRecord(c.ev[2 * kMaxChunks], st) == cudaSuccess &&
          cudaStreamWaitEvent(c.comp, c.ev[2 * kMaxChunks], 0) == cudaSuccess;
    if (!okp) return fail(CA_ERR_CUDA);
    const int kblocks = static_cast<int>(std::min<long long>((ke / 4 + 255) / 256 + 1, 148 * 8));
    if (!hr) {
      f32_to_bf16_kernel<<<kblocks, 256, 0, c.comp>>>(dk, hk, ke);
      f32_to_bf16_kernel<<<kblocks, 256, 0, c.comp>>>(dv, hv, ke);
    }
    for (int ch = 0; ch < n_chunks; ++ch) {
      const int64_t r0 = ch * rows_per;
      const int64_t rows = std::min<int64_t>(rows_per, nq - r0);
      if (rows <= 0) break;
      const int64_t e0 = r0 * row_e, n = rows * row_e;
      cudaEvent_t in_done = c.ev[2 * ch], att_done = c.ev[2 * ch + 1];
      if (hr) {
        rb->wait(kv_segs + ch);
        okp = cudaMemcpyAsync(hq + e0, pq + e0, n * 2, cudaMemcpyHostToDevice, st) == cudaSuccess;
      } else {
        okp = cudaMemcpyAsync(dq + e0, q + e0, n * 4, cudaMemcpyHostToDevice, st) == cudaSuccess;
      }
      okp = okp && cudaEventRecord(in_done, st) == cudaSuccess &&
            cudaStreamWaitEvent(c.comp, in_done, 0) == cudaSuccess;
      if (!okp) return fail(CA_ERR_CUDA);
      const int qblocks = static_cast<int>(std::min<long long>((n / 4 + 255) / 256 + 1, 148 * 8));
      if (!hr) f32_to_bf16_kernel<<<qblocks, 256, 0, c.comp>>>(dq + e0, hq + e0, n);
      if (cudaGetLastError() != cudaSuccess) return fail(CA_ERR_CUDA);
      ca_dev_args d{};
      d.q = hq + e0;
      d.k = hk;
      d.v = hv;
      d.out = dout + e0;
      d.out_f32 = 1;
      d.precise = 1;
      d.batch = 1;
      d.sq = static_cast<int32_t>(rows);
      d.sk = static_cast<int32_t>(nk);
      d.n_head = static_cast<int32_t>(s->n_head);
      d.n_head_kv = static_cast<int32_t>(s->n_head_kv);
      d.head_dim = hd;
      d.q_pos = dmeta + r0;
      d.k_pos = dmeta + nq;
      d.q_seq = qseq ? dmeta + off_qseq + r0 : (kseq ? dzero + r0 : nullptr);
      d.k_seq = kseq ? dmeta + off_kseq : (qseq ? dzero : nullptr);
      d.q_prefix = qpre ? dmeta + off_qpre + r0 : nullptr;
      d.sliding_window = s->sliding_window;
      d.causal_prefix = s->causal_prefix;
      d.scale = s->scale;
      d.softcap = s->softcap;
      d.status = dstatus;
      const int rc = attention_dev_impl(&d, c.comp);
      if (rc != CA_OK) return fail(rc);
      okp = cudaEventRecord(att_done, c.comp) == cudaSuccess &&
            cudaStreamWaitEvent(c.outs, att_done, 0) == cudaSuccess &&
            cudaMemcpyAsync(out + e0, dout + e0, n * 4, cudaMemcpyDeviceToHost, c.outs) ==
                cudaSuccess;
      if (!okp) return fail(CA_ERR_CUDA);
    }
    if (cudaStreamSynchronize(c.outs) != cudaSuccess ||
        cudaStreamSynchronize(c.comp) != cudaSuccess || cudaStreamSynchronize(st) != cudaSuccess)
      return fail(CA_ERR_CUDA);
    return call_status();
  }
  // Calls of a few MB and up without head_dim padding round on the host too
  // (see the pipelined form): one job, each of Q, K, V copied once rounded.
  const size_t one_pin = static_cast<size_t>(qe + 2 * ke) * 2;
  bool hr1 = host_round_enabled() && hd_p == hd && ke > 0 && one_pin >= (4u << 20);
  if (hr1 && one_pin > c.pin_cap) {
    if (c.pin) cudaFreeHost(c.pin);
    c.pin = nullptr;
    c.pin_cap = 0;
    if (cudaHostAlloc(reinterpret_cast<void**>(&c.pin), one_pin, cudaHostAllocDefault) ==
        cudaSuccess)
      c.pin_cap = one_pin;
    else
      cudaGetLastError();
  }
  hr1 = hr1 && c.pin_cap >= one_pin;
  bool ok = true;
  if (hr1) {
    const RoundSeg segs[3] = {{k, c.pin, static_cast<size_t>(ke)},
                              {v, c.pin + ke, static_cast<size_t>(ke)},
                              {q, c.pin + 2 * ke, static_cast<size_t>(qe)}};
    __nv_bfloat16* devs[3] = {hk, hv, hq};
    RoundBatch rb(segs, 3);
    for (int i = 0; i < 3; ++i) {
      rb.wait(i);
      ok = ok && cudaMemcpyAsync(devs[i], segs[i].dst, segs[i].n * 2, cudaMemcpyHostToDevice,
                                 st) == cudaSuccess;
    }
  } else {
    ok = cudaMemcpyAsync(dq, q, qe * 4, cudaMemcpyHostToDevice, st) == cudaSuccess;
    ok = ok && (ke == 0 || cudaMemcpyAsync(dk, k, ke * 4, cudaMemcpyHostToDevice, st) ==
                               cudaSuccess);
    ok = ok && (ke == 0 || cudaMemcpyAsync(dv, v, ke * 4, cudaMemcpyHostToDevice, st) ==
                               cudaSuccess);
  }
  ok = ok && cudaMemcpyAsync(dmeta, meta.data(), meta.size() * 4, cudaMemcpyHostToDevice, st) ==
                 cudaSuccess;
  if ((qseq != kseq) && ok)
    ok = cudaMemsetAsync(dzero, 0, 4 * (nq + nk), st) == cudaSuccess;
  ok = ok && cudaMemsetAsync(dstatus, 0, 4, st) == cudaSuccess;
  if (!ok) return CA_ERR_CUDA;
  auto conv = [&](const float* src, __nv_bfloat16* dst, long long n, long long n_p) {
    const int blocks = static_cast<int>(std::min<long long>((n_p / 4 + 255) / 256 + 1, 148 * 8));
    if (hd_p == hd)
      f32_to_bf16_kernel<<<blocks, 256, 0, st>>>(src, dst, n);
    else
      f32_to_bf16_pad_kernel<<<blocks, 256, 0, st>>>(src, dst, n / hd, hd, hd_p);
  };
  if (!hr1) {
    conv(dq, hq, qe, qe_p);
    if (ke > 0) {
      conv(dk, hk, ke, ke_p);
      conv(dv, hv, ke, ke_p);
    }
  }
  if (cudaGetLastError() != cudaSuccess) return CA_ERR_CUDA;
  ca_dev_args d{};
  d.q = hq;
  d.k = hk;
  d.v = hv;
  d.out = dout;
  d.out_f32 = 1;
  d.precise = 1;
  d.batch = 1;
  d.sq = static_cast<int32_t>(nq);
  d.sk = static_cast<int32_t>(nk);
  d.n_head = static_cast<int32_t>(s->n_head);
  d.n_head_kv = static_cast<int32_t>(s->n_head_kv);
  d.head_dim = hd_p;
  d.q_pos = dmeta;
  d.k_pos = dmeta + nq;
  d.q_seq = qseq ? dmeta + off_qseq : (kseq ? dzero : nullptr);
  d.k_seq = kseq ? dmeta + off_kseq : (qseq ? dzero : nullptr);
  d.q_prefix = qpre ? dmeta + off_qpre : nullptr;
  d.sliding_window = s->sliding_window;
  d.causal_prefix = s->causal_prefix;
  d.scale = s->scale;
  d.softcap = s->softcap;
  d.status = dstatus;
  int rc = nk == 0 ? CA_OK : attention_dev_impl(&d, st);
  if (rc != CA_OK) return rc;
  if (nk == 0) {  // no key at all: every row is 0 * (1 / 0)
    std::vector<float> nan(qe, std::nanf(""));
    std::memcpy(out, nan.data(), qe * 4);
    return cudaStreamSynchronize(st) == cudaSuccess ? CA_OK : CA_ERR_CUDA;
  }
  if (hd_p == hd) {
    if (cudaMemcpyAsync(out, dout, qe * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess)
      return CA_ERR_CUDA;
  } else if (cudaMemcpy2DAsync(out, hd * 4, dout, hd_p * 4, hd * 4, nq * s->n_head,
                               cudaMemcpyDeviceToHost, st) != cudaSuccess) {
    return CA_ERR_CUDA;
  }
  if (cudaStreamSynchronize(st) != cudaSuccess) return CA_ERR_CUDA;
  return call_status();
}

}  // namespace
}  // namespace ca

namespace ca {
namespace {

// Scratch of ca_attention_block_dev_noalloc: the post-norm, post-RoPE Q of
// one call. In host code this name is only a stand-in for the per-device
// copy; its device address comes from cudaGetSymbolAddress below.
constexpr size_t kNoAllocElems = CA_NOALLOC_SCRATCH_BYTES / sizeof(__nv_bfloat16);
static __device__ __align__(256) __nv_bfloat16 g_noalloc_qwork[kNoAllocElems];

// Per-device address of g_noalloc_qwork. Only a successful lookup is
// cached: a failed one (for example a first call made while the stream is
// being captured) is retried by the next call.
struct NoAllocSlot {
  std::mutex mu;
  void* ptr = nullptr;
};
NoAllocSlot g_noalloc[kMaxDevices];

int noalloc_scratch(int dev, void** out) {
  NoAllocSlot& slot = g_noalloc[dev];
  std::lock_guard<std::mutex> lock(slot.mu);
  if (!slot.ptr) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_qwork) != cudaSuccess || !ptr) {
      cudaGetLastError();  // clear the error so that it does not surface in a later call
      return CA_ERR_CUDA;
    }
    slot.ptr = ptr;
  }
  *out = slot.ptr;
  return CA_OK;
}

int noalloc_impl(const ca_block_args* a, cudaStream_t st) {
  if (!a) return CA_ERR_INVALID;
  if (a->q_work) return CA_ERR_INVALID;  // the library supplies the scratch
  if (a->batch < 0 || a->n_active < 0 || (a->cu_active && a->total_active < 0) ||
      a->n_head <= 0 || a->n_head_kv <= 0 ||
      a->head_dim <= 0)
    return CA_ERR_INVALID;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return CA_ERR_CUDA;
  void* scratch = nullptr;
  const int rc = noalloc_scratch(dev, &scratch);
  if (rc != CA_OK) return rc;
  ca_block_args b = *a;
  b.q_work = scratch;
  // The scratch holds the rotated queries only when the pre-ops pass writes
  // them; calls that rotate Q inside the attention kernel read none of it.
  // The size test divides step by step so that no product can wrap.
  if (!block_fuses_q(&b, block_vec(&b))) {
    unsigned long long room = kNoAllocElems;
    const int64_t f[4] = {a->cu_active ? 1 : a->batch,
                          a->cu_active ? a->total_active : a->n_active, a->n_head, a->head_dim};
    const bool empty = f[0] == 0 || f[1] == 0;
    for (int i = 0; i < 4 && !empty; ++i) {
      if (static_cast<unsigned long long>(f[i]) > room) return CA_ERR_SCRATCH;
      room /= static_cast<unsigned long long>(f[i]);
    }
  }
  return block_impl(&b, st);
}

// Failure-detection self-test: one CTA waits on an mbarrier that nothing
// arrives on, through the same bounded wait (mbar_wait_limit) every pipeline
// wait in the attention kernel uses, with a caller-chosen limit. The wait
// gives up, stores CA_ERR_TIMEOUT in the device error word and the kernel
// returns normally: the host sees the expiry through ca_device_status and
// the context stays usable. No trap, fault or unbounded loop is involved.
__global__ void selftest_wait_kernel(uint64_t limit_ns, int* status) {
  __shared__ __align__(8) uint64_t never;
  const uint32_t bar = smem_u32(&never);
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  bool dead = false;
  mbar_wait_limit(bar, 0, dead, limit_ns, status);
}

}  // namespace
}  // namespace ca

namespace ca {
namespace {

typedef CUresult (*AddrRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

AddrRangeFn addr_range_fn() {
  static AddrRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddrRangeFn>(p);
  });
  return fn;
}

// Pointers ca_ipc_import returned -> the mapped allocation base to close.
std::mutex g_ipc_mu;
std::vector<std::pair<void*, void*>> g_ipc_maps;

}  // namespace
}  // namespace ca

extern "C" {

int ca_ipc_export(const void* dev_ptr, void* handle, uint64_t* offset) {
  static_assert(sizeof(cudaIpcMemHandle_t) <= CA_IPC_HANDLE_BYTES, "IPC handle size");
  if (!dev_ptr || !handle || !offset) return CA_ERR_INVALID;
  ca::AddrRangeFn fn = ca::addr_range_fn();
  if (!fn) return CA_ERR_CUDA;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (fn(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS)
    return CA_ERR_INVALID;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) {
    cudaGetLastError();
    return CA_ERR_CUDA;
  }
  std::memset(handle, 0, CA_IPC_HANDLE_BYTES);
  std::memcpy(handle, &h, sizeof(h));
  *offset = reinterpret_cast<uint64_t>(dev_ptr) - static_cast<uint64_t>(base);
  return CA_OK;
}

int ca_ipc_import(const void* handle, uint64_t offset, void** dev_ptr) {
  if (!handle || !dev_ptr) return CA_ERR_INVALID;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  if (cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    cudaGetLastError();
    return CA_ERR_CUDA;
  }
  void* p = static_cast<char*>(base) + offset;
  std::lock_guard<std::mutex> lock(ca::g_ipc_mu);
  ca::g_ipc_maps.emplace_back(p, base);
  *dev_ptr = p;
  return CA_OK;
}

int ca_ipc_close(void* dev_ptr) {
  void* base = nullptr;
  {
    std::lock_guard<std::mutex> lock(ca::g_ipc_mu);
    for (size_t i = 0; i < ca::g_ipc_maps.size(); ++i)
      if (ca::g_ipc_maps[i].first == dev_ptr) {
        base = ca::g_ipc_maps[i].second;
        ca::g_ipc_maps.erase(ca::g_ipc_maps.begin() + i);
        break;
      }
  }
  if (!base) return CA_ERR_INVALID;
  return cudaIpcCloseMemHandle(base) == cudaSuccess ? CA_OK : CA_ERR_CUDA;
}

int ca_candidate_stats(const ca_cand_args* a, void* stream) {
  if (!a || !a->logits || !a->rows || !a->token || a->n_cand < 0 || a->n_vocab <= 0 ||
      a->n_vocab > INT_MAX || a->n_suppress < 0 || (a->n_suppress > 0 && !a->suppress))
    return CA_ERR_INVALID;
  if ((a->want_entropy && !a->entropy) || (a->want_prob && !a->prob)) return CA_ERR_INVALID;
  const int64_t rs = a->row_stride ? a->row_stride : a->n_vocab;
  if (rs < a->n_vocab) return CA_ERR_INVALID;
  if (a->n_cand == 0) return CA_OK;
  ca::CandParams p{};
  p.logits = a->logits;
  p.n_vocab = a->n_vocab;
  p.row_stride = rs;
  p.rows = a->rows;
  p.n_cand = a->n_cand;
  p.mask_id = a->mask_id;
  p.suppress = a->suppress;
  p.n_suppress = a->n_suppress;
  p.want_entropy = a->want_entropy;
  p.want_prob = a->want_prob;
  p.token = a->token;
  p.entropy = a->entropy;
  p.margin = a->margin;
  p.prob = a->prob;
  const int grid = std::min(a->n_cand, 148);
  ca::cand_stats_kernel<<<grid, ca::kCandThreads, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return cudaGetLastError() == cudaSuccess ? CA_OK : CA_ERR_CUDA;
}

// tokens_to_unmask (src/model/sampler.rs:115-132) in f32 as the reference.
int64_t ca_tokens_to_unmask(int64_t step, int64_t total_steps, int64_t masked, int32_t schedule) {
  if (step < 0 || total_steps < 0 || masked < 0 || (schedule != 0 && schedule != 1))
    return CA_ERR_INVALID;
  const int64_t steps_left = std::max<int64_t>(total_steps > step ? total_steps - step : 0, 1);
  const float t0 = static_cast<float>(step) / static_cast<float>(total_steps);
  const float t1 = static_cast<float>(step + 1) / static_cast<float>(total_steps);
  float frac;
  if (schedule == CA_SCHEDULE_COSINE) {
    const float half_pi = 1.57079632679489661923f;
    const float c0 = std::max(cosf(t0 * half_pi), 1e-6f);
    const float c1 = cosf(t1 * half_pi);
    frac = (c0 - c1) / c0;
  } else {
    frac = 1.0f / static_cast<float>(steps_left);
  }
  const float nf = roundf(frac * static_cast<float>(masked));
  // `as usize` saturates: NaN and negatives become 0.
  int64_t n = (nf != nf || nf <= 0.f) ? 0 : static_cast<int64_t>(nf);
  n = std::max<int64_t>(n, masked > 0 ? 1 : 0);
  return std::min<int64_t>(n, masked);
}

int ca_dequantize(int32_t qtype, const void* src, int64_t rows, int64_t cols,
                  const int32_t* row_ids, int64_t n_out, void* dst, int32_t dst_f32,
                  int64_t dst_stride, float scale, int32_t* status, void* stream) {
  using namespace ca;
  if (!src || !dst || rows < 0 || cols <= 0 || n_out < 0) return CA_ERR_INVALID;
  const int64_t unit = qtype == kQ4_K || qtype == kQ6_K ? 256
                       : qtype == kQ4_0 || qtype == kQ8_0 ? 32
                       : qtype == kQF16 ? 8 : 0;
  if (!unit) return CA_ERR_UNSUPPORTED;
  if (cols % unit) return CA_ERR_INVALID;
  const int64_t ds = dst_stride ? dst_stride : cols;
  if (ds < cols || ds % 8 || (reinterpret_cast<uintptr_t>(dst) & 15u)) return CA_ERR_INVALID;
  if (!row_ids && n_out > rows) return CA_ERR_INVALID;
  // Q4_K blocks are read with 32- and 64-bit loads.
  if (qtype == kQ4_K && (reinterpret_cast<uintptr_t>(src) & 7u)) return CA_ERR_INVALID;
  if (n_out == 0) return CA_OK;
  DequantParams p{};
  p.src = static_cast<const uint8_t*>(src);
  p.rows = rows;
  p.cols = cols;
  p.row_ids = row_ids;
  p.n_out = n_out;
  p.dst = dst;
  p.dst_f32 = dst_f32 ? 1 : 0;
  p.dst_stride = ds;
  p.scale = scale;
  p.qtype = qtype;
  p.err = status;
  const long long items = n_out * (((cols + 255) / 256 + kUnits - 1) / kUnits);
  if (items > UINT_MAX / 2) return CA_ERR_UNSUPPORTED;  // 32-bit work-item indices
  const int blocks = static_cast<int>(std::min<long long>((items + 7) / 8, 148LL * 16));
  dequant_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return cudaGetLastError() == cudaSuccess ? CA_OK : CA_ERR_CUDA;
}

}  // extern "C"

namespace ca {
namespace {

// cuBLASLt state of one device: handle, a 32 MiB workspace, and an fp32
// accumulator buffer for bf16 outputs with a bias (grown on demand), created
// on first use and kept for the process lifetime.
struct LtCtx {
  std::mutex mu;
  cublasLtHandle_t h = nullptr;
  void* ws = nullptr;
  size_t ws_bytes = 0;
  float* acc = nullptr;
  size_t acc_elems = 0;
};
LtCtx g_lt[kMaxDevices];

// out[t, r] = bf16(acc[t, r] + bias[r] (+ residual[t, r])): one rounding.
__global__ void bias_epilogue_kernel(const float* acc, const float* bias,
                                     const __nv_bfloat16* residual, __nv_bfloat16* out,
                                     long long n, long long rows) {
  const long long total = n * rows;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float v = __fadd_rn(acc[i], bias[i % rows]);
    if (residual) v = __fadd_rn(v, __bfloat162float(residual[i]));
    out[i] = __float2bfloat16_rn(v);
  }
}

int linear_impl(const ca_linear_args* a, cudaStream_t st) {
  if (!a || !a->act || !a->w || !a->out || a->n < 0 || a->rows <= 0 || a->cols <= 0)
    return CA_ERR_INVALID;
  if (a->n == 0) return CA_OK;
  const int64_t as = a->act_stride ? a->act_stride : a->cols;
  if (as < a->cols) return CA_ERR_INVALID;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return CA_ERR_CUDA;
  LtCtx& c = g_lt[dev];
  std::lock_guard<std::mutex> lock(c.mu);
  if (!c.h) {
    if (cublasLtCreate(&c.h) != CUBLAS_STATUS_SUCCESS) return CA_ERR_CUDA;
    c.ws_bytes = 32u << 20;
    if (cudaMalloc(&c.ws, c.ws_bytes) != cudaSuccess) {
      c.ws = nullptr;
      c.ws_bytes = 0;
    }
  }
  // bf16 output with a bias: cuBLASLt's bias epilogue wants a bf16 bias
  // there, so the product goes to an fp32 buffer and one kernel adds the
  // fp32 bias and the residual with a single rounding.
  const bool split = !a->out_f32 && a->bias;
  if (split) {
    const size_t need = static_cast<size_t>(a->n) * static_cast<size_t>(a->rows);
    if (need > c.acc_elems) {
      if (c.acc) cudaFree(c.acc);
      c.acc = nullptr;
      c.acc_elems = 0;
      if (cudaMalloc(&c.acc, need * sizeof(float)) != cudaSuccess) return CA_ERR_NOMEM;
      c.acc_elems = need;
    }
  }
  // Row-major out[n, rows] = act[n, cols] . W[rows, cols]^T is, column-major,
  // D[rows, n] = W^T(op T on a [cols, rows] matrix) x act^T ([cols, n]).
  const cudaDataType_t dt = (a->out_f32 || split) ? CUDA_R_32F : CUDA_R_16BF;
  cublasLtMatmulDesc_t op = nullptr;
  cublasLtMatrixLayout_t la = nullptr, lb = nullptr, lc = nullptr;
  cublasLtMatmulPreference_t pref = nullptr;
  int rc = CA_ERR_CUDA;
  do {
    if (cublasLtMatmulDescCreate(&op, CUBLAS_COMPUTE_32F, CUDA_R_32F) != CUBLAS_STATUS_SUCCESS) break;
    const cublasOperation_t tA = CUBLAS_OP_T, tB = CUBLAS_OP_N;
    cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_TRANSA, &tA, sizeof(tA));
    cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_TRANSB, &tB, sizeof(tB));
    if (a->bias && !split) {
      const cublasLtEpilogue_t ep = CUBLASLT_EPILOGUE_BIAS;
      const cudaDataType_t bt = CUDA_R_32F;
      cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_EPILOGUE, &ep, sizeof(ep));
      cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_BIAS_POINTER, &a->bias,
                                     sizeof(a->bias));
      cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_BIAS_DATA_TYPE, &bt, sizeof(bt));
    }
    if (cublasLtMatrixLayoutCreate(&la, CUDA_R_16BF, a->cols, a->rows, a->cols) !=
            CUBLAS_STATUS_SUCCESS ||
        cublasLtMatrixLayoutCreate(&lb, CUDA_R_16BF, a->cols, a->n, as) != CUBLAS_STATUS_SUCCESS ||
        cublasLtMatrixLayoutCreate(&lc, dt, a->rows, a->n, a->rows) != CUBLAS_STATUS_SUCCESS)
      break;
    if (cublasLtMatmulPreferenceCreate(&pref) != CUBLAS_STATUS_SUCCESS) break;
    cublasLtMatmulPreferenceSetAttribute(pref, CUBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES,
                                         &c.ws_bytes, sizeof(c.ws_bytes));
    cublasLtMatmulHeuristicResult_t heur;
    int found = 0;
    if (cublasLtMatmulAlgoGetHeuristic(c.h, op, la, lb, lc, lc, pref, 1, &heur, &found) !=
            CUBLAS_STATUS_SUCCESS ||
        found == 0) {
      rc = CA_ERR_UNSUPPORTED;
      break;
    }
    const float alpha = 1.f, beta = (a->residual && !split) ? 1.f : 0.f;
    void* dptr = split ? static_cast<void*>(c.acc) : a->out;
    const void* cptr = (a->residual && !split) ? a->residual : dptr;
    if (cublasLtMatmul(c.h, op, &alpha, a->w, la, a->act, lb, &beta, cptr, lc, dptr, lc,
                       &heur.algo, c.ws, c.ws_bytes, st) != CUBLAS_STATUS_SUCCESS)
      break;
    if (split) {
      const long long total = a->n * a->rows;
      const int blocks = static_cast<int>(std::min<long long>((total + 255) / 256, 148LL * 16));
      bias_epilogue_kernel<<<blocks, 256, 0, st>>>(
          c.acc, a->bias, static_cast<const __nv_bfloat16*>(a->residual),
          static_cast<__nv_bfloat16*>(a->out), a->n, a->rows);
      if (cudaGetLastError() != cudaSuccess) break;
    }
    rc = CA_OK;
  } while (false);
  if (pref) cublasLtMatmulPreferenceDestroy(pref);
  if (lc) cublasLtMatrixLayoutDestroy(lc);
  if (lb) cublasLtMatrixLayoutDestroy(lb);
  if (la) cublasLtMatrixLayoutDestroy(la);
  if (op) cublasLtMatmulDescDestroy(op);
  return rc;
}

}  // namespace
}  // namespace ca

extern "C" {

int ca_linear(const ca_linear_args* a, void* stream) {
  return ca::linear_impl(a, static_cast<cudaStream_t>(stream));
}

int ca_selftest_wait_timeout(int64_t limit_ns, void* stream) {
  if (limit_ns <= 0 || limit_ns > 1000000000ll) return CA_ERR_INVALID;
  ca::selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<uint64_t>(limit_ns), nullptr);
  return cudaGetLastError() == cudaSuccess ? CA_OK : CA_ERR_CUDA;
}

int ca_selftest_wait_timeout_status(int64_t limit_ns, int32_t* status, void* stream) {
  if (limit_ns <= 0 || limit_ns > 1000000000ll || !status) return CA_ERR_INVALID;
  ca::selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<uint64_t>(limit_ns), status);
  return cudaGetLastError() == cudaSuccess ? CA_OK : CA_ERR_CUDA;
}

int ca_attention_block_dev_noalloc(const ca_block_args* a, void* stream) {
  return ca::noalloc_impl(a, static_cast<cudaStream_t>(stream));
}

int ca_round_bf16_host(const float* src, uint16_t* dst, uint64_t n) {
  if (n == 0) return CA_OK;
  if (!src || !dst) return CA_ERR_INVALID;
  ca::host_round_bf16(src, dst, static_cast<size_t>(n));
  return CA_OK;
}

int ca_attention_host_f32(float* out, const float* q, const float* k, const float* v,
                          const ca_shape* s, const ca_rows* qr, const ca_rows* kr) {
  return ca::host_f32_impl(out, q, k, v, s, qr, kr);
}

int ca_attention_dev(const ca_dev_args* a, void* stream) {
  return ca::attention_dev_impl(a, static_cast<cudaStream_t>(stream));
}

int ca_attention_block_dev(const ca_block_args* a, void* stream) {
  return ca::block_impl(a, static_cast<cudaStream_t>(stream));
}

// build_rope_cache_ff (src/model/ops.rs:398-416): freq_i = 1 / theta^(2i/d)
// in f32, divided by freq_factors[i] when given; entry t*half+i = sin_cos(t*freq).
int ca_build_rope_table(float* out, int64_t max_seq_len, int64_t rope_dim, float theta,
                        const float* freq_factors) {
  if (!out || max_seq_len < 0 || rope_dim < 0 || rope_dim % 2) return CA_ERR_INVALID;
  const int64_t half = rope_dim / 2;
  std::vector<float> freq(half);
  for (int64_t i = 0; i < half; ++i) {
    float f = 1.0f / powf(theta, 2.0f * static_cast<float>(i) / static_cast<float>(rope_dim));
    if (freq_factors) f /= freq_factors[i];
    freq[i] = f;
  }
  for (int64_t t = 0; t < max_seq_len; ++t)
    for (int64_t i = 0; i < half; ++i) {
      const float x = static_cast<float>(t) * freq[i];
      out[2 * (t * half + i)] = sinf(x);
      out[2 * (t * half + i) + 1] = cosf(x);
    }
  return CA_OK;
}

int ca_device_status(void* stream) {
  if (cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) != cudaSuccess) return CA_ERR_CUDA;
  int derr = 0;
  if (cudaMemcpyFromSymbol(&derr, ca::g_device_error, sizeof(int)) != cudaSuccess)
    return CA_ERR_CUDA;
  if (derr == 0) return CA_OK;
  const int zero = 0;
  cudaMemcpyToSymbol(ca::g_device_error, &zero, sizeof(int));
  return derr;
}

const char* ca_status_string(int status) {
  switch (status) {
    case CA_OK: return "ok";
    case CA_ERR_INVALID: return "invalid argument";
    case CA_ERR_UNSUPPORTED: return "unsupported by this build";
    case CA_ERR_CUDA: return "CUDA error";
    case CA_ERR_TIMEOUT: return "device-side wait timed out";
    case CA_ERR_NOMEM: return "out of memory";
    case CA_ERR_SCRATCH: return "request exceeds the no-allocation entry point's fixed scratch";
    default: return "unknown status";
  }
}

const char* ca_version(void) { return "canvas_attn 0.1.0 sm_100a"; }


}  // extern "C"
