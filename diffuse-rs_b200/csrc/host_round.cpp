// host_round.cpp -- fp32 -> bf16 rounding on the host for the host-buffer
// entry point (ca_attention_host_f32). The attention kernels take bf16
// operands, so rounding before the host-to-device copy halves the bytes that
// cross PCIe, the bound of that entry point. The rounding is the GPU's
// (cvt.rn.bf16.f32: round to nearest even, every NaN to 0x7FFF, overflow to
// infinity), so the device sees bit-identical operands either way.
//
// Work is split over a small persistent pool of host threads (the calling
// thread takes part); the pool is created on first use and never destroyed,
// so no thread or lock outlives its objects at process exit.
#include <immintrin.h>
#include <sched.h>

#include <algorithm>
#include <atomic>
#include <condition_variable>
#include <cstdint>
#include <cstdlib>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

#include "host_round.h"

namespace ca {
namespace {

inline uint16_t round_one(uint32_t u) {
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fff;  // NaN
  return static_cast<uint16_t>((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}

void round_scalar(const float* src, uint16_t* dst, size_t n) {
  const uint32_t* s = reinterpret_cast<const uint32_t*>(src);
  for (size_t i = 0; i < n; ++i) dst[i] = round_one(s[i]);
}

__attribute__((target("avx2"))) inline __m256i round8(__m256i x) {
  const __m256i one = _mm256_set1_epi32(1);
  const __m256i bias = _mm256_set1_epi32(0x7fff);
  const __m256i lsb = _mm256_and_si256(_mm256_srli_epi32(x, 16), one);
  __m256i r = _mm256_srli_epi32(_mm256_add_epi32(x, _mm256_add_epi32(bias, lsb)), 16);
  const __m256i mag = _mm256_and_si256(x, _mm256_set1_epi32(0x7fffffff));
  const __m256i nan = _mm256_cmpgt_epi32(mag, _mm256_set1_epi32(0x7f800000));
  return _mm256_blendv_epi8(r, bias, nan);
}

// Stores bypass the cache (non-temporal): the bf16 copy is read next by the
// copy engine, not by this CPU, and skipping the read-for-ownership of the
// destination lines cuts the memory traffic per element from 8 to 6 bytes.
__attribute__((target("avx2"))) void round_avx2(const float* src, uint16_t* dst, size_t n) {
  size_t i = 0;
  while (i < n && (reinterpret_cast<uintptr_t>(dst + i) & 31u)) {
    dst[i] = round_one(reinterpret_cast<const uint32_t*>(src)[i]);
    ++i;
  }
  for (; i + 16 <= n; i += 16) {
    const __m256i a = round8(_mm256_loadu_si256(reinterpret_cast<const __m256i*>(src + i)));
    const __m256i b = round8(_mm256_loadu_si256(reinterpret_cast<const __m256i*>(src + i + 8)));
    // packus works per 128-bit lane: a0-3 b0-3 a4-7 b4-7 -> a0-7 b0-7.
    const __m256i p = _mm256_permute4x64_epi64(_mm256_packus_epi32(a, b), 0xD8);
    _mm256_stream_si256(reinterpret_cast<__m256i*>(dst + i), p);
  }
  _mm_sfence();
  round_scalar(src + i, dst + i, n - i);
}

// A rounding job: segments (src, dst, n) cut into tasks of kPart elements,
// claimed in order by the pool's workers and by the thread that waits on
// the job. Each segment counts its unfinished tasks, so the caller can hand
// a segment to the copy engine as soon as it is done while later segments
// are still being rounded.
constexpr size_t kPart = 1u << 16;  // 256 KiB of fp32 input per task

struct Job {
  std::vector<RoundSeg> seg;
  std::vector<size_t> first;               // first task of each segment
  std::vector<std::atomic<int>> left;      // unfinished tasks per segment
  size_t n_tasks = 0;
  std::atomic<size_t> next{0};             // next task to claim
  std::atomic<size_t> finished{0};
  void (*fn)(const float*, uint16_t*, size_t) = nullptr;

  // Claims and runs one task; false when none is left to claim.
  bool run_one() {
    const size_t t = next.fetch_add(1);
    if (t >= n_tasks) return false;
    const size_t si = std::upper_bound(first.begin(), first.end(), t) - first.begin() - 1;
    const RoundSeg& sg = seg[si];
    const size_t b = (t - first[si]) * kPart;
    fn(sg.src + b, sg.dst + b, std::min(kPart, sg.n - b));
    left[si].fetch_sub(1, std::memory_order_release);
    finished.fetch_add(1, std::memory_order_release);
    return true;
  }
};

class Pool {
 public:
  explicit Pool(int workers) : n_threads_(workers + 1) {
    for (int i = 0; i < workers; ++i) std::thread([this] { loop(); }).detach();
  }
  int threads() const { return n_threads_; }
  void start(Job* j) {
    {
      std::lock_guard<std::mutex> g(m_);
      job_ = j;
      ++gen_;
    }
    cv_.notify_all();
  }
  // Blocks until segment si of the running job is rounded (si < 0: every
  // task of the job), running tasks meanwhile.
  void wait(Job* j, int si) {
    for (;;) {
      if (si >= 0 ? j->left[si].load(std::memory_order_acquire) == 0
                  : j->finished.load(std::memory_order_acquire) == j->n_tasks)
        return;
      if (!j->run_one()) std::this_thread::yield();
    }
  }
  // Waits for the whole job, then detaches it: no worker touches it after.
  void finish(Job* j) {
    wait(j, -1);
    std::unique_lock<std::mutex> g(m_);
    job_ = nullptr;
    idle_.wait(g, [&] { return busy_ == 0; });
  }

 private:
  void loop() {
    uint64_t seen = 0;
    for (;;) {
      Job* j;
      {
        std::unique_lock<std::mutex> g(m_);
        cv_.wait(g, [&] { return gen_ != seen && job_ != nullptr; });
        seen = gen_;
        j = job_;
        ++busy_;
      }
      while (j->run_one()) {
      }
      std::lock_guard<std::mutex> g(m_);
      if (--busy_ == 0) idle_.notify_all();
    }
  }
  std::mutex m_;
  std::condition_variable cv_, idle_;
  Job* job_ = nullptr;
  uint64_t gen_ = 0;
  int busy_ = 0;
  int n_threads_ = 1;
};

int usable_cpus() {
  cpu_set_t set;
  if (sched_getaffinity(0, sizeof(set), &set) == 0) return std::max(1, CPU_COUNT(&set));
  return std::max(1u, std::thread::hardware_concurrency());
}

Pool& pool() {
  static Pool* p = [] {
    int t = std::min(usable_cpus(), 32);
    if (const char* e = std::getenv("CA_HOST_THREADS")) t = std::max(1, std::atoi(e));
    return new Pool(t - 1);  // never destroyed: detached workers outlive main
  }();
  return *p;
}

std::mutex g_round_mu;  // one job at a time

}  // namespace

struct RoundBatch::Impl {
  Job job;
  std::unique_lock<std::mutex> lock{g_round_mu};
};

RoundBatch::RoundBatch(const RoundSeg* segs, int n) : impl_(new Impl) {
  static const bool avx2 = __builtin_cpu_supports("avx2");
  Job& j = impl_->job;
  j.fn = avx2 ? round_avx2 : round_scalar;
  j.seg.assign(segs, segs + n);
  j.first.resize(n);
  j.left = std::vector<std::atomic<int>>(n);
  for (int i = 0; i < n; ++i) {
    j.first[i] = j.n_tasks;
    const size_t t = (segs[i].n + kPart - 1) / kPart;
    j.left[i].store(static_cast<int>(t));
    j.n_tasks += t;
  }
  pool().start(&j);
}

void RoundBatch::wait(int seg) { pool().wait(&impl_->job, seg); }

RoundBatch::~RoundBatch() {
  pool().finish(&impl_->job);
  delete impl_;
}

// Rounds n floats to bf16 bits into dst, in parallel on the host.
void host_round_bf16(const float* src, uint16_t* dst, size_t n) {
  if (n <= kPart) {
    static const bool avx2 = __builtin_cpu_supports("avx2");
    (avx2 ? round_avx2 : round_scalar)(src, dst, n);
    return;
  }
  RoundSeg sg{src, dst, n};
  RoundBatch b(&sg, 1);
  b.wait(0);
}

int host_round_threads() { return pool().threads(); }

}  // namespace ca
