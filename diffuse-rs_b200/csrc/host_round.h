// host_round.h -- fp32 -> bf16 rounding on host threads (host_round.cpp).
#pragma once

#include <cstddef>
#include <cstdint>

namespace ca {

struct RoundSeg {
  const float* src;
  uint16_t* dst;
  size_t n;
};

// Rounds n floats to bf16 bit patterns (round to nearest even, NaN to
// 0x7FFF: the GPU's cvt.rn.bf16.f32) on the host thread pool; blocks.
void host_round_bf16(const float* src, uint16_t* dst, size_t n);

// Rounds several segments as one job that starts at construction; wait(i)
// returns once segment i is rounded (the caller runs tasks meanwhile), so a
// caller can pass finished segments on while later ones are still being
// rounded. The destructor waits for the whole job. One batch at a time per
// process (a second one blocks until the first is destroyed).
class RoundBatch {
 public:
  RoundBatch(const RoundSeg* segs, int n);
  ~RoundBatch();
  RoundBatch(const RoundBatch&) = delete;
  RoundBatch& operator=(const RoundBatch&) = delete;
  void wait(int seg);

 private:
  struct Impl;
  Impl* impl_;
};

}  // namespace ca
