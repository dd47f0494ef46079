// Warp-level tau cumulative-mass expert selection for one token.
//
// Restates src/MoEBlock.py:68-91 (softmax_thresholding) with the rounding points of the
// reference's CPU bf16 path:
//   p_e  = bf16( exp(l_e - max) / sum_e exp(l_e - max) )      (fp32 inside)
//   order: p descending, ties -> lower expert index          (stable sort contract; the
//          reference Triton decode kernel picks the lowest index too, tl:368-369)
//   c_j  = bf16( p_(0) + ... + p_(j) )                       (sequential fp32 sum)
//   keep expert (j) iff c_j < bf16(tau)  or  j == 0          (forced top-1, MoEBlock.py:81-86)
//   w_e  = bf16( 1 / (1 + exp(-l_e)) ) on kept experts, 0 elsewhere.
// The cumulative sum is monotone, so the first rejected rank ends the selection; the
// selection loop is an iterative warp arg-max (one 64-bit max-reduction per kept expert),
// which visits experts in exactly the sorted order without sorting all of them.
#pragma once
#include "common.cuh"

namespace ppmoe {

constexpr int kMaxExpertsPerLane = 8;  // E <= 256

// l[i] holds the bf16-valued logit of expert e = lane + 32*i (i < epl, e < E).
// On return w[i] is the gate weight (0 when not selected) and the returned bitmask has
// bit i set when expert lane + 32*i was selected.
__device__ __forceinline__ uint32_t select_experts_warp(const float (&l)[kMaxExpertsPerLane], int E,
                                                        float tau_b, float (&w)[kMaxExpertsPerLane]) {
  const int lane = threadIdx.x & 31;
  const int epl = (E + 31) >> 5;
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < kMaxExpertsPerLane; ++i)
    if (i < epl && lane + 32 * i < E) m = fmaxf(m, l[i]);
  m = warp_max(m);
  float ex[kMaxExpertsPerLane];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxExpertsPerLane; ++i) {
    ex[i] = (i < epl && lane + 32 * i < E) ? expf(l[i] - m) : 0.f;
    s += ex[i];
  }
  s = warp_sum(s);
  unsigned long long key[kMaxExpertsPerLane];
#pragma unroll
  for (int i = 0; i < kMaxExpertsPerLane; ++i) {
    const int e = lane + 32 * i;
    if (i < epl && e < E) {
      const float p = bf16r(__fdiv_rn(ex[i], s));  // p >= 0: its bit pattern orders like p
      key[i] = (static_cast<unsigned long long>(__float_as_uint(p)) << 32) |
               static_cast<unsigned long long>(0xFFFFFFFFu - static_cast<uint32_t>(e));
    } else {
      key[i] = 0ull;  // never selected (below every real key)
    }
  }
  uint32_t bits = 0;
  float cum = 0.f;
  for (int j = 0; j < E; ++j) {
    unsigned long long k = 0ull;
#pragma unroll
    for (int i = 0; i < kMaxExpertsPerLane; ++i) k = key[i] > k ? key[i] : k;
    k = warp_max_u64(k);
    const float p = __uint_as_float(static_cast<uint32_t>(k >> 32));
    const int e = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(k & 0xFFFFFFFFull));
    cum += p;
    if (j > 0 && !(bf16r(cum) < tau_b)) break;
    if ((e & 31) == lane) {
      const int i = e >> 5;
#pragma unroll
      for (int q = 0; q < kMaxExpertsPerLane; ++q)
        if (q == i) { key[q] = 0ull; bits |= 1u << q; }
    }
  }
#pragma unroll
  for (int i = 0; i < kMaxExpertsPerLane; ++i)
    w[i] = (bits >> i) & 1u ? bf16r(__fdiv_rn(1.f, 1.f + expf(-l[i]))) : 0.f;
  return bits;
}

}  // namespace ppmoe
