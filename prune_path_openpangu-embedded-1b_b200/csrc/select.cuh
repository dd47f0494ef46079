// Warp-level tau cumulative-mass expert selection for one token.
//
// Restates src/MoEBlock.py:68-91 (softmax_thresholding) with the rounding points of the
// reference's CPU bf16 path:
//   p_e  = bf16( exp(l_e - max) * (1 / sum_e exp(l_e - max)) ) (fp32 inside)
//   order: p descending, ties -> lower expert index          (stable sort contract; the
//          reference Triton decode kernel picks the lowest index too, tl:368-369)
//   c_j  = bf16( p_(0) + ... + p_(j) )                       (sequential fp32 sum)
//   keep expert (j) iff c_j < bf16(tau)  or  j == 0          (forced top-1, MoEBlock.py:81-86)
//   w_e  = bf16( 1 / (1 + exp(-l_e)) ) on kept experts, 0 elsewhere.
// The cumulative sum is monotone, so the kept experts are a prefix of the sorted order.
// Requires E <= 256 (8 experts per lane; the 16-bit index field needs E < 65535).
#pragma once
#include "common.cuh"

namespace ppmoe {

constexpr int kMaxExpertsPerLane = 8;  // E <= 256

__device__ __forceinline__ uint32_t float_order_key(float f) {  // unsigned order == float order
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float float_from_order_key(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// Sequential selection over 32-bit keys (bf16 bits of p << 16 | 0xFFFF - e): one redux.sync
// max per kept expert, which visits experts in exactly the sorted order.  Exact for any
// probabilities; used when the parallel path's exactness condition does not hold.
__device__ __forceinline__ uint32_t select_sequential(uint32_t (&key)[kMaxExpertsPerLane], int E, float tau_b) {
  const int lane = threadIdx.x & 31;
  uint32_t bits = 0;
  float cum = 0.f;
  for (int j = 0; j < E; ++j) {
    uint32_t k = 0u;
#pragma unroll
    for (int i = 0; i < kMaxExpertsPerLane; ++i) k = max(k, key[i]);
    k = __reduce_max_sync(0xffffffffu, k);
    const float p = __uint_as_float(k & 0xFFFF0000u);
    const int e = static_cast<int>(0xFFFFu - (k & 0xFFFFu));
    cum += p;
    if (j > 0 && !(bf16r(cum) < tau_b)) break;
    if ((e & 31) == lane) {
      const int i = e >> 5;
#pragma unroll
      for (int q = 0; q < kMaxExpertsPerLane; ++q)
        if (q == i) { key[q] = 0u; bits |= 1u << q; }
    }
  }
  return bits;
}

// Parallel selection: warp bitonic sort of the keys (descending), prefix sums of the sorted
// probabilities, cutoff by a min-reduction.  Every probability is a bf16 value; when each
// one up to the cutoff is 0 or >= 2^-16 and the sums stay below 2, every partial sum is a
// multiple of 2^-23 below 2 and therefore exact in fp32, so any summation order gives the
// sequential sums bit for bit.  Otherwise returns false (warp-uniformly) and the caller
// falls back to select_sequential.
template <int EPL>
__device__ __forceinline__ bool select_parallel(const uint32_t (&key)[kMaxExpertsPerLane], int E, float tau_b,
                                                uint32_t& bits_out) {
  const int lane = threadIdx.x & 31;
  constexpr int n = 32 * EPL;
  uint32_t v[EPL];
#pragma unroll
  for (int r = 0; r < EPL; ++r) v[r] = key[r];
  // element index i = lane * EPL + r.  The stage loops stay rolled: this code runs once per
  // token and its size (instruction-cache misses) matters more than loop overhead.
#pragma unroll 1
  for (int k = 2; k <= n; k <<= 1) {
#pragma unroll 1
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j >= EPL) {
        const int lj = j / EPL;
#pragma unroll
        for (int r = 0; r < EPL; ++r) {
          const int i = lane * EPL + r;
          const uint32_t o = __shfl_xor_sync(0xffffffffu, v[r], lj);
          const bool keep_max = ((i & k) == 0) == ((i & j) == 0);
          v[r] = keep_max ? max(v[r], o) : min(v[r], o);
        }
      } else {
#pragma unroll
        for (int jj = 1; jj < EPL; jj <<= 1) {  // j < EPL: exchange inside the lane
          if (jj == j) {
#pragma unroll
            for (int r = 0; r < EPL; ++r) {
              const int rp = r ^ jj;
              if (rp > r) {
                const int i = lane * EPL + r;
                const uint32_t a = v[r], b = v[rp];
                const bool desc = (i & k) == 0;
                v[r] = desc ? max(a, b) : min(a, b);
                v[rp] = desc ? min(a, b) : max(a, b);
              }
            }
          }
        }
      }
    }
  }
  float loc[EPL];
  float run = 0.f;
#pragma unroll
  for (int r = 0; r < EPL; ++r) {
    run += __uint_as_float(v[r] & 0xFFFF0000u);
    loc[r] = run;
  }
  float incl = run;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  const float excl = incl - run;  // exact under the condition checked below
  uint32_t keep_lane = 0;
  int first_rej = n;
#pragma unroll
  for (int r = 0; r < EPL; ++r) {
    const int i = lane * EPL + r;
    const bool keep = i < E && (i == 0 || bf16r(excl + loc[r]) < tau_b);
    keep_lane |= (uint32_t)keep << r;
    if (!keep && i < first_rej) first_rej = i;
  }
  const int J = __reduce_min_sync(0xffffffffu, first_rej);  // sums up to index J decide
  uint32_t bad = excl + loc[EPL - 1] >= 2.f;
#pragma unroll
  for (int r = 0; r < EPL; ++r) {
    const int i = lane * EPL + r;
    const float p = __uint_as_float(v[r] & 0xFFFF0000u);
    if (i <= J && i < E && p != 0.f && p < 1.52587890625e-05f) bad = 1;  // 2^-16
  }
  if (__any_sync(0xffffffffu, bad)) return false;
  // kept experts -> per-owner-lane bits (expert e is owned by lane e % 32, slot e / 32)
  uint32_t bits = 0;
#pragma unroll
  for (int q = 0; q < kMaxExpertsPerLane; ++q) {
    if (q * 32 < E) {
      uint32_t wq = 0u;
#pragma unroll
      for (int r = 0; r < EPL; ++r) {
        const uint32_t e = 0xFFFFu - (v[r] & 0xFFFFu);
        wq |= (((keep_lane >> r) & 1u) && (e >> 5) == (uint32_t)q) ? (1u << (e & 31u)) : 0u;
      }
      wq = __reduce_or_sync(0xffffffffu, wq);
      bits |= ((wq >> lane) & 1u) << q;
    }
  }
  bits_out = bits;
  return true;
}

// Rank selection for E <= 64: each lane ranks its own (at most two) experts against all E
// keys (read four at a time from a 64-word per-warp shared buffer `kbuf`), accumulating
// S_i = sum of p over experts ahead of it.  Under
// the same exactness condition as select_parallel, S_i + p_i equals the sequential
// cumulative sum at expert i's sorted position bit for bit; no sort and no scatter needed.
template <int EPL>
__device__ __forceinline__ bool select_rank(const uint32_t (&key)[kMaxExpertsPerLane], int E, float tau_b,
                                            uint32_t& bits_out, uint32_t* kbuf) {
  const int lane = threadIdx.x & 31;
  // every key to shared memory (padding keys are 0), then 4 keys per broadcast load
#pragma unroll
  for (int r = 0; r < EPL; ++r) kbuf[lane + 32 * r] = key[r];
  __syncwarp();
  float S[EPL][2];
  int rank[EPL];
#pragma unroll
  for (int r = 0; r < EPL; ++r) { S[r][0] = S[r][1] = 0.f; rank[r] = 0; }
#pragma unroll
  for (int j4 = 0; j4 < 8 * EPL; ++j4) {
    const uint4 kq = reinterpret_cast<const uint4*>(kbuf)[j4];
    const uint32_t kk[4] = {kq.x, kq.y, kq.z, kq.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float pj = __uint_as_float(kk[q] & 0xFFFF0000u);
#pragma unroll
      for (int r = 0; r < EPL; ++r) {
        const bool g = kk[q] > key[r];
        S[r][q & 1] += g ? pj : 0.f;
        rank[r] += g;
      }
    }
  }
  __syncwarp();
  uint32_t keep_bits = 0;
  int first_rej = 1 << 20;
  float Sr[EPL];
#pragma unroll
  for (int r = 0; r < EPL; ++r) {
    Sr[r] = S[r][0] + S[r][1];  // exact under the condition checked below
    if (lane + 32 * r < E) {
      const float c = Sr[r] + __uint_as_float(key[r] & 0xFFFF0000u);
      const bool keep = rank[r] == 0 || bf16r(c) < tau_b;
      keep_bits |= (uint32_t)keep << r;
      if (!keep) first_rej = min(first_rej, rank[r]);
    }
  }
  const int J = __reduce_min_sync(0xffffffffu, first_rej);
  uint32_t bad = 0;
#pragma unroll
  for (int r = 0; r < EPL; ++r) {
    if (lane + 32 * r < E) {
      const float p = __uint_as_float(key[r] & 0xFFFF0000u);
      if (rank[r] <= J && p != 0.f && p < 1.52587890625e-05f) bad = 1;  // 2^-16
      if (Sr[r] + p >= 2.f) bad = 1;
    }
  }
  if (__any_sync(0xffffffffu, bad)) return false;
  bits_out = keep_bits;
  return true;
}

// l[i] holds the bf16-valued logit of expert e = lane + 32*i (e < E).  kbuf: 64 words of
// 16-byte aligned shared memory owned by the calling warp.  On return w[i] is the
// gate weight (0 when not selected) and the returned bitmask has bit i set when expert
// lane + 32*i was selected.  Each probability is a bf16 value, so its fp32 bit pattern has
// 16 zero low bits; the 32-bit key (bf16 bits of p) << 16 | (0xFFFF - e) orders candidates
// by p descending and then by expert index ascending.
template <int EPL = kMaxExpertsPerLane>
__device__ __forceinline__ uint32_t select_experts_warp(const float (&l)[kMaxExpertsPerLane], int E,
                                                        float tau_b, float (&w)[kMaxExpertsPerLane],
                                                        uint32_t* kbuf, bool throughput = false,
                                                        uint32_t* keys_out = nullptr) {
  // EPL < kMaxExpertsPerLane: the caller guarantees E <= 32 * EPL, and only the first EPL
  // slots are touched (the rest are compile-time zeros), so the code for larger E is not built
  const int lane = threadIdx.x & 31;
  uint32_t mk = 0u;
#pragma unroll
  for (int i = 0; i < EPL; ++i)
    if (lane + 32 * i < E) mk = max(mk, float_order_key(l[i]));
  const float m = float_from_order_key(__reduce_max_sync(0xffffffffu, mk));
  float ex[kMaxExpertsPerLane];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxExpertsPerLane; ++i) {
    ex[i] = (i < EPL && lane + 32 * i < E) ? expf(l[i] - m) : 0.f;
    s += ex[i];
  }
  s = warp_sum(s);
  const float rs = __frcp_rn(s);
  uint32_t key[kMaxExpertsPerLane];
#pragma unroll
  for (int i = 0; i < kMaxExpertsPerLane; ++i) {
    const int e = lane + 32 * i;
    if (i < EPL && e < E) {
      const float p = bf16r(__fmul_rn(ex[i], rs));  // p >= 0: its bit pattern orders like p
      key[i] = (__float_as_uint(p) & 0xFFFF0000u) | (0xFFFFu - static_cast<uint32_t>(e));
    } else {
      key[i] = 0u;  // never selected (below every real key)
    }
  }
  uint32_t bits = 0;
  bool done;
  // throughput: the bitonic network (O(E log E) work) instead of the rank count (O(E^2)
  // work, lower latency); measured slower for 16 tokens in the fused decode, so off there.
  if (EPL == 1 || (EPL > 1 && E <= 32))
    done = throughput ? select_parallel<1>(key, E, tau_b, bits) : select_rank<1>(key, E, tau_b, bits, kbuf);
  else if (EPL == 2 || (EPL > 2 && E <= 64))
    done = throughput ? select_parallel<2>(key, E, tau_b, bits) : select_rank<2>(key, E, tau_b, bits, kbuf);
  else if (EPL <= 4 || E <= 128) done = select_parallel<4>(key, E, tau_b, bits);
  else done = select_parallel<8>(key, E, tau_b, bits);
  if (keys_out) {
#pragma unroll
    for (int i = 0; i < kMaxExpertsPerLane; ++i) keys_out[i] = key[i];
  }
  if (!done) bits = select_sequential(key, E, tau_b);
#pragma unroll
  for (int i = 0; i < kMaxExpertsPerLane; ++i)
    w[i] = (i < EPL && ((bits >> i) & 1u)) ? bf16r(__frcp_rn(1.f + expf(-l[i]))) : 0.f;
  return bits;
}

// CTA-parallel selection of ONE token for E <= 64, used by the single-token decode: every
// warp computes the softmax keys redundantly (identical code, identical results); warp w
// ranks experts (w % 2) * 32 + lane against the experts of part w / 2 (NW / 2 parts), the
// partial ranks and mass sums meet in shared memory, and warp 0 finishes.  Same exactness
// condition and fallback as select_rank.  Warps 0 .. NW-1 of the CTA must all call it.
// scratch: 2 * (NW / 2) * 64 words of shared memory.  Returns the kept-expert bitmask of
// slot i (expert lane + 32 i) in warp 0 (other warps: 0) and writes w (warp 0 only valid).
template <int NW>
__device__ __forceinline__ uint32_t select_one_token_cta(const float* lg, int E, float tau_b,
                                                         float (&w)[kMaxExpertsPerLane], uint32_t* scratch) {
  constexpr int NP = NW / 2;  // rank parts
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float l[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) l[r] = lane + 32 * r < E ? lg[lane + 32 * r] : -INFINITY;
  uint32_t mk = 0u;
#pragma unroll
  for (int r = 0; r < 2; ++r)
    if (lane + 32 * r < E) mk = max(mk, float_order_key(l[r]));
  const float m = float_from_order_key(__reduce_max_sync(0xffffffffu, mk));
  float ex[2], s = 0.f;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    ex[r] = lane + 32 * r < E ? expf(l[r] - m) : 0.f;
    s += ex[r];
  }
  s = warp_sum(s);
  const float rs = __frcp_rn(s);
  uint32_t key[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int e = lane + 32 * r;
    key[r] = e < E ? (__float_as_uint(bf16r(__fmul_rn(ex[r], rs))) & 0xFFFF0000u) | (0xFFFFu - (uint32_t)e) : 0u;
  }
  // ---- partial ranks: own expert i = h*32 + lane against experts of part p
  int* prank = reinterpret_cast<int*>(scratch);           // [NP][64]
  float* psum = reinterpret_cast<float*>(scratch) + NP * 64;  // [NP][64]
  if (warp < 2 * NP) {
    const int h = warp & 1, p = warp >> 1;
    const uint32_t mine = h ? key[1] : key[0];
    const int j0 = (64 * p) / NP, j1 = (64 * (p + 1)) / NP;
    float S = 0.f;
    int rk = 0;
#pragma unroll 4
    for (int j = j0; j < j1; ++j) {
      const uint32_t kj = __shfl_sync(0xffffffffu, (j & 32) ? key[1] : key[0], j & 31);
      const bool g = kj > mine;
      S += g ? __uint_as_float(kj & 0xFFFF0000u) : 0.f;
      rk += g;
    }
    prank[p * 64 + h * 32 + lane] = rk;
    psum[p * 64 + h * 32 + lane] = S;
  }
  // the NW calling warps only (other warps of the CTA may be busy elsewhere)
  asm volatile("bar.sync 3, %0;" ::"n"(NW * 32) : "memory");
  uint32_t bits = 0;
  if (warp == 0) {
    float Sr[2];
    int rank[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      Sr[r] = 0.f;
      rank[r] = 0;
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        Sr[r] += psum[p * 64 + r * 32 + lane];
        rank[r] += prank[p * 64 + r * 32 + lane];
      }
    }
    uint32_t keep_bits = 0;
    int first_rej = 1 << 20;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      if (lane + 32 * r < E) {
        const float c = Sr[r] + __uint_as_float(key[r] & 0xFFFF0000u);
        const bool keep = rank[r] == 0 || bf16r(c) < tau_b;
        keep_bits |= (uint32_t)keep << r;
        if (!keep) first_rej = min(first_rej, rank[r]);
      }
    }
    const int J = __reduce_min_sync(0xffffffffu, first_rej);
    uint32_t bad = 0;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      if (lane + 32 * r < E) {
        const float p = __uint_as_float(key[r] & 0xFFFF0000u);
        if (rank[r] <= J && p != 0.f && p < 1.52587890625e-05f) bad = 1;  // 2^-16
        if (Sr[r] + p >= 2.f) bad = 1;
      }
    }
    if (__any_sync(0xffffffffu, bad)) {
      uint32_t k8[kMaxExpertsPerLane];
#pragma unroll
      for (int i = 0; i < kMaxExpertsPerLane; ++i) k8[i] = i < 2 ? key[i] : 0u;
      keep_bits = select_sequential(k8, E, tau_b);
    }
    bits = keep_bits;
#pragma unroll
    for (int i = 0; i < kMaxExpertsPerLane; ++i)
      w[i] = (i < 2 && ((bits >> i) & 1u)) ? bf16r(__frcp_rn(1.f + expf(-l[i & 1]))) : 0.f;
  }
  return bits;
}

}  // namespace ppmoe
