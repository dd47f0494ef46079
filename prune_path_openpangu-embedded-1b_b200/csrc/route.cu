// Selection from given logits: softmax_thresholding (src/MoEBlock.py:49-95) on the GPU,
// one warp per token (select.cuh).  Used by the prefill path after its router GEMM and
// exported on its own so the selection contract can be checked from fixed bf16 logits.
#include "common.cuh"
#include "select.cuh"

namespace ppmoe {

template <int EPL>  // experts per lane: E <= 32 EPL
__global__ void route_logits_kernel(const __nv_bfloat16* __restrict__ logits, int N, int E, float tau_b,
                                    const float* __restrict__ bias, __nv_bfloat16* __restrict__ w_out,
                                    uint8_t* __restrict__ mask_out, __nv_bfloat16* __restrict__ probs_out) {
  __shared__ __align__(16) uint32_t kbuf[8][64];
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= N) return;
  float l[kMaxExpertsPerLane], w[kMaxExpertsPerLane];
#pragma unroll
  for (int i = 0; i < kMaxExpertsPerLane; ++i) {
    const int e = lane + 32 * i;
    float v = -INFINITY;
    if (i < EPL && e < E) {
      v = __bfloat162float(logits[(size_t)t * E + e]);
      if (bias) v = bf16r(v + bias[e]);
    }
    l[i] = v;
  }
  const uint32_t bits = select_experts_warp<EPL>(l, E, tau_b, w, kbuf[threadIdx.x >> 5]);
  if (probs_out) {
    // training-mode output y_soft = softmax(logits) (src/MoEBlock.py:68, 93-94), computed with
    // the operations the selection uses, so these are exactly the probabilities it ranked
    uint32_t mk = 0u;
#pragma unroll
    for (int i = 0; i < EPL; ++i)
      if (lane + 32 * i < E) mk = max(mk, float_order_key(l[i]));
    const float m = float_from_order_key(__reduce_max_sync(0xffffffffu, mk));
    float ex[kMaxExpertsPerLane], sum = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxExpertsPerLane; ++i) {
      ex[i] = (i < EPL && lane + 32 * i < E) ? expf(l[i] - m) : 0.f;
      sum += ex[i];
    }
    sum = warp_sum(sum);
    const float rs = __frcp_rn(sum);
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int e = lane + 32 * i;
      if (e < E) probs_out[(size_t)t * E + e] = __float2bfloat16_rn(bf16r(__fmul_rn(ex[i], rs)));
    }
  }
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = lane + 32 * i;
    if (e < E) {
      w_out[(size_t)t * E + e] = __float2bfloat16_rn(w[i]);
      if (mask_out) mask_out[(size_t)t * E + e] = (bits >> i) & 1u;
    }
  }
}

// Compact active-expert list per token, the form the reference's decode router hands to its
// expert kernel (decode_active_idx / decode_active_weight / decode_num_active,
// src/tl_kernel_optimized_Ultimate_PanGU.py:488-490, written by the kernel at tl:335-380):
// ids[t][r] = the expert at position r of token t's selection in descending-probability
// order (ties to the lower index), w[t][r] its gate weight, n[t] the count; positions
// r >= n[t] hold id -1 and weight 0.  One warp per token; the kept experts are a prefix of
// the sorted order, so each kept expert's position is the number of kept keys above its own.
__global__ void route_compact_kernel(const __nv_bfloat16* __restrict__ logits, int N, int E, float tau_b,
                                     int32_t* __restrict__ ids, __nv_bfloat16* __restrict__ w_out,
                                     int32_t* __restrict__ n_out, uint8_t* __restrict__ mask_out) {
  __shared__ __align__(16) uint32_t kbuf[8][256];
  const int lane = threadIdx.x & 31, wi = threadIdx.x >> 5;
  const int t = blockIdx.x * (blockDim.x >> 5) + wi;
  if (t >= N) return;
  float l[kMaxExpertsPerLane], w[kMaxExpertsPerLane];
#pragma unroll
  for (int i = 0; i < kMaxExpertsPerLane; ++i) {
    const int e = lane + 32 * i;
    l[i] = e < E ? __bfloat162float(logits[(size_t)t * E + e]) : -INFINITY;
  }
  uint32_t key[kMaxExpertsPerLane];
  const uint32_t bits = select_experts_warp(l, E, tau_b, w, kbuf[wi], false, key);
  __syncwarp();
  // kept keys, compacted into the warp's buffer (any order)
  int k = 0;
#pragma unroll
  for (int i = 0; i < kMaxExpertsPerLane; ++i) {
    const bool kept = (bits >> i) & 1u;
    const uint32_t b = __ballot_sync(0xffffffffu, kept);
    if (kept) kbuf[wi][k + __popc(b & ((1u << lane) - 1u))] = key[i];
    k += __popc(b);
  }
  __syncwarp();
#pragma unroll
  for (int i = 0; i < kMaxExpertsPerLane; ++i) {
    const int e = lane + 32 * i;
    if (e >= E) continue;
    if ((bits >> i) & 1u) {
      int r = 0;
      #pragma unroll 4
      for (int j = 0; j < k; ++j) r += kbuf[wi][j] > key[i];
      ids[(size_t)t * E + r] = e;
      w_out[(size_t)t * E + r] = __float2bfloat16_rn(w[i]);
    }
    if (e >= k) {
      ids[(size_t)t * E + e] = -1;
      w_out[(size_t)t * E + e] = __float2bfloat16_rn(0.f);
    }
    if (mask_out) mask_out[(size_t)t * E + e] = (bits >> i) & 1u;
  }
  if (lane == 0) n_out[t] = k;
}

int route_compact_launch(const void* logits, int N, int E, float tau, int32_t* ids, void* w_out, int32_t* n_out,
                         uint8_t* mask_out, cudaStream_t st) {
  if (N == 0) return PPMOE_OK;
  const int warps = 8;
  route_compact_kernel<<<(N + warps - 1) / warps, warps * 32, 0, st>>>(
      static_cast<const __nv_bfloat16*>(logits), N, E, __bfloat162float(__float2bfloat16_rn(tau)), ids,
      static_cast<__nv_bfloat16*>(w_out), n_out, mask_out);
  PPMOE_CHECK_CUDA(cudaGetLastError());
  return PPMOE_OK;
}

int route_logits_launch(const void* logits, int N, int E, float tau, const float* bias, void* w_out,
                        uint8_t* mask_out, cudaStream_t st, void* probs_out = nullptr);
int route_logits_launch(const void* logits, int N, int E, float tau, const float* bias, void* w_out,
                        uint8_t* mask_out, cudaStream_t st, void* probs_out) {
  if (N == 0) return PPMOE_OK;
  const int warps = 8;
  auto kern = E <= 64 ? route_logits_kernel<2> : route_logits_kernel<kMaxExpertsPerLane>;
  kern<<<(N + warps - 1) / warps, warps * 32, 0, st>>>(
      static_cast<const __nv_bfloat16*>(logits), N, E, __bfloat162float(__float2bfloat16_rn(tau)), bias,
      static_cast<__nv_bfloat16*>(w_out), mask_out, static_cast<__nv_bfloat16*>(probs_out));
  PPMOE_CHECK_CUDA(cudaGetLastError());
  return PPMOE_OK;
}

}  // namespace ppmoe
