// Expert-parallel prefill, source side: add the partial rows that the expert-owning ranks
// returned for each token (fp32, or bf16 in the reduced-traffic mode) in rank order with fp32
// additions, and round once to bf16.
#include "common.cuh"

namespace ppmoe {

__device__ __forceinline__ float4 load4(const float4* p, size_t i) { return p[i]; }
__device__ __forceinline__ float4 load4(const uint2* p, size_t i) {  // 4 bf16 -> fp32
  const uint2 v = p[i];
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.y));
  return make_float4(a.x, a.y, b.x, b.y);
}

// row_of [P][n]: row of `back` holding rank d's partial for token t, or -1.  T = float4 (fp32
// partials) or uint2 (bf16 partials, the optional reduced-traffic mode).
template <typename T>
__global__ void ep_combine_kernel(const T* __restrict__ back, const int* __restrict__ row_of, int P, int n,
                                  int H4, uint2* __restrict__ out) {
  const int t = blockIdx.x;
  int rows[8];
#pragma unroll
  for (int d = 0; d < 8; ++d) rows[d] = d < P ? row_of[(size_t)d * n + t] : -1;
  for (int c = threadIdx.x; c < H4; c += blockDim.x) {
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int d = 0; d < 8; ++d) {
      if (rows[d] >= 0) {
        const float4 v = load4(back, (size_t)rows[d] * H4 + c);
        s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
      }
    }
    __nv_bfloat162 lo = __floats2bfloat162_rn(s.x, s.y), hi = __floats2bfloat162_rn(s.z, s.w);
    uint2 pk;
    pk.x = *reinterpret_cast<uint32_t*>(&lo);
    pk.y = *reinterpret_cast<uint32_t*>(&hi);
    out[(size_t)t * H4 + c] = pk;
  }
}

}  // namespace ppmoe

using namespace ppmoe;

static int ep_combine(const void* back, bool bf16, const int32_t* row_of, int ranks, int tokens, int hidden,
                      void* out, void* stream) {
  if (ranks < 1 || ranks > 8 || tokens < 0 || hidden <= 0 || hidden % 4 != 0) {
    set_error("ppmoe_ep_combine: ranks=%d (1..8), tokens=%d, hidden=%d (multiple of 4)", ranks, tokens, hidden);
    return PPMOE_ERR_UNSUPPORTED;
  }
  if (tokens == 0) return PPMOE_OK;
  if (!back || !row_of || !out) {
    set_error("ppmoe_ep_combine: null pointer");
    return PPMOE_ERR_INVALID_ARG;
  }
  if (bf16)
    ep_combine_kernel<<<tokens, 128, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint2*>(back), row_of, ranks, tokens, hidden / 4, static_cast<uint2*>(out));
  else
    ep_combine_kernel<<<tokens, 128, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const float4*>(back), row_of, ranks, tokens, hidden / 4, static_cast<uint2*>(out));
  PPMOE_CHECK_CUDA(cudaGetLastError());
  return PPMOE_OK;
}

extern "C" int ppmoe_ep_combine(const float* back, const int32_t* row_of, int ranks, int tokens, int hidden,
                                void* out, void* stream) {
  return ep_combine(back, false, row_of, ranks, tokens, hidden, out, stream);
}

extern "C" int ppmoe_ep_combine_bf16(const void* back, const int32_t* row_of, int ranks, int tokens, int hidden,
                                     void* out, void* stream) {
  return ep_combine(back, true, row_of, ranks, tokens, hidden, out, stream);
}
