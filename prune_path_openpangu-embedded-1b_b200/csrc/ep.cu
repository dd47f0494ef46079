// Expert-parallel prefill, source side: add the partial rows that the expert-owning ranks
// returned for each token (fp32, or bf16 in the reduced-traffic mode) in rank order with fp32
// additions, and round once to bf16.
#include <cuda_fp16.h>
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


// ------------------------------------------------------------------ dispatch
// Destination d owns, in expert group g (experts g P .. g P + P - 1), expert g P + d for even g
// and g P + P - 1 - d for odd g (snake order: balanced under a prior that falls with the expert
// index).  A token goes to d when it selected at least one of them (gate weight > 0).  The send buffer is chunk-major, then destination-major, tokens
// ascending inside each (chunk, destination) segment; each payload row is the token's H bf16
// activations followed by its gate weights for d's experts (owned order), padded to row_pitch
// bytes.  Chunk c covers token blocks [nb c / C, nb (c + 1) / C) of 256 tokens.
constexpr int kEpBlock = 256;
constexpr int kEpMaxRanks = 8;
constexpr int kEpMaxChunks = 8;

__host__ __device__ inline int ep_owner(int e, int P) {
  const int g = e / P, i = e - g * P;
  return (g & 1) ? P - 1 - i : i;
}
__host__ __device__ inline int ep_expert(int d, int j, int P) {  // destination d's j-th expert
  return j * P + ((j & 1) ? P - 1 - d : d);
}

__device__ __forceinline__ uint32_t ep_dest_bits(const __nv_bfloat16* w, int E, int P) {
  uint32_t bits = 0;
  for (int e = 0; e < E; ++e)
    if (__bfloat162float(w[e]) > 0.f) bits |= 1u << ep_owner(e, P);
  return bits;
}

__global__ void ep_count_kernel(const __nv_bfloat16* __restrict__ w, int n, int E, int P, int* __restrict__ blkcnt) {
  const int t = blockIdx.x * kEpBlock + threadIdx.x;
  const uint32_t bits = t < n ? ep_dest_bits(w + (size_t)t * E, E, P) : 0u;
  for (int d = 0; d < P; ++d) {
    const int c = __syncthreads_count((bits >> d) & 1u);
    if (threadIdx.x == 0) blkcnt[blockIdx.x * P + d] = c;
  }
}

// One thread per (chunk, destination): segment totals, then the first send row of every block.
__global__ void ep_scan_kernel(const int* __restrict__ blkcnt, int nb, int P, int C, int* __restrict__ blkoff,
                               long long* __restrict__ counts) {
  __shared__ int tot[kEpMaxChunks][kEpMaxRanks];
  const int c = threadIdx.x / kEpMaxRanks, d = threadIdx.x % kEpMaxRanks;
  const bool on = c < C && d < P;
  const int b0 = on ? (int)((long long)nb * c / C) : 0, b1 = on ? (int)((long long)nb * (c + 1) / C) : 0;
  int s = 0;
  for (int b = b0; b < b1; ++b) s += blkcnt[b * P + d];
  tot[c][d] = on ? s : 0;
  __syncthreads();
  if (!on) return;
  int run = 0;
  for (int cc = 0; cc < c; ++cc)
    for (int dd = 0; dd < P; ++dd) run += tot[cc][dd];
  for (int dd = 0; dd < d; ++dd) run += tot[c][dd];
  counts[d * C + c] = s;
  for (int b = b0; b < b1; ++b) {
    blkoff[b * P + d] = run;
    run += blkcnt[b * P + d];
  }
}

// Per 256-token block: each selected (token, destination) gets its send row (running ballot
// prefix in token order), row_of[d][t] records it (-1 otherwise), and one warp per token copies
// the activation row and the destination's gate weights into the payload.
__global__ void ep_scatter_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w, int n,
                                  int H, int E, int P, const int* __restrict__ blkoff, uint8_t* __restrict__ send,
                                  int pitch, int* __restrict__ row_of) {
  __shared__ int wcnt[kEpMaxRanks][kEpBlock / 32];
  __shared__ int pos_s[kEpBlock][kEpMaxRanks];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t = blockIdx.x * kEpBlock + tid;
  const uint32_t bits = t < n ? ep_dest_bits(w + (size_t)t * E, E, P) : 0u;
  uint32_t bal[kEpMaxRanks];
#pragma unroll
  for (int d = 0; d < kEpMaxRanks; ++d) {
    bal[d] = __ballot_sync(0xffffffffu, d < P && ((bits >> d) & 1u));
    if (lane == 0) wcnt[d][warp] = __popc(bal[d]);
  }
  __syncthreads();
  for (int d = 0; d < P; ++d) {
    int pos = -1;
    if ((bits >> d) & 1u) {
      pos = blkoff[blockIdx.x * P + d] + __popc(bal[d] & ((1u << lane) - 1u));
      for (int q = 0; q < warp; ++q) pos += wcnt[d][q];
    }
    pos_s[tid][d] = pos;
    if (t < n) row_of[(size_t)d * n + t] = pos;
  }
  __syncthreads();
  const int el = E / P, H8 = H / 8;
  for (int i = warp; i < kEpBlock; i += kEpBlock / 32) {
    const int tt = blockIdx.x * kEpBlock + i;
    if (tt >= n) break;
    const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)tt * H);
    for (int d = 0; d < P; ++d) {
      const int pos = pos_s[i][d];
      if (pos < 0) continue;
      uint8_t* row = send + (size_t)pos * pitch;
      for (int c = lane; c < H8; c += 32) reinterpret_cast<uint4*>(row)[c] = xr[c];
      for (int j = lane; j < el; j += 32)
        reinterpret_cast<__nv_bfloat16*>(row + (size_t)H * 2)[j] = w[(size_t)tt * E + ep_expert(d, j, P)];
    }
  }
}

// Scaled-fp16 partial rows (ppmoe_ep_experts partial_format 1): row d of token t at
// back + row_of[d][t] * pitch; values fp16 scaled by 2^s per 64-column slice, s (int8) after the
// H values.  Thread c owns columns 4c .. 4c + 3; fp32 sums in rank order, one bf16 rounding.
__global__ void ep_combine_f16s_kernel(const uint8_t* __restrict__ back, int pitch, const int* __restrict__ row_of,
                                       int P, int n, int H, uint2* __restrict__ out) {
  const int t = blockIdx.x;
  int rows[8];
#pragma unroll
  for (int d = 0; d < 8; ++d) rows[d] = d < P ? row_of[(size_t)d * n + t] : -1;
  for (int c = threadIdx.x; c < H / 4; c += blockDim.x) {
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int d = 0; d < 8; ++d) {
      if (rows[d] >= 0) {
        const uint8_t* row = back + (size_t)rows[d] * pitch;
        const uint2 v = reinterpret_cast<const uint2*>(row)[c];
        const int sc = reinterpret_cast<const int8_t*>(row + (size_t)H * 2)[c >> 4];
        const float inv = __uint_as_float((uint32_t)(127 - sc) << 23);
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
        s.x += a.x * inv; s.y += a.y * inv; s.z += b.x * inv; s.w += b.y * inv;
      }
    }
    __nv_bfloat162 lo = __floats2bfloat162_rn(s.x, s.y), hi = __floats2bfloat162_rn(s.z, s.w);
    uint2 pk;
    pk.x = *reinterpret_cast<uint32_t*>(&lo);
    pk.y = *reinterpret_cast<uint32_t*>(&hi);
    out[(size_t)t * (H / 4) + c] = pk;
  }
}

}  // namespace ppmoe

using namespace ppmoe;

extern "C" size_t ppmoe_ep_dispatch_workspace_bytes(int tokens, int ranks) {
  if (tokens < 0 || ranks < 1 || ranks > kEpMaxRanks) return 0;
  const size_t nb = (size_t)(tokens + kEpBlock - 1) / kEpBlock;
  return 2 * align_up(nb * ranks * 4, 256) + 256;
}

extern "C" int ppmoe_ep_dispatch(const void* x, const void* weights, int tokens, int hidden, int experts, int ranks,
                                 int chunks, void* send, int row_pitch, int64_t* counts, int32_t* row_of, void* ws,
                                 size_t ws_bytes, void* stream) {
  clear_error();
  if (ranks < 1 || ranks > kEpMaxRanks || chunks < 1 || chunks > kEpMaxChunks || tokens < 0 || hidden <= 0 ||
      hidden % 8 != 0 || experts < ranks || experts % ranks != 0 || experts > 256) {
    set_error("ppmoe_ep_dispatch: ranks=%d (1..%d), chunks=%d (1..%d), tokens=%d, hidden=%d (multiple of 8), "
              "experts=%d (a multiple of ranks)", ranks, kEpMaxRanks, chunks, kEpMaxChunks, tokens, hidden, experts);
    return PPMOE_ERR_UNSUPPORTED;
  }
  const int need = (int)align_up((size_t)(hidden + experts / ranks) * 2, 16);
  if (row_pitch < need || row_pitch % 16 != 0) {
    set_error("ppmoe_ep_dispatch: row_pitch=%d must be a multiple of 16 and >= %d", row_pitch, need);
    return PPMOE_ERR_INVALID_ARG;
  }
  if (ws_bytes < ppmoe_ep_dispatch_workspace_bytes(tokens, ranks)) {
    set_error("ppmoe_ep_dispatch: workspace %zu < %zu bytes", ws_bytes, ppmoe_ep_dispatch_workspace_bytes(tokens, ranks));
    return PPMOE_ERR_WORKSPACE;
  }
  if (!x || !weights || !send || !counts || !row_of || !ws || (reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(send)) % 16) {
    set_error("ppmoe_ep_dispatch: null pointer, or x / send not 16-byte aligned");
    return PPMOE_ERR_INVALID_ARG;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int nb = (tokens + kEpBlock - 1) / kEpBlock;
  int* blkcnt = static_cast<int*>(ws);
  int* blkoff = reinterpret_cast<int*>(static_cast<uint8_t*>(ws) + align_up((size_t)nb * ranks * 4, 256));
  if (nb > 0) {
    ep_count_kernel<<<nb, kEpBlock, 0, st>>>(static_cast<const __nv_bfloat16*>(weights), tokens, experts, ranks, blkcnt);
  }
  ep_scan_kernel<<<1, kEpMaxChunks * kEpMaxRanks, 0, st>>>(blkcnt, nb, ranks, chunks, blkoff,
                                                           reinterpret_cast<long long*>(counts));
  if (nb > 0) {
    ep_scatter_kernel<<<nb, kEpBlock, 0, st>>>(static_cast<const __nv_bfloat16*>(x),
                                               static_cast<const __nv_bfloat16*>(weights), tokens, hidden, experts,
                                               ranks, blkoff, static_cast<uint8_t*>(send), row_pitch, row_of);
  }
  PPMOE_CHECK_CUDA(cudaGetLastError());
  return PPMOE_OK;
}

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

extern "C" int ppmoe_ep_combine_f16s(const void* back, int pitch, const int32_t* row_of, int ranks, int tokens,
                                     int hidden, void* out, void* stream) {
  clear_error();
  if (ranks < 1 || ranks > 8 || tokens < 0 || hidden <= 0 || hidden % 64 != 0 || pitch < (int)f16s_pitch(hidden) ||
      pitch % 16 != 0) {
    set_error("ppmoe_ep_combine_f16s: ranks=%d (1..8), tokens=%d, hidden=%d (multiple of 64), pitch=%d (>= %zu, "
              "multiple of 16)", ranks, tokens, hidden, pitch, f16s_pitch(hidden > 0 ? hidden : 64));
    return PPMOE_ERR_UNSUPPORTED;
  }
  if (tokens == 0) return PPMOE_OK;
  if (!back || !row_of || !out) {
    set_error("ppmoe_ep_combine_f16s: null pointer");
    return PPMOE_ERR_INVALID_ARG;
  }
  ep_combine_f16s_kernel<<<tokens, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(back), pitch, row_of, ranks, tokens, hidden, static_cast<uint2*>(out));
  PPMOE_CHECK_CUDA(cudaGetLastError());
  return PPMOE_OK;
}
