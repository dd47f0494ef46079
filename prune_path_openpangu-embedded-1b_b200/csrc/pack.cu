// Packing pass: the reference-layout buffers that physical_reorder_for_inference mounts on
// TauSparseMoE (src/openpangu_moe.py:234-243: W_gate [H,I], W_up [H,I], W_down [I,H],
// router [H,E], neurons already grouped by expert) -> one packed blob (common.cuh):
//   router_eh [E][H]   transpose (one expert's router row contiguous: the decode router's
//                      per-rank rows and the K-major operand of the prefill router GEMM)
//   experts [E][G][3][H] per neuron n = e*G+j: W_gate[:,n] | W_up[:,n] | W_down[n,:]
//                      (one contiguous 3*H*2-byte record: what a decode CTA streams)
//   down_t [E][H][G]   per expert, W_down[e*G:(e+1)*G, :] transposed (K-major operand of
//                      the prefill down GEMM)
#include "common.cuh"

namespace ppmoe {

// dst[b][c * dst_ld + r] = src[b][r * src_ld + c], for r < R, c < C (bf16 bit patterns).
__global__ void transpose_bf16_kernel(const uint16_t* __restrict__ src, uint16_t* __restrict__ dst,
                                      int R, int C, long long src_ld, long long dst_ld,
                                      long long src_bs, long long dst_bs) {
  __shared__ uint16_t tile[32][33];
  const int b = blockIdx.z;
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  src += b * src_bs;
  dst += b * dst_bs;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int r = r0 + i, c = c0 + threadIdx.x;
    if (r < R && c < C) tile[i][threadIdx.x] = src[(long long)r * src_ld + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i, r = r0 + threadIdx.x;
    if (r < R && c < C) dst[(long long)c * dst_ld + r] = tile[threadIdx.x][i];
  }
}

static int transpose(const void* src, void* dst, int R, int C, long long src_ld, long long dst_ld,
                     int batch, long long src_bs, long long dst_bs, cudaStream_t st) {
  dim3 grid((C + 31) / 32, (R + 31) / 32, batch), block(32, 8);
  transpose_bf16_kernel<<<grid, block, 0, st>>>(static_cast<const uint16_t*>(src), static_cast<uint16_t*>(dst),
                                                 R, C, src_ld, dst_ld, src_bs, dst_bs);
  PPMOE_CHECK_CUDA(cudaGetLastError());
  return PPMOE_OK;
}

int pack_launch(const void* Wg, const void* Wu, const void* Wd, const void* R, int H, int E, int G,
                void* packed, cudaStream_t st) {
  const PackedLayout L = packed_layout(H, E, G);
  uint8_t* p = static_cast<uint8_t*>(packed);
  const long long I = (long long)E * G;
  int rc;
  if ((rc = transpose(R, p + L.router_eh, H, E, E, H, 1, 0, 0, st))) return rc;
  uint16_t* ex = reinterpret_cast<uint16_t*>(p + L.experts);
  if ((rc = transpose(Wg, ex, H, (int)I, I, 3LL * H, 1, 0, 0, st))) return rc;
  if ((rc = transpose(Wu, ex + H, H, (int)I, I, 3LL * H, 1, 0, 0, st))) return rc;
  PPMOE_CHECK_CUDA(cudaMemcpy2DAsync(ex + 2 * H, (size_t)3 * H * 2, Wd, (size_t)H * 2, (size_t)H * 2, (size_t)I,
                                     cudaMemcpyDeviceToDevice, st));
  if ((rc = transpose(Wd, p + L.down_t, G, H, H, G, E, (long long)G * H, (long long)G * H, st))) return rc;
  return PPMOE_OK;
}

}  // namespace ppmoe
