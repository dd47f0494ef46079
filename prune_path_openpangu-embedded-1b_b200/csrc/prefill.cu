// Prefill (more than 16 tokens): tcgen05 grouped GEMMs with device-side dispatch.
//
// Replaces TauSparseMoE.forward_prefill (src/tl_kernel_optimized_Ultimate_PanGU.py:532-604):
//   moe_router_kernel (tl:40-91)            -> router_gemm_kernel (tcgen05, M=128 tokens,
//                                             N=E, K=H) + route_logits_kernel (select.cuh)
//   torch.sort + moe_select_expert_kernel + scatter_ (tl:557-564)  -> route_logits_kernel
//   moe_local_scan / moe_global_scan (tl:133-212) + .item() sync   -> count / scan kernels;
//                                             the worst-case-sized workspace removes the host
//                                             sync and the 512-tile-per-expert cap (tl:176)
//   moe_dispatch_kernel (tl:217-266)        -> scatter_kernel (token order within expert)
//   moe_fused_expert_kernel (tl:271-328)    -> gu_gemm_pair_kernel (gathered token rows of
//                                             two 128-row tiles x the expert's interleaved
//                                             gate/up rows, SwiGLU and gate weight in the
//                                             epilogue -> a2 rows) + down_gemm_kernel (a2 x
//                                             down_t, one scaled-fp16 row per pair) +
//                                             pair_combine_kernel (per token, its rows in
//                                             expert order)
// Numerics follow the reference's bf16 rounding points; the per-token combine over experts
// accumulates in fp32 and rounds once (the reference Triton kernel adds bf16 atomics).
#include <cuda_fp16.h>
#include <mutex>
#include "umma.cuh"

namespace ppmoe {

int route_logits_launch(const void*, int, int, float, const float*, void*, uint8_t*, cudaStream_t,
                        void* probs_out = nullptr);
int route_compact_launch(const void*, int, int, float, int32_t*, void*, int32_t*, uint8_t*, cudaStream_t);

constexpr int kTileM = 128;
constexpr int kBK = 64;  // K elements per pipeline stage (one 128-byte swizzle row)
// Up to this many tokens the router GEMM splits K over kRouterSplit CTAs per 128-token tile
// (a lone CTA streaming all of K is latency-bound).
constexpr int kRouterSplit = 8;
constexpr int kRouterSplitMaxN = 512;

struct PrefillWs {
  size_t logits, weights, blockcnt, blockoff, count, exp_off, ntiles, tile_expert, tile_row0, unit_tile, pair_token,
      pair_w, a2, ypart, tok_pairs, tok_k, rpart, status, total;
  long long max_pairs, max_tiles;
  int nblocks;
};

static PrefillWs prefill_ws_layout(long long N, int H, int E, int G) {
  PrefillWs w;
  w.nblocks = (int)((N + 255) / 256);
  w.max_pairs = ((N * E + 127LL * E) + 127) / 128 * 128;
  w.max_tiles = w.max_pairs / 128;
  size_t o = 0;
  auto take = [&](size_t bytes) { size_t r = o; o = align_up(o + bytes, 1024); return r; };
  w.status = take(64);
  w.logits = take((size_t)N * E * 2);
  w.rpart = take(N <= kRouterSplitMaxN ? (size_t)kRouterSplit * N * E * 4 : 0);
  w.weights = take((size_t)N * E * 2);
  w.blockcnt = take((size_t)w.nblocks * E * 4);
  w.blockoff = take((size_t)w.nblocks * E * 4);
  w.count = take((size_t)E * 4);
  w.exp_off = take((size_t)E * 4);
  w.ntiles = take(16);
  w.tile_expert = take((size_t)w.max_tiles * 4);
  w.tile_row0 = take((size_t)w.max_tiles * 4);
  w.unit_tile = take((size_t)w.max_tiles * 4);
  w.pair_token = take((size_t)w.max_pairs * 4);
  w.pair_w = take((size_t)w.max_pairs * 4);
  w.a2 = take((size_t)w.max_pairs * G * 2);
  // down-projection row of every pair: fp16 values [pairs][H], then one int8 power-of-two
  // scale per 64-column slice [pairs][H / 64]
  w.ypart = take((size_t)w.max_pairs * H * 2 + align_up((size_t)w.max_pairs * (H / 64), 1024));
  w.tok_pairs = take((size_t)N * E * 4);        // per token: its pairs in expert order
  w.tok_k = take((size_t)N * 4);
  w.total = o;
  return w;
}

// ======================================================================== router GEMM
struct RouterArgs {
  int N, E, EP, H, stages;
  const float* bias;
  __nv_bfloat16* logits;
  uint32_t* status;
  int ksplit;   // > 1: CTA (tile, blockIdx.y) covers 1/ksplit of K and writes fp32 partials
  float* part;  // [ksplit][N][E] (ksplit > 1), summed in order by router_sum_kernel
};



__global__ void __launch_bounds__(192, 1)
router_gemm_kernel(const __grid_constant__ CUtensorMap mapX, const __grid_constant__ CUtensorMap mapR,
                   const RouterArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(align_up(reinterpret_cast<uintptr_t>(smem_raw), 1024));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t a_bytes = kTileM * 128, b_bytes = (uint32_t)a.EP * 128;
  const uint32_t stage_bytes = a_bytes + b_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.stages * stage_bytes);
  uint64_t* empty = full + a.stages;
  uint64_t* tfull = empty + a.stages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tfull + 1);
  const int KB = a.H / kBK;
  const uint32_t ncols = a.EP <= 32 ? 32 : a.EP <= 64 ? 64 : a.EP <= 128 ? 128 : 256;
  if (tid == 0) {
    for (int s = 0; s < a.stages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    mbar_init(tfull, 1);
    fence_mbar_init();
  }
  if (warp == 5) tmem_alloc(tmem_slot, ncols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int tile = blockIdx.x, ks = blockIdx.y;
  const int kb0 = KB * ks / a.ksplit, kb1 = KB * (ks + 1) / a.ksplit;  // this CTA's k-blocks

  if (warp == 4 && lane == 0) {  // TMA producer
    for (int kb = kb0; kb < kb1; ++kb) {
      const int j = kb - kb0, s = j % a.stages;
      mbar_wait_parked(&empty[s], ((j / a.stages) & 1) ^ 1, a.status);
      uint8_t* st = smem + s * stage_bytes;
      mbar_arrive_expect_tx(&full[s], stage_bytes);
      tma_load_2d(st, &mapX, kb * kBK, tile * kTileM, &full[s]);
      tma_load_2d(st + a_bytes, &mapR, kb * kBK, 0, &full[s]);
    }
  } else if (warp == 5 && lane == 0) {  // MMA issuer
    const uint32_t idesc = umma_idesc_bf16(kTileM, a.EP);
    for (int kb = kb0; kb < kb1; ++kb) {
      const int j = kb - kb0, s = j % a.stages;
      mbar_wait_parked(&full[s], (j / a.stages) & 1, a.status);
      tc_fence_after();
      const uint32_t sa = smem_u32(smem + s * stage_bytes);
      const uint64_t ad = umma_desc_sw128(sa), bd = umma_desc_sw128(sa + a_bytes);
#pragma unroll
      for (int k = 0; k < kBK / 16; ++k) umma_bf16(tmem, ad + 2 * k, bd + 2 * k, idesc, (j | k) != 0);
      umma_commit(&empty[s]);
    }
    umma_commit(tfull);
  } else if (warp < 4) {  // epilogue: row = token
    mbar_wait_parked(tfull, 0, a.status);
    tc_fence_after();
    const int t = tile * kTileM + warp * 32 + lane;
    for (int c0 = 0; c0 < a.EP; c0 += 32) {
      float v[32];
      tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + c0, v);
      if (t < a.N && a.ksplit > 1) {  // fp32 partial of this K range
        float* pr = a.part + ((size_t)ks * a.N + t) * a.E + c0;
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (c0 + j < a.E) pr[j] = v[j];
      } else if (t < a.N) {
        if (c0 + 32 <= a.E && a.E % 8 == 0 && (reinterpret_cast<uintptr_t>(a.logits) & 15) == 0) {
          // whole 32-expert chunk: four 16-byte stores
          uint32_t pk[16];
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            float l0 = bf16r(v[j]), l1 = bf16r(v[j + 1]);
            if (a.bias) { l0 = bf16r(l0 + a.bias[c0 + j]); l1 = bf16r(l1 + a.bias[c0 + j + 1]); }
            __nv_bfloat162 h2 = __floats2bfloat162_rn(l0, l1);
            pk[j / 2] = *reinterpret_cast<uint32_t*>(&h2);
          }
          uint4* dst = reinterpret_cast<uint4*>(a.logits + (size_t)t * a.E + c0);
#pragma unroll
          for (int q = 0; q < 4; ++q) dst[q] = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int e = c0 + j;
            if (e < a.E) {
              float l = bf16r(v[j]);
              if (a.bias) l = bf16r(l + a.bias[e]);
              a.logits[(size_t)t * a.E + e] = __float2bfloat16_rn(l);
            }
          }
        }
      }
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, ncols);
  }
}

// Logits of a K-split router GEMM: the ksplit fp32 partials summed in split order, rounded to
// bf16 (+ optional prior, rounded again), as the one-pass epilogue does.
__global__ void router_sum_kernel(const float* __restrict__ part, int ksplit, int N, int E, const float* __restrict__ bias,
                                  __nv_bfloat16* __restrict__ logits) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= N * E) return;
  float v = 0.f;
  for (int q = 0; q < ksplit; ++q) v += part[(size_t)q * N * E + i];
  float l = bf16r(v);
  if (bias) l = bf16r(l + bias[i % E]);
  logits[i] = __float2bfloat16_rn(l);
}

// ======================================================================== dispatch
__device__ __forceinline__ void count_body(int bx, const __nv_bfloat16* __restrict__ w, int wpitch, int N, int E,
                                           int* __restrict__ blockcnt) {
  // stage the block's 256 consecutive gate-weight rows (coalesced), then warp w counts
  // experts w, w + (warps), ... with one ballot per 32-token chunk
  extern __shared__ __align__(16) uint8_t cn_smem[];
  const int P = E + 2;
  __nv_bfloat16* ws = reinterpret_cast<__nv_bfloat16*>(cn_smem);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nw = blockDim.x >> 5;
  const int t0 = bx * 256, nt = min(256, N - t0);
  for (int i = tid; i < nt * E / 2; i += blockDim.x) {  // rows wpitch elements apart (E when dense)
    const int r = (2 * i) / E, c = (2 * i) % E;
    *reinterpret_cast<uint32_t*>(ws + r * P + c) =
        *reinterpret_cast<const uint32_t*>(w + (size_t)(t0 + r) * wpitch + c);
  }
  __syncthreads();
  for (int e = warp; e < E; e += nw) {
    int n = 0;
    for (int c = 0; c < 8; ++c) {
      const int r = c * 32 + lane;
      n += __popc(__ballot_sync(0xffffffffu, r < nt && __bfloat162float(ws[r * P + e]) > 0.f));
    }
    if (lane == 0) blockcnt[(size_t)bx * E + e] = n;
  }
}
__global__ void count_kernel(const __nv_bfloat16* __restrict__ w, int wpitch, int N, int E, int* __restrict__ blockcnt) {
  count_body(blockIdx.x, w, wpitch, N, E, blockcnt);
}

// One CTA of 1024 threads: per-expert prefix over token blocks, 128-padded expert offsets,
// tile list, gate/up units, padding rows, activation counts.  Warp w owns experts w, w + 32,
// ...: its lanes scan the expert's block counts 32 at a time (warp shuffles); warp 0 scans
// the experts' tile and unit counts.
__device__ __forceinline__ void scan_body(const int* __restrict__ blockcnt, int nblocks, int E,
                            int* __restrict__ blockoff, int* __restrict__ count, int* __restrict__ exp_off,
                            int* __restrict__ ntiles, int* __restrict__ tile_expert, int* __restrict__ tile_row0,
                            int* __restrict__ unit_tile, int* __restrict__ pair_token, float* __restrict__ pair_w,
                            long long* __restrict__ act_counts) {
  __shared__ int off_s[257];
  __shared__ int uoff_s[257];
  __shared__ int cnt_s[256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int e = warp; e < E; e += nw) {
    int carry = 0;
    for (int b0 = 0; b0 < nblocks; b0 += 32) {
      const int b = b0 + lane;
      const int v = b < nblocks ? blockcnt[(size_t)b * E + e] : 0;
      int inc = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += y;
      }
      if (b < nblocks) blockoff[(size_t)b * E + e] = carry + inc - v;
      carry += __shfl_sync(0xffffffffu, inc, 31);
    }
    if (lane == 0) {
      count[e] = carry;
      cnt_s[e] = carry;
      if (act_counts) act_counts[e] += carry;
    }
  }
  __syncthreads();
  if (warp == 0) {  // exclusive prefixes of the padded rows and of the units, in expert order
    int orow = 0, ou = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int e = e0 + lane;
      const int t = e < E ? (cnt_s[e] + kTileM - 1) / kTileM : 0;
      int it = t, iu = (t + 1) / 2;
      const int t0 = it, u0 = iu;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, it, o), z = __shfl_up_sync(0xffffffffu, iu, o);
        if (lane >= o) { it += y; iu += z; }
      }
      if (e < E) {
        off_s[e] = orow + (it - t0) * kTileM;
        uoff_s[e] = ou + (iu - u0);
      }
      orow += __shfl_sync(0xffffffffu, it, 31) * kTileM;
      ou += __shfl_sync(0xffffffffu, iu, 31);
    }
    if (lane == 0) {
      off_s[E] = orow;
      ntiles[0] = orow / kTileM;
      ntiles[1] = ou;
    }
  }
  __syncthreads();
  for (int e = warp; e < E; e += nw) {
    const int o = off_s[e], t = (off_s[e + 1] - o) / kTileM;
    if (lane == 0) exp_off[e] = o;
    for (int i = lane; i < t; i += 32) {
      tile_expert[o / kTileM + i] = e;
      tile_row0[o / kTileM + i] = o + i * kTileM;
    }
    // gate/up work units: consecutive tile pairs of one expert (first tile * 2 + has-second)
    for (int i = 2 * lane; i < t; i += 64) unit_tile[uoff_s[e] + i / 2] = (o / kTileM + i) * 2 + (i + 1 < t);
    // padding rows of the expert's last tile
    for (int p = o + cnt_s[e] + lane; p < off_s[e + 1]; p += 32) { pair_token[p] = -1; pair_w[p] = 0.f; }
  }
}
__global__ void __launch_bounds__(1024) scan_kernel(const int* __restrict__ blockcnt, int nblocks, int E,
                            int* __restrict__ blockoff, int* __restrict__ count, int* __restrict__ exp_off,
                            int* __restrict__ ntiles, int* __restrict__ tile_expert, int* __restrict__ tile_row0,
                            int* __restrict__ unit_tile, int* __restrict__ pair_token, float* __restrict__ pair_w,
                            long long* __restrict__ act_counts) {
  scan_body(blockcnt, nblocks, E, blockoff, count, exp_off, ntiles, tile_expert, tile_row0, unit_tile, pair_token,
            pair_w, act_counts);
}

// Per token block: (token, expert) pairs in token order within each expert.
__device__ __forceinline__ void scatter_body(int bx, const __nv_bfloat16* __restrict__ w, int wpitch, int N, int E, const int* __restrict__ blockoff,
                               const int* __restrict__ exp_off, int* __restrict__ pair_token,
                               float* __restrict__ pair_w, int* __restrict__ tok_pairs, int* __restrict__ tok_k) {
  // The block's 256 gate-weight rows are consecutive in memory: one coalesced copy into shared
  // memory (row pitch E + 2 elements against bank conflicts), plus each token's selection
  // bitmask.  Warp w owns experts w, w + (warps), ... and walks the 8 token chunks in order, so each
  // pair's slot is a running ballot prefix; the token-side index (its pairs in expert order)
  // comes from the bitmask.
  extern __shared__ __align__(16) uint8_t sc_smem[];
  const int P = E + 2;
  __nv_bfloat16* ws = reinterpret_cast<__nv_bfloat16*>(sc_smem);          // [256][E + 2]
  uint32_t* bm = reinterpret_cast<uint32_t*>(sc_smem + (size_t)256 * P * 2);  // [256][8]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t0 = bx * 256, nt = min(256, N - t0);
  const int nw = blockDim.x >> 5;
  for (int i = tid; i < nt * E / 2; i += blockDim.x) {  // rows wpitch elements apart (E when dense)
    const int r = (2 * i) / E, c = (2 * i) % E;
    *reinterpret_cast<uint32_t*>(ws + r * P + c) =
        *reinterpret_cast<const uint32_t*>(w + (size_t)(t0 + r) * wpitch + c);
  }
  __syncthreads();
  if (tid < nt) {
    int k = 0;
    for (int q = 0; q < (E + 31) / 32; ++q) {
      uint32_t m = 0;
      for (int b = 0; b < 32 && q * 32 + b < E; ++b)
        m |= (uint32_t)(__bfloat162float(ws[tid * P + q * 32 + b]) > 0.f) << b;
      bm[tid * 8 + q] = m;
      k += __popc(m);
    }
    tok_k[t0 + tid] = k;
  }
  __syncthreads();
  for (int e = warp; e < E; e += nw) {
    int run = exp_off[e] + blockoff[(size_t)bx * E + e];
    for (int c = 0; c < 8; ++c) {
      const int r = c * 32 + lane;
      const float wv = r < nt ? __bfloat162float(ws[r * P + e]) : 0.f;
      const uint32_t b = __ballot_sync(0xffffffffu, wv > 0.f);
      if (wv > 0.f) {
        const int pos = run + __popc(b & ((1u << lane) - 1u));
        pair_token[pos] = t0 + r;
        pair_w[pos] = wv;
        int j = __popc(bm[r * 8 + (e >> 5)] & ((1u << (e & 31)) - 1u));
        for (int q = 0; q < (e >> 5); ++q) j += __popc(bm[r * 8 + q]);
        tok_pairs[(size_t)(t0 + r) * E + j] = pos;
      }
      run += __popc(b);
    }
  }
}
__global__ void scatter_kernel(const __nv_bfloat16* __restrict__ w, int wpitch, int N, int E, const int* __restrict__ blockoff,
                               const int* __restrict__ exp_off, int* __restrict__ pair_token,
                               float* __restrict__ pair_w, int* __restrict__ tok_pairs, int* __restrict__ tok_k) {
  scatter_body(blockIdx.x, w, wpitch, N, E, blockoff, exp_off, pair_token, pair_w, tok_pairs, tok_k);
}

// At most 256 tokens (one token block): count, scan and scatter in one CTA, one launch.
__global__ void __launch_bounds__(1024) dispatch_one_block_kernel(
    const __nv_bfloat16* __restrict__ w, int wpitch, int N, int E, int* __restrict__ blockcnt,
    int* __restrict__ blockoff, int* __restrict__ count, int* __restrict__ exp_off, int* __restrict__ ntiles,
    int* __restrict__ tile_expert, int* __restrict__ tile_row0, int* __restrict__ unit_tile,
    int* __restrict__ pair_token, float* __restrict__ pair_w, long long* __restrict__ act_counts,
    int* __restrict__ tok_pairs, int* __restrict__ tok_k) {
  count_body(0, w, wpitch, N, E, blockcnt);
  __syncthreads();  // the block's own global writes are visible to it after the barrier
  scan_body(blockcnt, 1, E, blockoff, count, exp_off, ntiles, tile_expert, tile_row0, unit_tile, pair_token, pair_w,
            act_counts);
  __syncthreads();
  scatter_body(0, w, wpitch, N, E, blockoff, exp_off, pair_token, pair_w, tok_pairs, tok_k);
}

// ======================================================================== gate/up GEMM
struct GUArgs {
  const __nv_bfloat16* x;
  int H, G;
  int xpitch;  // elements between token rows (H when dense)
  const int* tile_expert;
  const int* tile_row0;
  const int* ntiles;
  const int* pair_token;
  const float* pair_w;
  __nv_bfloat16* a2;  // [pairs][G]
  uint32_t* status;
  int stages;  // pipeline depth (set from the shared-memory budget)
};

constexpr int kGUMaxStages = 5;  // cp.async groups kept in flight per producer thread

// Gate/up over tile PAIRS: two 128-row tiles of one expert share every B (weight) stage, so
// each expert's gate/up rows are read from L2 once per 256 pair rows instead of once per 128.
// Per 64-wide k-block: two 128 x 2G x 16 MMAs per k step (accumulators at TMEM columns 0 and
// 256).  Warps 0-15 are the epilogue (warp w: tile w / 8, column half (w / 4) % 2, TMEM lane
// quarter w % 4), warps 16-23 gather the 256 token rows with cp.async, warp 24 allocates TMEM
// and issues the MMAs.
// The one accumulator pair is not double-buffered (2 x 2G columns fill TMEM's 512), so a
// unit's epilogue runs before the next unit's first MMA.
struct GUPairArgs {
  GUArgs g;
  const int* unit_tile;  // per unit: first tile * 2 + (1 if the unit has a second tile)
  int nsplit;            // 1, or 2: each unit's neurons in two halves run as separate units
};

constexpr int kGUEpi = 16;                       // epilogue warps (8 or 16; 8 with 16 producers: 584 vs 562 us at config 3)
constexpr int kGUProd = 8;                       // producer warps (gathers), half per tile (8 or 16)
constexpr int kGUThreads = 32 * (kGUEpi + kGUProd + 1);  // + 1 MMA warp

__global__ void __launch_bounds__(kGUThreads, 1)
gu_gemm_pair_kernel(const __grid_constant__ CUtensorMap mapGU, const GUPairArgs pa) {
  const GUArgs& a = pa.g;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(align_up(reinterpret_cast<uintptr_t>(smem_raw), 1024));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int S = a.stages, LAG = S - 2;
  const int NS = pa.nsplit, GS = a.G / NS;  // neurons per (split) unit
  const int NB = 2 * GS;
  const uint32_t a_bytes = kTileM * 128, b_bytes = (uint32_t)NB * 128;
  const uint32_t stage_bytes = 2 * a_bytes + b_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * stage_bytes);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 1);
  const int KB = a.H / kBK;
  const int nunits = a.ntiles[1] * NS;  // unit u: tile pair u / NS, neuron half u % NS
  if (tid == 0) {
    for (int s = 0; s < S; ++s) { mbar_init(&full[s], 32 * kGUProd + 1); mbar_init(&empty[s], 1); }
    mbar_init(tfull, 1);
    mbar_init(tempty, 32 * kGUEpi);
    fence_mbar_init();
  }
  if (warp == kGUEpi + kGUProd) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp >= kGUEpi && warp < kGUEpi + kGUProd) {  // producers: gathered token rows; B via TMA
    // Producer warp pw fills RPW consecutive rows of tile pw / WPT.  Per instruction its 32
    // lanes copy the 128-byte k-slices of 4 rows (8 lanes per row, one 16-byte chunk each), so
    // every copy instruction reads 4 whole 128-byte lines.
    constexpr int WPT = kGUProd / 2, RPW = kTileM / WPT, NI = RPW / 4;
    const int pr = tid - 32 * kGUEpi, pw = warp - kGUEpi, h = pw / WPT, rbase = (pw % WPT) * RPW, sub = lane >> 3, ck = lane & 7;
    uint8_t* const a_base = smem + h * a_bytes;
    int it = 0;
    // padding rows and the absent second tile load nothing: their stale shared-memory rows
    // only reach accumulator rows that the epilogue discards.  Unit u + grid's row pointers are
    // loaded while unit u streams (three dependent global loads off the critical path).
    auto unit_src = [&](int u, const __nv_bfloat16* (&src)[NI], int& e) {
      e = 0;
#pragma unroll
      for (int i = 0; i < NI; ++i) src[i] = nullptr;
      if (u >= nunits) return;
      const int ut = pa.unit_tile[u / NS], t0 = ut >> 1;
      e = a.tile_expert[t0];
      if (h == 0 || (ut & 1)) {
        const int row0 = a.tile_row0[t0 + h];
#pragma unroll
        for (int i = 0; i < NI; ++i) {
          const int tok = a.pair_token[row0 + rbase + 4 * i + sub];
          src[i] = tok >= 0 ? a.x + (size_t)tok * a.xpitch + ck * 8 : nullptr;
        }
      }
    };
    const __nv_bfloat16* nsrc[NI];
    int ne;
    unit_src(blockIdx.x, nsrc, ne);
    for (int u = blockIdx.x; u < nunits; u += gridDim.x) {
      const int nh = u % NS, e = ne;
      const __nv_bfloat16* src[NI];
#pragma unroll
      for (int i = 0; i < NI; ++i) src[i] = nsrc[i];
      unit_src(u + gridDim.x, nsrc, ne);
      for (int kb = 0; kb < KB; ++kb, ++it) {
        const int s = it % S;
        mbar_wait_parked(&empty[s], ((it / S) & 1) ^ 1, a.status);
        uint8_t* st = a_base + s * stage_bytes;
#pragma unroll
        for (int i = 0; i < NI; ++i)
          if (src[i]) cp_async16(st + sw128_offset(rbase + 4 * i + sub, ck), src[i] + kb * kBK);
        cp_async_commit();
        if (pr == 0) {
          mbar_arrive_expect_tx(&full[s], b_bytes);
          tma_load_3d(smem + s * stage_bytes + 2 * a_bytes, &mapGU, kb * kBK, 0, e * a.G + nh * GS, &full[s]);
        }
        if (it >= LAG) {
          if (LAG == 3) cp_async_wait<3>(); else if (LAG == 2) cp_async_wait<2>(); else cp_async_wait<1>();
          fence_proxy_async();
          mbar_arrive(&full[(it - LAG) % S]);
        }
      }
    }
    cp_async_wait<0>();
    fence_proxy_async();
    for (int j = max(0, it - LAG); j < it; ++j) mbar_arrive(&full[j % S]);
  } else if (warp == kGUEpi + kGUProd && lane == 0) {  // MMA issuer
    const uint32_t idesc = umma_idesc_bf16(kTileM, NB);
    int it = 0, ul = 0;
    for (int u = blockIdx.x; u < nunits; u += gridDim.x, ++ul) {
      const bool two = pa.unit_tile[u / NS] & 1;
      mbar_wait_parked(tempty, (ul & 1) ^ 1, a.status);
      tc_fence_after();
      for (int kb = 0; kb < KB; ++kb, ++it) {
        const int s = it % S;
        mbar_wait_parked(&full[s], (it / S) & 1, a.status);
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + s * stage_bytes);
        const uint64_t ad0 = umma_desc_sw128(sa), ad1 = umma_desc_sw128(sa + a_bytes),
                       bd = umma_desc_sw128(sa + 2 * a_bytes);
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k) {
          umma_bf16(tmem, ad0 + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
          if (two) umma_bf16(tmem + 256, ad1 + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
        }
        umma_commit(&empty[s]);
      }
      umma_commit(tfull);
    }
  } else if (warp < kGUEpi) {  // epilogue: row r of tile h = pair; SwiGLU with the reference's rounding points
    // 16 warps: tile w / 8, column half (w / 4) % 2, TMEM lane quarter w % 4; 8 warps: tile w / 4
    constexpr int EPT = kGUEpi / 2;  // epilogue warps per tile
    const int h = warp / EPT, cw = EPT == 8 ? (warp >> 2) & 1 : 0, q = warp & 3, r = q * 32 + lane;
    const int cmid = EPT == 8 ? NB / 64 * 32 : NB, cbeg = cw ? cmid : 0, cend = cw ? NB : cmid;  // this warp's columns
    int ul = 0;
    for (int u = blockIdx.x; u < nunits; u += gridDim.x, ++ul) {
      // the unit's rows and gate weights are known before its accumulators: load them first so
      // that their latency overlaps the main loop
      const int ut = pa.unit_tile[u / NS], nh = u % NS;
      const bool has = h == 0 || (ut & 1);
      const int p = has ? a.tile_row0[(ut >> 1) + h] + r : 0;
      const float wg = has ? a.pair_w[p] : 0.f;
      mbar_wait_parked(tfull, ul & 1, a.status);
      tc_fence_after();
      if (has) {
        __nv_bfloat16* orow = a.a2 + (size_t)p * a.G + nh * GS;
        for (int c0 = cbeg; c0 < cend; c0 += 32) {
          float v[32];
          tmem_ld32(tmem + h * 256 + ((uint32_t)(q * 32) << 16) + c0, v);
          uint32_t pk[8];
#pragma unroll
          for (int j = 0; j < 16; j += 2) {
            float o2[2];
#pragma unroll
            for (int i = 0; i < 2; ++i) {
              const float gb = bf16r(v[2 * (j + i)]), ub = bf16r(v[2 * (j + i) + 1]);
              const float sb = bf16r(__fmul_rn(gb, __frcp_rn(1.f + expf(-gb))));  // silu
              o2[i] = bf16r(bf16r(sb * ub) * wg);
            }
            __nv_bfloat162 h2 = __floats2bfloat162_rn(o2[0], o2[1]);
            pk[j / 2] = *reinterpret_cast<uint32_t*>(&h2);
          }
          uint4* dst = reinterpret_cast<uint4*>(orow + c0 / 2);
          dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        }
      }
      tc_fence_before();
      mbar_arrive(tempty);
    }
  }
  __syncthreads();
  if (warp == kGUEpi + kGUProd) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ======================================================================== down GEMM + combine
struct DownArgs {
  int H, G, NCW;
  int NGRP;  // units per tile: tile t's column chunks in NGRP consecutive groups (small batches)
  int8_t* yscale;  // [pairs][H / 64] exponent s of each slice's scale 2^s
  const int* tile_expert;
  const int* tile_row0;
  const int* ntiles;
  const int* pair_token;
  uint32_t* status;
};

constexpr int kDownStages = 3;
constexpr int kDownEpiWarps = 8;  // two warpgroups, each converting alternate 64-column slices
constexpr int kDownThreads = 32 * (kDownEpiWarps + 2);

__global__ void __launch_bounds__(kDownThreads, 1)
down_gemm_kernel(const __grid_constant__ CUtensorMap mapA2, const __grid_constant__ CUtensorMap mapD,
                 const __grid_constant__ CUtensorMap mapYh, const DownArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(align_up(reinterpret_cast<uintptr_t>(smem_raw), 1024));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int KB2 = (a.G + kBK - 1) / kBK;  // 1 or 2 (G <= 128)
  const uint32_t a_kb = kTileM * 128;             // one 64-wide k-block of A
  const uint32_t b_kb = (uint32_t)a.NCW * 128;    // one 64-wide k-block of a B chunk
  const uint32_t a_bytes = KB2 * a_kb, b_bytes = KB2 * b_kb;
  uint8_t* sA = smem;  // two A tiles: the next tile's loads overlap this tile's chunks
  uint8_t* sB = smem + 2 * a_bytes;
  uint64_t* bfull = reinterpret_cast<uint64_t*>(sB + kDownStages * b_bytes);
  uint64_t* bempty = bfull + kDownStages;
  uint64_t* afull = bempty + kDownStages;  // [2]
  uint64_t* aempty = afull + 2;            // [2]
  uint64_t* tfull = aempty + 2;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  uint8_t* stg = reinterpret_cast<uint8_t*>(align_up(reinterpret_cast<uintptr_t>(tempty + 2) + 16, 1024));
  const int NCH = a.H / a.NCW, NCG = NCH / a.NGRP;
  const int nunits = *a.ntiles * a.NGRP;
  if (tid == 0) {
    for (int s = 0; s < kDownStages; ++s) { mbar_init(&bfull[s], 1); mbar_init(&bempty[s], 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(&afull[i], 1); mbar_init(&aempty[i], 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(&tfull[i], 1); mbar_init(&tempty[i], 32 * kDownEpiWarps); }
    fence_mbar_init();
  }
  if (warp == kDownEpiWarps + 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kDownEpiWarps && lane == 0) {  // TMA producer
    int tl = 0, ch = 0;
    for (int un = blockIdx.x; un < nunits; un += gridDim.x, ++tl) {
      const int tile = un / a.NGRP, cb = (un % a.NGRP) * NCG;
      const int e = a.tile_expert[tile], row0 = a.tile_row0[tile];
      const int ab = tl & 1;
      mbar_wait_parked(&aempty[ab], ((tl >> 1) & 1) ^ 1, a.status);
      mbar_arrive_expect_tx(&afull[ab], a_bytes);
      for (int kb = 0; kb < KB2; ++kb) tma_load_2d(sA + ab * a_bytes + kb * a_kb, &mapA2, kb * kBK, row0, &afull[ab]);
      for (int c = cb; c < cb + NCG; ++c, ++ch) {
        const int s = ch % kDownStages;
        mbar_wait_parked(&bempty[s], ((ch / kDownStages) & 1) ^ 1, a.status);
        mbar_arrive_expect_tx(&bfull[s], b_bytes);
        for (int kb = 0; kb < KB2; ++kb)
          tma_load_2d(sB + s * b_bytes + kb * b_kb, &mapD, kb * kBK, e * a.H + c * a.NCW, &bfull[s]);
      }
    }
  } else if (warp == kDownEpiWarps + 1 && lane == 0) {  // MMA issuer
    const uint32_t idesc = umma_idesc_bf16(kTileM, a.NCW);
    int tl = 0, ch = 0;
    for (int un = blockIdx.x; un < nunits; un += gridDim.x, ++tl) {
      const int ab = tl & 1;
      mbar_wait_parked(&afull[ab], (tl >> 1) & 1, a.status);
      tc_fence_after();
      for (int c = 0; c < NCG; ++c, ++ch) {
        const int s = ch % kDownStages, acc = ch & 1;
        mbar_wait_parked(&tempty[acc], ((ch >> 1) & 1) ^ 1, a.status);
        mbar_wait_parked(&bfull[s], (ch / kDownStages) & 1, a.status);
        tc_fence_after();
        for (int k16 = 0; k16 < a.G / 16; ++k16) {
          const int kb = k16 >> 2, kk = k16 & 3;
          const uint64_t ad = umma_desc_sw128(smem_u32(sA + ab * a_bytes + kb * a_kb)) + 2 * kk;
          const uint64_t bd = umma_desc_sw128(smem_u32(sB + s * b_bytes + kb * b_kb)) + 2 * kk;
          umma_bf16(tmem + acc * 256, ad, bd, idesc, k16 != 0);
        }
        umma_commit(&bempty[s]);
        umma_commit(&tfull[acc]);
      }
      umma_commit(&aempty[ab]);
    }
  } else if (warp < kDownEpiWarps) {  // epilogue: the tile's rows, stored in pair order as scaled fp16
    // Per 64-column slice of a row: s = 14 - exponent(max |v|) (clamped), the values scaled by
    // 2^s (exact) and rounded to fp16 (relative error <= 2^-11; |v 2^s| < 2^15, inside fp16's
    // range whatever the magnitudes), s stored beside the row.  Every thread writes its row of
    // the slice into a swizzled staging tile ([128 x 128 B], 128-byte swizzle, conflict-free),
    // the warpgroup's 4 warps meet at a named barrier, and one thread stores the tile with a
    // TMA tensor store.  Warpgroup hf takes slices hf, hf + 2, ... of each chunk (TMEM lane
    // quarter = warp % 4) and alternates two staging tiles of its own; a tile is rewritten only
    // after its store has read it.
    const int hf = warp >> 2, wq = warp & 3, r = wq * 32 + lane;
    constexpr int NWG = kDownEpiWarps / 4;
    const int S64 = a.H / 64;
    int ch = 0, sub = 0;
    for (int un = blockIdx.x; un < nunits; un += gridDim.x) {
      const int tile = un / a.NGRP, cb = (un % a.NGRP) * NCG;
      const int row0 = a.tile_row0[tile];
      for (int c = cb; c < cb + NCG; ++c, ++ch) {
        const int acc = ch & 1;
        mbar_wait_parked(&tfull[acc], (ch >> 1) & 1, a.status);
        tc_fence_after();
        for (int c0 = 64 * hf; c0 < a.NCW; c0 += 64 * NWG, ++sub) {
          uint8_t* hb = stg + (hf * 2 + (sub & 1)) * 16384;
          if (r == 0) bulk_wait_read<1>();
          named_bar_sync(1 + hf, 128);  // the buffer is free
          float v[2][32];
          tmem_ld32(tmem + acc * 256 + ((uint32_t)(wq * 32) << 16) + c0, v[0]);
          tmem_ld32(tmem + acc * 256 + ((uint32_t)(wq * 32) << 16) + c0 + 32, v[1]);
          float m = 0.f;
#pragma unroll
          for (int i = 0; i < 32; ++i) m = fmaxf(m, fmaxf(fabsf(v[0][i]), fabsf(v[1][i])));
          int sc = m > 0.f ? 14 - ((int)((__float_as_uint(m) >> 23) & 255u) - 127) : 0;
          sc = max(-126, min(126, sc));
          const float mul = __uint_as_float((uint32_t)(sc + 127) << 23);
          a.yscale[(size_t)(row0 + r) * S64 + (c * a.NCW + c0) / 64] = (int8_t)sc;
#pragma unroll
          for (int half = 0; half < 2; ++half) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              uint32_t pk[4];
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                __half2 h2 = __floats2half2_rn(v[half][8 * j + 2 * q] * mul, v[half][8 * j + 2 * q + 1] * mul);
                pk[q] = *reinterpret_cast<uint32_t*>(&h2);
              }
              *reinterpret_cast<uint4*>(hb + sw128_offset(r, 4 * half + j)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            }
          }
          fence_proxy_async();
          named_bar_sync(1 + hf, 128);  // the tile is complete
          if (r == 0) {
            tma_store_2d(&mapYh, hb, c * a.NCW + c0, row0);
            bulk_commit();
          }
        }
        tc_fence_before();
        mbar_arrive(&tempty[acc]);
      }
    }
    if (r == 0) bulk_wait<0>();
  }
  __syncthreads();
  if (warp == kDownEpiWarps + 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Per token: the rows of its pairs (scaled fp16, one power-of-two scale per 64-column slice)
// added in expert order in fp32 (deterministic), rounded once to bf16 (or written as fp32
// partial sums for expert-parallel ranks).  Thread c owns columns 8c .. 8c + 7.
__device__ __forceinline__ void unpack_h8(const uint4 h, int sc, float* f) {
  const float inv = __uint_as_float((uint32_t)(127 - sc) << 23);  // 2^-s, exact
  const __half2* p = reinterpret_cast<const __half2*>(&h);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __half22float2(p[i]);
    f[2 * i] = t.x * inv;
    f[2 * i + 1] = t.y * inv;
  }
}

// OUT: 0 bf16 rows, 1 fp32 partial rows, 2 scaled-fp16 partial rows of `opitch` bytes (H fp16,
// then H / 64 int8 slice exponents: the expert-parallel return format, f16s_pitch)
template <int OUT>
__global__ void pair_combine_kernel(const uint4* __restrict__ yv, const int8_t* __restrict__ ysc,
                                    const int* __restrict__ tok_pairs, const int* __restrict__ tok_k, int E, int H8,
                                    void* __restrict__ out, int opitch = 0) {
  __shared__ int rows[256];
  const int t = blockIdx.x;
  const int k = tok_k[t];
  const int S64 = H8 / 8;
  for (int j = threadIdx.x; j < k; j += blockDim.x) rows[j] = tok_pairs[(size_t)t * E + j];
  __syncthreads();
  for (int c = threadIdx.x; c < H8; c += blockDim.x) {
    float s[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i] = 0.f;
    int j = 0;
    for (; j + 4 <= k; j += 4) {  // four rows' loads in flight, added in order
      uint4 h[4];
      int sc[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        h[q] = yv[(size_t)rows[j + q] * H8 + c];
        sc[q] = ysc[(size_t)rows[j + q] * S64 + (c >> 3)];
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float f[8];
        unpack_h8(h[q], sc[q], f);
#pragma unroll
        for (int i = 0; i < 8; ++i) s[i] += f[i];
      }
    }
    for (; j < k; ++j) {
      float f[8];
      unpack_h8(yv[(size_t)rows[j] * H8 + c], ysc[(size_t)rows[j] * S64 + (c >> 3)], f);
#pragma unroll
      for (int i = 0; i < 8; ++i) s[i] += f[i];
    }
    if (OUT == 1) {
      float4* o = static_cast<float4*>(out) + ((size_t)t * H8 + c) * 2;
      o[0] = make_float4(s[0], s[1], s[2], s[3]);
      o[1] = make_float4(s[4], s[5], s[6], s[7]);
    } else if (OUT == 2) {
      // the slice's 8 threads (aligned lane groups: H is a multiple of 64) agree on its scale
      float m = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(s[i]));
      const unsigned am = __activemask();
      m = fmaxf(m, __shfl_xor_sync(am, m, 1));
      m = fmaxf(m, __shfl_xor_sync(am, m, 2));
      m = fmaxf(m, __shfl_xor_sync(am, m, 4));
      int sc = m > 0.f ? 14 - ((int)((__float_as_uint(m) >> 23) & 255u) - 127) : 0;
      sc = max(-126, min(126, sc));
      const float mul = __uint_as_float((uint32_t)(sc + 127) << 23);
      uint8_t* row = static_cast<uint8_t*>(out) + (size_t)t * opitch;
      uint32_t pk[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        __half2 h2 = __floats2half2_rn(s[2 * i] * mul, s[2 * i + 1] * mul);
        pk[i] = *reinterpret_cast<uint32_t*>(&h2);
      }
      reinterpret_cast<uint4*>(row)[c] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      if ((c & 7) == 0) reinterpret_cast<int8_t*>(row + (size_t)H8 * 16)[c >> 3] = (int8_t)sc;
    } else {
      uint32_t pk[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        __nv_bfloat162 b = __floats2bfloat162_rn(s[2 * i], s[2 * i + 1]);
        pk[i] = *reinterpret_cast<uint32_t*>(&b);
      }
      static_cast<uint4*>(out)[(size_t)t * H8 + c] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
  }
}

// ======================================================================== host
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// bf16 tensor map of rank 2 or 3, 128-byte swizzle, zero fill out of bounds.
static int make_map(CUtensorMap* m, const void* base, int rank, const cuuint64_t* dims, const cuuint64_t* strides_bytes,
                    const cuuint32_t* box) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is unavailable from the driver");
    return PPMOE_ERR_CUDA;
  }
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (cuuint32_t)rank, const_cast<void*>(base), dims, strides_bytes,
                  box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d)", (int)r);
    return PPMOE_ERR_CUDA;
  }
  return PPMOE_OK;
}

// Rank-2 map of any element type and swizzle, for the pair-row tile stores.
static int make_map_2d(CUtensorMap* m, const void* base, CUtensorMapDataType dt, CUtensorMapSwizzle sw,
                       const cuuint64_t* dims, const cuuint64_t* strides_bytes, const cuuint32_t* box) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is unavailable from the driver");
    return PPMOE_ERR_CUDA;
  }
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides_bytes, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled (pair rows) failed (%d)", (int)r);
    return PPMOE_ERR_CUDA;
  }
  return PPMOE_OK;
}

size_t prefill_workspace_bytes(long long N, int H, int E, int G) { return prefill_ws_layout(N, H, E, G).total; }
size_t route_workspace_bytes(long long N, int E);

// mode: kPrefillFull (router -> selection -> experts -> bf16 out), kPrefillRouteOnly (stop
// after the gate weights), kPrefillExperts (gate weights given in weights_out; expert compute
// only; `out` receives fp32 partial sums instead of bf16).
enum { kPrefillFull = 0, kPrefillRouteOnly = 1, kPrefillExperts = 2, kPrefillExpertsF16s = 3 };

int prefill_launch(const void* x, int N, const void* packed, int H, int E, int G, float tau, const float* bias,
                   void* out, void* logits_out, void* weights_out, int64_t* counts, void* wsp, size_t ws_bytes,
                   cudaStream_t st, int mode, int xpitch, int wpitch) {
  if (xpitch <= 0) xpitch = H;
  if (wpitch <= 0) wpitch = E;
  const PrefillWs W = prefill_ws_layout(N, H, E, G);
  // routing alone touches only the status word and the logits (the first two regions of the
  // layout, identical to the routing workspace of ppmoe_route)
  const size_t need = mode == kPrefillRouteOnly ? route_workspace_bytes(N, E) : W.total;
  if (ws_bytes < need) {
    set_error("ppmoe_prefill: workspace %zu < %zu bytes needed for %d tokens", ws_bytes, need, N);
    return PPMOE_ERR_WORKSPACE;
  }
  uint8_t* ws = static_cast<uint8_t*>(wsp);
  const PackedLayout PL = packed_layout(H, E, G);
  const uint8_t* pk = static_cast<const uint8_t*>(packed);
  uint32_t* status = reinterpret_cast<uint32_t*>(ws + W.status);
  __nv_bfloat16* logits = logits_out ? static_cast<__nv_bfloat16*>(logits_out)
                                     : reinterpret_cast<__nv_bfloat16*>(ws + W.logits);
  __nv_bfloat16* weights = weights_out ? static_cast<__nv_bfloat16*>(weights_out)
                                       : reinterpret_cast<__nv_bfloat16*>(ws + W.weights);
  int dev = 0, nsm = 0, rc;
  PPMOE_CHECK_CUDA(cudaGetDevice(&dev));
  PPMOE_CHECK_CUDA(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev));

  // ---- router GEMM + selection
  const int EP = (E + 15) / 16 * 16;
  CUtensorMap mX, mR, mGU, mA2, mD;
  // Batches of a few hundred tokens (about one or two 128-row tiles per expert) give the
  // grouped GEMMs fewer work units than SMs.  There each gate/up unit is split into two neuron
  // halves and each down tile into column groups, so that more SMs stream the experts' weights
  // (measured 3-4% faster from 128 to 1,024 tokens; slower below 128 tokens, where every
  // kernel is latency-bound and the extra units only add work).
  static const int small_split = [] { const char* v = getenv("PPMOE_SMALL_SPLIT"); return v ? atoi(v) : 1; }();
  const bool small = small_split && N > 128 && N <= 1024;
  const int gu_split = small && G % 32 == 0 ? 2 : 1;
  {
    cuuint64_t d[2] = {(cuuint64_t)H, (cuuint64_t)N}, s[1] = {(cuuint64_t)H * 2};
    cuuint32_t b[2] = {kBK, kTileM};
    if ((rc = make_map(&mX, x, 2, d, s, b))) return rc;
  }
  {
    cuuint64_t d[2] = {(cuuint64_t)H, (cuuint64_t)E}, s[1] = {(cuuint64_t)H * 2};
    cuuint32_t b[2] = {kBK, (cuuint32_t)EP};
    if ((rc = make_map(&mR, pk + PL.router_eh, 2, d, s, b))) return rc;
  }
  if (mode == kPrefillRouteOnly) {  // router GEMM + selection only: the router rows alone are read
    const int rstages = EP <= 64 ? 8 : EP <= 128 ? 6 : 4;
    RouterArgs ra{N, E, EP, H, rstages, bias, logits, status, 1, nullptr};
    const size_t r_smem = 1024 + rstages * (kTileM * 128 + (size_t)EP * 128) + 256;
    PPMOE_CHECK_CUDA(cudaFuncSetAttribute(router_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)r_smem));
    router_gemm_kernel<<<(N + kTileM - 1) / kTileM, 192, r_smem, st>>>(mX, mR, ra);
    PPMOE_CHECK_CUDA(cudaGetLastError());
    return route_logits_launch(logits, N, E, tau, nullptr, weights, nullptr, st);
  }
  {
    cuuint64_t d[3] = {(cuuint64_t)H, 2, (cuuint64_t)E * G}, s[2] = {(cuuint64_t)H * 2, (cuuint64_t)H * 6};
    cuuint32_t b[3] = {kBK, 2, (cuuint32_t)(G / gu_split)};
    if ((rc = make_map(&mGU, pk + PL.experts, 3, d, s, b))) return rc;
  }
  {
    cuuint64_t d[2] = {(cuuint64_t)G, (cuuint64_t)W.max_pairs}, s[1] = {(cuuint64_t)G * 2};
    cuuint32_t b[2] = {kBK, kTileM};
    if ((rc = make_map(&mA2, ws + W.a2, 2, d, s, b))) return rc;
  }
  const int NCW = H % 128 == 0 ? 128 : 64;  // B chunk stages stay small beside the staging rows
  {
    cuuint64_t d[2] = {(cuuint64_t)G, (cuuint64_t)E * H}, s[1] = {(cuuint64_t)G * 2};
    cuuint32_t b[2] = {kBK, (cuuint32_t)NCW};
    if ((rc = make_map(&mD, pk + PL.down_t, 2, d, s, b))) return rc;
  }

  if (mode != kPrefillExperts && mode != kPrefillExpertsF16s) {
  const int rstages = EP <= 64 ? 8 : EP <= 128 ? 6 : 4;  // stages in flight, within the shared-memory budget
  RouterArgs ra{N, E, EP, H, rstages, bias, logits, status, 1, nullptr};
  const size_t r_smem = 1024 + rstages * (kTileM * 128 + (size_t)EP * 128) + 256;
  PPMOE_CHECK_CUDA(cudaFuncSetAttribute(router_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)r_smem));
  if (N <= kRouterSplitMaxN && H / kBK >= kRouterSplit) {  // few tiles: split K, then sum in order
    ra.ksplit = kRouterSplit;
    ra.part = reinterpret_cast<float*>(ws + W.rpart);
    router_gemm_kernel<<<dim3((N + kTileM - 1) / kTileM, kRouterSplit), 192, r_smem, st>>>(mX, mR, ra);
    PPMOE_CHECK_CUDA(cudaGetLastError());
    router_sum_kernel<<<(N * E + 255) / 256, 256, 0, st>>>(ra.part, kRouterSplit, N, E, bias, logits);
  } else {
    router_gemm_kernel<<<(N + kTileM - 1) / kTileM, 192, r_smem, st>>>(mX, mR, ra);
  }
  PPMOE_CHECK_CUDA(cudaGetLastError());
  if ((rc = route_logits_launch(logits, N, E, tau, nullptr, weights, nullptr, st))) return rc;
  }
  if (mode == kPrefillRouteOnly) return PPMOE_OK;

  // ---- dispatch
  int* blockcnt = reinterpret_cast<int*>(ws + W.blockcnt);
  int* blockoff = reinterpret_cast<int*>(ws + W.blockoff);
  int* count = reinterpret_cast<int*>(ws + W.count);
  int* exp_off = reinterpret_cast<int*>(ws + W.exp_off);
  int* ntiles = reinterpret_cast<int*>(ws + W.ntiles);
  int* tile_expert = reinterpret_cast<int*>(ws + W.tile_expert);
  int* tile_row0 = reinterpret_cast<int*>(ws + W.tile_row0);
  int* pair_token = reinterpret_cast<int*>(ws + W.pair_token);
  float* pair_w = reinterpret_cast<float*>(ws + W.pair_w);
  const size_t sc_smem = (size_t)256 * (E + 2) * 2;
  PPMOE_CHECK_CUDA(cudaFuncSetAttribute(count_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sc_smem));
  PPMOE_CHECK_CUDA(cudaFuncSetAttribute(scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(sc_smem + 256 * 8 * 4)));
  if (W.nblocks == 1) {  // one token block: count, scan and scatter in one launch
    PPMOE_CHECK_CUDA(cudaFuncSetAttribute(dispatch_one_block_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)(sc_smem + 256 * 8 * 4)));
    dispatch_one_block_kernel<<<1, 1024, sc_smem + 256 * 8 * 4, st>>>(
        weights, wpitch, N, E, blockcnt, blockoff, count, exp_off, ntiles, tile_expert, tile_row0,
        reinterpret_cast<int*>(ws + W.unit_tile), pair_token, pair_w, reinterpret_cast<long long*>(counts),
        reinterpret_cast<int*>(ws + W.tok_pairs), reinterpret_cast<int*>(ws + W.tok_k));
  } else {
    count_kernel<<<W.nblocks, 256, sc_smem, st>>>(weights, wpitch, N, E, blockcnt);
    scan_kernel<<<1, 1024, 0, st>>>(blockcnt, W.nblocks, E, blockoff, count, exp_off, ntiles, tile_expert, tile_row0,
                                   reinterpret_cast<int*>(ws + W.unit_tile), pair_token, pair_w, reinterpret_cast<long long*>(counts));
    scatter_kernel<<<W.nblocks, 512, sc_smem + 256 * 8 * 4, st>>>(weights, wpitch, N, E, blockoff, exp_off, pair_token, pair_w,
                                                         reinterpret_cast<int*>(ws + W.tok_pairs), reinterpret_cast<int*>(ws + W.tok_k));
  }
  PPMOE_CHECK_CUDA(cudaGetLastError());

  // ---- experts
  // persistent grids: every SM, less the SMs left free for concurrent communication kernels
  // (expert-parallel callers set PPMOE_PREFILL_FREE_SMS so NCCL transfers overlap the GEMMs)
  static const int free_sms = [] { const char* v = getenv("PPMOE_PREFILL_FREE_SMS"); return v ? atoi(v) : 0; }();
  const int grid = (int)std::min<long long>(std::max(1, nsm - free_sms), W.max_tiles);
  GUArgs ga{static_cast<const __nv_bfloat16*>(x), H, G, xpitch, tile_expert, tile_row0, ntiles, pair_token, pair_w,
            reinterpret_cast<__nv_bfloat16*>(ws + W.a2), status, 0};
  // stages of (2 A tiles + B) that fit in 227 KB of shared memory: 5 up to G = 32, 4 at
  // G = 96, 3 at G = 128
  const size_t pair_stage = 2 * kTileM * 128 + (size_t)2 * (G / gu_split) * 128;
  GUPairArgs pa{ga, reinterpret_cast<const int*>(ws + W.unit_tile), gu_split};
  pa.g.stages = (int)std::min<size_t>(kGUMaxStages, (232448 - 1024 - 256) / pair_stage);
  const size_t p_smem = 1024 + (size_t)pa.g.stages * pair_stage + 256;
  PPMOE_CHECK_CUDA(cudaFuncSetAttribute(gu_gemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p_smem));
  gu_gemm_pair_kernel<<<grid, kGUThreads, p_smem, st>>>(mGU, pa);
  PPMOE_CHECK_CUDA(cudaGetLastError());
  CUtensorMap mYh;
  uint8_t* y_v = ws + W.ypart;
  int8_t* y_sc = reinterpret_cast<int8_t*>(y_v + (size_t)W.max_pairs * H * 2);
  {
    cuuint64_t d[2] = {(cuuint64_t)H, (cuuint64_t)W.max_pairs}, sh[1] = {(cuuint64_t)H * 2};
    cuuint32_t b[2] = {64, kTileM};
    if ((rc = make_map_2d(&mYh, y_v, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, CU_TENSOR_MAP_SWIZZLE_128B, d, sh, b))) return rc;
  }
  const int NCH = H / NCW;
  const int ngrp = !small ? 1 : NCH % 3 == 0 ? 3 : NCH % 2 == 0 ? 2 : 1;
  DownArgs da{H, G, NCW, ngrp, y_sc, tile_expert, tile_row0, ntiles, pair_token, status};
  const int KB2 = (G + kBK - 1) / kBK;
  const int NCW_ = NCW;
  const size_t d_smem = 1024 + (size_t)2 * KB2 * kTileM * 128 + (size_t)kDownStages * KB2 * NCW_ * 128 + 256 +
                        (kDownEpiWarps / 4) * 2 * 16384 + 1024;
  PPMOE_CHECK_CUDA(cudaFuncSetAttribute(down_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)d_smem));
  down_gemm_kernel<<<grid, kDownThreads, d_smem, st>>>(mA2, mD, mYh, da);
  PPMOE_CHECK_CUDA(cudaGetLastError());
  int* tok_pairs = reinterpret_cast<int*>(ws + W.tok_pairs);
  int* tok_k = reinterpret_cast<int*>(ws + W.tok_k);
  const uint4* yh = reinterpret_cast<const uint4*>(y_v);
  const int H8 = H / 8, cthreads = std::min(256, (H8 + 31) / 32 * 32);
  if (mode == kPrefillExperts)
    pair_combine_kernel<1><<<N, cthreads, 0, st>>>(yh, y_sc, tok_pairs, tok_k, E, H8, out);
  else if (mode == kPrefillExpertsF16s)
    pair_combine_kernel<2><<<N, cthreads, 0, st>>>(yh, y_sc, tok_pairs, tok_k, E, H8, out, (int)f16s_pitch(H));
  else
    pair_combine_kernel<0><<<N, cthreads, 0, st>>>(yh, y_sc, tok_pairs, tok_k, E, H8, out);
  PPMOE_CHECK_CUDA(cudaGetLastError());
  return PPMOE_OK;
}

// Router from token rows to the compact active-expert list: the tcgen05 router GEMM of the
// prefill path (bf16 logits, optional prior) into the workspace, then route_compact_kernel.
// Workspace: status word + N x E bf16 logits.
size_t route_workspace_bytes(long long N, int E) { return 1024 + align_up((size_t)N * E * 2, 1024); }

int route_launch(const void* x, int N, const void* packed, int H, int E, int G, float tau, const float* bias,
                 int32_t* ids, void* w_out, int32_t* n_out, uint8_t* mask, void* wsp, size_t ws_bytes,
                 cudaStream_t st) {
  if (ws_bytes < route_workspace_bytes(N, E)) {
    set_error("ppmoe_route: workspace %zu < %zu bytes needed for %d tokens", ws_bytes, route_workspace_bytes(N, E), N);
    return PPMOE_ERR_WORKSPACE;
  }
  uint8_t* ws = static_cast<uint8_t*>(wsp);
  const PackedLayout PL = packed_layout(H, E, G);
  const uint8_t* pk = static_cast<const uint8_t*>(packed);
  uint32_t* status = reinterpret_cast<uint32_t*>(ws);
  __nv_bfloat16* logits = reinterpret_cast<__nv_bfloat16*>(ws + 1024);
  const int EP = (E + 15) / 16 * 16;
  CUtensorMap mX, mR;
  int rc;
  {
    cuuint64_t d[2] = {(cuuint64_t)H, (cuuint64_t)N}, s[1] = {(cuuint64_t)H * 2};
    cuuint32_t b[2] = {kBK, kTileM};
    if ((rc = make_map(&mX, x, 2, d, s, b))) return rc;
  }
  {
    cuuint64_t d[2] = {(cuuint64_t)H, (cuuint64_t)E}, s[1] = {(cuuint64_t)H * 2};
    cuuint32_t b[2] = {kBK, (cuuint32_t)EP};
    if ((rc = make_map(&mR, pk + PL.router_eh, 2, d, s, b))) return rc;
  }
  const int rstages = EP <= 64 ? 8 : EP <= 128 ? 6 : 4;
  RouterArgs ra{N, E, EP, H, rstages, bias, logits, status, 1, nullptr};
  const size_t r_smem = 1024 + rstages * (kTileM * 128 + (size_t)EP * 128) + 256;
  PPMOE_CHECK_CUDA(cudaFuncSetAttribute(router_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)r_smem));
  router_gemm_kernel<<<(N + kTileM - 1) / kTileM, 192, r_smem, st>>>(mX, mR, ra);
  PPMOE_CHECK_CUDA(cudaGetLastError());
  return route_compact_launch(logits, N, E, tau, ids, w_out, n_out, mask, st);
}

}  // namespace ppmoe
