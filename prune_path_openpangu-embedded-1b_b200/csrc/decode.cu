// Fused decode: router GEMV + tau selection + expert SwiGLU + down projection, ONE launch.
//
// Replaces TauSparseMoE.forward_decode (src/tl_kernel_optimized_Ultimate_PanGU.py:494-530),
// i.e. moe_router_select_kernel_decode (tl:335-380) followed by
// moe_decode_swiglu_fused_kernel (tl:385-462), for 1..16 tokens.
//
// Grid: C clusters x 8 CTAs (C = the number of 8-CTA clusters the GPU co-schedules), 384
// threads per CTA, one CTA per SM.
//
//  1. Router.  Rank r of every cluster computes the logits of experts [r*E/8, (r+1)*E/8)
//     for all tokens on the tensor cores (their router_eh rows arrive by bulk copy); the
//     ranks' logits are exchanged over distributed shared memory.  Every cluster computes the
//     same logits with the same operation order, so every CTA holds bit-identical
//     selections without any grid-wide barrier.
//  2. Selection (select.cuh), redundantly in every CTA: gate weights, union of selected
//     experts, per-expert token bitmask.
//  3. Experts.  The union's neurons (|U| * G) are split evenly over all CTAs of the grid.
//     Each neuron is one contiguous 3*H*2-byte record (gate row | up row | down row) that
//     a bulk copy streams into a ring of shared-memory slots.  One token: gate/up GEMV on the
//     tensor cores per 4-neuron tile, SwiGLU, fp32 down rows by hidden column.  2..16 tokens
//     (H % 384 == 0): rounds of 8 neurons, gate/up and down both on the tensor cores.
//     Otherwise a CUDA-core path (one neuron per warp, tokens that selected its expert).
//     Rounding points everywhere: g,u -> bf16; s=bf16(silu(g)); a=bf16(s*u); a2=bf16(a*w).
//  4. Reduction.  The 8 CTA partials of a cluster are summed over distributed shared
//     memory (rank order) into one partial per cluster in global scratch; per 1/8-slice of
//     the hidden dimension an arrival counter elects the last cluster, whose CTA sums the
//     C cluster partials in cluster order and writes bf16 output, then re-arms the counter.
//     The result is deterministic (fixed summation order) and rounded to bf16 exactly once.
//
// No CTA ever waits for another cluster, so co-residency of the grid is not required.
// Every mbarrier wait is bounded (common.cuh) and records a status bit instead of hanging.
#include <cooperative_groups.h>
#include "common.cuh"
#include "select.cuh"

namespace cg = cooperative_groups;

namespace ppmoe {

constexpr int kDecThreads = 384;
constexpr int kDecWarps = kDecThreads / 32;
constexpr int kCluster = 8;
constexpr int kMaxClusters = 32;  // workspace sizing (148 SMs -> at most 18 clusters of 8)

struct DecodeArgs {
  const __nv_bfloat16* x;
  int N;
  const __nv_bfloat16* router_eh;  // [E][H]
  const __nv_bfloat16* experts;    // [E][G][3][H]
  int H, E, G;
  float tau_b;
  const float* bias;
  __nv_bfloat16* out;
  __nv_bfloat16* logits_out;
  __nv_bfloat16* weights_out;
  long long* counts;
  float* cpart;        // [clusters][N][H]
  uint32_t* counters;  // [8]
  uint32_t* status;
  int slots;           // ring depth
  int pdl;
  int x_host;  // x is pinned, device-mapped host memory: plain loads instead of a bulk copy
  unsigned long long* trace;  // optional per-CTA phase timestamps [grid][32] (diagnostics)
  float pf_thr;  // one token: L2-prefetch the records of experts with probability >= pf_thr (0: off;
                 // default 1 / E, PPMOE_DECODE_PF scales it)
};

__device__ __forceinline__ unsigned long long clk64() {  // diagnostics stamp: global ns timer
  unsigned long long c;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(c));
  return c;
}
#define PPMOE_TRACE(i) \
  do { if (a.trace && threadIdx.x == 0) a.trace[blockIdx.x * 32 + (i)] = clk64(); } while (0)

// Shared-memory carve-out (byte offsets from a 1 KiB aligned base).
struct DecSmem {
  uint32_t bars, x, part, lg, w, tokmask, ulist, misc, kbuf, a2, recv, ring, total;
};

// A neuron's gate, up and down rows are one contiguous record in its ring slot (one bulk copy);
// slots are 6H + 32 bytes apart, so the gate rows of 4 consecutive neurons start in 4
// different 16-byte bank groups and an 8-row tensor-core fragment load (4 neurons x gate/up)
// costs 2 shared-memory wavefronts instead of 8.
__host__ __device__ inline uint32_t dec_row_pitch(int H) { return 2u * (uint32_t)H; }
__host__ __device__ inline uint32_t dec_slot_bytes(int H) { return 6u * (uint32_t)H + 32u; }

__host__ __device__ inline DecSmem dec_smem(int NT, int H, int E, int slots) {
  DecSmem s;
  uint32_t o = 0;
  s.bars = o;    o += 8 * 64;                                   // <= 63 slot barriers + 1
  s.x = o;       o = (uint32_t)align_up(o + (size_t)NT * (H + 8) * 2, 128);
  s.part = o;    o = (uint32_t)align_up(o + (size_t)NT * E * 4, 128);
  s.lg = o;      o = (uint32_t)align_up(o + (size_t)NT * E * 4, 128);
  s.w = o;       o = (uint32_t)align_up(o + (size_t)NT * E * 4, 128);
  s.tokmask = o; o = (uint32_t)align_up(o + (size_t)E * 4, 128);
  s.ulist = o;   o = (uint32_t)align_up(o + (size_t)E * 4, 128);
  s.misc = o;    o = (uint32_t)align_up(o + 64, 128);
  s.kbuf = o;    o = (uint32_t)align_up(o + (size_t)kDecWarps * 64 * 4, 128);
  s.a2 = o;      o = (uint32_t)align_up(o + (size_t)max(64 * NT, kDecWarps * 8 + 32) * 4, 1024);  // >= max(warps, slots); direct-path partials
  s.recv = o;    o = (uint32_t)align_up(o + (NT == 1 ? (size_t)H * 4 : 0), 1024);  // one token: pushed partials
  s.ring = o;    o += (uint32_t)slots * dec_slot_bytes(H);
  s.total = o;
  return s;
}

template <int NT, int HCH, bool CTASEL>
__global__ void __launch_bounds__(kDecThreads, 1) decode_fused_kernel(const DecodeArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  cg::cluster_group cluster = cg::this_cluster();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rank = (int)cluster.block_rank();
  const int cid = blockIdx.x / kCluster;
  const int nclusters = gridDim.x / kCluster;
  const int H = a.H, E = a.E, G = a.G, N = a.N;
  const int HS = H / kCluster;  // output columns owned by this rank in the reduction
  const int XP = H + 8;          // token row pitch in shared memory (elements)
  const DecSmem L = dec_smem(NT, H, E, a.slots);

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* bar_in = bars + a.slots;  // x + router slice
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem + L.x);
  float* part = reinterpret_cast<float*>(smem + L.part);
  float* lg = reinterpret_cast<float*>(smem + L.lg);
  float* ws = reinterpret_cast<float*>(smem + L.w);
  uint32_t* tokmask = reinterpret_cast<uint32_t*>(smem + L.tokmask);
  int* ulist = reinterpret_cast<int*>(smem + L.ulist);
  int* misc = reinterpret_cast<int*>(smem + L.misc);  // [0]=|U| [1]=is_last
  float* a2s = reinterpret_cast<float*>(smem + L.a2);
  uint8_t* ring = smem + L.ring;
  const uint32_t rec_bytes = 3u * (uint32_t)H * 2u;  // one neuron record in the packed blob
  const uint32_t rowp = dec_row_pitch(H), slotb = dec_slot_bytes(H);

  PPMOE_TRACE(0);
  // ---- prologue: barriers; router slice prefetch (weights only: legal before the PDL wait)
  // one token: the router logits and the cluster reduction are pushed into the consumer's
  // shared memory; each pushing thread arrives (release, cluster scope) on the consumer's
  // barrier after its own store
  uint64_t* bar_lg = bars + a.slots + 1;   // the router logits of every rank (st.async bytes)
  uint64_t* bar_red = bars + a.slots + 2;  // one token: this rank's slice of every CTA partial
  if (tid == 0) {
    for (int s = 0; s <= a.slots; ++s) mbar_init(&bars[s], 1);
    // The router logits (and, for one token, the cluster reduction) land by st.async, which
    // completes bytes on these barriers: each is armed here with every byte it will receive,
    // before any peer can push (peers push only after the cluster barrier that follows).
    mbar_init(bar_lg, 1);
    if (NT == 1) mbar_init(bar_red, 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(bar_lg, (uint32_t)(N * E) * 4u);
    if (NT == 1) mbar_arrive_expect_tx(bar_red, (uint32_t)(kCluster * HS * 4));
  }
  __syncthreads();
  // every peer's barriers must be initialised before its first remote arrival: arrive here,
  // wait just before the first push (long after, so the wait is normally free)
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  // Router operands.  Rank r owns experts [r EPR, (r+1) EPR) (EPR = E / 8): their router_eh
  // rows (H contiguous bf16 each) land in padded ring slots (pitch 2H + 16 bytes) and the
  // token rows in xs at pitch XP = H + 8, so every 8-row fragment load below is
  // bank-conflict free.  Router rows are weights (legal before the PDL wait); x is not.
  const int EPR = E / kCluster;
  const uint32_t rrow = 2u * (uint32_t)H + 16u;
  const uint32_t h_bytes = 2u * (uint32_t)H;
  uint8_t* rsl = ring;  // router slots alias the ring
  if (warp == 0) {
    if (lane == 0) mbar_arrive_expect_tx(bar_in, (uint32_t)(EPR + (a.x_host ? 0 : N)) * h_bytes);
    __syncwarp();
    for (int e = lane; e < EPR; e += 32)
      bulk_g2s(rsl + (size_t)e * rrow, a.router_eh + (size_t)(rank * EPR + e) * H, h_bytes, bar_in,
               policy_evict_last());
  }
  PPMOE_TRACE(28);
  if (a.pdl) pdl_wait();
  PPMOE_TRACE(29);
  if (a.x_host) {
    // token rows straight from pinned host memory (no bulk copy from system memory): 16-byte
    // loads, ordered before their use by the barrier after the router-row wait below
    const int per = H / 8;
    #pragma unroll 1
    for (int i = tid; i < N * per; i += kDecThreads) {
      const int t = i / per, c = i - t * per;
      reinterpret_cast<uint4*>(xs + (size_t)t * XP)[c] = reinterpret_cast<const uint4*>(a.x + (size_t)t * H)[c];
    }
  } else if (warp == 0) {
    for (int t = lane; t < N; t += 32)
      bulk_g2s(xs + (size_t)t * XP, a.x + (size_t)t * H, h_bytes, bar_in, policy_evict_first());
  }
  // zero-fill padded token rows so that their (ignored) logits stay finite
  #pragma unroll 1
  for (int i = tid; i < (NT - N) * XP; i += kDecThreads) xs[(size_t)N * XP + i] = __float2bfloat16_rn(0.f);
  #pragma unroll 1
  for (int i = tid; i < E; i += kDecThreads) tokmask[i] = 0u;
  mbar_wait(bar_in, 0, a.status);
  if (a.x_host) __syncthreads();
  PPMOE_TRACE(1);

  // ---- 1. this rank's experts' logits on the tensor cores: D[16 tokens x 8 experts] per
  // expert tile, mma.sync m16n8k16 with the same permuted-k 8-byte fragments as the expert
  // GEMVs (A = token rows, B = router rows).  Warp w takes k-steps [w ks / 12, (w+1) ks / 12)
  // of every tile; the per-warp partials are summed in warp order, so every cluster computes
  // bit-identical logits for the rank's experts.
  if (NT == 1) {
    // One token: CUDA-core dot products.  Lane (e8 = lane % 8, k-quarter = lane / 8) of
    // warp w covers 8 elements of every 32-element chunk of warp w's k-range for expert
    // 8 j + e8; quarters meet by shuffle (fixed order), warps in warp order.
    const int e8 = lane & 7, kq = lane >> 3;
    const int nch = H >> 5;  // 32-element chunks; warp w takes [w nch / 12, (w+1) nch / 12)
    const int kb = 32 * ((nch * warp) / kDecWarps), ke = 32 * ((nch * (warp + 1)) / kDecWarps);
    float* rpart = reinterpret_cast<float*>(ring + align_up((size_t)EPR * rrow, 128));  // [12][EPR]
    #pragma unroll 1
    for (int j = 0; j < EPR; j += 8) {
      const int e = min(j + e8, EPR - 1);
      const __nv_bfloat16* rr = reinterpret_cast<const __nv_bfloat16*>(rsl + (size_t)e * rrow);
      float s0 = 0.f, s1 = 0.f;
      #pragma unroll 1
      for (int k = kb + kq * 8; k < ke; k += 32) {
        const uint4 rv = *reinterpret_cast<const uint4*>(rr + k);
        const uint4 xv = *reinterpret_cast<const uint4*>(xs + k);
        const __nv_bfloat162* rp = reinterpret_cast<const __nv_bfloat162*>(&rv);
        const __nv_bfloat162* xp = reinterpret_cast<const __nv_bfloat162*>(&xv);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 rf = __bfloat1622float2(rp[i]), xf = __bfloat1622float2(xp[i]);
          if (i & 1) s1 = fmaf(xf.y, rf.y, fmaf(xf.x, rf.x, s1));
          else s0 = fmaf(xf.y, rf.y, fmaf(xf.x, rf.x, s0));
        }
      }
      float v = s0 + s1;
      v += __shfl_xor_sync(0xffffffffu, v, 8);
      v += __shfl_xor_sync(0xffffffffu, v, 16);
      if (kq == 0 && j + e8 < EPR) rpart[warp * EPR + j + e8] = v;
    }
    __syncthreads();
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
    // thread (e, r) pushes this rank's logit of expert e into CTA r's `part` with st.async,
    // which completes its 4 bytes on CTA r's bar_lg (no separate arrival)
    for (int i = tid; i < EPR * kCluster; i += kDecThreads) {
      const int e = i / kCluster, r = i % kCluster;
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < kDecWarps; ++w) s += rpart[w * EPR + e];  // warp order
      asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];"
                   ::"r"(mapa_u32(part + rank * EPR + e, (uint32_t)r)), "r"(__float_as_uint(s)),
                   "r"(mapa_u32(bar_lg, (uint32_t)r))
                   : "memory");
    }
  } else {
    const int NTL = (EPR + 7) >> 3;  // expert tiles
    const int ks = H >> 4;
    const int k0 = (ks * warp) / kDecWarps, k1 = (ks * (warp + 1)) / kDecWarps;
    const int g8 = lane >> 2, q = lane & 3;
    float* rpart = reinterpret_cast<float*>(ring + align_up((size_t)EPR * rrow, 128));  // [12][NT][8 NTL]
    #pragma unroll 1
    for (int tl = 0; tl < NTL; ++tl) {
      const uint32_t brow = smem_u32(rsl + (size_t)min(8 * tl + g8, EPR - 1) * rrow) + 8 * q;
      const uint32_t xr0 = smem_u32(xs + (size_t)min(g8, NT - 1) * XP) + 8 * q;
      const uint32_t xr1 = smem_u32(xs + (size_t)min(g8 + 8, NT - 1) * XP) + 8 * q;
      float d[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      #pragma unroll 2
      for (int k = k0; k < k1; ++k) {
        uint2 bv, a0 = make_uint2(0u, 0u), a1 = make_uint2(0u, 0u);
        asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(bv.x), "=r"(bv.y) : "r"(brow + 32 * k));
        if (g8 < NT) asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(a0.x), "=r"(a0.y) : "r"(xr0 + 32 * k));
        if (g8 + 8 < NT) asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(a1.x), "=r"(a1.y) : "r"(xr1 + 32 * k));
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(d[k & 1][0]), "+f"(d[k & 1][1]), "+f"(d[k & 1][2]), "+f"(d[k & 1][3])
            : "r"(a0.x), "r"(a1.x), "r"(a0.y), "r"(a1.y), "r"(bv.x), "r"(bv.y));
      }
      const int e0 = 8 * tl + 2 * q;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int t = g8 + 8 * hh;
        if (t < NT)
          *reinterpret_cast<float2*>(rpart + ((size_t)warp * NT + t) * (8 * NTL) + e0) =
              make_float2(d[0][2 * hh] + d[1][2 * hh], d[0][2 * hh + 1] + d[1][2 * hh + 1]);
      }
    }
    __syncthreads();
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");  // peers' barriers exist
    // thread (t, e, r): this rank's logit of expert e for token t, summed in warp order, into
    // CTA r's lg[t][rank EPR + e] by st.async (completing 4 bytes on CTA r's bar_lg)
    #pragma unroll 1
    for (int i = tid; i < N * EPR * kCluster; i += kDecThreads) {
      const int r = i % kCluster, te = i / kCluster, t = te / EPR, e = te - t * EPR;
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < kDecWarps; ++w) s += rpart[((size_t)w * NT + t) * (8 * NTL) + e];  // warp order
      asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];"
                   ::"r"(mapa_u32(lg + t * E + rank * EPR + e, (uint32_t)r)), "r"(__float_as_uint(s)),
                   "r"(mapa_u32(bar_lg, (uint32_t)r))
                   : "memory");
    }
  }
  PPMOE_TRACE(2);
  if constexpr (NT == 1) {
    mbar_wait_cluster(bar_lg, 0u, a.status);  // all E logits pushed into `part`
    PPMOE_TRACE(3);
    for (int e = tid; e < E; e += kDecThreads) {
      float l = bf16r(part[e]);
      if (a.bias) l = bf16r(l + a.bias[e]);
      lg[e] = l;
    }
  } else {
    mbar_wait_cluster(bar_lg, 0u, a.status);  // every rank's logits pushed into lg
    PPMOE_TRACE(3);
    #pragma unroll 1
    for (int i = tid; i < N * E; i += kDecThreads) {
      float l = bf16r(lg[i]);
      if (a.bias) l = bf16r(l + a.bias[i % E]);
      lg[i] = l;
    }
  }
  __syncthreads();
  PPMOE_TRACE(4);

  // ---- 2. selection: a single token with E <= 64 is selected by the whole CTA, otherwise
  // one warp per token
  if constexpr (CTASEL) {  // one token, E <= 64 (chosen on the host)
    float w[kMaxExpertsPerLane];
    constexpr int kSelWarps = kDecWarps - 2;
    uint32_t bits = 0;
    if (warp >= kSelWarps) {
      // Speculative L2 prefetch while the other warps select: the records of every expert
      // whose probability reaches pf_thr (a superset of the selection), each CTA a contiguous
      // 1/grid share of the candidates' bytes in 16 KB pieces.  The copies issued after the
      // selection then read L2 instead of waiting on HBM.
      if (a.pf_thr > 0.f) {
        float l2[2];
        uint32_t mk = 0u;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          l2[r] = lane + 32 * r < E ? lg[lane + 32 * r] : -INFINITY;
          if (lane + 32 * r < E) mk = max(mk, float_order_key(l2[r]));
        }
        const float m = float_from_order_key(__reduce_max_sync(0xffffffffu, mk));
        float ex[2], sm = 0.f;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          ex[r] = lane + 32 * r < E ? expf(l2[r] - m) : 0.f;
          sm += ex[r];
        }
        sm = warp_sum(sm);
        const float lim = a.pf_thr * sm;
        const uint32_t c0 = __ballot_sync(0xffffffffu, ex[0] >= lim), c1 = __ballot_sync(0xffffffffu, ex[1] >= lim);
        const int nc = __popc(c0) + __popc(c1);
        const uint32_t rec = 6u * (uint32_t)H * (uint32_t)G;  // bytes of one expert's records
        const uint32_t piece = 16384u, ppe = (rec + piece - 1) / piece;
        const int total = nc * (int)ppe, P = gridDim.x;
        const int b0 = (int)((long long)total * blockIdx.x / P), b1 = (int)((long long)total * (blockIdx.x + 1) / P);
        for (int k = b0 + (warp - kSelWarps) * 32 + lane; k < b1; k += 64) {
          int ci = k / (int)ppe;
          const uint32_t off = (uint32_t)(k % (int)ppe) * piece;
          // ci-th set bit of (c1:c0), ascending expert order
          int e;
          if (ci < __popc(c0)) e = __fns(c0, 0, ci + 1);
          else e = 32 + __fns(c1, 0, ci - __popc(c0) + 1);
          const uint32_t sz = min(piece, rec - off);
          const char* src = reinterpret_cast<const char*>(a.experts) + (size_t)e * rec + off;
          asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(sz) : "memory");
        }
      }
    } else {
      bits = select_one_token_cta<kSelWarps>(lg, E, a.tau_b, w, reinterpret_cast<uint32_t*>(smem + L.kbuf));
    }
    if (warp == 0) {
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int e = lane + 32 * i;
        if (e < E) {
          ws[e] = w[i];
          tokmask[e] = (bits >> i) & 1u;
        }
      }
    }
  } else {
#pragma unroll 1
    for (int t = warp; t < N; t += kDecWarps) {
      float l[kMaxExpertsPerLane], w[kMaxExpertsPerLane];
#pragma unroll
      for (int i = 0; i < kMaxExpertsPerLane; ++i) {
        const int e = lane + 32 * i;
        l[i] = e < E ? lg[t * E + e] : -INFINITY;
      }
      if (t == 0) PPMOE_TRACE(12);
      uint32_t* kb = reinterpret_cast<uint32_t*>(smem + L.kbuf) + warp * 64;
      const uint32_t bits = E <= 64 ? select_experts_warp<2>(l, E, a.tau_b, w, kb) : select_experts_warp(l, E, a.tau_b, w, kb);
      if (t == 0) PPMOE_TRACE(13);
#pragma unroll
      for (int i = 0; i < kMaxExpertsPerLane; ++i) {
        const int e = lane + 32 * i;
        if (e < E) {
          ws[t * E + e] = w[i];
          if ((bits >> i) & 1u) atomicOr(&tokmask[e], 1u << t);
        }
      }
    }
  }
  __syncthreads();
  PPMOE_TRACE(5);

  // ---- 3. experts.  The union's neurons (|U| * G) are split evenly over the grid; CTA
  // neuron n lives in ring slot n % slots.  Warp 0 builds the union list (ascending expert
  // order, ballot compaction) and issues the first window: one bulk copy per run of neurons
  // that share an expert (contiguous in the packed blob and in the ring), completing on the
  // run head's barrier; the other slots of the run get a plain arrival so that every slot
  // barrier has finished exactly one phase before refills start.
  const uint64_t pol = policy_evict_first();
  int i0 = 0, cnt = 0;
  auto work_range = [&](int nU) {
    const int W = nU * G;
    if ((long long)W * gridDim.x < (1ll << 31)) {  // 32-bit division when the product fits
      i0 = (int)((uint32_t)W * blockIdx.x / gridDim.x);
      cnt = (int)((uint32_t)W * (blockIdx.x + 1) / gridDim.x) - i0;
    } else {
      i0 = (int)((long long)W * blockIdx.x / gridDim.x);
      cnt = (int)((long long)W * (blockIdx.x + 1) / gridDim.x) - i0;
    }
  };
  auto issue_neuron = [&](int n) {  // neuron n's three rows into slot n % slots
    const int gi = i0 + n;
    const int u = gi / G, j = gi - u * G;
    const int sl = n % a.slots;
    const __nv_bfloat16* src = a.experts + ((size_t)ulist[u] * G + j) * 3 * H;
    mbar_arrive_expect_tx(&bars[sl], rec_bytes);
    bulk_g2s(ring + (size_t)sl * slotb, src, rec_bytes, &bars[sl], pol);
  };
  if (warp == 0) {
    int base = 0;
    #pragma unroll 1
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int e = e0 + lane;
      const bool on = e < E && tokmask[e] != 0u;
      const uint32_t b = __ballot_sync(0xffffffffu, on);
      if (on) ulist[base + __popc(b & ((1u << lane) - 1u))] = e;
      base += __popc(b);
    }
    if (lane == 0) misc[0] = base;
    __syncwarp();
    PPMOE_TRACE(16);
  }
  // optional side outputs from the first CTA of the grid
  if (blockIdx.x == 0) {
    #pragma unroll 1
    for (int i = tid; i < N * E; i += kDecThreads) {
      if (a.logits_out) a.logits_out[i] = __float2bfloat16_rn(lg[i]);
      if (a.weights_out) a.weights_out[i] = __float2bfloat16_rn(ws[i]);
    }
    if (a.counts) {
      #pragma unroll 1
      for (int e = tid; e < E; e += kDecThreads) {
        long long c = 0;
        #pragma unroll 1
        for (int t = 0; t < N; ++t) c += ws[t * E + e] > 0.f;
        a.counts[e] += c;
      }
    }
  }
  __syncthreads();
  PPMOE_TRACE(17);
  work_range(misc[0]);
  // Single-token fast path: the whole CTA range fits the ring (at most 24 neurons).
  bool fast = false, tcb = false;
  if constexpr (NT == 1) fast = cnt <= min(a.slots, 24) && (H & 63) == 0;
  if constexpr (NT >= 2 && HCH == 1) tcb = (H % 384) == 0 && a.slots >= 16;
  // batched path: round r = neurons [8r, 8r + 8) into slots 8 (r & 1) .. +8, on bars[r & 1]
  auto issue_round = [&](int r) {
    const int nr = min(8, cnt - 8 * r);
    if (lane == 0) mbar_arrive_expect_tx(&bars[r & 1], (uint32_t)nr * rec_bytes);
    __syncwarp();
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (lane < nr) {
      const int gi = i0 + 8 * r + lane, u = gi / G;
      bulk_g2s(ring + (size_t)(8 * (r & 1) + lane) * slotb,
               a.experts + ((size_t)ulist[u] * G + (gi - u * G)) * 3 * H, rec_bytes, &bars[r & 1], pol);
    }
  };
  // the router slice / scratch in the ring is dead: every warp passed the barrier above
  if (fast) {
    // One bulk copy per neuron into its padded slot (pitch 6H + 32 staggers the banks of
    // the 8-row fragment loads); tile t (neurons 4t .. 4t+3) completes on bars[t].  Lane 0 of
    // warp w arms tile w and issues neurons w, w + 12, ...: copies issued by one thread are
    // serialised (~70 cycles each), so the issue is spread over the warps.  A copy may land
    // before its tile is armed: the phase cannot complete until the arming arrival.
    if (lane == 0 && cnt > 0) {
      if (warp < (cnt + 3) / 4) mbar_arrive_expect_tx(&bars[warp], (uint32_t)min(4, cnt - 4 * warp) * rec_bytes);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      for (int n = warp; n < cnt; n += kDecWarps) {
        const int gi = i0 + n, u = gi / G;
        bulk_g2s(ring + (size_t)n * slotb, a.experts + ((size_t)ulist[u] * G + (gi - u * G)) * 3 * H,
                 rec_bytes, &bars[n >> 2], pol);
      }
    }
  } else if (tcb) {
    if (warp == 0) {
      if (cnt > 0) issue_round(0);
      if (cnt > 8) issue_round(1);
    }
  } else if (warp == 0) {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    const int win = min(cnt, a.slots);
    for (int n = lane; n < win; n += 32) issue_neuron(n);
  }
  PPMOE_TRACE(6);

  float acc[HCH][NT][4];
#pragma unroll
  for (int c = 0; c < HCH; ++c)
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[c][t][q] = 0.f;

  if (fast) {
    // Single-token tensor-core path.  Gate/up: D[16 x 8] = A[16 x 16] * B[16 x 8] per k-step
    // with mma.sync m16n8k16: A row 0 is the token (other rows zero); B's 8 columns are the
    // gate/up rows of one tile of 4 neurons (column 2i: gate of neuron 4 t + i, 2i+1: its up
    // row).  Inside each 16-wide k-step the k order is permuted identically for A and B
    // (fragment positions 2q, 2q+1, 2q+8, 2q+9 <- elements 4q .. 4q+3), so each lane's B
    // fragment is one 8-byte shared load; the dot product is unchanged.  Warp w takes tile
    // w % T and k-part w / T of KS = 12 / T parts and waits only for its tile's copies; the
    // KS part sums meet in shared memory in part order.  Down: thread tid applies every
    // neuron's down row to hidden columns 4 tid .. 4 tid + 3 (fp32 FMA, loads ahead of FMAs).
    const int T = (cnt + 3) >> 2;  // row tiles, <= 6
    const int KS = kDecWarps / T;  // k-parts per tile
    const int ksteps = H >> 4;
    const int tile = warp % T, part = warp / T;
    const int g8 = lane >> 2, q = lane & 3;
    float* kpart = reinterpret_cast<float*>(smem + L.a2);  // [KS][T][8]
    if (part < KS) {
      const int k0 = (ksteps * part) / KS, k1 = (ksteps * (part + 1)) / KS;
      const int nr = min(4 * tile + (g8 >> 1), cnt - 1);  // padding columns read a valid row
      const uint32_t brow = smem_u32(ring + (size_t)nr * slotb + (g8 & 1) * rowp) + 8 * q;
      const uint32_t xrow = smem_u32(xs) + 8 * q;
      float d[4][4];
#pragma unroll
      for (int i = 0; i < 4; ++i) d[i][0] = d[i][1] = d[i][2] = d[i][3] = 0.f;
      mbar_wait(&bars[tile], 0u, a.status);
      PPMOE_TRACE(18);
      #pragma unroll 1
      for (int kk = k0; kk < k1; kk += 4) {
        uint2 xa[4], bv[4];
#pragma unroll
        for (int s2 = 0; s2 < 4; ++s2) {
          const int k = min(kk + s2, k1 - 1);
          asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(bv[s2].x), "=r"(bv[s2].y) : "r"(brow + 32 * k));
          asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(xa[s2].x), "=r"(xa[s2].y) : "r"(xrow + 32 * k));
          // only A row 0 (lanes 0-3) carries the token; steps past k1 contribute nothing
          if (lane >= 4 || kk + s2 >= k1) xa[s2] = make_uint2(0u, 0u);
        }
#pragma unroll
        for (int s2 = 0; s2 < 4; ++s2)
          asm volatile(
              "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
              "{%0,%1,%2,%3};"
              : "+f"(d[s2][0]), "+f"(d[s2][1]), "+f"(d[s2][2]), "+f"(d[s2][3])
              : "r"(xa[s2].x), "r"(0u), "r"(xa[s2].y), "r"(0u), "r"(bv[s2].x), "r"(bv[s2].y));
      }
      if (lane < 4) {
        kpart[(part * T + tile) * 8 + 2 * q] = (d[0][0] + d[1][0]) + (d[2][0] + d[3][0]);      // gate
        kpart[(part * T + tile) * 8 + 2 * q + 1] = (d[0][1] + d[1][1]) + (d[2][1] + d[3][1]);  // up
      }
    }
    PPMOE_TRACE(19);
    __syncthreads();
    float* a2k = kpart + kDecWarps * 8;
    PPMOE_TRACE(20);
    if (tid < cnt) {
      float gp[kDecWarps], up[kDecWarps];
#pragma unroll
      for (int p = 0; p < kDecWarps; ++p) {
        const int o = (min(p, KS - 1) * T + (tid >> 2)) * 8 + 2 * (tid & 3);
        gp[p] = kpart[o];
        up[p] = kpart[o + 1];
      }
      float g = 0.f, uu = 0.f;
#pragma unroll
      for (int p = 0; p < kDecWarps; ++p)  // part order
        if (p < KS) { g += gp[p]; uu += up[p]; }
      const float gb = bf16r(g), ub = bf16r(uu);
      const float sb = bf16r(__fmul_rn(gb, __frcp_rn(1.f + expf(-gb))));  // silu
      a2k[tid] = bf16r(bf16r(sb * ub) * ws[ulist[(i0 + tid) / G]]);
    }
    __syncthreads();
    PPMOE_TRACE(21);
#pragma unroll
    for (int c = 0; c < HCH; ++c) {
      const int h4 = tid + c * kDecThreads;
      if (h4 < H / 4) {
        #pragma unroll 1
        for (int m0 = 0; m0 < cnt; m0 += 8) {
          uint2 dv[8];
          float av[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int m = min(m0 + i, cnt - 1);
            dv[i] = *reinterpret_cast<const uint2*>(ring + (size_t)m * slotb + 2 * rowp + 8 * h4);
            av[i] = m0 + i < cnt ? a2k[m0 + i] : 0.f;  // 0 * finite weight adds exactly nothing
          }
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float2 d01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&dv[i].x));
            const float2 d23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&dv[i].y));
            acc[c][0][0] = fmaf(av[i], d01.x, acc[c][0][0]);
            acc[c][0][1] = fmaf(av[i], d01.y, acc[c][0][1]);
            acc[c][0][2] = fmaf(av[i], d23.x, acc[c][0][2]);
            acc[c][0][3] = fmaf(av[i], d23.y, acc[c][0][3]);
          }
        }
      }
    }
  } else if (tcb) {
    // Batched tensor-core path (2..16 tokens).  Rounds of 8 neurons (two tiles of 4),
    // double-buffered over ring slots 0-15; round r's copies complete on bars[r & 1].
    // Gate/up: mma.sync m16n8k16 with the tokens as A rows and, per tile, the gate/up rows
    // of 4 neurons as B columns (same permuted-k 8-byte fragments as the single-token path);
    // warp w owns k-steps [w KW, (w+1) KW) of every tile and keeps its x fragments in
    // registers for the whole launch, so the x region is reused for the per-warp partials
    // [12][2][NT][8] (summed in warp order).  Down: mma.sync m16n8k8, A = a2 [16 tokens x 8
    // neurons] (bf16, zero for tokens that did not select the neuron's expert), B = the
    // round's down rows read transposed by ldmatrix; warp w owns hidden columns
    // [H/12 w, H/12 (w + 1)) and accumulates them over all rounds in registers.
    constexpr int kMaxKW = 8;  // k-steps per warp (H <= 1536)
    const int KW = (H >> 4) / kDecWarps;
    const int g8 = lane >> 2, q = lane & 3;
    uint2 xa[kMaxKW][2];  // A fragments: token rows g8 and g8 + 8
#pragma unroll
    for (int s2 = 0; s2 < kMaxKW; ++s2) {
      const int k = warp * KW + min(s2, KW - 1);
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int t = g8 + 8 * hh;
        xa[s2][hh] = (t < NT && s2 < KW) ? *reinterpret_cast<const uint2*>(xs + (size_t)t * XP + 16 * k + 4 * q)
                                          : make_uint2(0u, 0u);
      }
    }
    __nv_bfloat16* a2t = reinterpret_cast<__nv_bfloat16*>(smem + L.a2);  // [16 tokens][8 neurons]
    if (tid < 64) reinterpret_cast<uint32_t*>(a2t)[tid] = 0u;
    __syncthreads();  // every warp holds its x fragments: the x region becomes the partials
    PPMOE_TRACE(22);
    float* kp = reinterpret_cast<float*>(xs);
    float dacc[16][4];
#pragma unroll
    for (int j = 0; j < 16; ++j) dacc[j][0] = dacc[j][1] = dacc[j][2] = dacc[j][3] = 0.f;
    const int colw = H / kDecWarps;  // hidden columns per warp (multiple of 32)
    const int rounds = (cnt + 7) >> 3;
    #pragma unroll 1
    for (int r = 0; r < rounds; ++r) {
      const int nr = min(8, cnt - 8 * r);
      const uint8_t* sb = ring + (size_t)(8 * (r & 1)) * slotb;
      mbar_wait(&bars[r & 1], (uint32_t)((r >> 1) & 1), a.status);
      if (r == 0) PPMOE_TRACE(23);
      if (r == 1) PPMOE_TRACE(27);
      // ---- gate/up
      float d[2][4];
#pragma unroll
      for (int t = 0; t < 2; ++t) d[t][0] = d[t][1] = d[t][2] = d[t][3] = 0.f;
      uint32_t brow[2];
#pragma unroll
      for (int t = 0; t < 2; ++t)
        brow[t] = smem_u32(sb + (size_t)min(4 * t + (g8 >> 1), nr - 1) * slotb + (g8 & 1) * rowp) + 8 * q +
                  32 * warp * KW;
#pragma unroll
      for (int s2 = 0; s2 < kMaxKW; ++s2) {
        if (s2 < KW) {
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            uint2 bv;
            asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(bv.x), "=r"(bv.y) : "r"(brow[t] + 32 * s2));
            asm volatile(
                "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                "{%0,%1,%2,%3};"
                : "+f"(d[t][0]), "+f"(d[t][1]), "+f"(d[t][2]), "+f"(d[t][3])
                : "r"(xa[s2][0].x), "r"(xa[s2][1].x), "r"(xa[s2][0].y), "r"(xa[s2][1].y), "r"(bv.x), "r"(bv.y));
          }
        }
      }
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        if (g8 < NT)
          *reinterpret_cast<float2*>(kp + ((warp * 2 + t) * NT + g8) * 8 + 2 * q) = make_float2(d[t][0], d[t][1]);
        if (g8 + 8 < NT)
          *reinterpret_cast<float2*>(kp + ((warp * 2 + t) * NT + g8 + 8) * 8 + 2 * q) = make_float2(d[t][2], d[t][3]);
      }
      __syncthreads();
      if (r == 0) PPMOE_TRACE(24);
      // ---- SwiGLU + gate weight per (token, neuron); warp order over the k partials
      if (tid < NT * 8) {
        const int t = tid >> 3, n = tid & 7, tl = n >> 2, i = n & 3;
        float g = 0.f, uu = 0.f;
#pragma unroll
        for (int w = 0; w < kDecWarps; ++w) {
          const float2 v = *reinterpret_cast<const float2*>(kp + ((w * 2 + tl) * NT + t) * 8 + 2 * i);
          g += v.x;
          uu += v.y;
        }
        float av = 0.f;
        if (t < N && n < nr) {
          const float gb = bf16r(g), ub = bf16r(uu);
          const float sbv = bf16r(__fmul_rn(gb, __frcp_rn(1.f + expf(-gb))));  // silu
          av = bf16r(sbv * ub) * ws[t * E + ulist[(i0 + 8 * r + n) / G]];     // 0 if not selected
        }
        a2t[t * 8 + n] = __float2bfloat16_rn(av);
      }
      __syncthreads();
      if (r == 0) PPMOE_TRACE(25);
      // ---- down: out[16 x 128 w..] += a2[16 x 8] * Wd[8 x ...]
      uint32_t af0, af1;
      asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
                   : "=r"(af0), "=r"(af1) : "r"(smem_u32(a2t) + (lane & 15) * 16));
      const uint32_t drow = smem_u32(sb + (size_t)min(lane & 7, nr - 1) * slotb + 2 * rowp) +
                            (uint32_t)(colw * warp + 8 * (lane >> 3)) * 2;
#pragma unroll
      for (int j4 = 0; j4 < 4; ++j4) {
        if (32 * j4 >= colw) break;
        uint32_t b0, b1, b2, b3;
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                     : "=r"(b0), "=r"(b1), "=r"(b2), "=r"(b3) : "r"(drow + j4 * 64));
        const uint32_t bb[4] = {b0, b1, b2, b3};
#pragma unroll
        for (int jj = 0; jj < 4; ++jj)
          asm volatile(
              "mma.sync.aligned.m16n8k8.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
              : "+f"(dacc[4 * j4 + jj][0]), "+f"(dacc[4 * j4 + jj][1]), "+f"(dacc[4 * j4 + jj][2]),
                "+f"(dacc[4 * j4 + jj][3])
              : "r"(af0), "r"(af1), "r"(bb[jj]));
      }
      __syncthreads();  // the round's slots and a2 are consumed
      if (r == 0) PPMOE_TRACE(26);
      if (warp == 0 && r + 2 < rounds) issue_round(r + 2);
    }
    // CTA partial straight from the fragments: column tile j of warp w covers hidden
    // columns H/12 w + 8 j + 2q, +1 for tokens g8 (c0, c1) and g8 + 8 (c2, c3)
    float* redt = reinterpret_cast<float*>(ring);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (8 * j >= colw) break;
      const int h = colw * warp + 8 * j + 2 * q;
      if (g8 < N) *reinterpret_cast<float2*>(redt + (size_t)g8 * H + h) = make_float2(dacc[j][0], dacc[j][1]);
      if (g8 + 8 < N)
        *reinterpret_cast<float2*>(redt + (size_t)(g8 + 8) * H + h) = make_float2(dacc[j][2], dacc[j][3]);
    }
  } else {
    // Wait for the whole first window before the batched loop reuses slots.
    const int win = min(cnt, a.slots);
#pragma unroll 1
    for (int n = 0; n < win; ++n) mbar_wait(&bars[n], 0u, a.status);
  }
  PPMOE_TRACE(7);

  for (int b0 = 0; b0 < ((fast || tcb) ? 0 : cnt); b0 += kDecWarps) {
    const int n = b0 + warp;
#pragma unroll
    for (int t = 0; t < NT; ++t)
      if (lane == t) a2s[warp * NT + t] = 0.f;
    __syncwarp();
    if (n < cnt) {
      const int s = n % a.slots;
      if (n >= a.slots) mbar_wait(&bars[s], (uint32_t)((n / a.slots) & 1), a.status);
      const int e = ulist[(i0 + n) / G];
      uint32_t tm = tokmask[e];
      const __nv_bfloat16* gate = reinterpret_cast<const __nv_bfloat16*>(ring + (size_t)s * slotb);
      const __nv_bfloat16* up = reinterpret_cast<const __nv_bfloat16*>(ring + (size_t)s * slotb + rowp);
      #pragma unroll 1
      while (tm) {
        const int t = __ffs(tm) - 1;
        tm &= tm - 1u;
        // four independent accumulators per row keep the FMA chains short
        float sg[4] = {0.f, 0.f, 0.f, 0.f}, su[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 2
        for (int v = lane; v < H / 8; v += 32) {
          const uint4 xv = *reinterpret_cast<const uint4*>(xs + t * XP + v * 8);
          const uint4 gv = *reinterpret_cast<const uint4*>(gate + v * 8);
          const uint4 uv = *reinterpret_cast<const uint4*>(up + v * 8);
          const __nv_bfloat162* xp = reinterpret_cast<const __nv_bfloat162*>(&xv);
          const __nv_bfloat162* gp = reinterpret_cast<const __nv_bfloat162*>(&gv);
          const __nv_bfloat162* up2 = reinterpret_cast<const __nv_bfloat162*>(&uv);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 xf = __bfloat1622float2(xp[q]);
            const float2 gf = __bfloat1622float2(gp[q]);
            const float2 uf = __bfloat1622float2(up2[q]);
            sg[q] = fmaf(xf.y, gf.y, fmaf(xf.x, gf.x, sg[q]));
            su[q] = fmaf(xf.y, uf.y, fmaf(xf.x, uf.x, su[q]));
          }
        }
        float g2 = (sg[0] + sg[1]) + (sg[2] + sg[3]);
        float u2 = (su[0] + su[1]) + (su[2] + su[3]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          g2 += __shfl_xor_sync(0xffffffffu, g2, o);
          u2 += __shfl_xor_sync(0xffffffffu, u2, o);
        }
        if (lane == 0) {
          const float gb = bf16r(g2), ub = bf16r(u2);
          const float sb = bf16r(__fmul_rn(gb, __frcp_rn(1.f + expf(-gb))));  // silu
          const float ab = bf16r(sb * ub);
          a2s[warp * NT + t] = bf16r(ab * ws[t * E + e]);
        }
      }
    }
    __syncthreads();
    const int nb = min(kDecWarps, cnt - b0);
    // down rows of this batch, four per step: loads first, then the dependent FMAs
    for (int m0 = 0; m0 < nb; m0 += 4) {
#pragma unroll
      for (int c = 0; c < HCH; ++c) {
        const int h4 = tid + c * kDecThreads;
        if (h4 < H / 4) {
          uint2 dv[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int m = min(m0 + q, nb - 1);
            const __nv_bfloat16* down =
                reinterpret_cast<const __nv_bfloat16*>(ring + (size_t)((b0 + m) % a.slots) * slotb + 2 * rowp);
            dv[q] = *reinterpret_cast<const uint2*>(down + h4 * 4);
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            if (m0 + q < nb) {
              const float2 d01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&dv[q].x));
              const float2 d23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&dv[q].y));
#pragma unroll
              for (int t = 0; t < NT; ++t) {
                const float av = a2s[(m0 + q) * NT + t];
                acc[c][t][0] = fmaf(av, d01.x, acc[c][t][0]);
                acc[c][t][1] = fmaf(av, d01.y, acc[c][t][1]);
                acc[c][t][2] = fmaf(av, d23.x, acc[c][t][2]);
                acc[c][t][3] = fmaf(av, d23.y, acc[c][t][3]);
              }
            }
          }
        }
      }
    }
    __syncthreads();
    if (warp == 0) {  // refill the slots this batch released
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      const int lo = b0 + a.slots, hi = min(cnt, b0 + nb + a.slots);
      #pragma unroll 1
      for (int n2 = lo + lane; n2 < hi; n2 += 32) issue_neuron(n2);
    }
  }
  PPMOE_TRACE(8);
  if (a.pdl) pdl_launch_dependents();

  if constexpr (NT == 1) {
    // ---- 4a'/4b'. one token: every float4 of the CTA partial is pushed to the rank that
    // owns its column slice (recv[source rank][HS]); the owner sums the 8 sources in rank
    // order once all have arrived.  No cluster barrier, no shared memory read by a peer.
    float* recv = reinterpret_cast<float*>(smem + L.recv);
#pragma unroll
    for (int c = 0; c < HCH; ++c) {
      const int h4 = tid + c * kDecThreads;
      if (h4 < H / 4) {
        const int col = 4 * h4, owner = col / HS;
        asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];"
                     ::"r"(mapa_u32(recv + rank * HS + (col - owner * HS), (uint32_t)owner)),
                     "r"(__float_as_uint(acc[c][0][0])), "r"(__float_as_uint(acc[c][0][1])),
                     "r"(__float_as_uint(acc[c][0][2])), "r"(__float_as_uint(acc[c][0][3])),
                     "r"(mapa_u32(bar_red, (uint32_t)owner))
                     : "memory");
      }
    }
    mbar_wait_cluster(bar_red, 0u, a.status);
    PPMOE_TRACE(9);
    #pragma unroll 1
    for (int i = tid; i < HS / 4; i += kDecThreads) {
      float4 s4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int q = 0; q < kCluster; ++q) {  // rank order
        const float4 v = *reinterpret_cast<const float4*>(recv + q * HS + 4 * i);
        s4.x += v.x; s4.y += v.y; s4.z += v.z; s4.w += v.w;
      }
      *reinterpret_cast<float4*>(a.cpart + (size_t)cid * H + rank * HS + 4 * i) = s4;
    }
  } else {
  // ---- 4a. CTA partial -> shared (ring is idle: every issued record has been consumed)
  float* red = reinterpret_cast<float*>(ring);
#pragma unroll
  for (int c = 0; c < HCH; ++c) {
    const int h4 = tid + c * kDecThreads;
    if (!tcb && h4 < H / 4) {  // the batched tensor-core path wrote its partial already
#pragma unroll
      for (int t = 0; t < NT; ++t)
        if (t < N)
          *reinterpret_cast<float4*>(red + (size_t)t * H + h4 * 4) =
              make_float4(acc[c][t][0], acc[c][t][1], acc[c][t][2], acc[c][t][3]);
    }
  }
  cluster.sync();
  PPMOE_TRACE(9);
  // ---- 4b. cluster partial of this rank's column slice, rank order
  #pragma unroll 1
  for (int i = tid; i < N * (HS / 4); i += kDecThreads) {
    const int t = i / (HS / 4), h = rank * HS + (i % (HS / 4)) * 4;
    float4 v[kCluster];
#pragma unroll
    for (int q = 0; q < kCluster; ++q)
      v[q] = *reinterpret_cast<const float4*>(cluster.map_shared_rank(red, q) + (size_t)t * H + h);
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int q = 0; q < kCluster; ++q) { s.x += v[q].x; s.y += v[q].y; s.z += v[q].z; s.w += v[q].w; }
    *reinterpret_cast<float4*>(a.cpart + ((size_t)cid * N + t) * H + h) = s;
  }
  // peers may still read this CTA's shared memory: arrive now, wait before exiting
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  }
  // ---- 4c. the last cluster to finish this column slice sums all cluster partials
  // The barrier orders every thread's partial store before thread 0's release; the
  // acquire side of the same atomic orders the last cluster's reads after all of them.
  __syncthreads();
  if (tid == 0) {
    uint32_t old;
    asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], 1;" : "=r"(old) : "l"(a.counters + rank) : "memory");
    misc[1] = (old == (uint32_t)nclusters - 1u);
  }
  __syncthreads();
  PPMOE_TRACE(10);
  const int nel = N * (HS / 4);  // float4 elements of this rank's column slice
  if (misc[1] && nel * nclusters <= 2 * kDecThreads) {
    // every cluster partial of the slice in one round of loads, then sums in cluster order
    float4* gat = reinterpret_cast<float4*>(ring + align_up((size_t)N * H * 4, 128));
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int j = tid + r * kDecThreads;
      if (j < nel * nclusters) {
        const int c = j / nel, i = j - c * nel;
        const int t = i / (HS / 4), h = rank * HS + (i % (HS / 4)) * 4;
        gat[j] = __ldcg(reinterpret_cast<const float4*>(a.cpart + ((size_t)c * N + t) * H + h));
      }
    }
    __syncthreads();
    if (tid < nel) {
      const int t = tid / (HS / 4), h = rank * HS + (tid % (HS / 4)) * 4;
      float4 s4 = make_float4(0.f, 0.f, 0.f, 0.f);
      #pragma unroll 1
      for (int c = 0; c < nclusters; ++c) {
        const float4 v = gat[c * nel + tid];
        s4.x += v.x; s4.y += v.y; s4.z += v.z; s4.w += v.w;
      }
      __nv_bfloat162 lo = __floats2bfloat162_rn(s4.x, s4.y), hi = __floats2bfloat162_rn(s4.z, s4.w);
      uint2 pk;
      pk.x = *reinterpret_cast<uint32_t*>(&lo);
      pk.y = *reinterpret_cast<uint32_t*>(&hi);
      *reinterpret_cast<uint2*>(a.out + (size_t)t * H + h) = pk;
    }
    if (tid == 0) a.counters[rank] = 0u;  // re-arm for the next launch
  } else if (misc[1]) {
    #pragma unroll 1
    for (int i = tid; i < N * (HS / 4); i += kDecThreads) {
      const int t = i / (HS / 4), h = rank * HS + (i % (HS / 4)) * 4;
      // eight independent L2 reads in flight per round; additions stay in cluster order
      float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
      #pragma unroll 1
      for (int c0 = 0; c0 < nclusters; c0 += 8) {
        float4 v[8];
#pragma unroll
        for (int c = 0; c < 8; ++c)
          if (c0 + c < nclusters)
            v[c] = __ldcg(reinterpret_cast<const float4*>(a.cpart + ((size_t)(c0 + c) * N + t) * H + h));
#pragma unroll
        for (int c = 0; c < 8; ++c)
          if (c0 + c < nclusters) { s.x += v[c].x; s.y += v[c].y; s.z += v[c].z; s.w += v[c].w; }
      }
      __nv_bfloat162 lo = __floats2bfloat162_rn(s.x, s.y), hi = __floats2bfloat162_rn(s.z, s.w);
      uint2 pk;
      pk.x = *reinterpret_cast<uint32_t*>(&lo);
      pk.y = *reinterpret_cast<uint32_t*>(&hi);
      *reinterpret_cast<uint2*>(a.out + (size_t)t * H + h) = pk;
    }
    if (tid == 0) a.counters[rank] = 0u;  // re-arm for the next launch
  }
  if constexpr (NT != 1) asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
  PPMOE_TRACE(11);
  if (a.trace && tid == 0) a.trace[blockIdx.x * 32 + 30] = (unsigned long long)cnt;
}

// ------------------------------------------------------------------ host side
using KernelFn = void (*)(const DecodeArgs);

static KernelFn pick_kernel(int NT, int HCH, bool ctasel) {
  // the one-token, E <= 64 variants carry only the CTA-wide selection (smaller code)
  if (ctasel) {
    if (HCH == 1) return decode_fused_kernel<1, 1, true>;
    if (HCH == 2) return decode_fused_kernel<1, 2, true>;
    if (HCH == 3) return decode_fused_kernel<1, 3, true>;
    return nullptr;
  }
#define PPMOE_K(nt, hch) if (NT == nt && HCH == hch) return decode_fused_kernel<nt, hch, false>;
  PPMOE_K(1, 1) PPMOE_K(1, 2) PPMOE_K(1, 3)
  PPMOE_K(2, 1) PPMOE_K(2, 2) PPMOE_K(2, 3)
  PPMOE_K(4, 1) PPMOE_K(4, 2) PPMOE_K(4, 3)
  PPMOE_K(8, 1) PPMOE_K(8, 2)
  PPMOE_K(16, 1)
#undef PPMOE_K
  return nullptr;
}

struct DecodeCfgCache {
  int dev = -1, NT = 0, H = 0, E = 0, slots = 0, pdl = -1;
  uint32_t smem = 0;
  int clusters = 0;
};
static thread_local DecodeCfgCache g_dec_cache;
static unsigned long long* g_trace = nullptr;
void decode_set_trace(void* buf) { g_trace = static_cast<unsigned long long*>(buf); }

int decode_launch(const void* x, int tokens, const void* packed, int H, int E, int G, float tau,
                  const float* bias, void* out, void* logits_out, void* weights_out, int64_t* counts,
                  void* wsp, size_t ws_bytes, int pdl, cudaStream_t stream, uint32_t* status,
                  uint32_t* counters, float* cpart, size_t cpart_bytes, int x_host) {
  if (E % kCluster != 0 || H % 32 != 0) {
    set_error("ppmoe_decode: experts (%d) must be a multiple of 8 and hidden (%d) of 32", E, H);
    return PPMOE_ERR_UNSUPPORTED;
  }
  int NT = 1;
  while (NT < tokens) NT <<= 1;
  const int HCH = (H / 4 + kDecThreads - 1) / kDecThreads;
  KernelFn fn = pick_kernel(NT, HCH, NT == 1 && E <= 64);
  if (!fn) {
    set_error("ppmoe_decode: tokens=%d with hidden=%d is outside the decode kernel's range", tokens, H);
    return PPMOE_ERR_UNSUPPORTED;
  }
  int dev = 0;
  PPMOE_CHECK_CUDA(cudaGetDevice(&dev));
  DecodeCfgCache& C = g_dec_cache;
  if (C.dev != dev || C.NT != NT || C.H != H || C.E != E || C.pdl != pdl) {
    int max_optin = 0;
    PPMOE_CHECK_CUDA(cudaDeviceGetAttribute(&max_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    int slots = 24;
    DecSmem L = dec_smem(NT, H, E, slots);
    while (slots > 2 && L.total + 1024 > (uint32_t)max_optin) L = dec_smem(NT, H, E, --slots);
    // the router slice and its group scratch alias the ring
    // router slots (E/8 padded rows) and the per-warp router partials alias the ring
    const size_t need_ring = align_up((size_t)(E / kCluster) * (2 * H + 16), 128) +
                             (size_t)kDecWarps * NT * 8 * ((E / kCluster + 7) / 8) * 4;
    const size_t red_ring = (size_t)NT * H * 4;
    if ((size_t)slots * dec_slot_bytes(H) < need_ring || (size_t)slots * dec_slot_bytes(H) < red_ring ||
        L.total + 1024 > (uint32_t)max_optin || slots < 2) {
      set_error("ppmoe_decode: shared memory budget exceeded (H=%d E=%d tokens=%d)", H, E, tokens);
      return PPMOE_ERR_UNSUPPORTED;
    }
    const uint32_t smem = L.total + 1024;
    PPMOE_CHECK_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kCluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    int nsm = 0;
    PPMOE_CHECK_CUDA(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev));
    cfg.gridDim = dim3((nsm / kCluster) * kCluster);
    cfg.blockDim = dim3(kDecThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    PPMOE_CHECK_CUDA(cudaOccupancyMaxActiveClusters(&clusters, fn, &cfg));
    if (clusters <= 0) {
      set_error("ppmoe_decode: no 8-CTA cluster fits (smem=%u)", smem);
      return PPMOE_ERR_UNSUPPORTED;
    }
    C.dev = dev; C.NT = NT; C.H = H; C.E = E; C.slots = slots; C.pdl = pdl;
    C.smem = smem; C.clusters = min(clusters, kMaxClusters);
  }
  if ((size_t)C.clusters * tokens * H * 4 > cpart_bytes) {
    set_error("ppmoe_decode: workspace sized for fewer tokens than %d", tokens);
    return PPMOE_ERR_WORKSPACE;
  }
  const PackedLayout PL = packed_layout(H, E, G);
  DecodeArgs a;
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.N = tokens;
  a.router_eh = reinterpret_cast<const __nv_bfloat16*>(static_cast<const uint8_t*>(packed) + PL.router_eh);
  a.experts = reinterpret_cast<const __nv_bfloat16*>(static_cast<const uint8_t*>(packed) + PL.experts);
  a.H = H; a.E = E; a.G = G;
  a.tau_b = __bfloat162float(__float2bfloat16_rn(tau));
  a.bias = bias;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.logits_out = static_cast<__nv_bfloat16*>(logits_out);
  a.weights_out = static_cast<__nv_bfloat16*>(weights_out);
  a.counts = reinterpret_cast<long long*>(counts);
  a.cpart = cpart;
  a.counters = counters;
  a.status = status;
  a.slots = C.slots;
  a.pdl = pdl;
  a.x_host = x_host;
  a.trace = g_trace;
  {
    static const float pf = [] { const char* v = getenv("PPMOE_DECODE_PF"); return v ? (float)atof(v) : 1.f; }();
    a.pf_thr = (tokens == 1 && E <= 64) ? pf / (float)E : 0.f;
  }

  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kCluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(C.clusters * kCluster);
  cfg.blockDim = dim3(kDecThreads);
  cfg.dynamicSmemBytes = C.smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  PPMOE_CHECK_CUDA(cudaLaunchKernelEx(&cfg, fn, a));
  return PPMOE_OK;
}

}  // namespace ppmoe
