// Fused decode of ONE token (the reference's decode case, tl:612-615): router GEMV + tau
// selection + expert SwiGLU + down projection in one launch, laid out so that consecutive
// layers overlap.
//
// Replaces TauSparseMoE.forward_decode (src/tl_kernel_optimized_Ultimate_PanGU.py:494-530):
// moe_router_select_kernel_decode (tl:335-380) + moe_decode_swiglu_fused_kernel (tl:385-462).
//
// Grid: one CTA per SM, as clusters of two CTAs; at most ~113 KB of shared memory and 80
// registers per thread, so that two CTAs fit on an SM.  The kernel signals its dependents
// (programmatic dependent launch) at its start: the next layer's CTAs become resident beside
// this layer's, load their router rows (weights) and park in griddepcontrol.wait, so the next
// layer starts from its activations the moment this one completes.
//
//  1. Router.  Rank r of a pair holds the router rows of experts [r E/2, (r+1) E/2) (bulk
//     copies issued before the dependency wait) and computes their logits on the tensor cores
//     (mma.sync m16n8k16, the token as A row 0, 8 experts' router rows as the B columns, warps
//     split K, partial sums added in warp order); each logit goes to the peer with st.async
//     (completing on the peer's mbarrier).  Every pair computes bit-identical logits.
//  2. Selection (select.cuh, CTA-wide rank count), redundantly per CTA.
//  3. Experts.  The union's |U| G neurons are split evenly over the grid; each neuron's record
//     (gate row | up row | down row, contiguous in the packed blob) is one bulk copy into a
//     shared-memory slot.  Gate/up on the tensor cores (the token as A row 0, 4 neurons'
//     gate/up rows as the 8 B columns; the k order inside each 16-wide step is permuted
//     identically for A and B so that every fragment is one 8-byte load), SwiGLU and the gate
//     weight per neuron, down rows by hidden column in fp32.  More neurons than slots: rounds.
//  4. Reduction.  Every CTA stores its fp32 partial [H] as 64-bit words (value | launch epoch
//     << 32); CTA c polls the words of its 1/grid slice of the hidden columns in every
//     partial until all carry this launch's epoch (no flag, fence or atomic on the critical
//     path), sums them in a fixed order and writes bf16.  CTA 0 advances the epoch word after
//     its own sums, i.e. after every CTA has read the epoch.  Deterministic; one bf16
//     rounding.  The polls need every CTA of the grid resident: the grid is one CTA per SM
//     (two fit), and with programmatic dependent launch a grid is only launched after every
//     CTA of its predecessor is running.
//
// Rounding points: logit = bf16(x.R) (+ bias, bf16); g,u -> bf16; s = bf16(silu(g));
// a = bf16(s u); a2 = bf16(a w); out = bf16(sum a2 Wd).  Every wait is bounded and records
// a status bit instead of hanging.
#include <cooperative_groups.h>
#include "common.cuh"
#include "select.cuh"

namespace cg = cooperative_groups;

namespace ppmoe {

constexpr int kD1Threads = 384;
constexpr int kD1Warps = kD1Threads / 32;
constexpr int kD1MaxHCH = 3;        // float4 column units per thread: H <= 4 * 384 * 3
constexpr int kD1TileBars = 12;     // tile barriers (slots <= 48)
constexpr int kD1MaxGrid = 160;     // partial rows in the workspace region

struct D1Args {
  const __nv_bfloat16* x;
  const __nv_bfloat16* router_eh;  // [E][H]
  const __nv_bfloat16* experts;    // [E][G][3][H]
  int H, E, G;
  float tau_b;
  const float* bias;
  __nv_bfloat16* out;
  __nv_bfloat16* logits_out;
  __nv_bfloat16* weights_out;
  long long* counts;
  unsigned long long* part;  // [H / 4][grid][4] tagged fp32 CTA partials (unit-major)
  uint32_t* epoch;           // launch epoch (advanced by CTA 0 at its end)
  uint32_t* status;
  int slots;
  int pdl;
  int trig_early;     // signal dependents at the start (1) or after the selection (0)
  unsigned long long* trace;  // optional [grid][32] globaltimer stamps (diagnostics)
};

__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
#define D1_TRACE(i) \
  do { if (a.trace && threadIdx.x == 0) a.trace[blockIdx.x * 32 + (i)] = gtimer(); } while (0)

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_v2u64(unsigned long long* p, unsigned long long a, unsigned long long b) {
  asm volatile("st.relaxed.gpu.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ void ld_relaxed_v2u64(const unsigned long long* p, unsigned long long& a,
                                                 unsigned long long& b) {
  asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
// 4-byte store into a peer CTA's shared memory that completes 4 transaction bytes on the
// peer's mbarrier (both addresses shared::cluster)
__device__ __forceinline__ void st_async_f32(uint32_t addr, float v, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];"
               ::"r"(addr), "r"(__float_as_uint(v)), "r"(bar) : "memory");
}

struct D1Smem {
  uint32_t bars, x, lg, w, ulist, misc, scr, ring, total;
};

__host__ __device__ inline uint32_t d1_slot_bytes(int H) { return 6u * (uint32_t)H + 32u; }
__host__ __device__ inline uint32_t d1_router_pitch(int H) { return 2u * (uint32_t)H + 32u; }

__host__ __device__ inline D1Smem d1_smem(int H, int E, int slots) {
  D1Smem s;
  uint32_t o = 0;
  s.bars = o;  o += 8 * 16;
  s.x = o;     o = (uint32_t)align_up(o + 2 * (size_t)H + 16, 128);
  s.lg = o;    o = (uint32_t)align_up(o + (size_t)E * 4, 128);
  s.w = o;     o = (uint32_t)align_up(o + (size_t)E * 4, 128);
  s.ulist = o; o = (uint32_t)align_up(o + (size_t)E * 4, 128);
  s.misc = o;  o = (uint32_t)align_up(o + 64, 128);
  s.scr = o;   o = (uint32_t)align_up(o + 3072 + 512, 1024);  // selection scratch | router / gate-up parts, a2
  s.ring = o;  o += (uint32_t)slots * d1_slot_bytes(H);
  s.total = o;
  return s;
}

__global__ void __launch_bounds__(kD1Threads, 2) decode1_kernel(const D1Args a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  cg::cluster_group cluster = cg::this_cluster();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rank = (int)cluster.block_rank();
  const int H = a.H, E = a.E, G = a.G, EH = a.E >> 1;
  const D1Smem L = d1_smem(H, E, a.slots);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* bar_in = bars + kD1TileBars;      // this rank's router rows
  uint64_t* bar_lg = bars + kD1TileBars + 1;  // the peer's E/2 logits (st.async bytes)
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem + L.x);
  float* lg = reinterpret_cast<float*>(smem + L.lg);
  float* ws = reinterpret_cast<float*>(smem + L.w);
  int* ulist = reinterpret_cast<int*>(smem + L.ulist);
  int* misc = reinterpret_cast<int*>(smem + L.misc);  // [0] |U|, [1] epoch
  float* scr = reinterpret_cast<float*>(smem + L.scr);
  uint8_t* ring = smem + L.ring;
  const uint32_t hb = 2u * (uint32_t)H, rpitch = d1_router_pitch(H), slotb = d1_slot_bytes(H);
  const uint32_t rec = 3u * hb;
  const int g8 = lane >> 2, q = lane & 3;

  D1_TRACE(0);
  if (tid == 0) {
    for (int s = 0; s < kD1TileBars; ++s) mbar_init(&bars[s], 1);
    mbar_init(bar_in, 1);
    mbar_init(bar_lg, 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(bar_lg, (uint32_t)EH * 4u);  // armed before the peer can push
  }
  __syncthreads();
  // the peer's barriers must exist before the first remote store: arrive now, wait later
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  if (warp == 0) {  // router rows are weights: legal before the dependency wait
    if (lane == 0) mbar_arrive_expect_tx(bar_in, (uint32_t)EH * hb);
    __syncwarp();
    const uint64_t pol = policy_evict_last();
    for (int e = lane; e < EH; e += 32)
      bulk_g2s(ring + (size_t)e * rpitch, a.router_eh + (size_t)(rank * EH + e) * H, hb, bar_in, pol);
  }
  if (a.trig_early) pdl_launch_dependents();
  if (a.pdl) pdl_wait();
  D1_TRACE(1);
  // token row: plain 16-byte loads (written by the previous kernel, normally still in L2)
  for (int i = tid; i < H / 8; i += kD1Threads)
    reinterpret_cast<uint4*>(xs)[i] = reinterpret_cast<const uint4*>(a.x)[i];
  if (tid == 0) misc[1] = (int)(ld_acquire_gpu(a.epoch) + 1u);
  mbar_wait(bar_in, 0u, a.status);
  __syncthreads();
  D1_TRACE(2);

  // ---- 1. router on the tensor cores: D[16 x 8] += A[16 x 16] B[16 x 8] per k-step and
  // expert tile; A row 0 = the token (lanes 0-3), B column n = router row of expert 8t + n.
  // Warp w takes k-steps [w KS / 12, (w+1) KS / 12) of every tile.
  {
    const int KS = H >> 4, NTL = (EH + 7) >> 3;
    const int k0 = (KS * warp) / kD1Warps, k1 = (KS * (warp + 1)) / kD1Warps;
    float* rpart = scr;  // [12][EH]
    const uint32_t xrow = smem_u32(xs) + 8 * q;
    #pragma unroll 1
    for (int t = 0; t < NTL; ++t) {
      const uint32_t brow = smem_u32(ring + (size_t)min(8 * t + g8, EH - 1) * rpitch) + 8 * q;
      float d[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      #pragma unroll 2
      for (int k = k0; k < k1; k += 2) {  // two independent accumulators
        uint2 bv[2], xa[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int kk = min(k + h, k1 - 1);
          asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(bv[h].x), "=r"(bv[h].y) : "r"(brow + 32 * kk));
          asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(xa[h].x), "=r"(xa[h].y) : "r"(xrow + 32 * kk));
          if (lane >= 4 || k + h >= k1) xa[h] = make_uint2(0u, 0u);
        }
#pragma unroll
        for (int h = 0; h < 2; ++h)
          asm volatile(
              "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
              "{%0,%1,%2,%3};"
              : "+f"(d[h][0]), "+f"(d[h][1]), "+f"(d[h][2]), "+f"(d[h][3])
              : "r"(xa[h].x), "r"(0u), "r"(xa[h].y), "r"(0u), "r"(bv[h].x), "r"(bv[h].y));
      }
      if (lane < 4) {
        const int e = 8 * t + 2 * q;
        if (e < EH) rpart[warp * EH + e] = d[0][0] + d[1][0];
        if (e + 1 < EH) rpart[warp * EH + e + 1] = d[0][1] + d[1][1];
      }
    }
    D1_TRACE(11);
    __syncthreads();
    D1_TRACE(12);
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
    D1_TRACE(13);
    if (tid < EH) {  // thread e: this rank's logit of expert rank EH + e, here and at the peer
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < kD1Warps; ++w) s += rpart[w * EH + tid];  // warp order
      float l = bf16r(s);
      if (a.bias) l = bf16r(l + a.bias[rank * EH + tid]);
      lg[rank * EH + tid] = l;
      st_async_f32(mapa_u32(lg + rank * EH + tid, (uint32_t)(rank ^ 1)), l, mapa_u32(bar_lg, (uint32_t)(rank ^ 1)));
    }
  }
  D1_TRACE(14);
  __syncthreads();                    // this rank's half of lg
  mbar_wait(bar_lg, 0u, a.status);    // the peer's half
  D1_TRACE(3);

  // ---- 2. selection (warp 0 holds the result), union list in ascending expert order
  {
    float wsel[kMaxExpertsPerLane];
    const uint32_t bits = select_one_token_cta<kD1Warps>(lg, E, a.tau_b, wsel, reinterpret_cast<uint32_t*>(scr));
    if (warp == 0) {
      int base = 0;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int e = lane + 32 * i;
        const bool on = e < E && ((bits >> i) & 1u);
        if (e < E) ws[e] = wsel[i];
        const uint32_t b = __ballot_sync(0xffffffffu, on);
        if (on) ulist[base + __popc(b & ((1u << lane) - 1u))] = e;
        base += __popc(b);
      }
      if (lane == 0) misc[0] = base;
    }
  }
  __syncthreads();
  D1_TRACE(4);
  if (!a.trig_early) pdl_launch_dependents();

  // ---- 3. experts: this CTA's neurons [i0, i0 + cnt) of the union's |U| G
  const int S = a.slots;
  const uint32_t Wn = (uint32_t)misc[0] * (uint32_t)G;  // <= 256 * 256
  const int i0 = (int)(Wn * blockIdx.x / gridDim.x);
  const int cnt = (int)(Wn * (blockIdx.x + 1) / gridDim.x) - i0;
  const int rounds = (cnt + S - 1) / S;
  const uint64_t pol = policy_evict_first();
  // round r: neurons [r S, r S + nr) into slots 0..nr-1; tile t (slots 4t..4t+3) completes on
  // bars[t].  Lane 0 of warp w arms tile w and issues neurons w, w + 12, ... (copies issued by
  // one thread are serialised, so the issue is spread over the warps).
  auto issue = [&](int r) {
    const int nb = r * S, nr = min(S, cnt - nb);
    if (lane == 0) {
      if (warp < (nr + 3) / 4) mbar_arrive_expect_tx(&bars[warp], (uint32_t)min(4, nr - 4 * warp) * rec);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      for (int n = warp; n < nr; n += kD1Warps) {
        const int gi = i0 + nb + n, u = gi / G;
        bulk_g2s(ring + (size_t)n * slotb, a.experts + ((size_t)ulist[u] * G + (gi - u * G)) * 3 * H, rec,
                 &bars[n >> 2], pol);
      }
    }
  };
  if (cnt > 0) issue(0);
  D1_TRACE(5);
  // optional side outputs from the first CTA (off the critical path of the others)
  if (blockIdx.x == 0) {
    for (int e = tid; e < E; e += kD1Threads) {
      if (a.logits_out) a.logits_out[e] = __float2bfloat16_rn(lg[e]);
      if (a.weights_out) a.weights_out[e] = __float2bfloat16_rn(ws[e]);
      if (a.counts && ws[e] > 0.f) a.counts[e] += 1;
    }
  }

  float acc[kD1MaxHCH][4];
#pragma unroll
  for (int c = 0; c < kD1MaxHCH; ++c) acc[c][0] = acc[c][1] = acc[c][2] = acc[c][3] = 0.f;
  const int ksteps = H >> 4;
  #pragma unroll 1
  for (int r = 0; r < rounds; ++r) {
    const int nb = r * S, nr = min(S, cnt - nb);
    if (r > 0) {
      __syncthreads();  // every slot of the previous round is consumed
      issue(r);
    }
    // gate/up: warp w takes tile w % T and k-part w / T of KS = 12 / T parts
    const int T = (nr + 3) >> 2;
    const int KS = kD1Warps / T;
    const int tile = warp % T, kpi = warp / T;
    float* kpart = scr;  // [KS][T][8]
    if (kpi < KS) {
      const int k0 = (ksteps * kpi) / KS, k1 = (ksteps * (kpi + 1)) / KS;
      const int nrow = min(4 * tile + (g8 >> 1), nr - 1);  // padding columns read a valid row
      const uint32_t brow = smem_u32(ring + (size_t)nrow * slotb + (g8 & 1) * hb) + 8 * q;
      const uint32_t xrow = smem_u32(xs) + 8 * q;
      float d[4][4];
#pragma unroll
      for (int i = 0; i < 4; ++i) d[i][0] = d[i][1] = d[i][2] = d[i][3] = 0.f;
      mbar_wait(&bars[tile], (uint32_t)(r & 1), a.status);
      if (r == 0 && warp == 0) D1_TRACE(6);
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
        kpart[(kpi * T + tile) * 8 + 2 * q] = (d[0][0] + d[1][0]) + (d[2][0] + d[3][0]);      // gate
        kpart[(kpi * T + tile) * 8 + 2 * q + 1] = (d[0][1] + d[1][1]) + (d[2][1] + d[3][1]);  // up
      }
    }
    __syncthreads();
    float* a2k = scr + kD1Warps * 8 * 2;
    if (tid < nr) {
      float g = 0.f, uu = 0.f;
      #pragma unroll 1
      for (int p = 0; p < KS; ++p) {  // part order
        const int o = (p * T + (tid >> 2)) * 8 + 2 * (tid & 3);
        g += kpart[o];
        uu += kpart[o + 1];
      }
      const float gb = bf16r(g), ub = bf16r(uu);
      const float sb = bf16r(__fmul_rn(gb, __frcp_rn(1.f + expf(-gb))));  // silu
      a2k[tid] = bf16r(bf16r(sb * ub) * ws[ulist[(i0 + nb + tid) / G]]);
    }
    __syncthreads();
    if (r == 0) D1_TRACE(7);
    // down rows: thread tid owns hidden columns 4 h4 .. 4 h4 + 3, h4 = tid + 384 c
#pragma unroll
    for (int c = 0; c < kD1MaxHCH; ++c) {
      const int h4 = tid + c * kD1Threads;
      if (h4 < H / 4) {
        #pragma unroll 1
        for (int m0 = 0; m0 < nr; m0 += 4) {
          uint2 dv[4];
          float av[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int m = min(m0 + i, nr - 1);
            dv[i] = *reinterpret_cast<const uint2*>(ring + (size_t)m * slotb + 2 * hb + 8 * h4);
            av[i] = m0 + i < nr ? a2k[m0 + i] : 0.f;  // 0 * finite weight adds exactly nothing
          }
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 d01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&dv[i].x));
            const float2 d23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&dv[i].y));
            acc[c][0] = fmaf(av[i], d01.x, acc[c][0]);
            acc[c][1] = fmaf(av[i], d01.y, acc[c][1]);
            acc[c][2] = fmaf(av[i], d23.x, acc[c][2]);
            acc[c][3] = fmaf(av[i], d23.y, acc[c][3]);
          }
        }
      }
    }
  }
  D1_TRACE(8);

  // ---- 4. grid reduction over epoch-tagged partials
  const unsigned long long ep = (unsigned long long)(uint32_t)misc[1] << 32;
  {
    // unit-major: a consumer's entries (its units x every partial) are contiguous
#pragma unroll
    for (int c = 0; c < kD1MaxHCH; ++c) {
      const int h4 = tid + c * kD1Threads;
      if (h4 < H / 4) {
        unsigned long long* dst = a.part + ((size_t)h4 * gridDim.x + blockIdx.x) * 4;
        st_relaxed_v2u64(dst, ep | __float_as_uint(acc[c][0]), ep | __float_as_uint(acc[c][1]));
        st_relaxed_v2u64(dst + 2, ep | __float_as_uint(acc[c][2]), ep | __float_as_uint(acc[c][3]));
      }
    }
  }
  D1_TRACE(9);
  {
    const int U = H >> 2, P = gridDim.x;
    const int u0 = (int)((uint32_t)U * blockIdx.x / (uint32_t)P);
    const int nu = (int)((uint32_t)U * (blockIdx.x + 1) / (uint32_t)P) - u0;
    float4* red = reinterpret_cast<float4*>(ring);  // [nu][P]; the ring is idle
    __syncthreads();  // every warp is done with the ring
    // entries (unit j, partial p); each thread polls its entries until all 4 words carry
    // this launch's epoch
    const uint32_t want = (uint32_t)(ep >> 32);
    for (int i = tid; i < nu * P; i += kD1Threads) {
      const unsigned long long* src = a.part + ((size_t)u0 * P + i) * 4;  // entry (u0 + i / P, i % P)
      unsigned long long w0, w1, w2, w3;
      uint32_t it = 0;
      #pragma unroll 1
      for (;;) {
        ld_relaxed_v2u64(src, w0, w1);
        ld_relaxed_v2u64(src + 2, w2, w3);
        if ((uint32_t)(w0 >> 32) == want && (uint32_t)(w1 >> 32) == want && (uint32_t)(w2 >> 32) == want &&
            (uint32_t)(w3 >> 32) == want)
          break;
        if (++it > kSpinLimit) {
          atomicOr(a.status, DEVERR_TIMEOUT);
          break;
        }
        __nanosleep(100);  // back off: early finishers must not crowd out the last CTAs' traffic
      }
      red[i] = make_float4(__uint_as_float((uint32_t)w0), __uint_as_float((uint32_t)w1),
                           __uint_as_float((uint32_t)w2), __uint_as_float((uint32_t)w3));
    }
    D1_TRACE(18);
    __syncthreads();
    D1_TRACE(19);
    for (int j = warp; j < nu; j += kD1Warps) {
      float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int p = lane; p < P; p += 32) {
        const float4 v = red[j * P + p];
        s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {  // fixed tree; lane 0's sum is reproducible
        s.x += __shfl_xor_sync(0xffffffffu, s.x, o);
        s.y += __shfl_xor_sync(0xffffffffu, s.y, o);
        s.z += __shfl_xor_sync(0xffffffffu, s.z, o);
        s.w += __shfl_xor_sync(0xffffffffu, s.w, o);
      }
      if (lane == 0) {
        __nv_bfloat162 lo = __floats2bfloat162_rn(s.x, s.y), hi = __floats2bfloat162_rn(s.z, s.w);
        uint2 pk;
        pk.x = *reinterpret_cast<uint32_t*>(&lo);
        pk.y = *reinterpret_cast<uint32_t*>(&hi);
        *reinterpret_cast<uint2*>(a.out + 4 * (size_t)(u0 + j)) = pk;
      }
    }
  }
  // CTA 0 has seen every CTA's partial of this launch, so every CTA has read the epoch
  if (blockIdx.x == 0 && tid == 0)
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(a.epoch), "r"((uint32_t)(ep >> 32)) : "memory");
  D1_TRACE(10);
  if (a.trace && tid == 0) a.trace[blockIdx.x * 32 + 30] = (unsigned long long)cnt;
}

// ------------------------------------------------------------------ host side
struct D1Cfg {
  int dev = -1, H = 0, E = 0;
  int ok = 0, slots = 0, grid = 0;
  uint32_t smem = 0;
};
static thread_local D1Cfg g_d1;
static int g_d1_mode = -1;  // PPMOE_DECODE1: 0 off, 1 signal dependents after selection, 2 early

static int d1_mode() {
  if (g_d1_mode < 0) {
    const char* v = getenv("PPMOE_DECODE1");
    g_d1_mode = v ? atoi(v) : 2;
  }
  return g_d1_mode;
}

// Bytes of the tagged-partial region the single-token kernel needs for hidden size H.
size_t decode1_region_bytes(int H) { return (size_t)kD1MaxGrid * H * 8; }

// Returns 1 if launched, 0 if the kernel does not apply (caller falls back), < 0 on error.
// part: the tagged-partial region (decode1_region_bytes); epoch: a word that only this kernel
// writes (zero-initialised with the workspace).
int decode1_launch(const void* x, const void* packed, int H, int E, int G, float tau, const float* bias, void* out,
                   void* logits_out, void* weights_out, int64_t* counts, int pdl, cudaStream_t stream,
                   uint32_t* status, uint32_t* epoch, void* part, size_t part_bytes, unsigned long long* trace) {
  const int mode = d1_mode();
  if (mode == 0 || E > 64 || (E & 1) || H % 64 != 0 || H > 4 * kD1Threads * kD1MaxHCH || !part) return 0;
  int dev = 0;
  PPMOE_CHECK_CUDA(cudaGetDevice(&dev));
  D1Cfg& C = g_d1;
  if (C.dev != dev || C.H != H || C.E != E) {
    C = D1Cfg();
    C.dev = dev; C.H = H; C.E = E;
    int nsm = 0, smem_sm = 0;
    PPMOE_CHECK_CUDA(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev));
    PPMOE_CHECK_CUDA(cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev));
    // two CTAs per SM: each gets half the SM's shared memory minus the per-CTA reservation
    const int budget = smem_sm / 2 - 1024 - 1024;  // -1024: alignment slack of the dynamic base
    int slots = 4 * kD1TileBars;  // tiles of 4 neurons <= warps
    while (slots > 1 && (int)d1_smem(H, E, slots).total > budget) --slots;
    const D1Smem Lm = d1_smem(H, E, slots);
    const size_t ring = (size_t)slots * d1_slot_bytes(H);
    const size_t router_need = (size_t)(E / 2) * d1_router_pitch(H);
    const int grid = (nsm / 2) * 2;
    const size_t red_need = (size_t)((H / 4 + grid - 1) / grid) * grid * 16;
    if (slots >= 4 && (int)Lm.total <= budget && router_need <= ring && red_need <= ring && grid <= kD1MaxGrid) {
      const uint32_t smem = Lm.total + 1024;
      PPMOE_CHECK_CUDA(cudaFuncSetAttribute(decode1_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      cudaLaunchConfig_t cfg = {};
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.gridDim = dim3(grid);
      cfg.blockDim = dim3(kD1Threads);
      cfg.dynamicSmemBytes = smem;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int clusters = 0;
      PPMOE_CHECK_CUDA(cudaOccupancyMaxActiveClusters(&clusters, decode1_kernel, &cfg));
      // the partial polls need the whole grid resident
      if (clusters * 2 >= grid) {
        C.ok = 1;
        C.slots = slots;
        C.grid = grid;
        C.smem = smem;
      }
    }
  }
  if (!C.ok || (size_t)C.grid * H * 8 > part_bytes) return 0;
  const PackedLayout PL = packed_layout(H, E, G);
  D1Args a;
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.router_eh = reinterpret_cast<const __nv_bfloat16*>(static_cast<const uint8_t*>(packed) + PL.router_eh);
  a.experts = reinterpret_cast<const __nv_bfloat16*>(static_cast<const uint8_t*>(packed) + PL.experts);
  a.H = H; a.E = E; a.G = G;
  a.tau_b = __bfloat162float(__float2bfloat16_rn(tau));
  a.bias = bias;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.logits_out = static_cast<__nv_bfloat16*>(logits_out);
  a.weights_out = static_cast<__nv_bfloat16*>(weights_out);
  a.counts = reinterpret_cast<long long*>(counts);
  a.part = static_cast<unsigned long long*>(part);
  a.epoch = epoch;
  a.status = status;
  a.slots = C.slots;
  a.pdl = pdl;
  a.trig_early = mode == 2;
  a.trace = trace;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(C.grid);
  cfg.blockDim = dim3(kD1Threads);
  cfg.dynamicSmemBytes = C.smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  PPMOE_CHECK_CUDA(cudaLaunchKernelEx(&cfg, decode1_kernel, a));
  return 1;
}

}  // namespace ppmoe
