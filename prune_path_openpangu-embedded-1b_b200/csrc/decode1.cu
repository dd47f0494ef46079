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
//     (mma.sync m16n8k16, the token as A row 0, 8 experts' router rows as the B columns, one
//     accumulator chain per expert tile and k parity, warps split K, partial sums added in
//     warp order); each logit goes to the peer with st.async (completing on the peer's
//     mbarrier).  Every pair computes bit-identical logits.
//  2. Selection (select.cuh, CTA-wide rank count), redundantly per CTA.
//  3. Gate/up by neuron.  The union's |U| G neurons are split evenly over the grid; each
//     neuron's gate and up rows (the first 4H bytes of its packed record) are one bulk copy
//     into a shared-memory slot; warp w computes the dot products of its neurons with the
//     token (fp32 FMA, lanes split K, butterfly sum), SwiGLU and the gate weight, and
//     publishes a2 = bf16(bf16(silu(g) u) w) as a 64-bit word (value | launch epoch << 32).
//  4. Down projection by hidden column.  CTA c owns columns [c H / grid, (c+1) H / grid); the
//     K-major down rows of those columns for every selected expert (down_t [E][H][G] of the
//     packed blob, one bulk copy per expert) stream into shared memory together with the
//     gate/up rows.  Every CTA polls the a2 words of all the union's neurons until they carry
//     this launch's epoch (no flag, fence or atomic on the critical path), then
//     out[h] = bf16(sum over experts, neurons of a2 * down_t[e][h][j]) in a fixed order, written
//     straight to the output: no cross-CTA reduction of outputs.  Experts beyond the shared
//     memory budget are processed in chunks (one a2 exchange each).
//  The epoch word is advanced by CTA 0 after it has seen every CTA's presence word of this
//  launch (each CTA writes one right after reading the epoch).  The polls need every CTA of
//  the grid resident: the grid is one CTA per SM (two fit), and with programmatic dependent
//  launch a grid is only launched after every CTA of its predecessor is running.
//
// Rounding points: logit = bf16(x.R) (+ bias, bf16); g,u -> bf16; s = bf16(silu(g));
// a = bf16(s u); a2 = bf16(a w); out = bf16(sum a2 Wd).  Deterministic (fixed summation
// orders).  Every wait is bounded and records a status bit instead of hanging.
#include <cooperative_groups.h>
#include "common.cuh"
#include "select.cuh"

namespace cg = cooperative_groups;

namespace ppmoe {

constexpr int kD1Threads = 384;
constexpr int kD1Warps = kD1Threads / 32;
constexpr int kD1MaxSlots = 24;     // gate/up slots (one mbarrier each)
constexpr int kD1MaxXI = 8;         // 16-byte token chunks per lane: H <= 2048
constexpr int kD1MaxGrid = 160;     // presence words in the workspace region

struct D1Args {
  const __nv_bfloat16* x;
  const __nv_bfloat16* router_eh;  // [E][H]
  const __nv_bfloat16* experts;    // [E][G][3][H]
  const __nv_bfloat16* down_t;     // [E][H][G]
  int H, E, G;
  float tau_b;
  const float* bias;
  __nv_bfloat16* out;
  __nv_bfloat16* logits_out;
  __nv_bfloat16* weights_out;
  long long* counts;
  unsigned long long* a2x;       // [E G] tagged a2 of the union's neurons (union order)
  unsigned long long* presence;  // [grid] tagged presence words
  uint32_t* epoch;               // launch epoch (advanced by CTA 0 at its end)
  uint32_t* status;
  int CE;     // experts per chunk
  int S;      // gate/up slots (>= neurons of one CTA in one chunk)
  int NC;     // >= hidden columns of one CTA
  int trig_early;             // signal dependents at the start (1) or after the selection (0)
  int pdl;
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
__device__ __forceinline__ void st_relaxed_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// 4-byte store into a peer CTA's shared memory that completes 4 transaction bytes on the
// peer's mbarrier (both addresses shared::cluster)
__device__ __forceinline__ void st_async_f32(uint32_t addr, float v, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];"
               ::"r"(addr), "r"(__float_as_uint(v)), "r"(bar) : "memory");
}
__device__ __forceinline__ float bf_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }

struct D1Smem {
  uint32_t bars, x, lg, w, ulist, misc, scr, alias, a2s, dred, dsl, ring, total;
};

__host__ __device__ inline uint32_t d1_slot_bytes(int H) { return 4u * (uint32_t)H + 32u; }
__host__ __device__ inline uint32_t d1_router_pitch(int H) { return 2u * (uint32_t)H + 32u; }

__host__ __device__ inline D1Smem d1_smem(int H, int E, int G, int CE, int S, int NC) {
  D1Smem s;
  uint32_t o = 0;
  s.bars = o;  o += 8 * 32;
  s.x = o;     o = (uint32_t)align_up(o + 2 * (size_t)H + 16, 128);
  s.lg = o;    o = (uint32_t)align_up(o + (size_t)E * 4, 128);
  s.w = o;     o = (uint32_t)align_up(o + (size_t)E * 4, 128);
  s.ulist = o; o = (uint32_t)align_up(o + (size_t)E * 4, 128);
  s.misc = o;  o = (uint32_t)align_up(o + 64, 128);
  s.scr = o;   o = (uint32_t)align_up(o + 3072 + 512, 1024);  // selection scratch | router warp parts
  // from here on the region also holds the router rows until the selection is done
  s.alias = o;
  s.a2s = o;   o = (uint32_t)align_up(o + (size_t)CE * G * 4, 128);
  s.dred = o;  o = (uint32_t)align_up(o + (size_t)NC * CE * 4, 128);
  s.dsl = o;   o = (uint32_t)align_up(o + (size_t)CE * NC * G * 2, 128);
  s.ring = o;  o += (uint32_t)S * d1_slot_bytes(H);
  s.total = o;
  return s;
}

__global__ void __launch_bounds__(kD1Threads, 2) decode1_kernel(const D1Args a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  cg::cluster_group cluster = cg::this_cluster();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rank = (int)cluster.block_rank();
  const int H = a.H, E = a.E, G = a.G, EH = a.E >> 1;
  const int P = gridDim.x, bid = blockIdx.x;
  const D1Smem L = d1_smem(H, E, G, a.CE, a.S, a.NC);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);  // [0, S): gate/up slots
  uint64_t* bar_dsl = bars + kD1MaxSlots;
  uint64_t* bar_in = bars + kD1MaxSlots + 1;  // this rank's router rows
  uint64_t* bar_lg = bars + kD1MaxSlots + 2;  // the peer's E/2 logits (st.async bytes)
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem + L.x);
  float* lg = reinterpret_cast<float*>(smem + L.lg);
  float* ws = reinterpret_cast<float*>(smem + L.w);
  int* ulist = reinterpret_cast<int*>(smem + L.ulist);
  int* misc = reinterpret_cast<int*>(smem + L.misc);  // [0] |U|, [1] epoch
  float* scr = reinterpret_cast<float*>(smem + L.scr);
  float* a2s = reinterpret_cast<float*>(smem + L.a2s);
  float* dred = reinterpret_cast<float*>(smem + L.dred);
  uint8_t* dsl = smem + L.dsl;
  uint8_t* ring = smem + L.ring;
  uint8_t* rrows = smem + L.alias;
  const uint32_t hb = 2u * (uint32_t)H, rpitch = d1_router_pitch(H), slotb = d1_slot_bytes(H);
  const int g8 = lane >> 2, q = lane & 3;

  D1_TRACE(0);
  if (tid == 0) {
    for (int s = 0; s < kD1MaxSlots; ++s) mbar_init(&bars[s], 1);
    mbar_init(bar_dsl, 1);
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
      bulk_g2s(rrows + (size_t)e * rpitch, a.router_eh + (size_t)(rank * EH + e) * H, hb, bar_in, pol);
  }
  if (a.trig_early) pdl_launch_dependents();
  if (a.pdl) pdl_wait();
  D1_TRACE(1);
  // token row: plain 16-byte loads (written by the previous kernel, normally still in L2)
  for (int i = tid; i < H / 8; i += kD1Threads)
    reinterpret_cast<uint4*>(xs)[i] = reinterpret_cast<const uint4*>(a.x)[i];
  if (tid == 0) {
    const uint32_t ep = ld_acquire_gpu(a.epoch) + 1u;
    misc[1] = (int)ep;
    st_relaxed_u64(a.presence + bid, (unsigned long long)ep << 32);
  }
  mbar_wait(bar_in, 0u, a.status);
  __syncthreads();
  D1_TRACE(2);

  // ---- 1. router on the tensor cores: D[16 x 8] += A[16 x 16] B[16 x 8] per k-step and
  // expert tile; A row 0 = the token (lanes 0-3), B column n = router row of expert 8t + n.
  // Warp w takes k-steps [w KS / 12, (w+1) KS / 12) of every tile; all tiles and both k
  // parities accumulate in independent chains.
  {
    const int KS = H >> 4, NTL = (EH + 7) >> 3;  // NTL <= 4 (E <= 64)
    const int k0 = (KS * warp) / kD1Warps, k1 = (KS * (warp + 1)) / kD1Warps;
    float* rpart = scr;  // [12][EH]
    const uint32_t xrow = smem_u32(xs) + 8 * q;
    uint32_t brow[4];
    float d[4][2][4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      brow[t] = smem_u32(rrows + (size_t)min(8 * t + g8, EH - 1) * rpitch) + 8 * q;
#pragma unroll
      for (int h = 0; h < 2; ++h) d[t][h][0] = d[t][h][1] = d[t][h][2] = d[t][h][3] = 0.f;
    }
    #pragma unroll 1
    for (int k = k0; k < k1; k += 2) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int kk = min(k + h, k1 - 1);
        uint2 xa;
        asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(xa.x), "=r"(xa.y) : "r"(xrow + 32 * kk));
        if (lane >= 4 || k + h >= k1) xa = make_uint2(0u, 0u);  // only A row 0 carries the token
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          if (t < NTL) {
            uint2 bv;
            asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(bv.x), "=r"(bv.y) : "r"(brow[t] + 32 * kk));
            asm volatile(
                "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                "{%0,%1,%2,%3};"
                : "+f"(d[t][h][0]), "+f"(d[t][h][1]), "+f"(d[t][h][2]), "+f"(d[t][h][3])
                : "r"(xa.x), "r"(0u), "r"(xa.y), "r"(0u), "r"(bv.x), "r"(bv.y));
          }
        }
      }
    }
    if (lane < 4) {
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int e = 8 * t + 2 * q;
        if (e < EH) rpart[warp * EH + e] = d[t][0][0] + d[t][1][0];
        if (e + 1 < EH) rpart[warp * EH + e + 1] = d[t][0][1] + d[t][1][1];
      }
    }
    __syncthreads();
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
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

  // ---- 3 + 4, per chunk of CE experts of the union
  const int nU = misc[0];
  const uint32_t want = (uint32_t)misc[1];
  const unsigned long long ep = (unsigned long long)want << 32;
  const int h0 = (int)((uint32_t)H * bid / P), ncols = (int)((uint32_t)H * (bid + 1) / P) - h0;
  const int NX = H >> 3;  // 16-byte token chunks; lane covers chunks lane + 32 i
  const uint64_t pol = policy_evict_first();
  float accv = 0.f;  // thread tid < ncols: output column h0 + tid
  const int nch = (nU + a.CE - 1) / a.CE;
  #pragma unroll 1
  for (int ch = 0; ch < nch; ++ch) {
    const int eb = ch * a.CE, nUc = min(a.CE, nU - eb);
    const uint32_t nb = (uint32_t)eb * G, Wc = (uint32_t)nUc * G;
    const int i0 = (int)(nb + Wc * bid / P), cnt = (int)(nb + Wc * (bid + 1) / P) - i0;
    const uint32_t par = (uint32_t)(ch & 1);
    if (ch > 0) __syncthreads();  // the previous chunk's slots, down rows and a2 are consumed
    // issue: lane 0 of warp w copies gate/up slots w, w + 12, ... and the down rows of chunk
    // experts w, w + 12, ... (copies issued by one thread are serialised)
    if (lane == 0) {
      if (warp == 0) mbar_arrive_expect_tx(bar_dsl, (uint32_t)nUc * ncols * G * 2);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      for (int s = warp; s < cnt; s += kD1Warps) {
        const int gi = i0 + s, u = gi / G;
        mbar_arrive_expect_tx(&bars[s], 2u * hb);
        bulk_g2s(ring + (size_t)s * slotb, a.experts + ((size_t)ulist[u] * G + (gi - u * G)) * 3 * H, 2u * hb,
                 &bars[s], pol);
      }
      for (int ei = warp; ei < nUc; ei += kD1Warps)
        bulk_g2s(dsl + (size_t)ei * a.NC * G * 2, a.down_t + ((size_t)ulist[eb + ei] * H + h0) * G,
                 (uint32_t)ncols * G * 2, bar_dsl, pol);
    }
    if (ch == 0) {
      D1_TRACE(5);
      if (bid == 0) {  // optional side outputs from the first CTA
        for (int e = tid; e < E; e += kD1Threads) {
          if (a.logits_out) a.logits_out[e] = __float2bfloat16_rn(lg[e]);
          if (a.weights_out) a.weights_out[e] = __float2bfloat16_rn(ws[e]);
          if (a.counts && ws[e] > 0.f) a.counts[e] += 1;
        }
      }
    }
    // gate/up: warp w takes slots w, w + 12, ...; lanes split K, butterfly sums (fixed order)
    #pragma unroll 1
    for (int s = warp; s < cnt; s += kD1Warps) {
      mbar_wait(&bars[s], par, a.status);
      if (ch == 0 && s == 0) D1_TRACE(6);
      const uint4* gr = reinterpret_cast<const uint4*>(ring + (size_t)s * slotb);
      const uint4* ur = reinterpret_cast<const uint4*>(ring + (size_t)s * slotb + hb);
      float g0 = 0.f, g1 = 0.f, u0 = 0.f, u1 = 0.f;
#pragma unroll
      for (int i = 0; i < kD1MaxXI; ++i) {
        const int c = lane + 32 * i;
        if (c < NX) {
          const uint4 gv = gr[c], uv = ur[c], xv = reinterpret_cast<const uint4*>(xs)[c];
          g0 = fmaf(bf_lo(xv.x), bf_lo(gv.x), g0); g1 = fmaf(bf_hi(xv.x), bf_hi(gv.x), g1);
          g0 = fmaf(bf_lo(xv.y), bf_lo(gv.y), g0); g1 = fmaf(bf_hi(xv.y), bf_hi(gv.y), g1);
          g0 = fmaf(bf_lo(xv.z), bf_lo(gv.z), g0); g1 = fmaf(bf_hi(xv.z), bf_hi(gv.z), g1);
          g0 = fmaf(bf_lo(xv.w), bf_lo(gv.w), g0); g1 = fmaf(bf_hi(xv.w), bf_hi(gv.w), g1);
          u0 = fmaf(bf_lo(xv.x), bf_lo(uv.x), u0); u1 = fmaf(bf_hi(xv.x), bf_hi(uv.x), u1);
          u0 = fmaf(bf_lo(xv.y), bf_lo(uv.y), u0); u1 = fmaf(bf_hi(xv.y), bf_hi(uv.y), u1);
          u0 = fmaf(bf_lo(xv.z), bf_lo(uv.z), u0); u1 = fmaf(bf_hi(xv.z), bf_hi(uv.z), u1);
          u0 = fmaf(bf_lo(xv.w), bf_lo(uv.w), u0); u1 = fmaf(bf_hi(xv.w), bf_hi(uv.w), u1);
        }
      }
      float g = g0 + g1, uu = u0 + u1;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        g += __shfl_xor_sync(0xffffffffu, g, o);
        uu += __shfl_xor_sync(0xffffffffu, uu, o);
      }
      if (lane == 0) {
        const int gi = i0 + s;
        const float gb = bf16r(g), ub = bf16r(uu);
        const float sb = bf16r(__fmul_rn(gb, __frcp_rn(1.f + expf(-gb))));  // silu
        const float a2 = bf16r(bf16r(sb * ub) * ws[ulist[gi / G]]);
        st_relaxed_u64(a.a2x + gi, ep | __float_as_uint(a2));
      }
    }
    if (ch == 0) D1_TRACE(7);
    if (a.trace) {  // diagnostics only: when every warp of the CTA is done with gate/up
      __syncthreads();
      if (ch == 0) D1_TRACE(16);
    }
    // every a2 of the chunk (and, in CTA 0's last chunk, every CTA's presence word) polled
    // until it carries this launch's epoch; four entries per thread in flight
    {
      const int n = (int)Wc + ((bid == 0 && ch == nch - 1) ? P : 0);
      #pragma unroll 1
      for (int b = 0; b < n; b += 4 * kD1Threads) {
        unsigned long long v[4];
        bool rdy[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          rdy[k] = b + tid + k * kD1Threads >= n;
          v[k] = 0ull;
        }
        uint32_t it = 0;
        #pragma unroll 1
        for (;;) {
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int idx = b + tid + k * kD1Threads;
            if (!rdy[k]) v[k] = ld_relaxed_u64(idx < (int)Wc ? a.a2x + nb + idx : a.presence + (idx - (int)Wc));
          }
          bool all = true;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            rdy[k] = rdy[k] || (uint32_t)(v[k] >> 32) == want;
            all = all && rdy[k];
          }
          if (all) break;
          if (++it > kSpinLimit) {
            atomicOr(a.status, DEVERR_TIMEOUT);
            break;
          }
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int idx = b + tid + k * kD1Threads;
          if (idx < (int)Wc) a2s[idx] = __uint_as_float((uint32_t)v[k]);
        }
      }
    }
    if (ch == 0) D1_TRACE(11);
    __syncthreads();
    if (ch == 0) D1_TRACE(8);
    mbar_wait(bar_dsl, par, a.status);
    if (ch == 0) D1_TRACE(12);
    // down: thread t -> (column t % ncols, chunk expert t / ncols), a G-long dot product read in
    // a rotated order (spreads the rows of neighbouring threads over the banks)
    {
      const int G8 = G >> 3;
      for (int t = tid; t < ncols * nUc; t += kD1Threads) {
        const int col = t % ncols, ei = t / ncols;
        const uint4* row = reinterpret_cast<const uint4*>(dsl + ((size_t)ei * a.NC + col) * G * 2);
        const float* av = a2s + ei * G;
        float s0 = 0.f, s1 = 0.f;
        int kk = t % G8;
        #pragma unroll 4
        for (int i = 0; i < G8; ++i) {
          const uint4 dv = row[kk];
          const float4 a0 = *reinterpret_cast<const float4*>(av + 8 * kk);
          const float4 a1 = *reinterpret_cast<const float4*>(av + 8 * kk + 4);
          s0 = fmaf(a0.x, bf_lo(dv.x), s0); s1 = fmaf(a0.y, bf_hi(dv.x), s1);
          s0 = fmaf(a0.z, bf_lo(dv.y), s0); s1 = fmaf(a0.w, bf_hi(dv.y), s1);
          s0 = fmaf(a1.x, bf_lo(dv.z), s0); s1 = fmaf(a1.y, bf_hi(dv.z), s1);
          s0 = fmaf(a1.z, bf_lo(dv.w), s0); s1 = fmaf(a1.w, bf_hi(dv.w), s1);
          kk = kk + 1 == G8 ? 0 : kk + 1;
        }
        dred[col * a.CE + ei] = s0 + s1;
      }
    }
    if (ch == 0) D1_TRACE(13);
    __syncthreads();
    if (ch == 0) D1_TRACE(14);
    if (tid < ncols) {
      float s = 0.f;
      for (int ei = 0; ei < nUc; ++ei) s += dred[tid * a.CE + ei];  // expert order
      accv += s;
    }
  }
  if (tid < ncols) a.out[h0 + tid] = __float2bfloat16_rn(accv);
  // CTA 0 has seen every CTA's presence word of this launch: every CTA has read the epoch
  if (bid == 0 && tid == 0)
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(a.epoch), "r"(want) : "memory");
  D1_TRACE(10);
  if (a.trace && tid == 0) a.trace[blockIdx.x * 32 + 30] = (unsigned long long)nch;
}

// ------------------------------------------------------------------ host side
struct D1Cfg {
  int dev = -1, H = 0, E = 0, G = 0;
  int ok = 0, grid = 0, CE = 0, S = 0, NC = 0;
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

// Bytes of the workspace region the single-token kernel needs: tagged a2 of every neuron and
// one presence word per CTA.
size_t decode1_region_bytes(int E, int G) { return ((size_t)E * G + kD1MaxGrid) * 8; }

// Returns 1 if launched, 0 if the kernel does not apply (caller falls back), < 0 on error.
// region: decode1_region_bytes; epoch: a word that only this kernel writes (zero-initialised
// with the workspace, like the region).
int decode1_launch(const void* x, const void* packed, int H, int E, int G, float tau, const float* bias, void* out,
                   void* logits_out, void* weights_out, int64_t* counts, int pdl, cudaStream_t stream,
                   uint32_t* status, uint32_t* epoch, void* region, size_t region_bytes,
                   unsigned long long* trace) {
  const int mode = d1_mode();
  if (mode == 0 || E > 64 || (E & 1) || H % 64 != 0 || H > 256 * kD1MaxXI || G % 8 != 0 || !region ||
      region_bytes < decode1_region_bytes(E, G))
    return 0;
  int dev = 0;
  PPMOE_CHECK_CUDA(cudaGetDevice(&dev));
  D1Cfg& C = g_d1;
  if (C.dev != dev || C.H != H || C.E != E || C.G != G) {
    C = D1Cfg();
    C.dev = dev; C.H = H; C.E = E; C.G = G;
    int nsm = 0, smem_sm = 0;
    PPMOE_CHECK_CUDA(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev));
    PPMOE_CHECK_CUDA(cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev));
    // two CTAs per SM: each gets half the SM's shared memory minus the per-CTA reservation
    const int budget = smem_sm / 2 - 1024 - 1024;  // -1024: alignment slack of the dynamic base
    const int grid = (nsm / 2) * 2;
    const int NC = (H + grid - 1) / grid;
    int CE = E, S = 0;
    D1Smem Lm{};
    for (; CE >= 1; --CE) {
      S = (CE * G + grid - 1) / grid;
      Lm = d1_smem(H, E, G, CE, S, NC);
      if (S <= kD1MaxSlots && (int)Lm.total <= budget) break;
    }
    const size_t router_need = (size_t)(E / 2) * d1_router_pitch(H);
    if (CE >= 1 && grid <= kD1MaxGrid && router_need <= Lm.total - Lm.alias) {
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
      if (clusters * 2 >= grid) {  // the a2 polls need the whole grid resident
        C.ok = 1;
        C.grid = grid;
        C.CE = CE;
        C.S = S;
        C.NC = NC;
        C.smem = smem;
      }
    }
  }
  if (!C.ok) return 0;
  const PackedLayout PL = packed_layout(H, E, G);
  const uint8_t* pk = static_cast<const uint8_t*>(packed);
  D1Args a;
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.router_eh = reinterpret_cast<const __nv_bfloat16*>(pk + PL.router_eh);
  a.experts = reinterpret_cast<const __nv_bfloat16*>(pk + PL.experts);
  a.down_t = reinterpret_cast<const __nv_bfloat16*>(pk + PL.down_t);
  a.H = H; a.E = E; a.G = G;
  a.tau_b = __bfloat162float(__float2bfloat16_rn(tau));
  a.bias = bias;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.logits_out = static_cast<__nv_bfloat16*>(logits_out);
  a.weights_out = static_cast<__nv_bfloat16*>(weights_out);
  a.counts = reinterpret_cast<long long*>(counts);
  a.a2x = static_cast<unsigned long long*>(region);
  a.presence = a.a2x + (size_t)E * G;
  a.epoch = epoch;
  a.status = status;
  a.CE = C.CE;
  a.S = C.S;
  a.NC = C.NC;
  a.trig_early = mode == 2;
  a.pdl = pdl;
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
