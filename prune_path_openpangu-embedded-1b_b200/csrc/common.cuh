// Shared device/host helpers for libppmoe (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>

#include "../../include/ppmoe.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "libppmoe is built for sm_100a only"
#endif

namespace ppmoe {

// ------------------------------------------------------------------ host error plumbing
void set_error(const char* fmt, ...);
void clear_error();  // empties the calling thread's last-error message
int cuda_fail(cudaError_t e, const char* what);

#define PPMOE_CHECK_CUDA(call)                                      \
  do {                                                              \
    cudaError_t _e = (call);                                        \
    if (_e != cudaSuccess) return ::ppmoe::cuda_fail(_e, #call);    \
  } while (0)

// Device status bits (workspace status word).
enum : uint32_t {
  DEVERR_TIMEOUT = 1u,      // a bounded mbarrier wait ran out
  DEVERR_OVERFLOW = 2u,     // a capacity bound was exceeded (work skipped)
};

// Size-bounded spin: ~2^22 polls with a short sleep ≈ well under a second.
constexpr uint32_t kSpinLimit = 1u << 22;

// ------------------------------------------------------------------ layout of the blob
struct PackedLayout {
  size_t router_eh, experts, down_t, total;
};

__host__ __device__ inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
// Bytes of one scaled-fp16 row of H values: H fp16 (each 64-column slice scaled by 2^s), then
// the H / 64 int8 exponents s, padded to 16 bytes.
__host__ __device__ inline size_t f16s_pitch(int H) { return align_up((size_t)H * 2 + (size_t)H / 64, 16); }

__host__ __device__ inline PackedLayout packed_layout(int H, int E, int G) {
  PackedLayout L;
  size_t off = 0;
  L.router_eh = off; off = align_up(off + (size_t)H * E * 2, 1024);
  L.experts = off;   off = align_up(off + (size_t)E * G * 3 * H * 2, 1024);
  L.down_t = off;    off = align_up(off + (size_t)E * G * H * 2, 1024);
  L.total = off;
  return L;
}

// ------------------------------------------------------------------ bf16 rounding helpers
__device__ __forceinline__ float bf16r(float v) {  // round to bf16 (RN-even), back to fp32
  return __bfloat162float(__float2bfloat16_rn(v));
}

// ------------------------------------------------------------------ PTX: mbarrier + bulk copy
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
               ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}

// Non-blocking probe of an mbarrier phase (returns at once; try_wait may suspend the thread
// for a system-defined time window before it re-checks).
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}

// Distributed-shared-memory helpers: the shared::cluster address of `p` in CTA `rank`, an
// arrival (release at cluster scope) on a barrier in another CTA of the cluster, and the
// acquire-at-cluster-scope probe used to wait for such arrivals.
__device__ __forceinline__ uint32_t mapa_u32(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase.  On timeout it records DEVERR_TIMEOUT in *status and
// returns false; the caller carries on (with garbage data) so that every CTA still reaches
// every cluster barrier and the launch ends.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* status) {
  const uint32_t a = smem_u32(bar);
#pragma unroll 1
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (i < 8192 ? mbar_test_wait(a, parity) : mbar_try_wait(a, parity)) return true;
    if (i > 16384) __nanosleep(32);
    // once any wait of this launch has given up, stop waiting quickly everywhere else
    if ((i & 1023u) == 1023u && status && *reinterpret_cast<volatile uint32_t*>(status)) return false;
  }
  if (status) atomicOr(status, DEVERR_TIMEOUT);
  return false;
}

// mbar_wait for waits that usually last long (pipeline stages, accumulator hand-offs): polls
// with the suspending try_wait from the first probe, so that waiting warps do not take issue
// slots from the warps that do the work.
__device__ __forceinline__ bool mbar_wait_parked(uint64_t* bar, uint32_t parity, uint32_t* status) {
  const uint32_t a = smem_u32(bar);
#pragma unroll 1
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(a, parity)) return true;
    if (i > 16384) __nanosleep(32);
    if ((i & 1023u) == 1023u && status && *reinterpret_cast<volatile uint32_t*>(status)) return false;
  }
  if (status) atomicOr(status, DEVERR_TIMEOUT);
  return false;
}

// mbar_wait with acquire at cluster scope (for phases completed by other CTAs' arrivals).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, uint32_t* status) {
  const uint32_t a = smem_u32(bar);
#pragma unroll 1
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait_cluster(a, parity)) return true;
    if (i > 16384) __nanosleep(32);
    if ((i & 1023u) == 1023u && status && *reinterpret_cast<volatile uint32_t*>(status)) return false;
  }
  if (status) atomicOr(status, DEVERR_TIMEOUT);
  return false;
}

// One-dimensional bulk copy global -> this CTA's shared memory, completing on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy) : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Programmatic dependent launch controls (no-ops when launched without the attribute).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------------------------------ warp helpers
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
    v = w > v ? w : v;
  }
  return v;
}

}  // namespace ppmoe
