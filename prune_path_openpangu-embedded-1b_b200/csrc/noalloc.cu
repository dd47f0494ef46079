// Allocation-free fused decode: the same single-launch decode kernel as ppmoe_decode, with
// its scratch (status word, arrival counters, cross-cluster partial sums) in a fixed-size
// array that lives in this library's own device memory instead of a caller workspace.
//
// For callers that cannot allocate device memory at the point of the call: code running
// under an allocator or memory pool that is not theirs to grow, plugin hosts that hand out
// only inputs and outputs, or hot paths where a cudaMalloc would synchronise the device.
#include <mutex>
#include "common.cuh"

namespace ppmoe {

int decode_launch(const void*, int, const void*, int, int, int, float, const float*, void*, void*, void*,
                  int64_t*, void*, size_t, int, cudaStream_t, uint32_t*, uint32_t*, float*, size_t, int x_host = 0);

// Scratch limit: tokens * hidden <= 8192 (e.g. 5 tokens at hidden 1536, 4 at 2048, 16 at
// 512) for up to 32 clusters of the decode grid: 32 * 8192 * 4 bytes of partials plus a
// 256-byte header.  Every GPU that loads the library holds this ~1 MiB until exit.
constexpr int kNoAllocMaxTokHidden = 8192;
constexpr size_t kNoAllocHeader = 256;
constexpr size_t kNoAllocBytes = kNoAllocHeader + (size_t)32 * kNoAllocMaxTokHidden * 4;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocBytes];

constexpr int kMaxDevices = 64;
static void* g_scratch_ptr[kMaxDevices] = {};
static std::mutex g_scratch_mu;

// Device address of the scratch array on the current device (looked up once per device;
// in host code the array's name is only a host-side stand-in, never a device address).
// The cached address belongs to the device's current primary context: after
// cudaDeviceReset the library's module is reloaded elsewhere and the address is stale, so
// these entry points must not be used across a device reset.
static int scratch_address(void** out) {
  int dev = 0;
  PPMOE_CHECK_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("ppmoe_decode_noalloc: device ordinal %d out of range", dev);
    return PPMOE_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    PPMOE_CHECK_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return PPMOE_OK;
}

}  // namespace ppmoe

using namespace ppmoe;

extern "C" int ppmoe_decode_noalloc(const void* x, int tokens, const void* packed, int hidden, int experts,
                                    int group, float tau, void* out, void* stream) {
  clear_error();
  if (tokens < 1 || tokens > PPMOE_DECODE_MAX_TOKENS || hidden <= 0 ||
      (long long)tokens * hidden > kNoAllocMaxTokHidden) {
    set_error("ppmoe_decode_noalloc: tokens * hidden = %lld exceeds the built-in scratch limit %d "
              "(tokens must also be in [1, %d]); use ppmoe_decode with a caller workspace",
              (long long)tokens * hidden, kNoAllocMaxTokHidden, PPMOE_DECODE_MAX_TOKENS);
    return PPMOE_ERR_UNSUPPORTED;
  }
  if (hidden % 64 != 0 || hidden > 4096 || experts < 2 || experts > 256 || experts % 2 != 0 ||
      group <= 0 || group % 8 != 0 || group > 256) {
    set_error("ppmoe_decode_noalloc: shape H=%d E=%d G=%d outside the supported range", hidden, experts, group);
    return PPMOE_ERR_UNSUPPORTED;
  }
  if (!x || !packed || !out) {
    set_error("ppmoe_decode_noalloc: null pointer");
    return PPMOE_ERR_INVALID_ARG;
  }
  if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(out) % 16 ||
      reinterpret_cast<uintptr_t>(packed) % 1024) {
    set_error("ppmoe_decode_noalloc: x/out must be 16-byte and packed 1024-byte aligned");
    return PPMOE_ERR_INVALID_ARG;
  }
  void* ws = nullptr;
  if (int rc = scratch_address(&ws)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // status word and arrival counters must start at zero (a previous call may have timed out)
  PPMOE_CHECK_CUDA(cudaMemsetAsync(ws, 0, kNoAllocHeader, st));
  uint8_t* w8 = static_cast<uint8_t*>(ws);
  return decode_launch(x, tokens, packed, hidden, experts, group, tau, nullptr, out, nullptr, nullptr, nullptr,
                       ws, kNoAllocBytes, 0, st, reinterpret_cast<uint32_t*>(w8),
                       reinterpret_cast<uint32_t*>(w8 + 64), reinterpret_cast<float*>(w8 + kNoAllocHeader),
                       kNoAllocBytes - kNoAllocHeader);
}

// Status of the allocation-free decode calls on the current device: synchronises `stream`,
// reads the status word in the library-owned scratch (the bits a bounded device-side wait or
// a capacity check set), and on an error re-arms the word and the arrival counters so that
// the next call starts clean.  Mirrors ppmoe_workspace_status for the caller-workspace path.
extern "C" int ppmoe_decode_noalloc_status(void* stream) {
  clear_error();
  void* ws = nullptr;
  if (int rc = scratch_address(&ws)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint32_t word = 0;
  PPMOE_CHECK_CUDA(cudaMemcpyAsync(&word, ws, 4, cudaMemcpyDeviceToHost, st));
  PPMOE_CHECK_CUDA(cudaStreamSynchronize(st));
  if (word == 0) return PPMOE_OK;
  PPMOE_CHECK_CUDA(cudaMemsetAsync(ws, 0, kNoAllocHeader, st));
  PPMOE_CHECK_CUDA(cudaStreamSynchronize(st));
  if (word & DEVERR_TIMEOUT) {
    set_error("ppmoe_decode_noalloc: a bounded device-side wait timed out (status 0x%x)", word);
    return PPMOE_ERR_TIMEOUT;
  }
  set_error("ppmoe_decode_noalloc: capacity exceeded on the device (status 0x%x)", word);
  return PPMOE_ERR_WORKSPACE;
}
