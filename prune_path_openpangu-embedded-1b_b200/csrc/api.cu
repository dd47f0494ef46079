// extern "C" entry points of libppmoe (declared in include/ppmoe.h): argument validation,
// workspace layout, error reporting.  The kernels live in pack.cu, route.cu, decode.cu.
#include <stdarg.h>
#include <string.h>
#include "common.cuh"

namespace ppmoe {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

void clear_error() { g_err[0] = 0; }

int cuda_fail(cudaError_t e, const char* what) {
  set_error("%s failed: %s", what, cudaGetErrorString(e));
  return PPMOE_ERR_CUDA;
}

int pack_launch(const void*, const void*, const void*, const void*, int, int, int, void*, cudaStream_t);
int route_logits_launch(const void*, int, int, float, const float*, void*, uint8_t*, cudaStream_t,
                        void* probs_out = nullptr);
int decode_launch(const void*, int, const void*, int, int, int, float, const float*, void*, void*, void*,
                  int64_t*, void*, size_t, int, cudaStream_t, uint32_t*, uint32_t*, float*, size_t, int x_host = 0);

void decode_set_trace(void*);
size_t route_workspace_bytes(long long, int);
int route_launch(const void*, int, const void*, int, int, int, float, const float*, int32_t*, void*, int32_t*,
                 uint8_t*, void*, size_t, cudaStream_t);
size_t prefill_workspace_bytes(long long, int, int, int);
int prefill_launch(const void*, int, const void*, int, int, int, float, const float*, void*, void*, void*, int64_t*,
                   void*, size_t, cudaStream_t, int, int xpitch = 0, int wpitch = 0);

// Workspace header: status word, decode arrival counters; then the decode cluster partials.
constexpr size_t kWsHeader = 256;
constexpr size_t kWsCounters = 64;
constexpr int kWsMaxClusters = 32;

static bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

static int check_shape(const char* fn, int H, int E, int G) {
  if (H <= 0 || H % 64 != 0 || H > 4096) {
    set_error("%s: hidden=%d must be a positive multiple of 64 <= 4096", fn, H);
    return PPMOE_ERR_UNSUPPORTED;
  }
  if (E <= 0 || E > 256 || E % 2 != 0) {
    set_error("%s: experts=%d must be even and in [2, 256]", fn, E);
    return PPMOE_ERR_UNSUPPORTED;
  }
  if (G <= 0 || G % 8 != 0 || G > 256) {
    set_error("%s: group=%d must be a positive multiple of 8 <= 256", fn, G);
    return PPMOE_ERR_UNSUPPORTED;
  }
  return PPMOE_OK;
}

}  // namespace ppmoe

using namespace ppmoe;

extern "C" {

int ppmoe_version(void) { return 100; }

const char* ppmoe_last_error(void) { return g_err; }

void ppmoe_debug_trace(void* buf) { decode_set_trace(buf); }

size_t ppmoe_packed_bytes(int hidden, int experts, int group) {
  if (check_shape("ppmoe_packed_bytes", hidden, experts, group)) return 0;
  return packed_layout(hidden, experts, group).total;
}

int ppmoe_pack(const void* W_gate, const void* W_up, const void* W_down, const void* router, int hidden,
               int experts, int group, void* packed, void* stream) {
  g_err[0] = 0;
  if (int rc = check_shape("ppmoe_pack", hidden, experts, group)) return rc;
  if (!W_gate || !W_up || !W_down || !router || !packed) {
    set_error("ppmoe_pack: null pointer");
    return PPMOE_ERR_INVALID_ARG;
  }
  if (!aligned(packed, 1024)) {
    set_error("ppmoe_pack: packed buffer must be 1024-byte aligned");
    return PPMOE_ERR_INVALID_ARG;
  }
  return pack_launch(W_gate, W_up, W_down, router, hidden, experts, group, packed,
                     static_cast<cudaStream_t>(stream));
}

size_t ppmoe_workspace_bytes(int max_tokens, int hidden, int experts, int group) {
  if (check_shape("ppmoe_workspace_bytes", hidden, experts, group) || max_tokens < 0) return 0;
  const size_t nt = (size_t)(max_tokens < PPMOE_DECODE_MAX_TOKENS ? max_tokens : PPMOE_DECODE_MAX_TOKENS);
  // cross-cluster partials of the decode kernel
  const size_t multi = (size_t)kWsMaxClusters * (nt ? nt : 1) * hidden * 4;
  return kWsHeader + multi;
}

int ppmoe_workspace_init(void* ws, size_t ws_bytes, void* stream) {
  g_err[0] = 0;
  if (!ws || ws_bytes < kWsHeader || !aligned(ws, 256)) {
    set_error("ppmoe_workspace_init: workspace must be >= %zu bytes and 256-byte aligned", kWsHeader);
    return PPMOE_ERR_INVALID_ARG;
  }
  // the whole workspace: prefill's fp32 accumulator must start at zero as well
  PPMOE_CHECK_CUDA(cudaMemsetAsync(ws, 0, ws_bytes, static_cast<cudaStream_t>(stream)));
  return PPMOE_OK;
}

int ppmoe_workspace_status(void* ws, void* stream) {
  g_err[0] = 0;
  if (!ws) {
    set_error("ppmoe_workspace_status: null workspace");
    return PPMOE_ERR_INVALID_ARG;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint32_t word = 0;
  PPMOE_CHECK_CUDA(cudaMemcpyAsync(&word, ws, 4, cudaMemcpyDeviceToHost, st));
  PPMOE_CHECK_CUDA(cudaStreamSynchronize(st));
  if (word == 0) return PPMOE_OK;
  PPMOE_CHECK_CUDA(cudaMemsetAsync(ws, 0, 4, st));
  // a timed-out launch may have left arrival counters armed: re-arm them too (words 0-7; word
  // 8 is the single-token kernel's launch epoch, which must keep counting)
  PPMOE_CHECK_CUDA(cudaMemsetAsync(static_cast<uint8_t*>(ws) + kWsCounters, 0, 32, st));
  PPMOE_CHECK_CUDA(cudaStreamSynchronize(st));
  if (word & DEVERR_TIMEOUT) {
    set_error("device: a bounded wait timed out (status 0x%x)", word);
    return PPMOE_ERR_TIMEOUT;
  }
  set_error("device: capacity exceeded (status 0x%x)", word);
  return PPMOE_ERR_WORKSPACE;
}

int ppmoe_route_logits(const void* logits, int tokens, int experts, float tau, void* weights_out,
                       uint8_t* mask_out, void* stream) {
  g_err[0] = 0;
  if (tokens < 0 || experts <= 0 || experts > 256) {
    set_error("ppmoe_route_logits: tokens=%d experts=%d out of range", tokens, experts);
    return PPMOE_ERR_UNSUPPORTED;
  }
  if (tokens > 0 && (!logits || !weights_out)) {
    set_error("ppmoe_route_logits: null pointer");
    return PPMOE_ERR_INVALID_ARG;
  }
  return route_logits_launch(logits, tokens, experts, tau, nullptr, weights_out, mask_out,
                             static_cast<cudaStream_t>(stream));
}

int ppmoe_route_logits_train(const void* logits, int tokens, int experts, float tau, void* weights_out,
                             uint8_t* mask_out, void* probs_out, void* stream) {
  g_err[0] = 0;
  if (tokens < 0 || experts <= 0 || experts > 256) {
    set_error("ppmoe_route_logits_train: tokens=%d experts=%d out of range", tokens, experts);
    return PPMOE_ERR_UNSUPPORTED;
  }
  if (tokens > 0 && (!logits || !weights_out || !probs_out)) {
    set_error("ppmoe_route_logits_train: null pointer");
    return PPMOE_ERR_INVALID_ARG;
  }
  return route_logits_launch(logits, tokens, experts, tau, nullptr, weights_out, mask_out,
                             static_cast<cudaStream_t>(stream), probs_out);
}

static int decode_checked(const char* fn, const void* x, int tokens, const void* packed, int hidden, int experts,
                          int group, float tau, const float* logit_bias, void* out, void* logits_out,
                          void* weights_out, int64_t* counts, void* ws, size_t ws_bytes, int pdl, void* stream,
                          int x_host) {
  if (int rc = check_shape(fn, hidden, experts, group)) return rc;
  if (tokens < 1 || tokens > PPMOE_DECODE_MAX_TOKENS) {
    set_error("%s: tokens=%d must be in [1, %d]", fn, tokens, PPMOE_DECODE_MAX_TOKENS);
    return PPMOE_ERR_UNSUPPORTED;
  }
  if (!x || !packed || !out || !ws) {
    set_error("%s: null pointer", fn);
    return PPMOE_ERR_INVALID_ARG;
  }
  if (!aligned(x, 16) || !aligned(out, 16) || !aligned(packed, 1024) || !aligned(ws, 256)) {
    set_error("%s: x/out must be 16-byte, packed 1024-byte, ws 256-byte aligned", fn);
    return PPMOE_ERR_INVALID_ARG;
  }
  if (ws_bytes < kWsHeader) {
    set_error("%s: workspace too small", fn);
    return PPMOE_ERR_WORKSPACE;
  }
  uint8_t* w8 = static_cast<uint8_t*>(ws);
  return decode_launch(x, tokens, packed, hidden, experts, group, tau, logit_bias, out, logits_out, weights_out,
                       counts, ws, ws_bytes, pdl, static_cast<cudaStream_t>(stream),
                       reinterpret_cast<uint32_t*>(w8), reinterpret_cast<uint32_t*>(w8 + kWsCounters),
                       reinterpret_cast<float*>(w8 + kWsHeader), ws_bytes - kWsHeader, x_host);
}

int ppmoe_decode(const void* x, int tokens, const void* packed, int hidden, int experts, int group, float tau,
                 const float* logit_bias, void* out, void* logits_out, void* weights_out, int64_t* counts,
                 void* ws, size_t ws_bytes, int pdl, void* stream) {
  g_err[0] = 0;
  return decode_checked("ppmoe_decode", x, tokens, packed, hidden, experts, group, tau, logit_bias, out, logits_out,
                        weights_out, counts, ws, ws_bytes, pdl, stream, 0);
}

// Token rows from pinned host memory into the staging buffer, one CTA, chained by
// programmatic dependent launch between the previous decode and the next one: it lets the
// next decode launch at once (its prologue loads only weights), copies while the previous
// decode is still finishing, and exits only after that decode has completed, so the next
// decode's griddepcontrol.wait also covers the previous decode (which used the same
// workspace).  Overwriting x_dev early is safe: this grid starts only after every CTA of the
// previous decode has signalled its dependents, which each does long after its rows landed.
__global__ void x_stage_kernel(const uint4* src_host, uint4* __restrict__ dst, int n16) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  for (int i = threadIdx.x; i < n16; i += blockDim.x) dst[i] = src_host[i];
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

static int launch_x_stage(const void* src_host, void* dst, size_t bytes, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  PPMOE_CHECK_CUDA(cudaLaunchKernelEx(&cfg, x_stage_kernel, static_cast<const uint4*>(src_host),
                                      static_cast<uint4*>(dst), (int)(bytes / 16)));
  return PPMOE_OK;
}

// Device address of pinned, mapped host memory, or null (pageable or unregistered memory).
static void* mapped_host(const void* p) {
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();  // clear the error of an unregistered pointer
    return nullptr;
  }
  return at.type == cudaMemoryTypeHost ? at.devicePointer : nullptr;
}

int ppmoe_decode_host(const void* x_host, int tokens, const void* packed, int hidden, int experts, int group,
                      float tau, const float* logit_bias, void* out_host, void* x_dev, void* out_dev, void* ws,
                      size_t ws_bytes, void* stream) {
  g_err[0] = 0;
  if (!x_host || !out_host) {
    set_error("ppmoe_decode_host: null host pointer");
    return PPMOE_ERR_INVALID_ARG;
  }
  // Token rows: pinned, mapped host memory is staged by a one-CTA kernel chained with
  // programmatic dependent launch (the copy overlaps the previous decode; reading host memory
  // from every CTA of the decode itself means thousands of small reads over the host link,
  // measured ~4x slower); pageable memory by a stream-ordered copy.  The output is small and
  // written by a few CTAs: into pinned, mapped host memory directly when out_host allows it
  // (no device-to-host copy operation), else via out_dev.
  const size_t bytes = (size_t)tokens * (size_t)hidden * 2;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  void* xm = mapped_host(x_host);
  const bool ok_tokens = tokens >= 1 && tokens <= PPMOE_DECODE_MAX_TOKENS && x_dev;
  if (ok_tokens && xm && aligned(xm, 16) && aligned(x_dev, 16)) {
    if (int rc = launch_x_stage(xm, x_dev, bytes, s)) return rc;
  } else {
    xm = nullptr;
    if (ok_tokens) PPMOE_CHECK_CUDA(cudaMemcpyAsync(x_dev, x_host, bytes, cudaMemcpyHostToDevice, s));
  }
  void* om = mapped_host(out_host);
  const int rc = decode_checked("ppmoe_decode_host", x_dev, tokens, packed, hidden, experts, group, tau, logit_bias,
                                om ? om : out_dev, nullptr, nullptr, nullptr, ws, ws_bytes, xm ? 1 : 0, stream, 0);
  if (rc != PPMOE_OK || om) return rc;
  PPMOE_CHECK_CUDA(cudaMemcpyAsync(out_host, out_dev, bytes, cudaMemcpyDeviceToHost, s));
  return PPMOE_OK;
}

size_t ppmoe_prefill_workspace_bytes(int tokens, int hidden, int experts, int group) {
  if (check_shape("ppmoe_prefill_workspace_bytes", hidden, experts, group) || tokens < 1) return 0;
  return prefill_workspace_bytes(tokens, hidden, experts, group);
}

static int prefill_checks(const char* fn, const void* x, int tokens, const void* packed, int hidden, int experts,
                          int group, const void* out, const void* ws) {
  if (int rc = check_shape(fn, hidden, experts, group)) return rc;
  if (group % 16 != 0 || group > 128) {
    set_error("%s: group=%d must be a multiple of 16 and <= 128", fn, group);
    return PPMOE_ERR_UNSUPPORTED;
  }
  if (tokens < 1) {
    set_error("%s: tokens=%d must be >= 1", fn, tokens);
    return PPMOE_ERR_UNSUPPORTED;
  }
  if (!x || !packed || !out || !ws) {
    set_error("%s: null pointer", fn);
    return PPMOE_ERR_INVALID_ARG;
  }
  if (!aligned(x, 16) || !aligned(out, 16) || !aligned(packed, 1024) || !aligned(ws, 1024)) {
    set_error("%s: x/out must be 16-byte, packed and ws 1024-byte aligned", fn);
    return PPMOE_ERR_INVALID_ARG;
  }
  return PPMOE_OK;
}

int ppmoe_prefill(const void* x, int tokens, const void* packed, int hidden, int experts, int group, float tau,
                  const float* logit_bias, void* out, void* logits_out, void* weights_out, int64_t* counts,
                  void* ws, size_t ws_bytes, void* stream) {
  g_err[0] = 0;
  if (int rc = prefill_checks("ppmoe_prefill", x, tokens, packed, hidden, experts, group, out, ws)) return rc;
  return prefill_launch(x, tokens, packed, hidden, experts, group, tau, logit_bias, out, logits_out, weights_out,
                        counts, ws, ws_bytes, static_cast<cudaStream_t>(stream), 0);
}

int ppmoe_prefill_route(const void* x, int tokens, const void* packed, int hidden, int experts, int group, float tau,
                        const float* logit_bias, void* logits_out, void* weights_out, void* ws, size_t ws_bytes,
                        void* stream) {
  g_err[0] = 0;
  if (int rc = prefill_checks("ppmoe_prefill_route", x, tokens, packed, hidden, experts, group, weights_out, ws))
    return rc;
  return prefill_launch(x, tokens, packed, hidden, experts, group, tau, logit_bias, weights_out, logits_out,
                        weights_out, nullptr, ws, ws_bytes, static_cast<cudaStream_t>(stream), 1);
}

int ppmoe_prefill_experts(const void* x, int tokens, const void* packed, int hidden, int experts, int group,
                          const void* weights, float* out_f32, int64_t* counts, void* ws, size_t ws_bytes,
                          void* stream) {
  g_err[0] = 0;
  if (int rc = prefill_checks("ppmoe_prefill_experts", x, tokens, packed, hidden, experts, group, out_f32, ws))
    return rc;
  if (!weights) {
    set_error("ppmoe_prefill_experts: null gate weights");
    return PPMOE_ERR_INVALID_ARG;
  }
  return prefill_launch(x, tokens, packed, hidden, experts, group, 0.f, nullptr, out_f32, nullptr,
                        const_cast<void*>(weights), counts, ws, ws_bytes, static_cast<cudaStream_t>(stream), 2);
}

int ppmoe_ep_experts(const void* payload, int rows, int row_pitch, const void* packed, int hidden, int experts,
                     int group, int partial_format, void* out, void* ws, size_t ws_bytes, void* stream) {
  g_err[0] = 0;
  if (int rc = prefill_checks("ppmoe_ep_experts", payload, rows, packed, hidden, experts, group, out, ws))
    return rc;
  const int need = (int)align_up((size_t)(hidden + experts) * 2, 16);
  if (row_pitch < need || row_pitch % 16 != 0) {
    set_error("ppmoe_ep_experts: row_pitch=%d must be a multiple of 16 and >= %d", row_pitch, need);
    return PPMOE_ERR_INVALID_ARG;
  }
  if (partial_format != 0 && partial_format != 1) {
    set_error("ppmoe_ep_experts: partial_format=%d (0 fp32 rows, 1 scaled fp16 rows)", partial_format);
    return PPMOE_ERR_INVALID_ARG;
  }
  const uint8_t* p = static_cast<const uint8_t*>(payload);
  return prefill_launch(p, rows, packed, hidden, experts, group, 0.f, nullptr, out, nullptr,
                        const_cast<uint8_t*>(p + (size_t)hidden * 2), nullptr, ws, ws_bytes,
                        static_cast<cudaStream_t>(stream), partial_format ? 3 : 2, row_pitch / 2, row_pitch / 2);
}

size_t ppmoe_ep_partial_pitch(int hidden) {
  if (hidden <= 0 || hidden % 64 != 0) return 0;
  return f16s_pitch(hidden);
}

size_t ppmoe_route_workspace_bytes(int tokens, int hidden, int experts, int group) {
  if (check_shape("ppmoe_route_workspace_bytes", hidden, experts, group) || tokens < 1) return 0;
  return route_workspace_bytes(tokens, experts);
}

int ppmoe_route(const void* x, int tokens, const void* packed, int hidden, int experts, int group, float tau,
                const float* logit_bias, int32_t* active_ids, void* active_w, int32_t* n_active, uint8_t* mask,
                void* ws, size_t ws_bytes, void* stream) {
  g_err[0] = 0;
  if (int rc = check_shape("ppmoe_route", hidden, experts, group)) return rc;
  if (tokens < 1) {
    set_error("ppmoe_route: tokens=%d must be >= 1", tokens);
    return PPMOE_ERR_UNSUPPORTED;
  }
  if (!x || !packed || !active_ids || !active_w || !n_active || !ws) {
    set_error("ppmoe_route: null pointer");
    return PPMOE_ERR_INVALID_ARG;
  }
  if (!aligned(x, 16) || !aligned(packed, 1024) || !aligned(ws, 1024)) {
    set_error("ppmoe_route: x must be 16-byte, packed and ws 1024-byte aligned");
    return PPMOE_ERR_INVALID_ARG;
  }
  return route_launch(x, tokens, packed, hidden, experts, group, tau, logit_bias, active_ids, active_w, n_active,
                      mask, ws, ws_bytes, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
