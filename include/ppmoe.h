/*
 * ppmoe.h -- C ABI of the B200 (sm_100a) PrunePath sparse-MoE MLP library (libppmoe.so).
 *
 * Plain pointers and sizes only.  Every tensor pointer is DEVICE memory owned by the caller
 * unless stated otherwise; bf16 tensors are passed as `void*` (2-byte IEEE bfloat16,
 * row-major, contiguous).  `stream` is a `cudaStream_t` passed as `void*` (NULL = legacy
 * default stream).  Every call returns an int status: 0 = ok, negative = error (see
 * PPMOE_ERR_*); `ppmoe_last_error()` gives the message of the last failing call on the
 * calling host thread.  Launches are asynchronous; device-side faults that the kernels
 * detect (a bounded wait that ran out) are recorded in the workspace and returned by
 * `ppmoe_workspace_status()`.
 *
 * Shapes: hidden H, experts E, neurons per expert G, intermediate I = E * G.
 * Supported: H % 64 == 0, H <= 4096, E even and 2 <= E <= 256, G % 8 == 0, G <= 256.
 *
 * The reference exposes this path only as the PyTorch module `TauSparseMoE`
 * (src/tl_kernel_optimized_Ultimate_PanGU.py:468-615); each entry point below names the
 * part of that module (or of its callers) it replaces.
 */
#ifndef PPMOE_H_
#define PPMOE_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define PPMOE_API __attribute__((visibility("default")))
#else
#define PPMOE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define PPMOE_OK 0
#define PPMOE_ERR_INVALID_ARG (-1)  /* null pointer, bad size or misaligned buffer */
#define PPMOE_ERR_UNSUPPORTED (-2)  /* shape outside the supported range */
#define PPMOE_ERR_TIMEOUT (-3)      /* a bounded device-side wait ran out (status word) */
#define PPMOE_ERR_CUDA (-4)         /* a CUDA runtime call failed */
#define PPMOE_ERR_WORKSPACE (-5)    /* workspace too small or not initialised */

/* Largest token count the fused decode kernel takes; larger batches use the prefill path
 * (the reference takes its decode path only at one token, tl:612-615). */
#define PPMOE_DECODE_MAX_TOKENS 16

/* Library version (major * 10000 + minor * 100 + patch). */
PPMOE_API int ppmoe_version(void);

/* Message of the last failing call on this host thread ("" if none). */
PPMOE_API const char* ppmoe_last_error(void);

/* ---------------------------------------------------------------------------------------
 * Packed weights.  Replaces the layout that `physical_reorder_for_inference`
 * (src/openpangu_moe.py:212-256) mounts on TauSparseMoE's buffers W_gate [H,I],
 * W_up [H,I], W_down [I,H], router [H,E] (tl:483-486): this call reads exactly those
 * buffers and writes one packed, 1 KiB-aligned blob:
 *   router_eh [E][H] | experts [E][G][3][H] (gate row, up row, down row of each neuron,
 *   contiguous) | down_t [E][H][G]
 * ------------------------------------------------------------------------------------- */
PPMOE_API size_t ppmoe_packed_bytes(int hidden, int experts, int group);
PPMOE_API int ppmoe_pack(const void* W_gate, const void* W_up, const void* W_down, const void* router,
               int hidden, int experts, int group, void* packed, void* stream);

/* ---------------------------------------------------------------------------------------
 * Workspace: scratch the kernels keep between calls (cross-cluster partial sums,
 * self-resetting arrival counters, the device status word).  Size it with
 * ppmoe_workspace_bytes for the largest token count the caller will pass and zero it once
 * with ppmoe_workspace_init (which clears the whole buffer).  One workspace must not be used by two calls that can run
 * concurrently (different streams).
 * ------------------------------------------------------------------------------------- */
PPMOE_API size_t ppmoe_workspace_bytes(int max_tokens, int hidden, int experts, int group);
PPMOE_API int ppmoe_workspace_init(void* ws, size_t ws_bytes, void* stream);
/* Synchronises `stream`, returns PPMOE_OK or the first device-side error recorded since the
 * last call, and clears it. */
PPMOE_API int ppmoe_workspace_status(void* ws, void* stream);

/* ---------------------------------------------------------------------------------------
 * Router selection from given bf16 logits [N][E] (softmax, descending-probability order with
 * ties to the lower expert index, bf16 cumulative mass < bf16(tau), forced top-1).
 * Replaces `softmax_thresholding` (src/MoEBlock.py:49-95) and the selection half of
 * moe_router_select_kernel_decode (tl:356-380) / moe_select_expert_kernel (tl:96-124).
 * weights_out [N][E] bf16: sigmoid(logit) on selected experts, 0 elsewhere (required).
 * mask_out [N][E] uint8 (optional, may be NULL).
 * ------------------------------------------------------------------------------------- */
PPMOE_API int ppmoe_route_logits(const void* logits, int tokens, int experts, float tau,
                       void* weights_out, uint8_t* mask_out, void* stream);
/* Training-mode variant: also writes probs_out [N][E] bf16 = softmax(logits), the second
 * output of softmax_thresholding(training=True) (src/MoEBlock.py:68, 93-94) that the
 * entropy and load-balance regularisers consume (src/openpangu_moe.py:282-307).  These are
 * exactly the probabilities the selection ranked. */
PPMOE_API int ppmoe_route_logits_train(const void* logits, int tokens, int experts, float tau,
                                       void* weights_out, uint8_t* mask_out, void* probs_out, void* stream);

/* Router from token rows to a compact active-expert list per token: router GEMM (tcgen05) over
 * the packed router rows, bf16 logits (+ optional fp32 prior logit_bias [E], then rounded to
 * bf16), and the selection above.  Replaces moe_router_select_kernel_decode
 * (src/tl_kernel_optimized_Ultimate_PanGU.py:335-380) and its outputs decode_active_idx,
 * decode_active_weight, decode_num_active (tl:488-490, filled at tl:502-509), for any
 * number of tokens:
 *   active_ids [N][E] int32: token t's selected experts in descending softmax probability
 *     (ties to the lower expert index), positions >= n_active[t] hold -1;
 *   active_w [N][E] bf16: their gate weights sigmoid(logit) in the same order, 0 past the end;
 *   n_active [N] int32: number of selected experts (>= 1: the forced top-1);
 *   mask [N][E] uint8: optional dense selection mask (NULL to skip).
 * Workspace: ppmoe_route_workspace_bytes(tokens, ...) bytes, 1024-byte aligned (no zeroing
 * needed). */
PPMOE_API size_t ppmoe_route_workspace_bytes(int tokens, int hidden, int experts, int group);
PPMOE_API int ppmoe_route(const void* x, int tokens, const void* packed, int hidden, int experts, int group,
                          float tau, const float* logit_bias, int32_t* active_ids, void* active_w,
                          int32_t* n_active, uint8_t* mask, void* ws, size_t ws_bytes, void* stream);

/* ---------------------------------------------------------------------------------------
 * Fused decode, 1 <= tokens <= PPMOE_DECODE_MAX_TOKENS: router GEMV + selection + expert
 * SwiGLU + down projection in ONE launch.  Replaces TauSparseMoE.forward_decode
 * (tl:494-530: moe_router_select_kernel_decode + moe_decode_swiglu_fused_kernel).
 *   x [N][H] bf16 -> out [N][H] bf16.
 *   logit_bias: optional fp32 [E] added to the bf16 logits (then rounded to bf16) before
 *     selection; NULL for the reference's bias-free router.
 *   logits_out [N][E] bf16, weights_out [N][E] bf16, counts [E] int64 (+= number of tokens
 *     that selected each expert, the reference's activated_statistics,
 *     src/MoEBlock.py:189-191): optional, NULL to skip.
 *   pdl != 0 launches with programmatic dependent launch: the kernel prefetches its router
 *     slice before waiting on the previous kernel in the stream.
 * ------------------------------------------------------------------------------------- */
PPMOE_API int ppmoe_decode(const void* x, int tokens, const void* packed, int hidden, int experts,
                 int group, float tau, const float* logit_bias, void* out, void* logits_out,
                 void* weights_out, int64_t* counts, void* ws, size_t ws_bytes, int pdl,
                 void* stream);

/* Host-buffer decode for callers that hold activations in host memory, e.g. a plugin host:
 * x_host [tokens][hidden] bf16 is staged into x_dev (pinned, mapped host memory: by a
 * one-CTA kernel chained to the decode with programmatic dependent launch, so the transfer
 * overlaps the previous call's decode; pageable memory: by a stream-ordered
 * cudaMemcpyAsync), then the fused decode.  When out_host is pinned and mapped into the device address space (cudaHostAlloc /
 * torch pin_memory on a UVA system) the kernel writes the bf16 output into it directly;
 * otherwise into out_dev followed by a cudaMemcpyAsync into out_host.  The caller
 * synchronises the stream before reading out_host.  x_dev / out_dev: device staging buffers
 * of tokens * hidden bf16, 16-byte aligned (out_dev unused when out_host is pinned).
 * Equivalent to TauSparseMoE.forward (tl:606-615) on a host tensor moved to the device and
 * back.  Other arguments and limits as for ppmoe_decode. */
PPMOE_API int ppmoe_decode_host(const void* x_host, int tokens, const void* packed, int hidden, int experts,
                                int group, float tau, const float* logit_bias, void* out_host, void* x_dev,
                                void* out_dev, void* ws, size_t ws_bytes, void* stream);

/* ---------------------------------------------------------------------------------------
 * Prefill, any token count: tcgen05 router GEMM + selection, device-side dispatch (per-expert
 * counts, 128-row tiles, token permutation; no host synchronisation), tcgen05 grouped
 * gate/up GEMM with the SwiGLU epilogue, tcgen05 down GEMM with an fp32 per-token combine,
 * one bf16 rounding.  Replaces TauSparseMoE.forward_prefill (tl:532-604) and its kernels
 * moe_router_kernel, moe_select_expert_kernel, moe_local/global_scan_kernel,
 * moe_dispatch_kernel, moe_fused_expert_kernel (tl:40-328).
 *   Needs group % 16 == 0 and group <= 128 in addition to the shapes above.
 *   Workspace: ppmoe_prefill_workspace_bytes(tokens, ...) bytes, 1024-byte aligned, zeroed once
 *   (e.g. with ppmoe_workspace_init over its full size); a workspace sized for N tokens serves
 *   any call with <= N tokens.  Its status word is read by ppmoe_workspace_status.
 *   Other arguments as for ppmoe_decode.
 * ------------------------------------------------------------------------------------- */
PPMOE_API size_t ppmoe_prefill_workspace_bytes(int tokens, int hidden, int experts, int group);
PPMOE_API int ppmoe_prefill(const void* x, int tokens, const void* packed, int hidden, int experts, int group,
                            float tau, const float* logit_bias, void* out, void* logits_out, void* weights_out,
                            int64_t* counts, void* ws, size_t ws_bytes, void* stream);

/* Router half of ppmoe_prefill (router GEMM + selection): gate weights [N][E] bf16 (0 where
 * unselected) into weights_out, bf16 logits into logits_out (optional).  Replaces
 * moe_router_kernel + torch.sort + moe_select_expert_kernel + scatter_ (tl:40-124, 550-564).
 * Used by expert-parallel prefill on each rank's token shard.  Needs only
 * ppmoe_route_workspace_bytes(tokens, ...) bytes of workspace, and reads only the router
 * section of `packed` (its first E * H * 2 bytes: router_eh [E][H]), so a 1024-byte aligned
 * buffer holding just those rows serves as `packed`. */
PPMOE_API int ppmoe_prefill_route(const void* x, int tokens, const void* packed, int hidden, int experts,
                                  int group, float tau, const float* logit_bias, void* logits_out,
                                  void* weights_out, void* ws, size_t ws_bytes, void* stream);
/* Expert half of ppmoe_prefill for rows whose gate weights are given (weights [N][E] bf16,
 * 0 = expert not selected): dispatch + grouped gate/up + down GEMMs; out_f32 [N][H] receives
 * the fp32 sums over the given experts (no bf16 rounding, so partial sums from several
 * expert shards can be added exactly as the single-device path would).  Replaces
 * moe_local/global_scan, moe_dispatch and moe_fused_expert kernels (tl:133-328, 566-604). */
PPMOE_API int ppmoe_prefill_experts(const void* x, int tokens, const void* packed, int hidden, int experts,
                                    int group, const void* weights, float* out_f32, int64_t* counts, void* ws,
                                    size_t ws_bytes, void* stream);

/* Expert-parallel prefill, source side: out[t] = bf16( sum over d = 0..ranks-1 of
 * back[row_of[d][t]] ) with fp32 additions in rank order, skipping row_of = -1.
 * back [rows][hidden] fp32 (the partial sums returned by the expert-owning ranks), row_of
 * [ranks][tokens] int32, out [tokens][hidden] bf16; ranks <= 8.  No reference counterpart
 * (the reference runs on one device). */
PPMOE_API int ppmoe_ep_combine(const float* back, const int32_t* row_of, int ranks, int tokens, int hidden,
                               void* out, void* stream);
/* Same with bf16 partial rows (back [rows][hidden] bf16): the optional reduced-traffic mode of
 * expert-parallel prefill, whose partials are rounded to bf16 once on the expert side. */
PPMOE_API int ppmoe_ep_combine_bf16(const void* back, const int32_t* row_of, int ranks, int tokens, int hidden,
                                    void* out, void* stream);

/* Expert-parallel prefill, dispatch side (no reference counterpart: the reference runs on one
 * device; this replaces the host-side send-list construction around the NCCL all-to-all).
 * Destination rank d owns, of each group of `ranks` consecutive experts g ranks .. g ranks +
 * ranks - 1, expert g ranks + d for even g and g ranks + ranks - 1 - d for odd g (snake order);
 * a token is sent to d when it selected at least one of them (weights [tokens][experts] bf16, 0 = not selected).  The tokens
 * go in `chunks` consecutive chunks of whole 256-token blocks (chunk c: blocks
 * [nb c / chunks, nb (c + 1) / chunks), nb = ceil(tokens / 256)).  `send` receives one payload
 * row of row_pitch bytes per (token, destination): hidden bf16 activations, then the token's
 * gate weights for the destination's experts in owned order; rows chunk-major, then
 * destination-major, tokens ascending.  counts [ranks][chunks] int64 = rows per segment;
 * row_of [ranks][tokens] int32 = the send row of (token, destination) or -1.  Device-side only
 * (no host synchronisation); send must hold tokens * ranks rows in the worst case.
 * row_pitch >= 2 (hidden + experts / ranks), a multiple of 16; ranks <= 8, chunks <= 8. */
PPMOE_API size_t ppmoe_ep_dispatch_workspace_bytes(int tokens, int ranks);
PPMOE_API int ppmoe_ep_dispatch(const void* x, const void* weights, int tokens, int hidden, int experts, int ranks,
                                int chunks, void* send, int row_pitch, int64_t* counts, int32_t* row_of, void* ws,
                                size_t ws_bytes, void* stream);
/* Expert-parallel prefill, expert side: ppmoe_prefill_experts over received payload rows
 * (ppmoe_ep_dispatch layout: activations, then the gate weights of this rank's `experts` local
 * experts) without unpacking them.  partial_format 0: out = [rows][hidden] fp32 partial sums;
 * 1: out = rows of ppmoe_ep_partial_pitch(hidden) bytes in the scaled-fp16 format (each
 * value's relative error <= 2^-11; half the bytes of fp32 rows on the way back).  Workspace
 * as ppmoe_prefill_workspace_bytes(rows, ...).  Replaces moe_local/global_scan, moe_dispatch and
 * moe_fused_expert_kernel (tl:133-328, 566-604) on the expert-owning rank. */
PPMOE_API int ppmoe_ep_experts(const void* payload, int rows, int row_pitch, const void* packed, int hidden,
                               int experts, int group, int partial_format, void* out, void* ws, size_t ws_bytes,
                               void* stream);
/* Bytes per row of the scaled-fp16 partial format (ppmoe_ep_experts partial_format 1): hidden
 * fp16 values, each 64-column slice multiplied by 2^s (exact) so that |value| < 2^15, then the
 * hidden / 64 int8 exponents s; padded to 16 bytes.  0 if hidden is not a multiple of 64. */
PPMOE_API size_t ppmoe_ep_partial_pitch(int hidden);
/* Source side for scaled-fp16 partial rows: out[t] = bf16( sum over d of row_of[d][t]'s row,
 * rescaled to fp32 ) with fp32 additions in rank order.  back: rows of `pitch` bytes. */
PPMOE_API int ppmoe_ep_combine_f16s(const void* back, int pitch, const int32_t* row_of, int ranks, int tokens,
                                    int hidden, void* out, void* stream);

/* ---------------------------------------------------------------------------------------
 * Fused decode that allocates nothing and takes no workspace: for callers that cannot call
 * cudaMalloc at this point (code running inside someone else's memory pool, plugin hosts
 * that only hand over inputs and outputs, latency-critical paths where an allocation would
 * synchronise the device).  No counterpart in the reference.  Same kernel and results as
 * ppmoe_decode without bias and side outputs; its scratch is a ~1 MiB array inside this
 * library's device memory, held by every GPU that loads the library until process exit.
 *   Limit: 1 <= tokens <= 16 and tokens * hidden <= 8192 (PPMOE_ERR_UNSUPPORTED beyond).
 *   The first call on a device looks up the array's device address; make that first call
 *   before any stream capture.  All calls share the one array: calls that can overlap on
 *   the GPU (different streams, or different host threads) race and must be serialised by
 *   the caller.  Each call clears the array's status word and counters before its launch, so
 *   read ppmoe_decode_noalloc_status after a call (before the next one) to learn whether the
 *   device reported an error.
 * ------------------------------------------------------------------------------------- */
PPMOE_API int ppmoe_decode_noalloc(const void* x, int tokens, const void* packed, int hidden, int experts,
                                   int group, float tau, void* out, void* stream);
/* Device-side status of the ppmoe_decode_noalloc calls made so far on the current device:
 * synchronises `stream` and returns PPMOE_OK, or PPMOE_ERR_TIMEOUT / PPMOE_ERR_WORKSPACE when a
 * launch recorded a bounded wait that ran out or a capacity overflow (its output is then not
 * valid); an error is cleared (status word and arrival counters re-armed) before returning.
 * Like ppmoe_decode_noalloc it allocates nothing.  The cached scratch address belongs to the
 * device's primary context: neither entry point may be used across cudaDeviceReset.
 * No counterpart in the reference. */
PPMOE_API int ppmoe_decode_noalloc_status(void* stream);

/* Diagnostics: when `buf` (device, >= 32 * 8 bytes per CTA of the decode grid) is non-NULL,
 * later ppmoe_decode launches record per-CTA phase timestamps (SM clock64) into it; NULL
 * switches recording off.  No counterpart in the reference (it has no tracing). */
PPMOE_API void ppmoe_debug_trace(void* buf);

#ifdef __cplusplus
}
#endif

#endif /* PPMOE_H_ */
