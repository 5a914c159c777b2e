/*
 * C ABI of the B200 (sm_100a) DeepSeek-V3/R1 FP8 block-scaled MoE forward.
 *
 * Plain pointers and sizes only; every device pointer is CUDA device memory on the
 * current device and every call is asynchronous on `stream` (a cudaStream_t, NULL for the
 * legacy default stream) unless stated otherwise. Functions return MOE_OK (0) or an error
 * code; moe_last_error() gives the message of the last failure on the calling thread.
 *
 * The three entry points the reference extension exports through pybind11
 * (kernels/moe.cu:902-909) map one to one:
 *   pack_w13    (kernels/moe.cu:700-720) -> moe_pack_w13  (+ moe_pack_w13_bytes)
 *   pack_w2     (kernels/moe.cu:722-742) -> moe_pack_w2   (+ moe_pack_w2_bytes)
 *   moe_forward (kernels/moe.cu:744-900) -> moe_forward   (+ moe_forward_workspace_bytes)
 * The reference allocates its scratch and output through the PyTorch caching allocator
 * (kernels/moe.cu:819-833); here the caller passes both, so the library itself never
 * allocates device memory on the forward path.
 */
#ifndef MOE_B200_H
#define MOE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MOE_OK 0
#define MOE_ERR_INVALID 1   /* bad argument; message names it (reference TORCH_CHECK text) */
#define MOE_ERR_CUDA 2      /* a CUDA runtime call or kernel launch failed */
#define MOE_ERR_WORKSPACE 3 /* workspace smaller than moe_forward_workspace_bytes() */

/* Fixed geometry (reference/moe_ref.py:26-42). */
#define MOE_HIDDEN 7168
#define MOE_INTER 2048
#define MOE_EXPERTS 256
#define MOE_TOPK 8

/* Message of the last failed call on this thread ("" if none). */
const char* moe_last_error(void);

/* Device status word written by kernels (bit 1/2/4: a bounded wait of the producer / MMA /
 * epilogue role timed out; bit 8: inconsistent routing metadata). Synchronises the device.
 * When reset != 0 the word is cleared after reading. No reference counterpart: the
 * reference never checks kernel-side failures. */
int moe_get_status(int* status, int reset);

/* Bytes of the packed W13 for E_local experts (the reference returns an int32 tensor of
 * the same byte count, kernels/moe.cu:712). */
size_t moe_pack_w13_bytes(int E_local);

/* Replaces pack_w13 (kernels/moe.cu:700-720). w13: e4m3 [E_local, 4096, 7168], contiguous,
 * 16-byte aligned. w13_packed: moe_pack_w13_bytes(E_local) bytes, 16-byte aligned; its
 * layout is private to this library (consumed only by moe_forward). */
int moe_pack_w13(const void* w13, int E_local, void* w13_packed, void* stream);

size_t moe_pack_w2_bytes(int E_local);

/* Replaces pack_w2 (kernels/moe.cu:722-742). w2: e4m3 [E_local, 7168, 2048]. */
int moe_pack_w2(const void* w2, int E_local, void* w2_packed, void* stream);

/* Scratch bytes moe_forward needs for T tokens and E_local local experts. */
size_t moe_forward_workspace_bytes(int T, int E_local);

/* Replaces moe_forward (kernels/moe.cu:744-900), same argument order plus explicit sizes,
 * output, workspace and stream:
 *   hidden        e4m3 [T, 7168]
 *   hidden_scale  fp32 [56, T]            (block-major, reference/moe_ref.py:45)
 *   w13_packed    from moe_pack_w13,      w13_scale fp32 [E_local, 32, 56]
 *   w2_packed     from moe_pack_w2,       w2_scale  fp32 [E_local, 56, 16]
 *   logits        fp32 [T, 256],          bias      fp32 [256]
 *   routed_scaling_factor, local_expert_offset: as reference/moe_ref.py:14-15
 *   out_bf16      bf16 [T, 7168]          (written completely; tokens without a local
 *                                          expert get zeros)
 *   T             0 <= T <= 65536
 * All device pointers 16-byte aligned. Asynchronous; no host synchronisation. */
int moe_forward(const void* hidden, const float* hidden_scale, const void* w13_packed,
                const float* w13_scale, const void* w2_packed, const float* w2_scale,
                const float* logits, const float* bias, float routed_scaling_factor,
                int local_expert_offset, int T, int E_local, void* out_bf16, void* workspace,
                size_t workspace_bytes, void* stream);

/* Size of the static device scratch used by moe_forward_noalloc: 72 MiB per device. */
#define MOE_NOALLOC_SCRATCH_BYTES (72u << 20)

/* moe_forward for callers that cannot allocate device memory - for example a plugin whose host
 * application owns all GPU memory through its own pool, or a code path where a cudaMalloc
 * (which may synchronise the device and fail under memory pressure) is not allowed. It takes
 * no workspace: its scratch is a static array inside this library, MOE_NOALLOC_SCRATCH_BYTES
 * bytes on every device that loads the library, held until the process exits. The caller still
 * passes all inputs and the output, exactly as for moe_forward.
 *   - Limit: moe_forward_workspace_bytes(T, E_local) must not exceed MOE_NOALLOC_SCRATCH_BYTES
 *     (e.g. T <= 64 tokens with 32 local experts); larger calls return MOE_ERR_WORKSPACE and
 *     do nothing.
 *   - The first call on a device looks up the scratch address (and does the same one-time
 *     kernel set-up as moe_forward); make that first call before any stream capture.
 *   - Every call on a device uses the same scratch, so calls that can overlap on the GPU (on
 *     different streams, or from different threads) race and must be serialised by the
 *     caller. The scratch keeps the previous call's contents; each call resets what it needs.
 *   - It calls no cudaMalloc, cudaFree or other allocating routine.
 * No counterpart in the reference (its moe_forward allocates through PyTorch,
 * kernels/moe.cu:819-833). */
int moe_forward_noalloc(const void* hidden, const float* hidden_scale, const void* w13_packed,
                        const float* w13_scale, const void* w2_packed, const float* w2_scale,
                        const float* logits, const float* bias, float routed_scaling_factor,
                        int local_expert_offset, int T, int E_local, void* out_bf16, void* stream);

/* moe_forward that also records events[0..5] (cudaEvent_t) on `stream`: before the first
 * launch and after each of its five kernels (route, gather, gemm1, gemm2, combine), for
 * per-kernel timing. No reference counterpart (instrumentation only). */
int moe_forward_profiled(const void* hidden, const float* hidden_scale, const void* w13_packed,
                         const float* w13_scale, const void* w2_packed, const float* w2_scale,
                         const float* logits, const float* bias, float routed_scaling_factor,
                         int local_expert_offset, int T, int E_local, void* out_bf16,
                         void* workspace, size_t workspace_bytes, void* stream,
                         void* const* events);

/* Router alone (the routing half of moe_forward, reference/moe_ref.py:82-107): writes the
 * 8 selected global experts per token in selection order (descending biased score, ties to
 * the lower index) and their weights. No reference counterpart as a separate entry: the
 * reference keeps the indices internal; this exposes them for index-parity checks. */
int moe_route(const float* logits, const float* bias, float routed_scaling_factor, int T,
              int* topk_idx, float* topk_w, void* stream);

/* Byte offsets of the internal workspace regions for (T, E_local), in this order:
 * counts, dense_base, topk_idx, topk_w, token_nr, token_route, route_token, route_w, a_tiled,
 * a_scale, c_hi, c_lo, c_scale, partial, total. Writes min(n, 15) values; returns the number of
 * regions (15). For tests and tooling. */
int moe_workspace_layout(int T, int E_local, size_t* offsets, int n);

/* ---- Seeded synthetic inputs on the GPU (bit-identical to the CPU generator) ----
 * table: device fp32 [65537] inverse-normal-CDF table (see the Python package).
 * No reference counterpart: the reference draws inputs with torch (moe_layer.py:47-74). */
int moe_synth_logits(const float* table, uint64_t seed, int T, int E, float* out, void* stream);
int moe_synth_bias(const float* table, uint64_t seed, int E, float stddev, const int* hot_dev,
                   int n_hot, float hot_value, uint16_t* out_bf16, void* stream);
int moe_synth_hidden(const float* table, uint64_t seed, int T, float stddev, void* hidden,
                     float* hidden_scale, void* stream);
int moe_synth_w13(const float* table, uint64_t seed, int e0, int E, float stddev, void* w13,
                  float* w13_scale, void* stream);
int moe_synth_w2(const float* table, uint64_t seed, int e0, int E, float stddev, void* w2,
                 float* w2_scale, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MOE_B200_H */
