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
 * epilogue role timed out; bit 8: inconsistent routing metadata; bit 16: an expert-parallel
 * barrier timed out waiting for a peer rank). Synchronises the device.
 * When reset != 0 the word is cleared after reading. No reference counterpart: the
 * reference never checks kernel-side failures. */
int moe_get_status(int* status, int reset);

/* Limit of every bounded wait in the kernels (mbarrier waits of the GEMM roles, the
 * expert-parallel flag barriers) on the current device, in nanoseconds; 2 s by default,
 * accepted range [1 ms, 60 s]. A wait that runs out sets its status bit and returns. No
 * reference counterpart (the reference has no waits). Synchronous. */
int moe_set_wait_limit_ns(unsigned long long ns);
int moe_get_wait_limit_ns(unsigned long long* ns);

/* Failure-path probes: each makes one bounded wait run out on purpose, on the host's request,
 * without a fault, so tests can check that the kernel returns and reports it.
 * moe_probe_ep_barrier_timeout: the expert-parallel barrier kernel of a 2-rank layout whose
 *   second rank never signals; buf = >= 256 zeroed device bytes standing for both ranks'
 *   buffers. Sets status bit 16 after the wait limit.
 * moe_probe_mbar_timeout: one thread waits on an mbarrier nothing arrives on; after the wait
 *   limit it sets status bit `who` (1, 2 or 4) and writes *aborted (device int) = 1.
 * No reference counterpart. */
int moe_probe_ep_barrier_timeout(void* buf, void* stream);
int moe_probe_mbar_timeout(int who, int* aborted, void* stream);

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
 *                                          expert get zeros; from 1024 tokens on, rows are
 *                                          written while inputs are still being read, so it
 *                                          must not overlap any input or the workspace:
 *                                          refused with MOE_ERR_INVALID)
 *   T             0 <= T <= 65536
 * All device pointers 16-byte aligned, the workspace 256-byte aligned (as cudaMalloc returns).
 * Asynchronous; no host synchronisation. */
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

/* moe_forward with the output left in fp32: out_f32 fp32 [T, 7168] receives the per-token sum
 * of the weighted expert outputs before the final bf16 rounding of reference/moe_ref.py:136
 * (moe_forward's result is exactly its bf16 rounding). For callers that add further fp32 terms
 * (another expert slice, a shared expert, the residual) and round once at the end. No
 * reference counterpart: the reference keeps this fp32 buffer internal (kernels/moe.cu:
 * 828-897). Other arguments as moe_forward. */
int moe_forward_f32(const void* hidden, const float* hidden_scale, const void* w13_packed,
                    const float* w13_scale, const void* w2_packed, const float* w2_scale,
                    const float* logits, const float* bias, float routed_scaling_factor,
                    int local_expert_offset, int T, int E_local, float* out_f32, void* workspace,
                    size_t workspace_bytes, void* stream);

/* DeepSeek-V3's shared-expert branch over the same FP8 block-scaled format: one expert
 * (w13_packed / w2_packed from moe_pack_w13 / moe_pack_w2 with E_local = 1, scales [1, 32, 56] /
 * [1, 56, 16]) applied to every token with weight 1, i.e. moe_forward's expert computation
 * (reference/moe_ref.py:126-134) with all tokens routed to it. out: bf16 [T, 7168], or fp32 when
 * out_fp32 != 0 (to add to moe_forward_f32's routed output before one final rounding).
 * Workspace: moe_forward_workspace_bytes(T, 1). No reference counterpart (the reference's layer
 * has no shared expert). */
int moe_shared_expert_forward(const void* hidden, const float* hidden_scale, const void* w13_packed,
                              const float* w13_scale, const void* w2_packed, const float* w2_scale, int T,
                              void* out, int out_fp32, void* workspace, size_t workspace_bytes, void* stream);

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

/* FP8 activation quantiser, the step before moe_forward: bf16 hidden [T, 7168] -> e4m3 codes
 * [T, 7168] and block-major fp32 scales [56, T] (the layout reference/moe_ref.py:44-45 takes).
 * Per (token, 128-column block): scale = amax / 448 (fp32 division; 1.0 for an all-zero block),
 * code = e4m3(x / scale), round to nearest even, saturating to +-448. Inputs must be finite.
 * No reference counterpart: the reference receives already-quantised activations. */
int moe_quantize_hidden(const void* hidden_bf16, int T, void* out_e4m3, float* out_scale, void* stream);

/* ---- MoE prologue: gate (router) GEMM fused with the FP8 quantiser ----
 * The DeepSeek-V3 gate computes the routing logits from the same normalised bf16 hidden rows
 * that the experts consume quantised. moe_gate_quantize reads those rows once and writes both:
 *   logits [T, 256] fp32 = hidden . W_gate^T (bf16 operands, fp32 accumulation; each token's
 *                          logits are independent of T and of its position in the batch),
 *   codes [T, 7168] e4m3 + scale [56, T] fp32, bit-identical to moe_quantize_hidden.
 * Together they are the routing_logits / hidden_states / hidden_states_scale inputs of
 * moe_forward (reference/moe_ref.py:5-16). No reference counterpart: the reference receives
 * logits and quantised activations as inputs.
 *
 * moe_pack_gate: W_gate bf16 [256, 7168] -> moe_gate_packed_bytes() bytes of packed images,
 * once per weight set. */
size_t moe_gate_packed_bytes(void);
int moe_pack_gate(const void* w_gate_bf16, void* gate_packed, void* stream);
int moe_gate_quantize(const void* hidden_bf16, const void* gate_packed, int T, float* logits,
                      void* out_e4m3, float* out_scale, void* stream);

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

/* ---- Expert-parallel layer over W GPUs of one node (W <= 8), one process per GPU ----
 *
 * Rank r owns e_rank global experts (world * e_rank <= 256): by default [r * e_rank,
 * (r + 1) * e_rank), or any placement given at moe_ep_create (for example one balanced by
 * expected load); picks of experts without an owner are dropped like non-local experts in
 * reference/moe_ref.py:115-116. Each rank holds its own tokens. moe_ep_forward returns, for the rank's own tokens, the
 * layer output over all owned experts of all ranks: per owner rank the fp32 sum of its routes
 * in ascending expert order (moe_forward_f32's result for that rank's experts), then the fp32
 * sum of those partials in ascending rank order, rounded once to bf16. Token rows and fp32
 * partial results move between the
 * GPUs as peer stores issued by the kernels (CUDA IPC mappings over NVLink); the only host
 * collective is the one-time exchange of the IPC handles (moe_ep_connect). Synchronisation
 * between ranks is by epoch flags with bounded waits (2 s; status bit 16 on timeout).
 *
 * No reference counterpart: the reference's moe_forward (kernels/moe.cu:744-900) runs on one
 * GPU over 32 local experts. Its semantics per rank are those of moe_forward_f32 with
 * local_expert_offset = r * e_rank, summed over ranks and rounded once.
 *
 * Protocol: every rank calls moe_ep_create (allocates its symmetric buffer, returns its IPC
 * handle), the handles are all-gathered in rank order, every rank calls moe_ep_connect, then
 * a host barrier; then all ranks call moe_ep_forward the same number of times, in the same
 * order (T may differ per rank and may be 0); teardown is a device synchronise and a host
 * barrier on every rank followed by moe_ep_destroy. */
#define MOE_EP_HANDLE_BYTES 64

/* Bytes of the per-rank symmetric buffer and of moe_ep_forward's workspace; 0 for an invalid
 * shape (world 1..8, t_rank_max >= 1, world * t_rank_max <= 65536, world * e_rank <= 256). */
size_t moe_ep_symmetric_bytes(int world, int t_rank_max, int e_rank);
size_t moe_ep_workspace_bytes(int world, int t_rank_max, int e_rank);

/* Creates rank `rank`'s context on the current device: allocates and zeroes the symmetric
 * buffer (synchronous) and writes its CUDA IPC handle (MOE_EP_HANDLE_BYTES) to ipc_handle.
 * placement: world * e_rank distinct global experts, rank-major (rank d owns
 * placement[d * e_rank ...] in that local order, the order of its weight arguments), the same
 * on every rank; NULL for the contiguous ranges [d * e_rank, (d + 1) * e_rank). Experts not
 * listed have no owner and their picks are dropped. */
int moe_ep_create(int rank, int world, int t_rank_max, int e_rank, const int* placement, void** ctx,
                  void* ipc_handle);

/* Maps the peers' buffers: handles = world * MOE_EP_HANDLE_BYTES, rank order. */
int moe_ep_connect(void* ctx, const void* handles);

/* Unmaps the peers and frees the buffer. Call only after every rank has finished its last
 * moe_ep_forward (device synchronise + host barrier). */
int moe_ep_destroy(void* ctx);

/* rank, world, t_rank_max, e_rank of a context. */
int moe_ep_info(void* ctx, int* out4);

/* One expert-parallel layer forward for this rank's T <= t_rank_max tokens:
 *   hidden e4m3 [T, 7168], hidden_scale fp32 [56, T], logits fp32 [T, 256], bias fp32 [256],
 *   w13_packed / w2_packed: this rank's e_rank experts in placement order (moe_pack_w13 /
 *                 moe_pack_w2),
 *   w13_scale fp32 [e_rank, 32, 56], w2_scale fp32 [e_rank, 56, 16],
 *   out_bf16 bf16 [T, 7168]; workspace of moe_ep_workspace_bytes(world, t_rank_max, e_rank),
 *   256-byte aligned.
 * Asynchronous on `stream`; the call itself never waits for other ranks. No per-call host state:
 * the barriers' epoch is kept and advanced in device memory, so the call can be captured into a
 * CUDA graph (after one eager call for the per-device set-up) and the graph replayed, one epoch
 * per replay, interleaved with eager calls. */
int moe_ep_forward(void* ctx, const void* hidden, const float* hidden_scale, const void* w13_packed,
                   const float* w13_scale, const void* w2_packed, const float* w2_scale,
                   const float* logits, const float* bias, float routed_scaling_factor, int T,
                   void* out_bf16, void* workspace, size_t workspace_bytes, void* stream);

/* moe_ep_forward recording events[0..9] on `stream`: before the first launch and after route,
 * dispatch, arrival barrier, gather, gemm1, gemm2, combine-send (+ counts reset), completion
 * barrier and final combine. Instrumentation only. */
int moe_ep_forward_profiled(void* ctx, const void* hidden, const float* hidden_scale,
                            const void* w13_packed, const float* w13_scale, const void* w2_packed,
                            const float* w2_scale, const float* logits, const float* bias,
                            float routed_scaling_factor, int T, void* out_bf16, void* workspace,
                            size_t workspace_bytes, void* stream, void* const* events);

#ifdef __cplusplus
}
#endif

#endif /* MOE_B200_H */
