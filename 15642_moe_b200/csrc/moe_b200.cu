/*
 * The one translation unit of libmoe_b200.so: every kernel plus the extern "C" boundary
 * declared in include/moe_b200.h.
 *
 * moe_forward pipeline (one stream, no host synchronisation):
 *   memset(counts) -> route_kernel -> gather_kernel -> gemm1_swiglu_kernel (tcgen05)
 *   -> gemm2_weighted_kernel (tcgen05) -> combine_kernel
 * replacing the reference's route_dispatch / stage1 / stage2 / bf16_convert launches
 * (kernels/moe.cu:842-897).
 *
 * moe_ep_forward (expert parallel over W GPUs, ep.cuh): route -> ep_dispatch (peer stores)
 *   -> barrier -> gather -> gemm1 -> gemm2 -> ep_combine_send (peer stores) -> memset(counts)
 *   -> barrier -> ep_final_combine.
 */
#include "moe_common.cuh"

#include "route.cuh"
#include "ep.cuh"
#include "gemm1.cuh"
#include "gemm2.cuh"
#include "pack.cuh"
#include "quant.cuh"
#include "gate.cuh"
#include "synth.cuh"
#include "moe_b200.h"

#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>
#include <utility>
#include <string>

using namespace moe;

namespace {

thread_local std::string g_err;

int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}

int cuda_check(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return MOE_OK;
  return fail(MOE_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

constexpr int DIRECT_MIN_TOKENS = 1024;

// Scratch of moe_forward_noalloc, for callers that cannot allocate device memory. One copy
// per device that loads this library, held until the process exits. Host code may not use the
// array's name as a device address: the address comes from cudaGetSymbolAddress, taken once
// per device with that device current (see noalloc_scratch()).
constexpr size_t NOALLOC_SCRATCH_BYTES = static_cast<size_t>(MOE_NOALLOC_SCRATCH_BYTES);
static __device__ __align__(256) uint8_t g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

struct DeviceInfo {
  bool ready = false;
  int num_sms = 0;
  void* noalloc_scratch = nullptr;  // device address of g_noalloc_scratch on this device
};
std::mutex g_dev_mu;
DeviceInfo g_dev[64];

// Per-device one-time set-up: SM count and the large dynamic shared-memory opt-in.
int device_info(DeviceInfo** out) {
  int dev = 0;
  if (int rc = cuda_check(cudaGetDevice(&dev), "cudaGetDevice")) return rc;
  if (dev < 0 || dev >= 64) return fail(MOE_ERR_CUDA, "device ordinal out of range");
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DeviceInfo& d = g_dev[dev];
  if (!d.ready) {
    if (int rc = cuda_check(cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev),
                            "cudaDeviceGetAttribute"))
      return rc;
    if (int rc = cuda_check(cudaFuncSetAttribute(gemm1_swiglu_kernel,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, G1_SMEM),
                            "cudaFuncSetAttribute(gemm1)"))
      return rc;
    if (int rc = cuda_check(cudaFuncSetAttribute(gemm2_weighted_kernel,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, G2_SMEM),
                            "cudaFuncSetAttribute(gemm2)"))
      return rc;
    if (int rc = cuda_check(cudaFuncSetAttribute(gate_quantize_kernel,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, GATE_SMEM),
                            "cudaFuncSetAttribute(gate)"))
      return rc;
    // setmaxnreg.inc in the epilogue warpgroups only completes if the CTA was launched with
    // enough registers for the whole split; refuse to launch a build where it could stall.
    cudaFuncAttributes fa1{}, fa2{};
    if (int rc = cuda_check(cudaFuncGetAttributes(&fa1, gemm1_swiglu_kernel), "cudaFuncGetAttributes(gemm1)")) return rc;
    if (int rc = cuda_check(cudaFuncGetAttributes(&fa2, gemm2_weighted_kernel), "cudaFuncGetAttributes(gemm2)")) return rc;
    if (fa1.numRegs < GEMM_LAUNCH_REGS_MIN || fa2.numRegs < GEMM_LAUNCH_REGS_MIN)
      return fail(MOE_ERR_CUDA, "GEMM kernels built with " + std::to_string(fa1.numRegs) + "/" +
                                    std::to_string(fa2.numRegs) + " registers per thread; the warpgroup "
                                    "register split needs " + std::to_string(GEMM_LAUNCH_REGS_MIN));
    d.ready = true;
  }
  *out = &d;
  return MOE_OK;
}

// Device address of this device's g_noalloc_scratch; looked up on the first call per device.
int noalloc_scratch(DeviceInfo* d, void** out) {
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (d->noalloc_scratch == nullptr) {
    void* p = nullptr;
    if (int rc = cuda_check(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress(scratch)"))
      return rc;
    d->noalloc_scratch = p;
  }
  *out = d->noalloc_scratch;
  return MOE_OK;
}

// cuTensorMapEncodeTiled from the driver, looked up once through the runtime (no -lcuda).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Tensor map of bf16 hidden [T, 7168] read as 128-row x 64-column boxes with the 128-byte
// swizzle (the K-major operand layout of the MMA); rows past T read as zero.
int hidden_bf16_map(const void* hidden, int T, CUtensorMap* map) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (encode == nullptr) return fail(MOE_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(T)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(H) * 2};
  const cuuint32_t box[2] = {64, TILE_M};
  const cuuint32_t elem[2] = {1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(hidden), dims, strides,
                            box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MOE_ERR_CUDA, "cuTensorMapEncodeTiled failed with code " + std::to_string(r));
  return MOE_OK;
}

// GEMM2 launched so that it may start on SMs that GEMM1's CTAs have left while GEMM1 still runs
// (programmatic dependent launch; GEMM1 allows it once all its CTAs are resident, GEMM2 waits per
// tile on the readiness counters GEMM1 publishes).
template <typename... KArgs, typename... Args>
cudaError_t launch_programmatic(void (*kernel)(KArgs...), int grid, int block, int smem, cudaStream_t st,
                                Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(static_cast<unsigned>(block));
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

cudaError_t launch_gemm2(const Gemm2Args& g2, int grid, cudaStream_t st) {
  return launch_programmatic(gemm2_weighted_kernel, grid, G2_THREADS, G2_SMEM, st, g2);
}

int grid_for(size_t work, int per_block, int cap) {
  size_t g = (work + per_block - 1) / per_block;
  if (g < 1) g = 1;
  if (g > static_cast<size_t>(cap)) g = cap;
  return static_cast<int>(g);
}

}  // namespace

extern "C" {

const char* moe_last_error(void) { return g_err.c_str(); }

int moe_get_status(int* status, int reset) {
  if (status == nullptr) return fail(MOE_ERR_INVALID, "status must not be null");
  if (int rc = cuda_check(cudaDeviceSynchronize(), "cudaDeviceSynchronize")) return rc;
  int v = 0;
  if (int rc = cuda_check(cudaMemcpyFromSymbol(&v, g_status, sizeof(int)), "read status")) return rc;
  *status = v;
  if (reset) {
    const int zero = 0;
    if (int rc = cuda_check(cudaMemcpyToSymbol(g_status, &zero, sizeof(int)), "reset status")) return rc;
  }
  return MOE_OK;
}

int moe_set_wait_limit_ns(unsigned long long ns) {
  if (ns < 1000000ull || ns > 60000000000ull)
    return fail(MOE_ERR_INVALID, "moe_set_wait_limit_ns: limit must be within [1 ms, 60 s]");
  return cuda_check(cudaMemcpyToSymbol(g_wait_limit_ns, &ns, sizeof(ns)), "set wait limit");
}

int moe_get_wait_limit_ns(unsigned long long* ns) {
  if (ns == nullptr) return fail(MOE_ERR_INVALID, "ns must not be null");
  return cuda_check(cudaMemcpyFromSymbol(ns, g_wait_limit_ns, sizeof(*ns)), "read wait limit");
}

int moe_probe_ep_barrier_timeout(void* buf, void* stream) {
  if (buf == nullptr || !aligned16(buf)) return fail(MOE_ERR_INVALID, "buf must be a 16-byte aligned device pointer");
  launch_ep_barrier_probe(static_cast<uint8_t*>(buf), static_cast<cudaStream_t>(stream));
  return cuda_check(cudaGetLastError(), "ep barrier probe launch");
}

int moe_probe_mbar_timeout(int who, int* aborted, void* stream) {
  if (who != ST_TIMEOUT_PRODUCER && who != ST_TIMEOUT_MMA && who != ST_TIMEOUT_EPILOGUE)
    return fail(MOE_ERR_INVALID, "who must be one of the role timeout bits 1, 2, 4");
  if (aborted == nullptr) return fail(MOE_ERR_INVALID, "aborted must not be null");
  mbar_probe_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(who, aborted);
  return cuda_check(cudaGetLastError(), "mbarrier probe launch");
}

size_t moe_pack_w13_bytes(int E_local) {
  return E_local > 0 ? static_cast<size_t>(E_local) * G1N * H : 0;
}

size_t moe_pack_w2_bytes(int E_local) {
  return E_local > 0 ? static_cast<size_t>(E_local) * H * I : 0;
}

int moe_pack_w13(const void* w13, int E_local, void* w13_packed, void* stream) {
  if (E_local < 1 || E_local > E_GLOBAL) return fail(MOE_ERR_INVALID, "W13 must be [E_local, 4096, 7168]");
  if (w13 == nullptr || w13_packed == nullptr) return fail(MOE_ERR_INVALID, "W13 must not be null");
  if (!aligned16(w13) || !aligned16(w13_packed)) return fail(MOE_ERR_INVALID, "W13 must be 16-byte aligned");
  DeviceInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  const size_t chunks = static_cast<size_t>(E_local) * G1_NT * 256 * (H / 16);
  pack_w13_kernel<<<grid_for(chunks, 256, d->num_sms * 16), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(w13), E_local, static_cast<uint8_t*>(w13_packed));
  return cuda_check(cudaGetLastError(), "pack_w13_kernel launch");
}

int moe_pack_w2(const void* w2, int E_local, void* w2_packed, void* stream) {
  if (E_local < 1 || E_local > E_GLOBAL) return fail(MOE_ERR_INVALID, "W2 must be [E_local, 7168, 2048]");
  if (w2 == nullptr || w2_packed == nullptr) return fail(MOE_ERR_INVALID, "W2 must not be null");
  if (!aligned16(w2) || !aligned16(w2_packed)) return fail(MOE_ERR_INVALID, "W2 must be 16-byte aligned");
  DeviceInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  const size_t chunks = static_cast<size_t>(E_local) * G2_NT * 256 * (I / 16);
  pack_w2_kernel<<<grid_for(chunks, 256, d->num_sms * 16), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(w2), E_local, static_cast<uint8_t*>(w2_packed));
  return cuda_check(cudaGetLastError(), "pack_w2_kernel launch");
}

size_t moe_forward_workspace_bytes(int T, int E_local) {
  if (T < 0 || E_local < 1 || E_local > E_GLOBAL) return 0;
  return make_workspace(T, E_local).total;
}

int moe_workspace_layout(int T, int E_local, size_t* offsets, int n) {
  if (T < 0 || E_local < 1 || E_local > E_GLOBAL) return fail(MOE_ERR_INVALID, "bad T or E_local");
  const Workspace w = make_workspace(T, E_local);
  const size_t v[16] = {w.counts,  w.dense_base, w.topk_idx, w.topk_w,  w.token_nr,
                        w.token_route, w.route_token, w.route_w, w.a_tiled, w.a_scale,
                        w.c_hi,    w.c_lo,       w.c_scale,  w.partial, w.tile_ready, w.total};
  for (int i = 0; i < n && i < 16; ++i) offsets[i] = v[i];
  return 16;
}

}  // extern "C"

namespace {

// The forward pipeline; when `events` is non-null, events[0..5] are recorded on the stream
// before the first launch and after each of the five kernels (route, gather, gemm1, gemm2,
// combine).
int forward_impl(const void* hidden, const float* hidden_scale, const void* w13_packed,
                 const float* w13_scale, const void* w2_packed, const float* w2_scale,
                 const float* logits, const float* bias, float routed_scaling_factor,
                 int local_expert_offset, int T, int E_local, void* out_bf16, void* workspace,
                 size_t workspace_bytes, void* stream, void* const* events, bool out_f32 = false,
                 bool shared = false) {
  if (T < 0) return fail(MOE_ERR_INVALID, "hidden must be [T, 7168]");
  if (E_local < 1 || E_local > E_GLOBAL) return fail(MOE_ERR_INVALID, "W13_packed must be [E_local, ...] with 1 <= E_local <= 256");
  if (T == 0) return MOE_OK;
  if (T > MAX_TOKENS) return fail(MOE_ERR_INVALID, "moe_forward: T must be at most 65536");
  if (!hidden || !hidden_scale || !w13_packed || !w13_scale || !w2_packed || !w2_scale ||
      (!shared && (!logits || !bias)) || !out_bf16 || !workspace)
    return fail(MOE_ERR_INVALID, "moe_forward: null pointer argument");
  const void* ptrs[] = {hidden, hidden_scale, w13_packed, w13_scale, w2_packed, w2_scale, logits, bias, out_bf16, workspace};
  for (const void* q : ptrs)
    if (!aligned16(q)) return fail(MOE_ERR_INVALID, "moe_forward: every tensor must be 16-byte aligned");
  const Workspace ws = make_workspace(T, E_local);
  if (workspace_bytes < ws.total)
    return fail(MOE_ERR_WORKSPACE, "workspace too small: need " + std::to_string(ws.total) + " bytes");
  // Kernels store 32-byte vectors into workspace regions (at 1024-byte offsets): the base must be
  // at least that aligned; 256 bytes is what cudaMalloc and the PyTorch allocator give.
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return fail(MOE_ERR_INVALID, "moe_forward: workspace must be 256-byte aligned");
  // Output rows are written while inputs are still being read (the router's zero rows before the
  // gather reads the hidden rows), so the output may overlap no input and not the workspace.
  {
    const size_t e = static_cast<size_t>(E_local), t = static_cast<size_t>(T);
    const struct {
      const void* p;
      size_t n;
    } in[] = {{hidden, t * H},
              {hidden_scale, sizeof(float) * HB * t},
              {w13_packed, e * 2 * I * H},
              {w13_scale, sizeof(float) * e * 2 * IB * HB},
              {w2_packed, e * H * I},
              {w2_scale, sizeof(float) * e * HB * IB},
              {logits, shared ? 0 : sizeof(float) * t * E_GLOBAL},
              {bias, shared ? 0 : sizeof(float) * E_GLOBAL},
              {workspace, ws.total}};
    const uintptr_t o0 = reinterpret_cast<uintptr_t>(out_bf16);
    const uintptr_t o1 = o0 + t * H * (out_f32 ? sizeof(float) : sizeof(uint16_t));
    for (const auto& r : in) {
      const uintptr_t a0 = reinterpret_cast<uintptr_t>(r.p);
      if (r.n != 0 && a0 < o1 && o0 < a0 + r.n)
        return fail(MOE_ERR_INVALID, "moe_forward: the output overlaps an input or the workspace");
    }
  }
  DeviceInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* W = static_cast<uint8_t*>(workspace);
  int* counts = reinterpret_cast<int*>(W + ws.counts);
  int* dense_base = reinterpret_cast<int*>(W + ws.dense_base);
  int* topk_idx = reinterpret_cast<int*>(W + ws.topk_idx);
  float* topk_w = reinterpret_cast<float*>(W + ws.topk_w);
  int* token_nr = reinterpret_cast<int*>(W + ws.token_nr);
  int* token_route = reinterpret_cast<int*>(W + ws.token_route);
  int* route_token = reinterpret_cast<int*>(W + ws.route_token);
  float* route_w = reinterpret_cast<float*>(W + ws.route_w);
  uint8_t* c_hi = W + ws.c_hi;
  uint8_t* c_lo = W + ws.c_lo;
  float* c_scale = reinterpret_cast<float*>(W + ws.c_scale);
  float* partial = reinterpret_cast<float*>(W + ws.partial);

  uint8_t* a_tiled = W + ws.a_tiled;
  float* a_scale = reinterpret_cast<float*>(W + ws.a_scale);
  int* tile_ready = reinterpret_cast<int*>(W + ws.tile_ready);
  Gemm1Args g1{a_tiled, a_scale, static_cast<const uint8_t*>(w13_packed), w13_scale, counts, T,
               ws.tiles_max, E_local, c_hi, c_lo, c_scale, tile_ready};
  // From DIRECT_MIN_TOKENS tokens on, GEMM2 writes the row of a token with one local route itself,
  // the router writes the zero row of a token with none, and the combine skips both (fewer fp32
  // route rows written and read back, fewer combine blocks); below, where that saved little and
  // GEMM2's extra loads cost a little, every token goes through the combine. The results are the
  // same either way.
  const int direct = T >= DIRECT_MIN_TOKENS ? 1 : 0;
  Gemm2Args g2{c_hi, c_lo, c_scale, static_cast<const uint8_t*>(w2_packed), w2_scale, counts, T,
               ws.tiles_max, E_local, route_w, partial, dense_base, tile_ready, tile_ready + ws.tiles_max,
               out_bf16, out_f32 ? 1 : 0, route_token, token_nr, direct};

  auto mark = [&](int i) {
    if (events != nullptr) cudaEventRecord(static_cast<cudaEvent_t>(events[i]), st);
  };
  mark(0);
  if (int rc = cuda_check(cudaMemsetAsync(counts, 0, sizeof(int) * E_local, st), "memset counts")) return rc;
  if (shared)
    shared_route_kernel<<<grid_for(static_cast<size_t>(T), 256, d->num_sms * 4), 256, 0, st>>>(
        T, counts, token_nr, token_route, route_token, route_w);
  else
    route_kernel<<<(T + 7) / 8, 256, 0, st>>>(logits, bias, T, routed_scaling_factor, local_expert_offset,
                                              E_local, topk_idx, topk_w, counts, token_nr, token_route,
                                              route_token, route_w, direct ? out_bf16 : nullptr,
                                              out_f32 ? H * 4 : H * 2);
  mark(1);
  const size_t route_max = static_cast<size_t>(T) * (E_local < TOP_K ? E_local : TOP_K);
  // gather and GEMM1 are launched programmatically: each may be scheduled while its predecessor
  // finishes and waits for it in hardware before touching its results.
  if (int rc = cuda_check(launch_programmatic(gather_kernel, grid_for(route_max, 8, d->num_sms * 8), 256, 0, st,
                                              static_cast<const uint8_t*>(hidden), hidden_scale, T,
                                              static_cast<const int*>(counts), E_local,
                                              static_cast<const int*>(route_token), ws.tiles_max, a_tiled, a_scale,
                                              tile_ready),
                          "gather launch"))
    return rc;
  mark(2);
  const int g1_grid = grid_for(static_cast<size_t>(ws.tiles_max) * G1_NT, 1, d->num_sms);
  if (int rc = cuda_check(launch_programmatic(gemm1_swiglu_kernel, g1_grid, G1_THREADS, G1_SMEM, st, g1),
                          "gemm1 launch"))
    return rc;
  mark(3);
  const int g2_grid = grid_for(static_cast<size_t>(ws.tiles_max) * G2_NT, 1, d->num_sms);
  if (int rc = cuda_check(launch_gemm2(g2, g2_grid, st), "gemm2 launch")) return rc;
  mark(4);
  if (out_f32)
    combine_kernel<float><<<T, COMBINE_THREADS, 0, st>>>(partial, token_nr, token_route, dense_base, T,
                                                         E_local, static_cast<float*>(out_bf16), direct);
  else
    combine_kernel<__nv_bfloat16><<<T, COMBINE_THREADS, 0, st>>>(partial, token_nr, token_route, dense_base,
                                                                 T, E_local, static_cast<__nv_bfloat16*>(out_bf16), direct);
  mark(5);
  return cuda_check(cudaGetLastError(), "moe_forward launch");
}

// ---- expert parallel -------------------------------------------------------------------

struct EpCtx {
  int rank = 0, world = 0, device = 0;
  EpLayout L{};
  uint8_t* local = nullptr;      // this rank's symmetric buffer (cudaMalloc)
  EpPeers peers{};
  bool opened[EP_MAX_RANKS] = {};  // peers[d] came from cudaIpcOpenMemHandle
  bool connected = false;
};

int ep_check_shape(int world, int t_rank_max, int e_rank) {
  if (world < 1 || world > EP_MAX_RANKS) return fail(MOE_ERR_INVALID, "moe_ep: world size must be 1..8");
  if (t_rank_max < 1) return fail(MOE_ERR_INVALID, "moe_ep: t_rank_max must be >= 1");
  if (static_cast<long long>(world) * t_rank_max > MAX_TOKENS)
    return fail(MOE_ERR_INVALID, "moe_ep: world * t_rank_max must be at most 65536");
  if (e_rank < 1 || static_cast<long long>(world) * e_rank > E_GLOBAL)
    return fail(MOE_ERR_INVALID, "moe_ep: e_rank must be >= 1 with world * e_rank <= 256");
  return MOE_OK;
}

int ep_forward_impl(EpCtx* c, const void* hidden, const float* hidden_scale, const void* w13_packed,
                    const float* w13_scale, const void* w2_packed, const float* w2_scale,
                    const float* logits, const float* bias, float routed_scaling_factor, int T,
                    void* out_bf16, void* workspace, size_t workspace_bytes, void* stream,
                    void* const* events) {
  if (c == nullptr || !c->connected) return fail(MOE_ERR_INVALID, "moe_ep_forward: context not connected");
  if (T < 0 || T > c->L.t_max)
    return fail(MOE_ERR_INVALID, "moe_ep_forward: T must be in [0, t_rank_max] (" + std::to_string(c->L.t_max) + ")");
  if (!w13_packed || !w13_scale || !w2_packed || !w2_scale || !bias || !workspace ||
      (T > 0 && (!hidden || !hidden_scale || !logits || !out_bf16)))
    return fail(MOE_ERR_INVALID, "moe_ep_forward: null pointer argument");
  const void* ptrs[] = {hidden, hidden_scale, w13_packed, w13_scale, w2_packed, w2_scale, logits, bias, out_bf16, workspace};
  for (const void* q : ptrs)
    if (!aligned16(q)) return fail(MOE_ERR_INVALID, "moe_ep_forward: every tensor must be 16-byte aligned");
  const EpLayout& L = c->L;
  const Workspace ws = make_workspace(L.r_cap, L.e_rank);
  const EpSourceWs sw = make_ep_source_ws(ws.total, L.t_max);
  if (workspace_bytes < sw.total)
    return fail(MOE_ERR_WORKSPACE, "workspace too small: need " + std::to_string(sw.total) + " bytes");
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return fail(MOE_ERR_INVALID, "moe_ep_forward: workspace must be 256-byte aligned");
  int dev = -1;
  if (int rc = cuda_check(cudaGetDevice(&dev), "cudaGetDevice")) return rc;
  if (dev != c->device) return fail(MOE_ERR_INVALID, "moe_ep_forward: current device differs from the context's");
  DeviceInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* W = static_cast<uint8_t*>(workspace);
  uint8_t* me = c->local;
  int* topk_idx = reinterpret_cast<int*>(W + ws.topk_idx);
  float* topk_w = reinterpret_cast<float*>(W + ws.topk_w);
  int* dense_base = reinterpret_cast<int*>(W + ws.dense_base);
  int* counts = ep_at<int>(me, L.counts);
  uint8_t* a_tiled = W + ws.a_tiled;
  float* a_scale = reinterpret_cast<float*>(W + ws.a_scale);
  uint8_t* c_hi = W + ws.c_hi;
  uint8_t* c_lo = W + ws.c_lo;
  float* c_scale = reinterpret_cast<float*>(W + ws.c_scale);
  float* partial = reinterpret_cast<float*>(W + ws.partial);
  int* tile_ready = reinterpret_cast<int*>(W + ws.tile_ready);
  Gemm1Args g1{a_tiled, a_scale, static_cast<const uint8_t*>(w13_packed), w13_scale, counts, L.r_cap,
               ws.tiles_max, L.e_rank, c_hi, c_lo, c_scale, tile_ready};
  Gemm2Args g2{c_hi, c_lo, c_scale, static_cast<const uint8_t*>(w2_packed), w2_scale, counts, L.r_cap,
               ws.tiles_max, L.e_rank, ep_at<float>(me, L.route_w), partial, dense_base, tile_ready,
               tile_ready + ws.tiles_max, nullptr, 0, nullptr, nullptr, 0};
  // Source side: local slot claims over all 256 experts (route_kernel with E_local = 256).
  int* local_counts = reinterpret_cast<int*>(W + sw.local_counts);
  int* reserve_base = reinterpret_cast<int*>(W + sw.base);
  int* token_nr = reinterpret_cast<int*>(W + sw.token_nr);
  int* token_route = reinterpret_cast<int*>(W + sw.token_route);
  int* route_token = reinterpret_cast<int*>(W + sw.route_token);
  float* route_w = reinterpret_cast<float*>(W + sw.route_w);
  auto mark = [&](int i) {
    if (events != nullptr) cudaEventRecord(static_cast<cudaEvent_t>(events[i]), st);
  };
  mark(0);
  if (int rc = cuda_check(cudaMemsetAsync(local_counts, 0, sizeof(int) * E_GLOBAL, st), "memset local counts"))
    return rc;
  if (T > 0)
    route_kernel<<<(T + 7) / 8, 256, 0, st>>>(logits, bias, T, routed_scaling_factor, 0, E_GLOBAL, topk_idx, topk_w,
                                              local_counts, token_nr, token_route, route_token, route_w);
  mark(1);
  ep_reserve_kernel<<<1, 256, 0, st>>>(c->peers, L, c->rank, local_counts, reserve_base);
  // Two warps (tokens) per block, so small per-rank batches still spread their peer stores
  // over every SM.
  ep_dispatch_kernel<<<grid_for(static_cast<size_t>(T), 2, d->num_sms * 32), 64, 0, st>>>(
      c->peers, L, c->rank, T, static_cast<const uint8_t*>(hidden), hidden_scale, token_nr, token_route, route_w,
      reserve_base);
  mark(2);
  ep_barrier_kernel<<<1, 32, 0, st>>>(c->peers, L.arrive, L.epoch, c->rank, L.world, 1);
  mark(3);
  const size_t route_max = static_cast<size_t>(L.r_cap) * (L.e_rank < TOP_K ? L.e_rank : TOP_K);
  if (int rc = cuda_check(launch_programmatic(gather_kernel, grid_for(route_max, 8, d->num_sms * 8), 256, 0, st,
                                              static_cast<const uint8_t*>(me + L.recv_rows),
                                              static_cast<const float*>(ep_at<float>(me, L.recv_scale)), L.r_cap,
                                              static_cast<const int*>(counts), L.e_rank,
                                              static_cast<const int*>(ep_at<int>(me, L.route_token)), ws.tiles_max,
                                              a_tiled, a_scale, tile_ready),
                          "gather launch"))
    return rc;
  mark(4);
  if (int rc = cuda_check(launch_programmatic(gemm1_swiglu_kernel,
                                              grid_for(static_cast<size_t>(ws.tiles_max) * G1_NT, 1, d->num_sms),
                                              G1_THREADS, G1_SMEM, st, g1),
                          "gemm1 launch"))
    return rc;
  mark(5);
  if (int rc = cuda_check(launch_gemm2(g2, grid_for(static_cast<size_t>(ws.tiles_max) * G2_NT, 1, d->num_sms), st),
                          "gemm2 launch"))
    return rc;
  mark(6);
  ep_combine_send_kernel<<<grid_for(static_cast<size_t>(L.r_cap), 1, d->num_sms * 4), COMBINE_THREADS, 0, st>>>(
      c->peers, L, c->rank, partial, dense_base);
  if (int rc = cuda_check(cudaMemsetAsync(counts, 0, sizeof(int) * L.e_rank, st), "memset counts")) return rc;
  mark(7);
  ep_barrier_kernel<<<1, 32, 0, st>>>(c->peers, L.done, L.epoch, c->rank, L.world, 0);
  mark(8);
  if (T > 0)
    if (int rc = cuda_check(launch_programmatic(ep_final_combine_kernel, T, COMBINE_THREADS, 0, st,
                                                static_cast<const uint8_t*>(me), L, T,
                                                static_cast<const int*>(topk_idx),
                                                static_cast<__nv_bfloat16*>(out_bf16)),
                            "final combine launch"))
      return rc;
  mark(9);
  return cuda_check(cudaGetLastError(), "moe_ep_forward launch");
}

}  // namespace

extern "C" {

int moe_forward(const void* hidden, const float* hidden_scale, const void* w13_packed,
                const float* w13_scale, const void* w2_packed, const float* w2_scale,
                const float* logits, const float* bias, float routed_scaling_factor,
                int local_expert_offset, int T, int E_local, void* out_bf16, void* workspace,
                size_t workspace_bytes, void* stream) {
  return forward_impl(hidden, hidden_scale, w13_packed, w13_scale, w2_packed, w2_scale, logits, bias,
                      routed_scaling_factor, local_expert_offset, T, E_local, out_bf16, workspace,
                      workspace_bytes, stream, nullptr);
}

int moe_forward_f32(const void* hidden, const float* hidden_scale, const void* w13_packed,
                    const float* w13_scale, const void* w2_packed, const float* w2_scale,
                    const float* logits, const float* bias, float routed_scaling_factor,
                    int local_expert_offset, int T, int E_local, float* out_f32, void* workspace,
                    size_t workspace_bytes, void* stream) {
  return forward_impl(hidden, hidden_scale, w13_packed, w13_scale, w2_packed, w2_scale, logits, bias,
                      routed_scaling_factor, local_expert_offset, T, E_local, out_f32, workspace,
                      workspace_bytes, stream, nullptr, true);
}

int moe_shared_expert_forward(const void* hidden, const float* hidden_scale, const void* w13_packed,
                              const float* w13_scale, const void* w2_packed, const float* w2_scale, int T,
                              void* out, int out_fp32, void* workspace, size_t workspace_bytes, void* stream) {
  return forward_impl(hidden, hidden_scale, w13_packed, w13_scale, w2_packed, w2_scale, nullptr, nullptr, 1.0f,
                      0, T, 1, out, workspace, workspace_bytes, stream, nullptr, out_fp32 != 0, true);
}

int moe_forward_noalloc(const void* hidden, const float* hidden_scale, const void* w13_packed,
                        const float* w13_scale, const void* w2_packed, const float* w2_scale,
                        const float* logits, const float* bias, float routed_scaling_factor,
                        int local_expert_offset, int T, int E_local, void* out_bf16, void* stream) {
  if (T < 0) return fail(MOE_ERR_INVALID, "hidden must be [T, 7168]");
  if (E_local < 1 || E_local > E_GLOBAL) return fail(MOE_ERR_INVALID, "W13_packed must be [E_local, ...] with 1 <= E_local <= 256");
  if (T == 0) return MOE_OK;
  const size_t need = make_workspace(T, E_local).total;
  if (need > NOALLOC_SCRATCH_BYTES)
    return fail(MOE_ERR_WORKSPACE,
                "moe_forward_noalloc: T=" + std::to_string(T) + " with E_local=" + std::to_string(E_local) +
                    " needs " + std::to_string(need) + " bytes of scratch, more than the " +
                    std::to_string(NOALLOC_SCRATCH_BYTES) +
                    " bytes of the library's static scratch (enough for T <= 64 with 32 local "
                    "experts); call moe_forward with a workspace instead");
  DeviceInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  void* scratch = nullptr;
  if (int rc = noalloc_scratch(d, &scratch)) return rc;
  return forward_impl(hidden, hidden_scale, w13_packed, w13_scale, w2_packed, w2_scale, logits, bias,
                      routed_scaling_factor, local_expert_offset, T, E_local, out_bf16, scratch,
                      NOALLOC_SCRATCH_BYTES, stream, nullptr);
}

int moe_forward_profiled(const void* hidden, const float* hidden_scale, const void* w13_packed,
                         const float* w13_scale, const void* w2_packed, const float* w2_scale,
                         const float* logits, const float* bias, float routed_scaling_factor,
                         int local_expert_offset, int T, int E_local, void* out_bf16,
                         void* workspace, size_t workspace_bytes, void* stream,
                         void* const* events) {
  if (events == nullptr) return fail(MOE_ERR_INVALID, "moe_forward_profiled: events must not be null");
  return forward_impl(hidden, hidden_scale, w13_packed, w13_scale, w2_packed, w2_scale, logits, bias,
                      routed_scaling_factor, local_expert_offset, T, E_local, out_bf16, workspace,
                      workspace_bytes, stream, events);
}

int moe_route(const float* logits, const float* bias, float routed_scaling_factor, int T,
              int* topk_idx, float* topk_w, void* stream) {
  if (T < 0) return fail(MOE_ERR_INVALID, "logits must be [T, 256]");
  if (T == 0) return MOE_OK;
  if (!logits || !bias || !topk_idx || !topk_w) return fail(MOE_ERR_INVALID, "moe_route: null pointer argument");
  if (!aligned16(logits) || !aligned16(bias)) return fail(MOE_ERR_INVALID, "moe_route: logits and bias must be 16-byte aligned");
  route_kernel<<<(T + 7) / 8, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      logits, bias, T, routed_scaling_factor, 0, 0, topk_idx, topk_w, nullptr, nullptr, nullptr,
      nullptr, nullptr);
  return cuda_check(cudaGetLastError(), "route_kernel launch");
}

int moe_quantize_hidden(const void* hidden_bf16, int T, void* out_e4m3, float* out_scale, void* stream) {
  if (T < 0) return fail(MOE_ERR_INVALID, "moe_quantize_hidden: hidden must be [T, 7168]");
  if (T == 0) return MOE_OK;
  if (T > MAX_TOKENS) return fail(MOE_ERR_INVALID, "moe_quantize_hidden: T must be at most 65536");
  if (!hidden_bf16 || !out_e4m3 || !out_scale) return fail(MOE_ERR_INVALID, "moe_quantize_hidden: null pointer argument");
  if (!aligned16(hidden_bf16) || !aligned16(out_e4m3) || !aligned16(out_scale))
    return fail(MOE_ERR_INVALID, "moe_quantize_hidden: every tensor must be 16-byte aligned");
  DeviceInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  const size_t warps = static_cast<size_t>(T) * (HB / QB_PER_WARP);
  quantize_hidden_kernel<<<grid_for(warps, 8, d->num_sms * 8), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(hidden_bf16), T, static_cast<uint8_t*>(out_e4m3), out_scale);
  return cuda_check(cudaGetLastError(), "quantize_hidden launch");
}

size_t moe_gate_packed_bytes(void) { return GATE_PACKED_BYTES; }

int moe_pack_gate(const void* w_gate_bf16, void* gate_packed, void* stream) {
  if (!w_gate_bf16 || !gate_packed) return fail(MOE_ERR_INVALID, "moe_pack_gate: null pointer argument");
  if (!aligned16(w_gate_bf16) || !aligned16(gate_packed))
    return fail(MOE_ERR_INVALID, "moe_pack_gate: W_gate and the packed buffer must be 16-byte aligned");
  DeviceInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  pack_gate_kernel<<<grid_for(static_cast<size_t>(E_GLOBAL) * H * 2 / 16, 256, d->num_sms * 8), 256, 0,
                     static_cast<cudaStream_t>(stream)>>>(static_cast<const uint8_t*>(w_gate_bf16),
                                                           static_cast<uint8_t*>(gate_packed));
  return cuda_check(cudaGetLastError(), "pack_gate_kernel launch");
}

int moe_gate_quantize(const void* hidden_bf16, const void* gate_packed, int T, float* logits,
                      void* out_e4m3, float* out_scale, void* stream) {
  if (T < 0) return fail(MOE_ERR_INVALID, "moe_gate_quantize: hidden must be [T, 7168]");
  if (T == 0) return MOE_OK;
  if (T > MAX_TOKENS) return fail(MOE_ERR_INVALID, "moe_gate_quantize: T must be at most 65536");
  if (!hidden_bf16 || !gate_packed || !logits || !out_e4m3 || !out_scale)
    return fail(MOE_ERR_INVALID, "moe_gate_quantize: null pointer argument");
  if (!aligned16(hidden_bf16) || !aligned16(gate_packed) || !aligned16(logits) || !aligned16(out_e4m3) ||
      !aligned16(out_scale))
    return fail(MOE_ERR_INVALID, "moe_gate_quantize: every tensor must be 16-byte aligned");
  DeviceInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  CUtensorMap map;
  if (int rc = hidden_bf16_map(hidden_bf16, T, &map)) return rc;
  const GateArgs args{static_cast<const uint8_t*>(gate_packed), T, logits, static_cast<uint8_t*>(out_e4m3),
                      out_scale};
  const dim3 grid(GATE_KS, (T + TILE_M - 1) / TILE_M);
  gate_quantize_kernel<<<grid, GATE_THREADS, GATE_SMEM, static_cast<cudaStream_t>(stream)>>>(map, args);
  return cuda_check(cudaGetLastError(), "gate_quantize launch");
}

int moe_synth_logits(const float* table, uint64_t seed, int T, int E, float* out, void* stream) {
  if (T < 0 || E < 0) return fail(MOE_ERR_INVALID, "moe_synth_logits: bad argument");
  const long n = static_cast<long>(T) * E;
  if (n == 0) return MOE_OK;
  if (!table || !out) return fail(MOE_ERR_INVALID, "moe_synth_logits: bad argument");
  synth_logits_kernel<<<grid_for(static_cast<size_t>(n), 256, 4096), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      table, seed, n, out);
  return cuda_check(cudaGetLastError(), "synth_logits launch");
}

int moe_synth_bias(const float* table, uint64_t seed, int E, float stddev, const int* hot_dev, int n_hot,
                   float hot_value, uint16_t* out_bf16, void* stream) {
  if (!table || !out_bf16 || E <= 0 || n_hot < 0 || (n_hot > 0 && !hot_dev))
    return fail(MOE_ERR_INVALID, "moe_synth_bias: bad argument");
  synth_bias_kernel<<<1, 256, 0, static_cast<cudaStream_t>(stream)>>>(table, seed, E, stddev, hot_dev, n_hot,
                                                                       hot_value, out_bf16);
  return cuda_check(cudaGetLastError(), "synth_bias launch");
}

int moe_synth_hidden(const float* table, uint64_t seed, int T, float stddev, void* hidden,
                     float* hidden_scale, void* stream) {
  if (T < 0) return fail(MOE_ERR_INVALID, "moe_synth_hidden: bad argument");
  if (T == 0) return MOE_OK;
  if (!table || !hidden || !hidden_scale) return fail(MOE_ERR_INVALID, "moe_synth_hidden: bad argument");
  const size_t warps = static_cast<size_t>(T) * HB;
  synth_hidden_kernel<<<grid_for(warps, 8, 8192), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      table, seed, T, stddev, static_cast<uint8_t*>(hidden), hidden_scale);
  return cuda_check(cudaGetLastError(), "synth_hidden launch");
}

int moe_synth_w13(const float* table, uint64_t seed, int e0, int E, float stddev, void* w13,
                  float* w13_scale, void* stream) {
  if (!table || !w13 || !w13_scale || E <= 0 || e0 < 0) return fail(MOE_ERR_INVALID, "moe_synth_w13: bad argument");
  const int blocks = E * (G1N / 128) * (H / 128);
  synth_weight_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      table, seed, SYN_W13, e0, G1N, H, stddev, static_cast<uint8_t*>(w13), w13_scale);
  return cuda_check(cudaGetLastError(), "synth_w13 launch");
}

int moe_synth_w2(const float* table, uint64_t seed, int e0, int E, float stddev, void* w2,
                 float* w2_scale, void* stream) {
  if (!table || !w2 || !w2_scale || E <= 0 || e0 < 0) return fail(MOE_ERR_INVALID, "moe_synth_w2: bad argument");
  const int blocks = E * (H / 128) * (I / 128);
  synth_weight_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      table, seed, SYN_W2, e0, H, I, stddev, static_cast<uint8_t*>(w2), w2_scale);
  return cuda_check(cudaGetLastError(), "synth_w2 launch");
}


size_t moe_ep_symmetric_bytes(int world, int t_rank_max, int e_rank) {
  if (ep_check_shape(world, t_rank_max, e_rank) != MOE_OK) return 0;
  return make_ep_layout(world, t_rank_max, e_rank).total;
}

size_t moe_ep_workspace_bytes(int world, int t_rank_max, int e_rank) {
  if (ep_check_shape(world, t_rank_max, e_rank) != MOE_OK) return 0;
  return make_ep_source_ws(make_workspace(world * t_rank_max, e_rank).total, t_rank_max).total;
}

int moe_ep_create(int rank, int world, int t_rank_max, int e_rank, const int* placement, void** ctx,
                  void* ipc_handle) {
  if (ctx == nullptr || ipc_handle == nullptr) return fail(MOE_ERR_INVALID, "moe_ep_create: null pointer argument");
  *ctx = nullptr;
  if (int rc = ep_check_shape(world, t_rank_max, e_rank)) return rc;
  if (rank < 0 || rank >= world) return fail(MOE_ERR_INVALID, "moe_ep_create: rank must be in [0, world)");
  // Placement table: global expert -> (owner << 16) | local index; -1 without an owner.
  int place[E_GLOBAL];
  for (int g = 0; g < E_GLOBAL; ++g) place[g] = -1;
  for (int i = 0; i < world * e_rank; ++i) {
    const int g = placement ? placement[i] : i;
    if (g < 0 || g >= E_GLOBAL || place[g] != -1)
      return fail(MOE_ERR_INVALID, "moe_ep_create: placement must list world * e_rank distinct experts in [0, 256)");
    place[g] = ((i / e_rank) << 16) | (i % e_rank);
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == MOE_EP_HANDLE_BYTES, "IPC handle size");
  EpCtx* c = new EpCtx();
  c->rank = rank;
  c->world = world;
  c->L = make_ep_layout(world, t_rank_max, e_rank);
  int rc = cuda_check(cudaGetDevice(&c->device), "cudaGetDevice");
  if (!rc) rc = cuda_check(cudaMalloc(&c->local, c->L.total), "cudaMalloc(symmetric buffer)");
  if (!rc) rc = cuda_check(cudaMemset(c->local, 0, c->L.total), "cudaMemset(symmetric buffer)");
  if (!rc)
    rc = cuda_check(cudaMemcpy(c->local + c->L.place, place, sizeof(place), cudaMemcpyHostToDevice),
                    "cudaMemcpy(placement)");
  cudaIpcMemHandle_t h{};
  if (!rc) rc = cuda_check(cudaIpcGetMemHandle(&h, c->local), "cudaIpcGetMemHandle");
  if (rc) {
    if (c->local) cudaFree(c->local);
    delete c;
    return rc;
  }
  std::memcpy(ipc_handle, &h, sizeof(h));
  *ctx = c;
  return MOE_OK;
}

int moe_ep_connect(void* ctx, const void* handles) {
  EpCtx* c = static_cast<EpCtx*>(ctx);
  if (c == nullptr || handles == nullptr) return fail(MOE_ERR_INVALID, "moe_ep_connect: null pointer argument");
  if (c->connected) return fail(MOE_ERR_INVALID, "moe_ep_connect: already connected");
  const uint8_t* hb = static_cast<const uint8_t*>(handles);
  for (int d = 0; d < c->world; ++d) {
    if (d == c->rank) {
      c->peers.base[d] = c->local;
      continue;
    }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, hb + static_cast<size_t>(d) * MOE_EP_HANDLE_BYTES, sizeof(h));
    void* p = nullptr;
    if (int rc = cuda_check(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle")) {
      for (int k = 0; k < d; ++k)
        if (c->opened[k]) {
          cudaIpcCloseMemHandle(c->peers.base[k]);
          c->opened[k] = false;
        }
      return rc;
    }
    c->peers.base[d] = static_cast<uint8_t*>(p);
    c->opened[d] = true;
  }
  c->connected = true;
  return MOE_OK;
}

int moe_ep_destroy(void* ctx) {
  EpCtx* c = static_cast<EpCtx*>(ctx);
  if (c == nullptr) return MOE_OK;
  int rc = MOE_OK;
  for (int d = 0; d < EP_MAX_RANKS; ++d)
    if (c->opened[d]) {
      int r = cuda_check(cudaIpcCloseMemHandle(c->peers.base[d]), "cudaIpcCloseMemHandle");
      if (!rc) rc = r;
    }
  if (c->local) {
    int r = cuda_check(cudaFree(c->local), "cudaFree(symmetric buffer)");
    if (!rc) rc = r;
  }
  delete c;
  return rc;
}

int moe_ep_forward(void* ctx, const void* hidden, const float* hidden_scale, const void* w13_packed,
                   const float* w13_scale, const void* w2_packed, const float* w2_scale,
                   const float* logits, const float* bias, float routed_scaling_factor, int T,
                   void* out_bf16, void* workspace, size_t workspace_bytes, void* stream) {
  return ep_forward_impl(static_cast<EpCtx*>(ctx), hidden, hidden_scale, w13_packed, w13_scale, w2_packed,
                         w2_scale, logits, bias, routed_scaling_factor, T, out_bf16, workspace,
                         workspace_bytes, stream, nullptr);
}

int moe_ep_forward_profiled(void* ctx, const void* hidden, const float* hidden_scale,
                            const void* w13_packed, const float* w13_scale, const void* w2_packed,
                            const float* w2_scale, const float* logits, const float* bias,
                            float routed_scaling_factor, int T, void* out_bf16, void* workspace,
                            size_t workspace_bytes, void* stream, void* const* events) {
  if (events == nullptr) return fail(MOE_ERR_INVALID, "moe_ep_forward_profiled: events must not be null");
  return ep_forward_impl(static_cast<EpCtx*>(ctx), hidden, hidden_scale, w13_packed, w13_scale, w2_packed,
                         w2_scale, logits, bias, routed_scaling_factor, T, out_bf16, workspace,
                         workspace_bytes, stream, events);
}

int moe_ep_info(void* ctx, int* out4) {
  EpCtx* c = static_cast<EpCtx*>(ctx);
  if (c == nullptr || out4 == nullptr) return fail(MOE_ERR_INVALID, "moe_ep_info: null pointer argument");
  out4[0] = c->rank;
  out4[1] = c->world;
  out4[2] = c->L.t_max;
  out4[3] = c->L.e_rank;
  return MOE_OK;
}

}  // extern "C"
