/*
 * Shared device definitions for the B200 (sm_100a) DeepSeek-V3/R1 FP8 MoE path:
 * fixed geometry, workspace layout, and thin inline-PTX wrappers for
 * mbarriers, bulk async copies and the 5th-generation tensor core (tcgen05).
 *
 * Geometry is the reference's fixed DeepSeek-V3/R1 shape
 * (reference/moe_ref.py:26-42, kernels/moe.cu:40-53).
 */
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <stdint.h>

namespace moe {

constexpr int H = 7168;          // hidden size
constexpr int I = 2048;          // expert intermediate size
constexpr int G1N = 2 * I;       // GEMM1 output columns (X1 | X2)
constexpr int E_GLOBAL = 256;    // routed experts
constexpr int N_GROUP = 8;       // expert groups
constexpr int GROUP_SIZE = 32;   // experts per group
constexpr int TOP_K = 8;         // experts per token
constexpr int TOPK_GROUP = 4;    // groups kept per token
constexpr int BLK = 128;         // FP8 scale block
constexpr int HB = H / BLK;      // 56 hidden blocks
constexpr int IB = I / BLK;      // 16 intermediate blocks
constexpr int G1B = G1N / BLK;   // 32 GEMM1 output blocks

constexpr int MAX_TOKENS = 65536;         // a route's slot is packed in 16 bits
constexpr int TILE_M = 128;              // routed rows per tile (UMMA M)
constexpr int TILE_BYTES = 128 * 128;    // one 128-row x 128-byte swizzled K block
constexpr int G1_NT = I / BLK;           // 16 GEMM1 column tiles (128 X1 + 128 X2 rows each)
constexpr int G2_NT = H / 256;           // 28 GEMM2 column tiles of 256 hidden rows

// Status bits reported through moe_get_status().
constexpr int ST_TIMEOUT_PRODUCER = 1;
constexpr int ST_TIMEOUT_MMA = 2;
constexpr int ST_TIMEOUT_EPILOGUE = 4;
constexpr int ST_BAD_INDEX = 8;
constexpr int ST_EP_TIMEOUT = 16;        // an expert-parallel barrier gave up waiting for a peer

// A bounded wait gives up after this long and reports ST_TIMEOUT_* / ST_EP_TIMEOUT. The limit
// is a device variable (one per device) so a test can shorten it through moe_set_wait_limit_ns;
// every wait reads it once when it starts.
constexpr unsigned long long WAIT_LIMIT_DEFAULT_NS = 2000000000ull;  // 2 s
__device__ unsigned long long g_wait_limit_ns = WAIT_LIMIT_DEFAULT_NS;

// Device status word (one per device), read by moe_get_status().
__device__ int g_status = 0;

__device__ __forceinline__ unsigned long long wait_limit_ns() {
  return *static_cast<volatile unsigned long long*>(&g_wait_limit_ns);
}
__device__ __forceinline__ int status_now() { return *static_cast<volatile int*>(&g_status); }

// ------------------------------------------------------------------------------------------
// Basic helpers
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void report_status(int bits) { atomicOr(&g_status, bits); }

// System-scope flag accesses for the expert-parallel barriers (peer memory over NVLink).
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// GPU-scope release / acquire on a counter in global memory (GEMM1 -> GEMM2 tile hand-off).
__device__ __forceinline__ void red_release_add(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Order this thread's earlier generic-proxy accesses of global memory before its later
// async-proxy (bulk copy) accesses.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
// Programmatic dependent launch: allow the next kernel of the stream (launched with the
// programmatic-serialization attribute) to be scheduled before this grid completes.
__device__ __forceinline__ void allow_dependent_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
// Wait until the grids this one depends on (the previous kernel of the stream) have completed and
// their memory operations are visible; returns at once for a normally launched kernel.
__device__ __forceinline__ void wait_prerequisite_grids() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Routing metadata is produced on the device; a consumer never trusts it for addressing.
__device__ __forceinline__ int clamp_tiles(int n, int tiles_max) {
  if (n < 0 || n > tiles_max) {
    report_status(ST_BAD_INDEX);
    return n < 0 ? 0 : tiles_max;
  }
  return n;
}
__device__ __forceinline__ int checked_expert(int e, int E_local) {
  if (e < 0 || e >= E_local) {
    report_status(ST_BAD_INDEX);
    return 0;
  }
  return e;
}

// ------------------------------------------------------------------------------------------
// mbarrier
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Test for completion of the phase with the given parity. When it is not complete the thread
// is suspended in hardware (no issue slots used) until it completes or about SUSPEND_NS pass,
// so waiting warps do not slow down the warps that share their SM sub-partition.
constexpr uint32_t SUSPEND_NS = 1000000;  // 1 ms per try; the caller bounds the total wait
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "n"(SUSPEND_NS)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity to complete. Returns false when the
// CTA-wide abort flag is raised or when the wait limit elapses (then it raises the flag and
// records `who` in g_status). Never spins forever.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          int who) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer(), limit = wait_limit_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer() - t0 > limit) {
      *abort_flag = 1;
      report_status(who);
      return false;
    }
  }
}

// Bounded wait that ignores the abort flag: used on teardown to let in-flight async copies
// and MMAs land before the CTA releases its shared memory and TMEM.
__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity) {
  const unsigned long long t0 = globaltimer(), limit = wait_limit_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > limit) return false;
  }
  return true;
}

// After a warp-wide wait has seen a phase complete: every lane observes the completion itself
// (an acquire of its own) before it reads data that the async proxy wrote under that barrier.
// The phase cannot advance meanwhile, because the slot is released only after these reads.
__device__ __forceinline__ void mbar_observe(uint64_t* bar, uint32_t parity) { (void)mbar_try_wait(bar, parity); }

// Non-suspending poll of an mbarrier phase.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait by polling, for the hand-offs on a GEMM's critical path (stage -> MMA -> epilogue ->
// MMA): a suspended try_wait wakes measurably later after the phase completes. The abort flag and
// the clock are checked every 64 polls. Same limits and error reporting as mbar_wait.
__device__ __forceinline__ bool mbar_wait_spin(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int who) {
  if (mbar_test_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer(), limit = wait_limit_ns();
  for (uint32_t n = 1;; ++n) {
    if (mbar_test_wait(bar, parity)) return true;
    if ((n & 63u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer() - t0 > limit) {
        *abort_flag = 1;
        report_status(who);
        return false;
      }
    }
  }
}

// Warp-uniform bounded wait: lane 0 waits, the result is broadcast to the warp.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity,
                                               volatile int* abort_flag, int who, bool spin = false) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0)
    ok = (spin ? mbar_wait_spin(bar, parity, abort_flag, who) : mbar_wait(bar, parity, abort_flag, who)) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  __syncwarp();
  return ok != 0;
}

// ------------------------------------------------------------------------------------------
// Bulk async copy global -> shared (no tensor map, no multicast)
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gsrc, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Same with an L2 eviction policy (policy from createpolicy).
__device__ __forceinline__ void bulk_g2s_hint(void* smem_dst, const void* gsrc, uint32_t bytes,
                                              uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], "
      "[%1], %2, [%3], %4;" ::"r"(smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
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

// ------------------------------------------------------------------------------------------
// tcgen05 (TMEM + UMMA)
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Arrive (once) on `bar` when every tcgen05 op issued so far by this thread has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// D(tmem) (+)= A(smem desc) x B(smem desc)^T, FP8 e4m3 inputs, fp32 accumulate.
__device__ __forceinline__ void tc_mma_f8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Load 32 consecutive fp32 columns of this thread's TMEM lane and wait for completion.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Two floats rounded to bf16 (nearest even), packed low word first.
__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

// acc[i] += v[i] * f for 32 values, as 16 packed fp32x2 FMAs (each lane IEEE fmaf).
__device__ __forceinline__ void fma32_scaled(float* acc, const float (&v)[32], float f) {
  uint64_t ff;
  asm("mov.b64 %0, {%1, %1};" : "=l"(ff) : "f"(f));
#pragma unroll
  for (int i = 0; i < 32; i += 2) {
    uint64_t a, b;
    asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "f"(acc[i]), "f"(acc[i + 1]));
    asm("mov.b64 %0, {%1, %2};" : "=l"(b) : "f"(v[i]), "f"(v[i + 1]));
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(a) : "l"(b), "l"(ff));
    asm("mov.b64 {%0, %1}, %2;" : "=f"(acc[i]), "=f"(acc[i + 1]) : "l"(a));
  }
}

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle, 8-row atoms of
// 1024 bytes (SBO), version 1 (sm_100). `saddr` is the shared-window byte address of the
// first row of the tile plus the K offset (multiples of 32 bytes inside the atom).
__device__ __forceinline__ uint64_t sdesc_k_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(1u) << 16;            // leading byte offset (unused, K-major SW128)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;    // stride byte offset: 8 rows x 128 B
  d |= static_cast<uint64_t>(1u) << 46;            // descriptor version for tcgen05
  d |= static_cast<uint64_t>(2u) << 61;            // SWIZZLE_128B
  return d;
}

// Instruction descriptor for kind::f8f6f4: e4m3 x e4m3 -> f32, both K-major.
__host__ __device__ constexpr uint32_t idesc_e4m3_f32(int m, int n) {
  return (1u << 4)                                   // D format f32
         | (0u << 7) | (0u << 10)                    // A, B = e4m3
         | (static_cast<uint32_t>(n >> 3) << 17)     // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);    // M / 16
}

// Byte offset of (row, byte k) inside a 128-row x 128-byte K-major SW128 tile.
__host__ __device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t k) {
  return row * 128u + ((((k >> 4) ^ (row & 7u)) << 4) | (k & 15u));
}

// Register re-balancing between warpgroups (all 128 threads of a warpgroup execute it).
template <int N>
__device__ __forceinline__ void regs_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void regs_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

// GEMM CTA shape shared by both tcgen05 kernels: warpgroup 0 = producer warp, MMA warp and
// two idle warps (56 registers each); warpgroups 1-2 = eight epilogue warps (224 registers).
// 128 * 56 + 256 * 224 = 64512 = 384 * 168, the launch allocation at 168 registers/thread;
// the host refuses to launch if ptxas gave the kernel fewer (setmaxnreg.inc would stall).
constexpr int GEMM_THREADS = 384;
constexpr int REGS_CTRL = 56;
constexpr int REGS_EPI = 224;
constexpr int GEMM_LAUNCH_REGS_MIN = (128 * REGS_CTRL + 256 * REGS_EPI + GEMM_THREADS - 1) / GEMM_THREADS;

// Named barrier among `nthreads` threads (ids 1..15; id 0 is __syncthreads) that also
// returns the OR of `pred` over the participants, so a decision to stop is uniform.
__device__ __forceinline__ bool named_bar_or(int id, int nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred)), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ uint8_t* align_1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) &
                                    ~static_cast<uintptr_t>(1023));
}

// ------------------------------------------------------------------------------------------
// Workspace layout of one moe_forward call (all offsets 1024-byte aligned).
// ------------------------------------------------------------------------------------------
struct Workspace {
  size_t counts;       // int32 [E_local]              routes per local expert (zeroed per call)
  size_t dense_base;   // int32 [E_local + 1]          routes of experts < e (written by GEMM2)
  size_t topk_idx;     // int32 [T, 8]                 selected global experts
  size_t topk_w;       // fp32  [T, 8]                 routing weights
  size_t token_nr;     // int32 [T]                    local routes per token
  size_t token_route;  // int32 [T, 8]                 (le << 16 | slot), ascending le
  size_t route_token;  // int32 [E_local, T]           token of each expert's slot
  size_t route_w;      // fp32  [E_local, T]           routing weight of each expert's slot
  size_t a_tiled;      // u8    [tiles_max, 56, 128, 128] routed hidden rows, SW128 tile images
  size_t a_scale;      // fp32  [tiles_max, 56, 128]   their per-128 block scales
  size_t c_hi;         // u8    [tiles_max, 16, 128, 128] SwiGLU output, e4m3 high part
  size_t c_lo;         // u8    [tiles_max, 16, 128, 128] e4m3 residual
  size_t c_scale;      // fp32  [tiles_max, 16, 128]   per (row, 128-block) scale
  size_t partial;      // fp32  [routes_max / 128, 224, 128, 32] weighted expert output per local route,
                       //       route d's 32-column group g at partial_offset(d, 32 g)
  size_t tile_ready;   // int32 [tiles_max + 1]         GEMM1 column blocks of each tile whose C is stored;
                       //                               the last entry is GEMM2's unit queue
  size_t total;
  int tiles_max;
};

__host__ __device__ inline size_t ws_align(size_t x) { return (x + 1023) & ~static_cast<size_t>(1023); }

inline Workspace make_workspace(int T, int E_local) {
  Workspace w{};
  // Tiles: each active expert pads its rows up to a multiple of 128, and there are at most
  // min(E_local, routes) active experts.
  int kmax = E_local < TOP_K ? E_local : TOP_K;
  long long routes = static_cast<long long>(T) * kmax;
  long long active = routes < E_local ? routes : E_local;
  long long rows = routes + active * (TILE_M - 1);
  w.tiles_max = static_cast<int>((rows + TILE_M - 1) / TILE_M);
  size_t tiles = static_cast<size_t>(w.tiles_max);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off = ws_align(off + bytes);
    return o;
  };
  const size_t e = static_cast<size_t>(E_local > 0 ? E_local : 1);
  w.counts = take(sizeof(int) * e);
  w.dense_base = take(sizeof(int) * (e + 1));
  w.topk_idx = take(sizeof(int) * TOP_K * static_cast<size_t>(T));
  w.topk_w = take(sizeof(float) * TOP_K * static_cast<size_t>(T));
  w.token_nr = take(sizeof(int) * static_cast<size_t>(T));
  w.token_route = take(sizeof(int) * TOP_K * static_cast<size_t>(T));
  w.route_token = take(sizeof(int) * e * static_cast<size_t>(T));
  w.route_w = take(sizeof(float) * e * static_cast<size_t>(T));
  w.a_tiled = take(tiles * HB * TILE_BYTES);
  w.a_scale = take(sizeof(float) * tiles * HB * TILE_M);
  w.c_hi = take(tiles * IB * TILE_BYTES);
  w.c_lo = take(tiles * IB * TILE_BYTES);
  w.c_scale = take(sizeof(float) * tiles * IB * TILE_M);
  w.partial = take(sizeof(float) * ((static_cast<size_t>(T) * kmax + TILE_M - 1) / TILE_M) * TILE_M * H);
  w.tile_ready = take(sizeof(int) * (tiles + 1));
  w.total = off;
  return w;
}

// Layout of the weighted per-route rows (GEMM2 -> combine): dense route rows in blocks of 128, each
// block stored as 224 column groups of [128 rows][32 floats]. GEMM2's epilogue (one row per thread)
// writes each 128-byte group with four full-sector 256-bit stores, and the combine reads a row's
// group as one whole 128-byte line.
constexpr int PART_G = H / 32;
__host__ __device__ __forceinline__ size_t partial_offset(size_t d, int col) {
  return ((d / TILE_M * PART_G + static_cast<size_t>(col >> 5)) * TILE_M + d % TILE_M) * 32 + (col & 31);
}

// 8 consecutive fp32 values to global memory in one 256-bit store (32-byte aligned address).
// One 256-bit store of 8 words to a 32-byte aligned global address.
__device__ __forceinline__ void st_global_v8_u32(void* p, const uint32_t* v) {
  asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(v[0]), "r"(v[1]), "r"(v[2]),
               "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}
__device__ __forceinline__ void st_global_v8(float* p, const float* v) {
  asm volatile("st.global.v8.f32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "f"(v[0]), "f"(v[1]), "f"(v[2]),
               "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7])
               : "memory");
}

// ------------------------------------------------------------------------------------------
// Expert tile map. From the per-expert route counts (each expert's rows padded to 128-row
// tiles, experts in ascending order): tile_off[e] = first tile of expert e, dense_off[e] =
// number of routes of experts < e. Entry [E_local] holds the totals.
// ------------------------------------------------------------------------------------------
struct TileMap {
  int tile_off[E_GLOBAL + 1];
  int dense_off[E_GLOBAL + 1];
};

// Built by one full warp; the caller synchronises before use. A count outside [0, cap] is
// reported and clamped; counts whose totals exceed what the workspace was sized for
// (cap * min(8, E_local) routes, tiles_max tiles) are reported and replaced by an empty map,
// so corrupted counts can never address past the workspace.
__device__ __forceinline__ void build_tile_map(TileMap* tm, const int* __restrict__ counts,
                                               int E_local, int cap, int tiles_max) {
  const int lane = threadIdx.x & 31;
  int c[8], tiles = 0, rows = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int e = lane * 8 + i;
    int v = e < E_local ? counts[e] : 0;
    if (v < 0 || v > cap) {
      report_status(ST_BAD_INDEX);
      v = v < 0 ? 0 : cap;
    }
    c[i] = v;
    tiles += (v + TILE_M - 1) / TILE_M;
    rows += v;
  }
  int t_incl = tiles, r_incl = rows;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int tn = __shfl_up_sync(0xffffffffu, t_incl, o);
    const int rn = __shfl_up_sync(0xffffffffu, r_incl, o);
    if (lane >= o) {
      t_incl += tn;
      r_incl += rn;
    }
  }
  int t = t_incl - tiles, r = r_incl - rows;
  const int all_tiles = __shfl_sync(0xffffffffu, t_incl, 31);
  const int all_rows = __shfl_sync(0xffffffffu, r_incl, 31);
  const long long rows_max = static_cast<long long>(cap) * (E_local < TOP_K ? E_local : TOP_K);
  if (all_tiles > tiles_max || all_rows > rows_max) {
    if (lane == 0) report_status(ST_BAD_INDEX);
    t = r = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) c[i] = 0;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int e = lane * 8 + i;
    if (e <= E_local) {
      tm->tile_off[e] = t;
      tm->dense_off[e] = r;
    }
    t += (c[i] + TILE_M - 1) / TILE_M;
    r += c[i];
  }
  if (lane == 31 && E_local == E_GLOBAL) {
    tm->tile_off[E_GLOBAL] = t;
    tm->dense_off[E_GLOBAL] = r;
  }
}

// Expert of tile t: the e with tile_off[e] <= t < tile_off[e + 1] (empty experts own no tile).
__device__ __forceinline__ int tile_expert(const TileMap* tm, int E_local, int t) {
  int lo = 0, hi = E_local;  // invariant: tile_off[lo] <= t < tile_off[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (tm->tile_off[mid] <= t) lo = mid; else hi = mid;
  }
  return lo;
}

}  // namespace moe
