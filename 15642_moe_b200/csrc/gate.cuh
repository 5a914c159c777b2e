/*
 * MoE prologue: the DeepSeek-V3 gate (router) GEMM and the FP8 activation quantiser in one
 * pass over the bf16 hidden states, the two consumers of the same normalised hidden rows x:
 *
 *   logits[t, e] = sum_k x[t, k] * W_gate[e, k]        fp32 [T, 256], the routing_logits input
 *                                                       of moe_forward (reference/moe_ref.py:5-6)
 *   codes, scale = quantise(x)                          e4m3 [T, 7168] + fp32 [56, T] block-major,
 *                                                       the hidden_states / hidden_states_scale
 *                                                       inputs (reference/moe_ref.py:44-45)
 *
 * The reference takes both as given inputs; this is the step that produces them. x and W_gate
 * are bf16, so every product is exact in fp32 and the tensor core's fp32 accumulation (bf16
 * tcgen05.mma, kind::f16) computes the same dot products as a fp32 GEMM of the upcast operands
 * up to the order of the additions.
 *
 * Work split: one cluster of GATE_KS CTAs per 128-token tile, CTA q owning hidden blocks
 * [14q, 14q + 14). Each CTA:
 *   warp 0      x producer: per 128-column block, two TMA tile loads (128 tokens x 64 columns,
 *               128-byte swizzle, zero fill past T) into a ring of GATE_A_STAGES blocks
 *   warp 1      W_gate producer: one bulk copy of a pre-swizzled 64-column half (256 experts) into
 *               a ring of GATE_B_STAGES halves (L2-resident: every token tile reads the same 3.7 MB)
 *   warp 2      MMA: 8 x (M=128, N=256, K=16) per block into one 256-column TMEM accumulator
 *   warps 3-18  quantiser: 4 threads per token row (32 columns each) read the same shared tile the
 *               MMA reads, release it, and write the e4m3 codes and the block scale; after the
 *               last block they copy the accumulator to shared memory
 * The x ring is the deep one: it keeps 4 blocks (128 KB) of HBM reads in flight per SM, and the
 * MMA's time on a block is not on the path that refills it. After the last block the cluster
 * sums its GATE_KS partial accumulators through distributed shared memory in K-slice order (CTA q
 * reduces rows [32q, 32q + 32)), so every token's logits are computed the same way whatever T is
 * and wherever the token sits in the batch.
 *
 * Quantisation is the convention of the benchmark configurations (bit-identical to
 * quantize_hidden_kernel): scale = amax / 448 (IEEE division, 1 for an all-zero block),
 * code = e4m3(x / scale) rounded to nearest even, saturated to +-448. x / scale is the correctly
 * rounded quotient from y = RN(1 / scale) by Markstein's method with two corrections (quotient2 in
 * quant.cuh), so the codes equal those of a true division. The block scale and y come from
 * 128-entry tables indexed by the amax mantissa (see block_scale). Blocks whose amax is below
 * 2^-80 (where the remainder could underflow) divide directly, out of line.
 */
#pragma once
#include "moe_common.cuh"
#include "quant.cuh"

#include <cuda.h>

namespace moe {

constexpr int GATE_KS = 4;                          // K slices per token tile (CTAs per cluster)
constexpr int GATE_KB = HB / GATE_KS;               // 14 hidden blocks per CTA
constexpr int GATE_A_ATOM = 128 * 128;              // 128 tokens x 64 bf16 columns (16 KB)
constexpr int GATE_A_BYTES = 2 * GATE_A_ATOM;       // one 128-column block of 128 tokens
constexpr int GATE_B_ATOM = E_GLOBAL * 128;         // 256 experts x 64 bf16 columns (32 KB)
constexpr int GATE_B_BYTES = 2 * GATE_B_ATOM;       // one 128-column block of W_gate
constexpr int GATE_A_STAGES = 4;                     // x ring: 4 blocks of 128 tokens (128 KB)
constexpr int GATE_B_STAGES = 3;                     // W_gate ring: 3 halves of 64 columns (96 KB)
constexpr int GATE_QWARPS = 16;
constexpr int GATE_QWARP0 = 3;                       // warps 0-2: x producer, W_gate producer, MMA
constexpr int GATE_THREADS = 32 * (GATE_QWARP0 + GATE_QWARPS);
constexpr int GATE_CTRL_BYTES = 2048;
constexpr int GATE_RING_BYTES = GATE_A_STAGES * GATE_A_BYTES + GATE_B_STAGES * GATE_B_ATOM;
constexpr int GATE_SMEM = GATE_RING_BYTES + GATE_CTRL_BYTES + 1024;
constexpr size_t GATE_PACKED_BYTES = static_cast<size_t>(HB) * GATE_B_BYTES;  // 3,670,016
constexpr int GATE_RED_ROW = E_GLOBAL * 4;          // bytes per accumulator row in shared memory
static_assert(TILE_M * GATE_RED_ROW <= GATE_A_STAGES * GATE_A_BYTES, "reduction buffer does not fit");
static_assert(GATE_SMEM <= 232448, "shared memory above the per-CTA limit");
static_assert(HB % GATE_KS == 0 && TILE_M % GATE_KS == 0, "bad K split");

struct GateArgs {
  const uint8_t* gate_packed;  // [56 blocks][2 halves][256 experts][128 B] (pack_gate_kernel)
  int T;
  float* logits;               // [T, 256]
  uint8_t* codes;              // [T, 7168] e4m3
  float* scale;                // [56, T]
};

struct GateCtrl {
  uint64_t a_full[GATE_A_STAGES];
  uint64_t a_empty[GATE_A_STAGES];
  uint64_t b_full[GATE_B_STAGES];
  uint64_t b_empty[GATE_B_STAGES];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort_flag;
  float scale_tab[128];   // RN((1 + f/128) / 448): block scale for amax mantissa f, exponent 0
  float recip_tab[128];   // RN(1 / scale_tab[f])
};
static_assert(sizeof(GateCtrl) <= GATE_CTRL_BYTES, "control block too large");

// W_gate bf16 [256, 7168] -> the shared-memory images the MMA reads: per 128-column block kb,
// two K-major 128-byte-swizzled halves of 256 rows x 64 columns. One thread per 16-byte chunk.
__global__ void __launch_bounds__(256) pack_gate_kernel(const uint8_t* __restrict__ w,
                                                        uint8_t* __restrict__ out) {
  constexpr int CHUNKS_PER_ROW = H * 2 / 16;  // 896
  const int total = E_GLOBAL * CHUNKS_PER_ROW;
  for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += gridDim.x * blockDim.x) {
    const int r = idx / CHUNKS_PER_ROW, qk = idx - r * CHUNKS_PER_ROW;
    const int kb = qk >> 4, half = (qk >> 3) & 1, c = qk & 7;
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(w + static_cast<size_t>(r) * H * 2) + qk);
    *reinterpret_cast<uint4*>(out + static_cast<size_t>(kb) * GATE_B_BYTES + half * GATE_B_ATOM + r * 128 +
                              ((c ^ (r & 7)) << 4)) = v;
  }
}

// ---- PTX wrappers used only here ---------------------------------------------------------

// 2-D tiled TMA load (no multicast) with an L2 policy; x is the column, y the row coordinate.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// D(tmem) (+)= A(smem desc) x B(smem desc)^T, bf16 inputs, fp32 accumulate.
__device__ __forceinline__ void tc_mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Instruction descriptor for kind::f16: bf16 x bf16 -> f32, both K-major.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int m, int n) {
  return (1u << 4)                                   // D format f32
         | (1u << 7) | (1u << 10)                    // A, B = bf16
         | (static_cast<uint32_t>(n >> 3) << 17)     // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);    // M / 16
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Every thread of every CTA in the cluster; orders shared-memory writes before the barrier
// with reads after it, cluster-wide.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_map(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}

__device__ __forceinline__ float4 ld_cluster_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// Block scale and its reciprocal from the bf16 bit pattern `mx` of the block's amax (sign
// cleared). For amax = (1 + f/128) 2^(E-127) with E >= 47, s = RN(amax / 448) and y = RN(1 / s)
// are the table entries for f scaled by 2^(E-127): scaling by a power of two commutes with
// rounding while the results stay normal, which holds for every E in [47, 254]. Returns false
// (s from a division, y unused) when amax < 2^-80 or amax = 0 (s = 1).
__device__ __forceinline__ bool block_scale(uint32_t mx, const GateCtrl* ctl, float& s, float& y) {
  const int E = static_cast<int>(mx >> 7);
  if (E >= 47) {
    const int f = static_cast<int>(mx & 0x7Fu), adj = (E - 127) << 23;
    s = __uint_as_float(__float_as_uint(ctl->scale_tab[f]) + adj);
    y = __uint_as_float(__float_as_uint(ctl->recip_tab[f]) - adj);
    return true;
  }
  s = mx ? __fdiv_rn(__uint_as_float(mx << 16), 448.0f) : 1.0f;
  y = 0.0f;
  return false;
}

struct Words16 {
  uint32_t v[16];
};
struct Codes8 {
  uint32_t v[8];
};

// Blocks whose amax is below 2^-80 (rare): IEEE division per value. Out of line and by value,
// so its code stays out of the quantiser's loop and the fast path keeps its operands in registers.
__device__ __noinline__ Codes8 quantise32_divide(Words16 w, float s) {
  Codes8 out;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    float2 q[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t u = w.v[2 * k + h];
      q[h] = make_float2(__fdiv_rn(__uint_as_float(u << 16), s), __fdiv_rn(__uint_as_float(u & 0xFFFF0000u), s));
    }
    out.v[k] = codes4(q[0], q[1], w.v[2 * k], w.v[2 * k + 1]);
  }
  return out;
}

// Quantise 32 bf16 values (16 words, two values per word, low half first) that share the block
// scale s (y = RN(1/s) when `fast`): returns 8 words of e4m3 codes in the same order. The sign
// of x is OR-ed into each code so that -0 codes as 0x80 (e4m3 is sign-magnitude; every other
// value already carries its sign through the quotient).
__device__ __forceinline__ void quantise32(const uint32_t (&w)[16], float s, float y, bool fast,
                                           uint32_t (&out)[8]) {
  if (!fast) {
    Words16 ww;
#pragma unroll
    for (int i = 0; i < 16; ++i) ww.v[i] = w[i];
    const Codes8 c = quantise32_divide(ww, s);
#pragma unroll
    for (int i = 0; i < 8; ++i) out[i] = c.v[i];
    return;
  }
  const uint64_t yy = f2_pack(y, y), ns = f2_pack(-s, -s);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    float2 q[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) q[h] = quotient2(bf16x2_to_f2(w[2 * k + h]), yy, ns);
    out[k] = codes4(q[0], q[1], w[2 * k], w[2 * k + 1]);
  }
}

// max(|a|, |b|) per bf16 half (the sign bit of each half is the XOR of the inputs' signs).
__device__ __forceinline__ uint32_t absmax_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

__global__ void __cluster_dims__(GATE_KS, 1, 1) __launch_bounds__(GATE_THREADS, 1)
    gate_quantize_kernel(const __grid_constant__ CUtensorMap x_map, const __grid_constant__ GateArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_1024(smem_raw);
  uint8_t* ring_a = smem;                                        // [4][2 halves][128 rows][128 B]
  uint8_t* ring_b = smem + GATE_A_STAGES * GATE_A_BYTES;         // [3][256 rows][128 B]
  GateCtrl* ctl = reinterpret_cast<GateCtrl*>(smem + GATE_RING_BYTES);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kb0 = static_cast<int>(blockIdx.x) * GATE_KB;  // cluster spans x: rank == blockIdx.x
  const int m0 = static_cast<int>(blockIdx.y) * TILE_M;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < GATE_A_STAGES; ++s) {
      mbar_init(&ctl->a_full[s], 1);
      mbar_init(&ctl->a_empty[s], 1 + GATE_QWARPS);
    }
#pragma unroll
    for (int s = 0; s < GATE_B_STAGES; ++s) {
      mbar_init(&ctl->b_full[s], 1);
      mbar_init(&ctl->b_empty[s], 1);
    }
    mbar_init(&ctl->mma_done, 1);
    ctl->abort_flag = 0;
    fence_mbar_init();
  }
  if (threadIdx.x < 128) {
    const float sc = __fdiv_rn(1.0f + static_cast<float>(threadIdx.x) * 0.0078125f, 448.0f);
    ctl->scale_tab[threadIdx.x] = sc;
    ctl->recip_tab[threadIdx.x] = __frcp_rn(sc);
  }
  if (warp == 2) {
    tmem_alloc(&ctl->tmem_base, E_GLOBAL);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  volatile int* abort_flag = &ctl->abort_flag;

  if (warp == 0) {
    // ---------------- x producer: two TMA boxes per 128-column block ----------------
    if (lane == 0) {
      const uint64_t pol_x = policy_evict_first();
      uint32_t it = 0;
      for (; it < GATE_KB && !*abort_flag; ++it) {
        const int s = it % GATE_A_STAGES;
        if (!mbar_wait(&ctl->a_empty[s], ((it / GATE_A_STAGES) & 1u) ^ 1u, abort_flag, ST_TIMEOUT_PRODUCER)) break;
        uint8_t* st = ring_a + s * GATE_A_BYTES;
        const int kb = kb0 + static_cast<int>(it);
        mbar_arrive_expect_tx(&ctl->a_full[s], GATE_A_BYTES);
        tma_load_2d(st, &x_map, kb * BLK, m0, &ctl->a_full[s], pol_x);
        tma_load_2d(st + GATE_A_ATOM, &x_map, kb * BLK + 64, m0, &ctl->a_full[s], pol_x);
      }
      if (*abort_flag) {
        // Let every copy in flight land before the CTA's shared memory is released.
        for (uint32_t i = 1; i <= GATE_A_STAGES && i <= it; ++i) {
          const uint32_t jt = it - i;
          mbar_wait_drain(&ctl->a_full[jt % GATE_A_STAGES], (jt / GATE_A_STAGES) & 1u);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- W_gate producer: one 32 KB bulk copy per 64-column half ----------------
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_last();
      uint32_t it = 0;
      for (; it < 2 * GATE_KB && !*abort_flag; ++it) {
        const int s = it % GATE_B_STAGES;
        if (!mbar_wait(&ctl->b_empty[s], ((it / GATE_B_STAGES) & 1u) ^ 1u, abort_flag, ST_TIMEOUT_PRODUCER)) break;
        mbar_arrive_expect_tx(&ctl->b_full[s], GATE_B_ATOM);
        bulk_g2s_hint(ring_b + s * GATE_B_ATOM,
                      p.gate_packed + static_cast<size_t>(kb0) * GATE_B_BYTES + static_cast<size_t>(it) * GATE_B_ATOM,
                      GATE_B_ATOM, &ctl->b_full[s], pol_w);
      }
      if (*abort_flag) {
        for (uint32_t i = 1; i <= GATE_B_STAGES && i <= it; ++i) {
          const uint32_t jt = it - i;
          mbar_wait_drain(&ctl->b_full[jt % GATE_B_STAGES], (jt / GATE_B_STAGES) & 1u);
        }
      }
    }
  } else if (warp == 2) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(128, E_GLOBAL);
      bool ok = true;
      for (uint32_t it = 0; it < GATE_KB && ok; ++it) {
        const int sa = it % GATE_A_STAGES;
        if (!mbar_wait(&ctl->a_full[sa], (it / GATE_A_STAGES) & 1u, abort_flag, ST_TIMEOUT_MMA)) break;
        const uint32_t a = smem_u32(ring_a + sa * GATE_A_BYTES);
#pragma unroll
        for (uint32_t half = 0; half < 2; ++half) {
          const uint32_t ib = 2 * it + half;
          const int sb = ib % GATE_B_STAGES;
          if (!mbar_wait(&ctl->b_full[sb], (ib / GATE_B_STAGES) & 1u, abort_flag, ST_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t b = smem_u32(ring_b + sb * GATE_B_ATOM);
#pragma unroll
          for (uint32_t kk = 0; kk < 4; ++kk)  // K = 16 bf16 = 32 bytes per MMA
            tc_mma_bf16(tmem, sdesc_k_sw128(a + half * GATE_A_ATOM + kk * 32), sdesc_k_sw128(b + kk * 32), idesc,
                        (it | half | kk) ? 1u : 0u);
          tc_commit(&ctl->b_empty[sb]);
        }
        if (ok) tc_commit(&ctl->a_empty[sa]);
      }
      // Arrives once every MMA issued above has completed (also after an abort).
      tc_commit(&ctl->mma_done);
    }
  } else {
    // ---------------- quantiser (warps 3..18) ----------------
    const int j = warp - GATE_QWARP0, rr = lane & 7, qq = lane >> 3;
    const int row = j * 8 + rr, t = m0 + row;
    const int half = qq >> 1, c0 = (qq & 1) * 4;
    bool aborted = false;
    for (uint32_t it = 0; it < GATE_KB; ++it) {
      const int s = it % GATE_A_STAGES;
      const uint32_t ph = (it / GATE_A_STAGES) & 1u;
      if (!mbar_wait_warp(&ctl->a_full[s], ph, abort_flag, ST_TIMEOUT_EPILOGUE)) {
        aborted = true;
        break;
      }
      mbar_try_wait(&ctl->a_full[s], ph);  // completed: gives this lane the acquire of the copies
      const uint8_t* a = ring_a + s * GATE_A_BYTES + half * GATE_A_ATOM + row * 128;
      uint32_t w[16];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint4 v = *reinterpret_cast<const uint4*>(a + (((c0 + c) ^ rr) << 4));
        w[4 * c] = v.x;
        w[4 * c + 1] = v.y;
        w[4 * c + 2] = v.z;
        w[4 * c + 3] = v.w;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl->a_empty[s]);
      // amax of |x| over the block's 128 columns: non-negative bf16 values order like their
      // bit patterns, so a packed 16-bit unsigned max finds it.
      uint32_t m2 = absmax_bf16x2(w[0], w[1]);
#pragma unroll
      for (int k = 2; k < 16; ++k) m2 = absmax_bf16x2(m2, w[k]);
      m2 &= 0x7FFF7FFFu;
      uint32_t mx = max(m2 & 0xFFFFu, m2 >> 16);
      mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
      mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
      float sc, rc;
      const bool fast = block_scale(mx, ctl, sc, rc);
      uint32_t code[8];
      quantise32(w, sc, rc, fast, code);
      if (t < p.T) {
        const int kb = kb0 + static_cast<int>(it);
        uint4* dst = reinterpret_cast<uint4*>(p.codes + static_cast<size_t>(t) * H + kb * BLK + qq * 32);
        dst[0] = make_uint4(code[0], code[1], code[2], code[3]);
        dst[1] = make_uint4(code[4], code[5], code[6], code[7]);
        if (qq == 0) p.scale[static_cast<size_t>(kb) * p.T + t] = sc;
      }
    }
    // Every quantiser has finished reading the x ring: it becomes the buffer that holds this
    // CTA's partial accumulator, [128 rows][64 float4 chunks], chunk c of row r at position
    // c ^ (r & 7) so a warp's 32 rows spread over all banks.
    asm volatile("bar.sync 1, %0;" ::"n"(32 * GATE_QWARPS) : "memory");
    if (lane == 0) mbar_wait_drain(&ctl->mma_done, 0);
    __syncwarp();
    mbar_try_wait(&ctl->mma_done, 0);
    tc_fence_after();
    if (!aborted && !*abort_flag) {
      const int lq = warp & 3;                   // TMEM lanes [32 lq, 32 lq + 32) of this warp
      const int r = lq * 32 + lane;
      const int cbase = (j >> 2) * 2;             // two 32-column chunks per warp
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int col = (cbase + cc) * 32;
        float v[32];
        tmem_ld32(tmem + (static_cast<uint32_t>(lq * 32) << 16) + col, v);
        uint8_t* rowp = smem + r * GATE_RED_ROW;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int c = col / 4 + i;
          *reinterpret_cast<float4*>(rowp + ((c ^ (r & 7)) << 4)) =
              make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        }
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  if (warp >= GATE_QWARP0) {
    // Rows [32q, 32q + 32) of the tile: sum of the GATE_KS partials in K-slice order.
    const uint32_t q = cluster_ctarank();
    const uint32_t red = smem_u32(smem);
    const int tid = threadIdx.x - 32 * GATE_QWARP0;
#pragma unroll
    for (int k = 0; k < (TILE_M / GATE_KS) * 64 / (32 * GATE_QWARPS); ++k) {
      const int idx = tid + k * 32 * GATE_QWARPS;
      const int r = static_cast<int>(q) * (TILE_M / GATE_KS) + idx / 64, c = idx & 63;
      const uint32_t off = r * GATE_RED_ROW + ((c ^ (r & 7)) << 4);
      float4 part[GATE_KS];
#pragma unroll
      for (int src = 0; src < GATE_KS; ++src) part[src] = ld_cluster_f4(cluster_map(red + off, src));
      float4 acc = part[0];
#pragma unroll
      for (int src = 1; src < GATE_KS; ++src) {
        acc.x += part[src].x;
        acc.y += part[src].y;
        acc.z += part[src].z;
        acc.w += part[src].w;
      }
      const int t = m0 + r;
      if (t < p.T) *reinterpret_cast<float4*>(p.logits + static_cast<size_t>(t) * E_GLOBAL + c * 4) = acc;
    }
  }
  // No CTA leaves (and releases its shared memory) while a peer may still read it.
  __syncwarp();
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  if (warp == 2) tmem_dealloc(tmem, E_GLOBAL);
}

}  // namespace moe
