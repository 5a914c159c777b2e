/*
 * GEMM1 + SwiGLU over the routed rows of every active local expert
 * (reference/moe_ref.py:126-130: G1 = A_e . W13[e]^T, C = X1 * SiLU(X2)).
 *
 * Work unit = (128-row tile, column tile j): the tile's rows against the 128 X1 rows
 * (128j..128j+127) and the matching 128 X2 rows (2048+128j..) of the expert's W13, so the
 * SwiGLU of one 128-wide intermediate block is computed inside one CTA.
 *
 * One persistent CTA per SM, warp-specialised:
 *   warp 0      producer: cp.async.bulk of pre-swizzled 16 KB A tiles and 32 KB W13 tiles
 *               into a 4-stage shared-memory ring (mbarrier complete_tx)
 *   warp 1      MMA: 4 x tcgen05.mma kind::f8f6f4 (M=128, N=256, K=32) per 128-K block into
 *               one of two TMEM accumulators (2 x 256 columns)
 *   warps 4-11  epilogue: after each 128-K block, read the raw partial from TMEM and promote it
 *               with the block scales, acc += raw * a_scale[row, kb] * w_scale[nblk, kb]
 *               (the reference's fp32 dequantisation, moe_ref.py:59-79, applied per block);
 *               at the end apply SwiGLU and write C as two e4m3 terms (hi + lo) with one fp32
 *               scale per (row, 128-column block), laid out as SW128 tiles for GEMM2.
 * The per-block promotion cannot use the hardware block-scaled MMA because the reference's
 * scales are arbitrary fp32 values, not powers of two.
 */
#pragma once
#include "moe_common.cuh"

namespace moe {

struct Gemm1Args {
  const uint8_t* a_tiled;   // [tiles, 56, 128, 128] SW128
  const float* a_scale;     // [tiles, 56, 128]
  const uint8_t* w13p;      // [E, 16, 56, 256, 128] SW128 (packed by pack_w13_kernel)
  const float* w13_scale;   // [E, 32, 56]
  const int* tile_expert;   // [tiles]
  const int* n_tiles;       // [1]
  int tiles_max;            // capacity of the workspace tile arrays
  int E_local;              // number of local experts (bounds of tile_expert)
  uint8_t* c_hi;            // [tiles, 16, 128, 128] SW128
  uint8_t* c_lo;            // [tiles, 16, 128, 128] SW128
  float* c_scale;           // [tiles, 16, 128]
};

constexpr int G1_STAGES = 4;
constexpr int G1_A_BYTES = TILE_BYTES;
constexpr int G1_B_BYTES = 2 * TILE_BYTES;
constexpr int G1_STAGE_BYTES = G1_A_BYTES + G1_B_BYTES;
constexpr int G1_THREADS = GEMM_THREADS;
constexpr int G1_CTRL_BYTES = 4096;
constexpr int G1_SMEM = G1_STAGES * G1_STAGE_BYTES + G1_CTRL_BYTES + 1024;

struct G1Ctrl {
  uint64_t full[G1_STAGES];
  uint64_t empty[G1_STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort_flag;
  float amax[2][2][TILE_M];  // [unit parity][column half][row]
};
static_assert(sizeof(G1Ctrl) <= G1_CTRL_BYTES, "control block too large");

// Pack 16 floats (already divided by the scale) into e4m3 hi and lo 16-byte chunks.
__device__ __forceinline__ void quant_hi_lo16(const float* x, uint4& hi, uint4& lo) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    uint32_t hw = 0, lw = 0;
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      float2 v = make_float2(x[w * 4 + p * 2], x[w * 4 + p * 2 + 1]);
      __nv_fp8x2_storage_t h2 = __nv_cvt_float2_to_fp8x2(v, __NV_SATFINITE, __NV_E4M3);
      __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(h2, __NV_E4M3);
      float2 hv = __half22float2(*reinterpret_cast<__half2*>(&hr));
      float2 r = make_float2(v.x - hv.x, v.y - hv.y);
      __nv_fp8x2_storage_t l2 = __nv_cvt_float2_to_fp8x2(r, __NV_SATFINITE, __NV_E4M3);
      hw |= static_cast<uint32_t>(h2) << (16 * p);
      lw |= static_cast<uint32_t>(l2) << (16 * p);
    }
    h[w] = hw;
    l[w] = lw;
  }
  hi = make_uint4(h[0], h[1], h[2], h[3]);
  lo = make_uint4(l[0], l[1], l[2], l[3]);
}

__global__ void __launch_bounds__(G1_THREADS, 1) gemm1_swiglu_kernel(Gemm1Args p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_1024(smem_raw);
  G1Ctrl* ctl = reinterpret_cast<G1Ctrl*>(smem + G1_STAGES * G1_STAGE_BYTES);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_units = clamp_tiles(*p.n_tiles, p.tiles_max) * G1_NT;
  if (static_cast<int>(blockIdx.x) >= n_units) return;  // uniform per CTA, before any TMEM use

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < G1_STAGES; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->empty[s], 1);
    }
#pragma unroll
    for (int b = 0; b < 2; ++b) {
      mbar_init(&ctl->tfull[b], 1);
      mbar_init(&ctl->tempty[b], 8);
    }
    mbar_init(&ctl->mma_done, 1);
    ctl->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&ctl->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  volatile int* abort_flag = &ctl->abort_flag;

  if (warp < 4) {
    regs_dec<REGS_CTRL>();
  }
  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      uint32_t it = 0;
      for (int u = blockIdx.x; u < n_units && !*abort_flag; u += gridDim.x) {
        const int tile = u / G1_NT, j = u % G1_NT;
        const int e = checked_expert(p.tile_expert[tile], p.E_local);
        const uint8_t* a_src = p.a_tiled + static_cast<size_t>(tile) * HB * TILE_BYTES;
        const uint8_t* b_src = p.w13p + (static_cast<size_t>(e) * G1_NT + j) * HB * G1_B_BYTES;
        for (int kb = 0; kb < HB; ++kb, ++it) {
          const int s = it % G1_STAGES;
          const uint32_t ph = (it / G1_STAGES) & 1u;
          if (!mbar_wait(&ctl->empty[s], ph ^ 1u, abort_flag, ST_TIMEOUT_PRODUCER)) break;
          uint8_t* sa = smem + s * G1_STAGE_BYTES;
          mbar_arrive_expect_tx(&ctl->full[s], G1_STAGE_BYTES);
          bulk_g2s(sa, a_src + static_cast<size_t>(kb) * TILE_BYTES, G1_A_BYTES, &ctl->full[s]);
          bulk_g2s_hint(sa + G1_A_BYTES, b_src + static_cast<size_t>(kb) * G1_B_BYTES, G1_B_BYTES,
                        &ctl->full[s], pol_w);
        }
      }
      const uint32_t issued = it;
      if (!*abort_flag) {
        // Drain: wait until the MMAs have released every stage, so no async arrive is pending.
        for (uint32_t jt = issued; jt < issued + G1_STAGES; ++jt) {
          if (!mbar_wait(&ctl->empty[jt % G1_STAGES], ((jt / G1_STAGES) & 1u) ^ 1u, abort_flag,
                         ST_TIMEOUT_PRODUCER))
            break;
        }
      }
      if (*abort_flag) {
        // Let the copies already issued land before shared memory is released.
        for (uint32_t i = 1; i <= G1_STAGES && i <= issued; ++i) {
          const uint32_t jt = issued - i;
          mbar_wait_drain(&ctl->full[jt % G1_STAGES], (jt / G1_STAGES) & 1u);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_e4m3_f32(128, 256);
      uint32_t it = 0;
      for (int u = blockIdx.x; u < n_units && !*abort_flag; u += gridDim.x) {
        for (int kb = 0; kb < HB; ++kb, ++it) {
          const int s = it % G1_STAGES;
          const uint32_t ph = (it / G1_STAGES) & 1u;
          const uint32_t b = it & 1u, use = it >> 1;
          if (!mbar_wait(&ctl->tempty[b], (use & 1u) ^ 1u, abort_flag, ST_TIMEOUT_MMA)) break;
          if (!mbar_wait(&ctl->full[s], ph, abort_flag, ST_TIMEOUT_MMA)) break;
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + s * G1_STAGE_BYTES);
          const uint32_t b_addr = a_addr + G1_A_BYTES;
          const uint32_t d = tmem + b * 256u;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            tc_mma_f8(d, sdesc_k_sw128(a_addr + kk * 32), sdesc_k_sw128(b_addr + kk * 32), idesc,
                      kk > 0 ? 1u : 0u);
          tc_commit(&ctl->empty[s]);
          tc_commit(&ctl->tfull[b]);
        }
      }
      if (*abort_flag) {
        // Let the MMAs already issued finish before TMEM is released.
        tc_commit(&ctl->mma_done);
        mbar_wait_drain(&ctl->mma_done, 0);
      }
    }
  } else if (warp >= 4) {
    // ---------------- epilogue (warps 4..11) ----------------
    regs_inc<REGS_EPI>();
    const int q = warp & 3;            // TMEM lane quadrant this warp may access
    const int hf = (warp - 4) >> 2;    // column half: 64 X1 + 64 X2 columns
    const int row = q * 32 + lane;
    const uint32_t t_lane = static_cast<uint32_t>(q * 32) << 16;
    uint32_t it = 0, unit_no = 0;
    for (int u = blockIdx.x; u < n_units; u += gridDim.x, ++unit_no) {
      const int tile = u / G1_NT, j = u % G1_NT;
      const int e = checked_expert(p.tile_expert[tile], p.E_local);
      const float* sa_ptr = p.a_scale + static_cast<size_t>(tile) * HB * TILE_M + row;
      const float* sg_ptr = p.w13_scale + (static_cast<size_t>(e) * G1B + j) * HB;
      const float* su_ptr = p.w13_scale + (static_cast<size_t>(e) * G1B + G1_NT + j) * HB;
      float accg[64], accu[64];
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        accg[i] = 0.0f;
        accu[i] = 0.0f;
      }
      float sa_next = __ldg(sa_ptr);
      bool aborted = false;
      for (int kb = 0; kb < HB; ++kb, ++it) {
        const float sa = sa_next;
        if (kb + 1 < HB) sa_next = __ldg(sa_ptr + (kb + 1) * TILE_M);
        const float fg = sa * __ldg(sg_ptr + kb);
        const float fu = sa * __ldg(su_ptr + kb);
        const uint32_t b = it & 1u, use = it >> 1;
        if (!mbar_wait_warp(&ctl->tfull[b], use & 1u, abort_flag, ST_TIMEOUT_EPILOGUE)) {
          aborted = true;
          break;
        }
        tc_fence_after();
        const uint32_t base = tmem + t_lane + b * 256u + hf * 64u;
        float v[32];
        tmem_ld32(base, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) accg[i] = fmaf(v[i], fg, accg[i]);
        tmem_ld32(base + 32u, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) accg[32 + i] = fmaf(v[i], fg, accg[32 + i]);
        tmem_ld32(base + 128u, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) accu[i] = fmaf(v[i], fu, accu[i]);
        tmem_ld32(base + 160u, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) accu[32 + i] = fmaf(v[i], fu, accu[32 + i]);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctl->tempty[b]);
      }
      // Every epilogue thread passes this barrier once per unit; the OR makes the decision
      // to stop uniform, so no thread is left waiting on a barrier the others skipped.
      if (named_bar_or(1, 256, aborted)) break;

      // SwiGLU: C = X1 * SiLU(X2)  (moe_ref.py:129-130)
      float amax = 0.0f;
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        const float x2 = accu[i];
        const float c = (x2 / (1.0f + expf(-x2))) * accg[i];
        accg[i] = c;
        amax = fmaxf(amax, fabsf(c));
      }
      ctl->amax[unit_no & 1][hf][row] = amax;
      named_bar_or(2, 256, false);
      amax = fmaxf(amax, ctl->amax[unit_no & 1][hf ^ 1][row]);
      const float scale = amax > 0.0f ? amax / 448.0f : 1.0f;
#pragma unroll
      for (int i = 0; i < 64; ++i) accg[i] = __fdiv_rn(accg[i], scale);

      const size_t blk = (static_cast<size_t>(tile) * IB + j) * TILE_BYTES + row * 128;
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) {
        uint4 hi, lo;
        quant_hi_lo16(&accg[ch * 16], hi, lo);
        const int c16 = hf * 4 + ch;
        const size_t off = blk + ((c16 ^ (row & 7)) << 4);
        *reinterpret_cast<uint4*>(p.c_hi + off) = hi;
        *reinterpret_cast<uint4*>(p.c_lo + off) = lo;
      }
      if (hf == 0) p.c_scale[(static_cast<size_t>(tile) * IB + j) * TILE_M + row] = scale;
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

}  // namespace moe
