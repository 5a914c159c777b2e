/*
 * GEMM1 + SwiGLU over the routed rows of every active local expert
 * (reference/moe_ref.py:126-130: G1 = A_e . W13[e]^T, C = X1 * SiLU(X2)).
 *
 * Work unit = (128-row tile, column tile j): the tile's rows against the 128 X1 rows
 * (128j..128j+127) and the matching 128 X2 rows (2048+128j..) of the expert's W13, so the
 * SwiGLU of one 128-wide intermediate block is computed inside one CTA.
 *
 * One persistent CTA per SM, warp-specialised (three warpgroups, 384 threads):
 *   warp 0      producer: cp.async.bulk of the 16 KB A tile image (routed rows, written by the
 *               gather kernel; 8 KB for a tile of at most 64 routes) and the pre-swizzled 32 KB
 *               W13 tile into a 4-stage ring, plus the block scales into shared memory (row
 *               scales eight K blocks at a time, W13 scales once per unit)
 *   warp 1      MMA: per 128-K block, 4 x tcgen05.mma kind::f8f6f4 (M=128, or 64 for a tile of
 *               at most 64 routes; K=32) over the
 *               256 columns, as ACC_SPLIT groups of N = 256 / ACC_SPLIT, each group into its
 *               own TMEM accumulator; all 512 TMEM columns rotate as accumulators so K blocks
 *               stay in flight while the epilogue promotes earlier ones.
 *   warps 4-11  epilogue: for every accumulator, read the raw 128-K partial from TMEM and
 *               promote it with the block scales, acc += raw * a_scale[row, kb] * w_scale[nb, kb]
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
  const uint8_t* a_tiled;   // [tiles, 56, 128, 128] SW128 images of the routed hidden rows
  const float* a_scale;     // [tiles, 56, 128]
  const uint8_t* w13p;      // [E, 16, 56, 256, 128] SW128 (packed by pack_w13_kernel)
  const float* w13_scale;   // [E, 32, 56]
  const int* counts;        // [E_local] routes per local expert
  int slots;                // bound on a count (T)
  int tiles_max;            // capacity of the tile arrays
  int E_local;
  uint8_t* c_hi;            // [tiles, 16, 128, 128] SW128
  uint8_t* c_lo;            // [tiles, 16, 128, 128] SW128
  float* c_scale;           // [tiles, 16, 128]
  int* tile_ready;          // [tiles] column blocks of the tile whose C is stored (release-add)
};

constexpr int G1_STAGES = 4;
constexpr int G1_A_BYTES = TILE_BYTES;
constexpr int G1_B_BYTES = 2 * TILE_BYTES;
constexpr int G1_STAGE_BYTES = G1_A_BYTES + G1_B_BYTES;
constexpr int G1_THREADS = GEMM_THREADS;
constexpr int G1_CTRL_BYTES = 20480;
// Block scales reach the epilogue through shared memory, copied by the producer ahead of the
// stages: the rows' scales a_scale[tile, kb, 0..127] for G1_SC_KB consecutive K blocks per copy,
// in a ring of G1_SC_RING slots, and W13's 2 x 56 scales once per unit (two slots by unit
// parity). Loading them from global memory in the epilogue stalled it on every K block.
constexpr int G1_SC_KB = 8;
constexpr int G1_SC_RING = 3;
static_assert(HB % G1_SC_KB == 0, "a unit's K blocks form whole scale groups");
constexpr int G1_SMEM = G1_STAGES * G1_STAGE_BYTES + G1_CTRL_BYTES + 1024;
static_assert(G1_STAGES <= HB, "the first unit fills every stage");
// TMEM accumulators: a 256-column unit is computed per 128-K block as ACC_SPLIT MMA groups of
// N = ACC_COLS, each into its own accumulator; all 512 TMEM columns rotate as ACC_BUFS
// accumulators, so ACC_BUFS / ACC_SPLIT K blocks can be in flight at once.
#ifndef MOE_ACC_SPLIT
#define MOE_ACC_SPLIT 1
#endif
constexpr int ACC_SPLIT = MOE_ACC_SPLIT;
constexpr int ACC_COLS = 256 / ACC_SPLIT;
constexpr int ACC_BUFS = 512 / ACC_COLS;
static_assert(ACC_SPLIT == 1 || ACC_SPLIT == 2, "unit is split into one or two accumulators");

struct G1Ctrl {
  uint64_t full[G1_STAGES];
  uint64_t empty[G1_STAGES];
  uint64_t tfull[ACC_BUFS];
  uint64_t tempty[ACC_BUFS];
  uint64_t sfull[G1_SC_RING];    // row scales of scale group g landed (slot g % G1_SC_RING)
  uint64_t sempty[G1_SC_RING];   // ... and read by the eight epilogue warps
  uint64_t ufull[2];             // W13 scales of the unit with this parity landed
  uint64_t uempty[2];            // ... and read
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort_flag;
  float amax[2][2][TILE_M];  // [unit parity][column half][row]
  alignas(16) float a_sc[G1_SC_RING][G1_SC_KB][TILE_M];   // a_scale[tile, kb, :] of a group
  alignas(16) float w_sc[2][2][HB];             // [unit parity][X1, X2][kb] of W13
  TileMap map;
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

// Load 64 consecutive fp32 columns of this thread's TMEM lane and wait for completion.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&v)[64]) {
  float a[32], b[32];
  tmem_ld32(taddr, a);
  tmem_ld32(taddr + 32u, b);
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    v[i] = a[i];
    v[32 + i] = b[i];
  }
}

// Epilogue step of one 128-K block of a 256-column unit, for this thread's row (TMEM lane
// quadrant `t_lane`): columns [64*hf, 64*hf + 64) of the unit's first 128-column half are
// promoted into acc0 with factor f0, the same columns of the second half into acc1 with f1.
// An accumulator is released as soon as its values are in registers, before the FMAs, so the
// tensor core can refill it while the promotion runs.
template <class Ctrl, bool kSpin = false>
__device__ __forceinline__ bool promote_block(Ctrl* ctl, uint32_t tmem, uint32_t t_lane, int hf,
                                              uint32_t it, float f0, float* acc0, float f1,
                                              float* acc1, volatile int* abort_flag) {
  float v[64];
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const uint32_t hidx = ACC_SPLIT == 2 ? 2 * it + half : it;
    const uint32_t q = hidx % ACC_BUFS, use = hidx / ACC_BUFS;
    if (ACC_SPLIT == 2 || half == 0) {
      if (!mbar_wait_warp(&ctl->tfull[q], use & 1u, abort_flag, ST_TIMEOUT_EPILOGUE, kSpin)) return false;
      tc_fence_after();
    }
    const uint32_t col = q * ACC_COLS + (ACC_SPLIT == 1 ? half * 128u : 0u) + hf * 64u;
    tmem_ld64(tmem + t_lane + col, v);
    if (ACC_SPLIT == 2 || half == 1) {
      tc_fence_before();
      __syncwarp();
      if ((threadIdx.x & 31) == 0) mbar_arrive(&ctl->tempty[q]);
    }
    float* acc = half == 0 ? acc0 : acc1;
    const float f = half == 0 ? f0 : f1;
    float w[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) w[i] = v[i];
    fma32_scaled(acc, w, f);
#pragma unroll
    for (int i = 0; i < 32; ++i) w[i] = v[32 + i];
    fma32_scaled(acc + 32, w, f);
  }
  return true;
}

// Expert, tile-in-expert and valid rows of global tile `tile`.
struct TileInfo {
  int e, m, rows;
};
__device__ __forceinline__ TileInfo locate(const TileMap* tm, const int* counts, int E_local,
                                           int tile, int cap) {
  TileInfo ti;
  ti.e = tile_expert(tm, E_local, tile);
  ti.m = tile - tm->tile_off[ti.e];
  const int c = min(max(counts[ti.e], 0), cap);
  ti.rows = min(TILE_M, c - ti.m * TILE_M);
  return ti;
}

__global__ void __launch_bounds__(G1_THREADS, 1) gemm1_swiglu_kernel(const __grid_constant__ Gemm1Args p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_1024(smem_raw);
  G1Ctrl* ctl = reinterpret_cast<G1Ctrl*>(smem + G1_STAGES * G1_STAGE_BYTES);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Launched programmatically after the gather, which lets this grid be scheduled only after its
  // own wait for the router's completion: the per-expert counts are final here, so every unit's
  // expert (and weight tiles) is known before the gathered rows are. The producer starts the
  // first unit's weight reads, then waits for the gather (below); every other thread waits before
  // its first read of the gather's output. GEMM2 may be scheduled once every CTA of this grid has
  // passed thread 0's wait, so it never sees the readiness counters before the gather zeroed
  // them; it then waits per tile on tile_ready and never needs this grid to finish.
  if (warp == 0) build_tile_map(&ctl->map, p.counts, p.E_local, p.slots, p.tiles_max);
  __syncthreads();
  const int n_units = clamp_tiles(ctl->map.tile_off[p.E_local], p.tiles_max) * G1_NT;
  if (static_cast<int>(blockIdx.x) >= n_units) return;  // uniform per CTA, before any TMEM use

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < G1_STAGES; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->empty[s], 1);
    }
#pragma unroll
    for (int b = 0; b < ACC_BUFS; ++b) {
      mbar_init(&ctl->tfull[b], 1);
      mbar_init(&ctl->tempty[b], 8);
    }
#pragma unroll
    for (int r = 0; r < G1_SC_RING; ++r) {
      mbar_init(&ctl->sfull[r], 1);
      mbar_init(&ctl->sempty[r], 8);
    }
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      mbar_init(&ctl->ufull[q], 1);
      mbar_init(&ctl->uempty[q], 8);
    }
    mbar_init(&ctl->mma_done, 1);
    ctl->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&ctl->tmem_base, ACC_BUFS * ACC_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  volatile int* abort_flag = &ctl->abort_flag;
  if (threadIdx.x != 0) wait_prerequisite_grids();

  if (warp < 4) {
    regs_dec<REGS_CTRL>();
  }
  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      // W13 block scales of unit number un (this CTA's count) into slot un & 1.
      auto issue_unit_scales = [&](uint32_t un, int e, int j) -> bool {
        const int q = un & 1;
        if (!mbar_wait(&ctl->uempty[q], ((un >> 1) & 1u) ^ 1u, abort_flag, ST_TIMEOUT_PRODUCER)) return false;
        mbar_arrive_expect_tx(&ctl->ufull[q], 2 * HB * 4);
        bulk_g2s(ctl->w_sc[q][0], p.w13_scale + (static_cast<size_t>(e) * G1B + j) * HB, HB * 4, &ctl->ufull[q]);
        bulk_g2s(ctl->w_sc[q][1], p.w13_scale + (static_cast<size_t>(e) * G1B + G1_NT + j) * HB, HB * 4,
                 &ctl->ufull[q]);
        return true;
      };
      // Row scales of the tile's K blocks kb0 .. kb0 + G1_SC_KB - 1 into the slot of group g.
      auto issue_scale_group = [&](uint32_t g, int tile, int kb0) -> bool {
        const int r = g % G1_SC_RING;
        if (!mbar_wait(&ctl->sempty[r], ((g / G1_SC_RING) & 1u) ^ 1u, abort_flag, ST_TIMEOUT_PRODUCER)) return false;
        mbar_arrive_expect_tx(&ctl->sfull[r], G1_SC_KB * TILE_M * 4);
        bulk_g2s(ctl->a_sc[r], p.a_scale + (static_cast<size_t>(tile) * HB + kb0) * TILE_M, G1_SC_KB * TILE_M * 4,
                 &ctl->sfull[r]);
        return true;
      };
      // Stage of K block number it (tile's K block kb): the routed-row tile and the weight tile.
      // A tile of at most 64 routes runs M = 64 MMAs and needs only its first 64 rows (a_bytes).
      auto issue_block = [&](uint32_t it, const uint8_t* a_src, uint32_t a_bytes, const uint8_t* b_src,
                             int kb) -> bool {
        const int s = it % G1_STAGES;
        if (!mbar_wait(&ctl->empty[s], ((it / G1_STAGES) & 1u) ^ 1u, abort_flag, ST_TIMEOUT_PRODUCER)) return false;
        uint8_t* sa = smem + s * G1_STAGE_BYTES;
        mbar_arrive_expect_tx(&ctl->full[s], a_bytes + G1_B_BYTES);
        bulk_g2s(sa, a_src + static_cast<size_t>(kb) * TILE_BYTES, a_bytes, &ctl->full[s]);
        bulk_g2s_hint(sa + G1_A_BYTES, b_src + static_cast<size_t>(kb) * G1_B_BYTES, G1_B_BYTES, &ctl->full[s],
                      pol_w);
        return true;
      };
      // First unit (blockIdx.x < n_units): while the gather still runs, fetch the unit's W13
      // scales and fill every stage with its weight tile, so HBM is busy before the first row
      // tile exists. Then wait for the gather, let GEMM2 be scheduled, and complete the stages
      // with their row tiles and row scales. (Pulling further weight tiles into L2 with bulk
      // prefetches at this point was measured slower.)
      uint32_t it = 0, units_issued = 0, groups_issued = 0;
      {
        const int tile = blockIdx.x / G1_NT, j = blockIdx.x % G1_NT;
        const TileInfo ti = locate(&ctl->map, p.counts, p.E_local, tile, p.slots);
        const int e = ti.e;
        const uint32_t a_bytes = ti.rows <= TILE_M / 2 ? G1_A_BYTES / 2 : G1_A_BYTES;
        const uint8_t* b_src = p.w13p + (static_cast<size_t>(e) * G1_NT + j) * HB * G1_B_BYTES;
        issue_unit_scales(0, e, j);   // slot 0 is free: the wait returns at once
        units_issued = 1;
#pragma unroll
        for (int s = 0; s < G1_STAGES; ++s) {
          mbar_arrive_expect_tx(&ctl->full[s], a_bytes + G1_B_BYTES);
          bulk_g2s_hint(smem + s * G1_STAGE_BYTES + G1_A_BYTES, b_src + static_cast<size_t>(s) * G1_B_BYTES,
                        G1_B_BYTES, &ctl->full[s], pol_w);
        }
        wait_prerequisite_grids();
        allow_dependent_launch();
        issue_scale_group(0, tile, 0);   // slot 0 is free: the wait returns at once
        groups_issued = 1;
        const uint8_t* a_src = p.a_tiled + static_cast<size_t>(tile) * HB * TILE_BYTES;
#pragma unroll
        for (int s = 0; s < G1_STAGES; ++s)
          bulk_g2s(smem + s * G1_STAGE_BYTES, a_src + static_cast<size_t>(s) * TILE_BYTES, a_bytes,
                   &ctl->full[s]);
        it = G1_STAGES;
      }
      static_assert(G1_STAGES <= G1_SC_KB, "the first stages lie in the first scale group");
      for (int u = blockIdx.x; u < n_units && !*abort_flag; u += gridDim.x) {
        const int tile = u / G1_NT, j = u % G1_NT;
        const TileInfo ti = locate(&ctl->map, p.counts, p.E_local, tile, p.slots);
        const int e = ti.e;
        const uint32_t a_bytes = ti.rows <= TILE_M / 2 ? G1_A_BYTES / 2 : G1_A_BYTES;
        const uint8_t* a_src = p.a_tiled + static_cast<size_t>(tile) * HB * TILE_BYTES;
        const uint8_t* b_src = p.w13p + (static_cast<size_t>(e) * G1_NT + j) * HB * G1_B_BYTES;
        const bool first = u == static_cast<int>(blockIdx.x);
        if (!first) {
          if (!issue_unit_scales(units_issued, e, j)) break;
          ++units_issued;
        }
        bool ok = true;
        for (int kb = first ? G1_STAGES : 0; kb < HB; ++kb, ++it) {
          if (kb % G1_SC_KB == 0) {
            if (!issue_scale_group(groups_issued, tile, kb)) {
              ok = false;
              break;
            }
            ++groups_issued;
          }
          if (!issue_block(it, a_src, a_bytes, b_src, kb)) {
            ok = false;
            break;
          }
        }
        if (!ok) break;
      }
      const uint32_t issued = it;
      if (!*abort_flag) {
        // Drain: wait until the MMAs have released every stage, so no async arrive is pending.
        // (Every scale copy is waited for by the epilogue.)
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
        for (uint32_t i = 1; i <= G1_SC_RING && i <= groups_issued; ++i) {
          const uint32_t g = groups_issued - i;
          mbar_wait_drain(&ctl->sfull[g % G1_SC_RING], (g / G1_SC_RING) & 1u);
        }
        for (uint32_t i = 1; i <= 2 && i <= units_issued; ++i) {
          const uint32_t un = units_issued - i;
          mbar_wait_drain(&ctl->ufull[un & 1], (un >> 1) & 1u);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t it = 0;
      bool stop = false;
      for (int u = blockIdx.x; u < n_units && !stop; u += gridDim.x) {
        // M = 64 for a tile of at most 64 routes: row 16 j + i of the accumulator is TMEM lane
        // 32 j + i (i < 16), half the tensor work of M = 128.
        const TileInfo ti = locate(&ctl->map, p.counts, p.E_local, u / G1_NT, p.slots);
        const uint32_t idesc = idesc_e4m3_f32(ti.rows <= TILE_M / 2 ? 64 : 128, ACC_COLS);
        for (int kb = 0; kb < HB && !stop; ++kb, ++it) {
          const int s = it % G1_STAGES;
          const uint32_t ph = (it / G1_STAGES) & 1u;
          if (!mbar_wait(&ctl->full[s], ph, abort_flag, ST_TIMEOUT_MMA)) {
            stop = true;
            break;
          }
          const uint32_t a_addr = smem_u32(smem + s * G1_STAGE_BYTES);
#pragma unroll
          for (int h = 0; h < ACC_SPLIT; ++h) {   // ACC_SPLIT = 2: h = 0 X1 rows, h = 1 X2 rows
            const uint32_t hidx = ACC_SPLIT * it + h;
            const uint32_t q = hidx % ACC_BUFS, use = hidx / ACC_BUFS;
            if (!mbar_wait(&ctl->tempty[q], (use & 1u) ^ 1u, abort_flag, ST_TIMEOUT_MMA)) {
              stop = true;
              break;
            }
            tc_fence_after();
            const uint32_t b_addr = a_addr + G1_A_BYTES + h * ACC_COLS * 128;
            const uint32_t d = tmem + q * ACC_COLS;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              tc_mma_f8(d, sdesc_k_sw128(a_addr + kk * 32), sdesc_k_sw128(b_addr + kk * 32), idesc,
                        kk > 0 ? 1u : 0u);
            tc_commit(&ctl->tfull[q]);
          }
          if (!stop) tc_commit(&ctl->empty[s]);
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
    const int q4 = warp & 3;            // TMEM lane quadrant this warp may access
    const int hf = (warp - 4) >> 2;     // column half: 64 X1 + 64 X2 columns
    const uint32_t t_lane = static_cast<uint32_t>(q4 * 32) << 16;
    uint32_t it = 0, unit_no = 0, grp = 0;
    for (int u = blockIdx.x; u < n_units; u += gridDim.x, ++unit_no) {
      const int tile = u / G1_NT, j = u % G1_NT;
      // Row of the tile this thread's TMEM lane holds: lane q4 * 32 + lane for M = 128; for the
      // M = 64 MMAs of a tile of at most 64 routes, row 16 q4 + lane in lanes 0-15 of each quarter
      // and none in lanes 16-31 (they compute on what their lanes hold and store nothing). The
      // rows past 64 of such a tile's C are never read: GEMM2 reads 64 rows of it.
      const bool small = locate(&ctl->map, p.counts, p.E_local, tile, p.slots).rows <= TILE_M / 2;
      const bool has_row = !small || lane < 16;
      const int row = small ? q4 * 16 + (lane & 15) : q4 * 32 + lane;
      float accg[64], accu[64];
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        accg[i] = 0.0f;
        accu[i] = 0.0f;
      }
      // The unit's W13 scales and each K block's row scales come through shared memory (copied by
      // the producer); each slot is released once this warp has read it.
      const int uq = unit_no & 1;
      bool aborted = !mbar_wait_warp(&ctl->ufull[uq], (unit_no >> 1) & 1u, abort_flag, ST_TIMEOUT_EPILOGUE);
      if (!aborted) mbar_observe(&ctl->ufull[uq], (unit_no >> 1) & 1u);
      const float* wg = ctl->w_sc[uq][0];
      const float* wu = ctl->w_sc[uq][1];
      for (int kb = 0; kb < HB && !aborted; ++kb, ++it) {
        const int r = grp % G1_SC_RING;
        if (kb % G1_SC_KB == 0) {
          if (!mbar_wait_warp(&ctl->sfull[r], (grp / G1_SC_RING) & 1u, abort_flag, ST_TIMEOUT_EPILOGUE)) {
            aborted = true;
            break;
          }
          mbar_observe(&ctl->sfull[r], (grp / G1_SC_RING) & 1u);
        }
        const float na = ctl->a_sc[r][kb % G1_SC_KB][row];
        const float fg = na * wg[kb], fu = na * wu[kb];
        if (kb % G1_SC_KB == G1_SC_KB - 1) {
          __syncwarp();
          if (lane == 0) mbar_arrive(&ctl->sempty[r]);
          ++grp;
        }
        if (!promote_block<G1Ctrl, true>(ctl, tmem, t_lane, hf, it, fg, accg, fu, accu, abort_flag)) {
          aborted = true;
          break;
        }
      }
      if (!aborted) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctl->uempty[uq]);
      }
      // Every epilogue thread passes this barrier once per unit; the OR makes the decision
      // to stop uniform, so no thread is left waiting on a barrier the others skipped.
      if (named_bar_or(1, 256, aborted)) break;

      // SwiGLU: C = X1 * SiLU(X2)  (moe_ref.py:129-130). C is re-encoded to ~2^-8 relative
      // precision below, so the fast exponential and division (a few ulp) are exact enough;
      // the IEEE-rounded versions made this once-per-unit step cost as much as the K loop.
      // For X2 -> -inf, __expf -> inf and __fdividef returns 0, the limit of SiLU.
      float amax = 0.0f;
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        const float x2 = accu[i];
        const float c = __fdividef(x2, 1.0f + __expf(-x2)) * accg[i];
        accg[i] = c;
        amax = fmaxf(amax, fabsf(c));
      }
      if (has_row) ctl->amax[unit_no & 1][hf][row] = amax;
      named_bar_or(2, 256, false);
      amax = fmaxf(amax, ctl->amax[unit_no & 1][hf ^ 1][row]);
      const float scale = amax > 0.0f ? amax / 448.0f : 1.0f;
      const float inv = amax > 0.0f ? 448.0f / amax : 1.0f;
#pragma unroll
      for (int i = 0; i < 64; ++i) accg[i] *= inv;

      const size_t blk = (static_cast<size_t>(tile) * IB + j) * TILE_BYTES + row * 128;
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) {
        uint4 hi, lo;
        quant_hi_lo16(&accg[ch * 16], hi, lo);
        const int c16 = hf * 4 + ch;
        const size_t off = blk + ((c16 ^ (row & 7)) << 4);
        if (has_row) {
          *reinterpret_cast<uint4*>(p.c_hi + off) = hi;
          *reinterpret_cast<uint4*>(p.c_lo + off) = lo;
        }
      }
      if (hf == 0 && has_row) p.c_scale[(static_cast<size_t>(tile) * IB + j) * TILE_M + row] = scale;
      // Publish: once every epilogue thread's C stores of this unit are visible GPU-wide, count
      // the column block as done for the tile (GEMM2 starts a tile at G1_NT).
      __threadfence();
      named_bar_or(3, 256, false);
      if (warp == 4 && lane == 0) red_release_add(p.tile_ready + tile, 1);
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, ACC_BUFS * ACC_COLS);
}

}  // namespace moe
