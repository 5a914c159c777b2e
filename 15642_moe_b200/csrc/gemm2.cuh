/*
 * GEMM2 with the routing weight over the routed rows of every active local expert
 * (reference/moe_ref.py:131-134: O = C . W2[e]^T, contribution = O * w[token, e]).
 *
 * C arrives from GEMM1 as two e4m3 terms sharing one fp32 scale per (row, 128-block):
 * C ~= scale * (hi + lo). Both terms are multiplied against the same W2 tile and accumulate
 * into the same TMEM accumulator, so the intermediate keeps ~2^-8 relative precision instead
 * of e4m3's 2^-4 while W2 stays FP8 in HBM.
 *
 * Work unit = (128-row tile, 256 hidden rows of W2 = two 128-wide output halves). Same warp
 * roles and rotating TMEM accumulators as GEMM1:
 *   warp 0      producer (bulk copies: 16 KB hi + 16 KB lo + 32 KB W2 per stage, 3 stages; 8 KB
 *               each of hi and lo for a tile of at most 64 routes), and per unit its block scales
 *               (c_scale of the tile, two rows of w2_scale) into shared memory
 *   warp 1      MMA: per 128-K block, hi then lo for each of the 4 K steps (M = 128, or 64 for a
 *               tile of at most 64 routes; K = 32), in ACC_SPLIT groups of N = 256 / ACC_SPLIT
 *               columns, each into its own accumulator
 *   warps 4-11  epilogue: per accumulator, promote with c_scale[row, kb] * w2_scale[hb, kb];
 *               at the end multiply by the route weight and write the fp32 rows to `partial`
 *               (dense: one row per local route).
 */
#pragma once
#include "moe_common.cuh"
#include "gemm1.cuh"

namespace moe {

struct Gemm2Args {
  const uint8_t* c_hi;      // [tiles, 16, 128, 128] SW128
  const uint8_t* c_lo;      // [tiles, 16, 128, 128] SW128
  const float* c_scale;     // [tiles, 16, 128]
  const uint8_t* w2p;       // [E, 28, 16, 256, 128] SW128 (packed by pack_w2_kernel)
  const float* w2_scale;    // [E, 56, 16]
  const int* counts;        // [E_local] routes per local expert
  int slots;                // slots per expert (row stride of route_w)
  int tiles_max;            // capacity of the c_* tile arrays
  int E_local;
  const float* route_w;     // [E_local, slots] routing weight of each expert slot
  float* partial;           // route (e, slot) is dense row dense_base[e] + slot (partial_offset layout)
  int* dense_base;          // [E_local + 1] written by CTA 0 for the combine
  const int* tile_ready;    // [tiles] GEMM1 column blocks done per tile; a tile is read at G1_NT
  int* unit_queue;          // zero at launch: the next unit to claim (dynamic schedule)
  // When `direct` is set, a route that is its token's only local route is written straight into
  // the token's output row (bf16, or fp32 when out_f32) instead of `partial`; the combine then
  // skips that token. Its value is the combine's for a one-route token: round(0 + x).
  void* out;
  int out_f32;
  const int* route_token;   // [E_local, slots] token of each expert slot
  const int* token_nr;      // [slots] local routes of each token
  int direct;
};

// Bounded wait until GEMM1 has stored all G1_NT column blocks of C for `tile` (acquire), then
// order the following bulk copies (async proxy) after it. Returns false on timeout or abort.
__device__ __forceinline__ bool wait_tile_ready(const int* ready, volatile int* abort_flag) {
  if (ld_acquire_gpu(ready) < G1_NT) {
    const unsigned long long t0 = globaltimer(), limit = wait_limit_ns();
    while (ld_acquire_gpu(ready) < G1_NT) {
      if (*abort_flag) return false;
      if (globaltimer() - t0 > limit) {
        *abort_flag = 1;
        report_status(ST_TIMEOUT_PRODUCER);
        return false;
      }
      __nanosleep(256);
    }
  }
  fence_proxy_async_global();
  return true;
}

constexpr int G2_STAGES = 3;
constexpr int G2_A_BYTES = TILE_BYTES;      // one of hi / lo
constexpr int G2_B_BYTES = 2 * TILE_BYTES;  // 256 W2 rows x 128 K bytes
constexpr int G2_STAGE_BYTES = 2 * G2_A_BYTES + G2_B_BYTES;
constexpr int G2_THREADS = GEMM_THREADS;
constexpr int G2_CTRL_BYTES = 20480;
constexpr int G2_SMEM = G2_STAGES * G2_STAGE_BYTES + G2_CTRL_BYTES + 1024;

// Units are claimed at run time from a global counter (tile-major order), so CTAs that start
// early - on SMs GEMM1 has already left - take more of them. The producer claims and passes each
// unit id to the MMA warp and the epilogue warps through a small ring in shared memory; -1 ends.
constexpr int G2_UNIT_RING = 4;

struct G2Ctrl {
  uint64_t full[G2_STAGES];
  uint64_t empty[G2_STAGES];
  uint64_t ufull[G2_UNIT_RING];
  uint64_t uempty[G2_UNIT_RING];
  int unit[G2_UNIT_RING];
  uint64_t tfull[ACC_BUFS];
  uint64_t tempty[ACC_BUFS];
  uint64_t sfull[2];             // block scales of the unit with this parity landed
  uint64_t sempty[2];            // ... and read by the eight epilogue warps
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort_flag;
  // Block scales of a unit, copied by the producer (loading them from global memory in the
  // epilogue stalled it on every K block): C's c_scale[tile, 0..15, 0..127] and W2's
  // w2_scale[e, 2 nt .. 2 nt + 1, 0..15], two slots by unit parity.
  alignas(16) float c_sc[2][IB][TILE_M];
  alignas(16) float w_sc[2][2][IB];
  TileMap map;
};
static_assert(sizeof(G2Ctrl) <= G2_CTRL_BYTES, "control block too large");

// Next unit id of this CTA's schedule (claim k), read by one thread (MMA) or one whole warp
// (epilogue); -1 when the schedule is over or the CTA aborted.
__device__ __forceinline__ int g2_next_unit(G2Ctrl* ctl, uint32_t k, volatile int* abort_flag, bool warp_wide) {
  const int r = k % G2_UNIT_RING;
  const uint32_t ph = (k / G2_UNIT_RING) & 1u;
  const bool ok = warp_wide ? mbar_wait_warp(&ctl->ufull[r], ph, abort_flag, ST_TIMEOUT_EPILOGUE)
                            : mbar_wait(&ctl->ufull[r], ph, abort_flag, ST_TIMEOUT_MMA);
  if (!ok) return -1;
  const int u = *static_cast<volatile int*>(&ctl->unit[r]);
  if (warp_wide) __syncwarp();
  if (!warp_wide || (threadIdx.x & 31) == 0) mbar_arrive(&ctl->uempty[r]);
  return u;
}

__global__ void __launch_bounds__(G2_THREADS, 1) gemm2_weighted_kernel(const __grid_constant__ Gemm2Args p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_1024(smem_raw);
  G2Ctrl* ctl = reinterpret_cast<G2Ctrl*>(smem + G2_STAGES * G2_STAGE_BYTES);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0) build_tile_map(&ctl->map, p.counts, p.E_local, p.slots, p.tiles_max);
  __syncthreads();
  if (blockIdx.x == 0)
    for (int e = threadIdx.x; e <= p.E_local; e += blockDim.x) p.dense_base[e] = ctl->map.dense_off[e];
  const int n_units = clamp_tiles(ctl->map.tile_off[p.E_local], p.tiles_max) * G2_NT;
  if (static_cast<int>(blockIdx.x) >= n_units) return;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < G2_STAGES; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->empty[s], 1);
    }
#pragma unroll
    for (int b = 0; b < ACC_BUFS; ++b) {
      mbar_init(&ctl->tfull[b], 1);
      mbar_init(&ctl->tempty[b], 8);
    }
#pragma unroll
    for (int r = 0; r < G2_UNIT_RING; ++r) {
      mbar_init(&ctl->ufull[r], 1);
      mbar_init(&ctl->uempty[r], 9);   // the MMA warp and the eight epilogue warps
    }
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      mbar_init(&ctl->sfull[q], 1);
      mbar_init(&ctl->sempty[q], 8);
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

  if (warp < 4) {
    regs_dec<REGS_CTRL>();
  }
  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      uint32_t it = 0, units_issued = 0;
      int ready_tile = -1;
      for (uint32_t k = 0; !*abort_flag; ++k) {
        // Claim the next unit and hand it to the MMA and epilogue warps.
        int u = atomicAdd(p.unit_queue, 1);
        if (u >= n_units) u = -1;
        const int r = k % G2_UNIT_RING;
        if (!mbar_wait(&ctl->uempty[r], ((k / G2_UNIT_RING) & 1u) ^ 1u, abort_flag, ST_TIMEOUT_PRODUCER)) break;
        ctl->unit[r] = u;
        mbar_arrive(&ctl->ufull[r]);
        if (u < 0) break;
        const int tile = u / G2_NT, nt = u % G2_NT;
        const TileInfo ti = locate(&ctl->map, p.counts, p.E_local, tile, p.slots);
        const int e = ti.e;
        // A tile of at most 64 routes runs M = 64 MMAs: only its first 64 rows of C are read.
        const uint32_t c_bytes = ti.rows <= TILE_M / 2 ? G2_A_BYTES / 2 : G2_A_BYTES;
        const size_t a_off = static_cast<size_t>(tile) * IB * TILE_BYTES;
        const uint8_t* b_src = p.w2p + (static_cast<size_t>(e) * G2_NT + nt) * IB * G2_B_BYTES;
        // This grid may start while GEMM1 still runs (programmatic launch): the tile's C must be
        // complete before its first copy is issued.
        if (tile != ready_tile) {
          if (!wait_tile_ready(p.tile_ready + tile, abort_flag)) break;
          ready_tile = tile;
        }
        {
          const int q = units_issued & 1;
          if (!mbar_wait(&ctl->sempty[q], ((units_issued >> 1) & 1u) ^ 1u, abort_flag, ST_TIMEOUT_PRODUCER)) break;
          mbar_arrive_expect_tx(&ctl->sfull[q], (IB * TILE_M + 2 * IB) * 4);
          bulk_g2s(ctl->c_sc[q], p.c_scale + static_cast<size_t>(tile) * IB * TILE_M, IB * TILE_M * 4, &ctl->sfull[q]);
          bulk_g2s(ctl->w_sc[q], p.w2_scale + (static_cast<size_t>(e) * HB + 2 * nt) * IB, 2 * IB * 4, &ctl->sfull[q]);
          ++units_issued;
        }
        for (int ib = 0; ib < IB; ++ib, ++it) {
          const int s = it % G2_STAGES;
          const uint32_t ph = (it / G2_STAGES) & 1u;
          if (!mbar_wait(&ctl->empty[s], ph ^ 1u, abort_flag, ST_TIMEOUT_PRODUCER)) break;
          uint8_t* st = smem + s * G2_STAGE_BYTES;
          mbar_arrive_expect_tx(&ctl->full[s], 2 * c_bytes + G2_B_BYTES);
          bulk_g2s(st, p.c_hi + a_off + static_cast<size_t>(ib) * TILE_BYTES, c_bytes, &ctl->full[s]);
          bulk_g2s(st + G2_A_BYTES, p.c_lo + a_off + static_cast<size_t>(ib) * TILE_BYTES, c_bytes, &ctl->full[s]);
          bulk_g2s_hint(st + 2 * G2_A_BYTES, b_src + static_cast<size_t>(ib) * G2_B_BYTES,
                        G2_B_BYTES, &ctl->full[s], pol_w);
        }
      }
      const uint32_t issued = it;
      if (!*abort_flag) {
        for (uint32_t jt = issued; jt < issued + G2_STAGES; ++jt) {
          if (!mbar_wait(&ctl->empty[jt % G2_STAGES], ((jt / G2_STAGES) & 1u) ^ 1u, abort_flag,
                         ST_TIMEOUT_PRODUCER))
            break;
        }
      }
      if (*abort_flag) {
        for (uint32_t i = 1; i <= G2_STAGES && i <= issued; ++i) {
          const uint32_t jt = issued - i;
          mbar_wait_drain(&ctl->full[jt % G2_STAGES], (jt / G2_STAGES) & 1u);
        }
        for (uint32_t i = 1; i <= 2 && i <= units_issued; ++i) {
          const uint32_t un = units_issued - i;
          mbar_wait_drain(&ctl->sfull[un & 1], (un >> 1) & 1u);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t it = 0;
      bool stop = false;
      for (uint32_t k = 0; !stop; ++k) {
        const int u = g2_next_unit(ctl, k, abort_flag, false);
        if (u < 0) break;
        // M = 64 for a tile of at most 64 routes: the accumulator then holds row 16 j + i in TMEM
        // lane 32 j + i (i < 16), half the tensor work of M = 128.
        const TileInfo ti = locate(&ctl->map, p.counts, p.E_local, u / G2_NT, p.slots);
        const uint32_t idesc = idesc_e4m3_f32(ti.rows <= TILE_M / 2 ? 64 : 128, ACC_COLS);
        for (int ib = 0; ib < IB && !stop; ++ib, ++it) {
          const int s = it % G2_STAGES;
          const uint32_t ph = (it / G2_STAGES) & 1u;
          if (!mbar_wait_spin(&ctl->full[s], ph, abort_flag, ST_TIMEOUT_MMA)) {
            stop = true;
            break;
          }
          const uint32_t hi_addr = smem_u32(smem + s * G2_STAGE_BYTES);
          const uint32_t lo_addr = hi_addr + G2_A_BYTES;
#pragma unroll
          for (int h = 0; h < ACC_SPLIT; ++h) {   // output columns [ACC_COLS h, ACC_COLS (h+1))
            const uint32_t hidx = ACC_SPLIT * it + h;
            const uint32_t q = hidx % ACC_BUFS, use = hidx / ACC_BUFS;
            if (!mbar_wait_spin(&ctl->tempty[q], (use & 1u) ^ 1u, abort_flag, ST_TIMEOUT_MMA)) {
              stop = true;
              break;
            }
            tc_fence_after();
            const uint32_t b_addr = hi_addr + 2 * G2_A_BYTES + h * ACC_COLS * 128;
            const uint32_t d = tmem + q * ACC_COLS;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t bd = sdesc_k_sw128(b_addr + kk * 32);
              tc_mma_f8(d, sdesc_k_sw128(hi_addr + kk * 32), bd, idesc, kk > 0 ? 1u : 0u);
              tc_mma_f8(d, sdesc_k_sw128(lo_addr + kk * 32), bd, idesc, 1u);
            }
            tc_commit(&ctl->tfull[q]);
          }
          if (!stop) tc_commit(&ctl->empty[s]);
        }
      }
      if (*abort_flag) {
        tc_commit(&ctl->mma_done);
        mbar_wait_drain(&ctl->mma_done, 0);
      }
    }
  } else if (warp >= 4) {
    // ---------------- epilogue (warps 4..11) ----------------
    regs_inc<REGS_EPI>();
    const int q4 = warp & 3;
    const int hf = (warp - 4) >> 2;    // which 64 columns of each 128-wide half
    const uint32_t t_lane = static_cast<uint32_t>(q4 * 32) << 16;
    uint32_t it = 0;
    for (uint32_t k = 0;; ++k) {
      const int u = g2_next_unit(ctl, k, abort_flag, true);
      if (u < 0) break;
      const int tile = u / G2_NT, nt = u % G2_NT;
      const TileInfo ti = locate(&ctl->map, p.counts, p.E_local, tile, p.slots);
      const int e = ti.e;
      // Row of the tile this thread's TMEM lane holds: lane q4 * 32 + lane for M = 128; for the
      // M = 64 MMAs of a tile of at most 64 routes, row 16 q4 + lane in lanes 0-15 of each
      // quarter, and no row (TILE_M) in lanes 16-31.
      const int row = ti.rows <= TILE_M / 2 ? (lane < 16 ? q4 * 16 + lane : TILE_M) : q4 * 32 + lane;
      const int slot = ti.m * TILE_M + row;
      // The route weight is first needed after the K loop; its load is issued now, and so is the
      // route's token, whose local route count is loaded after the first K block (off the unit
      // start): tok >= 0 marks a token's only local route.
      const float w = row < ti.rows ? __ldg(p.route_w + static_cast<size_t>(e) * p.slots + slot) : 0.0f;
      const int tk = p.direct && row < ti.rows ? __ldg(p.route_token + static_cast<size_t>(e) * p.slots + slot) : -1;
      int tk_nr = 0;
      float acc[128];
#pragma unroll
      for (int i = 0; i < 128; ++i) acc[i] = 0.0f;
      // The unit's scales come through shared memory: the producer copies them once the tile's
      // readiness counter shows GEMM1 has stored C and c_scale.
      const int uq = k & 1;
      bool aborted = !mbar_wait_warp(&ctl->sfull[uq], (k >> 1) & 1u, abort_flag, ST_TIMEOUT_EPILOGUE);
      if (!aborted) mbar_observe(&ctl->sfull[uq], (k >> 1) & 1u);
      const float* cs = &ctl->c_sc[uq][0][row < TILE_M ? row : 0];
      const float* ws0 = ctl->w_sc[uq][0];
      const float* ws1 = ctl->w_sc[uq][1];
      for (int ib = 0; ib < IB && !aborted; ++ib, ++it) {
        const float nc = cs[ib * TILE_M];
        const float f0 = nc * ws0[ib], f1 = nc * ws1[ib];
        if (!promote_block<G2Ctrl, true>(ctl, tmem, t_lane, hf, it, f0, acc, f1, acc + 64, abort_flag)) {
          aborted = true;
          break;
        }
        if (ib == 0 && tk >= 0 && tk < p.slots) tk_nr = __ldg(p.token_nr + tk);
      }
      const int tok = tk_nr == 1 ? tk : -1;
      if (!aborted) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctl->sempty[uq]);
      }
      if (named_bar_or(1, 256, aborted)) break;

      if (row < ti.rows && tok >= 0) {
        // The token's only local route: its output columns nt * 256 .. + 255, as the combine would
        // write them for a one-route token (0 + x, then one bf16 rounding or none). The output is
        // 16-byte aligned by contract; 256-bit stores only when it is also 32-byte aligned.
        const bool out32 = (reinterpret_cast<uintptr_t>(p.out) & 31u) == 0;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
#pragma unroll
          for (int g = 0; g < 8; g += 2) {
            // 16 columns: 64 bytes of fp32 or 32 bytes of bf16 per store pair / store.
            float v[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = __fadd_rn(0.0f, acc[h * 64 + 8 * g + i] * w);
            const size_t col = static_cast<size_t>(tok) * H + nt * 256 + h * 128 + hf * 64 + 8 * g;
            if (p.out_f32) {
              float* o = static_cast<float*>(p.out) + col;
              if (out32) {
                st_global_v8(o, v);
                st_global_v8(o + 8, v + 8);
              } else {
#pragma unroll
                for (int i = 0; i < 4; ++i)
                  reinterpret_cast<float4*>(o)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
              }
            } else {
              uint32_t q[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) q[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
              __nv_bfloat16* o = static_cast<__nv_bfloat16*>(p.out) + col;
              if (out32) {
                st_global_v8_u32(o, q);
              } else {
                reinterpret_cast<uint4*>(o)[0] = make_uint4(q[0], q[1], q[2], q[3]);
                reinterpret_cast<uint4*>(o)[1] = make_uint4(q[4], q[5], q[6], q[7]);
              }
            }
          }
        }
      } else if (row < ti.rows) {
        const size_t d = static_cast<size_t>(ctl->map.dense_off[e] + slot);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
#pragma unroll
          for (int g = 0; g < 8; ++g) {
            float v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = acc[h * 64 + 8 * g + i] * w;
            st_global_v8(p.partial + partial_offset(d, nt * 256 + h * 128 + hf * 64 + 8 * g), v);
          }
        }
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, ACC_BUFS * ACC_COLS);
}

}  // namespace moe
