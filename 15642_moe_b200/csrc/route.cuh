/*
 * Routing, local dispatch, row gather and the final combine of the MoE forward.
 *
 *   route_kernel     no-aux-loss grouped top-k routing (reference/moe_ref.py:82-107)
 *   dispatch_kernel  per-local-expert compaction into 128-row tiles, rows in token order
 *                    (the selection step of reference/moe_ref.py:110-124)
 *   gather_kernel    copies the routed FP8 hidden rows into K-major SW128 tiles
 *                    (the index_select of reference/moe_ref.py:124)
 *   combine_kernel   per-token sum of the weighted expert outputs in ascending expert
 *                    order, one bf16 rounding (reference/moe_ref.py:133-136)
 */
#pragma once
#include "moe_common.cuh"

namespace moe {

// Sigmoid rounded once to fp32: evaluated in double precision, then rounded to nearest.
// The reference's torch.sigmoid (fp32 1/(1+exp(-x))) can differ from this by one ulp.
__device__ __forceinline__ float sigmoid_rn(float x) {
  double d = 1.0 / (1.0 + exp(-static_cast<double>(x)));
  return __double2float_rn(d);
}

// Better-of for the top-k: larger value, ties to the lower index.
__device__ __forceinline__ bool better(float v, int i, float ov, int oi) {
  return ov > v || (ov == v && oi < i);
}

// One warp per token; lane l owns experts 8l..8l+7, so a group of 32 experts is four lanes.
__global__ void __launch_bounds__(256) route_kernel(const float* __restrict__ logits,
                                                    const float* __restrict__ bias, int T,
                                                    float rsf, int local_offset, int E_local,
                                                    int* __restrict__ topk_idx,
                                                    float* __restrict__ topk_w,
                                                    int* __restrict__ counts,
                                                    int* __restrict__ token_nr) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= T) return;

  const float4* lg = reinterpret_cast<const float4*>(logits + static_cast<size_t>(t) * E_GLOBAL + lane * 8);
  const float4* bp = reinterpret_cast<const float4*>(bias + lane * 8);
  float x[8], b[8];
  {
    float4 a0 = __ldg(lg), a1 = __ldg(lg + 1), c0 = __ldg(bp), c1 = __ldg(bp + 1);
    x[0] = a0.x; x[1] = a0.y; x[2] = a0.z; x[3] = a0.w;
    x[4] = a1.x; x[5] = a1.y; x[6] = a1.z; x[7] = a1.w;
    b[0] = c0.x; b[1] = c0.y; b[2] = c0.z; b[3] = c0.w;
    b[4] = c1.x; b[5] = c1.y; b[6] = c1.z; b[7] = c1.w;
  }
  float s[8], sb[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    s[i] = sigmoid_rn(x[i]);
    sb[i] = __fadd_rn(s[i], b[i]);
  }

  // Sum of the two largest biased scores of each group (moe_ref.py:91-92).
  float t1 = -INFINITY, t2 = -INFINITY;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (sb[i] > t1) {
      t2 = t1;
      t1 = sb[i];
    } else if (sb[i] > t2) {
      t2 = sb[i];
    }
  }
#pragma unroll
  for (int off = 1; off <= 2; off <<= 1) {
    float o1 = __shfl_xor_sync(0xffffffffu, t1, off);
    float o2 = __shfl_xor_sync(0xffffffffu, t2, off);
    if (t1 >= o1) {
      t2 = fmaxf(t2, o1);
    } else {
      t2 = fmaxf(t1, o2);
      t1 = o1;
    }
  }
  const float gscore = __fadd_rn(t1, t2);

  // Keep the 4 best groups, ties to the lower group (moe_ref.py:94-97).
  const int g = lane >> 2;
  int rank = 0;
#pragma unroll
  for (int og = 0; og < N_GROUP; ++og) {
    float os = __shfl_sync(0xffffffffu, gscore, og * 4);
    rank += (os > gscore || (os == gscore && og < g)) ? 1 : 0;
  }
  const bool group_kept = rank < TOPK_GROUP;

  // Top-8 of the biased scores inside the kept groups (moe_ref.py:99-101).
  uint32_t taken = group_kept ? 0u : 0xFFu;
  int sel_idx[TOP_K];
  float sel_s[TOP_K];
#pragma unroll
  for (int k = 0; k < TOP_K; ++k) {
    float bv = -INFINITY, bs = 0.0f;
    int bi = 0x7FFFFFFF;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (!((taken >> i) & 1u) && better(bv, bi, sb[i], lane * 8 + i)) {
        bv = sb[i];
        bi = lane * 8 + i;
        bs = s[i];
      }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
      float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      float os = __shfl_xor_sync(0xffffffffu, bs, off);
      if (better(bv, bi, ov, oi)) {
        bv = ov;
        bi = oi;
        bs = os;
      }
    }
    if ((bi >> 3) == lane) taken |= 1u << (bi & 7);
    sel_idx[k] = bi;
    sel_s[k] = bs;
  }

  // Weights: unbiased scores renormalised over the 8 picks, times the scaling factor
  // (moe_ref.py:103-107). The sum runs in ascending expert order.
  int rank_of[TOP_K];
#pragma unroll
  for (int k = 0; k < TOP_K; ++k) {
    int rk = 0;
#pragma unroll
    for (int j = 0; j < TOP_K; ++j) rk += sel_idx[j] < sel_idx[k] ? 1 : 0;
    rank_of[k] = rk;
  }
  float wsum = 0.0f;
#pragma unroll
  for (int r = 0; r < TOP_K; ++r) {
    float v = 0.0f;
#pragma unroll
    for (int k = 0; k < TOP_K; ++k) v = rank_of[k] == r ? sel_s[k] : v;
    wsum = __fadd_rn(wsum, v);
  }
  wsum = __fadd_rn(wsum, 1e-20f);

  int nlocal = 0;
#pragma unroll
  for (int k = 0; k < TOP_K; ++k) {
    int le = sel_idx[k] - local_offset;
    bool local = le >= 0 && le < E_local;
    nlocal += local ? 1 : 0;
    if (lane == k) {
      topk_idx[static_cast<size_t>(t) * TOP_K + k] = sel_idx[k];
      topk_w[static_cast<size_t>(t) * TOP_K + k] = __fmul_rn(__fdiv_rn(sel_s[k], wsum), rsf);
      if (local) atomicAdd(&counts[le], 1);
    }
  }
  if (lane == 0 && token_nr != nullptr) token_nr[t] = nlocal;
}

// One CTA per local expert: finds the expert's tokens in token order and lays them out as
// routed rows of its 128-row tiles. Tile offsets and the dense row base (index of the expert's
// first route among all local routes, used for the expert-output rows) come from the counts.
__global__ void __launch_bounds__(1024) dispatch_kernel(
    const int* __restrict__ topk_idx, const float* __restrict__ topk_w,
    const int* __restrict__ counts, int T, int E_local, int local_offset, int* __restrict__ n_tiles,
    int* __restrict__ tile_expert, int* __restrict__ tile_rows, int* __restrict__ tile_dense,
    int* __restrict__ route_token, float* __restrict__ route_w, int* __restrict__ token_row) {
  __shared__ int s_cnt[E_GLOBAL];
  __shared__ int s_off, s_base, s_running, s_total;
  __shared__ int warp_pre[32];
  const int e = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  if (tid < E_local) s_cnt[tid] = counts[tid];
  __syncthreads();
  if (tid == 0) {
    int off = 0, base = 0;
    for (int i = 0; i < e; ++i) {
      off += (s_cnt[i] + TILE_M - 1) / TILE_M;
      base += s_cnt[i];
    }
    s_off = off;
    s_base = base;
    s_running = 0;
    if (e == E_local - 1) *n_tiles = off + (s_cnt[e] + TILE_M - 1) / TILE_M;
  }
  __syncthreads();
  const int off = s_off, cnt = s_cnt[e], dense0 = s_base;
  const int nt = (cnt + TILE_M - 1) / TILE_M;
  for (int i = tid; i < nt; i += blockDim.x) {
    tile_expert[off + i] = e;
    tile_rows[off + i] = min(TILE_M, cnt - TILE_M * i);
    tile_dense[off + i] = dense0 + TILE_M * i;
  }
  const int ge = local_offset + e;
  const size_t row0 = static_cast<size_t>(off) * TILE_M;

  for (int base = 0; base < T; base += blockDim.x) {
    const int t = base + tid;
    int flag = 0, kslot = 0;
    float w = 0.0f;
    if (t < T) {
#pragma unroll
      for (int k = 0; k < TOP_K; ++k) {
        int gk = topk_idx[static_cast<size_t>(t) * TOP_K + k];
        if (gk == ge) {
          flag = 1;
          w = topk_w[static_cast<size_t>(t) * TOP_K + k];
        } else if (gk >= local_offset && gk < ge) {
          ++kslot;
        }
      }
    }
    const unsigned bal = __ballot_sync(0xffffffffu, flag);
    const int pre = __popc(bal & ((1u << lane) - 1u));
    if (lane == 0) warp_pre[wid] = __popc(bal);
    __syncthreads();
    if (wid == 0) {
      int v = lane < (blockDim.x >> 5) ? warp_pre[lane] : 0;
      int incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
      }
      warp_pre[lane] = incl - v;
      if (lane == 31) s_total = incl;
    }
    __syncthreads();
    if (flag) {
      const int slot = s_running + warp_pre[wid] + pre;
      if (slot < cnt) {
        const size_t row = row0 + slot;
        route_token[row] = t;
        route_w[row] = w;
        token_row[static_cast<size_t>(t) * TOP_K + kslot] = dense0 + slot;
      } else {
        report_status(ST_BAD_INDEX);
      }
    }
    __syncthreads();
    if (tid == 0) s_running += s_total;
    __syncthreads();
  }
  if (tid == 0 && s_running != cnt) report_status(ST_BAD_INDEX);
  for (int r = cnt + tid; r < nt * TILE_M; r += blockDim.x) {
    route_token[row0 + r] = -1;
    route_w[row0 + r] = 0.0f;
  }
}

// One warp per routed row: copies the FP8 hidden row of its token into the 56 K-major
// 128B-swizzled 16 KB tiles of its 128-row tile, and its 56 block scales. Pad rows are zero.
__global__ void __launch_bounds__(256) gather_kernel(const uint8_t* __restrict__ hidden,
                                                     const float* __restrict__ hidden_scale, int T,
                                                     const int* __restrict__ n_tiles,
                                                     int tiles_max,
                                                     const int* __restrict__ route_token,
                                                     uint8_t* __restrict__ a_tiled,
                                                     float* __restrict__ a_scale) {
  const int nrows = clamp_tiles(*n_tiles, tiles_max) * TILE_M;
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < nrows; row += warps) {
    const int tile = row >> 7, r = row & 127;
    const int tok = route_token[row];
    const bool ok = tok >= 0 && tok < T;
    const uint4* src = reinterpret_cast<const uint4*>(hidden + static_cast<size_t>(ok ? tok : 0) * H);
    uint8_t* dst = a_tiled + static_cast<size_t>(tile) * HB * TILE_BYTES;
#pragma unroll 2
    for (int q = lane; q < H / 16; q += 32) {
      uint4 v = ok ? __ldg(src + q) : make_uint4(0u, 0u, 0u, 0u);
      const int kb = q >> 3, c = q & 7;
      *reinterpret_cast<uint4*>(dst + static_cast<size_t>(kb) * TILE_BYTES + r * 128 +
                                ((c ^ (r & 7)) << 4)) = v;
    }
    for (int kb = lane; kb < HB; kb += 32)
      a_scale[(static_cast<size_t>(tile) * HB + kb) * TILE_M + r] =
          ok ? __ldg(hidden_scale + static_cast<size_t>(kb) * T + tok) : 0.0f;
  }
}

constexpr int COMBINE_THREADS = H / 16;  // 448: each thread owns 16 consecutive columns

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

// One CTA per token: out[t] = bf16( sum over its local routes, ascending expert order,
// of the weighted expert outputs ), starting from +0 like the reference's zero tensor.
__global__ void __launch_bounds__(COMBINE_THREADS) combine_kernel(const float* __restrict__ partial,
                                                                  const int* __restrict__ token_nr,
                                                                  const int* __restrict__ token_row,
                                                                  int T,
                                                                  __nv_bfloat16* __restrict__ out) {
  const int t = blockIdx.x;
  if (t >= T) return;
  const int n = token_nr[t];
  const int c0 = threadIdx.x * 16;
  float acc[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) acc[i] = 0.0f;
#pragma unroll
  for (int k = 0; k < TOP_K; ++k) {
    if (k < n) {
      const float4* src = reinterpret_cast<const float4*>(
          partial + static_cast<size_t>(token_row[static_cast<size_t>(t) * TOP_K + k]) * H + c0);
      float4 p[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) p[j] = __ldcs(src + j);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[4 * j + 0] = __fadd_rn(acc[4 * j + 0], p[j].x);
        acc[4 * j + 1] = __fadd_rn(acc[4 * j + 1], p[j].y);
        acc[4 * j + 2] = __fadd_rn(acc[4 * j + 2], p[j].z);
        acc[4 * j + 3] = __fadd_rn(acc[4 * j + 3], p[j].w);
      }
    }
  }
  uint4 o0, o1;
  o0.x = pack_bf16x2(acc[0], acc[1]);
  o0.y = pack_bf16x2(acc[2], acc[3]);
  o0.z = pack_bf16x2(acc[4], acc[5]);
  o0.w = pack_bf16x2(acc[6], acc[7]);
  o1.x = pack_bf16x2(acc[8], acc[9]);
  o1.y = pack_bf16x2(acc[10], acc[11]);
  o1.z = pack_bf16x2(acc[12], acc[13]);
  o1.w = pack_bf16x2(acc[14], acc[15]);
  uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(t) * H + c0);
  dst[0] = o0;
  dst[1] = o1;
}

}  // namespace moe
