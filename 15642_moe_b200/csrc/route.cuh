/*
 * Routing and the final combine of the MoE forward.
 *
 *   route_kernel     no-aux-loss grouped top-k routing (reference/moe_ref.py:82-107); every
 *                    local (token, expert) pair claims a slot in its expert's row list with one
 *                    atomic, which replaces the per-expert selection of moe_ref.py:110-124
 *   gather_kernel    copies each routed FP8 hidden row (and its 56 scales) into its expert's
 *                    128-row tile image, K-major with the 128-byte swizzle
 *                    (the index_select of reference/moe_ref.py:124)
 *   combine_kernel   per-token sum of the weighted expert outputs in ascending expert
 *                    order, one bf16 rounding (reference/moe_ref.py:133-136)
 *
 * The slot order inside an expert's list depends on atomic timing, but no result does: every
 * row of the expert GEMMs is computed independently of the other rows, and the combine adds a
 * token's contributions in ascending expert order.
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

// Order-preserving map of a float to an unsigned key (larger float -> larger key; +0 and -0
// differ, which never matters here).
__device__ __forceinline__ uint32_t order_key(float v) {
  const uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Compare-exchange: entry a ends up the better of the two (larger key; on equal keys the lower
// expert position), with its position and unbiased score alongside.
__device__ __forceinline__ void cx_best(uint32_t& ka, int& pa, float& sa, uint32_t& kb, int& pb, float& sbv) {
  const bool swap = kb > ka || (kb == ka && pb < pa);
  const uint32_t k0 = swap ? kb : ka, k1 = swap ? ka : kb;
  const int p0 = swap ? pb : pa, p1 = swap ? pa : pb;
  const float s0 = swap ? sbv : sa, s1 = swap ? sa : sbv;
  ka = k0; kb = k1; pa = p0; pb = p1; sa = s0; sbv = s1;
}

// Batcher's odd-even merge sort of eight entries (19 compare-exchanges), best first.
__device__ __forceinline__ void sort8_best_first(uint32_t (&k)[8], int (&p)[8], float (&v)[8]) {
#define MOE_CX(a, b) cx_best(k[a], p[a], v[a], k[b], p[b], v[b])
  MOE_CX(0, 1); MOE_CX(2, 3); MOE_CX(4, 5); MOE_CX(6, 7);
  MOE_CX(0, 2); MOE_CX(1, 3); MOE_CX(4, 6); MOE_CX(5, 7);
  MOE_CX(1, 2); MOE_CX(5, 6);
  MOE_CX(0, 4); MOE_CX(1, 5); MOE_CX(2, 6); MOE_CX(3, 7);
  MOE_CX(2, 4); MOE_CX(3, 5);
  MOE_CX(1, 2); MOE_CX(3, 4); MOE_CX(5, 6);
#undef MOE_CX
}

// One warp per token; lane l owns experts 8l..8l+7, so a group of 32 experts is four lanes.
// Outputs: topk_idx / topk_w [T, 8] in selection order. For the local picks (global expert g
// with 0 <= le = g - local_offset < E_local), when `counts` is given: counts[le] (atomic),
// route_token[le * T + slot] = t, route_w[le * T + slot] = weight, and the token's own list
// token_route[t * 8 + k] = (le << 16) | slot in ascending le, token_nr[t] = its length.
// When `zero_out` is given (rows of `zero_row_bytes`, 16-byte aligned), the output row of a token
// without a local route is written here as +0, and the combine skips that token.
__global__ void __launch_bounds__(256) route_kernel(const float* __restrict__ logits,
                                                    const float* __restrict__ bias, int T,
                                                    float rsf, int local_offset, int E_local,
                                                    int* __restrict__ topk_idx,
                                                    float* __restrict__ topk_w,
                                                    int* __restrict__ counts,
                                                    int* __restrict__ token_nr,
                                                    int* __restrict__ token_route,
                                                    int* __restrict__ route_token,
                                                    float* __restrict__ route_w,
                                                    void* __restrict__ zero_out = nullptr,
                                                    int zero_row_bytes = 0) {
  // The gather kernel may be scheduled once every block of this grid runs; it waits for this
  // grid's completion in hardware before reading anything written here.
  if (threadIdx.x == 0) allow_dependent_launch();
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

  // Top-8 of the biased scores inside the kept groups (moe_ref.py:99-101). Each round is two
  // hardware warp reductions: the largest order-preserving key, then the lowest expert index
  // among the lanes holding it (ties to the lower index). Key 0 marks excluded or taken entries
  // (below every real score's key; biased scores are never -0.0, so equal keys mean equal
  // scores).
  // Each lane first sorts its eight entries, best first (larger key, then lower expert index), so a
  // round only reads the lane's head and the winning lane shifts its list by one.
  uint32_t key[8];
  int pos[8];
  float sv[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    key[i] = group_kept ? order_key(sb[i]) : 0u;
    pos[i] = i;
    sv[i] = s[i];
  }
  sort8_best_first(key, pos, sv);
  int sel_idx[TOP_K];
  float sel_s[TOP_K];
#pragma unroll
  for (int k = 0; k < TOP_K; ++k) {
    const uint32_t mk = __reduce_max_sync(0xffffffffu, key[0]);
    const uint32_t wi = __reduce_min_sync(0xffffffffu, key[0] == mk ? static_cast<uint32_t>(lane * 8 + pos[0]) : 0xFFFFFFFFu);
    const float ws = __shfl_sync(0xffffffffu, sv[0], static_cast<int>(wi >> 3));
    if (static_cast<int>(wi >> 3) == lane) {
#pragma unroll
      for (int i = 0; i < 7; ++i) {
        key[i] = key[i + 1];
        pos[i] = pos[i + 1];
        sv[i] = sv[i + 1];
      }
      key[7] = 0u;
    }
    sel_idx[k] = static_cast<int>(wi);
    sel_s[k] = ws;
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
    const int le = sel_idx[k] - local_offset;
    nlocal += (le >= 0 && le < E_local) ? 1 : 0;
  }
  // Lane k < 8 handles pick k: all eight slot claims (atomics) and stores of a token are in
  // flight together rather than one after another.
  if (lane < TOP_K) {
    int my_idx = sel_idx[0];
    float my_s = sel_s[0];
#pragma unroll
    for (int k = 1; k < TOP_K; ++k) {
      my_idx = lane == k ? sel_idx[k] : my_idx;
      my_s = lane == k ? sel_s[k] : my_s;
    }
    const float w = __fmul_rn(__fdiv_rn(my_s, wsum), rsf);
    topk_idx[static_cast<size_t>(t) * TOP_K + lane] = my_idx;
    topk_w[static_cast<size_t>(t) * TOP_K + lane] = w;
    const int le = my_idx - local_offset;
    if (counts != nullptr && le >= 0 && le < E_local) {
      const int slot = atomicAdd(&counts[le], 1);
      route_token[static_cast<size_t>(le) * T + slot] = t;
      route_w[static_cast<size_t>(le) * T + slot] = w;
      // Position in the token's list: local picks with a lower expert id come first.
      int pos = 0;
#pragma unroll
      for (int j = 0; j < TOP_K; ++j) {
        const int lj = sel_idx[j] - local_offset;
        pos += (lj >= 0 && lj < le) ? 1 : 0;
      }
      token_route[static_cast<size_t>(t) * TOP_K + pos] = (le << 16) | slot;
    }
  }
  if (lane == 0 && token_nr != nullptr) token_nr[t] = nlocal;
  // A token without a local route: its output row is +0 (the combine's sum from +0 over no
  // routes). The router is bound by its load latency, so these stores cost it little, and the
  // combine no longer spends a block on each such token.
  if (zero_out != nullptr && nlocal == 0) {
    uint8_t* row = static_cast<uint8_t*>(zero_out) + static_cast<size_t>(t) * zero_row_bytes;
    if ((reinterpret_cast<uintptr_t>(zero_out) & 31u) == 0) {
      const uint32_t z[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int b = lane * 32; b < zero_row_bytes; b += 32 * 32) st_global_v8_u32(row + b, z);
    } else {
      for (int b = lane * 16; b < zero_row_bytes; b += 32 * 16)
        *reinterpret_cast<uint4*>(row + b) = make_uint4(0, 0, 0, 0);
    }
  }
}

// Routing of the shared expert: every token is slot t of the single local expert, weight 1.
// Replaces route_kernel when the forward computes DeepSeek-V3's shared-expert branch.
__global__ void __launch_bounds__(256) shared_route_kernel(int T, int* __restrict__ counts,
                                                           int* __restrict__ token_nr,
                                                           int* __restrict__ token_route,
                                                           int* __restrict__ route_token,
                                                           float* __restrict__ route_w) {
  if (blockIdx.x == 0 && threadIdx.x == 0) counts[0] = T;
  for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < T; t += gridDim.x * blockDim.x) {
    token_nr[t] = 1;
    token_route[static_cast<size_t>(t) * TOP_K] = t;  // (expert 0 << 16) | slot t
    route_token[t] = t;
    route_w[t] = 1.0f;
  }
}

// One warp per local route (dense index d over all experts' slot lists): the route's tile row
// is tile_off[e] * 128 + slot. Rows of a tile past its expert's last route are not written;
// every row of the expert GEMMs is independent and those rows' results are never stored.
__global__ void __launch_bounds__(256) gather_kernel(const uint8_t* __restrict__ hidden,
                                                     const float* __restrict__ hidden_scale, int T,
                                                     const int* __restrict__ counts, int E_local,
                                                     const int* __restrict__ route_token,
                                                     int tiles_max, uint8_t* __restrict__ a_tiled,
                                                     float* __restrict__ a_scale,
                                                     int* __restrict__ tile_ready) {
  __shared__ TileMap map;
  // Launched programmatically after the router: wait for its results, then let GEMM1's CTAs be
  // scheduled (GEMM1 waits for this grid in turn).
  wait_prerequisite_grids();
  if (threadIdx.x == 0) allow_dependent_launch();
  // The GEMM1 -> GEMM2 readiness counters of this call and GEMM2's unit queue (entry
  // tiles_max) start at zero; GEMM1 waits for this grid to complete.
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i <= tiles_max; i += gridDim.x * blockDim.x) tile_ready[i] = 0;
  if (threadIdx.x < 32) build_tile_map(&map, counts, E_local, T, tiles_max);
  __syncthreads();
  const int routes = map.dense_off[E_local];
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int d = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; d < routes; d += warps) {
    int lo = 0, hi = E_local;  // expert e with dense_off[e] <= d < dense_off[e + 1]
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (map.dense_off[mid] <= d) lo = mid; else hi = mid;
    }
    const int slot = d - map.dense_off[lo];
    const int tile = map.tile_off[lo] + slot / TILE_M, r = slot % TILE_M;
    const int tok = route_token[static_cast<size_t>(lo) * T + slot];
    if (tile >= tiles_max || tok < 0 || tok >= T) {
      report_status(ST_BAD_INDEX);
      continue;
    }
    // All 14 row loads and both scale loads are issued before any store (one round trip).
    const uint4* src = reinterpret_cast<const uint4*>(hidden + static_cast<size_t>(tok) * H);
    uint8_t* dst = a_tiled + static_cast<size_t>(tile) * HB * TILE_BYTES;
    uint4 v[H / 16 / 32];
#pragma unroll
    for (int i = 0; i < H / 16 / 32; ++i) v[i] = __ldg(src + lane + 32 * i);
    float s0 = 0.0f, s1 = 0.0f;
    if (lane < HB / 2) {
      s0 = __ldg(hidden_scale + static_cast<size_t>(lane) * T + tok);
      s1 = __ldg(hidden_scale + static_cast<size_t>(lane + HB / 2) * T + tok);
    }
#pragma unroll
    for (int i = 0; i < H / 16 / 32; ++i) {
      const int q = lane + 32 * i, kb = q >> 3, c = q & 7;
      *reinterpret_cast<uint4*>(dst + static_cast<size_t>(kb) * TILE_BYTES + r * 128 + ((c ^ (r & 7)) << 4)) = v[i];
    }
    if (lane < HB / 2) {
      a_scale[(static_cast<size_t>(tile) * HB + lane) * TILE_M + r] = s0;
      a_scale[(static_cast<size_t>(tile) * HB + lane + HB / 2) * TILE_M + r] = s1;
    }
  }
}

constexpr int COMBINE_THREADS = H / 16;  // 448 threads x 16 columns per row

// Row layout of the combine kernels: thread `tid` of a 448-thread CTA owns the four float4
// column groups q = tid + 448 j (j = 0..3) of a 7168-wide row, i.e. columns 4q..4q+3; acc[4j + c]
// is column 4q_j + c. A warp's access then covers 512 contiguous bytes per instruction.
constexpr int COMBINE_Q = H / 4 / COMBINE_THREADS;  // 4 float4 groups per thread

// Adds a token's weighted expert outputs to acc: `routes` holds n entries (le << 16) | slot in
// ascending le, and route (le, slot) is dense row dense_base[le] + slot of `partial` (layout of
// partial_offset; dense_base
// written by the GEMM2 kernel, entry [E_local] = all routes). Each entry is checked against the
// expert's row range before it addresses anything.
__device__ __forceinline__ void add_routes(float (&acc)[16], const float* __restrict__ partial,
                                           const int* __restrict__ routes, int n,
                                           const int* __restrict__ dense_base, int E_local, int tid) {
#pragma unroll
  for (int k = 0; k < TOP_K; ++k) {
    if (k < n) {
      const unsigned packed = static_cast<unsigned>(routes[k]);
      const int le = static_cast<int>(packed >> 16), slot = static_cast<int>(packed & 0xFFFFu);
      if (le >= E_local) {
        report_status(ST_BAD_INDEX);
        continue;
      }
      const int row = dense_base[le] + slot;
      if (row >= dense_base[le + 1]) {
        report_status(ST_BAD_INDEX);
        continue;
      }
      float4 p[COMBINE_Q];
#pragma unroll
      for (int j = 0; j < COMBINE_Q; ++j)
        p[j] = __ldcs(reinterpret_cast<const float4*>(partial + partial_offset(static_cast<size_t>(row),
                                                                               4 * (tid + j * COMBINE_THREADS))));
#pragma unroll
      for (int j = 0; j < COMBINE_Q; ++j) {
        acc[4 * j + 0] = __fadd_rn(acc[4 * j + 0], p[j].x);
        acc[4 * j + 1] = __fadd_rn(acc[4 * j + 1], p[j].y);
        acc[4 * j + 2] = __fadd_rn(acc[4 * j + 2], p[j].z);
        acc[4 * j + 3] = __fadd_rn(acc[4 * j + 3], p[j].w);
      }
    }
  }
}

// Rounds acc once to bf16 and stores it into the row at `row` (bf16 [7168]).
__device__ __forceinline__ void store_row_bf16(__nv_bfloat16* row, const float (&acc)[16], int tid) {
  uint2* d = reinterpret_cast<uint2*>(row) + tid;
#pragma unroll
  for (int j = 0; j < COMBINE_Q; ++j)
    d[j * COMBINE_THREADS] = make_uint2(pack_bf16x2(acc[4 * j], acc[4 * j + 1]), pack_bf16x2(acc[4 * j + 2], acc[4 * j + 3]));
}

// Stores acc unrounded into the row at `row` (fp32 [7168]).
__device__ __forceinline__ void store_row_f32(float* row, const float (&acc)[16], int tid) {
  float4* d = reinterpret_cast<float4*>(row) + tid;
#pragma unroll
  for (int j = 0; j < COMBINE_Q; ++j)
    d[j * COMBINE_THREADS] = make_float4(acc[4 * j], acc[4 * j + 1], acc[4 * j + 2], acc[4 * j + 3]);
}

// One CTA per token: out[t] = sum over its local routes, ascending expert order, of the
// weighted expert outputs, starting from +0 like the reference's zero tensor; rounded once to
// bf16 (OutT = __nv_bfloat16, moe_ref.py:136) or left in fp32 (OutT = float).
template <typename OutT>
__global__ void __launch_bounds__(COMBINE_THREADS) combine_kernel(const float* __restrict__ partial,
                                                                  const int* __restrict__ token_nr,
                                                                  const int* __restrict__ token_route,
                                                                  const int* __restrict__ dense_base,
                                                                  int T, int E_local, OutT* __restrict__ out,
                                                                  int skip_written) {
  const int t = blockIdx.x;
  if (t >= T) return;
  // With skip_written, the row of a token with one local route was written by the GEMM2 kernel
  // and that of a token with none by the router.
  if (skip_written && token_nr[t] <= 1) return;
  const int tid = threadIdx.x;
  float acc[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) acc[i] = 0.0f;
  add_routes(acc, partial, token_route + static_cast<size_t>(t) * TOP_K, token_nr[t], dense_base, E_local, tid);
  if constexpr (sizeof(OutT) == 2)
    store_row_bf16(out + static_cast<size_t>(t) * H, acc, tid);
  else
    store_row_f32(out + static_cast<size_t>(t) * H, acc, tid);
}

}  // namespace moe
