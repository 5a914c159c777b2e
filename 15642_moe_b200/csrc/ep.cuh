/*
 * Expert-parallel (EP) MoE layer: W ranks (one GPU each, W <= 8); rank r owns E_rank global
 * experts given by a placement table (by default [r * E_rank, (r + 1) * E_rank); any assignment
 * of distinct experts, e.g. one balanced by expected load) and holds its own T_r tokens. Token dispatch and the
 * return of expert outputs are peer stores over NVLink issued by these kernels; the only
 * host-side collective is the one-time exchange of CUDA IPC handles.
 *
 * Every rank owns one "symmetric" buffer with the same layout (EpLayout); each rank maps all
 * W buffers (its own plus the peers' through CUDA IPC) and passes their addresses as EpPeers.
 * A forward on rank r, epoch e (all ranks call it the same number of times):
 *
 *   route_kernel            top-8 of 256 for the own T_r tokens; every pick claims a local
 *                           slot of its expert (local atomics, as on one GPU)
 *   ep_reserve_kernel       per expert with local picks and an owner (placement table): one
 *                           system-scope atomic on the owner's count reserves a block of slots
 *   ep_dispatch_kernel      per token and owner rank d that it picked: its FP8 row and 56
 *                           scales -> d.recv[r * T_max + t]; per pick the (row, weight, slot)
 *                           records that d's gather / GEMM2 / combine read
 *   ep_barrier_kernel       release flag d.arrive[r] = e on every d, acquire own arrive[*] >= e
 *   gather, GEMM1, GEMM2    unchanged single-GPU kernels over the received rows
 *                           (row index = src * T_max + t, W * T_max "tokens")
 *   ep_combine_send_kernel  per received row: fp32 sum of its local routes in ascending
 *                           expert order, stored unrounded to src.comb[r][t]
 *   memset(own counts), ep_barrier_kernel on the `done` flags
 *   ep_final_combine_kernel out[t] = bf16( sum over owners d ascending of comb[d][t] )
 *
 * The partials travel in fp32 so the layer keeps the reference's single bf16 rounding of an
 * fp32 sum (moe_ref.py:110-136); rounding each owner's partial to bf16 first can move a
 * result by more than the reference tolerance where partials of different owners cancel.
 *
 * Reuse of buffers across epochs is safe without double buffering: a source starts epoch
 * e + 1's dispatch only after every owner signalled `done` for epoch e, which each owner does
 * after its last read of epoch e's received data and after zeroing its counts; an owner
 * writes epoch e + 1's comb rows only after every source signalled `arrive` for e + 1, which
 * each source does after its final combine of epoch e.
 *
 * Waits are bounded (the device wait limit, 2 s by default); on timeout the barrier reports
 * ST_EP_TIMEOUT and returns. Every consumer of peer-written metadata bounds-checks it before
 * addressing memory, so a timed-out forward never reads or writes out of range; once the status
 * word holds ST_EP_TIMEOUT the combine kernels stop exchanging data and the final combine writes
 * NaN rows, so a forward that ran into a timeout cannot return plausible-looking numbers. The
 * host learns of it through moe_get_status (ExpertParallel.forward(check=True) raises).
 * No load here uses TMA multicast; peers are read and written with plain loads and stores.
 */
#pragma once
#include "route.cuh"

namespace moe {

constexpr int EP_MAX_RANKS = 8;

struct EpLayout {
  int world, t_max, e_rank, r_cap;  // r_cap = world * t_max received-row slots
  size_t epoch, place, arrive, done, src_T, counts, recv_rows, recv_scale, route_token, route_w, tok_nr,
      tok_route, comb, total;
};

// Byte offsets of the symmetric buffer (identical on every rank).
//   epoch        u32                 this rank's forward count (read and advanced on the device,
//                                    so a captured CUDA graph can be replayed)
//   place        int [256]           expert placement: (owner rank << 16) | local index of each
//                                    global expert, -1 without an owner (same on every rank)
//   arrive/done  u32 [8]             epoch flags, index = signalling rank
//   src_T        int [8]             tokens each source sent this epoch
//   counts       int [E_rank]        routes per local expert (claimed by remote atomics)
//   recv_rows    u8  [r_cap, 7168]   received FP8 rows, row = src * t_max + t
//   recv_scale   f32 [56, r_cap]     their scales, block-major like hidden_states_scale
//   route_token  int [E_rank, r_cap] received row of each expert slot
//   route_w      f32 [E_rank, r_cap] routing weight of each expert slot
//   tok_nr       int [r_cap]         local routes of each received row
//   tok_route    int [r_cap, 8]      (le << 16) | slot of those routes, ascending le
//   comb         f32 [world, t_max, 7168]   returned partial sums, index = owner rank
inline EpLayout make_ep_layout(int world, int t_max, int e_rank) {
  EpLayout L{};
  L.world = world;
  L.t_max = t_max;
  L.e_rank = e_rank;
  L.r_cap = world * t_max;
  const size_t rc = static_cast<size_t>(L.r_cap), e = static_cast<size_t>(e_rank);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off = ws_align(off + bytes);
    return o;
  };
  L.epoch = take(sizeof(unsigned));
  L.place = take(sizeof(int) * E_GLOBAL);
  L.arrive = take(sizeof(unsigned) * EP_MAX_RANKS);
  L.done = take(sizeof(unsigned) * EP_MAX_RANKS);
  L.src_T = take(sizeof(int) * EP_MAX_RANKS);
  L.counts = take(sizeof(int) * e);
  L.recv_rows = take(rc * H);
  L.recv_scale = take(sizeof(float) * HB * rc);
  L.route_token = take(sizeof(int) * e * rc);
  L.route_w = take(sizeof(float) * e * rc);
  L.tok_nr = take(sizeof(int) * rc);
  L.tok_route = take(sizeof(int) * TOP_K * rc);
  L.comb = take(sizeof(float) * rc * H);
  L.total = off;
  return L;
}

// moe_ep_forward's workspace: the single-GPU layout over W * t_max rows and E_rank experts (the
// owner side), then the source side: its local route counts and reserved slot bases (256 ints
// each), its tokens' route lists ([t_max] counts, [t_max, 8] entries) and its per-expert slot
// lists over all 256 experts ([256, t_max] tokens and weights).
struct EpSourceWs {
  size_t local_counts, base, token_nr, token_route, route_token, route_w, total;
};
inline EpSourceWs make_ep_source_ws(size_t start, int t_max) {
  EpSourceWs w{};
  size_t off = start;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off = ws_align(off + bytes);
    return o;
  };
  const size_t t = static_cast<size_t>(t_max);
  w.local_counts = take(sizeof(int) * E_GLOBAL);
  w.base = take(sizeof(int) * E_GLOBAL);
  w.token_nr = take(sizeof(int) * t);
  w.token_route = take(sizeof(int) * TOP_K * t);
  w.route_token = take(sizeof(int) * E_GLOBAL * t);
  w.route_w = take(sizeof(float) * E_GLOBAL * t);
  w.total = off;
  return w;
}

struct EpPeers {
  uint8_t* base[EP_MAX_RANKS];  // symmetric buffer of each rank, mapped into this process
};

template <typename T_>
__host__ __device__ __forceinline__ T_* ep_at(uint8_t* base, size_t off) {
  return reinterpret_cast<T_*>(base + off);
}

// Owner rank and local index of global expert g from the placement table, or d = -1.
__device__ __forceinline__ void ep_owner(const int* place, const EpLayout& L, int g, int& d, int& le) {
  const int v = (g >= 0 && g < E_GLOBAL) ? place[g] : -1;
  d = v >> 16;
  le = v & 0xFFFF;
  if (v < 0 || d >= L.world || le >= L.e_rank) d = -1;
}

// One thread per global expert g with local routes and an owner: one system-scope atomic on the
// owner's count reserves a block of local_counts[g] consecutive slots, base[g] = its first.
// (One remote atomic per (source, expert) instead of one per route: a popular expert's count
// would otherwise serialise hundreds of atomics arriving over NVLink.)
__global__ void __launch_bounds__(256) ep_reserve_kernel(const __grid_constant__ EpPeers peers,
                                                         const __grid_constant__ EpLayout L, int rank,
                                                         const int* __restrict__ local_counts,
                                                         int* __restrict__ base) {
  const int* place = ep_at<int>(peers.base[rank], L.place);
  for (int g = threadIdx.x; g < E_GLOBAL; g += blockDim.x) {
    const int c = local_counts[g];
    int d, le;
    ep_owner(place, L, g, d, le);
    if (c <= 0 || d < 0) continue;
    base[g] = atomicAdd_system(ep_at<int>(peers.base[d], L.counts) + le, c);
  }
}

// One warp per own token. route_kernel (run over all 256 experts) gave the token its picks in
// ascending global expert order, token_route[t * 8 + k] = (g << 16) | local slot, and
// route_w[g * T + local slot] their weights; the owner of g comes from the placement table (picks
// of experts without an owner are dropped, as moe_ref.py:115-116 drops non-local ones). Lane k < n
// stores its pick into owner d's slot base[g] + local slot (row, weight, and the row's route
// list entry at its position among the token's picks of d); then the row (read once into
// registers) and its 56 scales are stored into every owner it picked.
__global__ void __launch_bounds__(256) ep_dispatch_kernel(const __grid_constant__ EpPeers peers, const __grid_constant__ EpLayout L, int rank, int T,
                                                          const uint8_t* __restrict__ hidden,
                                                          const float* __restrict__ hidden_scale,
                                                          const int* __restrict__ token_nr,
                                                          const int* __restrict__ token_route,
                                                          const float* __restrict__ route_w,
                                                          const int* __restrict__ base) {
  if (blockIdx.x == 0 && threadIdx.x < L.world)
    ep_at<int>(peers.base[threadIdx.x], L.src_T)[rank] = T;
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  const int* place = ep_at<int>(peers.base[rank], L.place);
  for (int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; t < T; t += warps) {
    const int n = min(max(token_nr[t], 0), TOP_K);
    int g = -1, ls = 0;
    if (lane < n) {
      const unsigned packed = static_cast<unsigned>(token_route[static_cast<size_t>(t) * TOP_K + lane]);
      g = static_cast<int>(packed >> 16);
      ls = static_cast<int>(packed & 0xFFFFu);
      if (g >= E_GLOBAL || ls >= T) {
        report_status(ST_BAD_INDEX);
        g = -1;
      }
    }
    int d = -1, le = 0;
    if (g >= 0) ep_owner(place, L, g, d, le);
    int pos = 0, nd = 0;
    unsigned mask = 0;
#pragma unroll
    for (int j = 0; j < TOP_K; ++j) {
      const int dj = __shfl_sync(0xffffffffu, d, j);
      pos += (d >= 0 && j < lane && dj == d) ? 1 : 0;
      nd += (dj == lane) ? 1 : 0;
      mask |= dj >= 0 ? (1u << dj) : 0u;
    }
    const int row = rank * L.t_max + t;
    if (lane < L.world) ep_at<int>(peers.base[lane], L.tok_nr)[row] = nd;
    if (d >= 0) {
      uint8_t* pb = peers.base[d];
      const int slot = base[g] + ls;
      if (slot >= 0 && slot < L.r_cap) {
        const size_t i = static_cast<size_t>(le) * L.r_cap + slot;
        ep_at<int>(pb, L.route_token)[i] = row;
        ep_at<float>(pb, L.route_w)[i] = route_w[static_cast<size_t>(g) * T + ls];
        ep_at<int>(pb, L.tok_route)[static_cast<size_t>(row) * TOP_K + pos] = (le << 16) | slot;
      } else {
        report_status(ST_BAD_INDEX);
      }
    }
    if (mask == 0) continue;
    // The row is read once into registers and stored to every owner that needs it.
    const uint4* src = reinterpret_cast<const uint4*>(hidden + static_cast<size_t>(t) * H);
    uint4 v[H / 16 / 32];
#pragma unroll
    for (int i = 0; i < H / 16 / 32; ++i) v[i] = __ldg(src + lane + 32 * i);
    float s0 = 0.0f, s1 = 0.0f;
    if (lane < HB / 2) {
      s0 = __ldg(hidden_scale + static_cast<size_t>(lane) * T + t);
      s1 = __ldg(hidden_scale + static_cast<size_t>(lane + HB / 2) * T + t);
    }
    for (int dd = 0; dd < L.world; ++dd) {
      if (!(mask & (1u << dd))) continue;
      uint8_t* pb = peers.base[dd];
      uint4* dst = reinterpret_cast<uint4*>(pb + L.recv_rows + static_cast<size_t>(row) * H);
#pragma unroll
      for (int i = 0; i < H / 16 / 32; ++i) dst[lane + 32 * i] = v[i];
      if (lane < HB / 2) {
        float* sc = ep_at<float>(pb, L.recv_scale);
        sc[static_cast<size_t>(lane) * L.r_cap + row] = s0;
        sc[static_cast<size_t>(lane + HB / 2) * L.r_cap + row] = s1;
      }
    }
  }
}

// One warp: lane d < world publishes this forward's epoch into rank d's flag slot [rank] (after
// a system-scope fence, so every store this rank issued before this kernel is visible first),
// then lane j < world waits, bounded, until this rank's flag [j] reaches the epoch. The epoch
// lives in this rank's buffer: the first barrier of a forward (`advance`) increments it, the
// second reads it, so no host value is baked into the launches.
__global__ void __launch_bounds__(32) ep_barrier_kernel(const __grid_constant__ EpPeers peers, size_t flag_off,
                                                        size_t epoch_off, int rank, int world, int advance) {
  // May be launched programmatically: everything the previous kernel stored must be complete
  // before this rank signals. The next kernel may then be scheduled (it waits for this one).
  wait_prerequisite_grids();
  allow_dependent_launch();
  const int lane = threadIdx.x;
  unsigned* ep = ep_at<unsigned>(peers.base[rank], epoch_off);
  unsigned epoch = 0;
  if (lane == 0) {
    epoch = *ep + (advance ? 1u : 0u);
    if (advance) *ep = epoch;
  }
  epoch = __shfl_sync(0xffffffffu, epoch, 0);
  if (lane < world) {
    __threadfence_system();
    st_release_sys(ep_at<unsigned>(peers.base[lane], flag_off) + rank, epoch);
    const unsigned* f = ep_at<unsigned>(peers.base[rank], flag_off) + lane;
    const unsigned long long t0 = globaltimer(), limit = wait_limit_ns();
    while (static_cast<int>(ld_acquire_sys(f) - epoch) < 0) {
      if (globaltimer() - t0 > limit) {
        report_status(ST_EP_TIMEOUT);
        break;
      }
      __nanosleep(128);
    }
  }
  __syncwarp();
}

// Grid-stride over the received rows (one CTA of 448 threads per row): the fp32
// sum of the row's local routes in ascending expert order from +0, stored into the source
// rank's comb[rank][t].
__global__ void __launch_bounds__(COMBINE_THREADS) ep_combine_send_kernel(const __grid_constant__ EpPeers peers, const __grid_constant__ EpLayout L,
                                                                          int rank,
                                                                          const float* __restrict__ partial,
                                                                          const int* __restrict__ dense_base) {
  uint8_t* me = peers.base[rank];
  const int* src_T = ep_at<int>(me, L.src_T);
  const int* tok_nr = ep_at<int>(me, L.tok_nr);
  const int* tok_route = ep_at<int>(me, L.tok_route);
  const int tid = threadIdx.x;
  if (status_now() & ST_EP_TIMEOUT) return;   // a peer is missing: send nothing this epoch
  for (int i = blockIdx.x; i < L.r_cap; i += gridDim.x) {
    const int src = i / L.t_max, t = i - src * L.t_max;
    int tn = src_T[src];
    if (tn > L.t_max) {
      if (threadIdx.x == 0) report_status(ST_BAD_INDEX);
      tn = L.t_max;
    }
    if (t >= tn) continue;
    const int n = tok_nr[i];
    if (n <= 0) continue;
    float acc[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) acc[k] = 0.0f;
    add_routes(acc, partial, tok_route + static_cast<size_t>(i) * TOP_K, n, dense_base, L.e_rank, tid);
    float* dst = ep_at<float>(peers.base[src], L.comb) + (static_cast<size_t>(rank) * L.t_max + t) * H;
    store_row_f32(dst, acc, tid);
  }
}

// Adds the fp32 row at `row` into acc (the combine kernels' column mapping).
__device__ __forceinline__ void add_row_f32(float (&acc)[16], const float* row, int tid) {
  const float4* q = reinterpret_cast<const float4*>(row) + tid;
  float4 v[COMBINE_Q];
#pragma unroll
  for (int j = 0; j < COMBINE_Q; ++j) v[j] = __ldcs(q + j * COMBINE_THREADS);
#pragma unroll
  for (int j = 0; j < COMBINE_Q; ++j) {
    acc[4 * j + 0] = __fadd_rn(acc[4 * j + 0], v[j].x);
    acc[4 * j + 1] = __fadd_rn(acc[4 * j + 1], v[j].y);
    acc[4 * j + 2] = __fadd_rn(acc[4 * j + 2], v[j].z);
    acc[4 * j + 3] = __fadd_rn(acc[4 * j + 3], v[j].w);
  }
}

// One CTA per own token: out[t] = bf16( sum over the owners of its picks, ascending rank,
// of comb[d][t] ) from +0; tokens whose picks have no owner get zeros.
__global__ void __launch_bounds__(COMBINE_THREADS) ep_final_combine_kernel(const uint8_t* __restrict__ me,
                                                                           EpLayout L, int T,
                                                                           const int* __restrict__ topk_idx,
                                                                           __nv_bfloat16* __restrict__ out) {
  wait_prerequisite_grids();                // launched programmatically after the done barrier
  const int t = blockIdx.x;
  if (t >= T) return;
  const int tid = threadIdx.x;
  if (status_now() & ST_EP_TIMEOUT) {       // the exchange did not complete: NaN, not stale data
    uint2* d = reinterpret_cast<uint2*>(out + static_cast<size_t>(t) * H) + tid;
#pragma unroll
    for (int j = 0; j < COMBINE_Q; ++j) d[j * COMBINE_THREADS] = make_uint2(0x7FC07FC0u, 0x7FC07FC0u);
    return;
  }
  const int* place = reinterpret_cast<const int*>(me + L.place);
  unsigned mask = 0;
#pragma unroll
  for (int k = 0; k < TOP_K; ++k) {
    int d, le;
    ep_owner(place, L, topk_idx[static_cast<size_t>(t) * TOP_K + k], d, le);
    if (d >= 0) mask |= 1u << d;
  }
  const float* comb = reinterpret_cast<const float*>(me + L.comb);
  float acc[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) acc[k] = 0.0f;
  for (int d = 0; d < L.world; ++d)
    if (mask & (1u << d)) add_row_f32(acc, comb + (static_cast<size_t>(d) * L.t_max + t) * H, tid);
  store_row_bf16(out + static_cast<size_t>(t) * H, acc, tid);
}

// Failure-path probe of ep_barrier_kernel on one GPU: the barrier of a 2-rank layout whose
// second rank never exists. `buf` (>= 256 zeroed bytes) stands for both ranks' buffers: the epoch
// lives at offset 0 and the flags at offset 64, so rank 0's own flag is set and the wait for
// rank 1's runs out after the wait limit, reporting ST_EP_TIMEOUT.
inline void launch_ep_barrier_probe(uint8_t* buf, cudaStream_t st) {
  EpPeers peers{};
  for (int d = 0; d < EP_MAX_RANKS; ++d) peers.base[d] = buf;
  ep_barrier_kernel<<<1, 32, 0, st>>>(peers, 64, 0, 0, 2, 1);
}

// Failure-path probe of mbar_wait: one thread waits on an mbarrier nothing arrives on; after the
// wait limit it raises the abort flag and reports `who`.
__global__ void __launch_bounds__(32) mbar_probe_kernel(int who, int* aborted) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncwarp();
  if (threadIdx.x == 0) {
    const bool ok = mbar_wait(&bar, 0, &abort_flag, who);
    *aborted = ok ? 0 : (abort_flag ? 1 : 2);
  }
}

}  // namespace moe
