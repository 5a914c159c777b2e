/*
 * GPU generator of the seeded synthetic MoE inputs; bit-identical to synth_cpu.c
 * (shared recipe in synth_core.h). Used by the benchmark and the GPU tests so that
 * gigabytes of expert weights need not be generated on the host.
 */
#pragma once
#include "moe_common.cuh"
#include "synth_core.h"

namespace moe {

__global__ void synth_logits_kernel(const float* __restrict__ table, uint64_t seed, long n,
                                    float* __restrict__ out) {
  const uint64_t base = syn_base(seed, SYN_LOGITS, 0);
  for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long>(gridDim.x) * blockDim.x)
    out[i] = syn_normal(table, syn_u32(base, static_cast<uint64_t>(i)));
}

__global__ void synth_bias_kernel(const float* __restrict__ table, uint64_t seed, int E, float stddev,
                                  const int* __restrict__ hot, int n_hot, float hot_value,
                                  uint16_t* __restrict__ out) {
  const uint64_t base = syn_base(seed, SYN_BIAS, 0);
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < E; e += gridDim.x * blockDim.x) {
    float v = syn_fmul(stddev, syn_normal(table, syn_u32(base, static_cast<uint64_t>(e))));
    for (int h = 0; h < n_hot; ++h)
      if (hot[h] == e) v = hot_value;
    out[e] = syn_bf16_bits(v);
  }
}

// One warp per (token, 128-column block).
__global__ void synth_hidden_kernel(const float* __restrict__ table, uint64_t seed, int T,
                                    float stddev, uint8_t* __restrict__ hidden,
                                    float* __restrict__ hidden_scale) {
  const uint64_t base = syn_base(seed, SYN_HIDDEN, 0);
  const int lane = threadIdx.x & 31;
  const long nblk = static_cast<long>(T) * HB;
  for (long w = (blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x) >> 5; w < nblk;
       w += (static_cast<long>(gridDim.x) * blockDim.x) >> 5) {
    const int t = static_cast<int>(w / HB), kb = static_cast<int>(w % HB);
    float v[4];
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint64_t idx = static_cast<uint64_t>(t) * H + kb * 128 + lane * 4 + i;
      v[i] = syn_bf16_round(syn_fmul(stddev, syn_normal(table, syn_u32(base, idx))));
      amax = fmaxf(amax, fabsf(v[i]));
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float scale = amax > 0.0f ? syn_fdiv(amax, 448.0f) : 1.0f;
    uint32_t packed = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) packed |= static_cast<uint32_t>(syn_e4m3(syn_fdiv(v[i], scale))) << (8 * i);
    *reinterpret_cast<uint32_t*>(hidden + static_cast<size_t>(t) * H + kb * 128 + lane * 4) = packed;
    if (lane == 0) hidden_scale[static_cast<size_t>(kb) * T + t] = scale;
  }
}

// One CTA (256 threads) per 128x128 block of one expert's weight matrix [rows, cols].
__global__ void __launch_bounds__(256) synth_weight_kernel(const float* __restrict__ table, uint64_t seed,
                                                           int stream, int e0, int rows, int cols,
                                                           float stddev, uint8_t* __restrict__ q,
                                                           float* __restrict__ scale) {
  __shared__ float red[8];
  const int rb = rows / 128, cb = cols / 128;
  const int e = blockIdx.x / (rb * cb);
  const int blk = blockIdx.x % (rb * cb);
  const int br = blk / cb, bc = blk % cb;
  const uint64_t base = syn_base(seed, static_cast<uint32_t>(stream), static_cast<uint32_t>(e0 + e));
  const int r = threadIdx.x >> 1, c0 = (threadIdx.x & 1) * 64;
  float v[64];
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 64; ++i) {
    const uint64_t idx = static_cast<uint64_t>(br * 128 + r) * cols + bc * 128 + c0 + i;
    v[i] = syn_bf16_round(syn_fmul(stddev, syn_normal(table, syn_u32(base, idx))));
    amax = fmaxf(amax, fabsf(v[i]));
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  amax = red[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) amax = fmaxf(amax, red[i]);
  const float s = amax > 0.0f ? syn_fdiv(amax, 448.0f) : 1.0f;
  uint8_t* dst = q + static_cast<size_t>(e) * rows * cols + static_cast<size_t>(br * 128 + r) * cols + bc * 128 + c0;
#pragma unroll
  for (int i = 0; i < 64; i += 16) {
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      uint32_t x = 0;
#pragma unroll
      for (int b = 0; b < 4; ++b) x |= static_cast<uint32_t>(syn_e4m3(syn_fdiv(v[i + 4 * k + b], s))) << (8 * b);
      w[k] = x;
    }
    *reinterpret_cast<uint4*>(dst + i) = make_uint4(w[0], w[1], w[2], w[3]);
  }
  if (threadIdx.x == 0) scale[static_cast<size_t>(e) * rb * cb + blk] = s;
}

}  // namespace moe
