/*
 * FP8 activation quantiser: the step before the MoE path. bf16 hidden states [T, 7168] become
 * the e4m3 codes [T, 7168] and the block-major fp32 scales [56, T] that moe_forward takes
 * (reference/moe_ref.py:44-45 input layout), with the convention of the benchmark
 * configurations: per (token, 128-column block) scale = amax / 448 (fp32 division, 1 for an
 * all-zero block), code = e4m3(x / scale) rounded to nearest even and saturated to +-448.
 * HBM-bound: 14,336 bytes read and 7,392 written per token.
 */
#pragma once
#include "moe_common.cuh"

#include <cuda_bf16.h>
#include <cuda_fp8.h>

namespace moe {

// One warp per (token, group of 8 blocks): four 512-byte loads per warp (16 bytes per lane) are
// issued before any is used, so each warp keeps 2 KB in flight. Lanes 0-15 hold block 2i and
// lanes 16-31 block 2i + 1 of load i; a block's amax is reduced over its 16 lanes.
constexpr int QB_PER_WARP = 8;  // 56 blocks per token = 7 warp items
__global__ void __launch_bounds__(256) quantize_hidden_kernel(const uint16_t* __restrict__ x, int T,
                                                              uint8_t* __restrict__ q,
                                                              float* __restrict__ scale) {
  const int lane = threadIdx.x & 31, sub = lane & 15, hi_half = lane >> 4;
  const long items = static_cast<long>(T) * (HB / QB_PER_WARP);
  const long warps = (static_cast<long>(gridDim.x) * blockDim.x) >> 5;
  for (long w = (blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x) >> 5; w < items; w += warps) {
    const int t = static_cast<int>(w / (HB / QB_PER_WARP));
    const int g = static_cast<int>(w - static_cast<long>(t) * (HB / QB_PER_WARP));
    const size_t row = static_cast<size_t>(t) * H + g * QB_PER_WARP * BLK;
    uint4 raw[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) raw[i] = __ldcs(reinterpret_cast<const uint4*>(x + row) + i * 32 + lane);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t u[4] = {raw[i].x, raw[i].y, raw[i].z, raw[i].w};
      float v[8];
      float amax = 0.0f;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        v[2 * k] = __uint_as_float(u[k] << 16);
        v[2 * k + 1] = __uint_as_float(u[k] & 0xFFFF0000u);
        amax = fmaxf(amax, fmaxf(fabsf(v[2 * k]), fabsf(v[2 * k + 1])));
      }
#pragma unroll
      for (int o = 8; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const float s = amax > 0.0f ? __fdiv_rn(amax, 448.0f) : 1.0f;
      uint32_t packed[2];
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const __nv_fp8x2_storage_t a = __nv_cvt_float2_to_fp8x2(
            make_float2(__fdiv_rn(v[4 * k], s), __fdiv_rn(v[4 * k + 1], s)), __NV_SATFINITE, __NV_E4M3);
        const __nv_fp8x2_storage_t b = __nv_cvt_float2_to_fp8x2(
            make_float2(__fdiv_rn(v[4 * k + 2], s), __fdiv_rn(v[4 * k + 3], s)), __NV_SATFINITE, __NV_E4M3);
        packed[k] = static_cast<uint32_t>(a) | (static_cast<uint32_t>(b) << 16);
      }
      // Codes of load i: 8 bytes per lane, 256 contiguous bytes per warp.
      __stcs(reinterpret_cast<uint2*>(q + row) + i * 32 + lane, make_uint2(packed[0], packed[1]));
      if (sub == 0) {
        const int kb = g * QB_PER_WARP + 2 * i + hi_half;
        scale[static_cast<size_t>(kb) * T + t] = s;
      }
    }
  }
}

}  // namespace moe
