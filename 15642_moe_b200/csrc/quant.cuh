/*
 * FP8 activation quantiser: the step before the MoE path. bf16 hidden states [T, 7168] become
 * the e4m3 codes [T, 7168] and the block-major fp32 scales [56, T] that moe_forward takes
 * (reference/moe_ref.py:44-45 input layout), with the convention of the benchmark
 * configurations: per (token, 128-column block) scale = amax / 448 (fp32 division, 1 for an
 * all-zero block), code = e4m3(x / scale) rounded to nearest even and saturated to +-448.
 * 14,336 bytes read and 7,392 written per token.
 *
 * x / scale is formed from y = RN(1 / scale) by Markstein's method (P. Markstein, "Computation of
 * elementary functions on the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990):
 * q1 = RN(x y), then twice r = x - scale q (exact with an FMA) and q = RN(q + r y). The first
 * correction brings q within one ulp of x / scale and the second then returns the correctly
 * rounded quotient, so the codes equal those of an IEEE division; two values at a time with the
 * packed f32x2 instructions. Blocks whose amax is below 2^-80 (where the remainder could
 * underflow) divide directly, out of line.
 */
#pragma once
#include "moe_common.cuh"

#include <cuda_bf16.h>
#include <cuda_fp8.h>

namespace moe {

__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float2 f2_unpack(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

// e4m3 codes (with the signs OR-ed in) of 8 consecutive values from their quotients q by the
// block scale: two cvt.rn.satfinite.e4m3x2 per 4 values.
__device__ __forceinline__ uint32_t codes4(float2 q0, float2 q1, uint32_t w0, uint32_t w1) {
  const uint32_t c0 = __nv_cvt_float2_to_fp8x2(q0, __NV_SATFINITE, __NV_E4M3);
  const uint32_t c1 = __nv_cvt_float2_to_fp8x2(q1, __NV_SATFINITE, __NV_E4M3);
  return (c0 | (c1 << 16)) | (__byte_perm(w0, w1, 0x7531) & 0x80808080u);
}

// x / s for the two values of a packed pair, correctly rounded, given y = RN(1/s) and
// ns = (-s, -s) (Markstein, two corrections; valid while s >= 2^-80 / 448).
__device__ __forceinline__ float2 quotient2(uint64_t x, uint64_t yy, uint64_t ns) {
  uint64_t t = f2_mul(x, yy);
  t = f2_fma(f2_fma(t, ns, x), yy, t);
  t = f2_fma(f2_fma(t, ns, x), yy, t);
  return f2_unpack(t);
}

// The two bf16 values of a word as a packed fp32 pair (low half first).
__device__ __forceinline__ uint64_t bf16x2_to_f2(uint32_t u) {
  return f2_pack(__uint_as_float(u << 16), __uint_as_float(u & 0xFFFF0000u));
}

constexpr float QUANT_FAST_MIN_AMAX = 0x1.0p-80f;

// 8 values (4 words) sharing the scale s with amax < 2^-80: IEEE division, out of line.
__device__ __noinline__ uint2 quantise8_divide(uint4 w, float s) {
  const uint32_t u[4] = {w.x, w.y, w.z, w.w};
  float2 q[4];
#pragma unroll
  for (int k = 0; k < 4; ++k)
    q[k] = make_float2(__fdiv_rn(__uint_as_float(u[k] << 16), s), __fdiv_rn(__uint_as_float(u[k] & 0xFFFF0000u), s));
  return make_uint2(codes4(q[0], q[1], u[0], u[1]), codes4(q[2], q[3], u[2], u[3]));
}

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
      uint2 packed;
      if (amax >= QUANT_FAST_MIN_AMAX) {
        const float y = __frcp_rn(s);
        const uint64_t yy = f2_pack(y, y), ns = f2_pack(-s, -s);
        packed.x = codes4(quotient2(bf16x2_to_f2(u[0]), yy, ns), quotient2(bf16x2_to_f2(u[1]), yy, ns), u[0], u[1]);
        packed.y = codes4(quotient2(bf16x2_to_f2(u[2]), yy, ns), quotient2(bf16x2_to_f2(u[3]), yy, ns), u[2], u[3]);
      } else {
        packed = quantise8_divide(raw[i], s);
      }
      // Codes of load i: 8 bytes per lane, 256 contiguous bytes per warp.
      __stcs(reinterpret_cast<uint2*>(q + row) + i * 32 + lane, packed);
      if (sub == 0) {
        const int kb = g * QB_PER_WARP + 2 * i + hi_half;
        scale[static_cast<size_t>(kb) * T + t] = s;
      }
    }
  }
}

}  // namespace moe
