/*
 * Seeded synthetic inputs for the DeepSeek-V3/R1 FP8 MoE forward, shared by
 * the CPU generator (synth_cpu.c, gcc) and the GPU generator (synth.cu, nvcc).
 *
 * Both sides must produce the same bytes for the same seed, so every step is
 * integer arithmetic or a single explicitly rounded IEEE fp32 operation:
 *   - uniform bits: the splitmix64 sequence  mix(base + idx * golden_gamma);
 *   - standard normal: piecewise-linear inverse CDF over a 65536-interval
 *     table of fp32 quantiles supplied by the caller (so the table bits are
 *     identical on host and device), which truncates the tails at about
 *     +-4.3 sigma;
 *   - bf16 rounding: round-to-nearest-even on the fp32 bit pattern;
 *   - e4m3 (OCP FP8, "fn": no infinities, 0x7F = NaN) rounding:
 *     round-to-nearest-even with saturation to +-448.
 * The scale of a 128-block is amax / 448 (fp32 division), the convention of
 * the configs in the reference benchmark description (amax-scaled e4m3).
 */
#ifndef MOE_SYNTH_CORE_H
#define MOE_SYNTH_CORE_H

#include <stdint.h>

#ifdef __CUDACC__
#define SYN_FN static __host__ __device__ __forceinline__
#else
#define SYN_FN static inline
#endif

#define SYN_TABLE_BITS 16
#define SYN_TABLE_N (1u << SYN_TABLE_BITS) /* intervals; table has N+1 entries */

/* Stream identifiers: one independent sequence per tensor kind. */
enum {
  SYN_LOGITS = 1,
  SYN_BIAS = 2,
  SYN_HIDDEN = 3,
  SYN_W13 = 4,
  SYN_W2 = 5
};

SYN_FN uint64_t syn_mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

/* Base of the sequence for (seed, stream, sub) where sub is e.g. an expert id. */
SYN_FN uint64_t syn_base(uint64_t seed, uint32_t stream, uint32_t sub) {
  return syn_mix64(syn_mix64(seed * 0x9E3779B97F4A7C15ull + stream) ^
                   ((uint64_t)sub * 0xD1B54A32D192ED03ull + 0x632BE59BD9B4E019ull));
}

SYN_FN uint32_t syn_u32(uint64_t base, uint64_t idx) {
  return (uint32_t)(syn_mix64(base + (idx + 1) * 0x9E3779B97F4A7C15ull) >> 32);
}

SYN_FN float syn_fmul(float a, float b) {
#ifdef __CUDA_ARCH__
  return __fmul_rn(a, b);
#else
  return a * b;
#endif
}
SYN_FN float syn_fadd(float a, float b) {
#ifdef __CUDA_ARCH__
  return __fadd_rn(a, b);
#else
  return a + b;
#endif
}
SYN_FN float syn_fsub(float a, float b) {
#ifdef __CUDA_ARCH__
  return __fsub_rn(a, b);
#else
  return a - b;
#endif
}
SYN_FN float syn_fdiv(float a, float b) {
#ifdef __CUDA_ARCH__
  return __fdiv_rn(a, b);
#else
  return a / b;
#endif
}

SYN_FN uint32_t syn_f2u(float f) {
#ifdef __CUDA_ARCH__
  return __float_as_uint(f);
#else
  union { float f; uint32_t u; } v; v.f = f; return v.u;
#endif
}
SYN_FN float syn_u2f(uint32_t u) {
#ifdef __CUDA_ARCH__
  return __uint_as_float(u);
#else
  union { float f; uint32_t u; } v; v.u = u; return v.f;
#endif
}

/* Standard normal sample from 32 uniform bits and the quantile table. */
SYN_FN float syn_normal(const float* table, uint32_t u) {
  uint32_t i = u >> (32 - SYN_TABLE_BITS);
  float frac = (float)(u & ((1u << (32 - SYN_TABLE_BITS)) - 1u)) *
               (1.0f / (float)(1u << (32 - SYN_TABLE_BITS)));
  float lo = table[i];
  float d = syn_fsub(table[i + 1], lo);
  return syn_fadd(lo, syn_fmul(frac, d));
}

/* fp32 -> bf16 bits, round to nearest even (finite inputs). */
SYN_FN uint16_t syn_bf16_bits(float x) {
  uint32_t b = syn_f2u(x);
  b += 0x7FFFu + ((b >> 16) & 1u);
  return (uint16_t)(b >> 16);
}
SYN_FN float syn_bf16_round(float x) { return syn_u2f((uint32_t)syn_bf16_bits(x) << 16); }

/* fp32 -> e4m3fn byte, round to nearest even, saturating to +-448. */
SYN_FN uint8_t syn_e4m3(float x) {
  uint32_t b = syn_f2u(x);
  uint8_t sign = (uint8_t)((b >> 24) & 0x80u);
  uint32_t a = b & 0x7FFFFFFFu;
  if (a >= 0x43E80000u) return (uint8_t)(sign | 0x7Eu); /* |x| >= 464: saturate */
  int e = (int)(a >> 23) - 127;
  if (e < -6) {
    /* subnormal range: value = m * 2^-9, m in 0..8 (8 carries into the min normal) */
    uint32_t mant = (a & 0x7FFFFFu) | (a ? 0x800000u : 0u); /* 24-bit significand */
    int shift = -e + 14; /* a * 2^9 = mant * 2^(e-23+9) -> integer part mant >> (14 - e) */
    if (a == 0 || shift > 31) return sign;
    uint32_t m = mant >> shift;
    uint32_t rem = mant & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (m & 1u))) m += 1;
    return (uint8_t)(sign | m); /* m == 8 encodes exponent field 1, mantissa 0 = 2^-6 */
  }
  uint32_t mant = a & 0x7FFFFFu;
  uint32_t r = mant >> 20;
  uint32_t rem = mant & 0xFFFFFu;
  if (rem > 0x80000u || (rem == 0x80000u && (r & 1u))) r += 1;
  if (r == 8) { r = 0; e += 1; }
  uint32_t code = ((uint32_t)(e + 7) << 3) | r;
  if (code > 0x7Eu) code = 0x7Eu;
  return (uint8_t)(sign | code);
}

#endif /* MOE_SYNTH_CORE_H */
