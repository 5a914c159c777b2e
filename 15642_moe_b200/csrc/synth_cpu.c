/*
 * CPU generator of the seeded synthetic MoE inputs (see synth_core.h for the
 * bit-exact recipe). Built with gcc -O2 -fopenmp -ffp-contract=off into
 * libmoe_synth_cpu.so; the GPU twin lives in synth.cu. Both produce identical
 * bytes for the same seed, so CPU-side checkers (the oracle) and the device
 * path consume the same inputs without copying weights through PCIe.
 *
 * Layouts (the reference oracle's, reference/moe_ref.py:44-52):
 *   logits      fp32 [T, 256]
 *   bias        bf16 [256]
 *   hidden      e4m3 [T, 7168],  hidden_scale fp32 [56, T]  (block-major)
 *   w13         e4m3 [E, 4096, 7168], w13_scale fp32 [E, 32, 56]
 *   w2          e4m3 [E, 7168, 2048], w2_scale  fp32 [E, 56, 16]
 * Expert e of a weight tensor is drawn from the stream (seed, kind, e0 + e),
 * so a slice of the global 256-expert layer can be generated on its own.
 */
#include <stdint.h>
#include <stddef.h>
#include <math.h>
#include "synth_core.h"

#define H_DIM 7168
#define I_DIM 2048

void moe_synth_cpu_logits(const float* table, uint64_t seed, int T, int E, float* out) {
  uint64_t base = syn_base(seed, SYN_LOGITS, 0);
  long n = (long)T * E;
#pragma omp parallel for schedule(static)
  for (long i = 0; i < n; ++i) out[i] = syn_normal(table, syn_u32(base, (uint64_t)i));
}

void moe_synth_cpu_bias(const float* table, uint64_t seed, int E, float stddev,
                        const int* hot, int n_hot, float hot_value, uint16_t* out) {
  uint64_t base = syn_base(seed, SYN_BIAS, 0);
  for (int e = 0; e < E; ++e) {
    float v = syn_fmul(stddev, syn_normal(table, syn_u32(base, (uint64_t)e)));
    for (int h = 0; h < n_hot; ++h)
      if (hot[h] == e) v = hot_value;
    out[e] = syn_bf16_bits(v);
  }
}

/* Quantise one row block of 128 values (already bf16-rounded) to e4m3. */
static float quant_block(const float* v, int n, int stride, uint8_t* q) {
  float amax = 0.0f;
  for (int i = 0; i < n; ++i) {
    float a = fabsf(v[(long)i * stride]);
    if (a > amax) amax = a;
  }
  float scale = amax > 0.0f ? syn_fdiv(amax, 448.0f) : 1.0f;
  for (int i = 0; i < n; ++i) q[(long)i * stride] = syn_e4m3(syn_fdiv(v[(long)i * stride], scale));
  return scale;
}

void moe_synth_cpu_hidden(const float* table, uint64_t seed, int T, float stddev,
                          uint8_t* hidden, float* hidden_scale) {
  uint64_t base = syn_base(seed, SYN_HIDDEN, 0);
  const int nkb = H_DIM / 128;
#pragma omp parallel for schedule(static)
  for (int t = 0; t < T; ++t) {
    float row[H_DIM];
    for (int h = 0; h < H_DIM; ++h)
      row[h] = syn_bf16_round(
          syn_fmul(stddev, syn_normal(table, syn_u32(base, (uint64_t)t * H_DIM + h))));
    for (int kb = 0; kb < nkb; ++kb)
      hidden_scale[(long)kb * T + t] =
          quant_block(row + kb * 128, 128, 1, hidden + (long)t * H_DIM + kb * 128);
  }
}

/* One weight matrix [rows, cols] of expert `sub` quantised per 128x128 block. */
static void weight_matrix(const float* table, uint64_t base, int rows, int cols, float stddev,
                          uint8_t* q, float* scale) {
  const int rb = rows / 128, cb = cols / 128;
#pragma omp parallel for schedule(static)
  for (int blk = 0; blk < rb * cb; ++blk) {
    int br = blk / cb, bc = blk % cb;
    static __thread float v[128 * 128];
    for (int r = 0; r < 128; ++r)
      for (int c = 0; c < 128; ++c) {
        uint64_t idx = (uint64_t)(br * 128 + r) * cols + (uint64_t)(bc * 128 + c);
        v[r * 128 + c] = syn_bf16_round(syn_fmul(stddev, syn_normal(table, syn_u32(base, idx))));
      }
    float amax = 0.0f;
    for (int i = 0; i < 128 * 128; ++i) {
      float a = fabsf(v[i]);
      if (a > amax) amax = a;
    }
    float s = amax > 0.0f ? syn_fdiv(amax, 448.0f) : 1.0f;
    for (int r = 0; r < 128; ++r)
      for (int c = 0; c < 128; ++c)
        q[(long)(br * 128 + r) * cols + bc * 128 + c] = syn_e4m3(syn_fdiv(v[r * 128 + c], s));
    scale[br * cb + bc] = s;
  }
}

void moe_synth_cpu_w13(const float* table, uint64_t seed, int e0, int E, float stddev,
                       uint8_t* w13, float* w13_scale) {
  for (int e = 0; e < E; ++e)
    weight_matrix(table, syn_base(seed, SYN_W13, (uint32_t)(e0 + e)), 2 * I_DIM, H_DIM, stddev,
                  w13 + (long)e * 2 * I_DIM * H_DIM, w13_scale + (long)e * 32 * 56);
}

void moe_synth_cpu_w2(const float* table, uint64_t seed, int e0, int E, float stddev,
                      uint8_t* w2, float* w2_scale) {
  for (int e = 0; e < E; ++e)
    weight_matrix(table, syn_base(seed, SYN_W2, (uint32_t)(e0 + e)), H_DIM, I_DIM, stddev,
                  w2 + (long)e * H_DIM * I_DIM, w2_scale + (long)e * 56 * 16);
}
