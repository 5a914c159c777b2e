/*
 * One-time weight packing (the role of pack_w13 / pack_w2, kernels/moe.cu:164-208):
 * FP8 weights are rearranged into the exact shared-memory images the GEMM kernels consume,
 * so each pipeline stage is one contiguous bulk copy and no tensor map is needed.
 *
 *   W13 [E, 4096, 7168] -> [E, 16 j, 56 kb, 256 rows, 128 B], rows 0..127 = W13 rows
 *       128j.. (X1 part), rows 128..255 = W13 rows 2048+128j.. (X2 part); each 32 KB block is
 *       K-major with the 128-byte swizzle (16-byte chunk c of row r stored at c ^ (r & 7)).
 *   W2  [E, 7168, 2048] -> [E, 28 nt, 16 ib, 256 rows, 128 B], rows = W2 rows 256nt.. .
 * Byte count is unchanged; the scales keep the reference layout.
 */
#pragma once
#include "moe_common.cuh"

namespace moe {

__global__ void __launch_bounds__(256) pack_w13_kernel(const uint8_t* __restrict__ w13, int E,
                                                       uint8_t* __restrict__ out) {
  // One thread per 16-byte chunk, ordered (e, j, row, k-chunk) so reads are contiguous.
  const size_t total = static_cast<size_t>(E) * G1_NT * 256 * (H / 16);
  for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int qk = static_cast<int>(idx % (H / 16));
    size_t t = idx / (H / 16);
    const int rho = static_cast<int>(t % 256);
    t /= 256;
    const int j = static_cast<int>(t % G1_NT);
    const int e = static_cast<int>(t / G1_NT);
    const int kb = qk >> 3, c = qk & 7;
    const int srow = rho < 128 ? 128 * j + rho : I + 128 * j + (rho - 128);
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(w13 + (static_cast<size_t>(e) * G1N + srow) * H) + qk);
    const size_t blk = ((static_cast<size_t>(e) * G1_NT + j) * HB + kb) * (2 * TILE_BYTES);
    *reinterpret_cast<uint4*>(out + blk + rho * 128 + ((c ^ (rho & 7)) << 4)) = v;
  }
}

__global__ void __launch_bounds__(256) pack_w2_kernel(const uint8_t* __restrict__ w2, int E,
                                                      uint8_t* __restrict__ out) {
  const size_t total = static_cast<size_t>(E) * G2_NT * 256 * (I / 16);
  for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int qk = static_cast<int>(idx % (I / 16));
    size_t t = idx / (I / 16);
    const int rho = static_cast<int>(t % 256);
    t /= 256;
    const int nt = static_cast<int>(t % G2_NT);
    const int e = static_cast<int>(t / G2_NT);
    const int ib = qk >> 3, c = qk & 7;
    const int srow = 256 * nt + rho;
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(w2 + (static_cast<size_t>(e) * H + srow) * I) + qk);
    const size_t blk = ((static_cast<size_t>(e) * G2_NT + nt) * IB + ib) * (2 * TILE_BYTES);
    *reinterpret_cast<uint4*>(out + blk + rho * 128 + ((c ^ (rho & 7)) << 4)) = v;
  }
}

}  // namespace moe
