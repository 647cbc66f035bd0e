// The six bf16 planes a tensor-core linear reads its f32 share activations from, and the device
// helpers that write them: each share split exactly into three bf16 terms, columns in the weight
// blocks' order.
#pragma once

#include <cuda_bf16.h>

#include <cstddef>
#include <cstdint>

namespace shd {

// The six bf16 planes a tensor-core linear reads ([share * 3 + term][Mp][KP], columns in the
// weight blocks' order), as a destination another kernel can write directly.
struct PlaneOut {  // plain data (it sits in kernel argument unions): value-initialise it, PlaneOut{}
  uint16_t* p;
  int Mp, KP;
};

// Physical column of logical column `col` in the planes (inverse of the weight blocks' column
// permutation: chunk of 256, slot l of 4 columns in each half, half).
__host__ __device__ __forceinline__ int plane_phys(int col) {
  const int c = col >> 8, r = col & 255;
  const int hi = r >= 128 ? 1 : 0;
  const int rr = r - 128 * hi;
  return c * 256 + (rr >> 2) * 8 + 4 * hi + (rr & 3);
}

// Exact three-term bf16 split of v: v = b0 + b1 + b2.
__device__ __forceinline__ void split3(float v, uint16_t (&b)[3]) {
  const __nv_bfloat16 b0 = __float2bfloat16_rn(v);
  const float r1 = __fsub_rn(v, __bfloat162float(b0));
  const __nv_bfloat16 b1 = __float2bfloat16_rn(r1);
  const float r2 = __fsub_rn(r1, __bfloat162float(b1));
  b[0] = __bfloat16_as_ushort(b0);
  b[1] = __bfloat16_as_ushort(b1);
  b[2] = __bfloat16_as_ushort(__float2bfloat16_rn(r2));
}

// Both shares (vc, vs) of row m, logical column col, into the planes.
__device__ __forceinline__ void planes_store(const PlaneOut& o, int m, int col, float vc, float vs) {
  const size_t plane = (size_t)o.Mp * o.KP;
  const size_t at = (size_t)m * o.KP + plane_phys(col);
  uint16_t b[3];
  split3(vc, b);
#pragma unroll
  for (int t = 0; t < 3; ++t) o.p[(size_t)t * plane + at] = b[t];
  split3(vs, b);
#pragma unroll
  for (int t = 0; t < 3; ++t) o.p[(size_t)(3 + t) * plane + at] = b[t];
}

}  // namespace shd
