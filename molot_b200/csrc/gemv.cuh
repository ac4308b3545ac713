// Q4 GEMV (gemm.h:223-254, gemv_q4): y = W x for a weight matrix in the
// reference's Q4 layout (quant.h:70-80: per 32-column group an FP32 scale
// and an int8 zero point, 4-bit values two per byte, element 2j in the low
// nibble of byte j) with the activations quantized once per call to int8
// per 32 values (gemm.h:44-70: scale absmax/127 rounded to fp16, values
// rounded half away from zero).  Per row and group the integer sum
// G = sum((nibble - zero) * q) is exact; y = sum_g (float)G * scale_w *
// scale_x.  The reference adds the groups in order; here each lane sums its
// own groups and the warp adds the lanes, a reassociation of the same terms.
//
// Two launches: q8_quantize_kernel packs the activations (per group: the 16
// even and the 16 odd int8 values as 4 + 4 words, the scale, the sum of the
// 32 values), gemv_q4_kernel streams the weights, one warp per row, each
// lane one 16-byte group of nibbles per step (a warp reads 512 contiguous
// bytes), 8 dp4a per group against the packed activations (L1/L2 hits).
// HBM-bound: cols/2 + 5*cols/32 bytes per row.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "ptx.cuh"

namespace molot {

constexpr int kGemvWarps = 8;

struct Q8Packed {  // one 32-value activation group
  int evens[4];    // q[0], q[2], ..., q[30] as bytes
  int odds[4];     // q[1], q[3], ..., q[31]
};

struct GemvQ4Args {
  const float* scales;   // [rows][ng]
  const int8_t* zeros;   // [rows][ng]
  const uint8_t* data;   // [rows][cols/2]
  const float* x;        // [cols]
  float* y;              // [rows]
  Q8Packed* xq;          // [ng] scratch
  float* xs;             // [ng] activation scales
  int* xsum;             // [ng] sum of the group's q
  int rows, cols, ng;
};

// One warp per activation group.
__global__ void __launch_bounds__(kGemvWarps * 32) q8_quantize_kernel(const __grid_constant__ GemvQ4Args a) {
  ptx::pdl_wait();
  if (threadIdx.x == 0) ptx::pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int g = blockIdx.x * kGemvWarps + (threadIdx.x >> 5);
  if (g >= a.ng) return;
  const float v = a.x[(long long)g * 32 + lane];
  float amax = fabsf(v);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  float xs = __fdiv_rn(amax, 127.0f);
  if (!(xs > 0.f)) xs = 1.0f;
  xs = __half2float(__float2half_rn(xs));  // the reference stores fp16 scales
  int q = (int)roundf(__fdiv_rn(v, xs));    // half away from zero
  q = q > 127 ? 127 : (q < -127 ? -127 : q);
  int sum = q;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
  // lanes 2k and 2k+1 hold elements 2k (even) and 2k+1 (odd): byte k of the
  // evens / odds rows
  __shared__ int8_t stage[kGemvWarps][2][16];
  const int w = threadIdx.x >> 5;
  stage[w][lane & 1][lane >> 1] = (int8_t)q;
  __syncwarp();
  if (lane < 8) {
    const int* src = reinterpret_cast<const int*>(&stage[w][lane >> 2][0]);
    int* dst = (lane >> 2) ? a.xq[g].odds : a.xq[g].evens;
    dst[lane & 3] = src[lane & 3];
  }
  if (lane == 0) {
    a.xs[g] = xs;
    a.xsum[g] = sum;
  }
}

// One warp per row; lane l takes groups l, l+32, ...
__global__ void __launch_bounds__(kGemvWarps * 32) gemv_q4_kernel(const __grid_constant__ GemvQ4Args a) {
  ptx::pdl_wait();  // the packed activations come from the preceding launch
  if (threadIdx.x == 0) ptx::pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int r = blockIdx.x * kGemvWarps + (threadIdx.x >> 5);
  if (r >= a.rows) return;
  const uint8_t* row = a.data + (long long)r * (a.cols / 2);
  const float* sc = a.scales + (long long)r * a.ng;
  const int8_t* zr = a.zeros + (long long)r * a.ng;
  float acc = 0.f;
  for (int g = lane; g < a.ng; g += 32) {
    const uint4 w = __ldcs(reinterpret_cast<const uint4*>(row) + g);  // streamed once
    const float s = __ldcs(sc + g);
    const int z = __ldcs(zr + g);
    const Q8Packed& p = a.xq[g];
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
    int dot = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      dot = __dp4a((int)(ws[i] & 0x0F0F0F0Fu), __ldg(p.evens + i), dot);
      dot = __dp4a((int)((ws[i] >> 4) & 0x0F0F0F0Fu), __ldg(p.odds + i), dot);
    }
    const int G = dot - z * __ldg(a.xsum + g);  // sum((nibble - zero) * q), exact
    acc += (float)G * s * __ldg(a.xs + g);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) a.y[r] = acc;
}

}  // namespace molot
