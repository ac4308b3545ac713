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
// One launch: every CTA first issues the loads of its rows' first weight
// groups, then waits for the preceding launch (x may be its output),
// quantizes x into shared memory (per group the 16 even and the 16 odd int8
// values, the scale, the sum of the 32 values; every CTA repeats this small
// step, which keeps the GEMV one launch), and finishes its rows: a warp owns
// two rows, each lane one 16-byte group of nibbles per row and step (a warp
// reads 512 contiguous bytes per row), 8 dp4a per group.  Reading weights
// before the wait is safe because the launch that precedes a GEMV on the
// stream does not write weights: the library's kernels release their
// dependents only after their own wait, and a kernel without that release
// completes before this one starts.  HBM-bound: cols/2 + 5*cols/32 bytes per
// row.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "ptx.cuh"

namespace molot {

constexpr int kGemvWarps = 8;  // per CTA (three CTAs fit an SM, so a grid is one wave)
constexpr int kGemvRowsPerWarp = 2;
constexpr int kGemvRows = kGemvWarps * kGemvRowsPerWarp;  // per CTA
constexpr int kGemvBatch = 4;  // groups per lane in flight per row

struct Q8Packed {  // one 32-value activation group
  int evens[4];    // q[0], q[2], ..., q[30] as bytes
  int odds[4];     // q[1], q[3], ..., q[31]
};

struct GemvQ4Args {
  const float* scales;  // [rows][ng]
  const int8_t* zeros;  // [rows][ng]
  const uint8_t* data;  // [rows][cols/2]
  const float* x;       // [cols]
  float* y;             // [rows]
  int rows, cols, ng;
};

// Shared memory of a CTA: packed groups, then scales, then sums.
__host__ __device__ constexpr int gemv_smem_bytes(int ng) { return ng * (int)sizeof(Q8Packed) + ng * 8; }

__global__ void __launch_bounds__(kGemvWarps * 32, 3) gemv_q4_kernel(const __grid_constant__ GemvQ4Args a) {
  extern __shared__ __align__(16) unsigned char gsm[];
  Q8Packed* xq = reinterpret_cast<Q8Packed*>(gsm);
  float* xs = reinterpret_cast<float*>(gsm + a.ng * sizeof(Q8Packed));
  int* xsum = reinterpret_cast<int*>(xs + a.ng);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r0 = blockIdx.x * kGemvRows + warp * kGemvRowsPerWarp;

  // ---- first weight batch of this warp's rows, before the wait
  uint4 w[kGemvRowsPerWarp][kGemvBatch];
  float s[kGemvRowsPerWarp][kGemvBatch];
  int z[kGemvRowsPerWarp][kGemvBatch];
  auto load_batch = [&](int g0) {
#pragma unroll
    for (int rr = 0; rr < kGemvRowsPerWarp; ++rr) {
      const int r = r0 + rr;
#pragma unroll
      for (int u = 0; u < kGemvBatch; ++u) {
        const int g = g0 + 32 * u;
        if (r < a.rows && g < a.ng) {
          w[rr][u] = __ldcs(reinterpret_cast<const uint4*>(a.data + (long long)r * (a.cols / 2)) + g);
          s[rr][u] = __ldcs(a.scales + (long long)r * a.ng + g);
          z[rr][u] = __ldcs(a.zeros + (long long)r * a.ng + g);
        }
      }
    }
  };
  load_batch(lane);

  // ---- x may be the preceding launch's output
  ptx::pdl_wait();
  if (threadIdx.x == 0) ptx::pdl_launch_dependents();

  // ---- quantize x (gemm.h:44-70): 8 lanes per group, 4 values per lane
  {
    const int j = lane & 7;  // lane of the group: elements 4j..4j+3
    // warp-uniform trip count: the shuffles below need every lane
    for (int gb = warp * 4; gb < a.ng; gb += kGemvWarps * 4) {
      const int g = gb + (lane >> 3);
      const bool ok = g < a.ng;
      const float4 t = ok ? reinterpret_cast<const float4*>(a.x + (long long)g * 32)[j]
                          : make_float4(0.f, 0.f, 0.f, 0.f);
      float amax = fmaxf(fmaxf(fabsf(t.x), fabsf(t.y)), fmaxf(fabsf(t.z), fabsf(t.w)));
#pragma unroll
      for (int off = 4; off > 0; off >>= 1)
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
      float sx = __fdiv_rn(amax, 127.0f);
      if (!(sx > 0.f)) sx = 1.0f;
      sx = __half2float(__float2half_rn(sx));  // the reference stores fp16 scales
      int q[4];
      const float vv[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        int v = (int)roundf(__fdiv_rn(vv[e], sx));  // half away from zero
        q[e] = v > 127 ? 127 : (v < -127 ? -127 : v);
      }
      int sum = q[0] + q[1] + q[2] + q[3];
#pragma unroll
      for (int off = 4; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      // element 4j+e -> evens slot 2j + e/2 (e even), odds slot 2j + e/2 (e odd)
      if (!ok) continue;
      reinterpret_cast<uint16_t*>(xq[g].evens)[j] = (uint16_t)((q[0] & 0xff) | ((q[2] & 0xff) << 8));
      reinterpret_cast<uint16_t*>(xq[g].odds)[j] = (uint16_t)((q[1] & 0xff) | ((q[3] & 0xff) << 8));
      if (j == 0) {
        xs[g] = sx;
        xsum[g] = sum;
      }
    }
  }
  __syncthreads();

  // ---- rows
  float acc[kGemvRowsPerWarp];
#pragma unroll
  for (int rr = 0; rr < kGemvRowsPerWarp; ++rr) acc[rr] = 0.f;
  for (int g0 = lane; g0 < a.ng; g0 += 32 * kGemvBatch) {
    if (g0 != lane) load_batch(g0);
#pragma unroll
    for (int u = 0; u < kGemvBatch; ++u) {
      const int g = g0 + 32 * u;
      if (g >= a.ng) continue;
      const Q8Packed p = xq[g];
      const float sxg = xs[g];
      const int sumg = xsum[g];
#pragma unroll
      for (int rr = 0; rr < kGemvRowsPerWarp; ++rr) {
        const uint32_t ws[4] = {w[rr][u].x, w[rr][u].y, w[rr][u].z, w[rr][u].w};
        int dot = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          dot = __dp4a((int)(ws[i] & 0x0F0F0F0Fu), p.evens[i], dot);
          dot = __dp4a((int)((ws[i] >> 4) & 0x0F0F0F0Fu), p.odds[i], dot);
        }
        const int G = dot - z[rr][u] * sumg;  // sum((nibble - zero) * q), exact
        acc[rr] += (float)G * s[rr][u] * sxg;
      }
    }
  }
#pragma unroll
  for (int rr = 0; rr < kGemvRowsPerWarp; ++rr) {
    float v = acc[rr];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if (lane == 0 && r0 + rr < a.rows) a.y[r0 + rr] = v;
  }
}

}  // namespace molot
