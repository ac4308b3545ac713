// Per-token attention prologue (forward.h:554-575) for sm_100a:
//   q: per-head weighted RMSNorm (rms_per_head, forward.h:138-140), then NEOX
//      RoPE (rope_apply, attn.h:19-28) -> q_out;
//   k: per-head weighted RMSNorm, NEOX RoPE -> cache slot;
//   v: plain RMSNorm over all nkv*hd values (rmsnorm_plain, norm.h:82-96)
//      when v_norm is set -> cache slot.
// One warp per head.  Sums of squares keep the reference's 16 fused
// accumulators (norm.h:10-18) and its reduction tree, so they are
// bit-identical to the reference's; the inverse square root is the correctly
// rounded 1/sqrt (the reference's -ffast-math build may use an rsqrt
// estimate there, an ulp-level difference).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "ptx.cuh"

namespace molot {

struct AppendArgs {
  // Inputs of sequence b: q [nq][D] at q_in + b*q_bstride; k, v [nkv][D] at
  // k_in / v_in + b*kv_in_bstride.
  const float* q_in;
  long long q_bstride;
  const float* k_in;
  const float* v_in;
  long long kv_in_bstride;
  float* q_out;  // [nq][D] per sequence, stride qo_bstride
  long long qo_bstride;
  const float* q_norm;  // [D] or null
  const float* k_norm;  // [D] or null
  int v_norm;
  float eps;
  const float* freq;  // [D/2] or null (NoPE)
  int nq, nkv;
  // Position and cache slot of the new token.
  int pos, slot;                            // when seq_pos is null
  // Several tokens of one sequence (prefill, forward.h:368-392): entry b
  // is the token at position pos + b*tok_step, written to slot
  // slot + b*tok_step (tok_step 0: one token per sequence).
  int tok_step;
  const int* seq_pos;                       // [B] or null
  const int* seq_slot;                      // [B] or null
  // Cache addressing (same conventions as DecodeArgs; elements of the
  // kernel's cache type).
  void* K;
  void* V;
  long long kv_bstride, stride_t, stride_h;
  const int* block_table;
  int bt_stride, page_size;
  long long page_stride, page_hstride;
};

constexpr int kAppendWarps = 4;

// Sum of squares of x[0..n) in the order of the reference's 16-lane FMA
// accumulators followed by _mm512_reduce_add_ps; every lane returns it.
__device__ __forceinline__ float warp_sumsq16(const float* x, int n, int lane) {
  const int a = lane & 15;
  float acc = 0.f;
#pragma unroll 8
  for (int i = a; i + 16 - a <= n; i += 16) acc = __fmaf_rn(x[i], x[i], acc);
  acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 8));
  acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 4));
  acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 2));
  acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 1));
  return acc;
}

// The cache's storage of a computed value: FP32 as is, BF16 rounded to
// nearest even.
__device__ __forceinline__ void cache_store(float* p, float x) { *p = x; }
__device__ __forceinline__ void cache_store(__nv_bfloat16* p, float x) {
  *p = __float2bfloat16_rn(x);
}

template <class CT>
__device__ __forceinline__ CT* cache_row(const AppendArgs& a, CT* base, int b, int g, int slot,
                                         int D) {
  if (a.block_table) {
    const int p = a.block_table[(long long)b * a.bt_stride + slot / a.page_size];
    return base + (long long)p * a.page_stride + (long long)g * a.page_hstride +
           (long long)(slot % a.page_size) * D;
  }
  return base + (long long)b * a.kv_bstride + (long long)slot * a.stride_t +
         (long long)g * a.stride_h;
}

template <int D, class CT = float>
__global__ void __launch_bounds__(kAppendWarps * 32)
    norm_rope_append_kernel(const __grid_constant__ AppendArgs a) {
  static_assert(D % 16 == 0, "head dim must be a multiple of 16");
  constexpr int H = D / 2;
  // Programmatic dependent launch: the next launch (the decode) may start at
  // once -- it streams only KV rows older than the one written here until it
  // waits for this grid.  Everything this kernel reads or writes comes after
  // the wait for the preceding grid.
  if (threadIdx.x == 0) ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int head = blockIdx.x * kAppendWarps + warp;
  const int b = blockIdx.y;
  if (head >= a.nq + a.nkv) return;
  const int pos = a.seq_pos ? a.seq_pos[b] : a.pos + b * a.tok_step;

  const bool is_q = head < a.nq;
  const int g = is_q ? head : head - a.nq;
  const float* x = is_q ? a.q_in + (long long)b * a.q_bstride + (long long)g * D
                        : a.k_in + (long long)b * a.kv_in_bstride + (long long)g * D;
  const float* w = is_q ? a.q_norm : a.k_norm;
  const int slot = is_q ? 0 : (a.seq_slot ? a.seq_slot[b] : a.slot + b * a.tok_step);
  float* qdst = is_q ? a.q_out + (long long)b * a.qo_bstride + (long long)g * D : nullptr;
  CT* kdst = is_q ? nullptr : cache_row(a, static_cast<CT*>(a.K), b, g, slot, D);

  float inv = 1.f;
  if (w) {
    const float ss = warp_sumsq16(x, D, lane);
    inv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), a.eps)));
  }
  for (int i = lane; i < H; i += 32) {
    float y0 = x[i], y1 = x[i + H];
    if (w) {
      y0 = __fmul_rn(__fmul_rn(y0, inv), w[i]);
      y1 = __fmul_rn(__fmul_rn(y1, inv), w[i + H]);
    }
    if (a.freq) {
      const float ang = __fmul_rn((float)pos, a.freq[i]);
      float s, c;
      sincosf(ang, &s, &c);
      const float z0 = __fsub_rn(__fmul_rn(y0, c), __fmul_rn(y1, s));
      const float z1 = __fadd_rn(__fmul_rn(y0, s), __fmul_rn(y1, c));
      y0 = z0;
      y1 = z1;
    }
    if (is_q) {
      qdst[i] = y0;
      qdst[i + H] = y1;
    } else {
      cache_store(kdst + i, y0);
      cache_store(kdst + i + H, y1);
    }
  }

  if (!is_q) {
    const float* vin = a.v_in + (long long)b * a.kv_in_bstride;
    float vinv = 1.f;
    if (a.v_norm) {
      const int nv = a.nkv * D;
      const float ss = warp_sumsq16(vin, nv, lane);
      vinv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)nv), a.eps)));
    }
    CT* vdst = cache_row(a, static_cast<CT*>(a.V), b, g, slot, D);
    const float* vh = vin + (long long)g * D;
    for (int i = lane; i < D; i += 32)
      cache_store(vdst + i, a.v_norm ? __fmul_rn(vh[i], vinv) : vh[i]);
  }
}

}  // namespace molot

namespace molot {

// Bulk write of nrows [nkv*D] FP32 rows (k and v, row pitch nkv*D) into
// slots slot0.. of a head-major cache (slot t of head g at base +
// g*stride_h + t*D) in the cache's element type; one CTA per (row, head).
template <class CT>
__global__ void kv_rows_to_cache_kernel(const float* __restrict__ k, const float* __restrict__ v,
                                        CT* kc, CT* vc, int slot0, int nkv, int D,
                                        long long stride_h) {
  const int r = blockIdx.x, g = blockIdx.y;
  const float* ks = k + ((long long)r * nkv + g) * D;
  const float* vs = v + ((long long)r * nkv + g) * D;
  const long long off = (long long)g * stride_h + (long long)(slot0 + r) * D;
  for (int j = threadIdx.x; j < D; j += blockDim.x) {
    cache_store(kc + off + j, ks[j]);
    cache_store(vc + off + j, vs[j]);
  }
}

}  // namespace molot
