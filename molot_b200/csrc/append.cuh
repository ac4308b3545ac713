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
#include <type_traits>

#include "ptx.cuh"

namespace molot {

// Q8 KV storage (the reduced format the reference's design names for its
// KV cache, DESIGN.md:48,87-88, left unimplemented there): a row of D
// values is D int8 followed by D/32 FP32 scales, one per 32 consecutive
// values, padded to a multiple of 16 bytes.  Each 32-value block is
// quantized with the reference's Q8 rule (quant.h:33-43, quantize_q8_row:
// s = absmax/127, 1 when that is not > 0; q = nearbyint(x/s) clamped to
// [-127, 127]) as the reference's -ffast-math build evaluates it: s =
// absmax * (1/127) and x/s = x * (127/absmax), each a correctly rounded FP32
// operation.  A value reads back as (float)q * s.  Strides and offsets of a
// Q8 cache count bytes.
struct Q8Row {};
static_assert(sizeof(Q8Row) == 1, "Q8 row pointers step in bytes");
__host__ __device__ constexpr int q8_row_bytes(int D) { return (D + D / 8 + 15) & ~15; }

// Row pitch of a cache in its stride units (elements; bytes for Q8).
template <class CT>
__host__ __device__ constexpr int row_pitch(int D) {
  return std::is_same<CT, Q8Row>::value ? q8_row_bytes(D) : D;
}

// One 32-value block held by a full warp (lane = element of the block):
// returns this lane's code, the block's scale in s.
__device__ __forceinline__ int q8_quantize(float x, float& s) {
  float amax = fabsf(x);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  s = __fmul_rn(amax, 0x1.020408p-7f);  // the FP32 value of 1/127
  if (!(s > 0.f)) {  // an all-zero block
    s = 1.0f;
    return 0;
  }
  const int v = __float2int_rn(__fmul_rn(x, __fdiv_rn(127.0f, amax)));  // ties to even
  return v > 127 ? 127 : (v < -127 ? -127 : v);
}

__device__ __forceinline__ void q8_put(unsigned char* row, int D, int block, int lane, int q,
                                       float s) {
  row[32 * block + lane] = (unsigned char)(signed char)q;
  if (lane == 0) *reinterpret_cast<float*>(row + D + 4 * block) = s;
}

// Quantizes block `block` of a row from one value per lane and stores it.
__device__ __forceinline__ void q8_store_block(float x, unsigned char* row, int D, int block,
                                               int lane) {
  float s;
  const int q = q8_quantize(x, s);
  q8_put(row, D, block, lane, q, s);
}

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
           (long long)(slot % a.page_size) * row_pitch<CT>(D);
  }
  return base + (long long)b * a.kv_bstride + (long long)slot * a.stride_t +
         (long long)g * a.stride_h;
}

template <int D, class CT = float>
__global__ void __launch_bounds__(kAppendWarps * 32)
    norm_rope_append_kernel(const __grid_constant__ AppendArgs a) {
  static_assert(D % 16 == 0, "head dim must be a multiple of 16");
  constexpr bool kQ8 = std::is_same<CT, Q8Row>::value;
  static_assert(!kQ8 || D % 64 == 0, "Q8 rows: both halves must be whole 32-value blocks");
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
    } else if constexpr (kQ8) {  // H % 32 == 0: the loop is warp-uniform
      unsigned char* row = reinterpret_cast<unsigned char*>(kdst);
      q8_store_block(y0, row, D, i >> 5, lane);
      q8_store_block(y1, row, D, (i + H) >> 5, lane);
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
    for (int i = lane; i < D; i += 32) {
      const float y = a.v_norm ? __fmul_rn(vh[i], vinv) : vh[i];
      if constexpr (kQ8)
        q8_store_block(y, reinterpret_cast<unsigned char*>(vdst), D, i >> 5, lane);
      else
        cache_store(vdst + i, y);
    }
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

// The same bulk write into a Q8 cache (row pitch q8_row_bytes(D), stride_h
// in bytes): one CTA of D threads per (row, head), warp w quantizes block w.
template <class CT>
__global__ void kv_rows_to_cache_q8_kernel(const float* __restrict__ k,
                                           const float* __restrict__ v, unsigned char* kc,
                                           unsigned char* vc, int slot0, int nkv, int D,
                                           long long stride_h) {
  static_assert(std::is_same<CT, Q8Row>::value, "Q8 caches only");
  const int r = blockIdx.x, g = blockIdx.y;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long src = ((long long)r * nkv + g) * D + threadIdx.x;
  const long long off = (long long)g * stride_h + (long long)(slot0 + r) * q8_row_bytes(D);
  q8_store_block(k[src], kc + off, D, w, lane);
  q8_store_block(v[src], vc + off, D, w, lane);
}

}  // namespace molot
