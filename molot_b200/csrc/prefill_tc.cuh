// Causal / sliding-window GQA prefill attention on the 5th-generation tensor
// cores (tcgen05), for FP32 caches at head_dim 64 and 128: the same
// contract as gqa_prefill_kernel (gemm.h:409-446, attn_prefill_gqa at
// forward.h:396) within the 1e-5 bar.
//
// Precision.  Both products keep FP32 accuracy by splitting operands:
//   S = Q K^T in split FP16.  Every query row and every key row is scaled
//     by a power of two (exact) so that its largest magnitude lies in
//     [2^14, 2^15); a scaled value x becomes h0 = fp16(x) and h1 = fp16(x -
//     h0) (x - h0 is exact in FP32), and S is formed as h0.h0 + h0.h1 +
//     h1.h0 by three kind::f16 MMAs accumulating in FP32.  The dropped h1.h1
//     term is ~2^-22 of the product; values below 2^-17 of their row's
//     largest keep an absolute error under 2^-39 of it.  The softmax undoes
//     both scales exactly before it applies the attention scale.
//   O += P V in split TF32: hi = round-to-nearest TF32 of x, lo = x - hi,
//     hi.hi + hi.lo + lo.hi by three kind::tf32 MMAs (P <= 2^8 and V are
//     used unscaled).
// FP16 pairs pack two K elements per 32-bit tensor-memory column, so Q's
// two halves take D columns in all and 64-key tiles fit: an S MMA costs the
// same issue time at N = 64 as at N = 32, so a key costs half the S issue
// time of 32-key tiles.
//
// CTA: one kv head x 128 query rows (row r = position (r / G) of the block,
// head (r % G) of the kv head's group), the MMA's M.  Tensor memory (512
// columns, all of the SM's): Q h0 / h1 (the A operand of S, D/2 columns
// each), two S buffers (BN columns each), P hi / lo (the A operand of O),
// the O accumulator (D columns); a thread of the softmax warpgroup owns its
// row's lane, so row maxima and sums never leave the thread.
// Warps:
//   0-3  softmax: Q row -> TMEM (scaled, split), then per key tile: S row
//        from TMEM, both scales and the attention scale, causal / window
//        mask, lazy online softmax in base 2 (the running max rises only
//        when a score exceeds it by 2^8; O is then rescaled in TMEM), P ->
//        TMEM (split); at the end O / l -> global.
//   4-11 converters: per key tile, K and V rows from global (L2-resident
//        across the query blocks; issued before the stage is free), each
//        key's scale (its largest magnitude, reduced over the four lanes
//        holding the key), K split in FP16 and V in TF32, into shared
//        memory in the no-swizzle K-major core-matrix layouts the MMAs read
//        (K as [key][dim], V transposed as [dim][key]), plus the keys'
//        inverse scales; 2 stages.
//   12   lane 0 issues the S MMAs (Q K^T) and their commits;
//   13   lane 0 issues the P V MMAs and theirs, in parallel with warp 12's.
// Barriers (all waits bounded; a wait that runs out records a status code,
// raises the abort flag and the CTA winds down without further MMAs):
//   kv_full / kv_empty per stage, s_full / s_free per S buffer, p_full,
//   pv_done, q_ready, done (the last commit, before TMEM is freed).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math_constants.h>

#include <cstdint>

#include "prefill.cuh"
#include "ptx.cuh"

namespace molot {

constexpr int kTcRows = 128;     // query rows per CTA (MMA M)
constexpr int kTcBN = 64;        // keys per tile (the S MMA's N)
constexpr int kTcStages = 2;     // K/V tile stages
constexpr int kTcConvWarps = 8;  // converter warps (4..11)
constexpr int kTcThreads = (4 + kTcConvWarps + 2) * 32;
constexpr int kTcTmemCols = 512;

template <int D>
struct TcShape {
  static_assert(D == 64 || D == 128, "tensor-core prefill: head_dim 64 or 128");
  static constexpr int BN = kTcBN;
  static constexpr int kKTile = BN * D * 2;  // one FP16 half (h0 or h1) of a K tile (bytes)
  // V tiles are transposed: 4-key chunks (leading byte offset kVChunk) of
  // 8-dim core matrices 160 bytes apart (stride byte offset), with a
  // 16-byte gap after each chunk, so the 32 lanes of a converter warp's
  // scalar stores (8 keys x 4 dim groups) fall on 32 different banks.
  static constexpr int kVSbo = 160;  // bytes between 8-dim core matrices of a 4-key chunk
  static constexpr int kVChunk = (D / 8) * kVSbo + 16;
  static constexpr int kVTile = (BN / 4) * kVChunk;  // one TF32 half of a V tile
  static constexpr int kKInv = BN * 4;               // the keys' inverse scales (floats)
  static constexpr int kStage = 2 * kKTile + 2 * kVTile + kKInv;
  static constexpr int kBarOff = kTcStages * kStage;
  static constexpr int kBars = 2 * kTcStages + 4 + 4;  // kv_full/empty, s_full/free x2, p, pv, q, done
  // Over half of the SM's shared memory, so a second CTA (which would wait
  // in tcgen05.alloc for the first one's 512 columns) never shares the SM.
  static constexpr int kUsed = kBarOff + kBars * 8 + 32;
  static constexpr int kTotal = kUsed > 116 * 1024 ? kUsed : 116 * 1024;
  // tensor-memory columns
  static constexpr uint32_t kQ0 = 0, kQ1 = D / 2, kS = D, kPhi = D + 2 * BN, kPlo = kPhi + BN,
                            kO = kPlo + BN;
  static_assert(kO + D <= kTcTmemCols, "tensor memory columns");
  static_assert(kTotal <= 227 * 1024, "shared memory");
  static_assert(kStage % 16 == 0 && kKTile % 16 == 0 && kVTile % 16 == 0, "16-byte operands");
  // K tile half, K-major B of S (N = keys, K = dims): core matrix = 8 keys x
  // 8 FP16 dims (16-byte rows)
  __device__ static int k_off(int key, int dim) {
    return (dim >> 3) * (BN * 16) + (key >> 3) * 128 + (key & 7) * 16 + (dim & 7) * 2;
  }
  // V tile half transposed, K-major B of O (N = dims, K = keys): 8 dims x 4 keys
  __device__ static int v_off(int key, int dim) {
    return (key >> 2) * kVChunk + (dim >> 3) * kVSbo + (dim & 7) * 16 + (key & 3) * 4;
  }
};

// Power-of-two exponent e that brings a largest magnitude m into [2^14,
// 2^15) (0 for m == 0), kept within the range where 2^e and 2^-e are normal.
__device__ __forceinline__ int fp16_split_exp(float m) {
  const int ex = (int)((__float_as_uint(m) >> 23) & 0xff);
  if (ex == 0) return m == 0.f ? 0 : 126;
  const int e = 141 - ex;
  return e > 126 ? 126 : (e < -126 ? -126 : e);
}
__device__ __forceinline__ float exp2i(int e) { return __uint_as_float((uint32_t)(e + 127) << 23); }
// Two scaled values y -> their FP16 high parts h0 (packed, y.x in the low
// half) and residual parts h1 = fp16(y - h0) (y - h0 exact in FP32).
__device__ __forceinline__ void fp16_split2(float2 y, uint32_t& h0, uint32_t& h1) {
  const __half2 a = __float22half2_rn(y);
  const float2 af = __half22float2(a);
  const __half2 b = __float22half2_rn(make_float2(y.x - af.x, y.y - af.y));
  h0 = *reinterpret_cast<const uint32_t*>(&a);
  h1 = *reinterpret_cast<const uint32_t*>(&b);
}

namespace tc {

// Round to nearest TF32, ties away from zero (cvt.rna.tf32.f32), in integer
// arithmetic on the bit pattern: add half of the dropped 13 bits' weight to
// the magnitude, then clear them (a carry moves into the exponent, as the
// rounding does).  Finite inputs only.
__device__ __forceinline__ float tf32_hi(float x) {
  return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xffffe000u);
}

// Shared-memory matrix descriptor, no swizzle (sm_100 layout: start, leading
// and stride byte offsets in 16-byte units, version 1).
__device__ __forceinline__ uint64_t sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((addr >> 4) & 0x3fff) | ((uint64_t)((lbo >> 4) & 0x3fff) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3fff) << 32) | (1ull << 46);
}
// Instruction descriptor: TF32 x TF32 -> F32, both K-major, M = 128.
__host__ __device__ constexpr uint32_t idesc(int n) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(kTcRows >> 4) << 24);
}
// Instruction descriptor: F16 x F16 -> F32, both K-major, M = 128.
__host__ __device__ constexpr uint32_t idesc16(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kTcRows >> 4) << 24);
}
// D[tmem] (+)= A[tmem] * B[smem desc], FP16 operands (A: two per column)
__device__ __forceinline__ void mma16(uint32_t d, uint32_t a, uint64_t b, uint32_t id, int acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(d),
      "r"(a), "l"(b), "r"(id), "r"(acc), "r"(0u));
}
// D[tmem] (+)= A[tmem] * B[smem desc], TF32 operands
__device__ __forceinline__ void mma(uint32_t d, uint32_t a, uint64_t b, uint32_t id, int acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(d),
      "r"(a), "l"(b), "r"(id), "r"(acc), "r"(0u));
}
__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   ptx::smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// 16 columns of this thread's lane, starting at addr.
__device__ __forceinline__ void ld16(uint32_t addr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(addr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void st16(uint32_t addr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16};" ::"r"(addr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15]))
      : "memory");
}
__device__ __forceinline__ void wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

}  // namespace tc

// Waits for `bar` to complete phase `par`, bounded by a.timeout_ns; on
// timeout records `code` and raises the abort flag.  Skipped once aborted.
__device__ __forceinline__ void tc_wait(uint64_t* bar, uint32_t par, const PrefillArgs& a,
                                        volatile int* abort_flag, int code) {
  if (*abort_flag) return;
  if (!ptx::mbar_wait_bounded(bar, par, a.timeout_ns)) {
    *abort_flag = 1;
    atomicCAS(a.status, 0, code);
  }
}

template <int D>
__global__ void __launch_bounds__(kTcThreads, 1)
    gqa_prefill_tc_kernel(const __grid_constant__ PrefillArgs a) {
  using TS = TcShape<D>;
  constexpr int BN = kTcBN;
  constexpr float kLog2e = 1.4426950408889634f;
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + TS::kBarOff);
  uint64_t* kv_full = bars;
  uint64_t* kv_empty = bars + kTcStages;
  uint64_t* s_full = bars + 2 * kTcStages;
  uint64_t* s_free = s_full + 2;
  uint64_t* p_full = s_full + 4;
  uint64_t* pv_done = p_full + 1;
  uint64_t* q_ready = p_full + 2;
  uint64_t* done_bar = p_full + 3;
  volatile uint32_t* tmem_sm = reinterpret_cast<volatile uint32_t*>(bars + TS::kBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + TS::kBars) + 1;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = blockIdx.y;
  const int mb = a.nblk_m - 1 - blockIdx.x;  // latest (longest) query blocks first
  const int G = a.G;
  const int BP = kTcRows / G;  // query positions per CTA
  const int m0 = mb * BP;
  // Keys the CTA attends: from the first position's window start to the
  // last position's causal end (capped at N).
  const int m_last = min(m0 + BP, a.M) - 1;
  const int pos_first = a.pos0 + m0, pos_last = a.pos0 + m_last;
  const int lo_key = a.window > 0 ? max(0, pos_first - a.window + 1) : 0;
  const int hi_key = min(pos_last + 1, a.N);
  const int kt0 = (lo_key / BN) * BN;
  const int ntiles = hi_key > kt0 ? (hi_key - kt0 + BN - 1) / BN : 0;

  if (tid == 0) {
    for (int i = 0; i < kTcStages; ++i) {
      ptx::mbar_init(kv_full + i, kTcConvWarps * 32);
      ptx::mbar_init(kv_empty + i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(s_full + i, 1);
      ptx::mbar_init(s_free + i, 128);
    }
    ptx::mbar_init(p_full, 128);
    ptx::mbar_init(pv_done, 1);
    ptx::mbar_init(q_ready, 128);
    ptx::mbar_init(done_bar, 2);  // one commit per issuing thread
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     ptx::smem_u32(const_cast<uint32_t*>(tmem_sm))),
                 "r"(kTcTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t T = *tmem_sm;
  // Q and the cache rows may come from the preceding launch.
  ptx::pdl_wait();
  if (tid == 0) ptx::pdl_launch_dependents();

  if (warp < 4) {
    // ------------------------------------------------------------ softmax
    const int r = tid;  // this thread's row == TMEM lane
    const uint32_t lane_base = T + ((uint32_t)(warp * 32) << 16);
    const int pl = r / G, h = r - pl * G;
    const int m = m0 + pl;
    const bool valid = pl < BP && m < a.M;
    const int pos = a.pos0 + m;
    const int t_hi = valid ? min(pos + 1, a.N) : 0;  // attended [t_lo, t_hi)
    const int t_lo = a.window > 0 ? max(0, pos - a.window + 1) : 0;
    const float* qrow = a.Q + (long long)m * a.q_tstride + (long long)(g * G + h) * D;
    // The row's scale 2^eq (its largest magnitude into [2^14, 2^15)), then
    // h0 / h1 into columns kQ0 / kQ1, two dims per column.
    int eq;
    {
      float amax = 0.f;
#pragma unroll 1
      for (int c = 0; c < D; c += 4) {
        const float4 x = valid ? *reinterpret_cast<const float4*>(qrow + c)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w))));
      }
      eq = fp16_split_exp(amax);
      const float sq = exp2i(eq);
#pragma unroll 1
      for (int c = 0; c < D; c += 32) {
        float w0[16], w1[16];
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          const float4 x = valid ? *reinterpret_cast<const float4*>(qrow + c + i)
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
          uint32_t a0, a1, b0, b1;
          fp16_split2(make_float2(x.x * sq, x.y * sq), a0, b0);
          fp16_split2(make_float2(x.z * sq, x.w * sq), a1, b1);
          w0[i / 2] = __uint_as_float(a0);
          w0[i / 2 + 1] = __uint_as_float(a1);
          w1[i / 2] = __uint_as_float(b0);
          w1[i / 2 + 1] = __uint_as_float(b1);
        }
        tc::st16(lane_base + TS::kQ0 + c / 2, w0);
        tc::st16(lane_base + TS::kQ1 + c / 2, w1);
      }
      tc::wait_st();
      tc::fence_before();
      ptx::mbar_arrive(q_ready);
    }
    // S * 2^-eq * 2^-ek[key] is the exact FP32 score; sl2 applies the
    // attention scale in base 2 with the single rounding of s * scale.
    const float sl2 = a.scale * kLog2e * exp2i(-eq);
    float mrow = -CUDART_INF_F, lrow = 0.f;
#pragma unroll 1
    for (int j = 0; j < ntiles; ++j) {
      const int sb = j & 1;
      const int st = j % kTcStages;
      tc_wait(s_full + sb, (j >> 1) & 1, a, abort_flag, 1);
      __syncwarp();  // lanes leave the wait loop on their own; tcgen05.ld is warp-collective
      tc::fence_after();
      float s[BN];
#pragma unroll
      for (int c = 0; c < BN; c += 16) tc::ld16(lane_base + TS::kS + sb * BN + c, s + c);
      tc::fence_before();
      ptx::mbar_arrive(s_free + sb);
      // The keys' inverse scales, written by the converters before they
      // released the stage (waited on here for ordering; it cannot refill
      // before this tile's P V completes).
      tc_wait(kv_full + st, (j / kTcStages) & 1, a, abort_flag, 1);
      const float* kinv = reinterpret_cast<const float*>(smem + st * TS::kStage + 2 * TS::kKTile +
                                                         2 * TS::kVTile);
      const int key0 = kt0 + j * BN;
      // s * 2^-ek (exact) then * sl2 (one rounding), two keys per packed
      // multiply; keys outside [t_lo, t_hi) only on the tiles that hold some.
#pragma unroll
      for (int i = 0; i < BN; i += 4) {
        const float4 ki = *reinterpret_cast<const float4*>(kinv + i);
        const float2 a0 = __fmul2_rn(__fmul2_rn(make_float2(s[i], s[i + 1]), make_float2(ki.x, ki.y)),
                                     make_float2(sl2, sl2));
        const float2 a1 = __fmul2_rn(__fmul2_rn(make_float2(s[i + 2], s[i + 3]), make_float2(ki.z, ki.w)),
                                     make_float2(sl2, sl2));
        s[i] = a0.x;
        s[i + 1] = a0.y;
        s[i + 2] = a1.x;
        s[i + 3] = a1.y;
      }
      if (key0 < t_lo || key0 + BN > t_hi) {
#pragma unroll
        for (int i = 0; i < BN; ++i) {
          const int t = key0 + i;
          if (t < t_lo || t >= t_hi) s[i] = -CUDART_INF_F;
        }
      }
      float mc4[4] = {-CUDART_INF_F, -CUDART_INF_F, -CUDART_INF_F, -CUDART_INF_F};
#pragma unroll
      for (int i = 0; i < BN; ++i) mc4[i & 3] = fmaxf(mc4[i & 3], s[i]);
      const float mc = fmaxf(fmaxf(mc4[0], mc4[1]), fmaxf(mc4[2], mc4[3]));
      // Lazy rescale: the running max rises only when a score exceeds it
      // by 2^8 (or is the row's first finite one).  The weights are formed
      // before the wait for the previous tile's P V (they depend on the
      // scores alone); O's rescale and the P stores come after it.
      const bool raise = mc > mrow + 8.f;
      const bool scale_o = raise && j > 0 && lrow > 0.f;
      const float alpha = scale_o ? prefill_ex2(mrow - mc) : 1.f;
      if (raise) mrow = mc;
      if (scale_o) lrow *= alpha;
      float l4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < BN; ++i) {
        s[i] = (s[i] == -CUDART_INF_F) ? 0.f : prefill_ex2(s[i] - mrow);
        l4[i & 3] += s[i];
      }
      lrow += (l4[0] + l4[1]) + (l4[2] + l4[3]);
      // P and O may be touched once the previous tile's P V has completed.
      if (j > 0) {
        tc_wait(pv_done, (j - 1) & 1, a, abort_flag, 2);
        __syncwarp();
        tc::fence_after();
      }
      // tcgen05.ld / st are warp-collective, so when any row of the warp
      // must rescale O the whole warp does it, the other rows with a factor
      // of 1.
      if (__any_sync(0xffffffffu, scale_o)) {
#pragma unroll 1
        for (int c = 0; c < D; c += 16) {
          float o[16];
          tc::ld16(lane_base + TS::kO + c, o);
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] *= alpha;
          tc::st16(lane_base + TS::kO + c, o);
        }
      }
#pragma unroll
      for (int c = 0; c < BN; c += 16) {
        float hi[16], lo[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          hi[i] = tc::tf32_hi(s[c + i]);
          lo[i] = s[c + i] - hi[i];
        }
        tc::st16(lane_base + TS::kPhi + c, hi);
        tc::st16(lane_base + TS::kPlo + c, lo);
      }
      tc::wait_st();
      tc::fence_before();
      ptx::mbar_arrive(p_full);
    }
    if (ntiles > 0) {
      tc_wait(pv_done, (ntiles - 1) & 1, a, abort_flag, 2);
      __syncwarp();
      tc::fence_after();
    }
    // Every lane of the warp reads O (warp-collective); valid rows store.
    float* orow = a.O + (long long)m * a.o_tstride + (long long)(g * G + h) * D;
    const float inv = lrow > 0.f ? 1.f / lrow : 0.f;  // an empty range gives zeros
#pragma unroll 1
    for (int c = 0; c < D; c += 16) {
      float o[16];
      if (ntiles > 0) {
        tc::ld16(lane_base + TS::kO + c, o);
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) o[i] = 0.f;
      }
      if (valid) {
#pragma unroll
        for (int i = 0; i < 16; i += 4)
          *reinterpret_cast<float4*>(orow + c + i) =
              make_float4(o[i] * inv, o[i + 1] * inv, o[i + 2] * inv, o[i + 3] * inv);
      }
    }
  } else if (warp < 4 + kTcConvWarps) {
    // ---------------------------------------------------------- converters
    // Converter warp cw takes keys 8cw..8cw+7 of a tile, four lanes per key:
    // lane l holds dims 4(l%4) + 16i of key 8cw + l/4, so a warp's loads
    // read 64 contiguous bytes of each of its 8 rows and a key's largest
    // magnitude is reduced over its four lanes with two shuffles.  A tile's
    // loads and scales are done before its stage is free.
    constexpr int NI = D / 16;  // float4 chunks of K (and of V) per thread
    static_assert(kTcConvWarps * 8 == BN, "eight keys per converter warp");
    const int key = 8 * (warp - 4) + (lane >> 2);
    const int dq = 4 * (lane & 3);
    const float* Kb = static_cast<const float*>(a.K) + (long long)g * a.stride_h;
    const float* Vb = static_cast<const float*>(a.V) + (long long)g * a.stride_h;
#pragma unroll 1
    for (int j = 0; j < ntiles; ++j) {
      const int st = j % kTcStages;
      const int t = kt0 + j * BN + key;
      float4 kx[NI], vx[NI];
#pragma unroll
      for (int i = 0; i < NI; ++i) {
        const long long row = (long long)t * a.stride_t + dq + 16 * i;
        kx[i] = t < a.N ? *reinterpret_cast<const float4*>(Kb + row) : make_float4(0.f, 0.f, 0.f, 0.f);
        vx[i] = t < a.N ? *reinterpret_cast<const float4*>(Vb + row) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      float am = 0.f;
#pragma unroll
      for (int i = 0; i < NI; ++i)
        am = fmaxf(am, fmaxf(fmaxf(fabsf(kx[i].x), fabsf(kx[i].y)),
                             fmaxf(fabsf(kx[i].z), fabsf(kx[i].w))));
      am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
      am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
      const int ek = fp16_split_exp(am);
      const float sk = exp2i(ek);
      if (j >= kTcStages) tc_wait(kv_empty + st, ((j / kTcStages) - 1) & 1, a, abort_flag, 3);
      unsigned char* base = smem + st * TS::kStage;
      unsigned char* kh0 = base;
      unsigned char* kh1 = base + TS::kKTile;
      unsigned char* vhi = base + 2 * TS::kKTile;
      unsigned char* vlo = vhi + TS::kVTile;
      float* kinv = reinterpret_cast<float*>(vlo + TS::kVTile);
      if (!*abort_flag) {
        if ((lane & 3) == 0) kinv[key] = exp2i(-ek);
#pragma unroll
        for (int i = 0; i < NI; ++i) {
          const int d0 = dq + 16 * i;
          uint32_t a0, a1, b0, b1;
          fp16_split2(make_float2(kx[i].x * sk, kx[i].y * sk), a0, b0);
          fp16_split2(make_float2(kx[i].z * sk, kx[i].w * sk), a1, b1);
          const int off = TS::k_off(key, d0);
          *reinterpret_cast<uint2*>(kh0 + off) = make_uint2(a0, a1);
          *reinterpret_cast<uint2*>(kh1 + off) = make_uint2(b0, b1);
          const float v4[4] = {vx[i].x, vx[i].y, vx[i].z, vx[i].w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float vh = tc::tf32_hi(v4[e]);
            const int vo = TS::v_off(key, d0 + e);
            *reinterpret_cast<float*>(vhi + vo) = vh;
            *reinterpret_cast<float*>(vlo + vo) = v4[e] - vh;
          }
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      ptx::mbar_arrive(kv_full + st);
    }
  } else if (warp == 4 + kTcConvWarps && lane == 0) {
    // --------------------------------------------------- S = Q K^T issuer
    // Fully unrolled: the descriptors advance by constant offsets (their
    // start-address field never carries: shared-memory offsets stay below
    // 2^18 bytes), so the thread issues at the tensor pipe's rate.
    const uint32_t ids = tc::idesc16(BN);
    tc_wait(q_ready, 0, a, abort_flag, 4);
    tc::fence_after();
#pragma unroll 1
    for (int j = 0; j < ntiles; ++j) {
      const int st = j % kTcStages, sb = j & 1;
      tc_wait(kv_full + st, (j / kTcStages) & 1, a, abort_flag, 4);
      if (j >= 2) tc_wait(s_free + sb, ((j >> 1) - 1) & 1, a, abort_flag, 4);
      tc::fence_after();
      if (!*abort_flag) {
        const uint32_t kb = ptx::smem_u32(smem + st * TS::kStage);
        const uint32_t d = T + TS::kS + sb * BN;
        const uint64_t b0 = tc::sdesc(kb, BN * 16, 128);
        const uint64_t b1 = tc::sdesc(kb + TS::kKTile, BN * 16, 128);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {  // S = Q0 K0 + Q0 K1 + Q1 K0 over dims 16k..16k+15
          const uint64_t step = (uint64_t)((2 * k * (BN * 16)) >> 4);
          tc::mma16(d, T + TS::kQ0 + 8 * k, b0 + step, ids, k > 0);
          tc::mma16(d, T + TS::kQ0 + 8 * k, b1 + step, ids, 1);
          tc::mma16(d, T + TS::kQ1 + 8 * k, b0 + step, ids, 1);
        }
      }
      tc::commit(s_full + sb);
    }
    tc::commit(done_bar);  // arrives once every MMA this thread issued has completed
  } else if (warp == 5 + kTcConvWarps && lane == 0) {
    // ------------------------------------------------------- O += P V issuer
    // A thread of its own, so tile j's P V is issued while the other thread
    // issues tile j+1's S.  kv_empty may follow P V(j) alone: S(j) completed
    // before the softmax released P(j).
    const uint32_t ido = tc::idesc(D);
#pragma unroll 1
    for (int jp = 0; jp < ntiles; ++jp) {
      const int st = jp % kTcStages;
      tc_wait(p_full, jp & 1, a, abort_flag, 4);
      tc::fence_after();
      if (!*abort_flag) {
        const uint32_t vb = ptx::smem_u32(smem + st * TS::kStage + 2 * TS::kKTile);
        const uint64_t bh0 = tc::sdesc(vb, TS::kVChunk, TS::kVSbo);
        const uint64_t bl0 = tc::sdesc(vb + TS::kVTile, TS::kVChunk, TS::kVSbo);
#pragma unroll
        for (int k = 0; k < BN / 8; ++k) {  // O += Ph Vh + Ph Vl + Pl Vh over keys 8k..8k+7
          const uint64_t step = (uint64_t)((2 * k * TS::kVChunk) >> 4);
          tc::mma(T + TS::kO, T + TS::kPhi + 8 * k, bh0 + step, ido, (jp > 0 || k > 0) ? 1 : 0);
          tc::mma(T + TS::kO, T + TS::kPhi + 8 * k, bl0 + step, ido, 1);
          tc::mma(T + TS::kO, T + TS::kPlo + 8 * k, bh0 + step, ido, 1);
        }
      }
      tc::commit(pv_done);
      tc::commit(kv_empty + st);
    }
    tc::commit(done_bar);
  }

  // Tensor memory is freed by the warp that allocated it, after every MMA
  // (done_bar) and every thread's tensor-memory access (the CTA barrier).
  tc::fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after();
    if (!ptx::mbar_wait_bounded(done_bar, 0, a.timeout_ns) && lane == 0)
      atomicCAS(a.status, 0, 5);
    __syncwarp();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(T),
                 "r"(kTcTmemCols));
  }
}

}  // namespace molot
