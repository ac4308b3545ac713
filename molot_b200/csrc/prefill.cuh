// Causal / sliding-window GQA prefill attention (gemm.h:409-446,
// attn_prefill_gqa, called at forward.h:396): M new queries at positions
// pos0..pos0+M-1 against the filled cache [0, N).  Query m of head h attends
// slots [t0, nn): nn = min(pos+1, N), t0 = max(0, pos-window+1) (window > 0)
// capped at N; an empty range yields zeros, as the reference's.
//
// One CTA = one kv head x 64 query rows (kPrefillRows / G positions, all G
// query heads of the kv head: each K/V row staged in shared memory serves
// every grouped head).  FP32 on the CUDA cores -- the reference's contract is
// FP32 to 1e-5 -- flash-attention style: a producer warp streams key tiles of
// BN slots through a two-stage shared-memory ring (one TMA bulk copy per K or
// V row, rows padded by 4 floats so the column reads of K are bank-conflict
// free; full/empty mbarriers per stage); the 8 consumer warps each own 8
// query rows (two groups of 16 lanes, 4 rows each): per tile S = Q K^T in
// registers (4 rows x BN/16 keys per thread), an online softmax in base 2, P
// to the warp's own rows of shared memory, O += P V in registers (4 rows x
// D/16 dims per thread).  No CTA-wide barrier runs inside the key loop: a
// warp only reads P it wrote itself, and stages are recycled through the
// empty barriers.  Grid: (query blocks, nkv), the longest (latest) query
// blocks first.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math_constants.h>

#include <cstdint>
#include <type_traits>

#include "append.cuh"
#include "ptx.cuh"

namespace molot {

constexpr int kPrefillConsumers = 256;  // 16 x 16: ty owns 4 rows, tx a column set
constexpr int kPrefillThreads = kPrefillConsumers + 32;  // + one producer warp
constexpr int kPrefillRows = 64;      // query rows (position, head) per CTA

// Four consecutive cache elements as floats (FP32 or BF16 storage).
__device__ __forceinline__ float4 load4(const float* p) {
  return *reinterpret_cast<const float4*>(p);
}
__device__ __forceinline__ float4 load4(const __nv_bfloat16* p) {
  const uint2 w = *reinterpret_cast<const uint2*>(p);
  return make_float4(__uint_as_float(w.x << 16), __uint_as_float(w.x & 0xffff0000u),
                     __uint_as_float(w.y << 16), __uint_as_float(w.y & 0xffff0000u));
}

// BF16 and Q8 caches (Q8Row, append.cuh): the raw rows of a tile arrive
// through the same ring and are expanded once per tile into FP32 tiles by
// the 256 consumer threads (bf16 values exactly; Q8 values as
// (float)code * scale, exactly as the quantizer defines them); the score
// and output loops then run on those tiles unchanged, instead of converting
// every value in their inner loops.
template <int D, class KT = float>
struct PrefillTile {
  static constexpr bool kQ8 = std::is_same<KT, Q8Row>::value;
  static constexpr bool kExpand = !std::is_same<KT, float>::value;  // expanded FP32 tiles
  static constexpr int EB = sizeof(KT);  // bytes per stride unit
  static constexpr int RB = kQ8 ? q8_row_bytes(D) : D * EB;  // bytes of a cache row
  static constexpr int BN = D > 128 ? 32 : 64;  // keys per tile
  static constexpr int NJ = BN / 16;            // score columns per thread
  static constexpr int LD = D + 4;              // padded Q row pitch (floats)
  static constexpr int LDK = (RB + 16) / EB;    // padded K/V row pitch (elements, +16 B)
  static constexpr int LDF = D + 4;             // expanded FP32 tile pitch (floats)
  static constexpr int PLD = BN + 4;            // P row pitch (floats)
  static constexpr int kQ = kPrefillRows * LD * 4;
  static constexpr int kKV = BN * LDK * EB;  // one K or V tile as it arrives
  static constexpr int kF = kExpand ? BN * LDF * 4 : 0;  // one expanded K or V tile
  static constexpr int kP = kPrefillRows * PLD * 4;
  static constexpr int kBars = 5 * 8;  // full[2], empty[2], q
  static constexpr int kTotal = kQ + 4 * kKV + 2 * kF + kP + kBars + 16;
  static_assert(kTotal <= 227 * 1024, "prefill CTA exceeds the shared-memory limit");
  static_assert(D % 64 == 0, "head dim must be a multiple of 64");
};

struct PrefillArgs {
  const float* Q;  // query m, head h: Q + m*q_tstride + h*D
  long long q_tstride;
  float* O;  // same layout, o_tstride
  long long o_tstride;
  const void* K;  // slot t of kv head g: K + t*stride_t + g*stride_h (elements)
  const void* V;
  long long stride_t, stride_h;
  int nq, nkv, G, M, N, pos0, window;
  float scale;
  int BP;      // query positions per CTA (kPrefillRows / G)
  int nblk_m;  // ceil(M / BP)
  int* status;
  unsigned long long timeout_ns;
};

__device__ __forceinline__ float prefill_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int D, class KT = float>
__global__ void __launch_bounds__(kPrefillThreads, 1)
    gqa_prefill_kernel(const __grid_constant__ PrefillArgs a) {
  using TP = PrefillTile<D, KT>;
  constexpr int BN = TP::BN, NJ = TP::NJ, LD = TP::LD, LDK = TP::LDK, PLD = TP::PLD;
  // the type and pitch of the tiles the score / output loops read
  using CT = typename std::conditional<TP::kExpand, float, KT>::type;
  constexpr int LDC = TP::kExpand ? TP::LDF : LDK;
  constexpr int DJ = D / 64;  // float4 groups of output columns per thread
  constexpr float kLog2e = 1.4426950408889634f;

  extern __shared__ __align__(128) unsigned char smem[];
  float* Qs = reinterpret_cast<float*>(smem);
  KT* KVs = reinterpret_cast<KT*>(smem + TP::kQ);  // [stage][K,V][BN][LDK]
  float* KVf = reinterpret_cast<float*>(smem + TP::kQ + 4 * TP::kKV);  // [K,V][BN][LDF]
  float* Ps = reinterpret_cast<float*>(smem + TP::kQ + 4 * TP::kKV + 2 * TP::kF);
  uint64_t* full =
      reinterpret_cast<uint64_t*>(smem + TP::kQ + 4 * TP::kKV + 2 * TP::kF + TP::kP);
  uint64_t* empty = full + 2;
  uint64_t* q_bar = full + 4;
  volatile int* abort_sm = reinterpret_cast<volatile int*>(full + 5);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int ty = tid >> 4, tx = tid & 15;  // a warp = two ty rows of 16 lanes
  const int g = blockIdx.y;
  const int mb = a.nblk_m - 1 - blockIdx.x;  // latest (longest) query blocks first
  const int G = a.G;

  if (tid == 0) {
    ptx::mbar_init(full + 0, 1);
    ptx::mbar_init(full + 1, 1);
    ptx::mbar_init(empty + 0, kPrefillConsumers / 32);
    ptx::mbar_init(empty + 1, kPrefillConsumers / 32);
    ptx::mbar_init(q_bar, 1);
    *abort_sm = 0;
    ptx::fence_mbar_init();
  }
  __syncthreads();
  // Inputs (q, the cache rows) may come from the preceding launch.
  ptx::pdl_wait();
  if (tid == 0) ptx::pdl_launch_dependents();

  // Block geometry: rows r = m_local*G + h_local.
  const int m_first = mb * a.BP;
  const int m_end = min(a.M, m_first + a.BP);
  auto row_t0 = [&](int m) {
    const int pos = a.pos0 + m;
    int t0 = (a.window > 0 && pos - a.window + 1 > 0) ? pos - a.window + 1 : 0;
    return t0 < a.N ? t0 : a.N;
  };
  auto row_nn = [&](int m) { return min(a.pos0 + m + 1, a.N); };
  const int t_lo = row_t0(m_first);
  const int t_hi = row_nn(m_end - 1);
  const int ntiles = t_hi > t_lo ? (t_hi - t_lo + BN - 1) / BN : 0;
  const int valid_rows = (m_end - m_first) * G;

  if (warp == kPrefillConsumers / 32) {
    // ---- producer warp: Q once, then the key tiles through the ring
    const uint64_t pol = ptx::policy_evict_first();
    if (lane == 0) ptx::mbar_arrive_expect_tx(q_bar, (uint32_t)valid_rows * D * 4u);
    __syncwarp();
    for (int r = lane; r < valid_rows; r += 32) {
      const int m = m_first + r / G, h = g * G + r % G;
      ptx::bulk_g2s(Qs + (size_t)r * LD, a.Q + (long long)m * a.q_tstride + (long long)h * D,
                    D * 4u, q_bar, pol);
    }
    for (int i = 0; i < ntiles; ++i) {
      const int stage = i & 1;
      if (i >= 2 && !ptx::mbar_wait_bounded(empty + stage, ((i >> 1) - 1) & 1, a.timeout_ns)) {
        if (lane == 0) {  // the results of this launch are void: say so now
          *abort_sm = 1;
          atomicCAS(a.status, 0, 3);
        }
      }
      __syncwarp();
      const int ts = t_lo + i * BN;
      const int rows = min(BN, t_hi - ts);
      KT* Kd = KVs + (size_t)(stage * 2) * BN * LDK;
      KT* Vd = Kd + (size_t)BN * LDK;
      if (lane == 0) ptx::mbar_arrive_expect_tx(full + stage, (uint32_t)rows * TP::RB * 2u);
      __syncwarp();
      for (int c = lane; c < rows; c += 32) {
        const long long off = (long long)(ts + c) * a.stride_t + (long long)g * a.stride_h;
        ptx::bulk_g2s(Kd + (size_t)c * LDK, static_cast<const KT*>(a.K) + off, TP::RB,
                      full + stage, pol);
        ptx::bulk_g2s(Vd + (size_t)c * LDK, static_cast<const KT*>(a.V) + off, TP::RB,
                      full + stage, pol);
      }
    }
    return;
  }

  // Per-row state (4 rows per thread, replicated over the 16 tx lanes).
  int rt0[4], rnn[4];
  float mrow[4], lrow[4];
  float o[4][DJ * 4];
#pragma unroll
  for (int ii = 0; ii < 4; ++ii) {
    const int r = ty * 4 + ii;
    const int m = m_first + r / G;
    const bool ok = r < valid_rows;
    rt0[ii] = ok ? row_t0(m) : 0;
    rnn[ii] = ok ? row_nn(m) : 0;  // invalid rows attend nothing
    mrow[ii] = -CUDART_INF_F;
    lrow[ii] = 0.f;
#pragma unroll
    for (int j = 0; j < DJ * 4; ++j) o[ii][j] = 0.f;
  }
  bool ok_waits = ptx::mbar_wait_bounded(q_bar, 0, a.timeout_ns);

  const float sl2 = a.scale * kLog2e;
  for (int i = 0; i < ntiles; ++i) {
    const int stage = i & 1;
    // A timed-out wait leaves this thread computing on stale data; the
    // results are then discarded (status word) and every loop still ends.
    ok_waits &= ptx::mbar_wait_bounded(full + stage, (i >> 1) & 1, a.timeout_ns);
    const CT* Kt;
    const CT* Vt;
    if constexpr (TP::kExpand) {
      // Every consumer is done with the previous expanded tiles; expand
      // this tile (4 values per task), publish, and hand the raw stage back
      // to the producer at once.
      ptx::named_bar_sync(1, kPrefillConsumers);
      const unsigned char* raw =
          reinterpret_cast<const unsigned char*>(KVs + (size_t)(stage * 2) * BN * LDK);
      constexpr int kWords = BN * D / 4;
      for (int w = tid; w < 2 * kWords; w += kPrefillConsumers) {
        const int kv = w / kWords, rem = w - kv * kWords;
        const int row = rem / (D / 4), c4 = rem - row * (D / 4);
        float4 f;
        if constexpr (TP::kQ8) {
          const unsigned char* rp = raw + (size_t)(kv * BN + row) * LDK;
          const uint32_t code = *reinterpret_cast<const uint32_t*>(rp + 4 * c4) ^ 0x80808080u;
          const float sc = *reinterpret_cast<const float*>(rp + D + 4 * (c4 >> 3));
          // code + 128 in the low mantissa bits of 2^23, minus 2^23 + 128
          f.x = __fmul_rn(__fsub_rn(__uint_as_float(__byte_perm(code, 0x4B000000u, 0x7650u)), 8388736.f), sc);
          f.y = __fmul_rn(__fsub_rn(__uint_as_float(__byte_perm(code, 0x4B000000u, 0x7651u)), 8388736.f), sc);
          f.z = __fmul_rn(__fsub_rn(__uint_as_float(__byte_perm(code, 0x4B000000u, 0x7652u)), 8388736.f), sc);
          f.w = __fmul_rn(__fsub_rn(__uint_as_float(__byte_perm(code, 0x4B000000u, 0x7653u)), 8388736.f), sc);
        } else {  // bf16: 4 values in 8 bytes
          f = load4(KVs + (size_t)(stage * 2 + kv) * BN * LDK + (size_t)row * LDK + 4 * c4);
        }
        *reinterpret_cast<float4*>(KVf + (size_t)(kv * BN + row) * LDC + 4 * c4) = f;
      }
      ptx::named_bar_sync(1, kPrefillConsumers);
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(empty + stage);
      Kt = KVf;
      Vt = KVf + (size_t)BN * LDC;
    } else {
      Kt = KVs + (size_t)(stage * 2) * BN * LDK;
      Vt = Kt + (size_t)BN * LDK;
    }
    const int ts = t_lo + i * BN;
    const int kc = min(BN, t_hi - ts);

    // ---- S = Q K^T for rows ty*4+ii, keys tx+16j
    float s[4][NJ];
#pragma unroll
    for (int ii = 0; ii < 4; ++ii)
#pragma unroll
      for (int j = 0; j < NJ; ++j) s[ii][j] = 0.f;
    const float* qb = Qs + (size_t)(ty * 4) * LD;
    const CT* kb = Kt + (size_t)tx * LDC;
#pragma unroll 4
    for (int k = 0; k < D; k += 4) {
      float4 qv[4], kv[NJ];
#pragma unroll
      for (int ii = 0; ii < 4; ++ii) qv[ii] = *reinterpret_cast<const float4*>(qb + ii * LD + k);
#pragma unroll
      for (int j = 0; j < NJ; ++j)
        kv[j] = load4(kb + (size_t)(16 * j) * LDC + k);
#pragma unroll
      for (int ii = 0; ii < 4; ++ii)
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
          s[ii][j] = fmaf(qv[ii].x, kv[j].x, s[ii][j]);
          s[ii][j] = fmaf(qv[ii].y, kv[j].y, s[ii][j]);
          s[ii][j] = fmaf(qv[ii].z, kv[j].z, s[ii][j]);
          s[ii][j] = fmaf(qv[ii].w, kv[j].w, s[ii][j]);
        }
    }

    // ---- online softmax (base 2), P to shared memory
#pragma unroll
    for (int ii = 0; ii < 4; ++ii) {
      float tmax = -CUDART_INF_F;
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const int t = ts + tx + 16 * j;
        const bool ok = t >= rt0[ii] && t < rnn[ii];
        s[ii][j] = ok ? s[ii][j] * sl2 : -CUDART_INF_F;
        tmax = fmaxf(tmax, s[ii][j]);
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1)
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
      const float mnew = fmaxf(mrow[ii], tmax);
      const float alpha = (mrow[ii] == -CUDART_INF_F) ? 0.f : prefill_ex2(mrow[ii] - mnew);
      float psum = 0.f;
      float* prow = Ps + (size_t)(ty * 4 + ii) * PLD;
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const float p = (s[ii][j] == -CUDART_INF_F) ? 0.f : prefill_ex2(s[ii][j] - mnew);
        psum += p;
        prow[tx + 16 * j] = p;
      }
      lrow[ii] = lrow[ii] * alpha + psum;  // this lane's share of the row sum
      mrow[ii] = mnew;
#pragma unroll
      for (int j = 0; j < DJ * 4; ++j) o[ii][j] *= alpha;
    }
    __syncwarp();  // P rows ty*4.. are written and read by this warp only

    // ---- O += P V over the kc valid keys of the tile
    const float* pb = Ps + (size_t)(ty * 4) * PLD;
    int c = 0;
    for (; c + 4 <= kc; c += 4) {
      float4 pv[4];
#pragma unroll
      for (int ii = 0; ii < 4; ++ii) pv[ii] = *reinterpret_cast<const float4*>(pb + ii * PLD + c);
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        const CT* vr = Vt + (size_t)(c + cc) * LDC + tx * 4;
#pragma unroll
        for (int jj = 0; jj < DJ; ++jj) {
          const float4 v4 = load4(vr + 64 * jj);
#pragma unroll
          for (int ii = 0; ii < 4; ++ii) {
            const float p = cc == 0 ? pv[ii].x : cc == 1 ? pv[ii].y : cc == 2 ? pv[ii].z : pv[ii].w;
            o[ii][jj * 4 + 0] = fmaf(p, v4.x, o[ii][jj * 4 + 0]);
            o[ii][jj * 4 + 1] = fmaf(p, v4.y, o[ii][jj * 4 + 1]);
            o[ii][jj * 4 + 2] = fmaf(p, v4.z, o[ii][jj * 4 + 2]);
            o[ii][jj * 4 + 3] = fmaf(p, v4.w, o[ii][jj * 4 + 3]);
          }
        }
      }
    }
    for (; c < kc; ++c) {  // ragged end of the last tile
      const CT* vr = Vt + (size_t)c * LDC + tx * 4;
#pragma unroll
      for (int jj = 0; jj < DJ; ++jj) {
        const float4 v4 = load4(vr + 64 * jj);
#pragma unroll
        for (int ii = 0; ii < 4; ++ii) {
          const float p = pb[ii * PLD + c];
          o[ii][jj * 4 + 0] = fmaf(p, v4.x, o[ii][jj * 4 + 0]);
          o[ii][jj * 4 + 1] = fmaf(p, v4.y, o[ii][jj * 4 + 1]);
          o[ii][jj * 4 + 2] = fmaf(p, v4.z, o[ii][jj * 4 + 2]);
          o[ii][jj * 4 + 3] = fmaf(p, v4.w, o[ii][jj * 4 + 3]);
        }
      }
    }
    __syncwarp();  // this warp's P rows may be rewritten by the next tile
    if (!TP::kExpand && lane == 0) ptx::mbar_arrive(empty + stage);
  }
  if (!ok_waits || *abort_sm) {
    atomicCAS(a.status, 0, 3);
    return;
  }

  // ---- epilogue: full row sums, normalise, store
#pragma unroll
  for (int ii = 0; ii < 4; ++ii) {
    float l = lrow[ii];
#pragma unroll
    for (int off = 1; off < 16; off <<= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
    const int r = ty * 4 + ii;
    if (r >= valid_rows) continue;
    const int m = m_first + r / G, h = g * G + r % G;
    const float inv = l > 0.f ? 1.f / l : 0.f;  // empty range: zeros (gemm.h:431-436)
    float* dst = a.O + (long long)m * a.o_tstride + (long long)h * D + tx * 4;
#pragma unroll
    for (int jj = 0; jj < DJ; ++jj) {
      float4 v;
      v.x = o[ii][jj * 4 + 0] * inv;
      v.y = o[ii][jj * 4 + 1] * inv;
      v.z = o[ii][jj * 4 + 2] * inv;
      v.w = o[ii][jj * 4 + 3] * inv;
      *reinterpret_cast<float4*>(dst + 64 * jj) = v;
    }
  }
}

}  // namespace molot
