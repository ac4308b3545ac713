// Split-KV GQA decode attention for sm_100a (flash-decoding, FP32, no tensor
// cores: batch-1 decode is a bandwidth-bound GEMV).
//
// Work decomposition
//   A *segment* is one (sequence b, kv head g) pair; its KV rows are the
//   slots [t0_b, n_b) (t0 > 0 for sliding-window layers, attn.h:137).  Slots
//   are grouped into 16-token *blocks* in absolute slot numbering (block k =
//   slots [16k, 16k+16), so a block never straddles a 16-token page).  All
//   segments' blocks are laid end to end (s = b*nkv + g) and the grid's CTAs
//   take equal contiguous block ranges: CTA c owns [c*NB/grid, (c+1)*NB/grid).
//   A segment that lies inside one CTA is finished there; one that spans CTAs
//   leaves a partial (running max, sum, unnormalised output) per CTA, and the
//   last CTA to finish it (atomic ticket) merges the partials.
//
// CTA structure (one CTA per SM, 8 consumer warps + 1 producer warp)
//   The producer streams tiles of 4 quarters x QR rows of K and V into a ring
//   of STAGES shared-memory stages with TMA bulk copies (one copy per quarter
//   when its rows are contiguous in HBM, one per row otherwise), signalling an
//   mbarrier with the byte count.  Quarters sit 32 bytes apart from one
//   another so the four 8-lane row groups of a warp read distinct banks.
//   A consumer warp works on 4 rows at once, 8 lanes per row: lane l of a row
//   group owns head dimensions {16m + l, 16m + l + 8}, i.e. exactly the two
//   accumulator lanes l and l+8 of the reference's 16-wide FMA dot
//   (gemm.h:17-28).  Each lane runs those two fused-multiply-add chains in
//   the reference's order and the row group finishes with the reference's
//   reduction tree (l+8 locally, then xor 4, 2, 1), so every QK score is
//   bit-identical to dot_fp32_avx512(q, k) * scale (attn.h:144).
//   Softmax is an exp2-based online softmax per row group; row groups, warps
//   and CTAs are merged with the usual (max, sum) rescaling.
//   The same lanes then accumulate p * V for their dimensions.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math_constants.h>

#include <cstdint>
#include <type_traits>

#include "append.cuh"
#include "ptx.cuh"

namespace molot {

constexpr int kBlk = 16;            // partition granularity (tokens)
constexpr int kConsumerWarps = 8;
// Three warpgroups: two of consumers, one whose first warp is the producer.
constexpr int kDecodeThreads = (kConsumerWarps + 4) * 32;
// Register split after launch (384 threads x 168 registers = 64512):
// consumers 256 x 232 + producer group 128 x 40 = 64512.
constexpr int kConsumerRegs = 232;
constexpr int kProducerRegs = 40;
static_assert(2 * 128 * kConsumerRegs + 128 * kProducerRegs <= kDecodeThreads * 168,
              "register split exceeds the launch allocation");
constexpr int kQuarterPadBytes = 32;
// Fused step: raw v values (nkv*D) a CTA stages for the new-row build; above
// this the build reads them from global memory.
constexpr int kMaxStagedV = 8 * kConsumerWarps * 32;

// KV element types of the cache.  FP32 keeps the reference's bit-exact
// score order: lane l8 of a row group owns dims {16m+l8, 16m+l8+8}, the
// reference's accumulator lanes.  BF16 (a storage format the reference
// specifies but does not implement) packs a lane's pair of dims into one
// 32-bit word, {16m+2*l8, 16m+2*l8+1}; its parity is against the reference
// run on the bf16-rounded cache, where only rounding-level order effects
// remain.
template <class KT>
struct KvElem;
template <>
struct KvElem<float> {
  static constexpr int kBytes = 4;
  __device__ __forceinline__ static int dim(int i, int l8) {
    return 16 * (i >> 1) + l8 + 8 * (i & 1);
  }
  template <int D>
  __device__ __forceinline__ static void load2(const float* row, int m, int l8, float& x0,
                                               float& x1) {
    x0 = row[16 * m + l8];
    x1 = row[16 * m + l8 + 8];
  }
  __device__ __forceinline__ static float store(float x) { return x; }
  // The reference's 16-accumulator tree over a row group: this lane holds
  // accumulators l8 (a0) and l8+8 (a1).
  __device__ __forceinline__ static float tree16(float a0, float a1) {
    float t = __fadd_rn(a0, a1);
    t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, 4));
    t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, 2));
    return __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, 1));
  }
};
template <>
struct KvElem<__nv_bfloat16> {
  static constexpr int kBytes = 2;
  __device__ __forceinline__ static int dim(int i, int l8) {
    return 16 * (i >> 1) + 2 * l8 + (i & 1);
  }
  template <int D>
  __device__ __forceinline__ static void load2(const __nv_bfloat16* row, int m, int l8,
                                               float& x0, float& x1) {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(row + 16 * m + 2 * l8);
    x0 = __uint_as_float(w << 16);
    x1 = __uint_as_float(w & 0xffff0000u);
  }
  __device__ __forceinline__ static __nv_bfloat16 store(float x) { return __float2bfloat16_rn(x); }
  // The same tree with this lane holding accumulators 2*l8 (a0) and 2*l8+1
  // (a1): acc[j] + acc[j+8] pairs lanes l8 and l8+4, then xor 2, xor 1, and
  // the last add joins the two components.
  __device__ __forceinline__ static float tree16(float a0, float a1) {
#pragma unroll
    for (int off = 4; off >= 1; off >>= 1) {
      a0 = __fadd_rn(a0, __shfl_xor_sync(0xffffffffu, a0, off));
      a1 = __fadd_rn(a1, __shfl_xor_sync(0xffffffffu, a1, off));
    }
    return __fadd_rn(a0, a1);
  }
};
// Q8 (Q8Row rows, see append.cuh): lane l8 owns dims {32m + 4*l8 + e},
// e = 0..3, of each 32-value block m -- one 32-bit word of codes per block
// -- so a row costs a lane D/32 word loads plus the block scales.  Index i
// of a lane's values is block i/4, e = i%4.
template <>
struct KvElem<Q8Row> {
  static constexpr int kBytes = 1;  // strides count bytes
  __device__ __forceinline__ static int dim(int i, int l8) {
    return 32 * (i >> 2) + 4 * l8 + (i & 3);
  }
  // Values 2m and 2m+1 of this lane: codes e, e+1 (e = 2*(m&1)) of block
  // m/2, each read back as (float)q * s exactly as the quantizer defines
  // (the integer-to-float conversion of a code is exact; it measured 8 %
  // faster on paged Q8 batches than a byte-permute-and-subtract form).
  template <int D>
  __device__ __forceinline__ static void load2(const Q8Row* row, int m, int l8, float& x0,
                                               float& x1) {
    const unsigned char* r = reinterpret_cast<const unsigned char*>(row);
    const int blk = m >> 1;
    const int w = *reinterpret_cast<const int*>(r + 32 * blk + 4 * l8);
    const float s = *reinterpret_cast<const float*>(r + D + 4 * blk);
    const int sh = (m & 1) * 16;
    const float c0 = __int2float_rn((int)(signed char)(w >> sh));
    const float c1 = __int2float_rn((int)(signed char)(w >> (sh + 8)));
    const float2 x = __fmul2_rn(make_float2(c0, c1), make_float2(s, s));
    x0 = x.x;
    x1 = x.y;
  }
};

// Two independent round-to-nearest FMAs in one packed-FP32 instruction
// (sm_100): (d0, d1) += (a0 * b0, a1 * b1).  Each half rounds exactly as
// __fmaf_rn does, so the reference's accumulation order and its bits are
// kept while the consumers issue half the FMA instructions.
__device__ __forceinline__ void fma2(float& d0, float& d1, float a0, float a1, float b0,
                                     float b1) {
  const float2 r = __ffma2_rn(make_float2(a0, a1), make_float2(b0, b1), make_float2(d0, d1));
  d0 = r.x;
  d1 = r.y;
}

// Sum of squares of one q head held in a row group's lane layout, equal bit
// for bit to the reference's (norm.h:10-18: 16 FMA accumulators, accumulator
// j taking dims j, j+16, j+32, ... in order, then the _mm512_reduce_add_ps
// tree pairing j with j+8, then j+4, j+2, j+1).  Every lane of the group
// returns it.
template <int D, class KT>
__device__ __forceinline__ float q_sumsq(const float (&x)[D / 8], int l8) {
  constexpr int DV = D / 16;
  if constexpr (std::is_same<KT, Q8Row>::value) {
    // Accumulator 4*(l8&3)+e takes its even terms (dims 32m + 4*(l8&3) + e)
    // from lane l8&3 and its odd ones (16 further) from lane (l8&3)+4: the
    // two lanes swap values and both run the same chain.
    const bool hi = l8 >= 4;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int mb = 0; mb < D / 32; ++mb) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float own = x[4 * mb + e];
        const float other = __shfl_xor_sync(0xffffffffu, own, 4);
        const float ev = hi ? other : own, od = hi ? own : other;
        acc[e] = __fmaf_rn(ev, ev, acc[e]);
        acc[e] = __fmaf_rn(od, od, acc[e]);
      }
    }
    // j + (j+8): lanes l8 and l8^2; j + (j+4): l8^1; then e + (e+2), e + (e+1).
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      acc[e] = __fadd_rn(acc[e], __shfl_xor_sync(0xffffffffu, acc[e], 2));
      acc[e] = __fadd_rn(acc[e], __shfl_xor_sync(0xffffffffu, acc[e], 1));
    }
    return __fadd_rn(__fadd_rn(acc[0], acc[2]), __fadd_rn(acc[1], acc[3]));
  } else {
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int mm = 0; mm < DV; ++mm) {
      a0 = __fmaf_rn(x[2 * mm], x[2 * mm], a0);
      a1 = __fmaf_rn(x[2 * mm + 1], x[2 * mm + 1], a1);
    }
    return KvElem<KT>::tree16(a0, a1);
  }
}

// Status codes written into the device status word.
constexpr int kDevErrConsumerTimeout = 1;
constexpr int kDevErrProducerTimeout = 2;
constexpr int kDevErrPeerTimeout = 3;

// Ranks of a peer-gather group (one GPU each, NVLink / NVSwitch).
constexpr int kMaxPeers = 8;
// Bound of the producer's final wait for its own copies in flight.  It is
// fixed, whatever the stage-wait bound of the launch: a CTA must never exit
// while a bulk copy into its shared memory is still landing, and copies
// from valid addresses always complete.
constexpr unsigned long long kDrainLimitNs = 2000000000ull;

struct DecodeArgs {
  // Query / output: head h of sequence b at Q + b*q_bstride + h*D.
  const float* Q;
  long long q_bstride;
  float* O;
  long long o_bstride;
  // Keys / values, contiguous form: slot t of kv head g of sequence b at
  // base + b*kv_bstride + t*stride_t + g*stride_h.
  const void* K;  // elements of the kernel's KV type (float or bf16)
  const void* V;
  long long kv_bstride, stride_t, stride_h;  // in elements
  // Paged form (block_table != nullptr): slot t of sequence b lives in page
  // p = block_table[b*bt_stride + t/page_size], row t%page_size, at
  // base + p*page_stride + g*page_hstride + (t%page_size)*D.
  const int* block_table;
  int bt_stride, page_size;
  long long page_stride, page_hstride;
  int nkv, G;
  float scale;
  // Segments.
  int uniform;  // 1: all segments share n / t0 below (single sequence)
  int n, t0;
  const int* seq_n;       // planned: [B]
  const int* seq_t0;      // planned: [B]
  const int* seg_prefix;  // planned: [S+1] global block offset of segment s
  const int* cta_seg;     // planned: [grid] segment holding the CTA's first block
  int S;
  long long NB;
  int nblk_u, blo_u;  // uniform: blocks per segment and first block index
  int grid;  // CTAs of the decode grid (the partition is computed from it)
  // Segment-aligned partition (uniform mode, grid >= S): every CTA works
  // inside one segment -- the first grid%S segments get grid/S+1 CTAs, the
  // rest grid/S -- and splits that segment's blocks evenly with its
  // neighbours.  No CTA then finalises a piece half-way through its range
  // (which stalls its stream and made segment-straddling CTAs the slowest).
  // Otherwise the blocks of all segments are split evenly (stream-K).
  int aligned;
  // Aligned partition: the last CTA of each segment takes a share of
  // (kShareW - tail_w) / kShareW of the others' (it also builds the fused
  // step's new row, which holds slot n-1).  0: equal shares.
  int tail_w;
  // Cluster merge (uniform launches, aligned partition): each segment's CTAs
  // form cl_per_seg thread-block clusters of `cluster` CTAs (grid = S *
  // cl_per_seg * cluster).  A cluster merges its CTAs' partials through
  // distributed shared memory; with one cluster per segment that merge
  // writes the output, otherwise each cluster leaves one partial record and
  // the last cluster to finish (ticket) merges the cl_per_seg records.
  // cluster < 2: off (per-CTA partials, ticket and last-CTA combine).
  int cluster;
  int cl_per_seg;
  // Programmatic dependent launch.  When set, the producer may stream each
  // segment's slots below its newest one (n-1) before the preceding launch
  // has completed: they were written two or more launches earlier (the
  // preceding launch is the append that wrote slot n-1).  When clear, it
  // waits before its first copy.
  int prefetch_old_rows;
  // Fused per-token prologue (forward.h:554-575), single sequence only.  When
  // fused != 0, Q holds the raw q projection and slot n-1 is the new token:
  // the kernel normalises and rotates q in registers, normalises/rotates the
  // new k and v rows, writes them to slot n-1 of K_w / V_w (the writable
  // views of K / V) and attends to them without streaming that slot.
  int fused;
  const float* k_raw;   // [nkv][D]
  const float* v_raw;   // [nkv][D]
  const float* q_norm;  // [D] or null
  const float* k_norm;  // [D] or null
  int v_norm;
  float eps;
  const float* freq;    // [D/2] or null (NoPE)
  int pos;              // RoPE position of the new token
  void* K_w;
  void* V_w;
  // Scratch.
  float* partials;  // [2*grid][partial_record_floats(G, D)]
  int* counters;    // [S] per-segment tickets, zero between launches
  int* status;
  // Bound of every wait for a stage (producer and consumers).
  unsigned long long timeout_ns;
  // Failure-detection test hook (molot_debug_withhold_next): the producer
  // issues no copy and exits, so the consumers' first wait runs out after
  // timeout_ns with nothing in flight.  0 in every normal launch.
  int withhold;
  // Peer gather (molot_paged_decode_gather): when npeer > 0 every final
  // output value goes to all npeer ranks' gathered buffers, peer_O[p] being
  // rank p's copy of what O addresses here (O == peer_O[own rank]).  After
  // its last store the grid's last CTA raises this rank's epoch flag in
  // every rank's buffer (peer_flag[p]); molot_comm_wait waits for them.
  int npeer;
  float* peer_O[kMaxPeers];
  unsigned long long* peer_flag[kMaxPeers];
  unsigned int* done_ctr;      // CTAs finished, zero between launches
  unsigned long long* epoch;   // this rank's launches so far
};

// Final output value: into O, or into every rank's gathered buffer.
__device__ __forceinline__ void put_out(const DecodeArgs& a, float* dst, float v) {
  if (a.npeer == 0) {
    *dst = v;
    return;
  }
  const long long off = dst - a.O;
  for (int p = 0; p < a.npeer; ++p) a.peer_O[p][off] = v;
}

template <int D, class KT = float>
struct TileShape {
  static constexpr bool kQ8 = std::is_same<KT, Q8Row>::value;
  static constexpr int EB = KvElem<KT>::kBytes;  // bytes per stride unit
  static constexpr int RB = kQ8 ? q8_row_bytes(D) : D * EB;  // bytes per row
  static constexpr int RS = RB / (int)sizeof(KT);            // row pitch in KT units
  // rows per quarter (a quarter holds 4.5-8 KB)
  static constexpr int QR =
      kQ8 ? (D > 128 ? 16 : (D > 64 ? 32 : 64)) : ((D > 128) ? 8 : 16) * (4 / EB);
  static constexpr int T = 4 * QR;                            // rows per tile
  static constexpr int TB = T / kBlk;                         // blocks per tile
  static constexpr int QB = QR * RB;                          // quarter bytes
  static constexpr int QSTRIDE = QB + kQuarterPadBytes;  // quarter pitch (bytes)
  static constexpr int KQ = 4 * QSTRIDE;                 // K (or V) part of a stage
  static constexpr int STAGE = 2 * KQ;
  static constexpr int STAGES_RAW = 204800 / STAGE;  // ~200 KB of ring
  static constexpr int STAGES = STAGES_RAW < 2 ? 2 : (STAGES_RAW > 8 ? 8 : STAGES_RAW);
};

template <int D, int GS, class KT = float>
struct DecodeSmem {
  using TS = TileShape<D, KT>;
  static constexpr int kStageBytes = TS::STAGES * TS::STAGE;
  // per-warp outputs for the CTA merge; reused as [256][6] scratch by the
  // cross-CTA combine
  static constexpr int kMergeO =
      4 * (kConsumerWarps * GS * D > 6 * kConsumerWarps * 32 ? kConsumerWarps * GS * D
                                                             : 6 * kConsumerWarps * 32);
  static constexpr int kMergeML = kConsumerWarps * GS * 2 * 4;
  // fused mode: the new k and v rows, then the launch's constants (cos and
  // sin of the RoPE angles [D/2] each, q_norm [D], k_norm [D])
  static constexpr int kNewRow = 2 * D * 4 + 3 * D * 4;
  static constexpr int kBars = 4 * TS::STAGES * 8;  // full and empty, K and V halves
  static constexpr int kTotal = kStageBytes + kMergeO + kMergeML + kNewRow + kBars + 16;
  static_assert(kTotal <= 227 * 1024, "decode CTA exceeds the shared-memory limit");
};

// Floats of one partial record: o[G][D], then m[G], l[G]; padded to a
// multiple of 4 so each record starts 16-byte aligned (float4 reads).
__host__ __device__ constexpr int partial_record_floats(int G, int D) {
  return (G * D + 2 * G + 3) & ~3;
}

// Aligned partition: first CTA of segment s and the number of its CTAs.
__device__ __forceinline__ int aligned_first_cta(const DecodeArgs& a, int s) {
  const int q = a.grid / a.S, r = a.grid % a.S;
  return s * q + min(s, r);
}
__device__ __forceinline__ int aligned_seg_of_cta(const DecodeArgs& a, int c) {
  const int q = a.grid / a.S, r = a.grid % a.S;
  return c < r * (q + 1) ? c / (q + 1) : r + (c - r * (q + 1)) / q;
}

constexpr int kShareW = 16;  // weight of a full CTA share in the aligned partition

// First block (global index) of CTA c's range; c == grid gives NB.  In the
// aligned partition local CTA j of a segment (cs CTAs) starts at
// floor(nblk_u * j * kShareW / T), T = cs * kShareW - tail_w.
__device__ __forceinline__ long long range_begin(const DecodeArgs& a, int c) {
  if (!a.aligned) return (long long)c * a.NB / a.grid;
  if (c >= a.grid) return a.NB;
  const int s = aligned_seg_of_cta(a, c);
  const int c0 = aligned_first_cta(a, s);
  const int cs = aligned_first_cta(a, s + 1) - c0;
  const long long T = (long long)cs * kShareW - a.tail_w;
  return (long long)s * a.nblk_u + (long long)a.nblk_u * (c - c0) * kShareW / T;
}

// CTA whose range holds block x: the largest c with range_begin(c) <= x.
__device__ __forceinline__ long long cta_of_block(const DecodeArgs& a, long long x) {
  if (!a.aligned) return ((x + 1) * a.grid + a.NB - 1) / a.NB - 1;
  const int s = (int)(x / a.nblk_u);
  const long long local = x - (long long)s * a.nblk_u;
  const int c0 = aligned_first_cta(a, s);
  const int cs = aligned_first_cta(a, s + 1) - c0;
  // largest j < cs with floor(A*j/T) <= local, A = nblk_u * kShareW
  const long long T = (long long)cs * kShareW - a.tail_w;
  const long long A = (long long)a.nblk_u * kShareW;
  const long long j = ((local + 1) * T + A - 1) / A - 1;
  return c0 + (j < cs - 1 ? j : cs - 1);
}

struct SegView {
  int b, g, n, t0, blo;
  long long gbeg, gend;
};

__device__ __forceinline__ SegView seg_view(const DecodeArgs& a, int s) {
  SegView v;
  v.b = s / a.nkv;
  v.g = s - v.b * a.nkv;
  if (a.uniform) {
    v.n = a.n;
    v.t0 = a.t0;
    v.gbeg = (long long)s * a.nblk_u;
    v.gend = v.gbeg + a.nblk_u;
    v.blo = a.blo_u;
  } else {
    v.n = __ldg(a.seq_n + v.b);
    v.t0 = __ldg(a.seq_t0 + v.b);
    v.gbeg = __ldg(a.seg_prefix + s);
    v.gend = __ldg(a.seg_prefix + s + 1);
    v.blo = v.t0 / kBlk;
  }
  return v;
}

__device__ __forceinline__ int first_seg_of_cta(const DecodeArgs& a, int c) {
  if (a.uniform) return (int)(range_begin(a, c) / a.nblk_u);
  return __ldg(a.cta_seg + c);
}

__device__ __forceinline__ void raise_status(const DecodeArgs& a, volatile int* abort_flag,
                                             int code) {
  *abort_flag = 1;
  atomicCAS(a.status, 0, code);
}

constexpr float kLog2e = 1.4426950408889634f;
// Lazy rescaling: the running maximum (log2 units) is only raised when a
// score exceeds it by more than this, so weights stay <= 2^8 while the
// accumulators are rescaled rarely.  Every merge uses the stored maxima,
// so the result does not depend on when rescales happened.
constexpr float kLazyLog2 = 8.0f;

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// One chunk of RC rows of a row group: QK scores in the reference's
// accumulation order, lazy online-softmax update, p * V accumulation.
// kr / vr point at the chunk's first K / V row in shared memory; rows are D
// elements apart; each lane reads its dims (KvElem<KT>).  FULL: every row is
// valid.
template <int D, int GS, int RC, bool FULL, class KT, class AfterQK, class BeforePV>
__device__ __forceinline__ void process_rows(const KT* kr, const KT* vr, int tok, int pt0,
                                             int pt1, float scale, float (&q)[GS][D / 8],
                                             float (&o)[GS][D / 8], float (&m2)[GS],
                                             float (&l)[GS], int new_tok, const KT* nk,
                                             const KT* nv, int l8, AfterQK after_qk,
                                             BeforePV before_pv) {
  constexpr int DV = D / 16;
  constexpr int RS = TileShape<D, KT>::RS;
  using E = KvElem<KT>;
  float sc[RC][GS];
  bool ok[RC];
#pragma unroll
  for (int r = 0; r < RC; ++r) {
    ok[r] = FULL || (tok + r >= pt0 && tok + r < pt1);
    // The fused step's new row (slot new_tok) is not in the stage; its k and
    // v sit in shared memory (nk, nv).  Full tiles never contain it.
    const KT* k = (!FULL && tok + r == new_tok) ? nk : kr + r * RS;
    float a0[GS], a1[GS];
#pragma unroll
    for (int h = 0; h < GS; ++h) {
      a0[h] = 0.f;
      a1[h] = 0.f;
    }
#pragma unroll
    for (int mm = 0; mm < DV; ++mm) {
      float k0, k1;
      E::template load2<D>(k, mm, l8, k0, k1);
#pragma unroll
      for (int h = 0; h < GS; ++h) fma2(a0[h], a1[h], q[h][2 * mm], q[h][2 * mm + 1], k0, k1);
    }
    // The reference's _mm512_reduce_add_ps tree: lanes l and l+8 (held by
    // this lane), then l^4, l^2, l^1 within the row group.
#pragma unroll
    for (int h = 0; h < GS; ++h) {
      float t = __fadd_rn(a0[h], a1[h]);
      t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, 4));
      t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, 2));
      t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, 1));
      const float s = __fmul_rn(t, scale);  // == dot_fp32_avx512(q, k) * scale
      sc[r][h] = ok[r] ? s : -CUDART_INF_F;
    }
  }
  after_qk();  // the chunk's K rows are read
  bool need_any = false;
  float mc2[GS];
#pragma unroll
  for (int h = 0; h < GS; ++h) {
    float mc = sc[0][h];
#pragma unroll
    for (int r = 1; r < RC; ++r) mc = fmaxf(mc, sc[r][h]);
    mc2[h] = mc * kLog2e;
    need_any |= mc2[h] > m2[h] + kLazyLog2;
  }
  if (__any_sync(0xffffffffu, need_any)) {
#pragma unroll
    for (int h = 0; h < GS; ++h) {
      const bool need = mc2[h] > m2[h] + kLazyLog2;
      const float alpha = need ? ex2(m2[h] - mc2[h]) : 1.f;
      l[h] *= alpha;
#pragma unroll
      for (int i = 0; i < 2 * DV; i += 2) {
        const float2 x = __fmul2_rn(make_float2(o[h][i], o[h][i + 1]), make_float2(alpha, alpha));
        o[h][i] = x.x;
        o[h][i + 1] = x.y;
      }
      m2[h] = need ? mc2[h] : m2[h];
    }
  }
  float p[RC][GS];
#pragma unroll
  for (int r = 0; r < RC; ++r) {
#pragma unroll
    for (int h = 0; h < GS; ++h) {
      const float e = ex2(__fmaf_rn(sc[r][h], kLog2e, -m2[h]));
      p[r][h] = FULL ? e : (ok[r] ? e : 0.f);
      l[h] += p[r][h];
    }
  }
  before_pv();  // the chunk's V rows may be read from here on
#pragma unroll
  for (int r = 0; r < RC; ++r) {
    const KT* v = (!FULL && tok + r == new_tok) ? nv : vr + r * RS;
#pragma unroll
    for (int mm = 0; mm < DV; ++mm) {
      float v0, v1;
      E::template load2<D>(v, mm, l8, v0, v1);
      if (!FULL && !ok[r]) {
        v0 = 0.f;
        v1 = 0.f;
      }
#pragma unroll
      for (int h = 0; h < GS; ++h)
        fma2(o[h][2 * mm], o[h][2 * mm + 1], p[r][h], p[r][h], v0, v1);
    }
  }
}

// Fused step, launch constants: cos/sin of the RoPE angles pos*freq[i]
// (tab[i], tab[D/2+i]) and the q_norm / k_norm weights (tab[D+i],
// tab[2D+i]), staged in shared memory once per CTA by the 256 consumer
// threads (the caller's named barrier publishes them).  They depend only on
// the launch's arguments and the layer's weights, never on the preceding
// kernel, so the consumers build them before the dependency wait, while the
// preceding launch drains.  forward.h:562-575 computes the same values per
// row.
template <int D>
__device__ __forceinline__ void fused_fill_tables(const DecodeArgs& a, float* tab, int ctid) {
  constexpr int NT = kConsumerWarps * 32;
  constexpr int IT = (D + NT - 1) / NT;
  float f[IT], wq[IT], wk[IT];
#pragma unroll
  for (int r = 0; r < IT; ++r) {
    const int i = ctid + r * NT;
    f[r] = (i < D / 2 && a.freq) ? ptx::ld_nc_issue(a.freq + i) : 0.f;
    wq[r] = (i < D && a.q_norm) ? ptx::ld_nc_issue(a.q_norm + i) : 0.f;
    wk[r] = (i < D && a.k_norm) ? ptx::ld_nc_issue(a.k_norm + i) : 0.f;
  }
#pragma unroll
  for (int r = 0; r < IT; ++r) {
    const int i = ctid + r * NT;
    if (i < D / 2 && a.freq) {
      float sn, cs;
      sincosf(__fmul_rn((float)a.pos, f[r]), &sn, &cs);
      tab[i] = cs;
      tab[D / 2 + i] = sn;
    }
    if (i < D) {
      tab[D + i] = wq[r];
      tab[2 * D + i] = wk[r];
    }
  }
}

// Fused step, the new token's raw rows for the CTA that builds it: the raw
// k row `kx` ([D]) and all nkv*D raw v values go to raw[0..D) and
// raw[D..D+nkv*D) (the caller's named barrier publishes them).  They are
// the preceding kernel's outputs, so this runs after the dependency wait;
// every load is issued before the first store.
template <int D>
__device__ __forceinline__ void fused_stage_raw(const DecodeArgs& a, float* raw, int ctid,
                                                const float* kx) {
  constexpr int NT = kConsumerWarps * 32;
  constexpr int IT = (D + NT - 1) / NT;
  constexpr int kMaxV = kMaxStagedV / NT;
  float kr[IT], vv[kMaxV];
  const int nv = a.nkv * D;
#pragma unroll
  for (int r = 0; r < IT; ++r) {
    const int i = ctid + r * NT;
    kr[r] = i < D ? ptx::ld_nc_issue(kx + i) : 0.f;
  }
#pragma unroll
  for (int r = 0; r < kMaxV; ++r) {
    const int j = ctid + r * NT;
    vv[r] = j < nv ? ptx::ld_nc_issue(a.v_raw + j) : 0.f;
  }
#pragma unroll
  for (int r = 0; r < IT; ++r) {
    const int i = ctid + r * NT;
    if (i < D) raw[i] = kr[r];
  }
#pragma unroll
  for (int r = 0; r < kMaxV; ++r) {
    const int j = ctid + r * NT;
    if (j < nv) raw[D + j] = vv[r];
  }
}

// Fused step, q side (forward.h:554-558): the warp's q registers hold the
// raw projection in the row-group lane layout (dims {16m+l8, 16m+l8+8}).
// Per-head weighted RMSNorm with the reference's sum-of-squares order (the
// same tree as the dot), then NEOX RoPE; a lane holds both halves of each
// of its rotation pairs (dim i and i + D/2), so no data moves between lanes.
// The arithmetic is operation for operation that of norm_rope_append_kernel.
template <int D, int GS, class KT>
__device__ __forceinline__ void fused_rotate_q(const DecodeArgs& a, float (&q)[GS][D / 8],
                                               int l8, const float* tab) {
  constexpr int DV = D / 16;
  constexpr int HV = DV / 2;
  using E = KvElem<KT>;
  if (a.q_norm) {
#pragma unroll
    for (int h = 0; h < GS; ++h) {
      const float t = q_sumsq<D, KT>(q[h], l8);
      const float inv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)D), a.eps)));
#pragma unroll
      for (int i = 0; i < 2 * DV; ++i) {
        const int dim = E::dim(i, l8);
        q[h][i] = __fmul_rn(__fmul_rn(q[h][i], inv), tab[D + dim]);
      }
    }
  }
  if (a.freq) {
#pragma unroll
    for (int i = 0; i < 2 * HV; ++i) {
      const int dim = E::dim(i, l8);  // < D/2; partner (index i + 2*HV) at dim + D/2
      const float c = tab[dim], s = tab[D / 2 + dim];
#pragma unroll
      for (int h = 0; h < GS; ++h) {
        const float y0 = q[h][i], y1 = q[h][i + 2 * HV];
        q[h][i] = __fsub_rn(__fmul_rn(y0, c), __fmul_rn(y1, s));
        q[h][i + 2 * HV] = __fadd_rn(__fmul_rn(y0, s), __fmul_rn(y1, c));
      }
    }
  }
}

// Fused step, k/v side (forward.h:562-575) for kv head sv.g: warp 0 builds
// the normalised, rotated k row, warp 1 the normalised v row (plain RMSNorm
// over all nkv*D values); both land in shared memory (for this launch) and
// in slot n-1 of the cache (for later ones).  Weights and angles come from
// the staged table.
template <int D, class KT>
__device__ __forceinline__ void fused_new_row(const DecodeArgs& a, const SegView& sv, int warp,
                                              int lane, KT* new_k, KT* new_v,
                                              const float* tab, const float* kx,
                                              const float* vx) {
  constexpr int H = D / 2;
  using E = KvElem<KT>;
  KT* K_w = static_cast<KT*>(a.K_w);
  KT* V_w = static_cast<KT*>(a.V_w);
  const long long row = (long long)sv.b * a.kv_bstride + (long long)(sv.n - 1) * a.stride_t +
                        (long long)sv.g * a.stride_h;
  if (warp == 0) {
    const float* x = kx;
    float inv = 1.f;
    if (a.k_norm) {
      const float ss = warp_sumsq16(x, D, lane);
      inv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), a.eps)));
    }
#pragma unroll
    for (int i = lane; i < H; i += 32) {
      float y0 = x[i], y1 = x[i + H];
      if (a.k_norm) {
        y0 = __fmul_rn(__fmul_rn(y0, inv), tab[2 * D + i]);
        y1 = __fmul_rn(__fmul_rn(y1, inv), tab[2 * D + i + H]);
      }
      if (a.freq) {
        const float c = tab[i], s = tab[H + i];
        const float z0 = __fsub_rn(__fmul_rn(y0, c), __fmul_rn(y1, s));
        const float z1 = __fadd_rn(__fmul_rn(y0, s), __fmul_rn(y1, c));
        y0 = z0;
        y1 = z1;
      }
      // the cache's format (bf16 rounds, Q8 quantizes here), the same
      // value in both copies
      if constexpr (std::is_same<KT, Q8Row>::value) {  // H % 32 == 0: warp-uniform
        unsigned char* sk = reinterpret_cast<unsigned char*>(new_k);
        unsigned char* gk = reinterpret_cast<unsigned char*>(K_w + row);
        float s0, s1;
        const int c0 = q8_quantize(y0, s0), c1 = q8_quantize(y1, s1);
        q8_put(sk, D, i >> 5, lane, c0, s0);
        q8_put(sk, D, (i + H) >> 5, lane, c1, s1);
        q8_put(gk, D, i >> 5, lane, c0, s0);
        q8_put(gk, D, (i + H) >> 5, lane, c1, s1);
      } else {
        const KT z0 = E::store(y0), z1 = E::store(y1);
        new_k[i] = z0;
        new_k[i + H] = z1;
        K_w[row + i] = z0;
        K_w[row + i + H] = z1;
      }
    }
  } else {
    float vinv = 1.f;
    if (a.v_norm) {
      const int nv = a.nkv * D;
      const float ss = warp_sumsq16(vx, nv, lane);
      vinv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)nv), a.eps)));
    }
    const float* vh = vx + (long long)sv.g * D;
#pragma unroll
    for (int i = lane; i < D; i += 32) {
      const float y = a.v_norm ? __fmul_rn(vh[i], vinv) : vh[i];
      if constexpr (std::is_same<KT, Q8Row>::value) {
        float sv;
        const int c = q8_quantize(y, sv);
        q8_put(reinterpret_cast<unsigned char*>(new_v), D, i >> 5, lane, c, sv);
        q8_put(reinterpret_cast<unsigned char*>(V_w + row), D, i >> 5, lane, c, sv);
      } else {
        const KT val = E::store(y);
        new_v[i] = val;
        V_w[row + i] = val;
      }
    }
  }
}

// Merge of a split segment's per-CTA partial records (log2-domain max m, sum
// l, unnormalised o), run by the 256 consumer threads of the CTA that drew
// the segment's last ticket.  CTAs cf..cl contributed; every CTA after the
// first starts inside the segment (its slot 0), the first keeps the segment
// in slot 0 only if its own range starts there too.  Each thread owns a
// float4 chunk of o[G][D] and a share (csplit) of the partials, issuing up
// to 16 partials' loads before merging them with online rescaling; shares
// are folded through `red` ([256][6] floats of shared memory).
// Slot of the first CTA's partial record: its second piece unless its own
// range starts in the segment.  Computed before the ticket, off the path.
__device__ __forceinline__ int combine_slot_first(const DecodeArgs& a, const SegView& sv,
                                                  long long cf) {
  return 2 * (int)cf + (range_begin(a, (int)cf) >= sv.gbeg ? 0 : 1);
}

template <int D>
__device__ __forceinline__ void combine_segment(const DecodeArgs& a, int slot_first, long long cf,
                                                long long cl, float* red, int ctid,
                                                float* out_seg) {
  constexpr int kBatch = 16;
  const int G = a.G;
  const int psz = partial_record_floats(G, D);
  const int nc = (int)(cl - cf + 1);
  const int nchunk = G * D / 4;
  const int csplit = max(1, (kConsumerWarps * 32) / nchunk);
  for (int task = ctid; task < nchunk * csplit; task += kConsumerWarps * 32) {
    const int chunk = task % nchunk;
    const int part_i = task / nchunk;
    const int hl = (chunk * 4) / D;
    float M = -CUDART_INF_F, L = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k0 = part_i; k0 < nc; k0 += kBatch * csplit) {
      float mc[kBatch], lc[kBatch];
      float4 oc[kBatch];
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int k = k0 + u * csplit;
        if (k < nc) {
          const int sl = k == 0 ? slot_first : 2 * ((int)cf + k);
          const float* pp = a.partials + (size_t)sl * psz;
          mc[u] = __ldcg(pp + G * D + hl);
          lc[u] = __ldcg(pp + G * D + G + hl);
          oc[u] = __ldcg(reinterpret_cast<const float4*>(pp) + chunk);
        } else {
          mc[u] = -CUDART_INF_F;
          lc[u] = 0.f;
          oc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
      // Batch maximum first, so the batch's weights are independent
      // exponentials rather than a chain of rescales.
      float Mn = M;
#pragma unroll
      for (int u = 0; u < kBatch; ++u) Mn = fmaxf(Mn, mc[u]);
      const float fa = (M == -CUDART_INF_F) ? 0.f : ex2(M - Mn);
      L *= fa;
      acc.x *= fa;
      acc.y *= fa;
      acc.z *= fa;
      acc.w *= fa;
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const float fb = (mc[u] == -CUDART_INF_F) ? 0.f : ex2(mc[u] - Mn);
        L = __fmaf_rn(lc[u], fb, L);
        acc.x = __fmaf_rn(oc[u].x, fb, acc.x);
        acc.y = __fmaf_rn(oc[u].y, fb, acc.y);
        acc.z = __fmaf_rn(oc[u].z, fb, acc.z);
        acc.w = __fmaf_rn(oc[u].w, fb, acc.w);
      }
      M = Mn;
    }
    if (csplit == 1) {
      float* dst = out_seg + chunk * 4;
      const float inv = 1.f / L;  // one division per chunk
      put_out(a, dst + 0, acc.x * inv);
      put_out(a, dst + 1, acc.y * inv);
      put_out(a, dst + 2, acc.z * inv);
      put_out(a, dst + 3, acc.w * inv);
    } else {
      // csplit > 1 implies nchunk * csplit <= 256: the task fits `red`.
      float* r = red + (size_t)task * 6;
      r[0] = M;
      r[1] = L;
      r[2] = acc.x;
      r[3] = acc.y;
      r[4] = acc.z;
      r[5] = acc.w;
    }
  }
  ptx::named_bar_sync(1, kConsumerWarps * 32);
  for (int chunk = ctid; csplit > 1 && chunk < nchunk; chunk += kConsumerWarps * 32) {
    float M = -CUDART_INF_F;
    for (int p = 0; p < csplit; ++p) M = fmaxf(M, red[(size_t)(p * nchunk + chunk) * 6]);
    float L = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int p = 0; p < csplit; ++p) {
      const float* r = red + (size_t)(p * nchunk + chunk) * 6;
      const float f = (r[0] == -CUDART_INF_F) ? 0.f : ex2(r[0] - M);
      L += r[1] * f;
      acc.x += r[2] * f;
      acc.y += r[3] * f;
      acc.z += r[4] * f;
      acc.w += r[5] * f;
    }
    float* dst = out_seg + chunk * 4;
    const float inv = 1.f / L;
    put_out(a, dst + 0, acc.x * inv);
    put_out(a, dst + 1, acc.y * inv);
    put_out(a, dst + 2, acc.z * inv);
    put_out(a, dst + 3, acc.w * inv);
  }
}

// Cluster merge of a segment (see DecodeArgs::cluster), run by the 256
// consumer threads of every CTA of the cluster after its piece: `cbuf` (this
// CTA's shared memory) holds the CTA's partial -- o[G][D], then m[G], l[G]
// in the log2 domain -- or, when the CTA had no slots, nothing yet.  The
// cluster's CTAs each merge a slice of the float4 chunks of o across the
// cluster, reading the peers' partials through distributed shared memory.
template <int D>
__device__ __forceinline__ void cluster_finish(const DecodeArgs& a, int cta, float* cbuf,
                                               bool have_part, int ctid,
                                               volatile int* ticket_sm) {
  constexpr int NT = kConsumerWarps * 32;
  const int G = a.G;
  const int GD = G * D;
  const int C = a.cluster;
  if (!have_part) {  // no slots in this CTA's range: a neutral partial
    for (int i = ctid; i < GD + 2 * G; i += NT)
      cbuf[i] = (i >= GD && i < GD + G) ? -CUDART_INF_F : 0.f;
  }
  ptx::cluster_sync();  // every CTA's partial is in its shared memory
  const int cs = C * a.cl_per_seg;  // CTAs per segment
  const int s = cta / cs;
  const int ci = (cta - s * cs) / C;  // cluster index within the segment
  const SegView sv = seg_view(a, s);
  float* out_seg = a.O + (long long)sv.b * a.o_bstride + (long long)sv.g * G * D;
  const int psz = partial_record_floats(G, D);
  float* rec = a.partials + (size_t)(s * a.cl_per_seg + ci) * psz;
  const uint32_t rank = ptx::cluster_ctarank();
  const int nchunk = GD / 4;
  // chunks interleaved over the cluster's CTAs, so every CTA merges a few
  for (int chunk = ctid * C + (int)rank; chunk < nchunk; chunk += C * NT) {
    const int hl = (chunk * 4) / D;
    float M = -CUDART_INF_F;
    for (int r = 0; r < C; ++r) M = fmaxf(M, ptx::ld_dsmem(ptx::dsmem_addr(cbuf + GD + hl, r)));
    float L = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r = 0; r < C; ++r) {
      const float mr = ptx::ld_dsmem(ptx::dsmem_addr(cbuf + GD + hl, r));
      const float lr = ptx::ld_dsmem(ptx::dsmem_addr(cbuf + GD + G + hl, r));
      const float4 o4 = ptx::ld_dsmem4(ptx::dsmem_addr(cbuf + chunk * 4, r));
      const float f = (mr == -CUDART_INF_F) ? 0.f : ex2(mr - M);
      L = __fmaf_rn(lr, f, L);
      acc.x = __fmaf_rn(o4.x, f, acc.x);
      acc.y = __fmaf_rn(o4.y, f, acc.y);
      acc.z = __fmaf_rn(o4.z, f, acc.z);
      acc.w = __fmaf_rn(o4.w, f, acc.w);
    }
    if (a.cl_per_seg == 1) {
      float* dst = out_seg + chunk * 4;
      put_out(a, dst + 0, acc.x / L);
      put_out(a, dst + 1, acc.y / L);
      put_out(a, dst + 2, acc.z / L);
      put_out(a, dst + 3, acc.w / L);
    } else {
      reinterpret_cast<float4*>(rec)[chunk] = acc;
      if ((chunk * 4) % D == 0) {
        rec[GD + hl] = M;
        rec[GD + G + hl] = L;
      }
    }
  }
  if (a.cl_per_seg > 1) __threadfence();  // the record slices, before the leader's ticket
  ptx::cluster_sync();  // no CTA reads a peer's shared memory after this
  if (a.cl_per_seg > 1 && rank == 0) {
    // The cluster's record is complete; the last cluster of the segment to
    // draw a ticket merges the segment's records.
    if (ctid == 0) *ticket_sm = ptx::atom_add_acq_rel_gpu(a.counters + s, 1);
    ptx::named_bar_sync(1, NT);
    if (*ticket_sm == a.cl_per_seg - 1) {
      const float* recs = a.partials + (size_t)s * a.cl_per_seg * psz;
      for (int chunk = ctid; chunk < nchunk; chunk += NT) {
        const int hl = (chunk * 4) / D;
        float M = -CUDART_INF_F;
        for (int k = 0; k < a.cl_per_seg; ++k) M = fmaxf(M, __ldcg(recs + k * psz + GD + hl));
        float L = 0.f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int k = 0; k < a.cl_per_seg; ++k) {
          const float* rk = recs + (size_t)k * psz;
          const float mr = __ldcg(rk + GD + hl);
          const float f = (mr == -CUDART_INF_F) ? 0.f : ex2(mr - M);
          const float4 o4 = __ldcg(reinterpret_cast<const float4*>(rk) + chunk);
          L = __fmaf_rn(__ldcg(rk + GD + G + hl), f, L);
          acc.x = __fmaf_rn(o4.x, f, acc.x);
          acc.y = __fmaf_rn(o4.y, f, acc.y);
          acc.z = __fmaf_rn(o4.z, f, acc.z);
          acc.w = __fmaf_rn(o4.w, f, acc.w);
        }
        float* dst = out_seg + chunk * 4;
        put_out(a, dst + 0, acc.x / L);
        put_out(a, dst + 1, acc.y / L);
        put_out(a, dst + 2, acc.z / L);
        put_out(a, dst + 3, acc.w / L);
      }
      if (ctid == 0) a.counters[s] = 0;
    }
  }
}

// SPLIT: the K and V halves of each ring stage fill and free on their own
// barriers, so a stage's K half is refilled as soon as every warp has its
// scores.  The host launches it where it measured faster: single-sequence
// FP32 launches at hd <= 128 with at least 8 tiles per CTA (cfg2 -3 %); it
// was slower with fewer tiles, for the consumer-bound BF16 / Q8 launches and
// for paged batches, which therefore run the one-barrier-pair form.
template <int D, int GS, int HS, class KT = float, bool SPLIT = false>
__global__ void __launch_bounds__(kDecodeThreads, 1)
    gqa_decode_kernel(const __grid_constant__ DecodeArgs a) {
  using TS = TileShape<D, KT>;
  using SM = DecodeSmem<D, GS, KT>;
  using E = KvElem<KT>;
  constexpr int EB = E::kBytes;
  constexpr int QR = TS::QR;
  constexpr int STAGES = TS::STAGES;
  constexpr int WPS = kConsumerWarps / HS;  // warps per head set
  constexpr int R = QR / WPS;               // rows per warp per quarter per tile
  // rows per online-softmax update: 2 at D = 256, where registers are
  // tightest, and for BF16, whose 4-row body is large enough to stall on
  // instruction fetch (2 rows measured 1-3 % faster there); 4 otherwise
  constexpr int RC = (D > 128 || EB == 2) ? (R < 2 ? R : 2) : (R < 4 ? R : 4);
  constexpr int DV = D / 16;
  static_assert(kConsumerWarps % HS == 0, "head sets must divide the consumer warps");
  static_assert(QR % WPS == 0 && R >= 1, "rows per quarter must divide among warps");
  static_assert(D % 16 == 0, "head dim must be a multiple of 16");
  static_assert(!TS::kQ8 || D % 64 == 0, "Q8 rows: both halves must be whole 32-value blocks");
  static_assert(R % RC == 0, "row chunks must tile the rows");

  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* stages = smem;
  float* merge_o = reinterpret_cast<float*>(smem + SM::kStageBytes);
  float* merge_ml = reinterpret_cast<float*>(smem + SM::kStageBytes + SM::kMergeO);
  // fused mode: the new k and v rows (cache format), then the tables (cos,
  // sin, q_norm, k_norm) at a fixed offset of 2*D floats
  KT* new_k = reinterpret_cast<KT*>(smem + SM::kStageBytes + SM::kMergeO + SM::kMergeML);
  KT* new_v = new_k + TS::RS;
  float* tab = reinterpret_cast<float*>(smem + SM::kStageBytes + SM::kMergeO + SM::kMergeML +
                                        2 * D * 4);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + SM::kStageBytes + SM::kMergeO +
                                                   SM::kMergeML + SM::kNewRow);
  // [stage][K, V]: in split mode the halves of a stage fill and free
  // separately; otherwise a stage uses its K half's barriers for both
  uint64_t* empty_bar = full_bar + 2 * STAGES;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty_bar + 2 * STAGES);
  volatile int* ticket_sm = abort_flag + 1;
  volatile int* seg_cta_sm = abort_flag + 2;  // [2]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2 * STAGES; ++i) {
      ptx::mbar_init(full_bar + i, 1);
      ptx::mbar_init(empty_bar + i, kConsumerWarps);
    }
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  __syncthreads();

  // Partition index: blocks in reverse.  The block scheduler hands out
  // blocks in index order, so the highest blocks of a launch start last,
  // on the SMs that the preceding launch's last CTAs free; they take the
  // lightest ranges (the first CTAs of a segment, never the new row's).
  const int cta = a.grid - 1 - (int)blockIdx.x;
  constexpr bool split = SPLIT;
  const long long cbeg = range_begin(a, cta);
  const long long cend = range_begin(a, cta + 1);
  const int s_first = first_seg_of_cta(a, cta);

  if (warp >= kConsumerWarps) {
    // ------------------------------------------------------------ producer
    ptx::setmaxnreg_dec<kProducerRegs>();
    if (warp != kConsumerWarps || a.withhold) return;
    const uint64_t pol = ptx::policy_evict_first();
    const bool rows_contig = (a.block_table != nullptr) || (a.stride_t * EB == TS::RB);
    bool waited = false;  // griddepcontrol.wait done by this warp
    int it = 0;
    long long pos = cbeg;
    int s = s_first;
    while (pos < cend) {
      const SegView sv = seg_view(a, s);
      const long long pend = sv.gend < cend ? sv.gend : cend;
      if (pend > pos) {
        const int lb = sv.blo + (int)(pos - sv.gbeg);
        const int le = sv.blo + (int)(pend - sv.gbeg);
        const int pt0 = max(sv.t0, lb * kBlk);
        const int pt1 = min(sv.n, le * kBlk);
        // Fused mode: slot n-1 is produced in this launch and never streamed.
        const int pt1c = a.fused ? min(pt1, sv.n - 1) : pt1;
        for (int blk = lb; blk < le; blk += TS::TB, ++it) {
          const int stage = it % STAGES;
          const int tok0 = blk * kBlk;
          int qa[4], qn[4];
          uint32_t bytes = 0;  // of one half (K or V)
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int lo = max(tok0 + q * QR, pt0);
            const int hi = min(tok0 + (q + 1) * QR, pt1c);
            qa[q] = lo;
            qn[q] = hi > lo ? hi - lo : 0;
            bytes += (uint32_t)qn[q] * TS::RB;
          }
          unsigned char* st_base = stages + (size_t)stage * TS::STAGE;
          // Split mode: the K and V halves are awaited and filled one after
          // the other, each on its own barriers (lanes 0-3 issue a half's
          // quarters).  Otherwise one round fills both halves through the K
          // half's barriers (lanes 0-7: quarter = lane & 3, half = lane >> 2).
          for (int kv = 0; kv < (split ? 2 : 1); ++kv) {
            uint64_t* fb = full_bar + 2 * stage + kv;
            if (it >= STAGES && !*abort_flag) {
              if (!ptx::mbar_wait_bounded(empty_bar + 2 * stage + kv, ((it / STAGES) - 1) & 1,
                                          a.timeout_ns)) {
                if (lane == 0) raise_status(a, abort_flag, kDevErrProducerTimeout);
              }
            }
            __syncwarp();
            // Slots written by the immediately preceding launch (the new
            // token's row) may only be read after that launch has completed.
            if (!waited && (!a.prefetch_old_rows || min(tok0 + TS::T, pt1c) >= sv.n)) {
              ptx::pdl_wait();
              waited = true;
            }
            if (*abort_flag) {
              // Consumers skip waits once aborted; complete the phase without data.
              if (lane == 0) ptx::mbar_arrive(fb);
              continue;
            }
            if (lane == 0) ptx::mbar_arrive_expect_tx(fb, split ? bytes : 2 * bytes);
            __syncwarp();
            if (rows_contig) {
              if (lane < (split ? 4 : 8)) {
                const int q = lane & 3;
                const int h = split ? kv : lane >> 2;  // K or V half
                if (qn[q] > 0) {
                  const unsigned char* base = static_cast<const unsigned char*>(h ? a.V : a.K);
                  long long off;  // stride units
                  if (a.block_table) {
                    const int p =
                        __ldg(a.block_table + (long long)sv.b * a.bt_stride + qa[q] / a.page_size);
                    off = (long long)p * a.page_stride + (long long)sv.g * a.page_hstride +
                          (long long)(qa[q] % a.page_size) * TS::RS;
                  } else {
                    off = (long long)sv.b * a.kv_bstride + (long long)qa[q] * a.stride_t +
                          (long long)sv.g * a.stride_h;
                  }
                  unsigned char* dst = st_base + h * TS::KQ + q * TS::QSTRIDE +
                                       (qa[q] - (tok0 + q * QR)) * TS::RB;
                  ptx::bulk_g2s(dst, base + off * EB, (uint32_t)qn[q] * TS::RB, fb, pol);
                }
              }
            } else {
              const int n_idx = (split ? 1 : 2) * 4 * QR;
              for (int idx = lane; idx < n_idx; idx += 32) {
                const int h = split ? kv : idx / (4 * QR);
                const int rem = split ? idx : idx - h * 4 * QR;
                const int q = rem / QR;
                const int r = rem - q * QR;
                const int t = tok0 + q * QR + r;
                if (t >= qa[q] && t < qa[q] + qn[q]) {
                  const unsigned char* base = static_cast<const unsigned char*>(h ? a.V : a.K);
                  const long long off = (long long)sv.b * a.kv_bstride +
                                        (long long)t * a.stride_t + (long long)sv.g * a.stride_h;
                  unsigned char* dst = st_base + h * TS::KQ + q * TS::QSTRIDE + r * TS::RB;
                  ptx::bulk_g2s(dst, base + off * EB, (uint32_t)TS::RB, fb, pol);
                }
              }
            }
          }
        }
      }
      pos = pend > pos ? pend : pos;
      ++s;
    }
    // Drain: every issued stage must have landed before the CTA may exit.
    if (lane == 0) {
      const int first = it > STAGES ? it - STAGES : 0;
      bool ok = true;
      for (int j = first; j < it && ok; ++j) {
        for (int kv = 0; kv < (split ? 2 : 1) && ok; ++kv) {
          if (!ptx::mbar_wait_bounded(full_bar + 2 * (j % STAGES) + kv, (j / STAGES) & 1,
                                      kDrainLimitNs)) {
            raise_status(a, abort_flag, kDevErrProducerTimeout);
            ok = false;
          }
        }
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  ptx::setmaxnreg_inc<kConsumerRegs>();
  // Fused step: the launch constants, before the dependency wait.
  if (a.fused) {
    fused_fill_tables<D>(a, tab, threadIdx.x);
    ptx::named_bar_sync(1, kConsumerWarps * 32);
  }
  // q, the KV row appended just before and the scratch the previous
  // decode/combine pair used are only touched after the preceding launch
  // completed.  The trigger comes after that wait: when the next grids
  // start early, everything up to the launch before this one is complete,
  // which is what makes a later decode's early reads of older KV rows safe.
  ptx::pdl_wait();
  if (threadIdx.x == 0) ptx::pdl_launch_dependents();
  const int set = warp / WPS;  // head set of this warp
  const int wi = warp - set * WPS;
  const int grp = lane >> 3;   // row group == quarter read
  const int l8 = lane & 7;
  const int ctid = threadIdx.x;  // 0..255

  float q[GS][2 * DV];
  float o[GS][2 * DV];
  float m[GS], l[GS];

  int it = 0;
  const bool clustered = a.cluster > 1;
  // cluster merge: this CTA's partial, in the ring (idle once the CTA's
  // last tile is consumed; a cluster-merged CTA has one piece)
  float* cbuf = reinterpret_cast<float*>(stages);
  bool have_part = false;
  long long pos = cbeg;
  int s = s_first;
  while (pos < cend) {
    const SegView sv = seg_view(a, s);
    const long long pend = sv.gend < cend ? sv.gend : cend;
    if (pend > pos) {
      const int lb = sv.blo + (int)(pos - sv.gbeg);
      const int le = sv.blo + (int)(pend - sv.gbeg);
      const int pt0 = max(sv.t0, lb * kBlk);
      const int pt1 = min(sv.n, le * kBlk);
      // A cluster-merged launch always merges, even a piece that is the
      // whole segment (its cluster peers then hold empty partials).
      const bool whole = !clustered && (pos == sv.gbeg) && (pend == sv.gend);
      // CTAs sharing this segment, for the merge after the piece: computed
      // here, off the critical path at the piece's end, and parked in shared
      // memory (read after the finalize barriers) rather than in registers.
      if (!whole && ctid == 0) {
        seg_cta_sm[0] = (int)cta_of_block(a, sv.gbeg);
        seg_cta_sm[1] = (int)cta_of_block(a, sv.gend - 1);
      }
      const int head0 = sv.g * a.G + set * GS;  // first query head of this warp's set

      {
        const float* qb = a.Q + (long long)sv.b * a.q_bstride + (long long)head0 * D;
#pragma unroll
        for (int h = 0; h < GS; ++h) {
#pragma unroll
          for (int i = 0; i < 2 * DV; ++i) {
            q[h][i] = ptx::ld_nc_issue(qb + h * D + E::dim(i, l8));
            o[h][i] = 0.f;
          }
          m[h] = -CUDART_INF_F;
          l[h] = 0.f;
        }
      }
      // Fused step: q arrived raw; the piece holding slot n-1 also builds
      // the new k/v row.
      const int new_tok = a.fused ? sv.n - 1 : -1;
      if (a.fused) {
        const bool newrow = pend == sv.gend;
        const float* kx = a.k_raw + (long long)sv.g * D;  // raw k row of head g
        const float* vx = a.v_raw;                          // raw v, all heads
        // merge_o is free until this piece's finalize: stage the raw rows
        // there when this piece builds the new row (the q loads above are in
        // flight meanwhile).
        if (newrow && a.nkv * D <= kMaxStagedV && (D + a.nkv * D) * 4 <= SM::kMergeO) {
          fused_stage_raw<D>(a, merge_o, ctid, kx);
          ptx::named_bar_sync(1, kConsumerWarps * 32);
          kx = merge_o;
          vx = merge_o + D;
        }
        fused_rotate_q<D, GS, KT>(a, q, l8, tab);
        if (newrow) {
          if (warp < 2) fused_new_row<D, KT>(a, sv, warp, lane, new_k, new_v, tab, kx, vx);
          ptx::named_bar_sync(1, kConsumerWarps * 32);
        }
      }

      for (int blk = lb; blk < le; blk += TS::TB, ++it) {
        const int stage = it % STAGES;
        const uint32_t par = (it / STAGES) & 1;
        uint64_t* fk = full_bar + 2 * stage;  // K half; fk + 1: V half
        uint64_t* ek = empty_bar + 2 * stage;
        if (!*abort_flag) {
          if (!ptx::mbar_wait_bounded(fk, par, a.timeout_ns)) {
            if (lane == 0) raise_status(a, abort_flag, kDevErrConsumerTimeout);
          }
        }
        __syncwarp();
        bool k_freed = false;  // this warp has released the K half
        if (!*abort_flag) {
          const KT* kq = reinterpret_cast<const KT*>(stages + (size_t)stage * TS::STAGE +
                                                     grp * TS::QSTRIDE);
          const KT* vq = reinterpret_cast<const KT*>(stages + (size_t)stage * TS::STAGE +
                                                     TS::KQ + grp * TS::QSTRIDE);
          const int tok_base = blk * kBlk + grp * QR + wi * R;
          // Only a piece's first and last tiles can hold rows outside
          // [pt0, pt1); the rest take the predicate-free path.
          const bool full = blk * kBlk >= pt0 && blk * kBlk + TS::T <= pt1 &&
                            !(new_tok >= blk * kBlk && new_tok < blk * kBlk + TS::T);
          // The K half is released once the warp's last chunk has its
          // scores; the V half is waited for before its first chunk's P*V.
          int r0 = 0;
          auto after_qk = [&]() {
            if (split && r0 + RC >= R) {
              __syncwarp();
              if (lane == 0) ptx::mbar_arrive(ek);
              k_freed = true;
            }
          };
          auto before_pv = [&]() {
            if (split && r0 == 0) {
              if (!*abort_flag && !ptx::mbar_wait_bounded(fk + 1, par, a.timeout_ns)) {
                if (lane == 0) raise_status(a, abort_flag, kDevErrConsumerTimeout);
              }
              __syncwarp();
            }
          };
          // One copy of each chunk body: the chunk loops stay rolled so the
          // instruction working set fits the SM's instruction cache.
          if (full) {
#pragma unroll 1
            for (r0 = 0; r0 < R; r0 += RC)
              process_rows<D, GS, RC, true>(kq + (wi * R + r0) * TS::RS, vq + (wi * R + r0) * TS::RS,
                                            tok_base + r0, pt0, pt1, a.scale, q, o, m, l,
                                            new_tok, new_k, new_v, l8, after_qk, before_pv);
          } else {
#pragma unroll 1
            for (r0 = 0; r0 < R; r0 += RC)
              process_rows<D, GS, RC, false>(kq + (wi * R + r0) * TS::RS, vq + (wi * R + r0) * TS::RS,
                                             tok_base + r0, pt0, pt1, a.scale, q, o, m, l,
                                             new_tok, new_k, new_v, l8, after_qk, before_pv);
          }
        }
        __syncwarp();
        if (lane == 0) {
          if (!k_freed) ptx::mbar_arrive(ek);
          if (split) ptx::mbar_arrive(ek + 1);
        }
      }

      // ---- finalize the piece: merge 4 row groups, then warps, then CTAs.
      // Row groups merge by reduce-scatter: the xor-16 round leaves each
      // lane half of its 2*DV values (the half its group bit 1 selects), the
      // xor-8 round a quarter, so group grp ends owning o-values
      // [grp*DV/2, (grp+1)*DV/2) of its lane's set; m and l are all-reduced.
      {
        const int bit1 = (lane >> 4) & 1, bit0 = (lane >> 3) & 1;
#pragma unroll
        for (int h = 0; h < GS; ++h) {
          // round 1 (xor 16): keep slot j of [0, DV) <- value j + bit1*DV
          float mo = __shfl_xor_sync(0xffffffffu, m[h], 16);
          float lo = __shfl_xor_sync(0xffffffffu, l[h], 16);
          float M = fmaxf(m[h], mo);
          float fs = (m[h] == -CUDART_INF_F) ? 0.f : ex2(m[h] - M);
          float fo = (mo == -CUDART_INF_F) ? 0.f : ex2(mo - M);
          l[h] = l[h] * fs + lo * fo;
#pragma unroll
          for (int j = 0; j < DV; ++j) {
            const float keep = bit1 ? o[h][DV + j] : o[h][j];
            const float send = bit1 ? o[h][j] : o[h][DV + j];
            const float recv = __shfl_xor_sync(0xffffffffu, send, 16);
            o[h][j] = keep * fs + recv * fo;
          }
          m[h] = M;
          // round 2 (xor 8): keep slot j of [0, DV/2) <- slot j + bit0*DV/2
          mo = __shfl_xor_sync(0xffffffffu, m[h], 8);
          lo = __shfl_xor_sync(0xffffffffu, l[h], 8);
          M = fmaxf(m[h], mo);
          fs = (m[h] == -CUDART_INF_F) ? 0.f : ex2(m[h] - M);
          fo = (mo == -CUDART_INF_F) ? 0.f : ex2(mo - M);
          l[h] = l[h] * fs + lo * fo;
#pragma unroll
          for (int j = 0; j < DV / 2; ++j) {
            const float keep = bit0 ? o[h][DV / 2 + j] : o[h][j];
            const float send = bit0 ? o[h][j] : o[h][DV / 2 + j];
            const float recv = __shfl_xor_sync(0xffffffffu, send, 8);
            o[h][j] = keep * fs + recv * fo;
          }
          m[h] = M;
          // slot j now holds o-value i = grp*DV/2 + j, i.e. dim E::dim(i, l8)
          float* dst = merge_o + ((size_t)warp * GS + h) * D;
#pragma unroll
          for (int j = 0; j < DV / 2; ++j) {
            const int i = (bit1 * 2 + bit0) * (DV / 2) + j;
            dst[E::dim(i, l8)] = o[h][j];
          }
          if (lane == 0) {
            merge_ml[(warp * GS + h) * 2] = m[h];
            merge_ml[(warp * GS + h) * 2 + 1] = l[h];
          }
        }
      }
      ptx::named_bar_sync(1, kConsumerWarps * 32);

      const int G = a.G;
      const int psz = partial_record_floats(G, D);
      const int slot = 2 * cta + (pos == cbeg ? 0 : 1);
      float* part = a.partials + (size_t)slot * psz;
      float* out_seg = a.O + (long long)sv.b * a.o_bstride + (long long)sv.g * G * D;
      for (int idx = ctid; idx < G * D; idx += kConsumerWarps * 32) {
        const int hl = idx / D;
        const int j = idx - hl * D;
        const int st = hl / GS;
        const int hh = hl - st * GS;
        float M = -CUDART_INF_F;
#pragma unroll
        for (int w = 0; w < WPS; ++w) M = fmaxf(M, merge_ml[((st * WPS + w) * GS + hh) * 2]);
        float L = 0.f, acc = 0.f;
#pragma unroll
        for (int w = 0; w < WPS; ++w) {
          const int ww = st * WPS + w;
          const float mw = merge_ml[(ww * GS + hh) * 2];
          const float f = (mw == -CUDART_INF_F) ? 0.f : ex2(mw - M);
          L += merge_ml[(ww * GS + hh) * 2 + 1] * f;
          acc += merge_o[((size_t)ww * GS + hh) * D + j] * f;
        }
        if (whole) {
          put_out(a, out_seg + idx, acc / L);
        } else {
          float* dst = clustered ? cbuf : part;
          dst[idx] = acc;
          if (j == 0) {
            dst[G * D + hl] = M;
            dst[G * D + G + hl] = L;
          }
        }
      }
      have_part = true;
      // Every partial (or output) write of this CTA is issued before the
      // barrier; the merge buffer is free again after it.
      ptx::named_bar_sync(1, kConsumerWarps * 32);
      if (!whole && !clustered) {
        // One thread publishes the CTA's partial and takes a ticket; the CTA
        // that draws the last ticket of the segment merges all partials.
        const long long cf = seg_cta_sm[0];
        const long long cl = seg_cta_sm[1];
        if (ctid == 0) *ticket_sm = ptx::atom_add_acq_rel_gpu(a.counters + s, 1);
        const int slot_first = combine_slot_first(a, sv, cf);  // while the ticket is out
        ptx::named_bar_sync(1, kConsumerWarps * 32);
        if (*ticket_sm == (int)(cl - cf)) {
          combine_segment<D>(a, slot_first, cf, cl, merge_o, ctid, out_seg);
          if (ctid == 0) a.counters[s] = 0;
        }
        ptx::named_bar_sync(1, kConsumerWarps * 32);
      }
    }
    pos = pend > pos ? pend : pos;
    ++s;
  }
  if (clustered) cluster_finish<D>(a, cta, cbuf, have_part, ctid, ticket_sm);
  if (a.npeer > 0) {
    // Peer gather: once every CTA's output stores are issued, the last CTA
    // to finish publishes this launch's epoch in every rank's buffer.  The
    // system-scope fences order the CTAs' stores to peer memory before the
    // count and the count before the flags.
    ptx::named_bar_sync(1, kConsumerWarps * 32);
    if (ctid == 0) {
      __threadfence_system();
      const unsigned int t = atomicAdd(a.done_ctr, 1u);
      if (t == (unsigned int)a.grid - 1) {
        __threadfence_system();
        *a.done_ctr = 0;
        const unsigned long long e = *a.epoch + 1;
        *a.epoch = e;
        for (int p = 0; p < a.npeer; ++p) ptx::st_release_sys(a.peer_flag[p], e);
      }
    }
  }
}

}  // namespace molot
