// Kernel selection across translation units.  Each storage type's decode
// kernels (and the prefill kernels) are instantiated in a translation unit
// of their own (kernels_*.cu), which the build compiles side by side; the
// rest of the library reaches them through these functions.
#pragma once

namespace molot {

// A kernel's host-side handle and its dynamic shared memory.
struct KernelRef {
  const void* fn = nullptr;
  int smem = 0;
};

// gqa_decode_kernel for a head_dim / group size and a cache storage type
// (molot_kv_dtype).  split: the FP32 kernel with split K/V stage barriers
// (head_dim <= 128).  false when that combination is not built.
bool pick_decode_f32(int D, int G, bool split, KernelRef* k);
bool pick_decode_bf16(int D, int G, KernelRef* k);
bool pick_decode_q8(int D, int G, KernelRef* k);
// gqa_prefill_kernel for a head_dim and a storage type.
bool pick_prefill_kv(int D, int kvt, KernelRef* k);
// gqa_prefill_tc_kernel (split-TF32 tcgen05; FP32 caches, head_dim 64/128).
bool pick_prefill_tc(int D, KernelRef* k);

// Thread-block clusters of this many CTAs that kernel k can keep resident
// at once on device dev (cached; 0 when the query fails).
int max_active_clusters(const KernelRef& k, int cluster, int dev);

// Partition of a single-sequence (uniform) decode launch of S segments
// (kv heads) of nblk 16-slot blocks each.
struct UniformPlan {
  int grid = 0;
  int aligned = 0;     // one segment per CTA (DecodeArgs::aligned)
  int cluster = 0;     // DecodeArgs::cluster
  int cl_per_seg = 0;  // DecodeArgs::cl_per_seg
};

constexpr int kClusterCtas = 8;       // CTAs per cluster (portable size)
constexpr int kClusterCtasWide = 16;  // one cluster per segment (non-portable size)
constexpr int kClusterMinBlocks = 4;  // blocks per CTA below which no extra cluster is added

// One CTA per SM at most.  Segment-aligned when there are at least as many
// CTAs as segments.  Launches too small to give every SM two blocks (the
// sliding-window layers) merge in thread-block clusters instead, when every
// segment can have a whole cluster resident at once: clusters of
// kClusterCtas CTAs merge the segment's partials in distributed shared
// memory -- k clusters per segment, as many as fit (each CTA keeping
// kClusterMinBlocks blocks or more).  On larger launches clusters measured
// slower (cfg2 step 0.88 -> 1.43 ms): a cluster starts only once kClusterCtas
// SMs of one GPC are free, which defeats the overlap of back-to-back
// launches.
//
// When a whole segment fits one 16-CTA cluster at once (wide_resident >= S),
// that form is taken: the merge then stays in distributed shared memory,
// with no ticket and no global record.
inline UniformPlan plan_uniform(long long NB, int S, int nblk, int sms, int clusters_resident,
                                int wide_resident = 0) {
  UniformPlan p;
  p.grid = (int)(NB < sms ? NB : sms);
  p.aligned = p.grid >= S ? 1 : 0;
  if (NB < 2LL * sms && wide_resident >= S && S * kClusterCtasWide <= sms &&
      nblk >= kClusterCtasWide) {
    p.grid = S * kClusterCtasWide;
    p.aligned = 1;
    p.cluster = kClusterCtasWide;
    p.cl_per_seg = 1;
    return p;
  }
  const int C = kClusterCtas;
  if (NB < 2LL * sms && clusters_resident >= S && S * C <= sms && nblk >= C) {
    int k = clusters_resident / S;
    if (k > sms / (S * C)) k = sms / (S * C);
    const int by_work = nblk / (C * kClusterMinBlocks);
    if (k > by_work) k = by_work > 1 ? by_work : 1;
    if (k >= 1 && nblk >= C * k) {
      p.grid = S * k * C;
      p.aligned = 1;
      p.cluster = C;
      p.cl_per_seg = k;
    }
  }
  return p;
}

// Launches of under 8 FP32-sized tiles (64 slots) per CTA, e.g. a 4096-slot
// context: every segment the same number of CTAs, the grid rounded down to
// a multiple of S, measured faster there (cfg1 0.425 -> 0.417 ms per token);
// longer launches keep every SM (cfg2 measured 0.3 % slower rounded).
// Every single-sequence decode entry applies it, so their partitions (and
// results) agree.
inline void balance_uniform_grid(UniformPlan& p, int S, int nblk) {
  const long long rows = (long long)nblk * 16 * S / p.grid;
  if (p.cluster < 2 && p.aligned && p.grid >= 2 * S && rows < 8LL * 64) p.grid -= p.grid % S;
}

}  // namespace molot
