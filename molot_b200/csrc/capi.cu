// C ABI of molot_b200 (include/molot_b200.h): argument checking, scratch
// workspaces, kernel dispatch, the KV-cache handle and paged plans.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "append.cuh"
#include "comm.cuh"
#include "decode.cuh"
#include "dispatch.cuh"
#include "gemv.cuh"
#include "molot_b200.h"
#include "prefill.cuh"
#include "prefill_tc.cuh"

namespace molot {

void take_withhold(DecodeArgs& a);
// No-alloc scratch status of device `dev` (noalloc.cu): MOLOT_OK when it was
// never set up there.
int noalloc_status_check(int dev, cudaStream_t st, bool clear);

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(e == cudaErrorMemoryAllocation ? MOLOT_ERR_NOMEM : MOLOT_ERR_CUDA,
              std::string(what) + ": " + cudaGetErrorString(e));
}

#define MOLOT_CUDA(call)                                 \
  do {                                                   \
    cudaError_t e_ = (call);                             \
    if (e_ != cudaSuccess) return cuda_fail(e_, #call);  \
  } while (0)

constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s per bounded wait
constexpr int kMaxPartialFloats = 4096 + 2 * 32;           // G*D + 2G upper bound

int current_device(int* dev) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0)
    return fail(MOLOT_ERR_NO_DEVICE, "no CUDA device visible");
  MOLOT_CUDA(cudaGetDevice(dev));
  return MOLOT_OK;
}

int sm_count(int dev) {
  static std::mutex mu;
  static std::vector<int> cache;
  std::lock_guard<std::mutex> lk(mu);
  if ((int)cache.size() <= dev) cache.resize(dev + 1, 0);
  if (!cache[dev]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = v > 0 ? v : 1;
  }
  return cache[dev];
}

// ------------------------------------------------------------- workspace

// Device scratch owned by one ordered stream of calls: split-KV partials,
// the device status word and plan arrays.  Grows only; growth synchronises
// the device.
struct Workspace {
  int device = -1;
  float* partials = nullptr;
  size_t partials_cap = 0;
  int* counters = nullptr;  // per-segment tickets, zero between launches
  size_t counters_cap = 0;
  int* status = nullptr;
  int* plan = nullptr;
  size_t plan_cap = 0;

  ~Workspace() { release(); }
  void release() {
    if (device < 0) return;
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    cudaFree(partials);
    cudaFree(counters);
    cudaFree(status);
    cudaFree(plan);
    if (prev >= 0) cudaSetDevice(prev);
    partials = nullptr;
    counters = nullptr;
    status = nullptr;
    plan = nullptr;
    partials_cap = counters_cap = plan_cap = 0;
  }

  int ensure(int dev, size_t partial_floats, size_t ncounters, size_t plan_ints) {
    if (device >= 0 && device != dev)
      return fail(MOLOT_ERR_INVALID, "workspace used on a different device than it was made on");
    device = dev;
    const bool grow = partial_floats > partials_cap || ncounters > counters_cap ||
                      plan_ints > plan_cap || !status;
    if (!grow) return MOLOT_OK;
    MOLOT_CUDA(cudaDeviceSynchronize());
    if (!status) {
      MOLOT_CUDA(cudaMalloc(&status, 256));
      MOLOT_CUDA(cudaMemset(status, 0, 256));
    }
    if (partial_floats > partials_cap) {
      cudaFree(partials);
      partials = nullptr;
      const size_t cap = std::max(partial_floats, (size_t)2 * sm_count(dev) * kMaxPartialFloats);
      MOLOT_CUDA(cudaMalloc(&partials, cap * sizeof(float)));
      partials_cap = cap;
    }
    if (ncounters > counters_cap) {
      cudaFree(counters);
      counters = nullptr;
      const size_t cap = std::max<size_t>(ncounters, 4096);
      MOLOT_CUDA(cudaMalloc(&counters, cap * sizeof(int)));
      MOLOT_CUDA(cudaMemset(counters, 0, cap * sizeof(int)));
      counters_cap = cap;
    }
    if (plan_ints > plan_cap) {
      cudaFree(plan);
      plan = nullptr;
      const size_t cap = std::max<size_t>(plan_ints, 4096);
      MOLOT_CUDA(cudaMalloc(&plan, cap * sizeof(int)));
      plan_cap = cap;
    }
    return MOLOT_OK;
  }

  int check(cudaStream_t st, bool clear) {
    if (!status) return MOLOT_OK;
    int h = 0;
    MOLOT_CUDA(cudaMemcpyAsync(&h, status, sizeof(int), cudaMemcpyDeviceToHost, st));
    MOLOT_CUDA(cudaStreamSynchronize(st));
    if (h != 0) {
      if (clear) {
        MOLOT_CUDA(cudaMemsetAsync(status, 0, sizeof(int), st));
        // A launch that gave up may have left tickets behind.
        MOLOT_CUDA(cudaMemsetAsync(counters, 0, counters_cap * sizeof(int), st));
        MOLOT_CUDA(cudaStreamSynchronize(st));
      }
      return fail(MOLOT_ERR_TIMEOUT, h == kDevErrConsumerTimeout
                                         ? "device wait for a KV tile timed out"
                                         : "device wait for a free KV stage timed out");
    }
    return MOLOT_OK;
  }
};

// ------------------------------------------------------------- dispatch

// FP32 kernels with split K/V stage barriers (hd <= 128; see gqa_decode_kernel).
bool pick_decode_split(int D, int G, KernelRef* k) { return pick_decode_f32(D, G, true, k); }

// kvt: the cache's molot_kv_dtype.
bool pick_decode_kv(int D, int G, int kvt, KernelRef* k) {
  switch (kvt) {
    case MOLOT_KV_BF16: return pick_decode_bf16(D, G, k);
    case MOLOT_KV_Q8: return pick_decode_q8(D, G, k);
  }
  return pick_decode_f32(D, G, false, k);
}

template <class CT>
const void* pick_append_t(int D) {
  switch (D) {
    case 64: return reinterpret_cast<const void*>(&norm_rope_append_kernel<64, CT>);
    case 128: return reinterpret_cast<const void*>(&norm_rope_append_kernel<128, CT>);
    case 256: return reinterpret_cast<const void*>(&norm_rope_append_kernel<256, CT>);
  }
  return nullptr;
}

const void* pick_append(int D, int kvt = MOLOT_KV_F32) {
  switch (kvt) {
    case MOLOT_KV_BF16: return pick_append_t<__nv_bfloat16>(D);
    case MOLOT_KV_Q8: return pick_append_t<Q8Row>(D);
  }
  return pick_append_t<float>(D);
}

int prepare_kernel(const KernelRef& k, int dev) {
  // The dynamic shared-memory opt-in is per function and device.
  static std::mutex mu;
  static std::vector<std::pair<const void*, int>> done;
  std::lock_guard<std::mutex> lk(mu);
  for (auto& p : done)
    if (p.first == k.fn && p.second == dev) return MOLOT_OK;
  MOLOT_CUDA(cudaFuncSetAttribute(k.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, k.smem));
  // 16-CTA clusters (plan_uniform) are a non-portable size.
  MOLOT_CUDA(cudaFuncSetAttribute(k.fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  done.emplace_back(k.fn, dev);
  return MOLOT_OK;
}

// Every kernel of the library is launched with programmatic stream
// serialisation: it may start while the preceding kernel drains, and reads
// what that kernel wrote only after griddepcontrol.wait.
int launch(const void* fn, dim3 grid, dim3 block, int smem, cudaStream_t st, void* arg) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* args[] = {arg};
  MOLOT_CUDA(cudaLaunchKernelExC(&cfg, fn, args));
  return MOLOT_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int window_start(int pos_cur, int window) {
  return (window > 0 && pos_cur - window + 1 > 0) ? pos_cur - window + 1 : 0;
}

int check_shape(int nq, int nkv, int d, KernelRef* k, int kvt = MOLOT_KV_F32) {
  if (nq <= 0 || nkv <= 0 || d <= 0) return fail(MOLOT_ERR_INVALID, "nq, nkv and d must be > 0");
  if (nq % nkv) return fail(MOLOT_ERR_INVALID, "nq must be a multiple of nkv");
  if (!pick_decode_kv(d, nq / nkv, kvt, k))
    return fail(MOLOT_ERR_UNSUPPORTED, "head_dim / group size combination not built: d=" +
                                           std::to_string(d) +
                                           " group=" + std::to_string(nq / nkv));
  return MOLOT_OK;
}

// One decode grid; split segments are merged inside it (by their last CTA,
// or by thread-block clusters, DecodeArgs::cluster).
int launch_decode(const KernelRef& k, DecodeArgs& a, cudaStream_t st) {
  take_withhold(a);
  if (a.cluster < 2) return launch(k.fn, dim3(a.grid), dim3(kDecodeThreads), k.smem, st, &a);
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = a.cluster;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.grid);
  cfg.blockDim = dim3(kDecodeThreads);
  cfg.dynamicSmemBytes = k.smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  void* args[] = {&a};
  MOLOT_CUDA(cudaLaunchKernelExC(&cfg, k.fn, args));
  return MOLOT_OK;
}

// Single-sequence decode over a strided contiguous cache.  prefetch_old_rows:
// see DecodeArgs (set only when the preceding launch is the library's append
// of slot n-1).
int decode_uniform(Workspace& ws, const float* Q, float* O, const void* K, const void* V,
                   int nq, int nkv, int n, int d, long long stride_t, long long stride_h,
                   float scale, int pos_cur, int window, cudaStream_t st,
                   bool prefetch_old_rows = false, const DecodeArgs* fused = nullptr,
                   int kvt = MOLOT_KV_F32) {
  KernelRef k;
  int rc = check_shape(nq, nkv, d, &k, kvt);
  if (rc) return rc;
  if (!Q || !O || !K || !V) return fail(MOLOT_ERR_INVALID, "null pointer");
  if (n < 0) return fail(MOLOT_ERR_INVALID, "n must be >= 0");
  if (!aligned16(K) || !aligned16(V) || (stride_t & 3) || (stride_h & 3))
    return fail(MOLOT_ERR_INVALID, "K/V must be 16-byte aligned with strides multiple of 4 floats");
  int dev;
  if ((rc = current_device(&dev))) return rc;
  const int t0 = window_start(pos_cur, window);
  if (n <= t0) {  // empty range: the reference leaves zeros (attn.h:163)
    MOLOT_CUDA(cudaMemsetAsync(O, 0, sizeof(float) * (size_t)nq * d, st));
    return MOLOT_OK;
  }
  const int blo = t0 / kBlk;
  const int nblk = (n + kBlk - 1) / kBlk - blo;
  const long long NB = (long long)nkv * nblk;
  if ((rc = prepare_kernel(k, dev))) return rc;
  UniformPlan up =
      plan_uniform(NB, nkv, nblk, sm_count(dev), max_active_clusters(k, kClusterCtas, dev),
                   max_active_clusters(k, kClusterCtasWide, dev));
  balance_uniform_grid(up, nkv, nblk);
  const int grid = up.grid;
  const int G = nq / nkv;
  if ((rc = ws.ensure(dev, (size_t)2 * grid * partial_record_floats(G, d), nkv, 0))) return rc;
  DecodeArgs a = {};
  a.grid = grid;
  a.aligned = up.aligned;  // one segment per CTA (see DecodeArgs)
  a.cluster = up.cluster;
  a.cl_per_seg = up.cl_per_seg;
  // The last CTA of a segment holds slot n-1: in a fused step it also
  // builds that row, in a decode right after the append that wrote it, it
  // can only stream that row once the append has completed.  Half a share
  // of slots for it measured best (cfg2 fused step, FP32 and BF16 caches),
  // a quarter on launches of under 8 tiles per CTA (cfg1 0.4167 -> 0.4135
  // ms per token; cfg3's clustered sliding-window layers 0.549 -> 0.533 ms
  // per token); the two forms keep one partition, so their results stay
  // bit-identical.
  const bool short_launch = (long long)nblk * kBlk * nkv / grid < 8LL * 64;
  a.tail_w = (fused || prefetch_old_rows) ? (short_launch ? kShareW * 3 / 4 : kShareW / 2) : 0;
  {
    // Split K/V stage barriers where they measured faster (see the kernel).
    const int tile_rows = d <= 64 ? TileShape<64, float>::T : TileShape<128, float>::T;
    const long long rows_per_cta = (long long)nblk * kBlk * nkv / grid;
    KernelRef ks;
    if (kvt == MOLOT_KV_F32 && d <= 128 && a.aligned && rows_per_cta >= 8LL * tile_rows &&
        pick_decode_split(d, G, &ks)) {
      k = ks;
      if ((rc = prepare_kernel(k, dev))) return rc;
    }
  }
  a.prefetch_old_rows = prefetch_old_rows ? 1 : 0;
  if (fused) {  // per-token prologue fused into this launch (slot n-1 is new)
    a.fused = 1;
    a.k_raw = fused->k_raw;
    a.v_raw = fused->v_raw;
    a.q_norm = fused->q_norm;
    a.k_norm = fused->k_norm;
    a.v_norm = fused->v_norm;
    a.eps = fused->eps;
    a.freq = fused->freq;
    a.pos = fused->pos;
    a.K_w = fused->K_w;
    a.V_w = fused->V_w;
  }
  a.Q = Q;
  a.q_bstride = (long long)nq * d;
  a.O = O;
  a.o_bstride = (long long)nq * d;
  a.K = K;
  a.V = V;
  a.kv_bstride = 0;
  a.stride_t = stride_t;
  a.stride_h = stride_h;
  a.block_table = nullptr;
  a.nkv = nkv;
  a.G = G;
  a.scale = scale;
  a.uniform = 1;
  a.n = n;
  a.t0 = t0;
  a.S = nkv;
  a.NB = NB;
  a.nblk_u = nblk;
  a.blo_u = blo;
  a.partials = ws.partials;
  a.counters = ws.counters;
  a.status = ws.status;
  a.timeout_ns = kWaitLimitNs;
  return launch_decode(k, a, st);
}

int append_launch(const AppendArgs& a, int d, int B, cudaStream_t st, int kvt = MOLOT_KV_F32) {
  const void* fn = pick_append(d, kvt);
  if (!fn) return fail(MOLOT_ERR_UNSUPPORTED, "head_dim not built: " + std::to_string(d));
  const int heads = a.nq + a.nkv;
  AppendArgs copy = a;
  return launch(fn, dim3((heads + kAppendWarps - 1) / kAppendWarps, B), dim3(kAppendWarps * 32), 0,
                st, &copy);
}

// ------------------------------------------------------------- host-call context

// Per-device state behind the synchronous host-buffer drop-ins.
struct HostCtx {
  std::mutex mu;
  int device = -1;
  cudaStream_t stream = nullptr;
  Workspace ws;
  float* buf = nullptr;
  size_t buf_cap = 0;  // floats

  int init(int dev) {
    if (device == dev) return MOLOT_OK;
    device = dev;
    MOLOT_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    return MOLOT_OK;
  }
  int reserve(size_t floats) {
    if (floats <= buf_cap) return MOLOT_OK;
    if (buf) cudaFree(buf);
    buf = nullptr;
    buf_cap = 0;
    MOLOT_CUDA(cudaMalloc(&buf, floats * sizeof(float)));
    buf_cap = floats;
    return MOLOT_OK;
  }
};

HostCtx& host_ctx(int dev) {
  static std::mutex mu;
  static std::vector<HostCtx*> ctxs;
  std::lock_guard<std::mutex> lk(mu);
  if ((int)ctxs.size() <= dev) ctxs.resize(dev + 1, nullptr);
  if (!ctxs[dev]) ctxs[dev] = new HostCtx();  // lives until process exit
  return *ctxs[dev];
}

size_t round4(size_t x) { return (x + 63) & ~size_t(63); }

// Copies Q/K/V in, runs decode_uniform over the staged copy, copies O out.
int host_decode(const float* Q, const float* K, const float* V, float* O, int nq, int nkv, int n,
                int d, bool head_major, float scale, int pos_cur, int window) {
  if (!Q || !K || !V || !O) return fail(MOLOT_ERR_INVALID, "null pointer");
  if (n < 0 || nq <= 0 || nkv <= 0 || d <= 0)
    return fail(MOLOT_ERR_INVALID, "sizes must be positive");
  int dev, rc;
  if ((rc = current_device(&dev))) return rc;
  HostCtx& c = host_ctx(dev);
  std::lock_guard<std::mutex> lk(c.mu);
  if ((rc = c.init(dev))) return rc;
  const size_t qn = (size_t)nq * d, kvn = (size_t)n * nkv * d;
  const size_t oq = 0, ok = round4(qn), ov = ok + round4(kvn), oo = ov + round4(kvn);
  if ((rc = c.reserve(oo + round4(qn)))) return rc;
  float* dq = c.buf + oq;
  float* dk = c.buf + ok;
  float* dv = c.buf + ov;
  float* dout = c.buf + oo;
  MOLOT_CUDA(cudaMemcpyAsync(dq, Q, qn * 4, cudaMemcpyHostToDevice, c.stream));
  if (kvn) {
    MOLOT_CUDA(cudaMemcpyAsync(dk, K, kvn * 4, cudaMemcpyHostToDevice, c.stream));
    MOLOT_CUDA(cudaMemcpyAsync(dv, V, kvn * 4, cudaMemcpyHostToDevice, c.stream));
  }
  const long long st_t = head_major ? d : (long long)nkv * d;
  const long long st_h = head_major ? (long long)n * d : d;
  rc = decode_uniform(c.ws, dq, dout, dk, dv, nq, nkv, n, d, st_t, st_h, scale, pos_cur, window,
                      c.stream);
  if (rc) return rc;
  MOLOT_CUDA(cudaMemcpyAsync(O, dout, qn * 4, cudaMemcpyDeviceToHost, c.stream));
  MOLOT_CUDA(cudaStreamSynchronize(c.stream));
  return c.ws.check(c.stream, true);
}

// ------------------------------------------------------------- prefill

// kvt: the cache's molot_kv_dtype.
bool pick_prefill(int D, KernelRef* k, int kvt = MOLOT_KV_F32) { return pick_prefill_kv(D, kvt, k); }

// gemm.h:409-446 on device buffers: Q/O [M][nq][d] (token stride q_tstride /
// o_tstride floats), slot t of kv head g at K + t*stride_t + g*stride_h.
int prefill_strided(Workspace& ws, const float* Q, long long q_tstride, float* O,
                    long long o_tstride, const void* K, const void* V, int nq, int nkv, int M,
                    int N, int d, long long stride_t, long long stride_h, float scale, int pos0,
                    int window, cudaStream_t st, int kvt = MOLOT_KV_F32) {
  if (!Q || !O || !K || !V) return fail(MOLOT_ERR_INVALID, "null pointer");
  if (nq <= 0 || nkv <= 0 || nq % nkv || M < 0 || N < 0 || pos0 < 0)
    return fail(MOLOT_ERR_INVALID, "bad sizes (nq must be a multiple of nkv)");
  const int G = nq / nkv;
  if (G > kPrefillRows || kPrefillRows % G)
    return fail(MOLOT_ERR_UNSUPPORTED, "prefill group size must divide 64");
  KernelRef k;
  if (!pick_prefill(d, &k, kvt)) return fail(MOLOT_ERR_UNSUPPORTED, "prefill head_dim not built");
  if (!aligned16(Q) || !aligned16(O) || !aligned16(K) || !aligned16(V) || (q_tstride & 3) ||
      (o_tstride & 3) || (stride_t & 3) || (stride_h & 3))
    return fail(MOLOT_ERR_INVALID, "buffers must be 16-byte aligned with strides multiple of 4");
  if (M == 0) return MOLOT_OK;
  int dev, rc;
  if ((rc = current_device(&dev))) return rc;
  if ((rc = ws.ensure(dev, 0, 0, 0))) return rc;
  // FP32 caches at head_dim 64/128: the split-TF32 tensor-core kernel
  // (128 query rows per CTA, so the group size must divide 128).
  KernelRef ktc;
  const bool tc = kvt == MOLOT_KV_F32 && kTcRows % G == 0 && pick_prefill_tc(d, &ktc);
  if (tc) k = ktc;
  if ((rc = prepare_kernel(k, dev))) return rc;
  PrefillArgs a = {};
  a.Q = Q;
  a.q_tstride = q_tstride;
  a.O = O;
  a.o_tstride = o_tstride;
  a.K = K;
  a.V = V;
  a.stride_t = stride_t;
  a.stride_h = stride_h;
  a.nq = nq;
  a.nkv = nkv;
  a.G = G;
  a.M = M;
  a.N = N;
  a.pos0 = pos0;
  a.window = window;
  a.scale = scale;
  a.BP = (tc ? kTcRows : kPrefillRows) / G;
  a.nblk_m = (M + a.BP - 1) / a.BP;
  a.status = ws.status;
  a.timeout_ns = kWaitLimitNs;
  return launch(k.fn, dim3(a.nblk_m, nkv), dim3(tc ? kTcThreads : kPrefillThreads), k.smem, st,
                &a);
}

// Host drop-in: stage Qm / K / V, run, copy Om back.
int host_prefill(const float* Qm, const float* K, const float* V, float* Om, int nq, int nkv,
                 int M, int N, int d, float scale, int pos0, int window) {
  if (!Qm || !K || !V || !Om) return fail(MOLOT_ERR_INVALID, "null pointer");
  if (M < 0 || N < 0 || nq <= 0 || nkv <= 0 || d <= 0)
    return fail(MOLOT_ERR_INVALID, "sizes must be non-negative");
  int dev, rc;
  if ((rc = current_device(&dev))) return rc;
  HostCtx& c = host_ctx(dev);
  std::lock_guard<std::mutex> lk(c.mu);
  if ((rc = c.init(dev))) return rc;
  const size_t qn = (size_t)M * nq * d, kvn = (size_t)N * nkv * d;
  const size_t oq = 0, ok = round4(qn), ov = ok + round4(kvn), oo = ov + round4(kvn);
  if ((rc = c.reserve(oo + round4(qn) + 4))) return rc;
  float* dq = c.buf + oq;
  float* dk = c.buf + ok;
  float* dv = c.buf + ov;
  float* dout = c.buf + oo;
  if (qn) MOLOT_CUDA(cudaMemcpyAsync(dq, Qm, qn * 4, cudaMemcpyHostToDevice, c.stream));
  if (kvn) {
    MOLOT_CUDA(cudaMemcpyAsync(dk, K, kvn * 4, cudaMemcpyHostToDevice, c.stream));
    MOLOT_CUDA(cudaMemcpyAsync(dv, V, kvn * 4, cudaMemcpyHostToDevice, c.stream));
  }
  rc = prefill_strided(c.ws, dq, (long long)nq * d, dout, (long long)nq * d, dk, dv, nq, nkv, M,
                       N, d, (long long)nkv * d, d, scale, pos0, window, c.stream);
  if (rc) return rc;
  if (qn) MOLOT_CUDA(cudaMemcpyAsync(Om, dout, qn * 4, cudaMemcpyDeviceToHost, c.stream));
  MOLOT_CUDA(cudaStreamSynchronize(c.stream));
  return c.ws.check(c.stream, true);
}

// ------------------------------------------------------------- Q4 GEMV

// y = W x in one launch (x is quantized inside it).
int gemv_q4_launch(const float* scales, const int8_t* zeros, const uint8_t* data, int rows,
                   int cols, const float* x, float* y, cudaStream_t st) {
  if (!scales || !zeros || !data || !x || !y) return fail(MOLOT_ERR_INVALID, "null pointer");
  if (rows <= 0 || cols <= 0 || cols % 32)
    return fail(MOLOT_ERR_INVALID, "rows > 0 and cols a positive multiple of 32 required");
  if (!aligned16(data) || !aligned16(x))
    return fail(MOLOT_ERR_INVALID, "data and x must be 16-byte aligned");
  const int ng = cols / 32;
  const int smem = gemv_smem_bytes(ng);
  if (smem > 200 * 1024) return fail(MOLOT_ERR_UNSUPPORTED, "cols too large for the Q4 GEMV");
  int dev, rc;
  if ((rc = current_device(&dev))) return rc;
  if ((rc = prepare_kernel({reinterpret_cast<const void*>(&gemv_q4_kernel), 200 * 1024}, dev)))
    return rc;
  GemvQ4Args a = {};
  a.scales = scales;
  a.zeros = zeros;
  a.data = data;
  a.x = x;
  a.y = y;
  a.rows = rows;
  a.cols = cols;
  a.ng = ng;
  return launch(reinterpret_cast<const void*>(&gemv_q4_kernel),
                dim3((rows + kGemvRows - 1) / kGemvRows), dim3(kGemvWarps * 32), smem, st, &a);
}

}  // namespace

// Lets other translation units of the library report through
// molot_last_error().
int set_last_error(int code, const char* msg) { return fail(code, msg); }

int max_active_clusters(const KernelRef& k, int cluster, int dev) {
  static std::mutex mu;
  struct Entry {
    const void* fn;
    int cluster, dev, n;
  };
  static std::vector<Entry> cache;
  std::lock_guard<std::mutex> lk(mu);
  for (auto& e : cache)
    if (e.fn == k.fn && e.cluster == cluster && e.dev == dev) return e.n;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cluster * 64);
  cfg.blockDim = dim3(kDecodeThreads);
  cfg.dynamicSmemBytes = k.smem;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, k.fn, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  cache.push_back({k.fn, cluster, dev, n});
  return n;
}

// molot_debug_withhold_next: pending request of the calling host thread.
thread_local unsigned long long g_withhold_ns = 0;

void take_withhold(DecodeArgs& a) {
  if (!g_withhold_ns) return;
  a.withhold = 1;
  a.timeout_ns = g_withhold_ns;
  g_withhold_ns = 0;
}

}  // namespace molot

using namespace molot;

// ===================================================================== C ABI

struct molot_kv_cache {
  int device = -1;
  int n_layers = 0, nkv = 0, hd = 0, cap = 0;
  int dtype = MOLOT_KV_F32;
  size_t elem = 4;         // bytes per stride unit (element; 1 for Q8)
  size_t layer_units = 0;  // stride units per K (or V) of one layer, padded
  unsigned char* base = nullptr;
  float* staging = nullptr;  // device copy of host rows for BF16 / Q8 writes
  size_t staging_cap = 0;    // floats
  // Row pitch in stride units: hd elements, or a Q8 row's bytes.
  int rs() const { return dtype == MOLOT_KV_Q8 ? q8_row_bytes(hd) : hd; }
  std::vector<int> len;
  Workspace ws;
  // The handle's two most recent kernel launches on its stream (index 0 =
  // latest), which decide whether a decode may stream older KV rows before
  // griddepcontrol.wait.  An append releases its successor at once; a decode
  // or step releases it only after its own wait, so when the preceding
  // launch is decode-type, everything before it is complete.
  enum Kind { kNone = 0, kAppend = 1, kDecode = 2 };
  int hist_kind[2] = {kNone, kNone};
  int hist_layer[2] = {-1, -1};  // layer whose cache that launch wrote
  void record(int kind, int layer) {
    hist_kind[1] = hist_kind[0];
    hist_layer[1] = hist_layer[0];
    hist_kind[0] = kind;
    hist_layer[0] = layer;
  }
  void ordered() {  // a copy in the stream completed everything before it
    hist_kind[0] = hist_kind[1] = kNone;
    hist_layer[0] = hist_layer[1] = -1;
  }
  // decode(L) right after append(L): rows below n-1 were written two or more
  // launches before the append, and the launch before the append neither
  // released early nor wrote layer L.
  bool decode_may_prefetch(int L) const {
    return hist_kind[0] == kAppend && hist_layer[0] == L && hist_kind[1] != kAppend &&
           hist_layer[1] != L;
  }
  // step(L): the preceding launch released this one only after its own
  // wait, and did not write layer L itself.
  bool step_may_prefetch(int L) const {
    return hist_kind[0] != kAppend && hist_layer[0] != L;
  }
};

struct molot_paged_plan {
  int device = -1;
  Workspace ws;
  int* h_plan = nullptr;  // pinned staging
  size_t h_cap = 0;
  cudaEvent_t uploaded = nullptr;
  bool built = false;
  int B = 0, nq = 0, nkv = 0, d = 0, window = 0, grid = 0, S = 0;
  long long NB = 0;
  // offsets (ints) into ws.plan
  size_t o_n = 0, o_t0 = 0, o_pos = 0, o_slot = 0, o_prefix = 0, o_cta = 0;
  std::vector<int> h_n, h_t0, h_pos, h_slot, h_prefix, h_cta;
  bool all_empty = false;
  // K pool whose newest slots the plan's most recent launch appended.
  const float* appended_pool = nullptr;
  int kvt = MOLOT_KV_F32;  // element type of the pools it is used with
  // Row pitch of the pools in stride units: d elements, or a Q8 row's bytes.
  int rs() const { return kvt == MOLOT_KV_Q8 ? q8_row_bytes(d) : d; }
};

extern "C" {

const char* molot_status_string(int status) {
  switch (status) {
    case MOLOT_OK: return "ok";
    case MOLOT_ERR_INVALID: return "invalid argument";
    case MOLOT_ERR_CUDA: return "CUDA error";
    case MOLOT_ERR_NOMEM: return "out of device memory";
    case MOLOT_ERR_CACHE_FULL: return "KV cache full";
    case MOLOT_ERR_CACHE_EMPTY: return "shared KV empty";
    case MOLOT_ERR_UNSUPPORTED: return "unsupported shape";
    case MOLOT_ERR_TIMEOUT: return "device wait timed out";
    case MOLOT_ERR_NO_DEVICE: return "no CUDA device";
  }
  return "unknown status";
}

const char* molot_last_error(void) { return g_last_error.c_str(); }

int molot_device_status(int clear) {
  int dev, rc;
  if ((rc = current_device(&dev))) return rc;
  HostCtx& c = host_ctx(dev);
  std::lock_guard<std::mutex> lk(c.mu);
  if ((rc = c.init(dev))) return rc;
  MOLOT_CUDA(cudaDeviceSynchronize());
  const int a = c.ws.check(c.stream, clear != 0);
  const int b = noalloc_status_check(dev, c.stream, clear != 0);
  return a ? a : b;
}

int molot_debug_withhold_next(unsigned long long wait_limit_ns) {
  g_withhold_ns = wait_limit_ns;
  return MOLOT_OK;
}

// ---------------------------------------------------------------- drop-ins

int molot_attn_decode_gqa_cache(const float* Q, const float* K, const float* V, float* O, int nq,
                                int nkv, int n, int qhd, float scale, int pos_cur, int window) {
  return host_decode(Q, K, V, O, nq, nkv, n, qhd, false, scale, pos_cur, window);
}

int molot_attn_decode_gqa(const float* Q, const float* K, const float* V, float* O, int nq,
                          int nkv, int n, int d, float scale) {
  // attn.h:106: the full causal prefix (window 0).
  return host_decode(Q, K, V, O, nq, nkv, n, d, true, scale, n > 0 ? n : 0, 0);
}

int molot_attn_decode_gqa_win(const float* Q, const float* K, const float* V, float* O, int nq,
                              int nkv, int n, int d, float scale, int pos_cur, int window) {
  return host_decode(Q, K, V, O, nq, nkv, n, d, true, scale, pos_cur, window);
}

int molot_attn_decode_head_win(const float* Q, const float* K, const float* V, float* out, int n,
                               int d, float scale, int pos_cur, int window) {
  return host_decode(Q, K, V, out, 1, 1, n, d, true, scale, pos_cur, window);
}

int molot_attn_decode_head(const float* Q, const float* K, const float* V, float* out, int n,
                           int d, float scale) {
  return host_decode(Q, K, V, out, 1, 1, n, d, true, scale, n > 0 ? n : 0, 0);
}

int molot_rope_apply(float* x, int d, int pos, const float* inv_freq) {
  if (!x || !inv_freq || d <= 0 || (d & 1)) return fail(MOLOT_ERR_INVALID, "bad rope arguments");
  if (!pick_append(d)) return fail(MOLOT_ERR_UNSUPPORTED, "head_dim not built");
  int dev, rc;
  if ((rc = current_device(&dev))) return rc;
  HostCtx& c = host_ctx(dev);
  std::lock_guard<std::mutex> lk(c.mu);
  if ((rc = c.init(dev))) return rc;
  if ((rc = c.reserve(round4(d) + round4(d / 2)))) return rc;
  float* dx = c.buf;
  float* df = c.buf + round4(d);
  MOLOT_CUDA(cudaMemcpyAsync(dx, x, (size_t)d * 4, cudaMemcpyHostToDevice, c.stream));
  MOLOT_CUDA(cudaMemcpyAsync(df, inv_freq, (size_t)(d / 2) * 4, cudaMemcpyHostToDevice, c.stream));
  AppendArgs a = {};
  a.q_in = dx;
  a.q_out = dx;
  a.freq = df;
  a.nq = 1;
  a.nkv = 0;
  a.pos = pos;
  if ((rc = append_launch(a, d, 1, c.stream))) return rc;
  MOLOT_CUDA(cudaMemcpyAsync(x, dx, (size_t)d * 4, cudaMemcpyDeviceToHost, c.stream));
  MOLOT_CUDA(cudaStreamSynchronize(c.stream));
  return MOLOT_OK;
}

int molot_rope_inv_freq(float base, int d, float* out) {
  if (!out || d <= 0) return fail(MOLOT_ERR_INVALID, "bad rope_inv_freq arguments");
  for (int i = 0; i < d / 2; ++i) out[i] = 1.0f / std::pow(base, (2.0f * (float)i) / (float)d);
  return MOLOT_OK;
}

// ---------------------------------------------------------------- device forms

int molot_attn_decode_strided_dev(const float* Q, const float* K, const float* V, float* O,
                                  int nq, int nkv, int n, int d, long long stride_t,
                                  long long stride_h, float scale, int pos_cur, int window,
                                  void* stream) {
  KernelRef k;
  int dev, rc;
  if ((rc = check_shape(nq, nkv, d, &k))) return rc;
  if ((rc = current_device(&dev))) return rc;
  HostCtx& c = host_ctx(dev);
  std::lock_guard<std::mutex> lk(c.mu);
  return decode_uniform(c.ws, Q, O, K, V, nq, nkv, n, d, stride_t, stride_h, scale, pos_cur,
                        window, (cudaStream_t)stream);
}

namespace molot {
namespace {
// The per-token prologue into a strided single-sequence cache: slot `slot`
// of kv head g lives at kc + slot*stride_t + g*stride_h.
int append_strided(const float* q, const float* k, const float* v, float* q_out,
                   const float* q_norm, const float* k_norm, int v_norm, float eps,
                   const float* freq, int pos, float* kc, float* vc, int slot, int nq, int nkv,
                   int d, long long stride_t, long long stride_h, cudaStream_t st,
                   int kvt = MOLOT_KV_F32) {
  // k, v, kc and vc all null: q only (a shared-KV layer's query, forward.h:554-558)
  const bool q_only = !k && !v && !kc && !vc;
  if (!q || !q_out || (!q_only && (!k || !v || !kc || !vc)))
    return fail(MOLOT_ERR_INVALID, "null pointer");
  if (nq <= 0 || nkv <= 0 || slot < 0) return fail(MOLOT_ERR_INVALID, "bad sizes");
  AppendArgs a = {};
  a.q_in = q;
  a.k_in = k;
  a.v_in = v;
  a.q_out = q_out;
  a.q_norm = q_norm;
  a.k_norm = k_norm;
  a.v_norm = v_norm;
  a.eps = eps;
  a.freq = freq;
  a.nq = nq;
  a.nkv = q_only ? 0 : nkv;  // the kernel runs one warp per q and k head
  a.pos = pos;
  a.slot = slot;
  a.K = kc;
  a.V = vc;
  a.stride_t = stride_t;
  a.stride_h = stride_h;
  return append_launch(a, d, 1, st, kvt);
}
}  // namespace
}  // namespace molot

int molot_norm_rope_append_dev(const float* q, const float* k, const float* v, float* q_out,
                               const float* q_norm, const float* k_norm, int v_norm, float eps,
                               const float* freq, int pos, float* kc, float* vc, int slot,
                               int nq, int nkv, int d, void* stream) {
  return append_strided(q, k, v, q_out, q_norm, k_norm, v_norm, eps, freq, pos, kc, vc, slot, nq,
                        nkv, d, (long long)nkv * d, d, (cudaStream_t)stream);
}

// ---------------------------------------------------------------- KV cache handle

int molot_kv_create(int n_layers, int nkv, int hd, int cap, molot_kv_cache** out) {
  return molot_kv_create_ex(n_layers, nkv, hd, cap, MOLOT_KV_F32, out);
}

int molot_kv_dtype(const molot_kv_cache* kv) {
  if (!kv) return fail(MOLOT_ERR_INVALID, "null handle");
  return kv->dtype;
}

int molot_kv_create_ex(int n_layers, int nkv, int hd, int cap, int kv_dtype,
                       molot_kv_cache** out) {
  if (!out) return fail(MOLOT_ERR_INVALID, "null out");
  *out = nullptr;
  if (n_layers <= 0 || nkv <= 0 || hd <= 0 || cap <= 0)
    return fail(MOLOT_ERR_INVALID, "sizes must be positive");
  if (kv_dtype != MOLOT_KV_F32 && kv_dtype != MOLOT_KV_BF16 && kv_dtype != MOLOT_KV_Q8)
    return fail(MOLOT_ERR_INVALID, "kv_dtype must be MOLOT_KV_F32, MOLOT_KV_BF16 or MOLOT_KV_Q8");
  if (!pick_append(hd, kv_dtype)) return fail(MOLOT_ERR_UNSUPPORTED, "head_dim not built");
  int dev, rc;
  if ((rc = current_device(&dev))) return rc;
  auto* kv = new molot_kv_cache();
  kv->device = dev;
  kv->n_layers = n_layers;
  kv->nkv = nkv;
  kv->hd = hd;
  kv->cap = cap;
  kv->dtype = kv_dtype;
  kv->elem = kv_dtype == MOLOT_KV_BF16 ? 2 : (kv_dtype == MOLOT_KV_Q8 ? 1 : 4);
  const size_t align = 256 / kv->elem;  // 256-byte aligned layers
  kv->layer_units = ((size_t)cap * nkv * kv->rs() + align - 1) & ~(align - 1);
  kv->len.assign(n_layers, 0);
  cudaError_t e = cudaMalloc(&kv->base, kv->layer_units * 2 * n_layers * kv->elem);
  if (e != cudaSuccess) {
    delete kv;
    return cuda_fail(e, "cudaMalloc(kv cache)");
  }
  *out = kv;
  return MOLOT_OK;
}

void molot_kv_destroy(molot_kv_cache* kv) {
  if (!kv) return;
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(kv->device);
  cudaDeviceSynchronize();
  cudaFree(kv->base);
  cudaFree(kv->staging);
  kv->ws.release();
  if (prev >= 0) cudaSetDevice(prev);
  delete kv;
}

int molot_kv_length(const molot_kv_cache* kv, int layer) {
  if (!kv || layer < 0 || layer >= kv->n_layers) return fail(MOLOT_ERR_INVALID, "bad layer");
  return kv->len[layer];
}

int molot_kv_set_length(molot_kv_cache* kv, int layer, int n) {
  if (!kv || layer < 0 || layer >= kv->n_layers || n < 0 || n > kv->cap)
    return fail(MOLOT_ERR_INVALID, "bad layer or length");
  kv->len[layer] = n;
  return MOLOT_OK;
}

int molot_kv_layer_data(molot_kv_cache* kv, int layer, float** k, float** v) {
  if (!kv || layer < 0 || layer >= kv->n_layers) return fail(MOLOT_ERR_INVALID, "bad layer");
  if (k) *k = reinterpret_cast<float*>(kv->base + (size_t)(2 * layer) * kv->layer_units * kv->elem);
  if (v) *v = reinterpret_cast<float*>(kv->base + (size_t)(2 * layer + 1) * kv->layer_units * kv->elem);
  return MOLOT_OK;
}

int molot_kv_write(molot_kv_cache* kv, int layer, int slot0, int nrows, const float* k,
                   const float* v, void* stream) {
  if (!kv || layer < 0 || layer >= kv->n_layers) return fail(MOLOT_ERR_INVALID, "bad layer");
  if (!k || !v || slot0 < 0 || nrows < 0 || slot0 + nrows > kv->cap)
    return fail(MOLOT_ERR_INVALID, "rows outside the cache");
  if (nrows == 0) return MOLOT_OK;
  kv->ordered();
  float *kc, *vc;
  molot_kv_layer_data(kv, layer, &kc, &vc);
  if (kv->dtype != MOLOT_KV_F32) {
    // Rows are converted on the device; host rows are staged there first.
    const size_t n = (size_t)nrows * kv->nkv * kv->hd;
    cudaPointerAttributes pa{};
    const bool dev_src = cudaPointerGetAttributes(&pa, k) == cudaSuccess &&
                         (pa.type == cudaMemoryTypeDevice || pa.type == cudaMemoryTypeManaged);
    cudaGetLastError();  // a host pointer may leave an error behind on older drivers
    const float *ks = k, *vs = v;
    cudaStream_t st = (cudaStream_t)stream;
    if (!dev_src) {
      if (kv->staging_cap < 2 * n) {
        MOLOT_CUDA(cudaStreamSynchronize(st));
        cudaFree(kv->staging);
        kv->staging = nullptr;
        kv->staging_cap = 0;
        MOLOT_CUDA(cudaMalloc(&kv->staging, 2 * n * sizeof(float)));
        kv->staging_cap = 2 * n;
      }
      MOLOT_CUDA(cudaMemcpyAsync(kv->staging, k, n * 4, cudaMemcpyHostToDevice, st));
      MOLOT_CUDA(cudaMemcpyAsync(kv->staging + n, v, n * 4, cudaMemcpyHostToDevice, st));
      ks = kv->staging;
      vs = kv->staging + n;
    }
    if (kv->dtype == MOLOT_KV_Q8)
      kv_rows_to_cache_q8_kernel<Q8Row><<<dim3(nrows, kv->nkv), kv->hd, 0, st>>>(
          ks, vs, reinterpret_cast<unsigned char*>(kc), reinterpret_cast<unsigned char*>(vc),
          slot0, kv->nkv, kv->hd, (long long)kv->cap * kv->rs());
    else
      kv_rows_to_cache_kernel<__nv_bfloat16><<<dim3(nrows, kv->nkv), 128, 0, st>>>(
          ks, vs, reinterpret_cast<__nv_bfloat16*>(kc), reinterpret_cast<__nv_bfloat16*>(vc),
          slot0, kv->nkv, kv->hd, (long long)kv->cap * kv->hd);
    MOLOT_CUDA(cudaGetLastError());
    return MOLOT_OK;
  }
  // [nrows][nkv*hd] rows in, [nkv][cap][hd] head-major cache out: one
  // strided copy per kv head.
  const size_t hd = kv->hd, src_pitch = (size_t)kv->nkv * hd * sizeof(float);
  cudaStream_t st = (cudaStream_t)stream;
  for (int g = 0; g < kv->nkv; ++g) {
    const size_t off = (size_t)g * kv->cap * hd + (size_t)slot0 * hd;
    MOLOT_CUDA(cudaMemcpy2DAsync(kc + off, hd * sizeof(float), k + g * hd, src_pitch,
                                 hd * sizeof(float), nrows, cudaMemcpyDefault, st));
    MOLOT_CUDA(cudaMemcpy2DAsync(vc + off, hd * sizeof(float), v + g * hd, src_pitch,
                                 hd * sizeof(float), nrows, cudaMemcpyDefault, st));
  }
  return MOLOT_OK;
}

int molot_attn_append_rope(molot_kv_cache* kv, int layer, const float* q, const float* k,
                           const float* v, float* q_out, const float* q_norm,
                           const float* k_norm, int v_norm, float eps, const float* freq,
                           int pos, int nq, void* stream) {
  if (!kv || layer < 0 || layer >= kv->n_layers) return fail(MOLOT_ERR_INVALID, "bad layer");
  if (kv->len[layer] >= kv->cap) return fail(MOLOT_ERR_CACHE_FULL, "fwd: KV cache full");
  float *kc, *vc;
  molot_kv_layer_data(kv, layer, &kc, &vc);
  int rc = append_strided(q, k, v, q_out, q_norm, k_norm, v_norm, eps, freq, pos, kc, vc,
                          kv->len[layer], nq, kv->nkv, kv->hd, kv->rs(), (long long)kv->cap * kv->rs(),
                          (cudaStream_t)stream, kv->dtype);
  if (rc) return rc;
  kv->len[layer]++;
  kv->record(molot_kv_cache::kAppend, layer);
  return MOLOT_OK;
}

int molot_attn_decode(molot_kv_cache* kv, int src_layer, const float* q, float* o, int nq,
                      float scale, int pos_cur, int window, void* stream) {
  if (!kv || src_layer < 0 || src_layer >= kv->n_layers)
    return fail(MOLOT_ERR_INVALID, "bad layer");
  const int n = kv->len[src_layer];
  if (n == 0) return fail(MOLOT_ERR_CACHE_EMPTY, "fwd: shared KV empty");
  float *kc, *vc;
  molot_kv_layer_data(kv, src_layer, &kc, &vc);
  const bool prefetch = kv->decode_may_prefetch(src_layer);
  int rc = decode_uniform(kv->ws, q, o, kc, vc, nq, kv->nkv, n, kv->hd, kv->rs(),
                          (long long)kv->cap * kv->rs(), scale, pos_cur, window,
                          (cudaStream_t)stream, prefetch, nullptr, kv->dtype);
  if (rc == MOLOT_OK) kv->record(molot_kv_cache::kDecode, -1);
  return rc;
}

int molot_attn_step(molot_kv_cache* kv, int layer, const float* q, const float* k,
                    const float* v, const float* q_norm, const float* k_norm, int v_norm,
                    float eps, const float* freq, int pos, float* o, int nq, float scale,
                    int window, void* stream) {
  if (!kv || layer < 0 || layer >= kv->n_layers) return fail(MOLOT_ERR_INVALID, "bad layer");
  if (!q || !k || !v || !o) return fail(MOLOT_ERR_INVALID, "null pointer");
  if (kv->len[layer] >= kv->cap) return fail(MOLOT_ERR_CACHE_FULL, "fwd: KV cache full");
  float *kc, *vc;
  molot_kv_layer_data(kv, layer, &kc, &vc);
  DecodeArgs f = {};
  f.k_raw = k;
  f.v_raw = v;
  f.q_norm = q_norm;
  f.k_norm = k_norm;
  f.v_norm = v_norm;
  f.eps = eps;
  f.freq = freq;
  f.pos = pos;
  f.K_w = kc;
  f.V_w = vc;
  const int n = kv->len[layer] + 1;  // the new token occupies slot n-1
  if (n <= window_start(pos, window)) {
    // Nothing to attend to (attn.h:163 leaves zeros); still append the row.
    // The rotated q goes to o, which the memset then clears.
    int rc = append_strided(q, k, v, o, q_norm, k_norm, v_norm, eps, freq, pos, kc, vc,
                            n - 1, nq, kv->nkv, kv->hd, kv->rs(), (long long)kv->cap * kv->rs(),
                            (cudaStream_t)stream, kv->dtype);
    if (rc) return rc;
    MOLOT_CUDA(cudaMemsetAsync(o, 0, sizeof(float) * (size_t)nq * kv->hd, (cudaStream_t)stream));
    kv->len[layer] = n;
    kv->ordered();
    return MOLOT_OK;
  }
  const bool prefetch = kv->step_may_prefetch(layer);
  int rc = decode_uniform(kv->ws, q, o, kc, vc, nq, kv->nkv, n, kv->hd, kv->rs(),
                          (long long)kv->cap * kv->rs(), scale, pos, window, (cudaStream_t)stream,
                          prefetch, &f, kv->dtype);
  if (rc) return rc;
  kv->len[layer] = n;
  kv->record(molot_kv_cache::kDecode, layer);
  return MOLOT_OK;
}

// forward.h:368-392 for M tokens of a KV-owning layer: per-token QK-norm /
// V-norm / RoPE at positions pos0..pos0+M-1, rows appended at slots
// n..n+M-1, n += M.
int molot_attn_append_rope_tokens(molot_kv_cache* kv, int layer, const float* q, const float* k,
                                  const float* v, float* q_out, const float* q_norm,
                                  const float* k_norm, int v_norm, float eps, const float* freq,
                                  int pos0, int M, int nq, void* stream) {
  if (!kv || layer < 0 || layer >= kv->n_layers) return fail(MOLOT_ERR_INVALID, "bad layer");
  if (!q || !k || !v || !q_out) return fail(MOLOT_ERR_INVALID, "null pointer");
  if (M < 0 || M > 65535 || nq <= 0 || nq % kv->nkv || pos0 < 0)
    return fail(MOLOT_ERR_INVALID, "bad token count / nq");
  if (M == 0) return MOLOT_OK;
  const int n = kv->len[layer];
  if (n + M > kv->cap) return fail(MOLOT_ERR_CACHE_FULL, "fwd: KV cache full");
  float *kc, *vc;
  molot_kv_layer_data(kv, layer, &kc, &vc);
  AppendArgs a = {};
  a.q_in = q;
  a.q_bstride = (long long)nq * kv->hd;
  a.k_in = k;
  a.v_in = v;
  a.kv_in_bstride = (long long)kv->nkv * kv->hd;
  a.q_out = q_out;
  a.qo_bstride = (long long)nq * kv->hd;
  a.q_norm = q_norm;
  a.k_norm = k_norm;
  a.v_norm = v_norm;
  a.eps = eps;
  a.freq = freq;
  a.nq = nq;
  a.nkv = kv->nkv;
  a.pos = pos0;
  a.slot = n;
  a.tok_step = 1;
  a.K = kc;
  a.V = vc;
  a.kv_bstride = 0;
  a.stride_t = kv->rs();
  a.stride_h = (long long)kv->cap * kv->rs();
  int rc = append_launch(a, kv->hd, M, (cudaStream_t)stream, kv->dtype);
  if (rc) return rc;
  kv->len[layer] = n + M;
  kv->record(molot_kv_cache::kAppend, layer);
  return MOLOT_OK;
}

// gemm.h:409-446 over the cache of src_layer (its current length N; the
// layer itself or its shared-KV source): q, o [M][nq][hd] device.
int molot_attn_prefill(molot_kv_cache* kv, int src_layer, const float* q, float* o, int nq, int M,
                       float scale, int pos0, int window, void* stream) {
  if (!kv || src_layer < 0 || src_layer >= kv->n_layers)
    return fail(MOLOT_ERR_INVALID, "bad layer");
  if (nq <= 0 || nq % kv->nkv) return fail(MOLOT_ERR_INVALID, "nq must be a multiple of nkv");
  float *kc, *vc;
  molot_kv_layer_data(kv, src_layer, &kc, &vc);
  const int hd = kv->hd;
  int rc = prefill_strided(kv->ws, q, (long long)nq * hd, o, (long long)nq * hd, kc, vc, nq,
                           kv->nkv, M, kv->len[src_layer], hd, kv->rs(),
                           (long long)kv->cap * kv->rs(), scale, pos0, window,
                           (cudaStream_t)stream, kv->dtype);
  if (rc) return rc;
  kv->record(molot_kv_cache::kDecode, -1);  // releases its successor after its own wait
  return MOLOT_OK;
}

int molot_attn_prefill_strided_dev(const float* Q, const float* K, const float* V, float* O,
                                   int nq, int nkv, int M, int N, int d, long long stride_t,
                                   long long stride_h, float scale, int pos0, int window,
                                   void* stream) {
  int dev, rc;
  if ((rc = current_device(&dev))) return rc;
  HostCtx& c = host_ctx(dev);
  std::lock_guard<std::mutex> lk(c.mu);
  return prefill_strided(c.ws, Q, (long long)nq * d, O, (long long)nq * d, K, V, nq, nkv, M, N,
                         d, stride_t, stride_h, scale, pos0, window, (cudaStream_t)stream);
}

int molot_attn_prefill_gqa(const float* Qm, const float* K, const float* V, float* Om, int nq,
                           int nkv, int M, int N, int d, float scale, int pos0, int window) {
  return host_prefill(Qm, K, V, Om, nq, nkv, M, N, d, scale, pos0, window);
}

int molot_gemv_q4_dev(const float* scales, const int8_t* zeros, const uint8_t* data, int rows,
                      int cols, const float* x, float* y, void* stream) {
  return gemv_q4_launch(scales, zeros, data, rows, cols, x, y, (cudaStream_t)stream);
}

int molot_gemv_q4(const float* scales, const int8_t* zeros, const uint8_t* data,
                  const int16_t* wsums, int rows, int cols, const float* x, float* y) {
  (void)wsums;  // the VNNI bias correction of the CPU path; not needed here
  if (!scales || !zeros || !data || !x || !y) return fail(MOLOT_ERR_INVALID, "null pointer");
  if (rows <= 0 || cols <= 0 || cols % 32)
    return fail(MOLOT_ERR_INVALID, "rows > 0 and cols a positive multiple of 32 required");
  int dev, rc;
  if ((rc = current_device(&dev))) return rc;
  HostCtx& c = host_ctx(dev);
  std::lock_guard<std::mutex> lk(c.mu);
  if ((rc = c.init(dev))) return rc;
  const size_t ng = cols / 32, nsc = rows * ng;
  // staging (floats): scales, x, y, then zeros and nibbles as bytes
  const size_t o_sc = 0, o_x = round4(nsc), o_y = o_x + round4(cols), o_b = o_y + round4(rows);
  const size_t bytes = nsc + (size_t)rows * cols / 2;
  if ((rc = c.reserve(o_b + round4((bytes + 3) / 4) + 16))) return rc;
  float* dsc = c.buf + o_sc;
  float* dx = c.buf + o_x;
  float* dy = c.buf + o_y;
  uint8_t* dz = reinterpret_cast<uint8_t*>(c.buf + o_b);
  uint8_t* dd = dz + ((nsc + 15) & ~size_t(15));
  MOLOT_CUDA(cudaMemcpyAsync(dsc, scales, nsc * 4, cudaMemcpyHostToDevice, c.stream));
  MOLOT_CUDA(cudaMemcpyAsync(dx, x, (size_t)cols * 4, cudaMemcpyHostToDevice, c.stream));
  MOLOT_CUDA(cudaMemcpyAsync(dz, zeros, nsc, cudaMemcpyHostToDevice, c.stream));
  MOLOT_CUDA(cudaMemcpyAsync(dd, data, (size_t)rows * cols / 2, cudaMemcpyHostToDevice, c.stream));
  rc = gemv_q4_launch(dsc, reinterpret_cast<const int8_t*>(dz), dd, rows, cols, dx, dy,
                      c.stream);
  if (rc) return rc;
  MOLOT_CUDA(cudaMemcpyAsync(y, dy, (size_t)rows * 4, cudaMemcpyDeviceToHost, c.stream));
  MOLOT_CUDA(cudaStreamSynchronize(c.stream));
  return c.ws.check(c.stream, true);
}

int molot_kv_check(molot_kv_cache* kv, void* stream) {
  if (!kv) return fail(MOLOT_ERR_INVALID, "null handle");
  MOLOT_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
  MOLOT_CUDA(cudaGetLastError());
  return kv->ws.check((cudaStream_t)stream, true);
}

// ---------------------------------------------------------------- paged plans

int molot_paged_plan_create(molot_paged_plan** out) {
  if (!out) return fail(MOLOT_ERR_INVALID, "null out");
  int dev, rc;
  if ((rc = current_device(&dev))) return rc;
  auto* p = new molot_paged_plan();
  p->device = dev;
  cudaError_t e = cudaEventCreateWithFlags(&p->uploaded, cudaEventDisableTiming);
  if (e != cudaSuccess) {
    delete p;
    return cuda_fail(e, "cudaEventCreate");
  }
  *out = p;
  return MOLOT_OK;
}

void molot_paged_plan_destroy(molot_paged_plan* p) {
  if (!p) return;
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(p->device);
  cudaDeviceSynchronize();
  if (p->h_plan) cudaFreeHost(p->h_plan);
  if (p->uploaded) cudaEventDestroy(p->uploaded);
  p->ws.release();
  if (prev >= 0) cudaSetDevice(prev);
  delete p;
}

int molot_paged_plan_set_kv_dtype(molot_paged_plan* p, int kv_dtype) {
  if (!p) return fail(MOLOT_ERR_INVALID, "null plan");
  if (kv_dtype != MOLOT_KV_F32 && kv_dtype != MOLOT_KV_BF16 && kv_dtype != MOLOT_KV_Q8)
    return fail(MOLOT_ERR_INVALID, "kv_dtype must be MOLOT_KV_F32, MOLOT_KV_BF16 or MOLOT_KV_Q8");
  p->kvt = kv_dtype;
  p->appended_pool = nullptr;
  return MOLOT_OK;
}

int molot_paged_plan_build(molot_paged_plan* p, int B, int nq, int nkv, int d,
                           const int* seq_lens, const int* positions, int window, void* stream) {
  if (!p || !seq_lens || B <= 0) return fail(MOLOT_ERR_INVALID, "bad plan arguments");
  KernelRef k;
  int rc = check_shape(nq, nkv, d, &k);
  if (rc) return rc;
  const int S = B * nkv;
  p->h_n.assign(seq_lens, seq_lens + B);
  p->h_t0.resize(B);
  p->h_pos.resize(B);
  p->h_slot.resize(B);
  p->h_prefix.resize(S + 1);
  long long NB = 0;
  for (int b = 0; b < B; ++b) {
    const int n = seq_lens[b];
    if (n < 0) return fail(MOLOT_ERR_INVALID, "negative sequence length");
    const int pos = positions ? positions[b] : n - 1;
    const int t0 = window_start(pos, window);
    p->h_pos[b] = pos;
    p->h_slot[b] = n - 1;
    p->h_t0[b] = t0;
    const int nblk = n > t0 ? (n + kBlk - 1) / kBlk - t0 / kBlk : 0;
    for (int g = 0; g < nkv; ++g) {
      p->h_prefix[b * nkv + g] = (int)NB;
      NB += nblk;
    }
  }
  p->h_prefix[S] = (int)NB;
  if (NB >= (1ll << 31)) return fail(MOLOT_ERR_INVALID, "batch too large");
  int dev;
  if ((rc = current_device(&dev))) return rc;
  if (dev != p->device) return fail(MOLOT_ERR_INVALID, "plan used on another device");
  const int grid = (int)std::max<long long>(1, std::min<long long>(NB, sm_count(dev)));
  p->h_cta.resize(grid);
  {
    int s = 0;
    for (int c = 0; c < grid; ++c) {
      const long long start = (long long)c * NB / grid;
      while (s < S && p->h_prefix[s + 1] <= start) ++s;
      p->h_cta[c] = std::min(s, S - 1);
    }
  }
  p->B = B;
  p->nq = nq;
  p->nkv = nkv;
  p->d = d;
  p->window = window;
  p->grid = grid;
  p->S = S;
  p->NB = NB;
  p->all_empty = NB == 0;
  // layout of the uploaded plan
  p->o_n = 0;
  p->o_t0 = p->o_n + B;
  p->o_pos = p->o_t0 + B;
  p->o_slot = p->o_pos + B;
  p->o_prefix = p->o_slot + B;
  p->o_cta = p->o_prefix + S + 1;
  const size_t total = p->o_cta + grid;
  const int G = nq / nkv;
  if ((rc = p->ws.ensure(dev, (size_t)2 * grid * partial_record_floats(G, d), S, total))) return rc;
  if (p->h_cap < total) {
    if (p->h_plan) {
      MOLOT_CUDA(cudaEventSynchronize(p->uploaded));
      cudaFreeHost(p->h_plan);
      p->h_plan = nullptr;
    }
    MOLOT_CUDA(cudaMallocHost(&p->h_plan, total * sizeof(int)));
    p->h_cap = total;
  } else if (p->built) {
    MOLOT_CUDA(cudaEventSynchronize(p->uploaded));  // staging still being read?
  }
  std::memcpy(p->h_plan + p->o_n, p->h_n.data(), B * sizeof(int));
  std::memcpy(p->h_plan + p->o_t0, p->h_t0.data(), B * sizeof(int));
  std::memcpy(p->h_plan + p->o_pos, p->h_pos.data(), B * sizeof(int));
  std::memcpy(p->h_plan + p->o_slot, p->h_slot.data(), B * sizeof(int));
  std::memcpy(p->h_plan + p->o_prefix, p->h_prefix.data(), (S + 1) * sizeof(int));
  std::memcpy(p->h_plan + p->o_cta, p->h_cta.data(), grid * sizeof(int));
  cudaStream_t st = (cudaStream_t)stream;
  MOLOT_CUDA(cudaMemcpyAsync(p->ws.plan, p->h_plan, total * sizeof(int), cudaMemcpyHostToDevice, st));
  MOLOT_CUDA(cudaEventRecord(p->uploaded, st));
  p->built = true;
  return MOLOT_OK;
}

}  // extern "C"

namespace molot {
namespace {
// molot_paged_decode, or with a comm its gathering form: outputs into every
// rank's gathered buffer at float offset out_offset ([B][nranks*nq][d]).
int paged_decode_impl(molot_paged_plan* p, const float* Q, float* O, const float* k_pool,
                      const float* v_pool, const int* block_table, int max_pages, int page_size,
                      float scale, cudaStream_t st, molot_comm* c, size_t out_offset) {
  if (!p || !p->built) return fail(MOLOT_ERR_INVALID, "plan not built");
  if (!Q || (!O && !c) || !k_pool || !v_pool || !block_table)
    return fail(MOLOT_ERR_INVALID, "null pointer");
  if (page_size <= 0 || page_size % kBlk) return fail(MOLOT_ERR_INVALID, "page_size must be a multiple of 16");
  if (!aligned16(k_pool) || !aligned16(v_pool)) return fail(MOLOT_ERR_INVALID, "pools must be 16-byte aligned");
  int dev, rc;
  if ((rc = current_device(&dev))) return rc;
  if (dev != p->device) return fail(MOLOT_ERR_INVALID, "plan used on another device");
  KernelRef k;
  if ((rc = check_shape(p->nq, p->nkv, p->d, &k, p->kvt))) return rc;
  DecodeArgs a = {};
  a.o_bstride = (long long)p->nq * p->d;
  if (c) {
    if (!c->opened) return fail(MOLOT_ERR_INVALID, "comm not opened");
    if (c->device != dev) return fail(MOLOT_ERR_INVALID, "comm used on another device");
    const size_t row = (size_t)c->nranks * p->nq * p->d;  // floats per sequence
    if (out_offset % 4 || (out_offset + (size_t)p->B * row) * sizeof(float) > c->data_bytes)
      return fail(MOLOT_ERR_INVALID, "gathered outputs outside the comm buffer (or offset not a "
                                     "multiple of 4 floats)");
    for (int b = 0; b < p->B; ++b)
      if (p->h_n[b] <= p->h_t0[b])
        return fail(MOLOT_ERR_INVALID, "peer gather needs every sequence to attend >= 1 slot");
    a.npeer = c->nranks;
    for (int r = 0; r < c->nranks; ++r) {
      a.peer_O[r] = reinterpret_cast<float*>(c->peer_base[r]) + out_offset +
                    (size_t)c->rank * p->nq * p->d;
      a.peer_flag[r] = &c->ctl(r)->flags[c->rank];
    }
    a.done_ctr = &c->own_ctl()->done;
    a.epoch = &c->own_ctl()->epoch;
    O = a.peer_O[c->rank];
    a.o_bstride = (long long)row;
  } else {
    // Sequences with an empty attended range produce zeros (attn.h:163).
    for (int b = 0; b < p->B; ++b)
      if (p->h_n[b] <= p->h_t0[b])
        MOLOT_CUDA(cudaMemsetAsync(O + (size_t)b * p->nq * p->d, 0, sizeof(float) * p->nq * p->d, st));
    if (p->all_empty) return MOLOT_OK;
  }
  if ((rc = prepare_kernel(k, dev))) return rc;
  a.Q = Q;
  a.q_bstride = (long long)p->nq * p->d;
  a.O = O;
  a.K = k_pool;
  a.V = v_pool;
  a.block_table = block_table;
  a.bt_stride = max_pages;
  a.page_size = page_size;
  a.page_stride = (long long)p->nkv * page_size * p->rs();
  a.page_hstride = (long long)page_size * p->rs();
  a.nkv = p->nkv;
  a.G = p->nq / p->nkv;
  a.scale = scale;
  a.uniform = 0;
  a.seq_n = p->ws.plan + p->o_n;
  a.seq_t0 = p->ws.plan + p->o_t0;
  a.seg_prefix = p->ws.plan + p->o_prefix;
  a.cta_seg = p->ws.plan + p->o_cta;
  a.S = p->S;
  a.NB = p->NB;
  a.partials = p->ws.partials;
  a.counters = p->ws.counters;
  a.status = p->ws.status;
  a.timeout_ns = kWaitLimitNs;
  a.grid = p->grid;
  // Older slots were written two or more launches back only when this
  // plan's most recent launch appended the newest slot of every sequence
  // (into these very pools).
  a.prefetch_old_rows = (p->appended_pool == k_pool) ? 1 : 0;
  p->appended_pool = nullptr;
  return launch_decode(k, a, st);
}
}  // namespace
}  // namespace molot

extern "C" {

int molot_paged_decode(molot_paged_plan* p, const float* Q, float* O, const float* k_pool,
                       const float* v_pool, const int* block_table, int max_pages,
                       int page_size, float scale, void* stream) {
  return paged_decode_impl(p, Q, O, k_pool, v_pool, block_table, max_pages, page_size, scale,
                           (cudaStream_t)stream, nullptr, 0);
}

int molot_paged_decode_gather(molot_paged_plan* p, molot_comm* c, const float* Q,
                              size_t out_offset, const float* k_pool, const float* v_pool,
                              const int* block_table, int max_pages, int page_size, float scale,
                              void* stream) {
  if (!c) return fail(MOLOT_ERR_INVALID, "null comm");
  return paged_decode_impl(p, Q, nullptr, k_pool, v_pool, block_table, max_pages, page_size,
                           scale, (cudaStream_t)stream, c, out_offset);
}

int molot_paged_append(molot_paged_plan* p, const float* q, const float* k, const float* v,
                       float* q_out, const float* q_norm, const float* k_norm, int v_norm,
                       float eps, const float* freq, float* k_pool, float* v_pool,
                       const int* block_table, int max_pages, int page_size, void* stream) {
  if (!p || !p->built) return fail(MOLOT_ERR_INVALID, "plan not built");
  if (!q || !k || !v || !q_out || !k_pool || !v_pool || !block_table)
    return fail(MOLOT_ERR_INVALID, "null pointer");
  if (page_size <= 0 || page_size % kBlk) return fail(MOLOT_ERR_INVALID, "page_size must be a multiple of 16");
  for (int b = 0; b < p->B; ++b)
    if (p->h_n[b] <= 0) return fail(MOLOT_ERR_INVALID, "append needs seq_lens >= 1");
  AppendArgs a = {};
  a.q_in = q;
  a.q_bstride = (long long)p->nq * p->d;
  a.k_in = k;
  a.v_in = v;
  a.kv_in_bstride = (long long)p->nkv * p->d;
  a.q_out = q_out;
  a.qo_bstride = (long long)p->nq * p->d;
  a.q_norm = q_norm;
  a.k_norm = k_norm;
  a.v_norm = v_norm;
  a.eps = eps;
  a.freq = freq;
  a.nq = p->nq;
  a.nkv = p->nkv;
  a.seq_pos = p->ws.plan + p->o_pos;
  a.seq_slot = p->ws.plan + p->o_slot;
  a.K = k_pool;
  a.V = v_pool;
  a.block_table = block_table;
  a.bt_stride = max_pages;
  a.page_size = page_size;
  a.page_stride = (long long)p->nkv * page_size * p->rs();
  a.page_hstride = (long long)page_size * p->rs();
  int rc = append_launch(a, p->d, p->B, (cudaStream_t)stream, p->kvt);
  p->appended_pool = rc == MOLOT_OK ? k_pool : nullptr;
  return rc;
}

int molot_paged_check(molot_paged_plan* p, void* stream) {
  if (!p) return fail(MOLOT_ERR_INVALID, "null plan");
  MOLOT_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
  MOLOT_CUDA(cudaGetLastError());
  return p->ws.check((cudaStream_t)stream, true);
}

}  // extern "C"
