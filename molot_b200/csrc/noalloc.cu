// molot_attn_decode_strided_noalloc: the strided single-sequence decode for
// callers that cannot allocate device memory.
//
// Some embedders run inside a host runtime that owns every device
// allocation (a custom caching allocator, a memory pool sized at start-up,
// or a region where cudaMalloc would synchronise the device and stall other
// streams), so a library call that allocates its own scratch on first use
// is not acceptable to them.  This entry point allocates nothing: the split-KV
// partial records, the per-head tickets and the status word live in one
// file-scope __device__ array of fixed size (kNoAllocScratchBytes, about
// 1.4 MB).  Every GPU on which the library's code is loaded holds that
// array until the process exits.
//
// Limits: head_dim in {64, 128, 256}, group size nq/nkv in {1, 2, 4, 8} with
// group * head_dim <= 1024, nkv <= 256, and at most kNoAllocMaxGrid CTAs.
// Larger requests are rejected with MOLOT_ERR_UNSUPPORTED.
//
// All calls share the one array, and it keeps what the last call left in it:
// each call clears the tickets (cudaMemsetAsync on the array, which
// allocates nothing) before its launch; the partial records are always
// written before they are read.  The status word is not cleared by a call:
// a call that gave up on a bounded wait leaves MOLOT_ERR_TIMEOUT there until
// molot_noalloc_status (or molot_device_status) reads and clears it.  Calls
// whose work overlaps on the GPU -- different streams, or different host
// threads without ordering -- race on the array; order them on one stream.
//
// The partition of the work and the kernel variant are those of
// molot_attn_decode_strided_dev, so both give bit-identical outputs.
//
// Set-up: on the first call on a device, with that device current, the
// array's device address is fetched once with cudaGetSymbolAddress (the
// array's name is only a host-side stand-in in host code) and cached; make
// that first call before any stream capture.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "decode.cuh"
#include "dispatch.cuh"
#include "molot_b200.h"

namespace molot {

int set_last_error(int code, const char* msg);
void take_withhold(DecodeArgs& a);

namespace {

constexpr int kNoAllocMaxGrid = 160;                      // >= 148 SMs of a B200
constexpr int kNoAllocMaxGroupDim = 1024;                 // G * head_dim
constexpr int kNoAllocMaxRecord = kNoAllocMaxGroupDim + 64;  // floats, >= partial_record_floats
constexpr int kNoAllocMaxSegments = 256;                  // nkv
constexpr size_t kNoAllocPartialBytes = 2ull * kNoAllocMaxGrid * kNoAllocMaxRecord * 4;
constexpr size_t kNoAllocCounterBytes = kNoAllocMaxSegments * 4;
constexpr size_t kNoAllocStatusBytes = 256;
constexpr size_t kNoAllocScratchBytes =
    kNoAllocPartialBytes + kNoAllocCounterBytes + kNoAllocStatusBytes;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of the scratch array on the current device (set-up once).
int scratch_for(int dev, unsigned char** out) {
  if (dev < 0 || dev >= kMaxDevices)
    return set_last_error(MOLOT_ERR_UNSUPPORTED, "device index beyond the no-alloc table");
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return set_last_error(MOLOT_ERR_CUDA, (std::string("cudaGetSymbolAddress(no-alloc scratch): ") +
                                             cudaGetErrorString(e)).c_str());
    g_scratch_addr[dev] = p;
  }
  *out = static_cast<unsigned char*>(g_scratch_addr[dev]);
  return MOLOT_OK;
}

// The FP32 decode kernels of molot_attn_decode_strided_dev, within the
// no-alloc limits (group <= 8).  split: the split K/V stage-barrier form.
bool pick(int d, int g, bool split, KernelRef* k) {
  return g <= 8 && pick_decode_f32(d, g, split, k);
}

int cuda_err(cudaError_t e, const char* what) {
  return set_last_error(MOLOT_ERR_CUDA, (std::string(what) + ": " + cudaGetErrorString(e)).c_str());
}

int* status_word(unsigned char* scratch) {
  return reinterpret_cast<int*>(scratch + kNoAllocPartialBytes + kNoAllocCounterBytes);
}

// Reads the status word on `st` into the host (no allocation: a pageable
// destination goes through the driver's own staging), clears it on request.
int read_status(unsigned char* scratch, cudaStream_t st, bool clear) {
  int h = 0;
  cudaError_t e = cudaMemcpyAsync(&h, status_word(scratch), sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_err(e, "reading the no-alloc status word");
  if (h == 0) return MOLOT_OK;
  if (clear) {
    e = cudaMemsetAsync(status_word(scratch), 0, sizeof(int), st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_err(e, "clearing the no-alloc status word");
  }
  return set_last_error(MOLOT_ERR_TIMEOUT, h == kDevErrConsumerTimeout
                                               ? "no-alloc decode: wait for a KV tile timed out"
                                               : "no-alloc decode: wait for a free stage timed out");
}

}  // namespace

int noalloc_status_check(int dev, cudaStream_t st, bool clear) {
  unsigned char* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (dev < 0 || dev >= kMaxDevices || !g_scratch_addr[dev]) return MOLOT_OK;
    scratch = static_cast<unsigned char*>(g_scratch_addr[dev]);
  }
  return read_status(scratch, st, clear);
}

}  // namespace molot

using namespace molot;

extern "C" int molot_attn_decode_strided_noalloc(const float* Q, const float* K, const float* V,
                                                 float* O, int nq, int nkv, int n, int d,
                                                 long long stride_t, long long stride_h,
                                                 float scale, int pos_cur, int window,
                                                 void* stream) {
  if (!Q || !K || !V || !O) return set_last_error(MOLOT_ERR_INVALID, "null pointer");
  if (nq <= 0 || nkv <= 0 || d <= 0 || n < 0 || nq % nkv)
    return set_last_error(MOLOT_ERR_INVALID, "bad sizes (nq must be a positive multiple of nkv)");
  const int G = nq / nkv;
  KernelRef k;
  if (nkv > kNoAllocMaxSegments || G * d > kNoAllocMaxGroupDim || !pick(d, G, false, &k))
    return set_last_error(MOLOT_ERR_UNSUPPORTED,
                          "no-alloc decode supports head_dim 64/128/256, group 1/2/4/8 with "
                          "group*head_dim <= 1024 and nkv <= 256");
  if ((reinterpret_cast<uintptr_t>(K) & 15) || (reinterpret_cast<uintptr_t>(V) & 15) ||
      (stride_t & 3) || (stride_h & 3))
    return set_last_error(MOLOT_ERR_INVALID,
                          "K/V must be 16-byte aligned with strides multiple of 4 floats");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_err(e, "cudaGetDevice");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int t0 = (window > 0 && pos_cur - window + 1 > 0) ? pos_cur - window + 1 : 0;
  if (n <= t0) {  // empty attended range: zeros, as the reference (attn.h:163)
    e = cudaMemsetAsync(O, 0, sizeof(float) * (size_t)nq * d, st);
    return e == cudaSuccess ? MOLOT_OK : cuda_err(e, "cudaMemsetAsync(O)");
  }
  unsigned char* scratch = nullptr;
  int rc = scratch_for(dev, &scratch);
  if (rc) return rc;
  int sms = 0;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return cuda_err(e, "cudaDeviceGetAttribute");
  const int blo = t0 / kBlk;
  const int nblk = (n + kBlk - 1) / kBlk - blo;
  const long long NB = (long long)nkv * nblk;
  if (partial_record_floats(G, d) > kNoAllocMaxRecord)
    return set_last_error(MOLOT_ERR_UNSUPPORTED, "partial record exceeds the no-alloc scratch");
  e = cudaFuncSetAttribute(k.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, k.smem);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(k.fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e != cudaSuccess) return cuda_err(e, "cudaFuncSetAttribute");
  // The partition of molot_attn_decode_strided_dev (at most kNoAllocMaxGrid
  // CTAs, which covers one per SM of a B200).
  UniformPlan up = plan_uniform(NB, nkv, nblk, sms < kNoAllocMaxGrid ? sms : kNoAllocMaxGrid,
                                max_active_clusters(k, kClusterCtas, dev),
                                max_active_clusters(k, kClusterCtasWide, dev));
  balance_uniform_grid(up, nkv, nblk);
  const int grid = up.grid;

  float* partials = reinterpret_cast<float*>(scratch);
  int* counters = reinterpret_cast<int*>(scratch + kNoAllocPartialBytes);
  int* status = status_word(scratch);
  // Tickets must start at zero; a previous call may have left them
  // otherwise if it gave up on a wait.  The status word is left for
  // molot_noalloc_status to report.
  e = cudaMemsetAsync(counters, 0, kNoAllocCounterBytes, st);
  if (e != cudaSuccess) return cuda_err(e, "cudaMemsetAsync(no-alloc tickets)");
  // The kernel variant of molot_attn_decode_strided_dev: split K/V stage
  // barriers for long FP32 launches at head_dim <= 128.
  const int aligned = up.aligned;
  {
    const int tile_rows = d <= 64 ? TileShape<64, float>::T : TileShape<128, float>::T;
    const long long rows_per_cta = (long long)nblk * kBlk * nkv / grid;
    KernelRef ks;
    if (d <= 128 && aligned && rows_per_cta >= 8LL * tile_rows && pick(d, G, true, &ks)) k = ks;
  }
  e = cudaFuncSetAttribute(k.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, k.smem);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(k.fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e != cudaSuccess) return cuda_err(e, "cudaFuncSetAttribute");

  DecodeArgs a = {};
  a.Q = Q;
  a.q_bstride = (long long)nq * d;
  a.O = O;
  a.o_bstride = (long long)nq * d;
  a.K = K;
  a.V = V;
  a.stride_t = stride_t;
  a.stride_h = stride_h;
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
  a.partials = partials;
  a.counters = counters;
  a.status = status;
  a.timeout_ns = 2000000000ull;
  a.grid = grid;
  a.aligned = aligned;
  a.cluster = up.cluster;
  a.cl_per_seg = up.cl_per_seg;
  a.prefetch_old_rows = 0;  // the caller's K/V may come from the preceding launch
  take_withhold(a);
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = up.cluster;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kDecodeThreads);
  cfg.dynamicSmemBytes = k.smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = up.cluster > 1 ? 2 : 1;
  void* args[] = {&a};
  e = cudaLaunchKernelExC(&cfg, k.fn, args);
  return e == cudaSuccess ? MOLOT_OK : cuda_err(e, "launch (no-alloc decode)");
}

extern "C" int molot_noalloc_status(void* stream, int clear) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_err(e, "cudaGetDevice");
  return noalloc_status_check(dev, static_cast<cudaStream_t>(stream), clear != 0);
}
