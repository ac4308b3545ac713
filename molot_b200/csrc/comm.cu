// molot_comm_*: the peer-gather group behind molot_paged_decode_gather (see
// comm.cuh for the buffer layout and the epoch protocol).
//
// The reference runs on one CPU and has no multi-device path; the call site
// this serves is forward.h:589-600 (attention of every head, then the output
// projection over all heads), with the kv heads split over the GPUs.
#include <cuda_runtime.h>

#include <cstring>
#include <string>

#include "comm.cuh"
#include "molot_b200.h"
#include "ptx.cuh"

namespace molot {

int set_last_error(int code, const char* msg);

namespace {

int cuda_err(cudaError_t e, const char* what) {
  return set_last_error(e == cudaErrorMemoryAllocation ? MOLOT_ERR_NOMEM : MOLOT_ERR_CUDA,
                        (std::string(what) + ": " + cudaGetErrorString(e)).c_str());
}

#define COMM_CUDA(call)                                \
  do {                                                 \
    cudaError_t e_ = (call);                           \
    if (e_ != cudaSuccess) return cuda_err(e_, #call); \
  } while (0)

struct CommWaitArgs {
  const CommCtl* ctl;  // this rank's control block (flags written by the peers)
  unsigned long long* wait_epoch;
  int* status;
  int nranks;
  unsigned long long limit_ns;
};

// One warp: lane p waits for rank p's flag to reach this wait's epoch.  A
// wait that gives up records kDevErrPeerTimeout and still counts the epoch,
// so the decode / wait pairs of later steps stay matched.
__global__ void comm_wait_kernel(const __grid_constant__ CommWaitArgs a) {
  const int p = threadIdx.x;
  const unsigned long long target = *a.wait_epoch + 1;
  bool ok = true;
  if (p < a.nranks) {
    const unsigned long long* f = &a.ctl->flags[p];
    if (ptx::ld_acquire_sys(f) < target) {
      const unsigned long long t0 = ptx::globaltimer_ns();
      while (ptx::ld_acquire_sys(f) < target) {
        if (ptx::globaltimer_ns() - t0 > a.limit_ns) {
          ok = false;
          break;
        }
        __nanosleep(64);
      }
    }
  }
  if (!ok) atomicCAS(a.status, 0, kDevErrPeerTimeout);
  __syncwarp();
  if (p == 0) *a.wait_epoch = target;
}

}  // namespace
}  // namespace molot

using namespace molot;

extern "C" {

int molot_comm_create(int nranks, int rank, size_t buf_bytes, molot_comm** out) {
  if (!out) return set_last_error(MOLOT_ERR_INVALID, "null out");
  *out = nullptr;
  if (nranks < 1 || nranks > kMaxPeers || rank < 0 || rank >= nranks)
    return set_last_error(MOLOT_ERR_INVALID, "nranks must be 1..8 and 0 <= rank < nranks");
  if (buf_bytes == 0 || buf_bytes % 16)
    return set_last_error(MOLOT_ERR_INVALID, "buf_bytes must be a positive multiple of 16");
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0)
    return set_last_error(MOLOT_ERR_NO_DEVICE, "no CUDA device visible");
  auto* c = new molot_comm();
  if (cudaGetDevice(&c->device) != cudaSuccess) {
    delete c;
    return set_last_error(MOLOT_ERR_CUDA, "cudaGetDevice");
  }
  c->nranks = nranks;
  c->rank = rank;
  c->data_bytes = buf_bytes;
  c->data_round = (buf_bytes + 255) & ~size_t(255);
  cudaError_t e = cudaMalloc(&c->base, c->data_round + kCommCtlBytes);
  if (e == cudaSuccess) e = cudaMemset(c->base, 0, c->data_round + kCommCtlBytes);
  if (e != cudaSuccess) {
    cudaFree(c->base);
    delete c;
    return cuda_err(e, "cudaMalloc(comm buffer)");
  }
  c->peer_base[rank] = c->base;
  c->opened = nranks == 1;
  *out = c;
  return MOLOT_OK;
}

int molot_comm_handle(const molot_comm* c, void* handle) {
  if (!c || !handle) return set_last_error(MOLOT_ERR_INVALID, "null argument");
  static_assert(sizeof(cudaIpcMemHandle_t) == MOLOT_COMM_HANDLE_BYTES, "IPC handle size");
  cudaIpcMemHandle_t h;
  COMM_CUDA(cudaIpcGetMemHandle(&h, c->base));
  std::memcpy(handle, &h, sizeof(h));
  return MOLOT_OK;
}

int molot_comm_open(molot_comm* c, const void* handles) {
  if (!c || !handles) return set_last_error(MOLOT_ERR_INVALID, "null argument");
  if (c->opened) return MOLOT_OK;
  int dev = -1;
  COMM_CUDA(cudaGetDevice(&dev));
  if (dev != c->device) return set_last_error(MOLOT_ERR_INVALID, "comm used on another device");
  const unsigned char* hs = static_cast<const unsigned char*>(handles);
  for (int r = 0; r < c->nranks; ++r) {
    if (r == c->rank) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, hs + (size_t)r * MOLOT_COMM_HANDLE_BYTES, sizeof(h));
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int q = 0; q < r; ++q)
        if (q != c->rank && c->peer_base[q]) {
          cudaIpcCloseMemHandle(c->peer_base[q]);
          c->peer_base[q] = nullptr;
        }
      return cuda_err(e, ("cudaIpcOpenMemHandle(rank " + std::to_string(r) + ")").c_str());
    }
    c->peer_base[r] = static_cast<unsigned char*>(p);
  }
  c->opened = true;
  return MOLOT_OK;
}

int molot_comm_buffer(const molot_comm* c, float** buf) {
  if (!c || !buf) return set_last_error(MOLOT_ERR_INVALID, "null argument");
  *buf = reinterpret_cast<float*>(c->base);
  return MOLOT_OK;
}

int molot_comm_wait(molot_comm* c, void* stream) {
  if (!c) return set_last_error(MOLOT_ERR_INVALID, "null comm");
  if (!c->opened) return set_last_error(MOLOT_ERR_INVALID, "comm not opened");
  CommWaitArgs a;
  a.ctl = c->own_ctl();
  a.wait_epoch = &c->own_ctl()->wait_epoch;
  a.status = &c->own_ctl()->status;
  a.nranks = c->nranks;
  a.limit_ns = kCommWaitLimitNs;
  // A plain launch (no programmatic serialisation): it starts only once
  // this rank's preceding work on the stream has completed.
  comm_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(a);
  COMM_CUDA(cudaGetLastError());
  return MOLOT_OK;
}

int molot_comm_check(molot_comm* c, void* stream) {
  if (!c) return set_last_error(MOLOT_ERR_INVALID, "null comm");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  COMM_CUDA(cudaStreamSynchronize(st));
  int h = 0;
  COMM_CUDA(cudaMemcpyAsync(&h, &c->own_ctl()->status, sizeof(int), cudaMemcpyDeviceToHost, st));
  COMM_CUDA(cudaStreamSynchronize(st));
  if (h != 0) {
    COMM_CUDA(cudaMemsetAsync(&c->own_ctl()->status, 0, sizeof(int), st));
    COMM_CUDA(cudaStreamSynchronize(st));
    return set_last_error(MOLOT_ERR_TIMEOUT, "wait for a peer rank's outputs timed out");
  }
  return MOLOT_OK;
}

void molot_comm_destroy(molot_comm* c) {
  if (!c) return;
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(c->device);
  cudaDeviceSynchronize();
  for (int r = 0; r < c->nranks; ++r)
    if (r != c->rank && c->peer_base[r]) cudaIpcCloseMemHandle(c->peer_base[r]);
  cudaFree(c->base);
  if (prev >= 0) cudaSetDevice(prev);
  delete c;
}

}  // extern "C"
