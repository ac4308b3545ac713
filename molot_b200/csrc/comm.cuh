// Peer-gather group (molot_comm_*): one process per GPU, each holding a
// gathered-output buffer that every rank of the group writes into directly
// over NVLink / NVSwitch (CUDA IPC mappings of the peers' buffers).
//
// Buffer of one rank (one cudaMalloc, mapped by every peer):
//   [0, data_round)            the gathered outputs (caller-sized)
//   [data_round, +kCommCtl)    CommCtl: one epoch flag per rank (written by
//                              that rank), then words only this rank uses.
// A paged decode launched with the group writes its final outputs into every
// rank's buffer and, from its last CTA, raises its own flag in every rank's
// buffer to its launch count (epoch).  molot_comm_wait is a one-warp kernel
// that waits, with a bounded spin, until every rank's flag in this rank's
// buffer has reached this rank's wait count.  Flags only grow, so nothing is
// ever reset between launches.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>

#include "decode.cuh"

namespace molot {

struct CommCtl {
  unsigned long long flags[kMaxPeers];  // flags[p]: rank p's decodes that have landed here
  unsigned long long epoch;             // this rank's gather launches so far
  unsigned long long wait_epoch;        // this rank's completed waits so far
  unsigned int done;                    // CTAs finished in the running launch
  int status;                           // kDevErrPeerTimeout after a wait that gave up
};
constexpr size_t kCommCtlBytes = 256;
static_assert(sizeof(CommCtl) <= kCommCtlBytes, "comm control block too large");

// Bound of one molot_comm_wait: the ranks of a step run in lockstep, so a
// wait that lasts seconds means a rank has stopped.
constexpr unsigned long long kCommWaitLimitNs = 5000000000ull;

}  // namespace molot

struct molot_comm {
  int device = -1;
  int nranks = 0, rank = 0;
  size_t data_bytes = 0;   // usable bytes of the gathered buffer
  size_t data_round = 0;   // data_bytes rounded up to 256
  unsigned char* base = nullptr;                  // this rank's buffer
  unsigned char* peer_base[molot::kMaxPeers] = {};  // every rank's buffer as mapped here
  bool opened = false;
  molot::CommCtl* ctl(int r) const {
    return reinterpret_cast<molot::CommCtl*>(peer_base[r] + data_round);
  }
  molot::CommCtl* own_ctl() const { return reinterpret_cast<molot::CommCtl*>(base + data_round); }
};
