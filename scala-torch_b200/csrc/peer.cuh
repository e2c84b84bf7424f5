// Peer-memory exchange for tensor-parallel decode: the row-split projections (o_proj, down_proj)
// write their partial sums straight into every rank's receive slots over NVLink and signal with
// system-scope atomics; a small reduce kernel sums the slots in rank order (identical on all ranks)
// and adds the residual.  This replaces one NCCL allreduce per row-split projection for decode-sized
// row counts.  Every wait is bounded by the global timer and reports through an error word.
//
// Buffer of each rank (one cudaMalloc, shared through CUDA IPC):
//   [0, 4096)  control: counter[2] (u64, incremented by every producing block of every rank),
//              epoch[2] (u64, uses consumed so far), done[2] (u32, reduce blocks finished)
//   [4096, ..) data: region r (0 = o_proj, 1 = down_proj), slot s (producing rank):
//              float[slot_elems] at 4096 + ((r * tp + s) * slot_elems) * 4
// Two regions alternate, so a rank can only rewrite a region after every rank has reduced it
// (it needs every rank's contribution to the other region first).
#pragma once

#include "common.cuh"

namespace stb {

constexpr int kMaxPeers = 8;
constexpr uint64_t kPeerControlBytes = 4096;

struct PeerArgs {
  float *slots[kMaxPeers];                     // each rank's data area (device address valid here)
  unsigned long long *counters[kMaxPeers];     // each rank's counter[2]
  unsigned long long *my_counter, *my_epoch;   // this rank's counter[2], epoch[2]
  unsigned int *my_done;                       // this rank's done[2]
  const float *my_slots;                       // this rank's data area
  uint64_t slot_elems;
  int tp, rank, region;
  unsigned long long wait_ns;
  int *err;
};

__device__ __forceinline__ unsigned long long peer_now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Spin until *counter >= target or wait_ns elapses (then record `code` in *err).  Returns success.
__device__ __forceinline__ bool peer_wait_geq(const unsigned long long *counter, unsigned long long target,
                                              unsigned long long wait_ns, int *err, int code) {
  const volatile unsigned long long *c = counter;
  const volatile int *e = err;
  if (*c >= target) return true;
  if (*e) return false;  // an earlier wait already failed: give up at once instead of waiting again
  const unsigned long long t0 = peer_now_ns();
  for (uint32_t i = 0;; i++) {
    if (*c >= target) return true;
    if ((i & 63) == 0 && (*e || peer_now_ns() - t0 > wait_ns)) {
      atomicCAS(err, 0, code);
      return false;
    }
    __nanosleep(64);
  }
}

// Producer side, called by one thread per block after the block's partial sums are stored to
// every rank: publish them (system fence) and count this block on every rank.
__device__ __forceinline__ void peer_signal(const PeerArgs &pa) {
  __threadfence_system();
  for (int r = 0; r < pa.tp; r++) atomicAdd_system(pa.counters[r] + pa.region, 1ull);
}

}  // namespace stb
