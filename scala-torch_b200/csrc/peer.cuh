// Peer-memory exchange for tensor-parallel decode: the row-split projections (o_proj, down_proj)
// store their partial sums straight into every rank's receive slots over NVLink; a small reduce
// kernel sums the slots in rank order (identical on all ranks) and adds the residual.  This
// replaces one NCCL allreduce per row-split projection for decode-sized row counts.
//
// Flag-in-data: every value travels as one 8-byte word (use number << 32 | float bits).  An 8-byte
// store is single-copy atomic, so the receiver knows a value has arrived when its word carries the
// expected use number -- no fence, counter or atomic is needed on the producer side, and the
// receiver polls its own (local) memory.  Every wait is bounded by the global timer and reports
// through the session's error word.
//
// Buffer of each rank (one cudaMalloc, shared through CUDA IPC):
//   [0, 4096)  control: epoch[2] (u64, uses of each region completed on this rank), done[2] (u32)
//   [4096, ..) data: region r (0 = o_proj, 1 = down_proj), slot s (producing rank):
//              u64[slot_elems] at 4096 + ((r * tp + s) * slot_elems) * 8
// Two regions alternate, so a rank can only rewrite a region after every rank has reduced it
// (it needs every rank's contribution to the other region first).
#pragma once

#include "common.cuh"

namespace stb {

constexpr int kMaxPeers = 8;
constexpr uint64_t kPeerControlBytes = 4096;

struct PeerArgs {
  unsigned long long *slots[kMaxPeers];  // each rank's data area (device address valid here)
  unsigned long long *my_epoch;          // this rank's epoch[2]
  unsigned int *my_done;                 // this rank's done[2]
  const unsigned long long *my_slots;    // this rank's data area
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

__device__ __forceinline__ unsigned long long peer_word(float v, uint32_t use) {
  return ((unsigned long long)use << 32) | (unsigned long long)__float_as_uint(v);
}

__device__ __forceinline__ unsigned long long peer_load(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void peer_store(unsigned long long *p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Wait until the word at p carries `use`; returns its value bits, or sets *ok = false after wait_ns
// (recording `code`) or as soon as another wait has already failed.
__device__ __forceinline__ float peer_take(const unsigned long long *p, uint32_t use, unsigned long long wait_ns,
                                           int *err, int code, bool *ok) {
  unsigned long long w = peer_load(p);
  if ((uint32_t)(w >> 32) == use) return __uint_as_float((uint32_t)w);
  const volatile int *e = err;
  const unsigned long long t0 = peer_now_ns();
  for (uint32_t i = 0;; i++) {
    w = peer_load(p);
    if ((uint32_t)(w >> 32) == use) return __uint_as_float((uint32_t)w);
    if ((i & 31) == 0 && (*e || peer_now_ns() - t0 > wait_ns)) {
      atomicCAS(err, 0, code);
      *ok = false;
      return 0.0f;
    }
    __nanosleep(32);
  }
}

// Spin until *counter >= target (used by the wait probe); same bounds and error reporting.
__device__ __forceinline__ bool peer_wait_geq(const unsigned long long *counter, unsigned long long target,
                                              unsigned long long wait_ns, int *err, int code) {
  const volatile unsigned long long *c = counter;
  const volatile int *e = err;
  if (*c >= target) return true;
  if (*e) return false;
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

}  // namespace stb
