// Tensor-parallel peer-memory exchange: IPC setup over the session's NCCL communicator, the rank-order
// reduce kernel, and a probe of the bounded device wait.  See peer.cuh for the protocol.
#include <nccl.h>

#include <cstdlib>
#include <cstring>
#include <vector>

#include "peer.cuh"

namespace stb {

struct PeerComm {
  uint64_t local = 0, bytes = 0;
  void *remote[kMaxPeers] = {};
  uint64_t base[kMaxPeers] = {};
  uint64_t slot_elems = 0;
  int tp = 1, rank = 0;
  unsigned long long wait_ns = 10000000000ull;
};

#define STB_NCCL_P(call)                                                                           \
  do {                                                                                             \
    ncclResult_t r_ = (call);                                                                      \
    if (r_ != ncclSuccess) throw Error(STB_ERR_NCCL, std::string(#call) + " failed: " + ncclGetErrorString(r_)); \
  } while (0)

// All ranks meet here (a one-element allreduce) and the stream is drained.
static void peer_barrier(stb_session *s) {
  uint64_t one = session_scratch(s, 64);
  STB_NCCL_P(ncclAllReduce((const void *)one, (void *)one, 1, ncclFloat32, ncclSum, (ncclComm_t)s->nccl, s->stream));
  STB_CUDA(cudaStreamSynchronize(s->stream));
}

void peer_setup(stb_session *s) {
  if (s->tp_size <= 1 || s->tp_size > kMaxPeers) return;
  const char *off = std::getenv("STB_TP_PEER");
  if (off && std::atoi(off) == 0) return;
  auto *pc = new PeerComm();
  try {
    const char *mb = std::getenv("STB_PEER_BUFFER_MB");
    pc->bytes = (uint64_t)(mb && *mb ? std::atoi(mb) : 64) << 20;
    const char *ms = std::getenv("STB_PEER_WAIT_MS");
    if (ms && *ms) pc->wait_ns = (unsigned long long)std::atoll(ms) * 1000000ull;
    pc->tp = s->tp_size;
    pc->rank = s->tp_rank;
    pc->local = session_alloc(s, pc->bytes);
    STB_CUDA(cudaMemsetAsync((void *)pc->local, 0, pc->bytes, s->stream));
    cudaIpcMemHandle_t mine;
    STB_CUDA(cudaIpcGetMemHandle(&mine, (void *)pc->local));
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    uint64_t dev = session_scratch(s, 64 * (kMaxPeers + 1));
    STB_CUDA(cudaMemcpyAsync((void *)dev, &mine, 64, cudaMemcpyHostToDevice, s->stream));
    STB_NCCL_P(ncclAllGather((const void *)dev, (void *)(dev + 64), 64, ncclUint8, (ncclComm_t)s->nccl, s->stream));
    std::vector<cudaIpcMemHandle_t> all(pc->tp);
    STB_CUDA(cudaMemcpyAsync(all.data(), (const void *)(dev + 64), 64 * pc->tp, cudaMemcpyDeviceToHost, s->stream));
    STB_CUDA(cudaStreamSynchronize(s->stream));
    for (int r = 0; r < pc->tp; r++) {
      if (r == pc->rank) {
        pc->base[r] = pc->local;
        continue;
      }
      STB_CUDA(cudaIpcOpenMemHandle(&pc->remote[r], all[r], cudaIpcMemLazyEnablePeerAccess));
      pc->base[r] = (uint64_t)pc->remote[r];
    }
    pc->slot_elems = ((pc->bytes - kPeerControlBytes) / (2ull * pc->tp * 8)) & ~3ull;
    s->peer = pc;
    peer_barrier(s);  // every rank has mapped every buffer before first use
  } catch (...) {
    for (int r = 0; r < kMaxPeers; r++)
      if (pc->remote[r]) cudaIpcCloseMemHandle(pc->remote[r]);
    if (pc->local) session_free(s, pc->local);
    s->peer = nullptr;
    delete pc;
    throw;
  }
}

void peer_teardown(stb_session *s) {
  // No collective here (a rank that failed must not hang the others at close).  Unmapping is safe
  // after completed steps: a peer's last stores into this buffer happen before this rank's last
  // reduce observed their signals.
  auto *pc = (PeerComm *)s->peer;
  if (!pc) return;
  cudaStreamSynchronize(s->stream);
  for (int r = 0; r < kMaxPeers; r++)
    if (pc->remote[r]) cudaIpcCloseMemHandle(pc->remote[r]);
  try {
    session_free(s, pc->local);
  } catch (...) {
  }
  s->peer = nullptr;
  delete pc;
}

// Zero every rank's counters and epochs (collective): a clean state for a new generation.
void peer_reset(stb_session *s) {
  auto *pc = (PeerComm *)s->peer;
  if (!pc) return;
  peer_barrier(s);
  // epochs restart at 0, so every slot word must lose its old use number too
  STB_CUDA(cudaMemsetAsync((void *)pc->local, 0, pc->bytes, s->stream));
  peer_barrier(s);
}

bool peer_usable(stb_session *s, uint64_t elems) {
  auto *pc = (PeerComm *)s->peer;
  return pc && elems <= pc->slot_elems;
}

PeerArgs peer_args(stb_session *s, int region) {
  auto *pc = (PeerComm *)s->peer;
  PeerArgs a{};
  for (int r = 0; r < pc->tp; r++) a.slots[r] = (unsigned long long *)(pc->base[r] + kPeerControlBytes);
  a.my_epoch = (unsigned long long *)pc->local;
  a.my_done = (unsigned int *)(pc->local + 64);
  a.my_slots = (const unsigned long long *)(pc->local + kPeerControlBytes);
  a.slot_elems = pc->slot_elems;
  a.tp = pc->tp;
  a.rank = pc->rank;
  a.region = region;
  a.wait_ns = pc->wait_ns;
  a.err = session_error_word(s);
  return a;
}

// out[i] = residual[i] + (((slot_0[i] + slot_1[i]) + slot_2[i]) + ...), each slot word taken once it
// carries this use of the region; the last block to finish advances the region's epoch.
__global__ void peer_reduce_kernel(PeerArgs pa, long total, const float *residual, float *out) {
  pdl_wait();
  pdl_trigger();
  const uint32_t use = (uint32_t)(pa.my_epoch[pa.region] + 1ull);
  const unsigned long long *base = pa.my_slots + (size_t)pa.region * pa.tp * pa.slot_elems;
  bool ok = true;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total && ok; i += (long)gridDim.x * blockDim.x) {
    float acc = peer_take(base + i, use, pa.wait_ns, pa.err, 16 + pa.region, &ok);
    for (int r = 1; r < pa.tp; r++)
      acc += peer_take(base + (size_t)r * pa.slot_elems + i, use, pa.wait_ns, pa.err, 16 + pa.region, &ok);
    if (ok) out[i] = residual[i] + acc;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(pa.my_done + pa.region, 1u);
    if (prev == gridDim.x - 1) {
      pa.my_done[pa.region] = 0u;
      pa.my_epoch[pa.region] += 1ull;
      __threadfence();
    }
  }
}

void peer_reduce_launch(stb_session *s, int region, long total, const float *residual, float *out) {
  PeerArgs pa = peer_args(s, region);
  long blocks = (total + 255) / 256;
  if (blocks > 148) blocks = 148;
  launch_kernel(peer_reduce_kernel, dim3((unsigned)blocks), dim3(256), 0, s->stream, true, pa, total, residual, out);
}

__global__ void wait_probe_kernel(const unsigned long long *counter, unsigned long long wait_ns, int *err) {
  if (threadIdx.x == 0) peer_wait_geq(counter, 1ull, wait_ns, err, 99);
}

}  // namespace stb

using namespace stb;

extern "C" {

int stb_check_bounded_wait(stb_session *s, uint64_t wait_ns, int *code) {
  return guarded([&] {
    enter(s);
    STB_REQUIRE(code && wait_ns > 0 && wait_ns <= 5000000000ull, "wait must be in (0, 5 s]");
    int *err = session_error_word(s);
    const uint64_t counter = session_scratch(s, 64);
    STB_CUDA(cudaMemsetAsync((void *)counter, 0, 8, s->stream));
    wait_probe_kernel<<<1, 32, 0, s->stream>>>((const unsigned long long *)counter, wait_ns, err);
    check_launch("wait_probe");
    count_launch(s);
    STB_CUDA(cudaStreamSynchronize(s->stream));
    STB_CUDA(cudaMemcpy(code, err, sizeof(int), cudaMemcpyDeviceToHost));
    STB_CUDA(cudaMemset(err, 0, sizeof(int)));
  });
}

int stb_session_tp_peer(stb_session *s, int *enabled, uint64_t *slot_elems) {
  return guarded([&] {
    enter(s);
    auto *pc = (PeerComm *)s->peer;
    if (enabled) *enabled = pc != nullptr;
    if (slot_elems) *slot_elems = pc ? pc->slot_elems : 0;
  });
}

}  // extern "C"
