// Tensor-parallel plumbing: one NCCL communicator per session.  Megatron column/row splits of the
// Llama projections are joined by one Float32 sum allreduce per row-split projection.  The
// reference has no distributed path (LlamaConfig rejects pretraining_tp != 1,
// models/.../LlamaConfig.scala:91); this is the one exchange step the B200 build adds.
#include <nccl.h>

#include <cstring>

#include "common.cuh"

namespace stb {

void peer_setup(stb_session *s);
void peer_teardown(stb_session *s);

#define STB_NCCL(call)                                                                            \
  do {                                                                                            \
    ncclResult_t r_ = (call);                                                                     \
    if (r_ != ncclSuccess) throw Error(STB_ERR_NCCL, std::string(#call) + " failed: " + ncclGetErrorString(r_)); \
  } while (0)

void allreduce_sum_f32(stb_session *s, void *buf, uint64_t count) {
  if (s->tp_size <= 1 || count == 0) return;
  if (!s->nccl) throw Error(STB_ERR_STATE, "tensor-parallel communicator not initialised");
  STB_NCCL(ncclAllReduce(buf, buf, count, ncclFloat32, ncclSum, (ncclComm_t)s->nccl, s->stream));
}

void allgather_bytes(stb_session *s, const void *send, void *recv, uint64_t bytes) {
  if (s->tp_size <= 1) {
    if (send != recv) STB_CUDA(cudaMemcpyAsync(recv, send, bytes, cudaMemcpyDeviceToDevice, s->stream));
    return;
  }
  if (!s->nccl) throw Error(STB_ERR_STATE, "tensor-parallel communicator not initialised");
  STB_NCCL(ncclAllGather(send, recv, bytes, ncclUint8, (ncclComm_t)s->nccl, s->stream));
}

}  // namespace stb

using namespace stb;

extern "C" {

void stb_session_close_tp(stb_session *s) {
  if (s && s->peer) peer_teardown(s);
  if (s && s->nccl) {
    ncclCommDestroy((ncclComm_t)s->nccl);
    s->nccl = nullptr;
  }
}

int stb_nccl_unique_id(uint8_t id[128]) {
  return guarded([&] {
    STB_REQUIRE(id, "output is null");
    static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id size");
    ncclUniqueId u;
    STB_NCCL(ncclGetUniqueId(&u));
    std::memcpy(id, &u, 128);
  });
}

int stb_session_init_tp(stb_session *s, int nranks, int rank, const uint8_t id[128]) {
  return guarded([&] {
    enter(s);
    STB_REQUIRE(nranks >= 1 && rank >= 0 && rank < nranks, "invalid tensor-parallel rank");
    STB_REQUIRE(!s->nccl, "communicator already initialised");
    s->tp_rank = rank;
    s->tp_size = nranks;
    if (nranks == 1) return;
    STB_REQUIRE(id, "unique id is null");
    ncclUniqueId u;
    std::memcpy(&u, id, 128);
    ncclComm_t comm;
    STB_NCCL(ncclCommInitRank(&comm, nranks, u, rank));
    s->nccl = comm;
    peer_setup(s);  // NVLink receive buffers for the fused row-split projections
  });
}

int stb_allreduce_sum_f32(stb_session *s, uint64_t buf, uint64_t count) {
  return guarded([&] {
    enter(s);
    STB_REQUIRE(count == 0 || buf, "null buffer");
    allreduce_sum_f32(s, (void *)buf, count);
  });
}

}  // extern "C"
