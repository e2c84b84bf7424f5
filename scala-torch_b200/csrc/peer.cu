// Tensor-parallel peer-memory exchange: IPC setup over the session's NCCL communicator, the rank-order
// reduce kernel, and a probe of the bounded device wait.  See peer.cuh for the protocol.
#include <nccl.h>

#include <cstdlib>
#include <cstring>
#include <vector>

#include "gemv.cuh"
#include "peer.cuh"
#include "tc_common.cuh"

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

// peer_reduce_kernel and the next projection's RMSNorm prologue in one (decode chunks of up to 64 rows
// on the skinny form): a cluster of 8 CTAs per token row, one float4 of the row per thread.  Every slot
// word of the thread is loaded at once (one round trip when the peers' stores have landed; words of an
// older use are then waited for one by one, bounded), the slots are added in rank order and the
// residual after them as peer_reduce_kernel does; the CTAs' double sums of squares are added in rank
// order through distributed shared memory, and each thread writes the three BF16 terms of its
// normalised values (the GEMV's expression) into x3n [3][NT][H].  Rows >= rows get zero terms.  The
// last block to finish advances the region's epoch.
constexpr int PR_CTAS = 8, PR_THREADS = 256;

__device__ __forceinline__ double pr_ld_cluster_f64(uint32_t cluster_addr) {
  double v;
  asm volatile("ld.shared::cluster.f64 %0, [%1];" : "=d"(v) : "r"(cluster_addr) : "memory");
  return v;
}

__global__ void __cluster_dims__(PR_CTAS, 1, 1) __launch_bounds__(PR_THREADS) peer_reduce_norm_kernel(
    PeerArgs pa, int rows, int H, const float *residual, float *out, const float *norm_w, double eps, uint16_t *x3n,
    int NT) {
  __shared__ double s_scratch[PR_THREADS / 32];
  __shared__ double s_cta, s_total;
  pdl_wait();
  const uint32_t use = (uint32_t)(pa.my_epoch[pa.region] + 1ull);
  const unsigned long long *base = pa.my_slots + (size_t)pa.region * pa.tp * pa.slot_elems;
  const int m = blockIdx.y, n4 = H / 4;
  const int c = blockIdx.x * PR_THREADS + threadIdx.x;  // float4 of the row
  const bool live = m < rows && c < n4;
  float4 v = make_float4(0.f, 0.f, 0.f, 0.f), nw = v;
  double sq = 0.0;
  bool ok = true;
  if (live) {
    const size_t i0 = (size_t)m * H + 4 * c;
    unsigned long long w[kMaxPeers][4];
#pragma unroll
    for (int r = 0; r < kMaxPeers; r++)
      if (r < pa.tp)
#pragma unroll
        for (int e = 0; e < 4; e++) w[r][e] = peer_load(base + (size_t)r * pa.slot_elems + i0 + e);
    v = *(const float4 *)(residual + i0);
    nw = *(const float4 *)(norm_w + 4 * c);
    float a[4];
    bool ready = true;
#pragma unroll
    for (int e = 0; e < 4; e++) {
      float acc = 0.0f;
#pragma unroll
      for (int r = 0; r < kMaxPeers; r++) {
        if (r < pa.tp) {
          ready = ready && (uint32_t)(w[r][e] >> 32) == use;
          const float x = __uint_as_float((uint32_t)w[r][e]);
          acc = r == 0 ? x : acc + x;
        }
      }
      a[e] = acc;
    }
    if (!ready) {  // some peer's words of this use had not landed: wait for each (bounded), same order
      for (int e = 0; e < 4; e++) {
        float acc = 0.0f;
        for (int r = 0; r < pa.tp; r++) {
          const float x = peer_take(base + (size_t)r * pa.slot_elems + i0 + e, use, pa.wait_ns, pa.err,
                                    16 + pa.region, &ok);
          acc = r == 0 ? x : acc + x;
        }
        a[e] = acc;
      }
    }
    v = make_float4(v.x + a[0], v.y + a[1], v.z + a[2], v.w + a[3]);
    *(float4 *)(out + i0) = v;
    const double d0 = v.x, d1 = v.y, d2 = v.z, d3 = v.w;
    sq = __dadd_rn(sq, __dmul_rn(d0, d0));
    sq = __dadd_rn(sq, __dmul_rn(d1, d1));
    sq = __dadd_rn(sq, __dmul_rn(d2, d2));
    sq = __dadd_rn(sq, __dmul_rn(d3, d3));
  }
  pdl_trigger();  // after this thread's loads: the next GEMM's weight stream would delay them
  double inv = 0.0;
  if (m < rows) {  // uniform over the cluster (one row)
    const double bs = block_sum_double(sq, s_scratch);
    if (threadIdx.x == 0) s_cta = bs;
    tc::cluster_sync_all();  // every CTA's sum is in its shared memory
    if (threadIdx.x == 0) {
      double total = 0.0;
      const uint32_t sa = tc::smem_u32(&s_cta);
      for (int r = 0; r < PR_CTAS; r++) total += pr_ld_cluster_f64(tc::map_to_rank(sa, (uint32_t)r));
      s_total = total;
    }
    tc::cluster_sync_all();  // no CTA leaves while its sum may still be read; s_total visible in the CTA
    inv = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(s_total, (double)H), eps)));
  }
  if (c < n4) {
    const float f[4] = {v.x, v.y, v.z, v.w}, nws[4] = {nw.x, nw.y, nw.z, nw.w};
    uint16_t h[3][4];
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const float g = m < rows ? __double2float_rn(__dmul_rn(__dmul_rn((double)f[e], inv), (double)nws[e])) : 0.0f;
      split3_bf16(g, h[0][e], h[1][e], h[2][e]);
    }
#pragma unroll
    for (int tm = 0; tm < 3; tm++) {
      uint2 u;
      u.x = (uint32_t)h[tm][0] | ((uint32_t)h[tm][1] << 16);
      u.y = (uint32_t)h[tm][2] | ((uint32_t)h[tm][3] << 16);
      *(uint2 *)(x3n + ((size_t)tm * NT + m) * H + 4 * c) = u;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(pa.my_done + pa.region, 1u);
    if (prev == gridDim.x * gridDim.y - 1) {
      pa.my_done[pa.region] = 0u;
      pa.my_epoch[pa.region] += 1ull;
      __threadfence();
    }
  }
}

bool peer_norm_fusable(int H) { return H % 4 == 0 && H <= PR_CTAS * PR_THREADS * 4; }

void peer_reduce_norm_launch(stb_session *s, int region, int rows, int H, const float *residual, float *out,
                             const float *norm_w, double eps, uint16_t *x3n, int NT) {
  STB_REQUIRE(rows >= 1 && rows <= NT && peer_norm_fusable(H) && x3n && norm_w, "fused peer reduce + RMSNorm shape");
  PeerArgs pa = peer_args(s, region);
  launch_kernel(peer_reduce_norm_kernel, dim3(PR_CTAS, NT), dim3(PR_THREADS), 0, s->stream, true, pa, rows, H, residual,
                out, norm_w, eps, x3n, NT);
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
