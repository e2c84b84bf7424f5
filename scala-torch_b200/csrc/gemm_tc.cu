// Prefill Linear on the tcgen05 tensor cores: y[M,N] = half(x)[M,K] . W[N,K]^T (+ bias), FP32
// accumulation in TMEM.  The same Linear as stb_linear (nn.Linear.apply, nn/src/main/scala/
// scalatorch/nn/Linear.scala:11-17) for prompt-sized M; the activations are rounded to the
// weight's type (round-to-nearest-even, SafeTensorsWriter.bfloat's rule for BF16) because a
// kind::f16 MMA takes both operands in one 16-bit type -- that rounding is the tolerance source.
//
// Two forms: gemm_tc2_kernel (below, the default) runs CTA pairs over 256x256 tiles;
// gemm_tc_kernel (STB_GEMM_PAIR=0) is the single-CTA form.
//
// Single-CTA kernel shape (one CTA per SM, persistent over 128x256 output tiles):
//   warp 0      TMA producer: x tile 128x64 and W tile 256x64 per stage (SWIZZLE_128B, K-major),
//               4-stage shared-memory ring guarded by full/empty mbarriers
//   warp 1      one thread issues tcgen05.mma (M=128, N=256, K=16) into a TMEM accumulator and
//               commits to the ring's empty barrier / the accumulator's full barrier
//   warp 2      allocates and frees the 512 TMEM columns (two 256-column accumulators)
//   warps 4..7  epilogue: tcgen05.ld 32 lanes x 32 columns at a time, + bias, Float32 stores;
//               accumulator double buffering overlaps a tile's epilogue with the next tile's MMAs
// Every mbarrier wait is bounded by the global timer; on expiry the kernel records an error code,
// stops issuing work, drains its MMAs (bounded) and frees TMEM before returning.
// Each CTA loads its own tiles from this GPU's memory; no load is shared across CTAs.
#include "tc_common.cuh"

namespace stb {

namespace {

using namespace tc;

constexpr int BM = 128, BN = 256, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2, STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int TMEM_COLS = 512;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;

struct TcParams {
  int M, N, K, ldy;
  float *y;
  const float *bias;
  int *err;
  const float *residual;  // optional: y = residual + (acc + bias); may alias y
  int ldr;
};

__global__ void __launch_bounds__(256, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb, TcParams p,
                   uint32_t idesc) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t *bars = (uint64_t *)(smem + STAGES * STAGE_BYTES);
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + STAGES);
  const uint32_t tfull0 = smem_u32(bars + 2 * STAGES), tempty0 = smem_u32(bars + 2 * STAGES + 2);
  const uint32_t drain = smem_u32(bars + 2 * STAGES + 4);
  uint32_t *tmem_slot = (uint32_t *)(bars + 2 * STAGES + 5);
  volatile int *abort_flag = (volatile int *)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mtiles = (p.M + BM - 1) / BM, ntiles = (p.N + BN - 1) / BN;
  const int tiles = mtiles * ntiles, kblocks = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int a = 0; a < 2; a++) {
      mbar_init(tfull0 + 8 * a, 1);
      mbar_init(tempty0 + 8 * a, 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sa0 = smem_u32(smem), sb0 = sa0 + STAGES * A_BYTES;

  if (warp == 0 && lane == 0) {
    int stage = 0;
    uint32_t phase = 0;
    for (int tile = blockIdx.x; tile < tiles && !*abort_flag; tile += gridDim.x) {
      const int mb = tile % mtiles, nb = tile / mtiles;
      for (int kb = 0; kb < kblocks; kb++) {
        if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, abort_flag, p.err, 1)) break;
        mbar_expect_tx(full0 + 8 * stage, STAGE_BYTES);
        tma_load_2d(sa0 + stage * A_BYTES, &ta, kb * BK, mb * BM, full0 + 8 * stage);
        tma_load_2d(sb0 + stage * B_BYTES, &tb, kb * BK, nb * BN, full0 + 8 * stage);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 1 && lane == 0) {
    int stage = 0, it = 0;
    uint32_t phase = 0;
    bool issued = false;
    for (int tile = blockIdx.x; tile < tiles && !*abort_flag; tile += gridDim.x, it++) {
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait(tempty0 + 8 * acc, acc_phase ^ 1, abort_flag, p.err, 2)) break;
      tc_fence_after();
      const uint32_t d = tmem + (uint32_t)(acc * BN);
      bool ok = true;
      for (int kb = 0; kb < kblocks; kb++) {
        if (!mbar_wait(full0 + 8 * stage, phase, abort_flag, p.err, 3)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t a = smem_desc(sa0 + stage * A_BYTES), b = smem_desc(sb0 + stage * B_BYTES);
#pragma unroll
        for (int k = 0; k < BK / 16; k++)  // +32 bytes of K per instruction inside the swizzle row
          mma_f16(d, a + (uint64_t)(2 * k), b + (uint64_t)(2 * k), idesc, (kb | k) != 0);
        issued = true;
        mma_commit(empty0 + 8 * stage);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
      mma_commit(tfull0 + 8 * acc);
    }
    if (issued) {  // all issued MMAs complete before TMEM is released
      mma_commit(drain);
      volatile int no_abort = 0;
      mbar_wait(drain, 0, &no_abort, p.err, 4);
    }
  } else if (warp >= 4) {
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    int it = 0;
    for (int tile = blockIdx.x; tile < tiles && !*abort_flag; tile += gridDim.x, it++) {
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      const int mb = tile % mtiles, nb = tile / mtiles;
      if (!mbar_wait(tfull0 + 8 * acc, acc_phase, abort_flag, p.err, 5)) break;
      tc_fence_after();
      const int row = mb * BM + q * 32 + lane;
      float *yrow = p.y + (size_t)row * p.ldy;
      const float *rrow = p.residual ? p.residual + (size_t)row * p.ldr : nullptr;
      for (int c = 0; c < BN / 32; c++) {
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + c * 32), r);
        const int n0 = nb * BN + c * 32;
        if (row < p.M && n0 < p.N) {
          // y = acc (+ bias) ; then y = residual + y (LlamaBlock's x + f(x), LlamaModel.scala:49-52)
          if (n0 + 32 <= p.N && (p.ldy & 3) == 0 && (!rrow || (p.ldr & 3) == 0)) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
              float4 v = make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]), __uint_as_float(r[j + 2]),
                                     __uint_as_float(r[j + 3]));
              if (p.bias) {
                v.x = v.x + p.bias[n0 + j];
                v.y = v.y + p.bias[n0 + j + 1];
                v.z = v.z + p.bias[n0 + j + 2];
                v.w = v.w + p.bias[n0 + j + 3];
              }
              if (rrow) {
                const float4 res = *reinterpret_cast<const float4 *>(rrow + n0 + j);
                v.x = res.x + v.x;
                v.y = res.y + v.y;
                v.z = res.z + v.z;
                v.w = res.w + v.w;
              }
              *reinterpret_cast<float4 *>(yrow + n0 + j) = v;
            }
          } else {
            for (int j = 0; j < 32 && n0 + j < p.N; j++) {
              float v = __uint_as_float(r[j]);
              if (p.bias) v = v + p.bias[n0 + j];
              if (rrow) v = rrow[n0 + j] + v;
              yrow[n0 + j] = v;
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(tempty0 + 8 * acc);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS)
                              : "memory");
}

// ---- CTA-pair form: a cluster of 2 CTAs (one per SM) computes 256 x 256 output tiles with
// tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 16).  CTA rank r loads rows [128 r, 128 r + 128)
// of the tile's x block and of its W block into its own shared memory (the MMA reads both halves of
// B from the two SMs), and holds rows [128 r, 128 r + 128) of the accumulator in its own TMEM.
// Per SM and K-block that is 32 KB of TMA writes for the same 128x256x64 multiply-adds per SM as the
// single-CTA form's 48 KB, so the same shared memory holds a 7-stage ring instead of 4: the refill
// loop (TMA latency ~1 us + commit) is covered by 1.8 us of MMA work instead of 1.0 us.
//   both CTAs  warp 0: TMA producer; completion bytes of both CTAs count on the leader's full barrier
//   leader     warp 1: issues the pair MMAs, commits to its own empty / accumulator barriers
//   leader     warp 3: forwards those phases to the peer's barriers (remote mbarrier arrivals)
//   both CTAs  warps 4..7: epilogue of their 128 rows; every epilogue thread of both CTAs arrives
//              on the leader's accumulator-empty barrier
// Waits are bounded as in gemm_tc_kernel and poll at CTA scope; the cross-CTA signals are relaxed
// remote arrivals that follow completed work (MMA commits, finished TMEM loads).  Both CTAs meet at
// cluster barriers before TMEM is freed.
constexpr int BM2 = 256, BN2 = 256, STAGES2 = 7;
constexpr int A2_BYTES = (BM2 / 2) * BK * 2, B2_BYTES = (BN2 / 2) * BK * 2, STAGE2_BYTES = A2_BYTES + B2_BYTES;
constexpr int SMEM2_BYTES = STAGES2 * STAGE2_BYTES + 1024 + 256;

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(256, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb, TcParams p,
                    uint32_t idesc) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t *bars = (uint64_t *)(smem + STAGES2 * STAGE2_BYTES);
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + STAGES2);
  const uint32_t tfull0 = smem_u32(bars + 2 * STAGES2), tempty0 = smem_u32(bars + 2 * STAGES2 + 2);
  const uint32_t drain = smem_u32(bars + 2 * STAGES2 + 4);
  uint32_t *tmem_slot = (uint32_t *)(bars + 2 * STAGES2 + 5);
  volatile int *abort_flag = (volatile int *)(tmem_slot + 1);

  const uint32_t rank = cluster_rank();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mtiles = (p.M + BM2 - 1) / BM2, ntiles = (p.N + BN2 - 1) / BN2;
  const int tiles = mtiles * ntiles, kblocks = (p.K + BK - 1) / BK;
  const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES2; s++) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int a = 0; a < 2; a++) {
      mbar_init(tfull0 + 8 * a, 1);
      mbar_init(tempty0 + 8 * a, 256);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers initialised and TMEM allocated before any cross-CTA use
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sa0 = smem_u32(smem), sb0 = sa0 + STAGES2 * A2_BYTES;
  const uint32_t full_lead0 = map_to_rank(full0, 0), tempty_lead0 = map_to_rank(tempty0, 0);

  if (warp == 0 && lane == 0) {
    int stage = 0;
    uint32_t phase = 0;
    for (int tile = pair; tile < tiles && !*abort_flag; tile += pairs) {
      const int mb = tile % mtiles, nb = tile / mtiles;
      for (int kb = 0; kb < kblocks; kb++) {
        if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, abort_flag, p.err, 11)) break;
        if (rank == 0) mbar_expect_tx(full0 + 8 * stage, 2 * STAGE2_BYTES);
        tma_load_2d_pair(sa0 + stage * A2_BYTES, &ta, kb * BK, mb * BM2 + (int)rank * (BM2 / 2),
                         full_lead0 + 8 * stage);
        tma_load_2d_pair(sb0 + stage * B2_BYTES, &tb, kb * BK, nb * BN2 + (int)rank * (BN2 / 2),
                         full_lead0 + 8 * stage);
        if (++stage == STAGES2) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 1 && lane == 0 && rank == 0) {
    int stage = 0, it = 0;
    uint32_t phase = 0;
    bool issued = false;
    for (int tile = pair; tile < tiles && !*abort_flag; tile += pairs, it++) {
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait(tempty0 + 8 * acc, acc_phase ^ 1, abort_flag, p.err, 12)) break;
      tc_fence_after();
      const uint32_t d = tmem + (uint32_t)(acc * BN2);
      bool ok = true;
      for (int kb = 0; kb < kblocks; kb++) {
        if (!mbar_wait(full0 + 8 * stage, phase, abort_flag, p.err, 13)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t a = smem_desc(sa0 + stage * A2_BYTES), b = smem_desc(sb0 + stage * B2_BYTES);
#pragma unroll
        for (int k = 0; k < BK / 16; k++)
          mma_f16_pair(d, a + (uint64_t)(2 * k), b + (uint64_t)(2 * k), idesc, (kb | k) != 0);
        issued = true;
        mma_commit_pair(empty0 + 8 * stage);
        if (++stage == STAGES2) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
      mma_commit_pair(tfull0 + 8 * acc);
    }
    if (issued) {
      mma_commit_pair(drain);
      volatile int no_abort = 0;
      mbar_wait(drain, 0, &no_abort, p.err, 14);
    }
  } else if (warp == 3 && lane == 0 && rank == 0) {
    // Forwarder: the leader's empty / accumulator-full phases, in the order the MMA thread
    // completes them, become arrivals on the peer's barriers of the same offsets.
    const uint32_t empty_peer0 = map_to_rank(empty0, 1), tfull_peer0 = map_to_rank(tfull0, 1);
    int stage = 0, it = 0;
    uint32_t phase = 0;
    for (int tile = pair; tile < tiles && !*abort_flag; tile += pairs, it++) {
      bool ok = true;
      for (int kb = 0; kb < kblocks; kb++) {
        if (!mbar_wait(empty0 + 8 * stage, phase, abort_flag, p.err, 15)) {
          ok = false;
          break;
        }
        mbar_arrive_cluster(empty_peer0 + 8 * stage);
        if (++stage == STAGES2) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
      const int acc = it & 1;
      if (!mbar_wait(tfull0 + 8 * acc, (it >> 1) & 1, abort_flag, p.err, 16)) break;
      mbar_arrive_cluster(tfull_peer0 + 8 * acc);
    }
  } else if (warp >= 4) {
    const int q = warp & 3;
    int it = 0;
    for (int tile = pair; tile < tiles && !*abort_flag; tile += pairs, it++) {
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      const int mb = tile % mtiles, nb = tile / mtiles;
      if (!mbar_wait(tfull0 + 8 * acc, acc_phase, abort_flag, p.err, 17)) break;
      tc_fence_after();
      const int row = mb * BM2 + (int)rank * (BM2 / 2) + q * 32 + lane;
      float *yrow = p.y + (size_t)row * p.ldy;
      const float *rrow = p.residual ? p.residual + (size_t)row * p.ldr : nullptr;
      for (int c = 0; c < BN2 / 32; c++) {
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN2 + c * 32), r);
        const int n0 = nb * BN2 + c * 32;
        if (row < p.M && n0 < p.N) {
          if (n0 + 32 <= p.N && (p.ldy & 3) == 0 && (!rrow || (p.ldr & 3) == 0)) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
              float4 v = make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]), __uint_as_float(r[j + 2]),
                                     __uint_as_float(r[j + 3]));
              if (p.bias) {
                v.x = v.x + p.bias[n0 + j];
                v.y = v.y + p.bias[n0 + j + 1];
                v.z = v.z + p.bias[n0 + j + 2];
                v.w = v.w + p.bias[n0 + j + 3];
              }
              if (rrow) {
                const float4 res = *reinterpret_cast<const float4 *>(rrow + n0 + j);
                v.x = res.x + v.x;
                v.y = res.y + v.y;
                v.z = res.z + v.z;
                v.w = res.w + v.w;
              }
              *reinterpret_cast<float4 *>(yrow + n0 + j) = v;
            }
          } else {
            for (int j = 0; j < 32 && n0 + j < p.N; j++) {
              float v = __uint_as_float(r[j]);
              if (p.bias) v = v + p.bias[n0 + j];
              if (rrow) v = rrow[n0 + j] + v;
              yrow[n0 + j] = v;
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive_cluster(tempty_lead0 + 8 * acc);
    }
  }
  tc_fence_before();
  cluster_sync_all();  // no CTA frees TMEM or exits while its pair may still signal its barriers
  tc_fence_after();
  if (warp == 2) asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS)
                              : "memory");
}

// x (Float32) -> weight type, round to nearest even, 8 elements per thread.
template <bool BF16>
__global__ void round_activations_kernel(const float *x, uint16_t *out, size_t count) {
  const size_t i = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) * 8;
  if (i + 8 <= count) {
    const float4 a = *reinterpret_cast<const float4 *>(x + i), b = *reinterpret_cast<const float4 *>(x + i + 4);
    const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    uint16_t h[8];
#pragma unroll
    for (int j = 0; j < 8; j++) h[j] = BF16 ? f32_to_bf16_rne(v[j]) : __half_as_ushort(__float2half_rn(v[j]));
    uint4 packed;
    packed.x = h[0] | ((uint32_t)h[1] << 16);
    packed.y = h[2] | ((uint32_t)h[3] << 16);
    packed.z = h[4] | ((uint32_t)h[5] << 16);
    packed.w = h[6] | ((uint32_t)h[7] << 16);
    *reinterpret_cast<uint4 *>(out + i) = packed;
  } else {
    for (size_t j = i; j < count; j++) out[j] = BF16 ? f32_to_bf16_rne(x[j]) : __half_as_ushort(__float2half_rn(x[j]));
  }
}

}  // namespace

// Instruction descriptor of kind::f16: D = F32 (bits 4-5 = 1), A/B = BF16 (1) or F16 (0) at bits
// 7-9 / 10-12, both K-major (bits 15/16 = 0), N >> 3 at bits 17-22, M >> 4 at bits 24-28.
uint32_t tc_idesc(int dtype) {
  const uint32_t ab = dtype == STB_BF16 ? 1u : 0u;
  return (1u << 4) | (ab << 7) | (ab << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

// The same for the CTA-pair MMA: M = 256, N = 256.
static uint32_t tc2_idesc(int dtype) {
  const uint32_t ab = dtype == STB_BF16 ? 1u : 0u;
  return (1u << 4) | (ab << 7) | (ab << 10) | ((uint32_t)(BN2 >> 3) << 17) | ((uint32_t)(BM2 >> 4) << 24);
}

// Pairs of SMs the CTA-pair kernel can keep resident at once (clusters of 2 at one CTA per SM).
static int resident_pairs(int device) {
  static std::mutex mu;
  static int pairs[64] = {};
  std::lock_guard<std::mutex> lock(mu);
  if (device >= 0 && device < 64 && pairs[device]) return pairs[device];
  STB_CUDA(cudaFuncSetAttribute(gemm_tc2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM2_BYTES));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(sm_count(device) & ~1));
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = SMEM2_BYTES;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 2;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, gemm_tc2_kernel, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = sm_count(device) / 2;
  }
  if (device >= 0 && device < 64) pairs[device] = n;
  return n;
}

static void gemm_tc2_launch(const void *xh, const void *w, int dtype, const float *bias, float *y, int ldy, int M,
                            int N, int K, int *err, int device, cudaStream_t stream, const float *residual,
                            int ldr) {
  const CUtensorMap ta = make_map(xh, dtype, (uint64_t)M, (uint64_t)K, BM2 / 2);
  const CUtensorMap tb = make_map(w, dtype, (uint64_t)N, (uint64_t)K, BN2 / 2);
  TcParams p{M, N, K, ldy, y, bias, err, residual, ldr};
  const int tiles = ((M + BM2 - 1) / BM2) * ((N + BN2 - 1) / BN2);
  const int pairs = std::min(tiles, resident_pairs(device));
  gemm_tc2_kernel<<<2 * pairs, 256, SMEM2_BYTES, stream>>>(ta, tb, p, tc2_idesc(dtype));
  check_launch("gemm_tc2");
}

// Enqueues the prefill GEMM on `stream`.  xh: the activations already in the weight's type
// (M x K, row-major); err: device int that receives a nonzero code if a wait expired.
// residual (optional, may alias y): y = residual + (x.W^T + bias), the residual add of a Llama block.
// The CTA-pair kernel by default; STB_GEMM_PAIR=0 selects the single-CTA kernel.
void gemm_tc_launch(const void *xh, const void *w, int dtype, const float *bias, float *y, int ldy, int M, int N,
                    int K, int *err, int device, cudaStream_t stream, const float *residual, int ldr) {
  static const int use_pair = env_int("STB_GEMM_PAIR", 1);
  if (use_pair) {
    gemm_tc2_launch(xh, w, dtype, bias, y, ldy, M, N, K, err, device, stream, residual, ldr);
    return;
  }
  const CUtensorMap ta = make_map(xh, dtype, (uint64_t)M, (uint64_t)K, BM);
  const CUtensorMap tb = make_map(w, dtype, (uint64_t)N, (uint64_t)K, BN);
  TcParams p{M, N, K, ldy, y, bias, err, residual, ldr};
  const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int grid = std::min(tiles, sm_count(device));
  static std::mutex mu;
  static bool configured[64] = {};
  {
    std::lock_guard<std::mutex> lock(mu);
    if (device < 0 || device >= 64 || !configured[device]) {
      STB_CUDA(cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
      if (device >= 0 && device < 64) configured[device] = true;
    }
  }
  gemm_tc_kernel<<<grid, 256, SMEM_BYTES, stream>>>(ta, tb, p, tc_idesc(dtype));
  check_launch("gemm_tc");
}

void gemm_tc_launch(const void *xh, const void *w, int dtype, const float *bias, float *y, int ldy, int M, int N,
                    int K, int *err, int device, cudaStream_t stream) {
  gemm_tc_launch(xh, w, dtype, bias, y, ldy, M, N, K, err, device, stream, nullptr, 0);
}

void round_activations(const float *x, uint16_t *out, size_t count, int dtype, cudaStream_t stream) {
  const size_t threads = (count + 7) / 8;
  const unsigned blocks = (unsigned)((threads + 255) / 256);
  if (dtype == STB_BF16) round_activations_kernel<true><<<blocks, 256, 0, stream>>>(x, out, count);
  else round_activations_kernel<false><<<blocks, 256, 0, stream>>>(x, out, count);
  check_launch("round_activations");
}

}  // namespace stb

using namespace stb;

extern "C" {

int stb_linear_prefill(stb_session *s, uint64_t x, uint64_t w, int w_dtype, uint64_t bias, uint64_t y, int M, int N,
                       int K) {
  return guarded([&] {
    enter(s);
    STB_REQUIRE(M >= 0 && N >= 0 && K >= 0, "Linear dimensions must be nonnegative");
    STB_REQUIRE(w_dtype == STB_BF16 || w_dtype == STB_F16, "tensor-core Linear needs BF16 or F16 weights");
    if (M == 0 || N == 0) return;
    STB_REQUIRE(K > 0 && K % 8 == 0, "tensor-core Linear needs K a positive multiple of 8");
    STB_REQUIRE(x && w && y, "null buffer");
    STB_REQUIRE(x % 16 == 0 && w % 16 == 0 && y % 16 == 0, "buffers must be 16-byte aligned");
    const uint64_t xbytes = (uint64_t)M * K * 2;
    int *err = session_error_word(s);
    const uint64_t scratch = session_scratch(s, xbytes);
    round_activations((const float *)x, (uint16_t *)scratch, (size_t)M * K, w_dtype, s->stream);
    gemm_tc_launch((const void *)scratch, (const void *)w, w_dtype, (const float *)bias, (float *)y, N, M, N, K, err,
                   s->device, s->stream);
    count_launch(s, 2);
  });
}

}  // extern "C"
