// Decode-sized Linear on the tcgen05 tensor cores with Float32-accurate activations:
//   y[M,N] = x[M,K] . W[N,K]^T (+ bias) (+ residual),  8 <= M <= 64 token rows, BF16 weights.
//
// The SIMT decode GEMV keeps FP32 activations with FP32 FMA, which is bound by FP32 issue once M
// reaches ~10 (2M flop per weight byte).  Here each activation is split into three BF16 terms
//   x0 = rne(x), x1 = rne(x - x0), x2 = rne(x - x0 - x1)   (x - x0 and x - x0 - x1 are exact),
// which together carry x's 24-bit significand (the remainder is ~2^-27 |x|).  BF16 x BF16 products
// are exact in FP32.  The tensor core's FP32 accumulation is not round-to-nearest (a chain of
// ~200 MMAs drifted by ~3e-5 relative here), so each 64-wide K block gets a fresh TMEM accumulator
// (12 MMAs: x2, x1, x0 terms x 4 K steps) from a ring of four, and the epilogue warps add the block
// partials in FP32 in K order.  The result keeps Float32-activation accuracy (within the decode
// GEMV's 1e-5 * (1 + |e|)) at tensor-core throughput: the kernel is bound by streaming W from HBM.
//
// Grid: (N / 128 weight-row tiles) x KSPLIT.  Each CTA streams a 128 x (K / KSPLIT) slice of W
// through a 4-stage TMA ring (SWIZZLE_128B, K-major) together with the matching 3 x NT x 64 slice
// of the split activations (NT = M rounded up to 32 or 64), one thread issues
// tcgen05.mma.cta_group::1.kind::f16 (M = 128, N = NT), four warps read and sum TMEM and store the
// CTA's partial sums.  A second kernel adds the KSPLIT partials in split order (deterministic) and applies the
// epilogue.  Every mbarrier wait is bounded; each CTA loads its own tiles.
#include "tc_common.cuh"

namespace stb {

namespace {

using namespace tc;

constexpr int SK_BM = 128, SK_STAGES = 4, SK_ACC = 4;

template <int NT>
struct SkinnyShape {
  static constexpr int A_BYTES = SK_BM * BK * 2;
  static constexpr int B_BYTES = 3 * NT * BK * 2;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int SMEM = SK_STAGES * STAGE + 1024 + 256;
  static constexpr int TMEM_COLS = SK_ACC * NT;  // 128 or 256 columns, a power of two
};

// x [M][K] (row stride ldx) -> x3 [3][NT][K] BF16 terms; rows M..NT-1 are zero.
__global__ void split3_kernel(const float *x, int ldx, uint16_t *x3, int M, int NT, int K) {
  pdl_wait();
  pdl_trigger();
  const long total = (long)NT * K;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int m = (int)(i / K), k = (int)(i % K);
    const float v = m < M ? x[(size_t)m * ldx + k] : 0.0f;
    const uint16_t h0 = f32_to_bf16_rne(v);
    const float r1 = v - __uint_as_float((uint32_t)h0 << 16);  // exact
    const uint16_t h1 = f32_to_bf16_rne(r1);
    const float r2 = r1 - __uint_as_float((uint32_t)h1 << 16);  // exact
    const uint16_t h2 = f32_to_bf16_rne(r2);
    x3[(size_t)m * K + k] = h0;
    x3[((size_t)NT + m) * K + k] = h1;
    x3[((size_t)2 * NT + m) * K + k] = h2;
  }
}

template <int NT>
__global__ void __launch_bounds__(192, 1)
    gemm_skinny_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tx, float *part,
                       int M, int N, int K, int kb_per_split, uint32_t idesc, int *err) {
  using S = SkinnyShape<NT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t *bars = (uint64_t *)(smem + SK_STAGES * S::STAGE);
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + SK_STAGES);
  const uint32_t accf0 = smem_u32(bars + 2 * SK_STAGES), acce0 = smem_u32(bars + 2 * SK_STAGES + SK_ACC);
  const uint32_t drain = smem_u32(bars + 2 * SK_STAGES + 2 * SK_ACC);
  uint32_t *tmem_slot = (uint32_t *)(bars + 2 * SK_STAGES + 2 * SK_ACC + 1);
  volatile int *abort_flag = (volatile int *)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = blockIdx.x, ks = blockIdx.y;
  const int kblocks = (K + BK - 1) / BK;
  const int kb0 = ks * kb_per_split, kb1 = min(kblocks, kb0 + kb_per_split);

  if (threadIdx.x == 0) {
    for (int s = 0; s < SK_STAGES; s++) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int r = 0; r < SK_ACC; r++) {
      mbar_init(accf0 + 8 * r, 1);
      mbar_init(acce0 + 8 * r, 4);  // one arrival per epilogue warp
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(S::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sa0 = smem_u32(smem), sb0 = sa0 + SK_STAGES * S::A_BYTES;
  pdl_wait();  // the split activations come from the previous kernel

  if (warp == 0 && lane == 0) {
    int stage = 0;
    uint32_t phase = 0;
    for (int kb = kb0; kb < kb1; kb++) {
      if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, abort_flag, err, 31)) break;
      mbar_expect_tx(full0 + 8 * stage, S::STAGE);
      tma_load_2d(sa0 + stage * S::A_BYTES, &tw, kb * BK, nb * SK_BM, full0 + 8 * stage);
      tma_load_2d(sb0 + stage * S::B_BYTES, &tx, kb * BK, 0, full0 + 8 * stage);
      if (++stage == SK_STAGES) {
        stage = 0;
        phase ^= 1;
      }
    }
  } else if (warp == 1 && lane == 0) {
    // One K block (64 x 3 terms = 12 MMAs) per accumulator: short tensor-core chains, the block
    // partials are added in FP32 by the epilogue warps.
    int stage = 0;
    uint32_t phase = 0;
    bool issued = false;
    for (int kb = kb0, j = 0; kb < kb1; kb++, j++) {
      const int r = j % SK_ACC;
      if (!mbar_wait(acce0 + 8 * r, ((uint32_t)(j / SK_ACC) & 1u) ^ 1u, abort_flag, err, 35)) break;
      if (!mbar_wait(full0 + 8 * stage, phase, abort_flag, err, 32)) break;
      tc_fence_after();
      const uint64_t a = smem_desc(sa0 + stage * S::A_BYTES);
      const uint32_t d = tmem + (uint32_t)(r * NT);
#pragma unroll
      for (int t = 2; t >= 0; t--) {  // smallest term first: x2, x1, x0, each NT rows of the B tile
        const uint64_t b = smem_desc(sb0 + stage * S::B_BYTES + t * NT * BK * 2);
#pragma unroll
        for (int k = 0; k < BK / 16; k++)
          mma_f16(d, a + (uint64_t)(2 * k), b + (uint64_t)(2 * k), idesc, (t != 2 || k != 0));
      }
      issued = true;
      mma_commit(empty0 + 8 * stage);
      mma_commit(accf0 + 8 * r);
      if (++stage == SK_STAGES) {
        stage = 0;
        phase ^= 1;
      }
    }
    if (issued) {
      mma_commit(drain);
      volatile int no_abort = 0;
      mbar_wait(drain, 0, &no_abort, err, 33);
    }
  } else if (warp >= 2) {
    const int q = warp & 3;  // TMEM lane quarter of this warp
    const int row = nb * SK_BM + q * 32 + lane;
    float acc[NT];
#pragma unroll
    for (int m = 0; m < NT; m++) acc[m] = 0.0f;
    bool ok = true;
    for (int kb = kb0, j = 0; kb < kb1; kb++, j++) {
      const int r = j % SK_ACC;
      int got = 0;
      if (lane == 0) got = mbar_wait(accf0 + 8 * r, (uint32_t)(j / SK_ACC) & 1u, abort_flag, err, 34);
      if (!__shfl_sync(0xffffffffu, got, 0)) {
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < NT / 32; c++) {
        uint32_t v[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(r * NT + c * 32), v);
#pragma unroll
        for (int jj = 0; jj < 32; jj++) acc[c * 32 + jj] += __uint_as_float(v[jj]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acce0 + 8 * r);
    }
    if (ok && row < N) {
      float *pp = part + (size_t)ks * M * N;
#pragma unroll
      for (int m = 0; m < NT; m++)
        if (m < M) pp[(size_t)m * N + row] = acc[m];
    }
  }
  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(S::TMEM_COLS) : "memory");
}

// y[m][n] = residual + ((part_0 + part_1) + ... + bias): split-K partials in split order.
__global__ void skinny_reduce_kernel(const float *part, int splits, int M, int N, const float *bias,
                                     const float *residual, int ldr, float *y, int ldy) {
  pdl_wait();
  pdl_trigger();
  const long total = (long)M * N;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    float acc = part[i];
    for (int s = 1; s < splits; s++) acc += part[(size_t)s * total + i];
    const int m = (int)(i / N), n = (int)(i % N);
    if (bias) acc = acc + bias[n];
    if (residual) acc = residual[(size_t)m * ldr + n] + acc;
    y[(size_t)m * ldy + n] = acc;
  }
}

uint32_t skinny_idesc(int nt) {
  // D = F32, A = B = BF16, both K-major, N >> 3 at bits 17-22, M >> 4 at bits 24-28
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(nt >> 3) << 17) | ((uint32_t)(SK_BM >> 4) << 24);
}

}  // namespace

// Scratch bytes the skinny path needs for (M, N, K): split activations + split-K partials.
uint64_t skinny_scratch_bytes(int M, int N, int K, int *splits_out, int device) {
  const int nt = M <= 32 ? 32 : 64;
  const int tiles = (N + SK_BM - 1) / SK_BM;
  const int kblocks = (K + BK - 1) / BK;
  const int sms = sm_count(device);
  int splits = std::max(1, std::min(kblocks, (2 * sms + tiles - 1) / tiles));  // cover the SMs twice
  const int kbps = (kblocks + splits - 1) / splits;
  splits = (kblocks + kbps - 1) / kbps;
  if (splits_out) *splits_out = splits;
  const uint64_t x3 = ((uint64_t)3 * nt * K * 2 + 255) & ~255ull;
  return x3 + (uint64_t)splits * M * N * 4;
}

// Enqueues split -> skinny GEMM -> reduce on `stream`.  scratch: skinny_scratch_bytes() bytes.
void skinny_launch(const float *x, int ldx, const void *w, const float *bias, const float *residual, int ldr,
                   float *y, int ldy, int M, int N, int K, void *scratch, int *err, int device, cudaStream_t stream,
                   bool pdl) {
  int splits = 1;
  skinny_scratch_bytes(M, N, K, &splits, device);
  const int nt = M <= 32 ? 32 : 64;
  const int kblocks = (K + BK - 1) / BK;
  const int kbps = (kblocks + splits - 1) / splits;
  uint16_t *x3 = (uint16_t *)scratch;
  float *part = (float *)((char *)scratch + (((uint64_t)3 * nt * K * 2 + 255) & ~255ull));
  const long total = (long)nt * K;
  launch_kernel(split3_kernel, dim3((unsigned)std::min<long>((total + 255) / 256, 148 * 8)), dim3(256), 0, stream,
                pdl, x, ldx, x3, M, nt, K);
  const CUtensorMap tw = make_map(w, STB_BF16, (uint64_t)N, (uint64_t)K, SK_BM);
  const CUtensorMap tx = make_map(x3, STB_BF16, (uint64_t)3 * nt, (uint64_t)K, 3 * nt);
  const dim3 grid((N + SK_BM - 1) / SK_BM, splits);
  static std::mutex mu;
  static bool configured[64][2] = {};
  const int which = nt == 32 ? 0 : 1;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (device < 0 || device >= 64 || !configured[device][which]) {
      if (nt == 32)
        STB_CUDA(cudaFuncSetAttribute(gemm_skinny_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      SkinnyShape<32>::SMEM));
      else
        STB_CUDA(cudaFuncSetAttribute(gemm_skinny_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      SkinnyShape<64>::SMEM));
      if (device >= 0 && device < 64) configured[device][which] = true;
    }
  }
  if (nt == 32)
    launch_kernel(gemm_skinny_kernel<32>, grid, dim3(192), (size_t)SkinnyShape<32>::SMEM, stream, true, tw, tx, part,
                  M, N, K, kbps, skinny_idesc(32), err);
  else
    launch_kernel(gemm_skinny_kernel<64>, grid, dim3(192), (size_t)SkinnyShape<64>::SMEM, stream, true, tw, tx, part,
                  M, N, K, kbps, skinny_idesc(64), err);
  const long outs = (long)M * N;
  launch_kernel(skinny_reduce_kernel, dim3((unsigned)std::min<long>((outs + 255) / 256, 148 * 4)), dim3(256), 0,
                stream, true, (const float *)part, splits, M, N, bias, residual, ldr, y, ldy);
}

}  // namespace stb
