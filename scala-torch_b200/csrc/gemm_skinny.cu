// Decode-sized Linear on the tcgen05 tensor cores with Float32-accurate activations:
//   y[M,N] = epilogue(x[M,K] . W[N,K]^T),  M >= 1 token rows (blocks of 64), BF16 weights,
// with the vector GEMV's optional RMSNorm prologue and its epilogues (gemv.cuh).
//
// The SIMT decode GEMV keeps FP32 activations with FP32 FMA, which is bound by FP32 issue once M
// reaches ~10 (2M flop per weight byte).  Here each activation is split into three BF16 terms
//   x0 = rne(x), x1 = rne(x - x0), x2 = rne(x - x0 - x1)   (x - x0 and x - x0 - x1 are exact),
// which together carry x's 24-bit significand (the remainder is ~2^-27 |x|).  BF16 x BF16 products
// are exact in FP32.  The B operand of one MMA is the whole [x0; x1; x2] tile (N = 3 NT rows), so a
// 64-wide K block takes 4 MMAs (M = 128, N = 3 NT, K = 16) rather than 12 dependent small ones, and
// the three term products land in separate TMEM column groups.  The tensor core's FP32
// accumulation is not round-to-nearest (a chain of ~200 MMAs drifted by ~3e-5 relative), so each
// group of 1 / 4 / 8 K blocks (NT = 16 / 32 / 64; chains of at most 32 MMAs) gets a fresh
// accumulator from a ring, and the epilogue warps combine the terms ((x2 + x1) + x0) and add the
// group partials in FP32 in K order.  Larger groups give the epilogue, which reads 3 NT columns per
// group, fewer turns where NT is wide.  The result keeps
// Float32-activation accuracy (within the decode GEMV's 1e-5 * (1 + |e|)) at tensor-core
// throughput: the kernel is bound by streaming W from HBM.
//
// Three kernels:
//   1. prologue: RMSNorm (the GEMV's expression) and the split into x3[3][NT][K] (NT = M rounded up
//      to 16, 32 or 64; rows M..NT-1 zero), one block per 1024 elements of a row;
//   2. stream-K GEMM: persistent CTAs, two per SM (one for 64-row term tiles).  The iterations
//      (128-row weight tile t, 64-wide K block kb), t-major, are cut into gridDim.x equal contiguous
//      ranges, so every SM streams the same number of weight bytes whatever the tile count.  Warp 0
//      issues TMA loads of the W tile and the matching 3 x NT x 64 slice of x3 through a 3-5 stage
//      ring (SWIZZLE_128B,
//      K-major; the first stages' W loads go out before the programmatic-dependency wait, since
//      weights never depend on the previous kernel), warp 1 issues
//      tcgen05.mma.cta_group::1.kind::f16 (M = 128, N = 3 NT), warps 2-5 sum the accumulators and
//      store one partial per (tile, piece): the part of a tile's K range this CTA covered;
//   3. fixup: adds each tile's pieces in piece (= K) order and applies the epilogue.
// Deterministic for a given SM count.  Every mbarrier wait is bounded; each CTA loads its own tiles.
#include "gemv.cuh"
#include "tc_common.cuh"

namespace stb {

namespace {

using namespace tc;

constexpr int SK_BM = 128, SK_ACC_MAX = 4;

template <int NT>
struct SkinnyShape {
  // Two CTAs per SM for 16- and 32-row term tiles (their MMA and epilogue latencies overlap: the 70B
  // gate/up shard at M = 8 took 169 us with one 9-stage CTA per SM and 155 us with two 5-stage CTAs),
  // one for 64-row tiles, whose stages are too large to fit two rings.
  static constexpr int CTAS_PER_SM = NT == 64 ? 1 : 2;
  static constexpr int STAGES = NT == 16 ? 5 : (NT == 32 ? 3 : 5);
  static constexpr int A_BYTES = SK_BM * BK * 2;
  static constexpr int B_BYTES = 3 * NT * BK * 2;  // multiple of 1024: the tile stays swizzle-aligned
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int SMEM = STAGES * STAGE + 1024 + 256;
  static constexpr int ACC_STRIDE = NT == 16 ? 64 : (NT == 32 ? 128 : 256);  // >= 3 NT TMEM columns
  static constexpr int ACC = NT == 16 ? 4 : 2;                                // accumulators in the ring
  static constexpr int GK = NT == 16 ? 1 : (NT == 32 ? 4 : 8);  // K blocks per accumulator (4 GK MMAs per chain)
  static constexpr int TMEM_COLS = ACC * ACC_STRIDE;                          // 256 or 512
  static_assert(SMEM <= 232448, "shared memory per CTA");
  static_assert(CTAS_PER_SM * (SMEM + 1024) <= 233472, "shared memory per SM");
  static_assert(CTAS_PER_SM * TMEM_COLS <= 512 && ACC <= SK_ACC_MAX, "tensor memory");
  static_assert((2 * STAGES + 2 * SK_ACC_MAX + 1) * 8 + 8 <= 256, "barrier area");
};

// Three W-column TMEM loads (the x2, x1 and x0 term columns of one chunk) and one wait, in a
// single asm statement so no use of the registers can be scheduled before the wait.
template <int W>
__device__ __forceinline__ void tmem_ld3(uint32_t a2, uint32_t a1, uint32_t a0, float (&t2)[W], float (&t1)[W],
                                         float (&t0)[W]) {
  static_assert(W == 16 || W == 32, "load width");
  uint32_t r[3 * W];
  if constexpr (W == 16) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%48];\n"
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%49];\n"
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47}, [%50];\n"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47])
        : "r"(a2), "r"(a1), "r"(a0)
        : "memory");
  } else {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%96];\n"
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%97];\n"
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%64, %65, %66, %67, %68, %69, %70, %71, %72, %73, %74, %75, %76, %77, %78, %79, %80, %81, %82, %83, %84, %85, %86, %87, %88, %89, %90, %91, %92, %93, %94, %95}, [%98];\n"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63]), "=r"(r[64]), "=r"(r[65]), "=r"(r[66]), "=r"(r[67]), "=r"(r[68]), "=r"(r[69]), "=r"(r[70]), "=r"(r[71]), "=r"(r[72]), "=r"(r[73]), "=r"(r[74]), "=r"(r[75]), "=r"(r[76]), "=r"(r[77]), "=r"(r[78]), "=r"(r[79]), "=r"(r[80]), "=r"(r[81]), "=r"(r[82]), "=r"(r[83]), "=r"(r[84]), "=r"(r[85]), "=r"(r[86]), "=r"(r[87]), "=r"(r[88]), "=r"(r[89]), "=r"(r[90]), "=r"(r[91]), "=r"(r[92]), "=r"(r[93]), "=r"(r[94]), "=r"(r[95])
        : "r"(a2), "r"(a1), "r"(a0)
        : "memory");
  }
#pragma unroll
  for (int j = 0; j < W; j++) {
    t2[j] = __uint_as_float(r[j]);
    t1[j] = __uint_as_float(r[W + j]);
    t0[j] = __uint_as_float(r[2 * W + j]);
  }
}

// First iteration of CTA c when T iterations are cut into G ranges.
__host__ __device__ __forceinline__ long long sk_start(int c, long long T, int G) { return (long long)c * T / G; }

__device__ __forceinline__ int sk_cta_of(long long i, long long T, int G) { return skinny_cta_of(i, T, G); }

// x [M][K] (row stride ldx), optionally RMS-normalised as the vector GEMV does it, -> x3 [3][NT][K].
// Block (kb, m) converts elements [kb * 1024, kb * 1024 + 1024) of row m, four per thread; with
// RMSNorm every block of a row recomputes the row's inverse RMS with the GEMV's exact loop and
// reduction order, so all blocks (and the GEMV) agree bit for bit.  The kernel is latency-bound
// (a few microseconds between two GEMMs), so every global load is issued before its first use:
// the thread's four elements and norm weights with the first 32 terms of the sum of squares, the
// rest of the sum 32 terms per round trip, still added in the loop's order.
__global__ void __launch_bounds__(256) skinny_prep_kernel(const float *x, int ldx, const float *norm_w,
                                                          double eps, uint16_t *x3, int M, int NT, int K) {
  __shared__ double s_scratch[8];
  pdl_wait();
  pdl_trigger();
  const int m = blockIdx.y;
  const int k0 = blockIdx.x * 1024 + threadIdx.x * 4;
  const bool vec = k0 + 4 <= K && (ldx & 3) == 0 && ((uintptr_t)x & 15) == 0;
  float v[4] = {0.0f, 0.0f, 0.0f, 0.0f}, nw[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  if (m < M) {
    const float *xr = x + (size_t)m * ldx;
    if (vec) {
      const float4 f = *(const float4 *)(xr + k0);
      v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
    } else {
#pragma unroll
      for (int e = 0; e < 4; e++)
        if (k0 + e < K) v[e] = xr[k0 + e];
    }
    if (norm_w) {
#pragma unroll
      for (int e = 0; e < 4; e++)
        if (k0 + e < K) nw[e] = norm_w[k0 + e];
    }
  }
  double inv = 1.0;
  if (m < M && norm_w) {
    const float *xr = x + (size_t)m * ldx;
    double sq = 0.0;
    int k = threadIdx.x;
    for (; k + 31 * 256 < K; k += 32 * 256) {
      float t[32];
#pragma unroll
      for (int i = 0; i < 32; i++) t[i] = xr[k + i * 256];
#pragma unroll
      for (int i = 0; i < 32; i++) {
        const double d = (double)t[i];
        sq = __dadd_rn(sq, __dmul_rn(d, d));
      }
    }
    for (; k < K; k += 256) {
      const double d = (double)xr[k];
      sq = __dadd_rn(sq, __dmul_rn(d, d));
    }
    const double total = block_sum_double(sq, s_scratch);
    inv = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(total, (double)K), eps)));
  }
  uint16_t h[3][4] = {};
#pragma unroll
  for (int e = 0; e < 4; e++) {
    float f = v[e];
    if (m < M && norm_w) f = __double2float_rn(__dmul_rn(__dmul_rn((double)f, inv), (double)nw[e]));
    split3_bf16(f, h[0][e], h[1][e], h[2][e]);
  }
  if (k0 + 4 <= K && (K & 3) == 0) {  // rows of x3 are 8-byte aligned: one 8-byte store per term
#pragma unroll
    for (int tm = 0; tm < 3; tm++) {
      uint2 u;
      u.x = (uint32_t)h[tm][0] | ((uint32_t)h[tm][1] << 16);
      u.y = (uint32_t)h[tm][2] | ((uint32_t)h[tm][3] << 16);
      *(uint2 *)(x3 + ((size_t)tm * NT + m) * K + k0) = u;
    }
  } else {
#pragma unroll
    for (int e = 0; e < 4; e++)
      if (k0 + e < K)
#pragma unroll
        for (int tm = 0; tm < 3; tm++) x3[((size_t)tm * NT + m) * K + k0 + e] = h[tm][e];
  }
}

template <int NT>
__global__ void __launch_bounds__(192, 2)
    gemm_skinny_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tx, float *part,
                       int M, int N, int kbs, long long T, int pmax, uint32_t idesc, int *err) {
  using S = SkinnyShape<NT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t *bars = (uint64_t *)(smem + S::STAGES * S::STAGE);
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + S::STAGES);
  const uint32_t accf0 = smem_u32(bars + 2 * S::STAGES), acce0 = smem_u32(bars + 2 * S::STAGES + SK_ACC_MAX);
  const uint32_t drain = smem_u32(bars + 2 * S::STAGES + 2 * SK_ACC_MAX);
  uint32_t *tmem_slot = (uint32_t *)(bars + 2 * S::STAGES + 2 * SK_ACC_MAX + 1);
  volatile int *abort_flag = (volatile int *)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta = blockIdx.x, G = gridDim.x;
  const long long i0 = sk_start(cta, T, G), i1 = sk_start(cta + 1, T, G);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::STAGES; s++) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int r = 0; r < S::ACC; r++) {
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
  const uint32_t sa0 = smem_u32(smem), sb0 = sa0 + S::STAGES * S::A_BYTES;

  if (warp == 0) {
    if (lane == 0) {
      // Weights never depend on the previous kernel: the first ring's W tiles load before the wait
      // for the split activations.
      const int pre = (int)min((long long)S::STAGES, i1 - i0);
      // (tile, K block) of the next load, advanced without dividing the 64-bit iteration index
      int t = (int)(i0 / kbs), kb = (int)(i0 % kbs);
      for (int j = 0; j < pre; j++) {
        mbar_expect_tx(full0 + 8 * j, S::STAGE);
        tma_load_2d(sa0 + j * S::A_BYTES, &tw, kb * BK, t * SK_BM, full0 + 8 * j);
        if (++kb == kbs) {
          kb = 0;
          t++;
        }
      }
      pdl_wait();
      {
        int kx = (int)(i0 % kbs);
        for (int j = 0; j < pre; j++) {
          tma_load_2d(sb0 + j * S::B_BYTES, &tx, kx * BK, 0, full0 + 8 * j);
          if (++kx == kbs) kx = 0;
        }
      }
      int stage = pre % S::STAGES;
      uint32_t phase = pre == S::STAGES ? 1u : 0u;
      for (long long i = i0 + pre; i < i1; i++) {
        if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, abort_flag, err, 31)) break;
        mbar_expect_tx(full0 + 8 * stage, S::STAGE);
        tma_load_2d(sa0 + stage * S::A_BYTES, &tw, kb * BK, t * SK_BM, full0 + 8 * stage);
        tma_load_2d(sb0 + stage * S::B_BYTES, &tx, kb * BK, 0, full0 + 8 * stage);
        if (++kb == kbs) {
          kb = 0;
          t++;
        }
        if (++stage == S::STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // Accumulator groups: up to GK consecutive K blocks of one tile; a group also ends at the end of
      // a tile or of this CTA's range (the epilogue walks the same groups).
      int stage = 0;
      uint32_t phase = 0;
      bool issued = false;
      int grp = 0, cnt = 0, kb = (int)(i0 % kbs);
      for (long long i = i0; i < i1; i++) {
        const int r = grp % S::ACC;
        if (cnt == 0 && !mbar_wait(acce0 + 8 * r, ((uint32_t)(grp / S::ACC) & 1u) ^ 1u, abort_flag, err, 35)) break;
        if (!mbar_wait(full0 + 8 * stage, phase, abort_flag, err, 32)) break;
        tc_fence_after();
        const uint64_t a = smem_desc(sa0 + stage * S::A_BYTES);
        const uint64_t b = smem_desc(sb0 + stage * S::B_BYTES);  // [x0; x1; x2]: N = 3 NT rows
        const uint32_t d = tmem + (uint32_t)(r * S::ACC_STRIDE);
#pragma unroll
        for (int k = 0; k < BK / 16; k++)
          mma_f16(d, a + (uint64_t)(2 * k), b + (uint64_t)(2 * k), idesc, cnt != 0 || k != 0);
        issued = true;
        mma_commit(empty0 + 8 * stage);
        if (++kb == kbs) kb = 0;  // kb == 0: the next iteration starts a tile
        if (++cnt == S::GK || kb == 0 || i + 1 == i1) {
          mma_commit(accf0 + 8 * r);
          grp++;
          cnt = 0;
        }
        if (++stage == S::STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (issued) {
        mma_commit(drain);
        volatile int no_abort = 0;
        mbar_wait(drain, 0, &no_abort, err, 33);
      }
    }
  } else {
    pdl_wait();  // the previous fixup may still read `part`
    const int q = warp & 3;  // TMEM lane quarter of this warp
    float acc[NT];
#pragma unroll
    for (int m = 0; m < NT; m++) acc[m] = 0.0f;
    int grp = 0, cnt = 0, kb = (int)(i0 % kbs), t = (int)(i0 / kbs);
    for (long long i = i0; i < i1; i++) {
      const bool tile_end = ++kb == kbs;
      if (tile_end) kb = 0;
      if (!(++cnt == S::GK || tile_end || i + 1 == i1)) continue;  // inside an accumulator group
      cnt = 0;
      const int r = grp % S::ACC;
      int got = 0;
      if (lane == 0) got = mbar_wait(accf0 + 8 * r, (uint32_t)(grp / S::ACC) & 1u, abort_flag, err, 34);
      if (!__shfl_sync(0xffffffffu, got, 0)) break;
      tc_fence_after();
      constexpr int W = NT == 16 ? 16 : 32;
      const uint32_t base = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(r * S::ACC_STRIDE);
#pragma unroll
      for (int c = 0; c < NT / W; c++) {  // columns t * NT + m hold term t of token row m
        float lo[W], mid[W], hi[W];
        tmem_ld3<W>(base + (uint32_t)(2 * NT + c * W), base + (uint32_t)(NT + c * W), base + (uint32_t)(c * W), lo,
                    mid, hi);
#pragma unroll
        for (int jj = 0; jj < W; jj++) acc[c * W + jj] += (lo[jj] + mid[jj]) + hi[jj];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acce0 + 8 * r);
      grp++;
      if (i + 1 == i1 || tile_end) {  // end of this CTA's piece of tile t
        const int piece = cta - sk_cta_of((long long)t * kbs, T, G);
        const int row = t * SK_BM + q * 32 + lane;
        if (row < N) {
          float *pp = part + ((size_t)t * pmax + piece) * M * SK_BM + q * 32 + lane;
#pragma unroll
          for (int m = 0; m < NT; m++)
            if (m < M) pp[(size_t)m * SK_BM] = acc[m];
        }
#pragma unroll
        for (int m = 0; m < NT; m++) acc[m] = 0.0f;
        t++;
      }
    }
  }
  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(S::TMEM_COLS) : "memory");
}

// Sum of the pieces of output (m, row) in piece order.
__device__ __forceinline__ float sk_gather(const float *part, int m, int row, int M, int kbs, long long T, int G,
                                           int pmax) {
  const int t = row / SK_BM;
  const int first = sk_cta_of((long long)t * kbs, T, G), last = sk_cta_of((long long)(t + 1) * kbs - 1, T, G);
  const float *pp = part + ((size_t)t * pmax * M + m) * SK_BM + (row % SK_BM);
  const size_t stride = (size_t)M * SK_BM;
  const int n = last - first + 1;
  // pieces four loads at a time (one round trip each), added in piece order
  float s = 0.0f;
  for (int p0 = 0; p0 < n; p0 += 4) {
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; j++) v[j] = p0 + j < n ? pp[(size_t)(p0 + j) * stride] : 0.0f;
#pragma unroll
    for (int j = 0; j < 4; j++)
      if (p0 + j < n) s = p0 + j == 0 ? v[0] : s + v[j];
  }
  return s;
}

// One thread per (token row, output row) -- per row pair for SiLU / QKV -- with the vector GEMV's
// epilogue expressions.  This launch covers rows m0 .. m0 + mb - 1 of the problem (blockIdx.y = row
// within the block; `part` holds mb rows); mg is the row in the problem's own indexing.
template <int EPI>
__global__ void __launch_bounds__(256) skinny_fixup_kernel(const GemvParams p, const float *part, int kbs,
                                                           long long T, int G, int pmax, int m0, int mb) {
  pdl_wait();
  pdl_trigger();
  constexpr bool paired = EPI == EPI_SILU || EPI == EPI_QKV;
  const int m = blockIdx.y, mg = m0 + m;
  const int units = paired ? p.N / 2 : p.N;
  const int u = blockIdx.x * 256 + threadIdx.x;
  if constexpr (EPI == EPI_LOGITS) {
    __shared__ unsigned long long s_best[8];
    unsigned long long key = 0ull;
    if (u < units) {
      const float v = sk_gather(part, m, u, mb, kbs, T, G, pmax);
      p.y[(size_t)mg * p.ldy + u] = v;
      key = argmax_key(v, u + p.row_offset);
    }
    if (p.best) {  // uniform: every thread of the block reaches the reduction
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        const unsigned long long o = __shfl_xor_sync(0xffffffffu, key, off);
        key = o > key ? o : key;
      }
      if ((threadIdx.x & 31) == 0) s_best[threadIdx.x >> 5] = key;
      __syncthreads();
      if (threadIdx.x == 0) {
        unsigned long long b = s_best[0];
        for (int w = 1; w < 8; w++) b = s_best[w] > b ? s_best[w] : b;
        if (b) atomicMax(&p.best[mg], b);
      }
    }
    return;
  }
  if (u >= units) return;
  if constexpr (EPI == EPI_PLAIN) {
    float v = sk_gather(part, m, u, mb, kbs, T, G, pmax);
    if (p.bias) v = v + p.bias[u];
    p.y[(size_t)mg * p.ldy + u] = v;
  } else if constexpr (EPI == EPI_RESID) {
    const float v = sk_gather(part, m, u, mb, kbs, T, G, pmax);
    p.y[(size_t)mg * p.ldy + u] = p.residual[(size_t)mg * p.ldr + u] + v;
  } else if constexpr (EPI == EPI_PEER) {
    const float v = sk_gather(part, m, u, mb, kbs, T, G, pmax);
    const uint32_t use = (uint32_t)(p.peer.my_epoch[p.peer.region] + 1ull);
    const size_t off = ((size_t)p.peer.region * p.peer.tp + p.peer.rank) * p.peer.slot_elems + (size_t)mg * p.ldy + u;
    const unsigned long long w = peer_word(v, use);
    for (int r = 0; r < p.peer.tp; r++) peer_store(p.peer.slots[r] + off, w);
  } else if constexpr (EPI == EPI_SILU) {
    const float gate = sk_gather(part, m, 2 * u, mb, kbs, T, G, pmax);
    const float up = sk_gather(part, m, 2 * u + 1, mb, kbs, T, G, pmax);
    p.y[(size_t)mg * p.ldy + u] = silu_ref(gate) * up;
  } else if constexpr (EPI == EPI_QKV) {
    const float fa = sk_gather(part, m, 2 * u, mb, kbs, T, G, pmax);
    const float fb = sk_gather(part, m, 2 * u + 1, mb, kbs, T, G, pmax);
    qkv_store_pair(p, mg, u, fa, fb, p.pos_dev ? *p.pos_dev : p.pos0);
  }
}

// The next projection's prologue fused into this projection's fixup (decode chunks of one 64-row block):
// both kernels write the next projection's activation terms x3n [3][NT][Kn] (rows M .. NT - 1 zero),
// so the next GEMM starts on them without a prologue launch of its own.

// SiLU(gate) * up of the interleaved gate/up projection (EPI_SILU's expression), split into three BF16
// terms for the down projection (Kn = N / 2).  Thread (token row, units 4 u .. 4 u + 3): the 8
// interleaved projection rows of its 4 units are two float4 per stream-K piece, every piece's loads in
// flight together; one 8-byte store per term.  blockIdx.y < NT; rows mb .. NT - 1 get zeros.
__global__ void __launch_bounds__(256) skinny_fixup_silu_split_kernel(const float *part, int N, int kbs, long long T,
                                                                      int G, int pmax, int mb, uint16_t *x3n,
                                                                      int NT) {
  pdl_wait();
  const int m = blockIdx.y, units = N / 2;
  const int u0 = 4 * (blockIdx.x * 256 + threadIdx.x);
  if (u0 >= units) return;
  float f[4] = {0.f, 0.f, 0.f, 0.f};
  if (m < mb) {
    const int row = 2 * u0, t = row / SK_BM;  // 8 rows, within one 128-row tile
    const int first = sk_cta_of((long long)t * kbs, T, G);
    const int n = sk_cta_of((long long)(t + 1) * kbs - 1, T, G) - first + 1;
    const float *pp = part + ((size_t)t * pmax * mb + m) * SK_BM + (row % SK_BM);
    const size_t stride = (size_t)mb * SK_BM;
    float4 w[4][2];
#pragma unroll
    for (int q = 0; q < 4; q++)
      if (q < n) {
        w[q][0] = __ldcg((const float4 *)(pp + q * stride));
        w[q][1] = __ldcg((const float4 *)(pp + q * stride + 4));
      }
    float4 a = w[0][0], b = w[0][1];
#pragma unroll
    for (int q = 1; q < 4; q++)
      if (q < n) {
        a.x = a.x + w[q][0].x; a.y = a.y + w[q][0].y; a.z = a.z + w[q][0].z; a.w = a.w + w[q][0].w;
        b.x = b.x + w[q][1].x; b.y = b.y + w[q][1].y; b.z = b.z + w[q][1].z; b.w = b.w + w[q][1].w;
      }
    for (int q = 4; q < n; q++) {  // more than four pieces: one round trip each
      const float4 c = __ldcg((const float4 *)(pp + q * stride)), d = __ldcg((const float4 *)(pp + q * stride + 4));
      a.x = a.x + c.x; a.y = a.y + c.y; a.z = a.z + c.z; a.w = a.w + c.w;
      b.x = b.x + d.x; b.y = b.y + d.y; b.z = b.z + d.z; b.w = b.w + d.w;
    }
    f[0] = silu_ref(a.x) * a.y;  // (gate, up) pairs
    f[1] = silu_ref(a.z) * a.w;
    f[2] = silu_ref(b.x) * b.y;
    f[3] = silu_ref(b.z) * b.w;
  }
  pdl_trigger();  // after this thread's loads: the next GEMM's weight stream would delay them
  uint16_t h[3][4];
#pragma unroll
  for (int e = 0; e < 4; e++) split3_bf16(f[e], h[0][e], h[1][e], h[2][e]);
#pragma unroll
  for (int tm = 0; tm < 3; tm++) {
    uint2 v;
    v.x = (uint32_t)h[tm][0] | ((uint32_t)h[tm][1] << 16);
    v.y = (uint32_t)h[tm][2] | ((uint32_t)h[tm][3] << 16);
    *(uint2 *)(x3n + ((size_t)tm * NT + m) * units + u0) = v;
  }
}

constexpr int SK_NORM_CTAS = 8, SK_NORM_THREADS = 256;  // a cluster per row: 8 x 256 x 4 = 8192 values

__device__ __forceinline__ double ld_cluster_f64(uint32_t cluster_addr) {
  double v;
  asm volatile("ld.shared::cluster.f64 %0, [%1];" : "=d"(v) : "r"(cluster_addr) : "memory");
  return v;
}

// The residual projection's fixup (EPI_RESID: y = residual + sum of the pieces in piece order) and the
// next projection's RMSNorm prologue on the updated row.  A cluster of 8 CTAs per token row, one float4
// of the row per thread (every load in flight together); each CTA reduces its sum of squares (double,
// the block's fixed order) and the row's total is its CTAs' sums added in cluster-rank order through
// distributed shared memory; then each thread scales its values with the GEMV's expression and writes
// their three BF16 terms (Kn = N).  Clusters of rows m >= mb write zero rows.
__global__ void __cluster_dims__(SK_NORM_CTAS, 1, 1) __launch_bounds__(SK_NORM_THREADS) skinny_fixup_norm_kernel(
    const GemvParams p, const float *part, int kbs, long long T, int G, int pmax, int mb, const float *norm_w,
    double eps, uint16_t *x3n, int NT) {
  __shared__ double s_scratch[SK_NORM_THREADS / 32];
  __shared__ double s_cta, s_total;
  pdl_wait();
  const int m = blockIdx.y, mg = m;  // one 64-row block: its rows are the problem's own
  const int N = p.N, n4 = N / 4;
  const int c = blockIdx.x * SK_NORM_THREADS + threadIdx.x;  // float4 of the row
  const bool live = m < mb && c < n4;
  float4 v = make_float4(0.f, 0.f, 0.f, 0.f), nw = v;
  double sq = 0.0;
  if (live) {
    const int row = 4 * c, t = row / SK_BM;  // a four-row group never straddles a 128-row tile
    const int n = sk_cta_of((long long)(t + 1) * kbs - 1, T, G) - sk_cta_of((long long)t * kbs, T, G) + 1;
    const float *pp = part + ((size_t)t * pmax * mb + m) * SK_BM + (row % SK_BM);
    const size_t stride = (size_t)mb * SK_BM;
    v = *(const float4 *)(p.residual + (size_t)mg * p.ldr + row);
    nw = *(const float4 *)(norm_w + row);
    float4 w[4];
#pragma unroll
    for (int q = 0; q < 4; q++)
      if (q < n) w[q] = __ldcg((const float4 *)(pp + q * stride));
    float4 acc = w[0];
#pragma unroll
    for (int q = 1; q < 4; q++)
      if (q < n) {
        acc.x = acc.x + w[q].x; acc.y = acc.y + w[q].y; acc.z = acc.z + w[q].z; acc.w = acc.w + w[q].w;
      }
    for (int q = 4; q < n; q++) {  // more than four pieces: one round trip each
      const float4 x = __ldcg((const float4 *)(pp + q * stride));
      acc.x = acc.x + x.x; acc.y = acc.y + x.y; acc.z = acc.z + x.z; acc.w = acc.w + x.w;
    }
    v = make_float4(v.x + acc.x, v.y + acc.y, v.z + acc.z, v.w + acc.w);
    *(float4 *)(p.y + (size_t)mg * p.ldy + row) = v;
    const double a = v.x, b = v.y, cc = v.z, d = v.w;
    sq = __dadd_rn(sq, __dmul_rn(a, a));
    sq = __dadd_rn(sq, __dmul_rn(b, b));
    sq = __dadd_rn(sq, __dmul_rn(cc, cc));
    sq = __dadd_rn(sq, __dmul_rn(d, d));
  }
  // The next GEMM's CTAs start streaming weights once every block triggers: after this block's loads
  // (triggering at entry measured slower: the weight stream delays these loads).
  pdl_trigger();
  double inv = 0.0;
  if (m < mb) {  // uniform over the cluster (one row)
    const double bs = block_sum_double(sq, s_scratch);
    if (threadIdx.x == 0) s_cta = bs;
    cluster_sync_all();  // every CTA's sum is in its shared memory
    if (threadIdx.x == 0) {
      double total = 0.0;
      const uint32_t a = smem_u32(&s_cta);
      for (int r = 0; r < SK_NORM_CTAS; r++) total += ld_cluster_f64(map_to_rank(a, (uint32_t)r));
      s_total = total;
    }
    cluster_sync_all();  // no CTA leaves while its sum may still be read; s_total visible in the CTA
    inv = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(s_total, (double)N), eps)));
  }
  if (c >= n4) return;
  const float f[4] = {v.x, v.y, v.z, v.w}, nws[4] = {nw.x, nw.y, nw.z, nw.w};
  uint16_t h[3][4];
#pragma unroll
  for (int e = 0; e < 4; e++) {
    const float g = m < mb ? __double2float_rn(__dmul_rn(__dmul_rn((double)f[e], inv), (double)nws[e])) : 0.0f;
    split3_bf16(g, h[0][e], h[1][e], h[2][e]);
  }
#pragma unroll
  for (int tm = 0; tm < 3; tm++) {
    uint2 u;
    u.x = (uint32_t)h[tm][0] | ((uint32_t)h[tm][1] << 16);
    u.y = (uint32_t)h[tm][2] | ((uint32_t)h[tm][3] << 16);
    *(uint2 *)(x3n + ((size_t)tm * NT + m) * N + 4 * c) = u;
  }
}

uint32_t skinny_idesc(int nt) {
  // D = F32, A = B = BF16, both K-major, N = 3 NT (>> 3 at bits 17-22), M = 128 (>> 4 at bits 24-28)
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)((3 * nt) >> 3) << 17) | ((uint32_t)(SK_BM >> 4) << 24);
}

struct SkinnyPlan {
  int nt, tiles, kbs, grid, pmax;
  long long iters;
  uint64_t x3_bytes, part_bytes;
};

SkinnyPlan skinny_plan(int M, int N, int K, int device) {
  SkinnyPlan q;
  q.nt = skinny_nt(M);
  q.tiles = (N + SK_BM - 1) / SK_BM;
  q.kbs = (K + BK - 1) / BK;
  q.iters = (long long)q.tiles * q.kbs;
  const int per_sm = q.nt == 16 ? SkinnyShape<16>::CTAS_PER_SM
                                : (q.nt == 32 ? SkinnyShape<32>::CTAS_PER_SM : SkinnyShape<64>::CTAS_PER_SM);
  q.grid = (int)std::min<long long>((long long)per_sm * sm_count(device), q.iters);
  const long long per = q.iters / q.grid;  // every range holds per or per + 1 iterations
  q.pmax = (int)std::min<long long>(q.grid, (q.kbs + per - 1) / per + 1);
  q.x3_bytes = ((uint64_t)3 * q.nt * K * 2 + 255) & ~255ull;
  q.part_bytes = (uint64_t)q.tiles * q.pmax * M * SK_BM * 4;
  return q;
}

template <int NT>
void configure(int device) {
  static std::mutex mu;
  static bool configured[64] = {};
  std::lock_guard<std::mutex> lock(mu);
  if (device < 0 || device >= 64 || !configured[device]) {
    STB_CUDA(cudaFuncSetAttribute(gemm_skinny_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  SkinnyShape<NT>::SMEM));
    if (device >= 0 && device < 64) configured[device] = true;
  }
}

template <int NT>
void launch_gemm(const SkinnyPlan &q, const CUtensorMap &tw, const CUtensorMap &tx, float *part, int M, int N,
                 int *err, int device, cudaStream_t stream) {
  configure<NT>(device);
  launch_kernel(gemm_skinny_kernel<NT>, dim3(q.grid), dim3(192), (size_t)SkinnyShape<NT>::SMEM, stream, true, tw, tx,
                part, M, N, q.kbs, q.iters, q.pmax, skinny_idesc(NT), err);
}

}  // namespace

bool skinny_eligible(int M, int N, int K, int w_dtype, const void *w) {
  static const int enabled = env_int("STB_SKINNY", 1);
  // One row too: above the work threshold the form streams weights faster than the SIMT GEMV even for
  // a single token (70B gate/up shard at M = 1: 146 us here, 160 us on the GEMV; the 70B-shaped
  // batch-1 decode 42.7 vs 31.5 tok/s).
  static const int min_rows = env_int("STB_SKINNY_MIN_ROWS", 1);
  static const int max_rows = env_int("STB_SKINNY_MAX_ROWS", 1 << 30);
  // Below ~16M multiply-adds the three launches cost more than the SIMT GEMV's one (measured: the
  // single-Linear 16 x 1536 x 576 takes 12.3 us on the GEMV, 13.3 us here; 32 x 1536 x 576 takes
  // 18.4 us on the GEMV, 13.3 us here).
  static const int min_work = env_int("STB_SKINNY_MIN_WORK", 1 << 24);
  return enabled && w_dtype == STB_BF16 && M >= std::max(1, min_rows) && M <= max_rows && K % 8 == 0 && K >= BK &&
         N >= SK_BM && ((uintptr_t)w % 16) == 0 && (int64_t)M * N * K > (int64_t)min_work;
}

void skinny_prepare(int device) {
  configure<16>(device);
  configure<32>(device);
  configure<64>(device);
}

uint64_t skinny_scratch_bytes(int M, int N, int K, int device) {
  const SkinnyPlan q = skinny_plan(std::min(M, 64), N, K, device);  // one 64-row block at a time
  return q.x3_bytes + q.part_bytes;
}

int skinny_nt(int M) { return M <= 16 ? 16 : (M <= 32 ? 32 : 64); }

bool skinny_norm_fusable(int N) { return N % 4 == 0 && N <= SK_NORM_CTAS * SK_NORM_THREADS * 4; }

template <int EPI>
int skinny_launch(const GemvParams &p, void *scratch, uint64_t scratch_bytes, int *err, int device,
                  cudaStream_t stream, const uint16_t *x3_ready, const SkinnyNext *next, SkinnyParts *deferred) {
  STB_REQUIRE(p.M >= 1 && p.K % 8 == 0 && p.K >= BK && p.N >= SK_BM, "skinny Linear shape");
  STB_REQUIRE(!deferred || (p.M <= 64 && !next), "deferred fixup: one block, no fused next prologue");
  STB_REQUIRE(!x3_ready || (p.M <= 64 && p.norm_w == nullptr && ((uintptr_t)x3_ready % 16) == 0),
              "prepared skinny activations: one block, no norm");
  STB_REQUIRE(p.stop == nullptr, "skinny Linear takes no stop flag");
  STB_REQUIRE(scratch && ((uintptr_t)scratch % 256) == 0 && scratch_bytes >= skinny_scratch_bytes(p.M, p.N, p.K, device),
              "skinny Linear scratch too small");
  if (next) {
    STB_REQUIRE(p.M <= 64 && next->x3 && ((uintptr_t)next->x3 % 16) == 0, "fused next prologue: one block");
    STB_REQUIRE((EPI == EPI_SILU && p.N % 8 == 0) ||
                    (EPI == EPI_RESID && next->norm_w && skinny_norm_fusable(p.N) && p.ldy % 4 == 0 && p.ldr % 4 == 0),
                "fused next prologue: SiLU split (N a multiple of 8), or residual + RMSNorm on rows of at most 8192 "
                "values");
  }
  const CUtensorMap tw = make_map(p.w, STB_BF16, (uint64_t)p.N, (uint64_t)p.K, SK_BM);
  constexpr bool paired = EPI == EPI_SILU || EPI == EPI_QKV;
  const int units = paired ? p.N / 2 : p.N;
  int launches = 0;
  // blocks of up to 64 token rows, in order, through the same scratch (each block's prologue waits
  // for the previous block's fixup)
  for (int m0 = 0; m0 < p.M; m0 += 64) {
    const int mb = std::min(64, p.M - m0);
    const SkinnyPlan q = skinny_plan(mb, p.N, p.K, device);
    const uint16_t *x3 = x3_ready ? x3_ready : (const uint16_t *)scratch;
    float *part = (float *)((char *)scratch + q.x3_bytes);
    if (!x3_ready)
      launch_kernel(skinny_prep_kernel, dim3((p.K + 1023) / 1024, q.nt), dim3(256), 0, stream, m0 > 0 || p.pdl,
                    p.x + (size_t)m0 * p.ldx, p.ldx, p.norm_w, p.norm_eps, (uint16_t *)scratch, mb, q.nt, p.K);
    const CUtensorMap tx = make_map(x3, STB_BF16, (uint64_t)3 * q.nt, (uint64_t)p.K, 3 * q.nt);
    if (q.nt == 16) launch_gemm<16>(q, tw, tx, part, mb, p.N, err, device, stream);
    else if (q.nt == 32) launch_gemm<32>(q, tw, tx, part, mb, p.N, err, device, stream);
    else launch_gemm<64>(q, tw, tx, part, mb, p.N, err, device, stream);
    if (deferred) {  // the consumer adds the pieces itself
      deferred->part = part;
      deferred->kbs = q.kbs;
      deferred->T = q.iters;
      deferred->G = q.grid;
      deferred->pmax = q.pmax;
      deferred->M = mb;
      launches += x3_ready ? 1 : 2;
      continue;
    }
    if (next && EPI == EPI_SILU)
      launch_kernel(skinny_fixup_silu_split_kernel, dim3((units / 4 + 255) / 256, q.nt), dim3(256), 0, stream, true,
                    (const float *)part, p.N, q.kbs, q.iters, q.grid, q.pmax, mb, next->x3, q.nt);
    else if (next)
      launch_kernel(skinny_fixup_norm_kernel, dim3(SK_NORM_CTAS, q.nt), dim3(SK_NORM_THREADS), 0, stream, true, p,
                    (const float *)part, q.kbs, q.iters, q.grid, q.pmax, mb, next->norm_w, next->eps, next->x3, q.nt);
    else
      launch_kernel(skinny_fixup_kernel<EPI>, dim3((units + 255) / 256, mb), dim3(256), 0, stream, true, p,
                    (const float *)part, q.kbs, q.iters, q.grid, q.pmax, m0, mb);
    launches += x3_ready ? 2 : 3;
  }
  check_launch("skinny");
  return launches;
}

template int skinny_launch<EPI_PLAIN>(const GemvParams &, void *, uint64_t, int *, int, cudaStream_t, const uint16_t *,
                                           const SkinnyNext *, SkinnyParts *);
template int skinny_launch<EPI_RESID>(const GemvParams &, void *, uint64_t, int *, int, cudaStream_t, const uint16_t *,
                                           const SkinnyNext *, SkinnyParts *);
template int skinny_launch<EPI_SILU>(const GemvParams &, void *, uint64_t, int *, int, cudaStream_t, const uint16_t *,
                                           const SkinnyNext *, SkinnyParts *);
template int skinny_launch<EPI_QKV>(const GemvParams &, void *, uint64_t, int *, int, cudaStream_t, const uint16_t *,
                                           const SkinnyNext *, SkinnyParts *);
template int skinny_launch<EPI_LOGITS>(const GemvParams &, void *, uint64_t, int *, int, cudaStream_t, const uint16_t *,
                                           const SkinnyNext *, SkinnyParts *);
template int skinny_launch<EPI_PEER>(const GemvParams &, void *, uint64_t, int *, int, cudaStream_t, const uint16_t *,
                                           const SkinnyNext *, SkinnyParts *);

}  // namespace stb
