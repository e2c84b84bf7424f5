// Prefill attention on the tcgen05 tensor cores, for prompt chunks that already run their
// projections on the tensor cores (chunks of at least tc_prefill_rows token rows, whose activations
// are rounded to the weight type: the prefill tolerance).
//
// The reference's causal grouped-query attention (cpu/src/main/scala/scalatorch/cpu/
// CpuAttention.scala:20-50: scores over the visible keys, softmax, weighted sum, in double) as a
// flash-attention tile loop: one CTA per (128 queries of one batch row, query head), 4 warps.
// Per 128-key tile of the head's KV group:
//   1. the 128 threads convert the Float32 K rows to BF16 (round to nearest even) into a K-major,
//      128-byte-swizzled shared-memory tile and the V rows, transposed, into a [hd][keys] tile --
//      the layouts a TMA SWIZZLE_128B load would produce, so the usual sm_100 descriptors apply;
//   2. one thread issues S = Q.K^T (tcgen05.mma.cta_group::1.kind::f16, M = 128, N = 128, K = hd)
//      into TMEM columns [0, 128);
//   3. each thread takes its query row of S from TMEM (tcgen05.ld), applies the causal mask
//      (key j visible to the query at position p iff j <= p) and the online softmax in Float32 (row
//      max, exp2 of the log2-scaled scores, running sum, rescale factor for earlier tiles), and
//      writes P rounded to BF16 over the K tile (already consumed by step 2);
//   4. one thread issues O += P.V (M = 128, N = hd, K = 128 keys) into the TMEM accumulator at
//      columns [128, 128 + hd).  Before that, a warp whose rows' running maximum moved rescales its
//      rows of O in place (tcgen05.ld, multiply by exp2(m_old - m_new), tcgen05.st).
// The output is O / sum in Float32.  Q, K, V and P are BF16 on the tensor cores (the tolerance
// source, as for the prefill projections); scores, softmax statistics and the output accumulate in
// FP32.  Shared memory: Q 128 x hd, K / P 128 x 128, V^T hd x 128 BF16 (96 KB at hd = 128, two CTAs
// per SM); TMEM: 256 columns.  Every wait on an MMA completion is bounded (2 s; then the session's
// error word is set, the kernel waits -- bounded again -- for the MMAs it issued and frees TMEM).
// No TMA and no cross-CTA sharing: each CTA reads the Float32 cache rows it needs itself.
#include "tc_common.cuh"

namespace stb {

namespace {

using namespace tc;

constexpr int AT_Q = 128, AT_K = 128, AT_THREADS = 128;
constexpr int AT_SMEM_FLOOR = 100 * 1024;  // at most two CTAs per SM (TMEM: 2 x 256 columns of 512)

template <int HD>
struct AttnTcShape {
  static constexpr int Q_BYTES = AT_Q * HD * 2;            // [128 q][hd]: hd / 64 subtiles of 16 KB
  static constexpr int KP_BYTES = AT_K * 128 * 2;          // K [128 keys][hd <= 128] or P [128 q][128 keys]
  static constexpr int V_BYTES = HD * AT_K * 2;            // V^T [hd][128 keys]: 2 subtiles of hd x 128 B
  static constexpr int SMEM_USED = Q_BYTES + KP_BYTES + V_BYTES + 1024 + 64;
  static constexpr int SMEM = SMEM_USED > AT_SMEM_FLOOR ? SMEM_USED : AT_SMEM_FLOOR;
  static_assert(SMEM <= 232448, "shared memory");
};

// Byte offset of the 16-byte chunk `c` (of 8 BF16 along K) of row `r` in a K-major, 128-byte
// swizzled tile: rows of 128 bytes, the chunk index XOR-ed with r mod 8 (TMA's SWIZZLE_128B).
__device__ __forceinline__ uint32_t swz(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  return (uint32_t)f32_to_bf16_rne(a) | ((uint32_t)f32_to_bf16_rne(b) << 16);
}

// Plain (compiler-visible) shared-memory store: the compiler may keep the next global loads in flight
// across it; the fences and barriers that publish the tiles to the tensor cores order it.
__device__ __forceinline__ void st_shared_v4(uint8_t *base, uint32_t off, uint4 v) {
  *reinterpret_cast<uint4 *>(base + off) = v;
}

// Stores 32 consecutive TMEM columns of this thread's lane (the inverse of tmem_ld32) and waits.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

template <int HD>
__global__ void __launch_bounds__(AT_THREADS, 2)
    flash_tc_kernel(const float *q, int ldq, const float *kcache, const float *vcache, float *out, int ldo, int count,
                    int nh, int kvh, int capacity, const int *pos_dev, int pos0, uint32_t idesc_s, uint32_t idesc_o,
                    int *err, uint16_t *out_half, int half_bf16) {
  static_assert(HD == 64 || HD == 128, "head size");
  using S = AttnTcShape<HD>;
  extern __shared__ uint8_t at_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)at_raw + 1023) & ~(uintptr_t)1023);
  uint8_t *qp = smem, *kp = smem + S::Q_BYTES, *vp = kp + S::KP_BYTES;  // generic pointers of the tiles
  const uint32_t qs = smem_u32(qp), kps = smem_u32(kp), vs = smem_u32(vp);
  uint64_t *bars = (uint64_t *)(smem + S::Q_BYTES + S::KP_BYTES + S::V_BYTES);
  const uint32_t bar = smem_u32(bars);
  uint32_t *tmem_slot = (uint32_t *)(bars + 1);
  __shared__ volatile int s_abort;
  __shared__ int s_ok;

  const int tid = threadIdx.x, warp = tid >> 5;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int g = h / (nh / kvh);
  const int base = pos_dev ? *pos_dev : pos0;
  const int t0 = qt * AT_Q;
  const int nq = min(AT_Q, count - t0);
  const int nkeys = base + t0 + nq;  // keys 0 .. position of the tile's last query
  const int ntiles = (nkeys + AT_K - 1) / AT_K;
  const float *kb = kcache + ((size_t)b * kvh + g) * capacity * HD;
  const float *vb = vcache + ((size_t)b * kvh + g) * capacity * HD;

  if (tid == 0) {
    s_abort = 0;
    mbar_init(bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(256)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // Q tile -> BF16, K-major swizzled (rows past the chunk are zero)
  for (int i = tid; i < AT_Q * (HD / 8); i += AT_THREADS) {
    const int r = i / (HD / 8), ch = i % (HD / 8);
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f), c = a;
    if (r < nq) {
      const float *src = q + ((size_t)b * count + t0 + r) * ldq + (size_t)h * HD + ch * 8;
      a = *reinterpret_cast<const float4 *>(src);
      c = *reinterpret_cast<const float4 *>(src + 4);
    }
    st_shared_v4(qp, (ch >> 3) * 16384 + swz(r, ch & 7),
                 make_uint4(pack_bf16(a.x, a.y), pack_bf16(a.z, a.w), pack_bf16(c.x, c.y), pack_bf16(c.z, c.w)));
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t row_tmem = tmem + ((uint32_t)(warp * 32) << 16);

  const int r = tid;                      // this thread's query row of the tile
  const int qpos = base + t0 + r;         // its absolute position
  const bool row_valid = r < nq;
  const float scale_log2 = (float)(1.4426950408889634 / sqrt((double)HD));
  float m_run = -INFINITY, l_run = 0.0f;
  uint32_t phase = 0;
  bool ok = true;
  int issued = 0;

  for (int kt = 0; kt < ntiles && ok; kt++) {
    const int j0 = kt * AT_K;
    // 1. K -> BF16 [keys][hd] and V -> BF16 V^T [hd][keys] (keys past the visible range are zero)
#pragma unroll 4
    for (int i = tid; i < AT_K * (HD / 8); i += AT_THREADS) {
      const int kr = i / (HD / 8), ch = i % (HD / 8);
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f), c = a;
      if (j0 + kr < nkeys) {
        const float *src = kb + (size_t)(j0 + kr) * HD + ch * 8;
        a = *reinterpret_cast<const float4 *>(src);
        c = *reinterpret_cast<const float4 *>(src + 4);
      }
      st_shared_v4(kp, (ch >> 3) * 16384 + swz(kr, ch & 7),
                   make_uint4(pack_bf16(a.x, a.y), pack_bf16(a.z, a.w), pack_bf16(c.x, c.y), pack_bf16(c.z, c.w)));
    }
    for (int i = tid; i < (HD / 4) * (AT_K / 8); i += AT_THREADS) {
      const int dq = i % (HD / 4), kg = i / (HD / 4);  // dimensions 4 dq .. 4 dq + 3, keys 8 kg .. 8 kg + 7
      float v[8][4];
#pragma unroll
      for (int e = 0; e < 8; e++) {
        float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
        if (j0 + kg * 8 + e < nkeys) x = *reinterpret_cast<const float4 *>(vb + (size_t)(j0 + kg * 8 + e) * HD + dq * 4);
        v[e][0] = x.x;
        v[e][1] = x.y;
        v[e][2] = x.z;
        v[e][3] = x.w;
      }
#pragma unroll
      for (int dd = 0; dd < 4; dd++) {
        const int d = dq * 4 + dd;
        st_shared_v4(vp, (kg >> 3) * (HD * 128) + swz(d, kg & 7),
                     make_uint4(pack_bf16(v[0][dd], v[1][dd]), pack_bf16(v[2][dd], v[3][dd]),
                                pack_bf16(v[4][dd], v[5][dd]), pack_bf16(v[6][dd], v[7][dd])));
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    // 2. S = Q . K^T
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < HD / 16; kk++) {
        const uint64_t a = smem_desc(qs + (kk >> 2) * 16384) + (uint64_t)(2 * (kk & 3));
        const uint64_t bdesc = smem_desc(kps + (kk >> 2) * 16384) + (uint64_t)(2 * (kk & 3));
        mma_f16(tmem, a, bdesc, idesc_s, kk != 0);
      }
      mma_commit(bar);
      issued++;
    }
    if (tid == 0) s_ok = mbar_wait(bar, phase, &s_abort, err, 50);
    __syncthreads();
    if (!s_ok) {
      ok = false;
      break;
    }
    phase ^= 1;
    tc_fence_after();
    // 3. online softmax of this row; P (BF16) over the K tile
    float mx = -INFINITY;
#pragma unroll
    for (int c = 0; c < AT_K / 32; c++) {
      uint32_t sr[32];
      tmem_ld32(row_tmem + (uint32_t)(c * 32), sr);
#pragma unroll
      for (int jj = 0; jj < 32; jj++) {
        const int j = j0 + c * 32 + jj;
        if (row_valid && j <= qpos && j < nkeys) mx = fmaxf(mx, __uint_as_float(sr[jj]) * scale_log2);
      }
    }
    const float m_new = fmaxf(m_run, mx);
    const float alpha = m_new == -INFINITY ? 1.0f : exp2f(m_run - m_new);
    float sum = 0.0f;
#pragma unroll
    for (int c = 0; c < AT_K / 32; c++) {
      uint32_t sr[32];
      tmem_ld32(row_tmem + (uint32_t)(c * 32), sr);
      float p[32];
#pragma unroll
      for (int jj = 0; jj < 32; jj++) {
        const int j = j0 + c * 32 + jj;
        const bool vis = row_valid && j <= qpos && j < nkeys;
        p[jj] = vis ? exp2f(__uint_as_float(sr[jj]) * scale_log2 - m_new) : 0.0f;
        sum += p[jj];
      }
      // keys c * 32 .. c * 32 + 31 of P: subtile (c >> 1), chunks 4 (c & 1) .. 4 (c & 1) + 3
#pragma unroll
      for (int k8 = 0; k8 < 4; k8++)
        st_shared_v4(kp, (c >> 1) * 16384 + swz(r, (c & 1) * 4 + k8),
                     make_uint4(pack_bf16(p[8 * k8], p[8 * k8 + 1]), pack_bf16(p[8 * k8 + 2], p[8 * k8 + 3]),
                                pack_bf16(p[8 * k8 + 4], p[8 * k8 + 5]), pack_bf16(p[8 * k8 + 6], p[8 * k8 + 7])));
    }
    l_run = l_run * alpha + sum;
    m_run = m_new;
    // rows whose maximum moved: O (the earlier tiles' P.V) scaled by alpha in TMEM, warp by warp
    if (kt > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll
      for (int c = 0; c < HD / 32; c++) {
        uint32_t orr[32];
        tmem_ld32(row_tmem + 128 + (uint32_t)(c * 32), orr);
#pragma unroll
        for (int jj = 0; jj < 32; jj++) orr[jj] = __float_as_uint(__uint_as_float(orr[jj]) * alpha);
        tmem_st32(row_tmem + 128 + (uint32_t)(c * 32), orr);
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    // 4. O += P . V
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < AT_K / 16; kk++) {
        const uint64_t a = smem_desc(kps + (kk >> 2) * 16384) + (uint64_t)(2 * (kk & 3));
        const uint64_t bdesc = smem_desc(vs + (kk >> 2) * (HD * 128)) + (uint64_t)(2 * (kk & 3));
        mma_f16(tmem + 128, a, bdesc, idesc_o, (kt | kk) != 0);
      }
      mma_commit(bar);
      issued++;
    }
    if (tid == 0) s_ok = mbar_wait(bar, phase, &s_abort, err, 51);
    __syncthreads();
    if (!s_ok) {
      ok = false;
      break;
    }
    phase ^= 1;
    tc_fence_after();  // the next tile overwrites K / P and V only after this tile's MMAs are done
  }
  if (!ok && tid == 0 && issued) {  // a wait expired: let the issued MMAs finish before TMEM is freed
    volatile int no_abort = 0;
    mbar_wait(bar, phase, &no_abort, err, 52);
  }
  if (ok) {
    const size_t off = ((size_t)b * count + t0 + r) * ldo + (size_t)h * HD;
    const float inv = row_valid ? 1.0f / l_run : 0.0f;
#pragma unroll
    for (int c = 0; c < HD / 32; c++) {
      uint32_t orr[32];
      tmem_ld32(row_tmem + 128 + (uint32_t)(c * 32), orr);
      if (!row_valid) continue;
      if (out_half) {  // the o projection's operand, rounded to the weight type (Float32 first, then half)
        uint16_t *dst = out_half + off + c * 32;
#pragma unroll
        for (int jj = 0; jj < 32; jj += 8) {
          uint32_t w4[4];
#pragma unroll
          for (int e = 0; e < 4; e++) {
            const float a = __uint_as_float(orr[jj + 2 * e]) * inv, bb = __uint_as_float(orr[jj + 2 * e + 1]) * inv;
            w4[e] = half_bf16 ? pack_bf16(a, bb)
                              : (uint32_t)__half_as_ushort(__float2half_rn(a)) |
                                    ((uint32_t)__half_as_ushort(__float2half_rn(bb)) << 16);
          }
          *reinterpret_cast<uint4 *>(dst + jj) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
        }
      } else {
        float *dst = out + off + c * 32;
#pragma unroll
        for (int jj = 0; jj < 32; jj += 4)
          *reinterpret_cast<float4 *>(dst + jj) =
              make_float4(__uint_as_float(orr[jj]) * inv, __uint_as_float(orr[jj + 1]) * inv,
                          __uint_as_float(orr[jj + 2]) * inv, __uint_as_float(orr[jj + 3]) * inv);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256) : "memory");
}

// kind::f16 instruction descriptor: D = F32, A = B = BF16, both K-major, N >> 3 at bits 17-22,
// M >> 4 at bits 24-28.
uint32_t at_idesc(int n) { return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(AT_Q >> 4) << 24); }

template <int HD>
void at_launch(dim3 grid, const float *q, int ldq, const float *kc, const float *vc, float *out, int ldo, int count,
               int nh, int kvh, int capacity, const int *posd, int pos0, int *err, int device, cudaStream_t st,
               uint16_t *out_half, int half_bf16) {
  static std::mutex mu;
  static bool configured[64] = {};
  {
    std::lock_guard<std::mutex> lock(mu);
    if (device < 0 || device >= 64 || !configured[device]) {
      STB_CUDA(cudaFuncSetAttribute(flash_tc_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    AttnTcShape<HD>::SMEM));
      if (device >= 0 && device < 64) configured[device] = true;
    }
  }
  launch_kernel(flash_tc_kernel<HD>, grid, dim3(AT_THREADS), (size_t)AttnTcShape<HD>::SMEM, st, false, q, ldq, kc, vc,
                out, ldo, count, nh, kvh, capacity, posd, pos0, at_idesc(128), at_idesc(HD), err, out_half, half_bf16);
}

}  // namespace

// Launches the tensor-core prefill attention for head sizes 64 and 128 (STB_TC_ATTENTION=0 keeps the
// FP32 tiled kernel); returns false when it does not apply.  q rows are (batch row, token) with
// `count` tokens per batch row; the chunk's keys are already in the cache.  With out_half the output
// goes there in half_dtype (STB_BF16 / STB_F16) -- the next tensor-core GEMM's operand -- instead of
// Float32 to out.
bool launch_flash_attention_tc(const float *q, int ldq, const float *kc, const float *vc, float *out, int ldo,
                               int rows, int count, int nh, int kvh, int hd, int capacity, const int *posd, int pos0,
                               int *err, int device, cudaStream_t st, uint16_t *out_half, int half_dtype) {
  static const int enabled = env_int("STB_TC_ATTENTION", 1);
  if (!enabled || rows % count != 0 || nh % kvh != 0 || (ldq % 4) != 0 || (ldo % 8) != 0) return false;
  const dim3 grid((count + AT_Q - 1) / AT_Q, nh, rows / count);
  const int bf = half_dtype == STB_BF16 ? 1 : 0;
  if (hd == 128)
    at_launch<128>(grid, q, ldq, kc, vc, out, ldo, count, nh, kvh, capacity, posd, pos0, err, device, st, out_half, bf);
  else if (hd == 64)
    at_launch<64>(grid, q, ldq, kc, vc, out, ldo, count, nh, kvh, capacity, posd, pos0, err, device, st, out_half, bf);
  else
    return false;
  return true;
}

}  // namespace stb
