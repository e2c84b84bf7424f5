// Single-token (decode) attention for head size 128 and grouped-query groups of up to 8 query
// heads, as a stream through shared memory, and the split merge fused into the next projection's
// prologue.
//
// The reference's causal grouped-query attention (cpu/src/main/scala/scalatorch/cpu/
// CpuAttention.scala:20-50) for one new token per batch row: scores of the query against every
// visible key, softmax, weighted sum of the values.  On the GPU each (batch row, KV head) pair's
// visible keys are cut into splits of `kps` keys (a multiple of 8, chosen from the cache capacity
// so that about two blocks per SM cover all pairs: every block is resident at once, no second
// wave).  Block (split, KV head, row), 256 threads, streams its split's K rows and then its V rows
// in chunks of 32 keys (16 KB) through a 5-stage ring:
//   * K chunks: four 2-D TMA box loads (32 dims x 32 keys of Float32, 128-byte swizzle) from one
//     tensor map over the whole cache; V chunks: one bulk copy of the contiguous rows.  The first
//     five chunks are issued before the programmatic-dependency wait (the cache rows of earlier
//     steps never depend on the previous kernel); the newest key, which the QKV projection just
//     wrote, is patched into its chunk from global memory after the wait.
//   * scores: lane (key k, head quad h4) computes the dot of key k with query heads 4 h4 .. 4 h4 + 3
//     over its warp's share of the dimensions (16 FMAs per 128-bit K load; the swizzle puts the keys
//     a warp reads in distinct banks; the query rows are broadcast reads); the shares are added in
//     order through shared memory.  Groups of more than 4 heads take two head quads per key (16
//     keys x 2 quads per warp, 4 dimension shares); smaller groups one (32 keys, 8 shares).
//   * after the last K chunk: softmax statistics per head over the split (max, exp, sum), a warp
//     per head;
//   * V chunks: warp w owns output dimensions 32 (w mod 4) .. + 31 of every head over the keys of
//     parity w / 4, with 8 accumulators per lane; the two parities are added at the end.
// The per-warp work is short chains of shared-memory loads and FMAs, so the block has 8 warps (16
// per SM) to hide their latency.  Each block writes its split's unnormalised sums and (max, sum) per
// head.  The merge (rescale every split by exp(max_s - max), sum in split order, divide) runs in
// attention_merge_split_kernel, which is the o projection's prologue: it writes the three BF16 terms
// of the merged output that the skinny GEMM reads (or the Float32 output for the other forms of the
// projection).  Every mbarrier wait is bounded (2 s; then the session's error word is set, the block
// waits -- bounded again -- for the copies it issued, and leaves without writing).
#include "attention_decode.cuh"
#include "gemv.cuh"
#include "tc_common.cuh"

namespace stb {

namespace {

using namespace tc;

constexpr int DS_HD = 128, DS_CH = 32, DS_RING = 5, DS_THREADS = 256, DS_WARPS = DS_THREADS / 32, DS_GMAX = 8,
              DS_KPS_MAX = 256;
constexpr int DS_CHUNK = DS_CH * DS_HD * 4;  // 16 KB: 32 K rows (4 swizzled boxes of 4 KB) or V rows
constexpr int DS_QROW = 132;                 // padded query row (floats)
constexpr int DS_SHARES = 8;                 // dimension shares of the scores (at most)
constexpr size_t DS_SMEM = 1024 + (size_t)DS_RING * DS_CHUNK + DS_GMAX * DS_QROW * 4 +
                           (size_t)DS_SHARES * DS_CH * DS_GMAX * 4 + (size_t)DS_KPS_MAX * DS_GMAX * 4 +
                           DS_GMAX * 2 * 4 + DS_RING * 8;

// Byte offset of float d of key row r inside a K chunk: box d / 32 (4 KB), row r (128 bytes), 16-byte
// chunk (d % 32) / 4 XOR-ed with r mod 8 (TMA's SWIZZLE_128B on a 1024-byte-aligned box).
__device__ __forceinline__ uint32_t ds_koff(int r, int d) {
  return (uint32_t)((d >> 5) * 4096 + r * 128 + ((((d & 31) >> 2) ^ (r & 7)) << 4) + (d & 3) * 4);
}

// Partial scores of key `sk` against query heads 4 sq .. 4 sq + 3 over dimensions [d0, d0 + DLEN).
template <int DLEN>
__device__ __forceinline__ float4 ds_scores(const uint8_t *chunk, const float *Qs, int sk, int sq, int d0) {
  float s4[4] = {0.f, 0.f, 0.f, 0.f};
  const float *qr = Qs + 4 * sq * DS_QROW + d0;
  const uint8_t *kr = chunk + (d0 >> 5) * 4096 + sk * 128;
  const int rx = sk & 7, c0 = (d0 & 31) >> 2;
#pragma unroll
  for (int i = 0; i < DLEN / 4; i++) {
    const int cc = c0 + i;  // 16-byte chunk along the dimensions (boxes of 8 chunks)
    const float4 kv = *(const float4 *)(kr + (cc >> 3) * 4096 + (((cc & 7) ^ rx) << 4));
#pragma unroll
    for (int h = 0; h < 4; h++) {
      const float4 qv = *(const float4 *)(qr + h * DS_QROW + 4 * i);
      s4[h] = fmaf(qv.x, kv.x, s4[h]);
      s4[h] = fmaf(qv.y, kv.y, s4[h]);
      s4[h] = fmaf(qv.z, kv.z, s4[h]);
      s4[h] = fmaf(qv.w, kv.w, s4[h]);
    }
  }
  return make_float4(s4[0], s4[1], s4[2], s4[3]);
}

// TWOQ: more than 4 query heads per KV head (two head quads per key).
template <bool TWOQ>
__global__ void __launch_bounds__(DS_THREADS, 2) decode_attention_stream_kernel(
    const __grid_constant__ CUtensorMap kmap, long long krow0, const float *q, int ldq, const float *kcache,
    const float *vcache, int count, int nh, int kvh, int capacity, const int *pos_dev, int pos0, int kps,
    float *part, int smax, int *err) {
  extern __shared__ uint8_t ds_raw[];
  uint8_t *ring = (uint8_t *)(((uintptr_t)ds_raw + 1023) & ~(uintptr_t)1023);
  float *Qs = (float *)(ring + DS_RING * DS_CHUNK);  // [8][DS_QROW]
  float *pscr = Qs + DS_GMAX * DS_QROW;              // [dimension shares][32 keys][8 heads]; V parity sums
  float *pt = pscr + DS_SHARES * DS_CH * DS_GMAX;    // [kps][8]: scores, then exp(score - max)
  float *red = pt + DS_KPS_MAX * DS_GMAX;            // [8][2]: max, sum
  uint64_t *bar = (uint64_t *)(red + DS_GMAX * 2);   // [DS_RING]
  __shared__ int s_ok;
  __shared__ volatile int s_abort;
  pdl_trigger();
  const int split = blockIdx.x, g0 = blockIdx.y, m = blockIdx.z;
  const int G = nh / kvh;
  const int b = m / count, t = m % count;
  const int keys = (pos_dev ? *pos_dev : pos0) + t + 1;
  const int S = (keys + kps - 1) / kps;
  if (split >= S) return;  // the grid covers the longest visible range
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int j0 = split * kps, nk = min(kps, keys - j0);
  const int nck = (nk + DS_CH - 1) / DS_CH, total = 2 * nck;  // K chunks, then V chunks
  const int fresh = keys - 1 - j0;                              // in [0, nk) only in the last split
  const long long kvrow0 = ((long long)b * kvh + g0) * capacity + j0;
  const uint32_t ring_a = smem_u32(ring), bar0 = smem_u32(bar);
  int issued = 0;  // thread 0: chunks whose loads are issued
  auto issue = [&](int c) {
    const int st = c % DS_RING;
    const uint32_t dst = ring_a + st * DS_CHUNK, br = bar0 + 8 * st;
    if (c < nck) {
      mbar_expect_tx(br, DS_CHUNK);
      const int y = (int)(krow0 + kvrow0 + (long long)c * DS_CH);
#pragma unroll
      for (int bx = 0; bx < 4; bx++) tma_load_2d(dst + bx * 4096, &kmap, bx * 32, y, br);
    } else {
      const int cv = c - nck, rows = min(DS_CH, nk - cv * DS_CH);
      const uint32_t bytes = (uint32_t)rows * DS_HD * 4;
      mbar_expect_tx(br, bytes);
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                   "l"(vcache + (kvrow0 + (long long)cv * DS_CH) * DS_HD), "r"(bytes), "r"(br)
                   : "memory");
    }
  };
  if (tid == 0) {
    s_abort = 0;
    for (int st = 0; st < DS_RING; st++) mbar_init(bar0 + 8 * st, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (; issued < min(DS_RING, total); issued++) issue(issued);
  }
  pdl_wait();
  {  // the group's query rows (zero past G): one float4 per thread
    const int g = tid / (DS_HD / 4), d4 = tid % (DS_HD / 4);
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (g < G) v = *(const float4 *)(q + (size_t)m * ldq + (size_t)(g0 * G + g) * DS_HD + d4 * 4);
    *(float4 *)(Qs + g * DS_QROW + d4 * 4) = v;
  }
  // the newest key's row, loaded now (after the wait) and stored once its chunk has landed
  const bool patch = fresh < nk && tid < DS_HD;
  const float kf = patch ? kcache[(kvrow0 + fresh) * DS_HD + tid] : 0.0f;
  const float vf = patch ? vcache[(kvrow0 + fresh) * DS_HD + tid] : 0.0f;
  const float scale = (float)(1.0 / sqrt((double)DS_HD));
  constexpr int NSH = TWOQ ? 4 : 8, DLEN = DS_HD / NSH;
  const int sk = TWOQ ? (warp & 1) * 16 + (lane & 15) : lane;  // key of this lane in a chunk
  const int sq = TWOQ ? lane >> 4 : 0;                          // head quad
  const int dsh = TWOQ ? warp >> 1 : warp;                      // dimension share
  float acc[DS_GMAX];
#pragma unroll
  for (int g = 0; g < DS_GMAX; g++) acc[g] = 0.0f;
  const int d = (warp & 3) * 32 + lane, par = warp >> 2;  // V phase: output dimension, key parity

  for (int c = 0; c < total; c++) {
    const int st = c % DS_RING;
    uint8_t *chunk = ring + st * DS_CHUNK;
    if (tid == 0) {
      s_ok = mbar_wait(bar0 + 8 * st, (uint32_t)(c / DS_RING) & 1u, &s_abort, err, 60);
      if (!s_ok) {  // leave only once every copy into this block's shared memory is done (bounded again)
        volatile int no_abort = 0;
        for (int cc = c; cc < issued; cc++)
          mbar_wait(bar0 + 8 * (cc % DS_RING), (uint32_t)(cc / DS_RING) & 1u, &no_abort, err, 61);
      }
    }
    __syncthreads();
    if (!s_ok) return;
    if (c < nck) {
      const int r = fresh - c * DS_CH;
      if (r >= 0 && r < DS_CH) {  // block-uniform
        if (tid < DS_HD) *(float *)(chunk + ds_koff(r, tid)) = kf;
        __syncthreads();
      }
      if (c * DS_CH + sk < nk)
        *(float4 *)(pscr + (dsh * DS_CH + sk) * DS_GMAX + 4 * sq) =
            ds_scores<DLEN>(chunk, Qs, sk, sq, dsh * DLEN);
      __syncthreads();
      {  // dimension shares added in order: one (key, head) per thread
        const int j = tid / DS_GMAX, g = tid % DS_GMAX;
        if (c * DS_CH + j < nk && g < G) {
          float sc = pscr[j * DS_GMAX + g];
#pragma unroll
          for (int sh = 1; sh < NSH; sh++) sc += pscr[(sh * DS_CH + j) * DS_GMAX + g];
          pt[(c * DS_CH + j) * DS_GMAX + g] = sc * scale;
        }
      }
      if (c == nck - 1) {  // all scores: softmax statistics of head `warp` over the split
        __syncthreads();
        const int g = warp;
        if (g < G) {
          float mx = -INFINITY;
          for (int j = lane; j < nk; j += 32) mx = fmaxf(mx, pt[j * DS_GMAX + g]);
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
          float sum = 0.0f;
          for (int j = lane; j < nk; j += 32) {
            const float e = expf(pt[j * DS_GMAX + g] - mx);
            pt[j * DS_GMAX + g] = e;
            sum += e;
          }
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
          if (lane == 0) {
            red[g * 2] = mx;
            red[g * 2 + 1] = sum;
          }
        }
      }
    } else {
      const int cv = c - nck, rows = min(DS_CH, nk - cv * DS_CH);
      const float *vt = (const float *)chunk;
      const int r = fresh - cv * DS_CH;
      if (r >= 0 && r < DS_CH) {  // block-uniform
        if (tid < DS_HD) ((float *)chunk)[r * DS_HD + tid] = vf;
        __syncthreads();
      }
      const float *pr = pt + (size_t)cv * DS_CH * DS_GMAX;
#pragma unroll 4
      for (int j = par; j < rows; j += 2) {
        const float v = vt[j * DS_HD + d];
        const float4 pa = *(const float4 *)(pr + j * DS_GMAX), pb = *(const float4 *)(pr + j * DS_GMAX + 4);
        acc[0] = fmaf(pa.x, v, acc[0]);
        acc[1] = fmaf(pa.y, v, acc[1]);
        acc[2] = fmaf(pa.z, v, acc[2]);
        acc[3] = fmaf(pa.w, v, acc[3]);
        acc[4] = fmaf(pb.x, v, acc[4]);
        acc[5] = fmaf(pb.y, v, acc[5]);
        acc[6] = fmaf(pb.z, v, acc[6]);
        acc[7] = fmaf(pb.w, v, acc[7]);
      }
    }
    __syncthreads();  // chunk consumed: its stage takes the chunk DS_RING ahead
    if (tid == 0 && issued < total) issue(issued++);
  }
  // odd-key sums (warps 4-7) onto the even-key sums (warps 0-3)
  if (par == 1) {
#pragma unroll
    for (int g = 0; g < DS_GMAX; g++) pscr[g * DS_HD + d] = acc[g];
  }
  __syncthreads();
  if (par == 1) return;
  const size_t slot = ((size_t)m * kvh + g0) * smax + split;
  float *po = part, *pml = part + (size_t)gridDim.z * kvh * smax * DS_GMAX * DS_HD;
#pragma unroll
  for (int g = 0; g < DS_GMAX; g++)
    if (g < G) po[(slot * DS_GMAX + g) * DS_HD + d] = acc[g] + pscr[g * DS_HD + d];
  if (tid < G) {
    pml[(slot * DS_GMAX + tid) * 2 + 0] = red[tid * 2];
    pml[(slot * DS_GMAX + tid) * 2 + 1] = red[tid * 2 + 1];
  }
}

// Sum of the stream-K pieces of 4 consecutive outputs (n0 % 4 == 0) of row m, in piece order.
__device__ __forceinline__ float4 ds_gather4(const DecodeStreamFused &fu, int m, int n0) {
  const int t = n0 >> 7;
  const int first = skinny_cta_of((long long)t * fu.kbs, fu.T, fu.G);
  const int n = skinny_cta_of((long long)(t + 1) * fu.kbs - 1, fu.T, fu.G) - first + 1;
  const float *pp = fu.part + ((size_t)t * fu.pmax * fu.M + m) * 128 + (n0 & 127);
  const size_t stride = (size_t)fu.M * 128;
  float4 w[4];
#pragma unroll
  for (int j = 0; j < 4; j++)
    if (j < n) w[j] = __ldcg((const float4 *)(pp + j * stride));
  float4 a = w[0];
#pragma unroll
  for (int j = 1; j < 4; j++)
    if (j < n) {
      a.x = a.x + w[j].x;
      a.y = a.y + w[j].y;
      a.z = a.z + w[j].z;
      a.w = a.w + w[j].w;
    }
  for (int j = 4; j < n; j++) {  // more than four pieces: one round trip each
    const float4 c = __ldcg((const float4 *)(pp + j * stride));
    a.x = a.x + c.x;
    a.y = a.y + c.y;
    a.z = a.z + c.z;
    a.w = a.w + c.w;
  }
  return a;
}

// The same for 2 consecutive outputs (n0 even).
__device__ __forceinline__ float2 ds_gather2(const DecodeStreamFused &fu, int m, int n0) {
  const int t = n0 >> 7;
  const int first = skinny_cta_of((long long)t * fu.kbs, fu.T, fu.G);
  const int n = skinny_cta_of((long long)(t + 1) * fu.kbs - 1, fu.T, fu.G) - first + 1;
  const float *pp = fu.part + ((size_t)t * fu.pmax * fu.M + m) * 128 + (n0 & 127);
  const size_t stride = (size_t)fu.M * 128;
  float2 w[4];
#pragma unroll
  for (int j = 0; j < 4; j++)
    if (j < n) w[j] = __ldcg((const float2 *)(pp + j * stride));
  float2 a = w[0];
#pragma unroll
  for (int j = 1; j < 4; j++)
    if (j < n) {
      a.x = a.x + w[j].x;
      a.y = a.y + w[j].y;
    }
  for (int j = 4; j < n; j++) {
    const float2 c = __ldcg((const float2 *)(pp + j * stride));
    a.x = a.x + c.x;
    a.y = a.y + c.y;
  }
  return a;
}

// Merge of the S split records of (row, KV head) at slot `base` for head g, dimensions d .. d + 3:
// max over splits, weights exp(max_s - max), numerator and denominator summed in split order.
__device__ __forceinline__ void ds_merge4(const float *po, const float *ml, size_t base, int S, int g, int d,
                                          float (&o)[4]) {
  float mx = -INFINITY;
  for (int s = 0; s < S; s++) mx = fmaxf(mx, __ldcg(&ml[((base + s) * DS_GMAX + g) * 2]));
  float num[4] = {0.f, 0.f, 0.f, 0.f}, den = 0.0f;
  for (int s0 = 0; s0 < S; s0 += 4) {  // four splits' loads per round trip
    float2 r[4];
    float4 v[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      if (s0 + j < S) {
        r[j] = __ldcg((const float2 *)&ml[((base + s0 + j) * DS_GMAX + g) * 2]);
        v[j] = __ldcg((const float4 *)&po[((base + s0 + j) * DS_GMAX + g) * DS_HD + d]);
      }
    }
#pragma unroll
    for (int j = 0; j < 4; j++) {
      if (s0 + j < S) {
        const float w = expf(r[j].x - mx);
        num[0] = fmaf(w, v[j].x, num[0]);
        num[1] = fmaf(w, v[j].y, num[1]);
        num[2] = fmaf(w, v[j].z, num[2]);
        num[3] = fmaf(w, v[j].w, num[3]);
        den = fmaf(w, r[j].y, den);
      }
    }
  }
#pragma unroll
  for (int e = 0; e < 4; e++) o[e] = num[e] / den;
}

// Groups of 5 to 8 query heads per KV head (the Llama-3-70B shape): the same blocks, ring and split
// records as decode_attention_stream_kernel, with the arithmetic laid out so that a chunk costs few
// shared-memory loads and no cross-warp reduction:
//   * scores: warp w takes keys 4 w .. 4 w + 3 of each K chunk; lane (head quad hq = lane / 16, dimension
//     group dg = lane % 16) keeps its 8 query dimensions of heads 4 hq .. 4 hq + 3 in registers (16-byte
//     chunk dg % 8 of boxes dg / 8 and dg / 8 + 2, the same 16 chunks of every key row: with the 128-byte
//     swizzle the 16 lanes of a quad read two whole 128-byte rows, no bank conflict), forms the 4 keys x
//     4 heads partial dots over them (8 K loads, 128 FMAs), and one reduce-scatter butterfly over the 16
//     lanes of its quad (15 shuffles) leaves lane dg with the whole dot of key dg / 4 and head dg % 4;
//   * softmax statistics per head over the split, as before;
//   * weighted V sum: warp w takes the same 4 keys of each V chunk, lane l owns dimensions 4 l .. 4 l + 3
//     of all 8 heads (32 accumulators; one 16-byte V load and two broadcast loads of the 8 weights per
//     key), and the 8 warps' sums are added in warp order at the end through the (then idle) ring.
constexpr size_t DS8_SMEM = 1024 + (size_t)DS_RING * DS_CHUNK + (size_t)DS_KPS_MAX * DS_GMAX * 4 +
                            DS_GMAX * 2 * 4 + (size_t)(DS_GMAX + 2) * DS_HD * 4 + 2 * DS_RING * 8;
static_assert(DS_RING * DS_CHUNK >= DS_WARPS * DS_GMAX * DS_HD * 4, "the ring holds the warps' value sums");

// FUSED: the QKV projection's fixup and the split merge happen here too (see DecodeStreamFused): q, and
// in the block holding the newest key its k (rotated) and v, are summed from the projection's stream-K
// pieces right after the dependency wait, the newest k / v row is written to the cache, and the last
// block of each (row, KV head) to finish merges the splits' records as attention_merge_split_kernel does.
template <bool FUSED>
__global__ void __launch_bounds__(DS_THREADS, 2) decode_attention_stream_g8_kernel(
    const __grid_constant__ CUtensorMap kmap, long long krow0, const float *q, int ldq, float *kcache, float *vcache,
    int count, int nh, int kvh, int capacity, const int *pos_dev, int pos0, int kps, float *part, int smax, int *err,
    const DecodeStreamFused fu) {
  extern __shared__ uint8_t ds_raw[];
  uint8_t *ring = (uint8_t *)(((uintptr_t)ds_raw + 1023) & ~(uintptr_t)1023);
  float *pt = (float *)(ring + DS_RING * DS_CHUNK);  // [kps][8]: scores, then exp(score - max)
  float *red = pt + DS_KPS_MAX * DS_GMAX;            // [8][2]: max, sum
  float *Qs = red + DS_GMAX * 2;                     // FUSED: [8][128] query rows, then the newest k and v rows
  uint64_t *bar = (uint64_t *)(Qs + (DS_GMAX + 2) * DS_HD);  // [DS_RING] full, then [DS_RING] empty
  __shared__ int s_last;
  __shared__ volatile int s_abort;
  pdl_trigger();
  const int split = blockIdx.x, g0 = blockIdx.y, m = blockIdx.z;
  const int G = nh / kvh;
  const int b = m / count, t = m % count;
  const int keys = (pos_dev ? *pos_dev : pos0) + t + 1;
  const int S = (keys + kps - 1) / kps;
  if (split >= S) return;  // the grid covers the longest visible range
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int j0 = split * kps, nk = min(kps, keys - j0);
  const int nck = (nk + DS_CH - 1) / DS_CH, total = 2 * nck;  // K chunks, then V chunks
  const int fresh = keys - 1 - j0;                              // in [0, nk) only in the last split
  const long long kvrow0 = ((long long)b * kvh + g0) * capacity + j0;
  const uint32_t ring_a = smem_u32(ring), bar0 = smem_u32(bar);
  int issued = 0;  // thread 0: chunks whose loads are issued
  auto issue = [&](int c) {
    const int st = c % DS_RING;
    const uint32_t dst = ring_a + st * DS_CHUNK, br = bar0 + 8 * st;
    if (c < nck) {
      mbar_expect_tx(br, DS_CHUNK);
      const int y = (int)(krow0 + kvrow0 + (long long)c * DS_CH);
#pragma unroll
      for (int bx = 0; bx < 4; bx++) tma_load_2d(dst + bx * 4096, &kmap, bx * 32, y, br);
    } else {
      const int cv = c - nck, rows = min(DS_CH, nk - cv * DS_CH);
      const uint32_t bytes = (uint32_t)rows * DS_HD * 4;
      mbar_expect_tx(br, bytes);
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                   "l"(vcache + (kvrow0 + (long long)cv * DS_CH) * DS_HD), "r"(bytes), "r"(br)
                   : "memory");
    }
  };
  if (tid == 0) {
    s_abort = 0;
    for (int st = 0; st < DS_RING; st++) {
      mbar_init(bar0 + 8 * st, 1);                            // full: the copies' bytes
      mbar_init(bar0 + 8 * (DS_RING + st), DS_WARPS);         // empty: one arrival per warp
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (; issued < min(DS_RING, total); issued++) issue(issued);
  }
  pdl_wait();
  const int hq = lane >> 4, dg = lane & 15;
  const int box = dg >> 3, ck = dg & 7;  // this lane's dimensions: 32 box + 4 ck .. + 3 and 32 (box + 2) + 4 ck .. + 3
  const int pos = keys - 1;               // this token's position
  float qa[4][4], qb[4][4];
  // The newest key's row, stored into its chunk once that has landed: thread tid < 128 holds dimension
  // tid of k and v (kf0, vf0) -- or, FUSED, they sit in shared memory after the query rows.
  float kf0 = 0.f, vf0 = 0.f;
  float *kvnew = Qs + DS_GMAX * DS_HD;  // FUSED: [2][128] newest k, v
  if constexpr (FUSED) {
    // One round trip for all of it: thread (head g = tid / 32, j = tid % 32) sums the pieces of q rows
    // 4 j .. 4 j + 3 of head hg -- rows 2 (hg 64 + d) and 2 (hg 64 + d) + 1 hold the rotary pair
    // (d, d + 64), so these are the pairs d = 2 j, 2 j + 1 -- rotates them into the shared query rows;
    // threads below 128 also sum the newest key's k pair d = tid (rotated) or v pair d = tid - 64,
    // write it to the cache and keep it for the chunk that holds that key.
    const int g = tid >> 5, j = tid & 31;
    float4 qv = make_float4(0.f, 0.f, 0.f, 0.f);
    double2 cq[2];
    if (g < G) {
      cq[0] = fu.rope[(size_t)pos * 64 + 2 * j];
      cq[1] = fu.rope[(size_t)pos * 64 + 2 * j + 1];
      qv = ds_gather4(fu, m, 2 * ((g0 * G + g) * 64) + 4 * j);
    }
    const bool kv = fresh < nk && tid < 2 * 64;
    const bool isv = tid >= 64;
    float2 ab = make_float2(0.f, 0.f);
    double2 crk = make_double2(0.0, 0.0);
    if (kv) {
      if (!isv) crk = fu.rope[(size_t)pos * 64 + tid];
      ab = ds_gather2(fu, m, 2 * (nh * 64 + (isv ? kvh * 64 : 0) + g0 * 64 + (tid & 63)));
    }
    if (g < G) {
      const float in[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
      for (int i = 0; i < 2; i++) {  // EPI_QKV's rotation: (a c - b s, b c + a s) in double
        const double a = (double)in[2 * i], bb = (double)in[2 * i + 1];
        Qs[g * DS_HD + 2 * j + i] = __double2float_rn(__dsub_rn(__dmul_rn(a, cq[i].x), __dmul_rn(bb, cq[i].y)));
        Qs[g * DS_HD + 2 * j + i + 64] = __double2float_rn(__dadd_rn(__dmul_rn(bb, cq[i].x), __dmul_rn(a, cq[i].y)));
      }
    } else {
#pragma unroll
      for (int i = 0; i < 2; i++) Qs[g * DS_HD + 2 * j + i] = Qs[g * DS_HD + 2 * j + i + 64] = 0.0f;
    }
    if (kv) {
      const int d = tid & 63;
      const size_t row = (size_t)(kvrow0 + fresh) * DS_HD;
      if (!isv) {
        const double a = (double)ab.x, bb = (double)ab.y;
        const float k0 = __double2float_rn(__dsub_rn(__dmul_rn(a, crk.x), __dmul_rn(bb, crk.y)));
        const float k1 = __double2float_rn(__dadd_rn(__dmul_rn(bb, crk.x), __dmul_rn(a, crk.y)));
        kcache[row + d] = k0;
        kcache[row + d + 64] = k1;
        kvnew[d] = k0;
        kvnew[d + 64] = k1;
      } else {
        vcache[row + d] = ab.x;
        vcache[row + d + 64] = ab.y;
        kvnew[DS_HD + d] = ab.x;
        kvnew[DS_HD + d + 64] = ab.y;
      }
    }
    __syncthreads();
#pragma unroll
    for (int h = 0; h < 4; h++) {
      const float *qr = Qs + (4 * hq + h) * DS_HD;
      const float4 a = *(const float4 *)(qr + 32 * box + 4 * ck);
      const float4 c4 = *(const float4 *)(qr + 32 * (box + 2) + 4 * ck);
      qa[h][0] = a.x; qa[h][1] = a.y; qa[h][2] = a.z; qa[h][3] = a.w;
      qb[h][0] = c4.x; qb[h][1] = c4.y; qb[h][2] = c4.z; qb[h][3] = c4.w;
    }
  } else {
#pragma unroll
    for (int h = 0; h < 4; h++) {
      const int g = 4 * hq + h;
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f), c4 = a;
      if (g < G) {
        const float *qr = q + (size_t)m * ldq + (size_t)(g0 * G + g) * DS_HD;
        a = *(const float4 *)(qr + 32 * box + 4 * ck);
        c4 = *(const float4 *)(qr + 32 * (box + 2) + 4 * ck);
      }
      qa[h][0] = a.x; qa[h][1] = a.y; qa[h][2] = a.z; qa[h][3] = a.w;
      qb[h][0] = c4.x; qb[h][1] = c4.y; qb[h][2] = c4.z; qb[h][3] = c4.w;
    }
    // the newest key's row, loaded now (after the wait): the copies issued earlier may predate it
    const bool patch = fresh < nk && tid < DS_HD;
    kf0 = patch ? kcache[(kvrow0 + fresh) * DS_HD + tid] : 0.0f;
    vf0 = patch ? vcache[(kvrow0 + fresh) * DS_HD + tid] : 0.0f;
    if (patch) {
      kvnew[tid] = kf0;
      kvnew[DS_HD + tid] = vf0;
    }
    __syncthreads();
  }
  const float scale = (float)(1.0 / sqrt((double)DS_HD));
  float acc[DS_GMAX][4];
#pragma unroll
  for (int g = 0; g < DS_GMAX; g++) acc[g][0] = acc[g][1] = acc[g][2] = acc[g][3] = 0.0f;

  // The warps consume the ring independently: lane 0 of each warp waits for a chunk's copies itself, and
  // a warp done with a chunk arrives on its stage's `empty` barrier (8 arrivals); thread 0 refills the
  // stage once all eight have.  The newest key's row is read from kvnew, not from its chunk.  If a wait
  // expires the abort flag makes every later wait return at once: the warps run on over stale data
  // (every barrier of the block is still reached) and the block writes nothing.
  const uint32_t empty0 = bar0 + 8 * DS_RING;
  auto wait_full = [&](int c) {
    int ok = 1;
    if (lane == 0) ok = mbar_wait(bar0 + 8 * (c % DS_RING), (uint32_t)(c / DS_RING) & 1u, &s_abort, err, 62);
    __syncwarp();
    return __shfl_sync(0xffffffffu, ok, 0);
  };
  auto release = [&](int c) {
    __syncwarp();
    if (lane == 0) mbar_arrive(empty0 + 8 * (c % DS_RING));
    if (tid == 0 && c + DS_RING < total &&
        mbar_wait(empty0 + 8 * (c % DS_RING), (uint32_t)(c / DS_RING) & 1u, &s_abort, err, 64))
      issue(issued++);  // chunk c + DS_RING into the stage chunk c held
  };
  for (int c = 0; c < nck; c++) {  // scores
    wait_full(c);
    const uint8_t *chunk = ring + (c % DS_RING) * DS_CHUNK;
    float v[16];  // [key j][head h]: partial dots over this lane's 8 dimensions
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int kr = 4 * warp + j;
      const uint32_t sw = (uint32_t)((ck ^ (kr & 7)) << 4);
      const bool isf = c * DS_CH + kr == fresh;
      const float4 ka = isf ? *(const float4 *)(kvnew + 32 * box + 4 * ck)
                            : *(const float4 *)(chunk + box * 4096 + kr * 128 + sw);
      const float4 kb = isf ? *(const float4 *)(kvnew + 32 * (box + 2) + 4 * ck)
                            : *(const float4 *)(chunk + (box + 2) * 4096 + kr * 128 + sw);
      const float kd[8] = {ka.x, ka.y, ka.z, ka.w, kb.x, kb.y, kb.z, kb.w};
#pragma unroll
      for (int h = 0; h < 4; h += 2) {  // heads h, h + 1 in one packed FP32 FMA (each lane an IEEE fma)
        float2 x = make_float2(qa[h][0] * kd[0], qa[h + 1][0] * kd[0]);
#pragma unroll
        for (int e = 1; e < 8; e++) {
          const float2 qq = e < 4 ? make_float2(qa[h][e], qa[h + 1][e]) : make_float2(qb[h][e - 4], qb[h + 1][e - 4]);
          x = __ffma2_rn(qq, make_float2(kd[e], kd[e]), x);
        }
        v[4 * j + h] = x.x;
        v[4 * j + h + 1] = x.y;
      }
    }
    release(c);  // the chunk's K rows are in registers now
    // reduce-scatter over the 16 lanes of the quad: after the level of offset o, a lane keeps the half
    // of its values selected by its bit o
#pragma unroll
    for (int o = 8; o >= 1; o >>= 1) {
      const bool up = (dg & o) != 0;
#pragma unroll
      for (int i = 0; i < o; i++) {
        const float send = up ? v[i] : v[i + o];
        const float keep = up ? v[i + o] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
      }
    }
    {  // lane dg: key dg / 4 of the warp's four, head 4 hq + dg % 4
      const int kr = 4 * warp + (dg >> 2), g = 4 * hq + (dg & 3);
      if (c * DS_CH + kr < nk && g < G) pt[(c * DS_CH + kr) * DS_GMAX + g] = v[0] * scale;
    }
  }
  __syncthreads();  // all scores: softmax statistics of head `warp` over the split
  {
    const int g = warp;
    if (g < G) {
      float mx = -INFINITY;
      for (int j = lane; j < nk; j += 32) mx = fmaxf(mx, pt[j * DS_GMAX + g]);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      float sum = 0.0f;
      for (int j = lane; j < nk; j += 32) {
        const float e = expf(pt[j * DS_GMAX + g] - mx);
        pt[j * DS_GMAX + g] = e;
        sum += e;
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      if (lane == 0) {
        red[g * 2] = mx;
        red[g * 2 + 1] = sum;
      }
    }
  }
  __syncthreads();
  for (int c = nck; c < total; c++) {  // weighted V sum
    wait_full(c);
    const uint8_t *chunk = ring + (c % DS_RING) * DS_CHUNK;
    const int cv = c - nck, rows = min(DS_CH, nk - cv * DS_CH);
    const float *pr = pt + (size_t)cv * DS_CH * DS_GMAX;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int kr = 4 * warp + j;
      if (kr < rows) {
        const float4 vv = cv * DS_CH + kr == fresh ? *(const float4 *)(kvnew + DS_HD + 4 * lane)
                                                   : *(const float4 *)(chunk + kr * (DS_HD * 4) + lane * 16);
        const float4 pa = *(const float4 *)(pr + kr * DS_GMAX), pb = *(const float4 *)(pr + kr * DS_GMAX + 4);
        const float p8[8] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y, pb.z, pb.w};
#pragma unroll
        for (int g = 0; g < DS_GMAX; g++) {  // packed FP32 FMAs: two dimensions per instruction
          const float2 pp = make_float2(p8[g], p8[g]);
          const float2 lo = __ffma2_rn(pp, make_float2(vv.x, vv.y), make_float2(acc[g][0], acc[g][1]));
          const float2 hi = __ffma2_rn(pp, make_float2(vv.z, vv.w), make_float2(acc[g][2], acc[g][3]));
          acc[g][0] = lo.x;
          acc[g][1] = lo.y;
          acc[g][2] = hi.x;
          acc[g][3] = hi.y;
        }
      }
    }
    release(c);
  }
  __syncthreads();
  if (s_abort) {  // leave only once every copy into this block's shared memory is done (bounded again)
    if (tid == 0) {
      volatile int no_abort = 0;
      for (int cc = max(0, issued - DS_RING); cc < issued; cc++)
        mbar_wait(bar0 + 8 * (cc % DS_RING), (uint32_t)(cc / DS_RING) & 1u, &no_abort, err, 63);
    }
    return;
  }
  // the warps' value sums, added in warp order through the ring (every copy into it has completed)
  float *ws = (float *)ring;  // [warp][8 heads][128]
#pragma unroll
  for (int g = 0; g < DS_GMAX; g++)
    *(float4 *)(ws + (warp * DS_GMAX + g) * DS_HD + 4 * lane) = make_float4(acc[g][0], acc[g][1], acc[g][2], acc[g][3]);
  __syncthreads();
  const size_t slot = ((size_t)m * kvh + g0) * smax + split;
  float *po = part, *pml = part + (size_t)gridDim.z * kvh * smax * DS_GMAX * DS_HD;
  {  // thread: head tid / 32, dimensions 4 (tid % 32) .. + 3
    const int g = tid >> 5, d = 4 * lane;
    if (g < G) {
      float4 sum = *(const float4 *)(ws + g * DS_HD + d);
#pragma unroll
      for (int w = 1; w < DS_WARPS; w++) {
        const float4 x = *(const float4 *)(ws + (w * DS_GMAX + g) * DS_HD + d);
        sum.x += x.x;
        sum.y += x.y;
        sum.z += x.z;
        sum.w += x.w;
      }
      *(float4 *)(po + (slot * DS_GMAX + g) * DS_HD + d) = sum;
    }
  }
  if (tid < G) {
    pml[(slot * DS_GMAX + tid) * 2 + 0] = red[tid * 2];
    pml[(slot * DS_GMAX + tid) * 2 + 1] = red[tid * 2 + 1];
  }
  if constexpr (FUSED) {
    // the last of the S blocks of (row, KV head) to get here merges their records
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(&fu.counter[m * kvh + g0], 1) == S - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const int g = tid >> 5, d = 4 * lane;  // head, dimensions d .. d + 3
    if (g < G) {
      const size_t base = ((size_t)m * kvh + g0) * smax;
      float o[4];
      ds_merge4(po, pml, base, S, g, d, o);
      const int K = nh * DS_HD, k0 = (g0 * G + g) * DS_HD + d;
      uint16_t h[3][4];
#pragma unroll
      for (int e = 0; e < 4; e++) split3_bf16(o[e], h[0][e], h[1][e], h[2][e]);  // the skinny prologue's split
#pragma unroll
      for (int tm = 0; tm < 3; tm++) {
        uint2 u;
        u.x = (uint32_t)h[tm][0] | ((uint32_t)h[tm][1] << 16);
        u.y = (uint32_t)h[tm][2] | ((uint32_t)h[tm][3] << 16);
        *(uint2 *)(fu.x3 + ((size_t)tm * fu.NT + m) * K + k0) = u;
      }
    }
    if (tid == 0) fu.counter[m * kvh + g0] = 0;  // for the next launch
  }
}

// The split merge and the o projection's prologue in one: block (kb, m) takes elements
// [kb * 1024, kb * 1024 + 1024) of token row m's attention output (four per thread, one query head),
// merges the splits' records (max over splits, weights exp(max_s - max), numerator and denominator
// summed in split order), and writes the three BF16 terms of each output into x3 [3][NT][K] (K = nh
// x 128) as the skinny prologue does; rows M .. NT - 1 get zeros.  With out != null the Float32
// outputs go there instead (the other forms of the projection).
__global__ void __launch_bounds__(256) attention_merge_split_kernel(
    const float *part, int kps, const int *pos_dev, int pos0, int count, int nh, int kvh, int smax, int M, int NT,
    uint16_t *x3, float *out, int ldo) {
  pdl_wait();
  pdl_trigger();
  const int K = nh * DS_HD, G = nh / kvh;
  const int m = blockIdx.y;
  const int k0 = blockIdx.x * 1024 + threadIdx.x * 4;
  if (k0 >= K) return;
  float o[4] = {0.f, 0.f, 0.f, 0.f};
  if (m < M) {
    const int gq = k0 / DS_HD, g0 = gq / G, g = gq % G, d = k0 % DS_HD;
    const int keys = (pos_dev ? *pos_dev : pos0) + m % count + 1;
    const int S = (keys + kps - 1) / kps;
    const float *po = part, *ml = part + (size_t)M * kvh * smax * DS_GMAX * DS_HD;  // sums, then (max, sum)
    ds_merge4(po, ml, ((size_t)m * kvh + g0) * smax, S, g, d, o);
  }
  if (out) {
    if (m < M) *(float4 *)(out + (size_t)m * ldo + k0) = make_float4(o[0], o[1], o[2], o[3]);
    return;
  }
  uint16_t h[3][4];
#pragma unroll
  for (int e = 0; e < 4; e++) split3_bf16(o[e], h[0][e], h[1][e], h[2][e]);  // the skinny prologue's split
#pragma unroll
  for (int tm = 0; tm < 3; tm++) {
    uint2 u;
    u.x = (uint32_t)h[tm][0] | ((uint32_t)h[tm][1] << 16);
    u.y = (uint32_t)h[tm][2] | ((uint32_t)h[tm][3] << 16);
    *(uint2 *)(x3 + ((size_t)tm * NT + m) * K + k0) = u;
  }
}

}  // namespace

DecodeStreamPlan decode_stream_plan(int rows, int kvh, int capacity, int device) {
  static const int forced = env_int("STB_DS_KPS", 0);  // keys per split, a multiple of 8 up to 256
  const int pairs = rows * kvh;
  const int splits = std::max(1, 2 * sm_count(device) / std::max(pairs, 1));
  // equal splits (rounded to 8 keys, not to whole 32-key chunks: the last chunk of a split is partly
  // masked), so the SMs that hold two blocks carry as few keys as possible
  int kps = ((capacity + splits - 1) / splits + 7) / 8 * 8;
  if (forced > 0 && forced % 8 == 0) kps = forced;
  kps = std::min(std::max(kps, DS_CH), DS_KPS_MAX);
  DecodeStreamPlan p;
  p.kps = kps;
  p.smax = (capacity + kps - 1) / kps;
  return p;
}

size_t decode_stream_part_floats(int rows, int kvh, int capacity) {
  const size_t smax = (size_t)(capacity + DS_CH - 1) / DS_CH;  // the smallest split: 32 keys
  return (size_t)rows * kvh * smax * DS_GMAX * (DS_HD + 2);
}

CUtensorMap make_kv_map(const float *kv, uint64_t rows) {
  CUtensorMap m;
  const cuuint64_t dims[2] = {(cuuint64_t)DS_HD, rows};
  const cuuint64_t strides[1] = {(cuuint64_t)DS_HD * 4};
  const cuuint32_t box[2] = {32, (cuuint32_t)DS_CH};
  const cuuint32_t elem[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(kv), dims, strides, box, elem,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw Error(STB_ERR_CUDA, "cuTensorMapEncodeTiled (KV cache) failed: " + std::to_string((int)r));
  return m;
}

bool decode_stream_fusable(int nh, int kvh) {
  static const int g8 = env_int("STB_DS_G8", 1);  // 0: groups above 4 heads take the general kernel
  return g8 && nh % kvh == 0 && nh / kvh > 4 && nh / kvh <= DS_GMAX;
}

bool decode_stream_applies(int hd, int nh, int kvh) {
  static const int enabled = env_int("STB_DECODE_STREAM", 1);
  return enabled && hd == DS_HD && nh % kvh == 0 && nh / kvh <= DS_GMAX;
}

void launch_decode_attention_stream(const CUtensorMap &kmap, long long krow0, const float *q, int ldq, float *kc,
                                    float *vc, int rows, int count, int nh, int kvh, int capacity, const int *posd,
                                    int pos0, const DecodeStreamPlan &plan, float *part, bool pdl, cudaStream_t st,
                                    int device, int *err, const DecodeStreamFused *fused) {
  {
    static std::mutex mu;
    static bool configured[64] = {};
    std::lock_guard<std::mutex> lock(mu);
    if (device < 0 || device >= 64 || !configured[device]) {
      STB_CUDA(cudaFuncSetAttribute(decode_attention_stream_kernel<true>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, (int)DS_SMEM));
      STB_CUDA(cudaFuncSetAttribute(decode_attention_stream_kernel<false>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, (int)DS_SMEM));
      STB_CUDA(cudaFuncSetAttribute(decode_attention_stream_g8_kernel<false>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, (int)DS8_SMEM));
      STB_CUDA(cudaFuncSetAttribute(decode_attention_stream_g8_kernel<true>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, (int)DS8_SMEM));
      if (device >= 0 && device < 64) configured[device] = true;
    }
  }
  STB_REQUIRE(!fused || decode_stream_fusable(nh, kvh), "fused decode attention: 5 to 8 query heads per KV head");
  if (fused) {
    STB_REQUIRE(fused->part && fused->rope && fused->counter && fused->x3 && fused->M == rows && count == 1 &&
                    fused->NT >= rows,
                "fused decode attention arguments");
    launch_kernel(decode_attention_stream_g8_kernel<true>, dim3(plan.smax, kvh, rows), dim3(DS_THREADS), DS8_SMEM, st,
                  pdl, kmap, krow0, q, ldq, kc, vc, count, nh, kvh, capacity, posd, pos0, plan.kps, part, plan.smax,
                  err, *fused);
    return;
  }
  if (decode_stream_fusable(nh, kvh)) {
    launch_kernel(decode_attention_stream_g8_kernel<false>, dim3(plan.smax, kvh, rows), dim3(DS_THREADS), DS8_SMEM,
                  st, pdl, kmap, krow0, q, ldq, kc, vc, count, nh, kvh, capacity, posd, pos0, plan.kps, part,
                  plan.smax, err, DecodeStreamFused{});
    return;
  }
  auto kernel = nh / kvh > 4 ? decode_attention_stream_kernel<true> : decode_attention_stream_kernel<false>;
  launch_kernel(kernel, dim3(plan.smax, kvh, rows), dim3(DS_THREADS), DS_SMEM, st, pdl, kmap, krow0, q, ldq, kc, vc,
                count, nh, kvh, capacity, posd, pos0, plan.kps, part, plan.smax, err);
}

void launch_attention_merge_split(const float *part, const DecodeStreamPlan &plan, const int *posd, int pos0,
                                  int rows, int count, int nh, int kvh, int NT, uint16_t *x3, float *out, int ldo,
                                  cudaStream_t st) {
  const int K = nh * DS_HD;
  launch_kernel(attention_merge_split_kernel, dim3((K + 1023) / 1024, out ? rows : NT), dim3(256), 0, st, true, part,
                plan.kps, posd, pos0, count, nh, kvh, plan.smax, rows, NT, x3, out, ldo);
}

}  // namespace stb
