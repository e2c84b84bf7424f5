// Persistent whole-generation decode for small single-GPU models; see decode_mega.cuh.
#include <mutex>

#include "decode_mega.cuh"
#include "gemv.cuh"
#include "tc_common.cuh"

namespace stb {

namespace {

constexpr int MG_THREADS = 256, MG_WARPS = MG_THREADS / 32;
constexpr unsigned long long MG_WAIT_NS = 2000000000ull;  // per barrier

__device__ __forceinline__ unsigned long long mg_now() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned mg_ld_acquire(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Grid-wide barrier of the cooperative launch: one monotonic arrival counter (zeroed by the host
// before the launch); barrier number k of the launch completes when it reaches (k + 1) * gridDim.x.
// `target` is that running threshold, kept alike by every thread of every block.  Data written
// before it by any block is visible after it to loads that bypass L1 (__ldcg).  Returns false when
// the wait ran out (the error word gets 41) or another block already reported an error.
__device__ bool grid_sync(unsigned *bar, unsigned &target, int *err, int *s_ok) {
  __syncthreads();
  target += gridDim.x;
  if (threadIdx.x == 0) {
    int ok = 1;
    __threadfence();
    atomicAdd(bar, 1u);
    if (mg_ld_acquire(bar) < target) {
      const unsigned long long t0 = mg_now();
      for (unsigned i = 1; mg_ld_acquire(bar) < target; i++) {
        if ((i & 63) == 0) {
          if (*(volatile int *)err) {
            ok = 0;
            break;
          }
          if (mg_now() - t0 > MG_WAIT_NS) {
            atomicCAS(err, 0, 41);
            ok = 0;
            break;
          }
        }
      }
    }
    *s_ok = ok;
  }
  __syncthreads();
  return *s_ok != 0;
}

// RMSNorm of one row, the vector GEMV prologue's loop, reduction and expression.
__device__ void mg_rmsnorm(const float *x, const float *w, float *y, int H, double eps, double *scr) {
  double sq = 0.0;
  for (int k = threadIdx.x; k < H; k += MG_THREADS) {
    const double v = (double)x[k];
    sq = __dadd_rn(sq, __dmul_rn(v, v));
  }
  const double total = block_sum_double(sq, scr);
  const double inv = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(total, (double)H), eps)));
  for (int k = threadIdx.x; k < H; k += MG_THREADS)
    y[k] = __double2float_rn(__dmul_rn(__dmul_rn((double)x[k], inv), (double)w[k]));
  __syncthreads();
}

__device__ __forceinline__ void mg_fma8(uint4 u, const float *x, float &acc) {
  const float4 xa = *reinterpret_cast<const float4 *>(x), xb = *reinterpret_cast<const float4 *>(x + 4);
  const float2 w01 = widen2<__nv_bfloat16>(u.x), w23 = widen2<__nv_bfloat16>(u.y);
  const float2 w45 = widen2<__nv_bfloat16>(u.z), w67 = widen2<__nv_bfloat16>(u.w);
  acc = fmaf(w01.x, xa.x, acc);
  acc = fmaf(w01.y, xa.y, acc);
  acc = fmaf(w23.x, xa.z, acc);
  acc = fmaf(w23.y, xa.w, acc);
  acc = fmaf(w45.x, xb.x, acc);
  acc = fmaf(w45.y, xb.y, acc);
  acc = fmaf(w67.x, xb.z, acc);
  acc = fmaf(w67.y, xb.w, acc);
}

__device__ __forceinline__ float mg_warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

// x . W[r] for R rows at once over K (K % 8 == 0, x in shared memory), by one warp, all R rows'
// loads in flight together; every lane gets the sums.  SHARED: the rows are staged in shared memory.
template <int R, bool SHARED>
__device__ __forceinline__ void mg_dots(const uint16_t *const (&w)[R], const float *x, int K, int lane,
                                        float (&out)[R]) {
  float acc[R];
#pragma unroll
  for (int r = 0; r < R; r++) acc[r] = 0.0f;
  const int C = K >> 3;
#pragma unroll 2
  for (int c = lane; c < C; c += 32) {
    uint4 u[R];
#pragma unroll
    for (int r = 0; r < R; r++)
      u[r] = SHARED ? *reinterpret_cast<const uint4 *>(w[r] + (size_t)c * 8) : ld_stream_u4(w[r] + (size_t)c * 8);
#pragma unroll
    for (int r = 0; r < R; r++) mg_fma8(u[r], x + c * 8, acc[r]);
  }
#pragma unroll
  for (int r = 0; r < R; r++) out[r] = mg_warp_sum(acc[r]);
}

// Weight staging: a bulk copy of global bytes into this block's shared memory that completes on
// an mbarrier.  mg_stage_begin (after the buffer's last reader passed a __syncthreads): thread 0
// orders the earlier generic reads before the async writes and arms the barrier with the byte
// count; the block then issues the copies (mg_copy*) and the consumer waits (mg_stage_wait).
__device__ __forceinline__ void mg_stage_begin(uint32_t bar, uint32_t bytes) {
  if (threadIdx.x == 0) {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc::mbar_expect_tx(bar, bytes);
  }
  __syncthreads();
}

__device__ __forceinline__ void mg_bulk(void *dst, const void *src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   tc::smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

// Contiguous range, 16 KB pieces spread over the block's threads (bytes % 16 == 0).
__device__ __forceinline__ void mg_copy(void *dst, const void *src, uint32_t bytes, uint32_t bar) {
  for (uint32_t off = threadIdx.x * 16384u; off < bytes; off += MG_THREADS * 16384u) {
    const uint32_t n = bytes - off < 16384u ? bytes - off : 16384u;
    mg_bulk((char *)dst + off, (const char *)src + off, n, bar);
  }
}

// Bounded wait of the whole block on a staging barrier; false (error word 42) if it ran out.
__device__ __forceinline__ bool mg_stage_wait(uint32_t bar, uint32_t parity, int *err, int *s_ok) {
  if (threadIdx.x == 0) {
    volatile int no_abort = 0;
    *s_ok = tc::mbar_wait(bar, parity, &no_abort, err, 42) ? 1 : 0;
  }
  __syncthreads();
  return *s_ok != 0;
}

// dst[k] = src[k] for k < n (src written by other blocks: L2 loads), eight loads in flight per thread.
__device__ __forceinline__ void mg_stage(float *dst, const float *src, int n) {
  for (int base = threadIdx.x; base < n; base += MG_THREADS * 8) {
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const int k = base + u * MG_THREADS;
      v[u] = k < n ? __ldcg(src + k) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const int k = base + u * MG_THREADS;
      if (k < n) dst[k] = v[u];
    }
  }
}

// L2 prefetch of a contiguous byte range, spread over the block's threads in 32 KB pieces.
__device__ __forceinline__ void mg_prefetch(const void *p, size_t bytes) {
  const char *c = (const char *)p;
  for (size_t off = (size_t)threadIdx.x * 32768; off < bytes; off += (size_t)MG_THREADS * 32768) {
    const size_t n = (bytes - off < 32768 ? bytes - off : 32768) & ~(size_t)15;
    if (n) prefetch_l2(c + off, (uint32_t)n);
  }
}

__device__ __forceinline__ float mg_block_max(float v, float *red) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = red[0];
  for (int i = 1; i < MG_WARPS; i++) r = fmaxf(r, red[i]);
  __syncthreads();
  return r;
}

__device__ __forceinline__ float mg_block_sum(float v, float *red) {
  v = mg_warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = 0.0f;
  for (int i = 0; i < MG_WARPS; i++) r += red[i];
  __syncthreads();
  return r;
}

// qkv_store_pair for one token row at `pos` with the position's (cos, sin) already in shared
// memory: q and k pairs rotated (double, no contraction), v pairs stored as they are.
template <int HD>
__device__ __forceinline__ void mg_qkv_store(float *qbuf, float *kc, float *vc, int NH, int KV, int cap, int pos,
                                             int pi, float fa, float fb, const double2 *rs) {
  constexpr int half = HD / 2;
  const int qpairs = NH * half, kpairs = KV * half;
  if (pi < qpairs + kpairs) {
    const int local = pi < qpairs ? pi : pi - qpairs;
    const int h = local / half, d = local % half;
    const double2 cs = rs[d];
    const double x0 = (double)fa, x1 = (double)fb;
    const float oa = __double2float_rn(__dsub_rn(__dmul_rn(x0, cs.x), __dmul_rn(x1, cs.y)));
    const float ob = __double2float_rn(__dadd_rn(__dmul_rn(x1, cs.x), __dmul_rn(x0, cs.y)));
    float *dst = pi < qpairs ? qbuf + (size_t)h * HD : kc + ((size_t)h * cap + pos) * HD;
    dst[d] = oa;
    dst[d + half] = ob;
  } else {
    const int local = pi - qpairs - kpairs;
    const int h = local / half, d = local % half;
    float *dst = vc + ((size_t)h * cap + pos) * HD;
    dst[d] = fa;
    dst[d + half] = fb;
  }
}

// Per-block staged weight slices (elements): the largest share any block takes of q/k/v row
// pairs, gate/up pairs and down rows, and the o projection's column slice of one head.
struct MgShares {
  int qp, gp, dn;
};
__host__ __device__ __forceinline__ MgShares mg_shares(int NH, int KV, int hd, int H, int I, int G) {
  const int qkv_pairs = (NH + 2 * KV) * hd / 2;
  return MgShares{(qkv_pairs + G - 1) / G, (I + G - 1) / G, (H + G - 1) / G};
}

template <int HD>
__global__ void __launch_bounds__(MG_THREADS, 1) decode_mega_kernel(const MegaArgs a) {
  static_assert(HD == 16 || HD == 32 || HD == 64 || HD == 128, "head size");
  constexpr int F = HD / 4, KG = MG_THREADS / F;  // weighted sum: quads x key groups
  extern __shared__ __align__(16) float mg_sm[];
  __shared__ double s_dscr[8];
  __shared__ float s_red[MG_WARPS];
  __shared__ int s_ok, s_pos, s_stop;
  __shared__ long long s_tok;
  __shared__ unsigned long long s_best[MG_WARPS];
  __shared__ __align__(8) uint64_t s_bar[6];  // staging barriers: q/k/v, o slice, gate/up, down, 2 norms
  __shared__ double2 s_rope[64];               // (cos, sin) of this step's position, hd / 2 pairs
  const int H = a.H, I = a.I, NH = a.NH, KV = a.KV, cap = a.capacity;
  const int G = gridDim.x, b = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int XW = H > I ? H : I;
  const int capr = (cap + 31) & ~31;  // keeps every later array 16-byte aligned (float4 access)
  const MgShares sh = mg_shares(NH, KV, HD, H, I, G);
  float *hs = mg_sm;                  // [H] residual stream of the current token (every block)
  float *xs = hs + H;                 // [max(H, I)] normalised input / staged act
  float *sc = xs + XW;                // [capacity, rounded up to 32] attention scores / probabilities
  float *qs = sc + capr;              // [HD]
  float *att = qs + HD;               // [HD]
  float *pv = att + HD;               // [1024] weighted-sum partials
  uint16_t *wq = reinterpret_cast<uint16_t *>(pv + 1024);  // [2 sh.qp][H]  this block's q/k/v rows
  uint16_t *wo = wq + (size_t)2 * sh.qp * H;                // [H][HD]       o columns of head b
  uint16_t *wg = wo + (size_t)H * HD;                       // [2 sh.gp][H]  gate/up rows
  uint16_t *wd = wg + (size_t)2 * sh.gp * H;                // [sh.dn][I]    down rows
  float *nin = reinterpret_cast<float *>(wd + (size_t)sh.dn * I);  // [H] input RMSNorm weight
  float *npost = nin + H;                                           // [H] post-attention RMSNorm weight
  MegaLayer *lt = reinterpret_cast<MegaLayer *>(npost + H);         // [L] layer table
  const int qkv_pairs = (NH + 2 * KV) * HD / 2;
  const int qp0 = (int)((long)b * qkv_pairs / G), qp1 = (int)((long)(b + 1) * qkv_pairs / G);
  const int gp0 = (int)((long)b * I / G), gp1 = (int)((long)(b + 1) * I / G);  // gate/up pairs
  const int dn0 = (int)((long)b * H / G), dn1 = (int)((long)(b + 1) * H / G);  // down rows
  const int lv0 = (int)((long)b * a.V / G), lv1 = (int)((long)(b + 1) * a.V / G);
  const int qw = NH * HD;
  const size_t kv_layer = (size_t)2 * KV * cap * HD;
  const float scale = (float)(1.0 / sqrt((double)HD));
  const uint32_t bq = tc::smem_u32(&s_bar[0]), bo = tc::smem_u32(&s_bar[1]);
  const uint32_t bg = tc::smem_u32(&s_bar[2]), bd = tc::smem_u32(&s_bar[3]);
  const uint32_t bni = tc::smem_u32(&s_bar[4]), bnp = tc::smem_u32(&s_bar[5]);
  const bool has_q = qp1 > qp0, has_g = gp1 > gp0, has_d = dn1 > dn0;
  const int smax = (cap + 63) / 64;  // split records per head
  // attention roles, fixed per step: block h * S + s takes key range s of head h; s == 0 merges
  int S = 1, KS = 64, ah = 0, as = 0;
  bool att_block = false, has_o = false;
  unsigned target = 0;            // grid_sync threshold
  uint32_t uq = 0, uo = 0, ug = 0, ud = 0, uni = 0, unp = 0;  // completed uses per staging barrier
  bool pq = false, po = false, pg = false, pd = false, pni = false, pnp = false;  // copies in flight

  if (tid == 0) {
    for (int i = 0; i < 6; i++) tc::mbar_init(tc::smem_u32(&s_bar[i]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  {  // the layer table, once
    const uint32_t *src = reinterpret_cast<const uint32_t *>(a.layers);
    uint32_t *dst = reinterpret_cast<uint32_t *>(lt);
    const int words = a.L * (int)(sizeof(MegaLayer) / 4);
    for (int i = tid; i < words; i += MG_THREADS) dst[i] = src[i];
  }
  __syncthreads();

  auto stage_q = [&](int l) {
    if (!has_q) return;
    const uint32_t bytes = (uint32_t)(2 * (qp1 - qp0)) * H * 2;
    mg_stage_begin(bq, bytes);
    mg_copy(wq, lt[l].qkv + (size_t)2 * qp0 * H, bytes, bq);
    pq = true;
  };
  auto stage_o = [&](int l) {
    if (!has_o) return;
    mg_stage_begin(bo, (uint32_t)H * HD * 2);
    const uint16_t *src = lt[l].o + (size_t)ah * HD;
    for (int n = tid; n < H; n += MG_THREADS) mg_bulk(wo + (size_t)n * HD, src + (size_t)n * qw, HD * 2, bo);
    po = true;
  };
  auto stage_g = [&](int l) {
    if (!has_g) return;
    const uint32_t bytes = (uint32_t)(2 * (gp1 - gp0)) * H * 2;
    mg_stage_begin(bg, bytes);
    mg_copy(wg, lt[l].gu + (size_t)2 * gp0 * H, bytes, bg);
    pg = true;
  };
  auto stage_d = [&](int l) {
    if (!has_d) return;
    const uint32_t bytes = (uint32_t)(dn1 - dn0) * I * 2;
    mg_stage_begin(bd, bytes);
    mg_copy(wd, lt[l].down + (size_t)dn0 * I, bytes, bd);
    pd = true;
  };
  auto stage_ni = [&](int l) {
    mg_stage_begin(bni, (uint32_t)H * 4);
    mg_copy(nin, lt[l].in_norm, (uint32_t)H * 4, bni);
    pni = true;
  };
  auto stage_np = [&](int l) {
    mg_stage_begin(bnp, (uint32_t)H * 4);
    mg_copy(npost, lt[l].post_norm, (uint32_t)H * 4, bnp);
    pnp = true;
  };
  // on an early exit: no bulk copy may still be writing this block's shared memory
  auto drain = [&]() {
    if (tid == 0) {
      volatile int no_abort = 0;
      if (pq) tc::mbar_wait(bq, uq & 1, &no_abort, a.err, 43);
      if (po) tc::mbar_wait(bo, uo & 1, &no_abort, a.err, 43);
      if (pg) tc::mbar_wait(bg, ug & 1, &no_abort, a.err, 43);
      if (pd) tc::mbar_wait(bd, ud & 1, &no_abort, a.err, 43);
      if (pni) tc::mbar_wait(bni, uni & 1, &no_abort, a.err, 43);
      if (pnp) tc::mbar_wait(bnp, unp & 1, &no_abort, a.err, 43);
    }
    __syncthreads();
  };

  for (int step = 0; step < a.steps; step++) {
    if (tid == 0) {
      s_stop = __ldcg(a.state + 1);
      s_pos = __ldcg(a.state);
      s_tok = __ldcg((const long long *)a.tokens);
    }
    __syncthreads();
    if (s_stop) break;  // read after a barrier: every block sees the same flag
    const int pos = s_pos;
    const int keys = pos + 1;
    S = (keys + 63) / 64;
    if (S > G / NH) S = G / NH;
    KS = (keys + S - 1) / S;
    ah = b / S;
    as = b % S;
    att_block = b < NH * S;
    has_o = att_block && as == 0;
    if (tid < HD / 2) s_rope[tid] = a.rope[(size_t)pos * (HD / 2) + tid];
    stage_ni(0);
    stage_np(0);
    stage_q(0);
    stage_o(0);
    stage_g(0);
    stage_d(0);
    for (int k = tid; k < H; k += MG_THREADS) hs[k] = widen1<__nv_bfloat16>(a.embed[(size_t)s_tok * H + k]);
    __syncthreads();

    for (int l = 0; l < a.L; l++) {
      float *kc = a.kv + (size_t)l * kv_layer;
      const bool more = l + 1 < a.L;
      // A: RMSNorm -> q/k/v pairs of this block -> RoPE, cache append
      if (!mg_stage_wait(bni, uni & 1, a.err, &s_ok)) {
        drain();
        return;
      }
      uni++;
      pni = false;
      mg_rmsnorm(hs, nin, xs, H, a.eps, s_dscr);  // ends with __syncthreads: nin is free again
      if (more) stage_ni(l + 1);
      if (has_q) {
        if (!mg_stage_wait(bq, uq & 1, a.err, &s_ok)) {
          drain();
          return;
        }
        uq++;
        pq = false;
        for (int p = qp0 + warp; p < qp1; p += MG_WARPS) {
          const uint16_t *rows[2] = {wq + (size_t)(2 * (p - qp0)) * H, wq + (size_t)(2 * (p - qp0) + 1) * H};
          float r[2];
          mg_dots<2, true>(rows, xs, H, lane, r);
          if (lane == 0) mg_qkv_store<HD>(a.qbuf, kc, kc + (size_t)KV * cap * HD, NH, KV, cap, pos, p, r[0], r[1], s_rope);
        }
        __syncthreads();
        if (more) stage_q(l + 1);
      }
      if (!grid_sync(a.bar, target, a.err, &s_ok)) {
        drain();
        return;
      }

      // B: attention split over (head, key range) blocks; the head's range-0 block merges the
      // splits and applies the head's slice of the o projection
      if (att_block) {
        const int h = ah, g = h / (NH / KV);
        const float *kr = kc + (size_t)g * cap * HD;
        const float *vr = kc + (size_t)KV * cap * HD + (size_t)g * cap * HD;
        const int j0 = as * KS, j1 = min(keys, j0 + KS), nk = j1 - j0;
        const int f = tid % F, kg = tid / F;  // weighted-sum role: quad f of keys kg, kg + KG, ...
        float4 v0[8];                          // the first eight of them, loaded with the K rows
#pragma unroll
        for (int u = 0; u < 8; u++) {
          const int j = kg + u * KG;
          v0[u] = j < nk ? __ldcg(reinterpret_cast<const float4 *>(vr + (size_t)(j0 + j) * HD) + f)
                         : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        if (tid < HD) qs[tid] = __ldcg(a.qbuf + (size_t)h * HD + tid);
        __syncthreads();
        {  // scores: four threads per key, hd / 4 dimensions each
          constexpr int QD = HD / 4;
          const int qt = tid & 3;
          for (int base = 0; base < nk; base += MG_THREADS / 4) {  // uniform trip count: all lanes shuffle
            const int j = j0 + base + (tid >> 2);
            float dot = 0.0f;
            if (j < j1) {
              const float4 *k4 = reinterpret_cast<const float4 *>(kr + (size_t)j * HD + qt * QD);
              float4 kv[QD / 4];
#pragma unroll
              for (int u = 0; u < QD / 4; u++) kv[u] = __ldcg(k4 + u);
#pragma unroll
              for (int u = 0; u < QD / 4; u++) {
                const float *q4 = qs + qt * QD + 4 * u;
                dot = fmaf(q4[0], kv[u].x, dot);
                dot = fmaf(q4[1], kv[u].y, dot);
                dot = fmaf(q4[2], kv[u].z, dot);
                dot = fmaf(q4[3], kv[u].w, dot);
              }
            }
            dot += __shfl_xor_sync(0xffffffffu, dot, 1);
            dot += __shfl_xor_sync(0xffffffffu, dot, 2);
            if (qt == 0 && j < j1) sc[j - j0] = dot * scale;
          }
        }
        __syncthreads();
        float mx = -INFINITY;
        for (int j = tid; j < nk; j += MG_THREADS) mx = fmaxf(mx, sc[j]);
        mx = mg_block_max(mx, s_red);
        float sum = 0.0f;
        for (int j = tid; j < nk; j += MG_THREADS) {
          const float e = expf(sc[j] - mx);
          sc[j] = e;
          sum += e;
        }
        sum = mg_block_sum(sum, s_red);
        {  // unnormalised weighted V sum of the range: thread (key group kg, quad f), groups in order
          float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
          for (int jb = kg; jb < nk; jb += 8 * KG) {
            float4 v[8];
#pragma unroll
            for (int u = 0; u < 8; u++) {
              const int j = jb + u * KG;
              v[u] = jb == kg ? v0[u]
                              : (j < nk ? __ldcg(reinterpret_cast<const float4 *>(vr + (size_t)(j0 + j) * HD) + f)
                                        : make_float4(0.f, 0.f, 0.f, 0.f));
            }
#pragma unroll
            for (int u = 0; u < 8; u++) {
              const int j = jb + u * KG;
              const float p = j < nk ? sc[j] : 0.0f;
              o0 = fmaf(p, v[u].x, o0);
              o1 = fmaf(p, v[u].y, o1);
              o2 = fmaf(p, v[u].z, o2);
              o3 = fmaf(p, v[u].w, o3);
            }
          }
          *reinterpret_cast<float4 *>(pv + kg * HD + 4 * f) = make_float4(o0, o1, o2, o3);
        }
        __syncthreads();
        float *rec = a.apart + ((size_t)h * smax + as) * (HD + 2);
        if (tid < HD) {
          float o = 0.0f;
#pragma unroll
          for (int k = 0; k < KG; k++) o += pv[k * HD + tid];
          if (S == 1) att[tid] = o / sum;
          else rec[2 + tid] = o;
        }
        if (S > 1) {
          if (tid == 0) {
            rec[0] = mx;
            rec[1] = sum;
          }
          __threadfence();
          __syncthreads();
          unsigned *done = a.bar + 16 + h;
          if (tid == 0) atomicAdd(done, 1u);
          if (has_o) {  // merge the head's S ranges in range order
            if (tid == 0) {
              int ok = 1;
              const unsigned long long t0 = mg_now();
              for (unsigned i = 1; mg_ld_acquire(done) < (unsigned)S; i++) {
                if ((i & 63) == 0 && (*(volatile int *)a.err || mg_now() - t0 > MG_WAIT_NS)) {
                  atomicCAS(a.err, 0, 44);
                  ok = 0;
                  break;
                }
              }
              *done = 0u;  // every range has arrived: ready for the next layer
              s_ok = ok;
            }
            __syncthreads();
            if (!s_ok) {
              drain();
              return;
            }
            const float *hrec = a.apart + (size_t)h * smax * (HD + 2);
            if (tid < HD) {
              float M = -INFINITY;
              for (int r = 0; r < S; r++) M = fmaxf(M, __ldcg(hrec + (size_t)r * (HD + 2)));
              float num = 0.0f, den = 0.0f;
              for (int r = 0; r < S; r++) {
                const float w = expf(__ldcg(hrec + (size_t)r * (HD + 2)) - M);
                num = fmaf(w, __ldcg(hrec + (size_t)r * (HD + 2) + 2 + tid), num);
                den = fmaf(w, __ldcg(hrec + (size_t)r * (HD + 2) + 1), den);
              }
              att[tid] = num / den;
            }
          }
        }
        if (has_o) {
          if (!mg_stage_wait(bo, uo & 1, a.err, &s_ok)) {  // (its __syncthreads also publishes att)
            drain();
            return;
          }
          uo++;
          po = false;
          {  // CH lanes per row (one 16-byte chunk each), 32 / CH rows per warp: conflict-free rows
            constexpr int CH = HD / 8, RPW = 32 / CH;
            const int rr = lane / CH, cc = lane % CH;
            for (int n0 = warp * RPW; n0 < H; n0 += MG_WARPS * RPW) {
              const int n = n0 + rr;
              float acc = 0.0f;
              if (n < H) mg_fma8(*reinterpret_cast<const uint4 *>(wo + (size_t)n * HD + cc * 8), att + cc * 8, acc);
#pragma unroll
              for (int off = CH / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
              if (cc == 0 && n < H) a.opart[(size_t)h * H + n] = acc;
            }
          }
          __syncthreads();
          if (more) stage_o(l + 1);
        }
      }
      if (!grid_sync(a.bar, target, a.err, &s_ok)) {
        drain();
        return;
      }

      // C: residual + o (heads in order), post-attention RMSNorm, gate/up pairs -> act
      for (int n0 = tid; n0 < H; n0 += 4 * MG_THREADS) {
        float s4[4] = {0.f, 0.f, 0.f, 0.f};
        for (int h0 = 0; h0 < NH; h0 += 16) {
          float v[4][16];
#pragma unroll
          for (int r = 0; r < 4; r++) {
            const int n = n0 + r * MG_THREADS;
#pragma unroll
            for (int u = 0; u < 16; u++)
              v[r][u] = (n < H && h0 + u < NH) ? __ldcg(a.opart + (size_t)(h0 + u) * H + n) : 0.0f;
          }
#pragma unroll
          for (int r = 0; r < 4; r++)
#pragma unroll
            for (int u = 0; u < 16; u++)
              if (h0 + u < NH) s4[r] += v[r][u];
        }
#pragma unroll
        for (int r = 0; r < 4; r++) {
          const int n = n0 + r * MG_THREADS;
          if (n < H) hs[n] = hs[n] + s4[r];
        }
      }
      __syncthreads();
      if (!mg_stage_wait(bnp, unp & 1, a.err, &s_ok)) {
        drain();
        return;
      }
      unp++;
      pnp = false;
      mg_rmsnorm(hs, npost, xs, H, a.eps, s_dscr);
      if (more) stage_np(l + 1);
      if (has_g) {
        if (!mg_stage_wait(bg, ug & 1, a.err, &s_ok)) {
          drain();
          return;
        }
        ug++;
        pg = false;
        for (int p = gp0 + 2 * warp; p < gp1; p += 2 * MG_WARPS) {  // two pairs per warp
          const int p2 = p + 1 < gp1 ? p + 1 : p;
          const uint16_t *rows[4] = {wg + (size_t)(2 * (p - gp0)) * H, wg + (size_t)(2 * (p - gp0) + 1) * H,
                                     wg + (size_t)(2 * (p2 - gp0)) * H, wg + (size_t)(2 * (p2 - gp0) + 1) * H};
          float r[4];
          mg_dots<4, true>(rows, xs, H, lane, r);
          if (lane == 0) {
            a.act[p] = silu_ref(r[0]) * r[1];
            if (p2 != p) a.act[p2] = silu_ref(r[2]) * r[3];
          }
        }
        __syncthreads();
        if (more) stage_g(l + 1);
      }
      if (!grid_sync(a.bar, target, a.err, &s_ok)) {
        drain();
        return;
      }

      // D: down rows of this block with the residual
      mg_stage(xs, a.act, I);
      __syncthreads();
      if (has_d) {
        if (!mg_stage_wait(bd, ud & 1, a.err, &s_ok)) {
          drain();
          return;
        }
        ud++;
        pd = false;
        for (int n = dn0 + warp; n < dn1; n += MG_WARPS) {
          const uint16_t *rows[1] = {wd + (size_t)(n - dn0) * I};
          float r[1];
          mg_dots<1, true>(rows, xs, I, lane, r);
          if (lane == 0) a.hid[n] = hs[n] + r[0];
        }
        __syncthreads();
        if (more) stage_d(l + 1);
      }
      if (!more) mg_prefetch(a.lm_head + (size_t)lv0 * H, (size_t)(lv1 - lv0) * H * 2);
      if (!grid_sync(a.bar, target, a.err, &s_ok)) {
        drain();
        return;
      }
      mg_stage(hs, a.hid, H);
      __syncthreads();
    }

    // final RMSNorm, lm_head rows of this block (four per warp in flight), greedy candidate
    mg_rmsnorm(hs, a.final_norm, xs, H, a.eps, s_dscr);
    unsigned long long best = 0ull;
    for (int v = lv0 + 4 * warp; v < lv1; v += 4 * MG_WARPS) {
      const uint16_t *rows[4];
#pragma unroll
      for (int r = 0; r < 4; r++) rows[r] = a.lm_head + (size_t)(v + r < lv1 ? v + r : v) * H;
      float d[4];
      mg_dots<4, false>(rows, xs, H, lane, d);
#pragma unroll
      for (int r = 0; r < 4; r++) {
        if (v + r < lv1) {
          const unsigned long long key = argmax_key(d[r], v + r);
          best = key > best ? key : best;
        }
      }
    }
    if (lane == 0) s_best[warp] = best;
    __syncthreads();
    if (tid == 0) {
      unsigned long long m = s_best[0];
      for (int w = 1; w < MG_WARPS; w++) m = s_best[w] > m ? s_best[w] : m;
      if (m) atomicMax(a.best, m);
    }
    if (!grid_sync(a.bar, target, a.err, &s_ok)) return;
    if (b == 0 && tid == 0) {  // finalize_kernel for one batch row
      const unsigned long long key = atomicExch(a.best, 0ull);
      const int pick = argmax_key_index(key);
      int stopped = a.state[2];
      if (!stopped) {
        a.out_ids[a.state[3]] = pick;
        a.state[3] += 1;
        for (int e = 0; e < a.eos_count; e++)
          if (a.eos[e] == pick) stopped = 1;
        a.state[2] = stopped;
      }
      a.tokens[0] = pick;
      a.state[0] += 1;
      a.state[1] = stopped;
    }
    if (!grid_sync(a.bar, target, a.err, &s_ok)) return;
  }
}

// Shared memory of one block: hs [H], xs [max(H, I)], scores [capacity rounded up to 32], q [hd],
// att [hd], weighted-sum partials [1024] (floats), then the staged BF16 weight slices (q/k/v pairs,
// the o columns of one head, gate/up pairs, down rows) for a grid of G blocks, the two staged RMSNorm
// weights [H] each and the layer table [L].  H % 8 == 0,
// I % 8 == 0 and hd % 16 == 0 keep each array 16-byte aligned.
size_t mega_smem(int H, int I, int capacity, int hd, int NH, int KV, int G, int L) {
  const MgShares sh = mg_shares(NH, KV, hd, H, I, G);
  const size_t floats = (size_t)H + (H > I ? H : I) + ((capacity + 31) & ~31) + 2 * hd + 1024;
  const size_t halves = (size_t)2 * sh.qp * H + (size_t)H * hd + (size_t)2 * sh.gp * H + (size_t)sh.dn * I;
  return floats * sizeof(float) + halves * 2 + (size_t)2 * H * sizeof(float) + (size_t)L * sizeof(MegaLayer);
}

int mega_sms(int device) {
  int n = 0;
  STB_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device));
  return n;
}

}  // namespace

bool mega_eligible(int H, int NH, int KV, int hd, int I, int V, int L, int capacity, int batch, int tp,
                   int w_dtype, int device) {
  // Opt-in: measured on the SmolLM2-shaped bench it decodes at ~1320 tok/s against ~1720 for the
  // graph-replayed step (a grid barrier costs ~1.4 us and the o slice waits on one small strided
  // bulk copy per row), so the graph path stays the default.
  static const int enabled = env_int("STB_DECODE_PERSISTENT", 0);
  if (!enabled || batch != 1 || tp != 1 || w_dtype != STB_BF16) return false;
  if (H % 8 || I % 8 || (hd != 16 && hd != 32 && hd != 64 && hd != 128) || KV <= 0 || NH % KV) return false;
  if (V <= 0 || NH > mega_sms(device)) return false;
  int coop = 0;
  STB_CUDA(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, device));
  return coop && mega_smem(H, I, capacity, hd, NH, KV, mega_sms(device), L) <= 200 * 1024;
}

namespace {

template <int HD>
void mega_launch_hd(const MegaArgs &a, size_t smem, int device, cudaStream_t st) {
  static std::mutex mu;
  static size_t configured[64] = {};
  {
    std::lock_guard<std::mutex> lock(mu);
    if (device < 0 || device >= 64 || configured[device] < smem) {
      STB_CUDA(cudaFuncSetAttribute(decode_mega_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      if (device >= 0 && device < 64) configured[device] = smem;
    }
  }
  int per_sm = 0;
  STB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_mega_kernel<HD>, MG_THREADS, smem));
  if (per_sm < 1) throw Error(STB_ERR_CUDA, "persistent decode does not fit on an SM");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(mega_sms(device));
  cfg.blockDim = dim3(MG_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, decode_mega_kernel<HD>, a);
  if (e != cudaSuccess) throw Error(STB_ERR_CUDA, std::string("persistent decode launch failed: ") + cudaGetErrorString(e));
}

}  // namespace

void mega_launch(const MegaArgs &a, int device, cudaStream_t st) {
  const size_t smem = mega_smem(a.H, a.I, a.capacity, a.hd, a.NH, a.KV, mega_sms(device), a.L);
  switch (a.hd) {
    case 16: mega_launch_hd<16>(a, smem, device, st); break;
    case 32: mega_launch_hd<32>(a, smem, device, st); break;
    case 64: mega_launch_hd<64>(a, smem, device, st); break;
    case 128: mega_launch_hd<128>(a, smem, device, st); break;
    default: throw Error(STB_ERR_INVALID, "persistent decode head size");
  }
}

}  // namespace stb
