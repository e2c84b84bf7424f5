// Llama decode runtime: the prepared, resident model of BackendLlama (models/src/main/scala/
// scalatorch/models/BackendLlama.scala) with its resident KV cache (BackendLlamaCache.scala),
// rebuilt around the B200 GEMV family.
//
// Per layer the reference runs ~20 separate backend ops with a stream synchronisation after each
// (CudaSession.scala:829-850).  Here one layer is five launches on the session stream:
//   1. QKV GEMV: input RMSNorm prologue, RoPE + KV-cache append epilogue  (q,k,v rows paired)
//   2. causal GQA attention over the HBM-resident cache (double accumulation as CpuAttention)
//   3. O GEMV with the residual add fused (h = x + attn)
//   4. gate/up GEMV: post RMSNorm prologue, SiLU(gate)*up epilogue (interleaved rows)
//   5. down GEMV with the residual add fused
// then the final-norm + lm_head GEMV with per-block greedy candidates and one finalize kernel that
// picks the token (TokenSampler strict '>'), feeds it back as the next input, appends it to the
// output and advances the device-side position.  A decode step therefore needs no host
// interaction and is captured once as a CUDA graph and replayed per generated token.
//
// Batched decode rows (2 .. 64 per chunk) take the tensor-core skinny form of each projection
// (gemm_skinny.cu: prologue, stream-K GEMM, fixup).  On one GPU the prologues are folded into the
// previous kernel: the attention merge writes the o projection's activation terms, the o fixup adds
// the residual and does the post-attention RMSNorm and split for gate/up, the gate/up fixup writes
// SiLU(gate)*up as the down projection's terms, and the down fixup adds the residual and does the
// next layer's input RMSNorm and split -- 9 launches per layer instead of 13.  With 5 to 8 query heads
// per KV head the attention also takes over the QKV fixup (RoPE, cache append) and its own split
// merge (attention_decode.cu): 8 launches per layer -- QKV GEMM, attention, o GEMM + fixup, gate/up
// GEMM + fixup, down GEMM + fixup.
//
// Tensor parallel (tp_size > 1): q/k/v/gate/up are split by output rows (heads / intermediate),
// o/down by input columns; each row-split projection's partial sums are joined by one NCCL
// allreduce which also carries the residual (rank 0 adds it before the reduction).  lm_head is
// split by vocabulary; ranks exchange their (value, index) candidates with one allgather.
#include <algorithm>
#include <climits>
#include <cmath>
#include <cstring>
#include <mutex>
#include <vector>

#include "attention_decode.cuh"
#include "gemv.cuh"
#include "rng.cuh"
#include "tc_common.cuh"

namespace stb {
void allreduce_sum_f32(stb_session *s, void *buf, uint64_t count);
void allgather_bytes(stb_session *s, const void *send, void *recv, uint64_t bytes);
void gemm_tc_launch(const void *xh, const void *w, int dtype, const float *bias, float *y, int ldy, int M, int N,
                    int K, int *err, int device, cudaStream_t stream, const float *residual, int ldr);
void round_activations(const float *x, uint16_t *out, size_t count, int dtype, cudaStream_t stream);
bool peer_usable(stb_session *s, uint64_t elems);
PeerArgs peer_args(stb_session *s, int region);
void peer_reduce_launch(stb_session *s, int region, long total, const float *residual, float *out);
bool peer_norm_fusable(int H);
void peer_reduce_norm_launch(stb_session *s, int region, int rows, int H, const float *residual, float *out,
                             const float *norm_w, double eps, uint16_t *x3n, int NT);
void peer_reset(stb_session *s);
bool launch_flash_attention_tc(const float *q, int ldq, const float *kc, const float *vc, float *out, int ldo,
                               int rows, int count, int nh, int kvh, int hd, int capacity, const int *posd, int pos0,
                               int *err, int device, cudaStream_t st, uint16_t *out_half = nullptr,
                               int half_dtype = STB_BF16);
}  // namespace stb

using namespace stb;

namespace {

struct Layer {
  uint64_t in_norm = 0, post_norm = 0;  // f32 [H]
  uint64_t qkv = 0;                     // half [(nh+2kv)*hd][H], rows paired (d, d+hd/2)
  uint64_t o = 0;                       // half [H][nh*hd] (this rank's input columns)
  uint64_t gu = 0;                      // half [2*I][H], rows interleaved gate/up
  uint64_t down = 0;                    // half [H][I] (this rank's input columns)
};

}  // namespace

struct stb_llama {
  stb_session *s = nullptr;
  stb_llama_config c{};
  int H = 0, NH = 0, KV = 0, hd = 0, I = 0, V = 0;  // local (this rank) sizes; H full
  int v0 = 0;                                       // vocabulary offset of this rank's lm_head rows
  int rank = 0, tp = 1;
  uint64_t embed = 0, final_norm = 0, lm_head = 0;  // lm_head may alias embed (tied, tp == 1)
  bool head_aliases_embed = false;
  std::vector<Layer> layers;
  uint64_t rope = 0;  // double2 [max_positions][hd/2]
  std::vector<uint64_t> owned;
  uint64_t weight_bytes = 0;
  int tc_rows = 256;  // chunks of >= tc_rows token rows use the tensor-core prefill (INT_MAX: never)
  // the last stb_llama_generate call's cache and decode graph, reused by the next call of the same
  // shape (batch, prompt + new, new, EOS count, prefill chunk)
  stb_llama_cache *gen = nullptr;
  int gen_key[5] = {};
};

struct stb_llama_cache {
  stb_llama *m = nullptr;
  int batch = 0, capacity = 0, used = 0;
  uint64_t kv = 0;  // [layers][2][batch][kvh][capacity][hd] f32
  // scratch sized for `rows` token rows
  int rows = 0;
  uint64_t hidden = 0, qbuf = 0, att = 0, act = 0, sum = 0, logits = 0;
  uint64_t best = 0;      // u64 [batch] greedy candidate keys of this rank (zero between steps)
  uint64_t best_all = 0;  // u64 [tp][batch] after the cross-rank gather
  // tensor-core prefill buffers (allocated when rows >= tc_rows): normalised x, half activations,
  // paired q/k/v projection, interleaved gate/up projection
  uint64_t xn = 0, xh = 0, qkvbuf = 0, gubuf = 0;
  uint64_t skin = 0, skin_bytes = 0;  // tensor-core skinny path scratch (one 64-row block)
  uint64_t skin_next = 0;             // next projection's activation terms written by a fused fixup
  uint64_t att_part = 0, att_count = 0;  // split decode attention records and counters (batch rows)
  CUtensorMap kv_map;                    // the whole K/V cache as rows of hd Float32 (streamed attention)
  bool kv_map_ok = false;
  int att_rows = 0;
  int graph_launches = 0;  // kernels in one replay of `graph`
  uint64_t tokens = 0;  // int64 [rows]
  uint64_t state = 0;   // int32: [0] position, [1] all stopped, [2..2+batch) stopped, [2+batch..) out count
  uint64_t out_ids = 0;
  int out_stride = 0;
  uint64_t eos = 0;
  int eos_count = 0;
  cudaGraphExec_t graph = nullptr;
  int graph_nodes = 0;
  std::vector<uint64_t> owned;
};

namespace {

uint64_t alloc_owned(stb_session *s, std::vector<uint64_t> &owned, uint64_t bytes) {
  uint64_t p = session_alloc(s, bytes);
  owned.push_back(p);
  return p;
}

void free_owned(stb_session *s, std::vector<uint64_t> &owned) {
  for (auto it = owned.rbegin(); it != owned.rend(); ++it) {
    try {
      session_free(s, *it);
    } catch (...) {
    }
  }
  owned.clear();
}

size_t esize(int dtype) { return dtype == STB_F32 ? 4 : 2; }

// ---------------------------------------------------------------- kernels

// hidden[m] = widen(table[tokens[m]]): 8 elements (one 16-byte load, H % 8 == 0) per thread, blocks
// (chunk group, row), so a row's loads are all in flight at once.
__global__ void embed_kernel(const int64_t *tokens, const uint16_t *table, int dtype, int H, int V, float *hidden,
                             int rows, const int *stop) {
  pdl_wait();
  if (stop && *stop) return;
  const int m = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= rows || c * 8 >= H) return;
  int64_t id = tokens[m];
  if (id < 0 || id >= V) id = 0;  // host validates; device-fed ids come from argmax over [0, V)
  const uint4 raw = *reinterpret_cast<const uint4 *>(table + (size_t)id * H + c * 8);
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
  float v[8];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const float2 f = dtype == STB_BF16 ? widen2<__nv_bfloat16>(w[i]) : widen2<__half>(w[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
  float *dst = hidden + (size_t)m * H + c * 8;
  *reinterpret_cast<float4 *>(dst) = make_float4(v[0], v[1], v[2], v[3]);
  *reinterpret_cast<float4 *>(dst + 4) = make_float4(v[4], v[5], v[6], v[7]);
}

// Causal grouped-query attention of CpuAttention.causal (cpu/.../CpuAttention.scala:20-50):
// scores, softmax and the weighted value sum in double (the reference's precision); one block of
// ATT_THREADS per (token row, query head).  Decode is latency-bound, so the kernel keeps memory
// round trips few: one key per thread for the scores (its whole K row in flight as float4 loads),
// and for the weighted sum each thread owns 4 output dimensions of a key subset with 8 V rows in
// flight; the subsets are combined in a fixed order.  hd must be a multiple of 4 and <= 256.
constexpr int ATT_THREADS = 256;
constexpr int ATT_UNROLL = 8;

__global__ void __launch_bounds__(ATT_THREADS) attention_kernel(const float *q, int ldq, const float *kcache,
                                                                const float *vcache, float *out, int ldo, int rows,
                                                                int count, int nh, int kvh, int hd, int capacity,
                                                                const int *pos_dev, int pos0, const int *stop) {
  // [capacity] probabilities | [32] reductions | [hd] q in double | [ATT_THREADS*4] partial sums
  extern __shared__ double s_p[];
  pdl_wait();
  pdl_trigger();
  if (stop && *stop) return;
  const int m = blockIdx.x / nh, h = blockIdx.x % nh;
  if (m >= rows) return;
  const int b = m / count, t = m % count;
  const int pos = (pos_dev ? *pos_dev : pos0) + t;
  const int keys = pos + 1;
  const int g = h / (nh / kvh);
  const float *qr = q + (size_t)m * ldq + (size_t)h * hd;
  const size_t base = ((size_t)b * kvh + g) * capacity;
  const float4 *K4 = reinterpret_cast<const float4 *>(kcache + base * hd);
  const float4 *V4 = reinterpret_cast<const float4 *>(vcache + base * hd);
  double *red = s_p + capacity;
  double *qs = red + 32;
  double *part = qs + hd;
  constexpr int NW = ATT_THREADS / 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int F = hd >> 2;  // float4 slots per row
  for (int d = threadIdx.x; d < hd; d += ATT_THREADS) qs[d] = (double)qr[d];
  __syncthreads();
  const double scale = 1.0 / sqrt((double)hd);
  double local_max = -(double)INFINITY;
  for (int j = threadIdx.x; j < keys; j += ATT_THREADS) {
    const float4 *kr = K4 + (size_t)j * F;
    double dot = 0.0;
    for (int f0 = 0; f0 < F; f0 += ATT_UNROLL) {
      float4 kv[ATT_UNROLL];
#pragma unroll
      for (int u = 0; u < ATT_UNROLL; u++) kv[u] = f0 + u < F ? kr[f0 + u] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int u = 0; u < ATT_UNROLL; u++) {
        if (f0 + u < F) {
          const double *qd = qs + 4 * (f0 + u);
          dot += qd[0] * (double)kv[u].x;
          dot += qd[1] * (double)kv[u].y;
          dot += qd[2] * (double)kv[u].z;
          dot += qd[3] * (double)kv[u].w;
        }
      }
    }
    const double sc = dot * scale;
    s_p[j] = sc;
    local_max = fmax(local_max, sc);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) local_max = fmax(local_max, __shfl_xor_sync(0xffffffffu, local_max, off));
  if (lane == 0) red[warp] = local_max;
  __syncthreads();
  double mx = red[0];
  for (int i = 1; i < NW; i++) mx = fmax(mx, red[i]);
  double local_sum = 0.0;
  for (int j = threadIdx.x; j < keys; j += ATT_THREADS) {
    const double e = exp(s_p[j] - mx);
    s_p[j] = e;
    local_sum += e;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) local_sum += __shfl_xor_sync(0xffffffffu, local_sum, off);
  __syncthreads();  // every thread has read red[] for the max
  if (lane == 0) red[warp] = local_sum;
  __syncthreads();
  double den = 0.0;
  for (int i = 0; i < NW; i++) den += red[i];
  for (int j = threadIdx.x; j < keys; j += ATT_THREADS) s_p[j] = s_p[j] / den;
  __syncthreads();
  // weighted value sum: thread (grp, f) owns dimensions 4f..4f+3 for keys j = grp (mod groups)
  const int groups = ATT_THREADS / F;
  const int f = threadIdx.x % F, grp = threadIdx.x / F;
  if (grp < groups) {
    double a0 = 0.0, a1 = 0.0, a2 = 0.0, a3 = 0.0;
    for (int j0 = grp; j0 < keys; j0 += groups * ATT_UNROLL) {
      float4 vv[ATT_UNROLL];
#pragma unroll
      for (int u = 0; u < ATT_UNROLL; u++) {
        const int j = j0 + u * groups;
        vv[u] = j < keys ? V4[(size_t)j * F + f] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < ATT_UNROLL; u++) {
        const int j = j0 + u * groups;
        if (j < keys) {
          const double pj = s_p[j];
          a0 += pj * (double)vv[u].x;
          a1 += pj * (double)vv[u].y;
          a2 += pj * (double)vv[u].z;
          a3 += pj * (double)vv[u].w;
        }
      }
    }
    double *pp = part + (size_t)(grp * F + f) * 4;
    pp[0] = a0; pp[1] = a1; pp[2] = a2; pp[3] = a3;
  }
  __syncthreads();
  for (int d = threadIdx.x; d < hd; d += ATT_THREADS) {
    double sum = 0.0;
    for (int gi = 0; gi < groups; gi++) sum += part[(size_t)(gi * F + (d >> 2)) * 4 + (d & 3)];
    out[(size_t)m * ldo + (size_t)h * hd + d] = (float)sum;
  }
}

size_t attention_smem(int capacity, int hd) {
  return (size_t)(capacity + 32 + hd + ATT_THREADS * 4) * sizeof(double);
}

// Causal grouped-query attention of a long prefill chunk in Float32 (the tensor-core prefill path,
// whose projections already round activations to BF16): flash-style tiles instead of one block
// per query row, so each K/V row is read once per 64 queries rather than once per query.
// Block (query tile, head, batch row) holds 64 queries; per 64-key tile it forms the 64 x 64
// scores (thread (ty, tx): queries 4ty..4ty+3 x keys 4tx..4tx+3, FP32 FMA over hd from shared
// memory), applies the causal mask, updates the running row max / sum (online softmax: earlier
// tiles rescaled by exp(m_old - m_new)) and accumulates P.V (queries 4ty.. x hd/16 dimensions).
// Keys are positions 0..base+t of this batch row's cache; the chunk's own keys were appended
// before the launch.
constexpr int FA_BQ = 64, FA_BK = 64, FA_PAD = 4;

template <int HD>
constexpr size_t flash_smem() {
  return (size_t)(HD * FA_BQ + HD * (FA_BK + FA_PAD) + FA_BK * HD + FA_BK * (FA_BQ + FA_PAD)) * sizeof(float);
}

template <int HD>
__global__ void __launch_bounds__(256) flash_attention_kernel(const float *q, int ldq, const float *kcache,
                                                              const float *vcache, float *out, int ldo, int count,
                                                              int nh, int kvh, int capacity, const int *pos_dev,
                                                              int pos0) {
  static_assert(HD == 16 || HD == 32 || HD == 64 || HD == 128, "head size");
  constexpr int DPT = HD / 16;  // output dimensions per thread
  extern __shared__ float fsm[];
  float *Qs = fsm;                           // [HD][BQ]        d-major
  float *Ks = Qs + HD * FA_BQ;               // [HD][BK + PAD]  d-major
  float *Vs = Ks + HD * (FA_BK + FA_PAD);    // [BK][HD]
  float *Ps = Vs + FA_BK * HD;               // [BK][BQ + PAD]  key-major
  pdl_wait();
  pdl_trigger();
  const int t0 = blockIdx.x * FA_BQ, h = blockIdx.y, b = blockIdx.z;
  const int g = h / (nh / kvh);
  const int base = pos_dev ? *pos_dev : pos0;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int nq = min(FA_BQ, count - t0);
  const int nkeys = base + t0 + nq;  // keys 0 .. position of the tile's last query
  const float scale = (float)(1.0 / sqrt((double)HD));
  const float *kb = kcache + ((size_t)b * kvh + g) * capacity * HD;
  const float *vb = vcache + ((size_t)b * kvh + g) * capacity * HD;

  for (int idx = tid; idx < FA_BQ * (HD / 4); idx += 256) {
    const int i = idx / (HD / 4), d = (idx % (HD / 4)) * 4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (i < nq) v = *reinterpret_cast<const float4 *>(q + (size_t)(b * count + t0 + i) * ldq + (size_t)h * HD + d);
    Qs[(d + 0) * FA_BQ + i] = v.x;
    Qs[(d + 1) * FA_BQ + i] = v.y;
    Qs[(d + 2) * FA_BQ + i] = v.z;
    Qs[(d + 3) * FA_BQ + i] = v.w;
  }

  float o[4][DPT];
  float mrow[4], lrow[4];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    mrow[i] = -INFINITY;
    lrow[i] = 0.0f;
#pragma unroll
    for (int e = 0; e < DPT; e++) o[i][e] = 0.0f;
  }

  for (int j0 = 0; j0 < nkeys; j0 += FA_BK) {
    __syncthreads();  // previous tile's K, V and P are no longer read
    for (int idx = tid; idx < FA_BK * (HD / 4); idx += 256) {
      const int jj = idx / (HD / 4), d = (idx % (HD / 4)) * 4;
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
      if (j0 + jj < nkeys) {
        kv = *reinterpret_cast<const float4 *>(kb + (size_t)(j0 + jj) * HD + d);
        vv = *reinterpret_cast<const float4 *>(vb + (size_t)(j0 + jj) * HD + d);
      }
      Ks[(d + 0) * (FA_BK + FA_PAD) + jj] = kv.x;
      Ks[(d + 1) * (FA_BK + FA_PAD) + jj] = kv.y;
      Ks[(d + 2) * (FA_BK + FA_PAD) + jj] = kv.z;
      Ks[(d + 3) * (FA_BK + FA_PAD) + jj] = kv.w;
      *reinterpret_cast<float4 *>(Vs + jj * HD + d) = vv;
    }
    __syncthreads();

    float s[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
      for (int jj = 0; jj < 4; jj++) s[i][jj] = 0.0f;
#pragma unroll 8
    for (int d = 0; d < HD; d++) {
      const float4 qv = *reinterpret_cast<const float4 *>(Qs + d * FA_BQ + 4 * ty);
      const float4 kv = *reinterpret_cast<const float4 *>(Ks + d * (FA_BK + FA_PAD) + 4 * tx);
      const float qa[4] = {qv.x, qv.y, qv.z, qv.w}, ka[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int jj = 0; jj < 4; jj++) s[i][jj] = fmaf(qa[i], ka[jj], s[i][jj]);
    }

#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int qpos = base + t0 + 4 * ty + i;
      float mt = -INFINITY;
#pragma unroll
      for (int jj = 0; jj < 4; jj++) {
        const int key = j0 + 4 * tx + jj;
        s[i][jj] = key <= qpos ? s[i][jj] * scale : -INFINITY;
        mt = fmaxf(mt, s[i][jj]);
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, off));
      const float mnew = fmaxf(mrow[i], mt);
      const float alpha = mnew == -INFINITY ? 1.0f : expf(mrow[i] - mnew);
      float rs = 0.0f;
#pragma unroll
      for (int jj = 0; jj < 4; jj++) {
        const float p = mnew == -INFINITY ? 0.0f : expf(s[i][jj] - mnew);
        s[i][jj] = p;
        rs += p;
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, off);
      lrow[i] = lrow[i] * alpha + rs;
      mrow[i] = mnew;
#pragma unroll
      for (int e = 0; e < DPT; e++) o[i][e] *= alpha;
    }
#pragma unroll
    for (int jj = 0; jj < 4; jj++)
      *reinterpret_cast<float4 *>(Ps + (4 * tx + jj) * (FA_BQ + FA_PAD) + 4 * ty) =
          make_float4(s[0][jj], s[1][jj], s[2][jj], s[3][jj]);
    __syncthreads();

    const int kmax = min(FA_BK, nkeys - j0);
    for (int jj = 0; jj < kmax; jj++) {
      const float4 pv = *reinterpret_cast<const float4 *>(Ps + jj * (FA_BQ + FA_PAD) + 4 * ty);
      const float pa[4] = {pv.x, pv.y, pv.z, pv.w};
      float va[DPT];
      if constexpr (DPT >= 4) {
#pragma unroll
        for (int c = 0; c < DPT / 4; c++) {
          const float4 v = *reinterpret_cast<const float4 *>(Vs + jj * HD + 64 * c + 4 * tx);
          va[4 * c + 0] = v.x;
          va[4 * c + 1] = v.y;
          va[4 * c + 2] = v.z;
          va[4 * c + 3] = v.w;
        }
      } else if constexpr (DPT == 2) {
        const float2 v = *reinterpret_cast<const float2 *>(Vs + jj * HD + 2 * tx);
        va[0] = v.x;
        va[1] = v.y;
      } else {
        va[0] = Vs[jj * HD + tx];
      }
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int e = 0; e < DPT; e++) o[i][e] = fmaf(pa[i], va[e], o[i][e]);
    }
  }

#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int t = t0 + 4 * ty + i;
    if (4 * ty + i >= nq) continue;
    float *orow = out + (size_t)(b * count + t) * ldo + (size_t)h * HD;
    const float inv = 1.0f / lrow[i];
#pragma unroll
    for (int e = 0; e < DPT; e++) {
      const int d = DPT >= 4 ? 64 * (e / 4) + 4 * tx + (e % 4) : (DPT == 2 ? 2 * tx + e : tx);
      orow[d] = o[i][e] * inv;
    }
  }
}

// Decode attention (one query token per batch row) in Float32, split over keys and shared by the
// query heads of a KV group: block (split s, KV head, token row) takes keys [128 s, 128 s + 128) of
// the visible range for all G = nh / kvh query heads of the group, so each K and V row is read once
// per group.  Decode is latency-bound, so every thread issues its K half-row and its V rows into
// registers at the start (one memory round trip for the whole block), then: scores by two threads
// per key (FMA over half of hd, one xor shuffle), per head max and sum of exp over the split (a warp
// per head), the weighted V sum by (key group, dimension quad) threads with the key groups added in
// order through shared memory.  A single split writes the normalised output; otherwise each split
// stores (max, sum, unnormalised sum) and the last split to finish (a per-(row, KV head) counter,
// reset by that block) merges them in split order, rescaling by exp(max_s - max).
constexpr int RA_KPS = 128, RA_GMAX = 8, RA_THREADS = 256;

// KPS keys per split: 128 (two threads per key) or, for head sizes up to 64 when the 128-key grid
// would leave SMs idle, 256 (one thread per key, one split for contexts up to 256 keys).
template <int HD, int KPS>
__global__ void __launch_bounds__(RA_THREADS) decode_attention_reg_kernel(
    const float *q, int ldq, const float *kcache, const float *vcache, float *out, int ldo, int count, int nh,
    int kvh, int capacity, const int *pos_dev, int pos0, float *part, int *counters, int smax) {
  static_assert(HD == 16 || HD == 32 || HD == 64 || HD == 128, "head size");
  static_assert(KPS == 128 || KPS == 256, "keys per split");
  constexpr int TPK = RA_THREADS / KPS, SEG = HD / TPK, NK4 = SEG / 4;
  constexpr int F = HD / 4, KG = RA_THREADS / F, VPT = KPS / KG;
  __shared__ __align__(16) float qs[RA_GMAX][HD];
  __shared__ float sp[RA_GMAX][KPS];
  __shared__ float red[RA_GMAX][2];
  __shared__ __align__(16) float opart[KG][RA_GMAX][HD];
  __shared__ int s_last;
  // Before the programmatic-dependency wait: the position (written by the previous step's finalize,
  // a graph launch earlier) and every K/V row but the newest (written by earlier steps).  The newest
  // row and q come from the projection kernel just before this one: loaded after the wait.
  pdl_trigger();
  const int split = blockIdx.x, g0 = blockIdx.y, m = blockIdx.z;
  const int G = nh / kvh;
  const int b = m / count, t = m % count;
  const int keys = (pos_dev ? *pos_dev : pos0) + t + 1;
  const int S = (keys + KPS - 1) / KPS;
  if (split >= S) return;  // the grid covers the longest visible range
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int j0 = split * KPS, nk = min(KPS, keys - j0);
  const int fresh = keys - 1 - j0;  // this split's index of the newest key (may be outside [0, nk))
  const size_t kvrow0 = ((size_t)b * kvh + g0) * capacity + j0;
  const float scale = (float)(1.0 / sqrt((double)HD));

  // every load of the block in flight at once
  const int jj = tid / TPK, hf = tid % TPK;  // score role: key jj, dimension segment hf
  const int f = tid % F, kg = tid / F;    // value role: dimensions 4f..4f+3 of keys kg, kg + KG, ...
  float4 kreg[NK4], vreg[VPT];
#pragma unroll
  for (int i = 0; i < NK4; i++)
    kreg[i] = jj < nk && jj != fresh
                  ? *reinterpret_cast<const float4 *>(kcache + (kvrow0 + jj) * HD + hf * SEG + 4 * i)
                  : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int i = 0; i < VPT; i++) {
    const int j = kg + i * KG;
    vreg[i] = j < nk && j != fresh ? *reinterpret_cast<const float4 *>(vcache + (kvrow0 + j) * HD + 4 * f)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  pdl_wait();
  if (jj == fresh) {
#pragma unroll
    for (int i = 0; i < NK4; i++)
      kreg[i] = *reinterpret_cast<const float4 *>(kcache + (kvrow0 + jj) * HD + hf * SEG + 4 * i);
  }
#pragma unroll
  for (int i = 0; i < VPT; i++) {
    const int j = kg + i * KG;
    if (j == fresh) vreg[i] = *reinterpret_cast<const float4 *>(vcache + (kvrow0 + j) * HD + 4 * f);
  }
  for (int i = tid; i < G * HD; i += RA_THREADS)
    qs[i / HD][i % HD] = q[(size_t)m * ldq + (size_t)(g0 * G) * HD + i];
  __syncthreads();

  {  // scores
    float dots[RA_GMAX];
#pragma unroll
    for (int g = 0; g < RA_GMAX; g++) {
      dots[g] = 0.0f;
      if (g < G) {
#pragma unroll
        for (int i = 0; i < NK4; i++) {
          const float4 qv = *reinterpret_cast<const float4 *>(&qs[g][hf * SEG + 4 * i]);
          dots[g] = fmaf(qv.x, kreg[i].x, dots[g]);
          dots[g] = fmaf(qv.y, kreg[i].y, dots[g]);
          dots[g] = fmaf(qv.z, kreg[i].z, dots[g]);
          dots[g] = fmaf(qv.w, kreg[i].w, dots[g]);
        }
      }
    }
    if constexpr (TPK == 2) {
#pragma unroll
      for (int g = 0; g < RA_GMAX; g++) dots[g] += __shfl_xor_sync(0xffffffffu, dots[g], 1);
    }
    if (hf == 0 && jj < nk) {
#pragma unroll
      for (int g = 0; g < RA_GMAX; g++)
        if (g < G) sp[g][jj] = dots[g] * scale;
    }
  }
  __syncthreads();
  for (int g = warp; g < G; g += RA_THREADS / 32) {  // per head: max and sum of exp over the split
    float mx = -INFINITY;
    for (int j = lane; j < nk; j += 32) mx = fmaxf(mx, sp[g][j]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    float sum = 0.0f;
    for (int j = lane; j < nk; j += 32) {
      const float e = expf(sp[g][j] - mx);
      sp[g][j] = e;
      sum += e;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    if (lane == 0) {
      red[g][0] = mx;
      red[g][1] = sum;
    }
  }
  __syncthreads();
  {  // unnormalised weighted V sum
#pragma unroll
    for (int g = 0; g < RA_GMAX; g++) {
      if (g < G) {
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
        for (int i = 0; i < VPT; i++) {
          const int j = kg + i * KG;
          const float p = j < nk ? sp[g][j] : 0.0f;
          a0 = fmaf(p, vreg[i].x, a0);
          a1 = fmaf(p, vreg[i].y, a1);
          a2 = fmaf(p, vreg[i].z, a2);
          a3 = fmaf(p, vreg[i].w, a3);
        }
        *reinterpret_cast<float4 *>(&opart[kg][g][4 * f]) = make_float4(a0, a1, a2, a3);
      }
    }
  }
  __syncthreads();
  const size_t slot = ((size_t)m * kvh + g0) * smax;  // this (row, KV head)'s split records
  float *po = part, *pml = part + (size_t)gridDim.z * kvh * smax * RA_GMAX * HD;
  for (int i = tid; i < G * HD; i += RA_THREADS) {
    const int g = i / HD, d = i % HD;
    float o = 0.0f;
    for (int k = 0; k < KG; k++) o += opart[k][g][d];
    if (S == 1) out[(size_t)m * ldo + (size_t)(g0 * G + g) * HD + d] = o / red[g][1];
    else po[((slot + split) * RA_GMAX + g) * HD + d] = o;
  }
  if (S == 1) return;
  if (tid < G) {
    pml[((slot + split) * RA_GMAX + tid) * 2 + 0] = red[tid][0];
    pml[((slot + split) * RA_GMAX + tid) * 2 + 1] = red[tid][1];
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(&counters[(size_t)m * kvh + g0], 1) == S - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int i = tid; i < G * HD; i += RA_THREADS) {
    const int g = i / HD, d = i % HD;
    float M = -INFINITY;
    for (int s = 0; s < S; s++) M = fmaxf(M, __ldcg(&pml[((slot + s) * RA_GMAX + g) * 2]));
    float num = 0.0f, den = 0.0f;
    for (int s = 0; s < S; s++) {
      const float w = expf(__ldcg(&pml[((slot + s) * RA_GMAX + g) * 2]) - M);
      num = fmaf(w, __ldcg(&po[((slot + s) * RA_GMAX + g) * HD + d]), num);
      den = fmaf(w, __ldcg(&pml[((slot + s) * RA_GMAX + g) * 2 + 1]), den);
    }
    out[(size_t)m * ldo + (size_t)(g0 * G + g) * HD + d] = num / den;
  }
  if (tid == 0) counters[(size_t)m * kvh + g0] = 0;
}

// Floats of split records decode_attention_reg_kernel needs for `rows` token rows.
size_t decode_attention_reg_part_floats(int rows, int kvh, int capacity, int hd) {
  const size_t smax = (size_t)(capacity + RA_KPS - 1) / RA_KPS;
  return (size_t)rows * kvh * smax * RA_GMAX * ((size_t)hd + 2);
}

// Launches the split decode attention when the head size and group size have a form (hd in
// {16, 32, 64, 128}, nh / kvh <= 8) and STB_DECODE_ATTENTION is not 0; returns false otherwise.
bool launch_decode_attention_reg(const float *q, int ldq, const float *kc, const float *vc, float *out, int ldo,
                             int rows, int count, int nh, int kvh, int hd, int capacity, const int *posd, int pos0,
                             float *part, int *counters, bool pdl, cudaStream_t st) {
  static const int enabled = env_int("STB_DECODE_ATTENTION", 1);
  if (!enabled || !part || !counters || nh % kvh != 0 || nh / kvh > RA_GMAX) return false;
  const int smax128 = (capacity + RA_KPS - 1) / RA_KPS;
  // 256-key splits when 128-key splits would not fill the SMs anyway (small batch, few KV heads)
  const bool wide = hd <= 64 && (long)rows * kvh * smax128 < 148;
  const int smax = wide ? (capacity + 255) / 256 : smax128;
  const dim3 grid(smax, kvh, rows);
#define STB_RA_LAUNCH(HDV, KPSV)                                                                                   \
  launch_kernel(decode_attention_reg_kernel<HDV, KPSV>, grid, dim3(RA_THREADS), 0, st, pdl, q, ldq, kc, vc, out, ldo,   \
                count, nh, kvh, capacity, posd, pos0, part, counters, smax)
  switch (hd) {
    case 16:
      if (wide) STB_RA_LAUNCH(16, 256);
      else STB_RA_LAUNCH(16, 128);
      return true;
    case 32:
      if (wide) STB_RA_LAUNCH(32, 256);
      else STB_RA_LAUNCH(32, 128);
      return true;
    case 64:
      if (wide) STB_RA_LAUNCH(64, 256);
      else STB_RA_LAUNCH(64, 128);
      return true;
    case 128: STB_RA_LAUNCH(128, 128); return true;
    default: return false;
  }
#undef STB_RA_LAUNCH
}

// Decode attention (one query token per batch row) in Float32, split over keys and shared by the
// query heads of a KV group: block (split s, KV head, token row) takes keys [KPS s, KPS s + KPS) of
// the visible range for all G = nh / kvh query heads of the group, so each K and V row is read once
// per group.  The cache keeps a (row, KV head)'s keys contiguous, so one thread moves the split's K
// and V rows into shared memory with two bulk copies (cp.async.bulk, TMA's 1-D form, this GPU's own
// memory, no multicast) issued before the programmatic-dependency wait -- every row but the newest,
// which the projection just before this kernel wrote and the threads load after the wait.  Blocks
// are small (128 threads, 2 * KPS * hd * 4 bytes of shared memory) and KPS adapts to the grid, so
// several blocks per SM keep the cache streaming.  Scores: each warp takes keys w, w + 4, ...; a lane
// holds hd/32 dimensions of the G query rows and of the key row; the G partial dots are reduced
// across the warp in one butterfly (9 shuffles for 8 heads).  Softmax per head by a warp, the
// weighted V sum per key by the same key split, warp partials added in order through shared memory.
// A single split writes the normalised output; otherwise each split stores (max, sum, unnormalised
// sum) and the last split to finish (a per-(row, KV head) counter, reset by that block) merges them
// in split order, rescaling by exp(max_s - max).  The copy wait is bounded (2 s, then the session's
// error word is set and the block leaves without writing).
constexpr int DA_GMAX = 8, DA_THREADS = 128, DA_WARPS = DA_THREADS / 32, DA_KPS_MIN = 32;

template <int HD, int KPS>
constexpr size_t da_smem() {
  return (size_t)2 * KPS * HD * 4 + (size_t)DA_GMAX * KPS * 4 + DA_GMAX * 2 * 4 + 16;
}

template <int HD, int KPS>
__global__ void __launch_bounds__(DA_THREADS) decode_attention_kernel(
    const float *q, int ldq, const float *kcache, const float *vcache, float *out, int ldo, int count, int nh,
    int kvh, int capacity, const int *pos_dev, int pos0, float *part, int *counters, int smax, int *err) {
  static_assert(HD == 32 || HD == 64 || HD == 128, "head size");
  static_assert(KPS % (4 * DA_WARPS) == 0 && KPS >= DA_KPS_MIN, "keys per split");
  static_assert(DA_WARPS * DA_GMAX * HD <= KPS * HD, "warp partials reuse the K tile");
  constexpr int DPL = HD / 32;  // dimensions per lane
  extern __shared__ __align__(128) uint8_t da_raw[];
  float *Ks = (float *)da_raw;               // [KPS][HD]
  float *Vs = Ks + KPS * HD;                 // [KPS][HD]
  float *sp = Vs + KPS * HD;                 // [G][KPS] scores, then probabilities
  float *red = sp + DA_GMAX * KPS;           // [G][2] max, sum
  uint64_t *bar = (uint64_t *)(red + DA_GMAX * 2);
  __shared__ int s_last, s_ok;
  __shared__ volatile int s_abort;
  pdl_trigger();
  const int split = blockIdx.x, g0 = blockIdx.y, m = blockIdx.z;
  const int G = nh / kvh;
  const int b = m / count, t = m % count;
  // position: written by the previous step's finalize, a graph launch earlier
  const int keys = (pos_dev ? *pos_dev : pos0) + t + 1;
  const int S = (keys + KPS - 1) / KPS;
  if (split >= S) return;  // the grid covers the longest visible range
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int j0 = split * KPS, nk = min(KPS, keys - j0);
  const int fresh = keys - 1 - j0;      // this split's index of the newest key (in [0, nk) only in the last split)
  const int old = fresh < nk ? fresh : nk;  // rows [0, old) were written by earlier steps
  const size_t kvrow0 = ((size_t)b * kvh + g0) * capacity + j0;
  const uint32_t bar_a = tc::smem_u32(bar);
  if (tid == 0) {
    s_abort = 0;
    tc::mbar_init(bar_a, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    if (old > 0) {
      const uint32_t bytes = (uint32_t)old * HD * 4;
      tc::mbar_expect_tx(bar_a, 2 * bytes);
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                       tc::smem_u32(Ks)),
                   "l"(kcache + kvrow0 * HD), "r"(bytes), "r"(bar_a)
                   : "memory");
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                       tc::smem_u32(Vs)),
                   "l"(vcache + kvrow0 * HD), "r"(bytes), "r"(bar_a)
                   : "memory");
    } else {
      tc::mbar_arrive(bar_a);
    }
  }
  __syncthreads();
  pdl_wait();
  if (fresh < nk) {  // the newest key, written by the projection just before this kernel
    for (int i = tid; i < HD; i += DA_THREADS) {
      Ks[fresh * HD + i] = kcache[(kvrow0 + fresh) * HD + i];
      Vs[fresh * HD + i] = vcache[(kvrow0 + fresh) * HD + i];
    }
  }
  float qr[DA_GMAX][DPL];
#pragma unroll
  for (int g = 0; g < DA_GMAX; g++)
#pragma unroll
    for (int d = 0; d < DPL; d++)
      qr[g][d] = g < G ? q[(size_t)m * ldq + (size_t)(g0 * G + g) * HD + lane * DPL + d] : 0.0f;
  if (tid == 0) {
    s_ok = tc::mbar_wait(bar_a, 0, &s_abort, err, 40);
    if (!s_ok) {  // leave only once the copies into this block's shared memory are done (bounded again)
      volatile int no_abort = 0;
      tc::mbar_wait(bar_a, 0, &no_abort, err, 41);
    }
  }
  __syncthreads();
  if (!s_ok) return;
  const float scale = (float)(1.0 / sqrt((double)HD));

  // scores: warp w takes the key quads [4 w + 16 i, 4 w + 16 i + 4); a lane sums its dimensions for the
  // 4 keys x 8 heads, then one reduce-scatter butterfly (31 shuffles, 5 levels) leaves lane l with
  // the whole dot of key l / 8 and head l % 8.
  for (int jb = 4 * warp; jb < nk; jb += 4 * DA_WARPS) {
    float a[32];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      float kv[DPL];
#pragma unroll
      for (int d = 0; d < DPL; d++) kv[d] = jb + k < nk ? Ks[(jb + k) * HD + lane * DPL + d] : 0.0f;
#pragma unroll
      for (int g = 0; g < DA_GMAX; g++) {
        float sacc = 0.0f;
#pragma unroll
        for (int d = 0; d < DPL; d++) sacc = fmaf(qr[g][d], kv[d], sacc);
        a[k * DA_GMAX + g] = sacc;
      }
    }
#pragma unroll
    for (int half = 16; half >= 1; half >>= 1) {
      const bool up = lane & half;
#pragma unroll
      for (int i = 0; i < half; i++) {
        const float send = up ? a[i] : a[i + half], keep = up ? a[i + half] : a[i];
        a[i] = keep + __shfl_xor_sync(0xffffffffu, send, half);
      }
    }
    const int k = lane >> 3, h = lane & 7;
    if (h < G && jb + k < nk) sp[h * KPS + jb + k] = a[0] * scale;
  }
  __syncthreads();
  for (int g = warp; g < G; g += DA_WARPS) {  // per head: max and sum of exp over the split
    float mx = -INFINITY;
    for (int j = lane; j < nk; j += 32) mx = fmaxf(mx, sp[g * KPS + j]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    float sum = 0.0f;
    for (int j = lane; j < nk; j += 32) {
      const float e = expf(sp[g * KPS + j] - mx);
      sp[g * KPS + j] = e;
      sum += e;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    if (lane == 0) {
      red[g * 2] = mx;
      red[g * 2 + 1] = sum;
    }
  }
  __syncthreads();
  float acc[DA_GMAX][DPL];
#pragma unroll
  for (int g = 0; g < DA_GMAX; g++)
#pragma unroll
    for (int d = 0; d < DPL; d++) acc[g][d] = 0.0f;
  for (int j = warp; j < nk; j += DA_WARPS) {  // unnormalised weighted V sum
    float vv[DPL];
#pragma unroll
    for (int d = 0; d < DPL; d++) vv[d] = Vs[j * HD + lane * DPL + d];
#pragma unroll
    for (int g = 0; g < DA_GMAX; g++) {
      if (g < G) {
        const float p = sp[g * KPS + j];
#pragma unroll
        for (int d = 0; d < DPL; d++) acc[g][d] = fmaf(p, vv[d], acc[g][d]);
      }
    }
  }
  float *opart = Ks;  // [warp][G][HD]: the K tile is no longer read
#pragma unroll
  for (int g = 0; g < DA_GMAX; g++)
    if (g < G)
#pragma unroll
      for (int d = 0; d < DPL; d++) opart[(warp * DA_GMAX + g) * HD + lane * DPL + d] = acc[g][d];
  __syncthreads();
  const size_t slot = ((size_t)m * kvh + g0) * smax;  // this (row, KV head)'s split records
  float *po = part, *pml = part + (size_t)gridDim.z * kvh * smax * DA_GMAX * HD;
  for (int i = tid; i < G * HD; i += DA_THREADS) {
    const int g = i / HD, d = i % HD;
    float o = 0.0f;
#pragma unroll
    for (int w = 0; w < DA_WARPS; w++) o += opart[(w * DA_GMAX + g) * HD + d];
    if (S == 1) out[(size_t)m * ldo + (size_t)(g0 * G + g) * HD + d] = o / red[g * 2 + 1];
    else po[((slot + split) * DA_GMAX + g) * HD + d] = o;
  }
  if (S == 1) return;
  if (tid < G) {
    pml[((slot + split) * DA_GMAX + tid) * 2 + 0] = red[tid * 2];
    pml[((slot + split) * DA_GMAX + tid) * 2 + 1] = red[tid * 2 + 1];
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(&counters[(size_t)m * kvh + g0], 1) == S - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int i = tid; i < G * HD; i += DA_THREADS) {
    const int g = i / HD, d = i % HD;
    float M = -INFINITY;
    for (int s = 0; s < S; s++) M = fmaxf(M, __ldcg(&pml[((slot + s) * DA_GMAX + g) * 2]));
    float num = 0.0f, den = 0.0f;
    for (int s = 0; s < S; s++) {
      const float w = expf(__ldcg(&pml[((slot + s) * DA_GMAX + g) * 2]) - M);
      num = fmaf(w, __ldcg(&po[((slot + s) * DA_GMAX + g) * HD + d]), num);
      den = fmaf(w, __ldcg(&pml[((slot + s) * DA_GMAX + g) * 2 + 1]), den);
    }
    out[(size_t)m * ldo + (size_t)(g0 * G + g) * HD + d] = num / den;
  }
  if (tid == 0) counters[(size_t)m * kvh + g0] = 0;
}

// Decode attention for head size 128, GQA groups of up to 8 query heads: the same blocks, split
// records and merge as decode_attention_kernel, with the arithmetic arranged so that no cross-lane
// reduction is needed.  Scores: lane (key k, head quad h4) of a warp computes the whole 128-term
// dot of key k with query heads 4 h4 .. 4 h4 + 3 (16 FMAs per 128-bit K load; the K rows land in
// shared memory padded to 132 floats by one bulk copy per row, so the 16 keys a warp reads fall in
// distinct banks, and the query rows are read as broadcasts).  Weighted V sum: warp w owns output
// dimensions 32 w .. 32 w + 31 of every head, so each lane runs over all keys with its own 8
// accumulators and no partials are combined across warps.  K and V complete on separate
// mbarriers: the scores start while V is still in flight.  The copy waits are bounded (2 s, then
// the session's error word is set and the block leaves without writing).
constexpr int DA2_KROW = 132;  // padded K row (floats)

template <int KPS>
constexpr size_t da2_smem() {
  return (size_t)KPS * DA2_KROW * 4 + (size_t)KPS * 128 * 4 + (size_t)DA_GMAX * DA2_KROW * 4 +
         (size_t)2 * DA_GMAX * KPS * 4 + DA_GMAX * 2 * 4 + 32;
}

template <int KPS>
__global__ void __launch_bounds__(DA_THREADS) decode_attention_hd128_kernel(
    const float *q, int ldq, const float *kcache, const float *vcache, float *out, int ldo, int count, int nh,
    int kvh, int capacity, const int *pos_dev, int pos0, float *part, int *counters, int smax, int *err) {
  constexpr int HD = 128;
  static_assert(KPS % 16 == 0 && KPS >= DA_KPS_MIN, "keys per split");
  extern __shared__ __align__(128) uint8_t da_raw[];
  float *Kp = (float *)da_raw;              // [KPS][DA2_KROW]
  float *Vs = Kp + KPS * DA2_KROW;          // [KPS][HD]
  float *Qs = Vs + KPS * HD;                // [G][DA2_KROW]
  float *sp = Qs + DA_GMAX * DA2_KROW;      // [G][KPS] scores, then probabilities
  float *pt = sp + DA_GMAX * KPS;           // [KPS][8] probabilities by key
  float *red = pt + DA_GMAX * KPS;          // [G][2] max, sum
  uint64_t *bar = (uint64_t *)(red + DA_GMAX * 2);  // [2]: K, V
  __shared__ int s_last, s_ok;
  __shared__ volatile int s_abort;
  pdl_trigger();
  const int split = blockIdx.x, g0 = blockIdx.y, m = blockIdx.z;
  const int G = nh / kvh;
  const int b = m / count, t = m % count;
  const int keys = (pos_dev ? *pos_dev : pos0) + t + 1;
  const int S = (keys + KPS - 1) / KPS;
  if (split >= S) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int j0 = split * KPS, nk = min(KPS, keys - j0);
  const int fresh = keys - 1 - j0;
  const int old = fresh < nk ? fresh : nk;  // rows [0, old) were written by earlier steps
  const size_t kvrow0 = ((size_t)b * kvh + g0) * capacity + j0;
  const uint32_t bar_k = tc::smem_u32(bar), bar_v = bar_k + 8;
  if (tid == 0) {
    s_abort = 0;
    tc::mbar_init(bar_k, 1);
    tc::mbar_init(bar_v, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (warp == 0) {
    if (lane == 0) {
      if (old > 0) {
        tc::mbar_expect_tx(bar_k, (uint32_t)old * HD * 4);
        tc::mbar_expect_tx(bar_v, (uint32_t)old * HD * 4);
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                         tc::smem_u32(Vs)),
                     "l"(vcache + kvrow0 * HD), "r"((uint32_t)old * HD * 4), "r"(bar_v)
                     : "memory");
      } else {
        tc::mbar_arrive(bar_k);
        tc::mbar_arrive(bar_v);
      }
    }
    __syncwarp();
    for (int r = lane; r < old; r += 32)  // one 512-byte copy per K row into its padded slot
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                       tc::smem_u32(Kp + r * DA2_KROW)),
                   "l"(kcache + (kvrow0 + r) * HD), "r"((uint32_t)HD * 4), "r"(bar_k)
                   : "memory");
  }
  pdl_wait();
  if (fresh < nk) {  // the newest key, written by the projection just before this kernel
    Kp[fresh * DA2_KROW + tid] = kcache[(kvrow0 + fresh) * HD + tid];
    Vs[fresh * HD + tid] = vcache[(kvrow0 + fresh) * HD + tid];
  }
  for (int i = tid; i < DA_GMAX * (HD / 4); i += DA_THREADS) {  // the group's query rows (zero past G)
    const int g = i / (HD / 4), d4 = i % (HD / 4);
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (g < G) v = *(const float4 *)(q + (size_t)m * ldq + (size_t)(g0 * G + g) * HD + d4 * 4);
    *(float4 *)(Qs + g * DA2_KROW + d4 * 4) = v;
  }
  if (tid == 0) {
    s_ok = tc::mbar_wait(bar_k, 0, &s_abort, err, 42);
    if (!s_ok) {  // leave only once every copy into this block's shared memory is done (bounded again)
      volatile int no_abort = 0;
      tc::mbar_wait(bar_k, 0, &no_abort, err, 42);
      tc::mbar_wait(bar_v, 0, &no_abort, err, 43);
    }
  }
  __syncthreads();
  if (!s_ok) return;
  const float scale = (float)(1.0 / sqrt((double)HD));

  // scores: 16 keys x 2 head quads per warp pass (32 keys x 1 quad when G <= 4)
  {
    const int quads = G > 4 ? 2 : 1, kpw = 32 / quads;
    const int kk = lane % kpw, h4 = lane / kpw;
    for (int jb = warp * kpw; jb < nk; jb += DA_WARPS * kpw) {
      const int j = jb + kk;
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      if (j < nk) {
        const float *kr = Kp + j * DA2_KROW;
        const float *qr = Qs + 4 * h4 * DA2_KROW;
#pragma unroll 8
        for (int d = 0; d < HD; d += 4) {
          const float4 kv = *(const float4 *)(kr + d);
#pragma unroll
          for (int h = 0; h < 4; h++) {
            const float4 qv = *(const float4 *)(qr + h * DA2_KROW + d);
            acc[h] = fmaf(qv.x, kv.x, acc[h]);
            acc[h] = fmaf(qv.y, kv.y, acc[h]);
            acc[h] = fmaf(qv.z, kv.z, acc[h]);
            acc[h] = fmaf(qv.w, kv.w, acc[h]);
          }
        }
#pragma unroll
        for (int h = 0; h < 4; h++)
          if (4 * h4 + h < G) sp[(4 * h4 + h) * KPS + j] = acc[h] * scale;
      }
    }
  }
  __syncthreads();
  for (int g = warp; g < G; g += DA_WARPS) {  // per head: max and sum of exp over the split
    float mx = -INFINITY;
    for (int j = lane; j < nk; j += 32) mx = fmaxf(mx, sp[g * KPS + j]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    float sum = 0.0f;
    for (int j = lane; j < nk; j += 32) {
      const float e = expf(sp[g * KPS + j] - mx);
      pt[j * DA_GMAX + g] = e;
      sum += e;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    if (lane == 0) {
      red[g * 2] = mx;
      red[g * 2 + 1] = sum;
    }
  }
  if (tid == 0) {
    s_ok = tc::mbar_wait(bar_v, 0, &s_abort, err, 43);
    if (!s_ok) {
      volatile int no_abort = 0;
      tc::mbar_wait(bar_v, 0, &no_abort, err, 43);
    }
  }
  __syncthreads();
  if (!s_ok) return;
  // weighted V sum: lane owns dimension d of every head
  const int d = warp * 32 + lane;
  float acc[DA_GMAX];
#pragma unroll
  for (int g = 0; g < DA_GMAX; g++) acc[g] = 0.0f;
#pragma unroll 4
  for (int j = 0; j < nk; j++) {
    const float v = Vs[j * HD + d];
    const float4 pa = *(const float4 *)(pt + j * DA_GMAX), pb = *(const float4 *)(pt + j * DA_GMAX + 4);
    acc[0] = fmaf(pa.x, v, acc[0]);
    acc[1] = fmaf(pa.y, v, acc[1]);
    acc[2] = fmaf(pa.z, v, acc[2]);
    acc[3] = fmaf(pa.w, v, acc[3]);
    acc[4] = fmaf(pb.x, v, acc[4]);
    acc[5] = fmaf(pb.y, v, acc[5]);
    acc[6] = fmaf(pb.z, v, acc[6]);
    acc[7] = fmaf(pb.w, v, acc[7]);
  }
  const size_t slot = ((size_t)m * kvh + g0) * smax;
  float *po = part, *pml = part + (size_t)gridDim.z * kvh * smax * DA_GMAX * HD;
  if (S == 1) {
#pragma unroll
    for (int g = 0; g < DA_GMAX; g++)
      if (g < G) out[(size_t)m * ldo + (size_t)(g0 * G + g) * HD + d] = acc[g] / red[g * 2 + 1];
    return;
  }
#pragma unroll
  for (int g = 0; g < DA_GMAX; g++)
    if (g < G) po[((slot + split) * DA_GMAX + g) * HD + d] = acc[g];
  if (tid < G) {
    pml[((slot + split) * DA_GMAX + tid) * 2 + 0] = red[tid * 2];
    pml[((slot + split) * DA_GMAX + tid) * 2 + 1] = red[tid * 2 + 1];
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(&counters[(size_t)m * kvh + g0], 1) == S - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int i = tid; i < G * HD; i += DA_THREADS) {  // the last split merges all, in split order
    const int g = i / HD, dd = i % HD;
    float M = -INFINITY;
    for (int s = 0; s < S; s++) M = fmaxf(M, __ldcg(&pml[((slot + s) * DA_GMAX + g) * 2]));
    float num = 0.0f, den = 0.0f;
    for (int s = 0; s < S; s++) {
      const float w = expf(__ldcg(&pml[((slot + s) * DA_GMAX + g) * 2]) - M);
      num = fmaf(w, __ldcg(&po[((slot + s) * DA_GMAX + g) * HD + dd]), num);
      den = fmaf(w, __ldcg(&pml[((slot + s) * DA_GMAX + g) * 2 + 1]), den);
    }
    out[(size_t)m * ldo + (size_t)(g0 * G + g) * HD + dd] = num / den;
  }
  if (tid == 0) counters[(size_t)m * kvh + g0] = 0;
}

// Floats of split records decode_attention_kernel needs for `rows` token rows (sized for the
// smallest split, DA_KPS_MIN keys).
size_t decode_attention_part_floats(int rows, int kvh, int capacity, int hd) {
  const size_t smax = (size_t)(capacity + DA_KPS_MIN - 1) / DA_KPS_MIN;
  return (size_t)rows * kvh * smax * DA_GMAX * ((size_t)hd + 2);
}

template <int HD, int KPS>
void da_launch(dim3 grid, bool pdl, cudaStream_t st, int device, const float *q, int ldq, const float *kc,
               const float *vc, float *out, int ldo, int count, int nh, int kvh, int capacity, const int *posd,
               int pos0, float *part, int *counters, int smax, int *err) {
  constexpr size_t smem = da_smem<HD, KPS>();
  if constexpr (smem > 48 * 1024) {
    static std::mutex mu;
    static bool configured[64] = {};
    std::lock_guard<std::mutex> lock(mu);
    if (device < 0 || device >= 64 || !configured[device]) {
      STB_CUDA(cudaFuncSetAttribute(decode_attention_kernel<HD, KPS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)smem));
      if (device >= 0 && device < 64) configured[device] = true;
    }
  }
  launch_kernel(decode_attention_kernel<HD, KPS>, grid, dim3(DA_THREADS), smem, st, pdl, q, ldq, kc, vc, out, ldo,
                count, nh, kvh, capacity, posd, pos0, part, counters, smax, err);
}

template <int KPS>
void da2_launch(dim3 grid, bool pdl, cudaStream_t st, int device, const float *q, int ldq, const float *kc,
                const float *vc, float *out, int ldo, int count, int nh, int kvh, int capacity, const int *posd,
                int pos0, float *part, int *counters, int smax, int *err) {
  constexpr size_t smem = da2_smem<KPS>();
  {
    static std::mutex mu;
    static bool configured[64] = {};
    std::lock_guard<std::mutex> lock(mu);
    if (device < 0 || device >= 64 || !configured[device]) {
      STB_CUDA(cudaFuncSetAttribute(decode_attention_hd128_kernel<KPS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)smem));
      if (device >= 0 && device < 64) configured[device] = true;
    }
  }
  launch_kernel(decode_attention_hd128_kernel<KPS>, grid, dim3(DA_THREADS), smem, st, pdl, q, ldq, kc, vc, out, ldo,
                count, nh, kvh, capacity, posd, pos0, part, counters, smax, err);
}

// Launches the split decode attention when the head size and group size have a form (hd in
// {32, 64, 128}, nh / kvh <= 8) and STB_DECODE_ATTENTION is not 0; returns false otherwise.  Keys per
// split: the smallest of 32 / 64 / 128 that keeps the grid within ~6 blocks per SM.  Head size 128
// takes decode_attention_hd128_kernel unless STB_DA_HD128 is 0.
bool launch_decode_attention(const float *q, int ldq, const float *kc, const float *vc, float *out, int ldo,
                             int rows, int count, int nh, int kvh, int hd, int capacity, const int *posd, int pos0,
                             float *part, int *counters, bool pdl, cudaStream_t st, int device, int *err) {
  static const int enabled = env_int("STB_DECODE_ATTENTION", 1);
  if (!enabled || !part || !counters || nh % kvh != 0 || nh / kvh > DA_GMAX) return false;
  if (hd != 32 && hd != 64 && hd != 128) return false;
  static const int forced = env_int("STB_DA_KPS", 0);  // 32 / 64 / 128 / 256: fixed keys per split
  const long units = (long)rows * kvh;
  const long budget = 6L * tc::sm_count(device);
  int kps = units * ((capacity + 31) / 32) <= budget ? 32 : (units * ((capacity + 63) / 64) <= budget ? 64 : 128);
  if (forced == 32 || forced == 64 || forced == 128 || (forced == 256 && hd <= 64)) kps = forced;
  const int smax = (capacity + kps - 1) / kps;
  const dim3 grid(smax, kvh, rows);
  static const int hd128 = env_int("STB_DA_HD128", 1);
  if (hd == 128 && hd128 && kps <= 128) {
    if (kps == 32)
      da2_launch<32>(grid, pdl, st, device, q, ldq, kc, vc, out, ldo, count, nh, kvh, capacity, posd, pos0, part,
                     counters, smax, err);
    else if (kps == 64)
      da2_launch<64>(grid, pdl, st, device, q, ldq, kc, vc, out, ldo, count, nh, kvh, capacity, posd, pos0, part,
                     counters, smax, err);
    else
      da2_launch<128>(grid, pdl, st, device, q, ldq, kc, vc, out, ldo, count, nh, kvh, capacity, posd, pos0, part,
                      counters, smax, err);
    return true;
  }
#define STB_DA(HDV, KPSV)                                                                                          \
  da_launch<HDV, KPSV>(grid, pdl, st, device, q, ldq, kc, vc, out, ldo, count, nh, kvh, capacity, posd, pos0, part, \
                       counters, smax, err)
#define STB_DA_HD(HDV)             \
  if (kps == 32) STB_DA(HDV, 32);      \
  else if (kps == 64) STB_DA(HDV, 64); \
  else STB_DA(HDV, 128);
  switch (hd) {
    case 32: STB_DA_HD(32); break;
    case 64:
      if (kps == 256) STB_DA(64, 256);
      else STB_DA_HD(64);
      break;
    default: STB_DA_HD(128); break;
  }
#undef STB_DA_HD
#undef STB_DA
  return true;
}

// Two forms of the split decode attention: the register form (every K/V load of a block issued into
// registers at entry, 256 threads, one memory round trip) is faster when the grid is small -- a few
// blocks, where latency is everything (SmolLM2-shaped batch 1: 1756 vs 1607 decode tokens/s) -- and the
// bulk-copy form when the grid spans the GPU several times (Llama-3-70B-shaped batch 8: 12 us less per
// layer).  The register form is chosen when its grid (128-key splits) has fewer blocks than SMs;
// STB_DA_IMPL = 0 / 1 forces the register / bulk-copy form.
bool use_register_attention(int rows, int kvh, int hd, int capacity, int device) {
  static const int forced = env_int("STB_DA_IMPL", -1);
  if (forced == 0 || forced == 1) return forced == 0;
  if (hd == 16) return true;  // the bulk-copy form has no head size 16
  return (long)rows * kvh * ((capacity + 127) / 128) < tc::sm_count(device);
}

template <int HD>
void flash_launch(dim3 grid, const float *q, int ldq, const float *kc, const float *vc, float *out, int ldo,
                  int count, int nh, int kvh, int capacity, const int *posd, int pos0, int device, cudaStream_t st) {
  static std::mutex mu;
  static bool configured[64] = {};  // per head size: one static set per instantiation
  {
    std::lock_guard<std::mutex> lock(mu);
    if (device < 0 || device >= 64 || !configured[device]) {
      STB_CUDA(cudaFuncSetAttribute(flash_attention_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)flash_smem<HD>()));
      if (device >= 0 && device < 64) configured[device] = true;
    }
  }
  launch_kernel(flash_attention_kernel<HD>, grid, dim3(256), flash_smem<HD>(), st, false, q, ldq, kc, vc, out, ldo,
                count, nh, kvh, capacity, posd, pos0);
}

// Launches the tiled prefill attention when the head size has an instantiation (16, 32, 64, 128)
// and STB_FLASH_ATTENTION is not 0; returns false otherwise.
bool launch_flash_attention(const float *q, int ldq, const float *kc, const float *vc, float *out, int ldo,
                            int rows, int count, int nh, int kvh, int hd, int capacity, const int *posd, int pos0,
                            int device, cudaStream_t st) {
  static const int enabled = env_int("STB_FLASH_ATTENTION", 1);
  if (!enabled || rows % count != 0) return false;
  const dim3 grid((count + FA_BQ - 1) / FA_BQ, nh, rows / count);
  switch (hd) {
    case 16: flash_launch<16>(grid, q, ldq, kc, vc, out, ldo, count, nh, kvh, capacity, posd, pos0, device, st); break;
    case 32: flash_launch<32>(grid, q, ldq, kc, vc, out, ldo, count, nh, kvh, capacity, posd, pos0, device, st); break;
    case 64: flash_launch<64>(grid, q, ldq, kc, vc, out, ldo, count, nh, kvh, capacity, posd, pos0, device, st); break;
    case 128:
      flash_launch<128>(grid, q, ldq, kc, vc, out, ldo, count, nh, kvh, capacity, posd, pos0, device, st);
      break;
    default: return false;
  }
  return true;
}

// Greedy pick from every rank's candidate key (argmax_key: largest logit, lowest id on ties --
// TokenSampler's strict '>'), token feedback, output append, EOS stop and position advance.  The
// local candidate slots are cleared for the next step.
__global__ void finalize_kernel(const unsigned long long *best_all, unsigned long long *best_local, int nranks,
                                int batch, int count, int64_t *tokens, int *state, int64_t *out_ids, int out_stride,
                                const int64_t *eos, int eos_count, int advance) {
  pdl_wait();
  if (state[1]) return;
  int *stopped = state + 2;
  int *out_count = state + 2 + batch;
  for (int b = threadIdx.x; b < batch; b += blockDim.x) {
    unsigned long long key = 0;
    for (int r = 0; r < nranks; r++) key = max(key, best_all[(size_t)r * batch + b]);
    const int besti = argmax_key_index(key);
    best_local[b] = 0ull;
    if (out_ids && !stopped[b]) {
      out_ids[(size_t)b * out_stride + out_count[b]] = besti;
      out_count[b] += 1;
      for (int e = 0; e < eos_count; e++)
        if (eos[e] == besti) stopped[b] = 1;
    }
    tokens[(size_t)b * count + (count - 1)] = besti;  // next step's input (count == 1 in decode)
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (advance) state[0] += advance;
    if (out_ids) {
      int all = 1;
      for (int b = 0; b < batch; b++) all &= stopped[b];
      state[1] = all;
    }
  }
}

// ---- tensor-core prefill helpers (chunks of >= tc_rows token rows)

// CpuFloatBackend.rmsNorm per row (CpuFloatBackend.scala:78-93), double accumulation; one block per row.
__global__ void rmsnorm_rows_kernel(const float *x, const float *w, double eps, float *out, int H) {
  __shared__ double s_red[8];
  pdl_wait();
  pdl_trigger();
  const float *xr = x + (size_t)blockIdx.x * H;
  double sq = 0.0;
  for (int k = threadIdx.x; k < H; k += blockDim.x) {
    const double v = (double)xr[k];
    sq = __dadd_rn(sq, __dmul_rn(v, v));
  }
  const double total = block_sum_double(sq, s_red);
  const double inv = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(total, (double)H), eps)));
  for (int k = threadIdx.x; k < H; k += blockDim.x)
    out[(size_t)blockIdx.x * H + k] = __double2float_rn(__dmul_rn(__dmul_rn((double)xr[k], inv), (double)w[k]));
}

// RoPE + KV append from a paired q/k/v projection row (the QKV GEMV epilogue's arithmetic, applied
// to a tensor-core GEMM output): one thread per (row, pair).
__global__ void rope_append_kernel(const float *qkv, int ldq, const double2 *rope, const int *pos_dev, int pos0,
                                   int count, int nh, int kvh, int hd, int capacity, float *q_out, int ldo,
                                   float *k_cache, float *v_cache, int rows) {
  pdl_wait();
  pdl_trigger();
  const int half = hd >> 1;
  const int pairs = (nh + 2 * kvh) * half;
  const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
  if (i >= (long)rows * pairs) return;
  const int mm = (int)(i / pairs), pi = (int)(i % pairs);
  const float fa = qkv[(size_t)mm * ldq + 2 * pi], fb = qkv[(size_t)mm * ldq + 2 * pi + 1];
  const int qpairs = nh * half, kpairs = kvh * half;
  const int bb = mm / count, t = mm % count;
  const int pos = (pos_dev ? *pos_dev : pos0) + t;
  if (pi < qpairs + kpairs) {
    const int local = pi < qpairs ? pi : pi - qpairs;
    const int h = local / half, d = local % half;
    const double2 cs = rope[(size_t)pos * half + d];
    const double a = (double)fa, b = (double)fb;
    const float oa = __double2float_rn(__dsub_rn(__dmul_rn(a, cs.x), __dmul_rn(b, cs.y)));
    const float ob = __double2float_rn(__dadd_rn(__dmul_rn(b, cs.x), __dmul_rn(a, cs.y)));
    float *dst = pi < qpairs ? q_out + (size_t)mm * ldo + (size_t)h * hd
                             : k_cache + (((size_t)bb * kvh + h) * capacity + pos) * hd;
    dst[d] = oa;
    dst[d + half] = ob;
  } else {
    const int local = pi - qpairs - kpairs;
    const int h = local / half, d = local % half;
    float *vc = v_cache + (((size_t)bb * kvh + h) * capacity + pos) * hd;
    vc[d] = fa;
    vc[d + half] = fb;
  }
}


// Float32 -> the weight type (BF16 round-to-nearest-even, or F16), for tensor-core operands.
__device__ __forceinline__ uint16_t to_half_bits(float v, bool bf16) {
  return bf16 ? f32_to_bf16_rne(v) : __half_as_ushort(__float2half_rn(v));
}

// rmsnorm_rows_kernel's arithmetic with the result rounded straight to the weight type for the next
// tensor-core GEMM (the Float32 row and the separate rounding pass are skipped; the two roundings,
// double -> Float32 -> half, are the same).  One block per row; the row stays in registers between
// the sum of squares and the scaling (H <= 8192 with 256 threads, H % 4 == 0).
template <bool BF16>
__global__ void __launch_bounds__(256) rmsnorm_round_kernel(const float *x, const float *w, double eps, uint16_t *out,
                                                            int H) {
  __shared__ double s_red[8];
  constexpr int CH = 8;  // float4 chunks per thread
  const float *xr = x + (size_t)blockIdx.x * H;
  float4 v[CH];
  double sq = 0.0;
#pragma unroll
  for (int j = 0; j < CH; j++) {
    const int c = threadIdx.x + 256 * j;
    v[j] = c * 4 < H ? *reinterpret_cast<const float4 *>(xr + c * 4) : make_float4(0.f, 0.f, 0.f, 0.f);
    const double a = v[j].x, b = v[j].y, cc = v[j].z, d = v[j].w;
    sq = __dadd_rn(sq, __dmul_rn(a, a));
    sq = __dadd_rn(sq, __dmul_rn(b, b));
    sq = __dadd_rn(sq, __dmul_rn(cc, cc));
    sq = __dadd_rn(sq, __dmul_rn(d, d));
  }
  const double total = block_sum_double(sq, s_red);
  const double inv = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(total, (double)H), eps)));
  uint16_t *orow = out + (size_t)blockIdx.x * H;
#pragma unroll
  for (int j = 0; j < CH; j++) {
    const int c = threadIdx.x + 256 * j;
    if (c * 4 >= H) break;
    const float4 wv = *reinterpret_cast<const float4 *>(w + c * 4);
    const float e[4] = {v[j].x, v[j].y, v[j].z, v[j].w}, ww[4] = {wv.x, wv.y, wv.z, wv.w};
    uint16_t h[4];
#pragma unroll
    for (int i = 0; i < 4; i++)
      h[i] = to_half_bits(__double2float_rn(__dmul_rn(__dmul_rn((double)e[i], inv), (double)ww[i])), BF16);
    *reinterpret_cast<uint2 *>(orow + c * 4) = make_uint2(h[0] | ((uint32_t)h[1] << 16), h[2] | ((uint32_t)h[3] << 16));
  }
}

// SiLU(gate) * up of the interleaved gate/up projection, rounded straight to the weight type for the
// down projection's tensor-core GEMM.  The sigmoid is evaluated in Float32 here (the Float32 decode
// path keeps the reference's double expression): the half rounding that follows is the prefill
// tolerance and dominates the difference.  Four outputs per thread (I % 4 == 0).
template <bool BF16>
__global__ void silu_mul_round_kernel(const float *gu, uint16_t *act, int I, long total4) {
  const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
  if (i >= total4) return;
  const long m = (i * 4) / I, j = (i * 4) % I;
  const float *src = gu + (size_t)m * 2 * I + 2 * j;
  const float4 a = *reinterpret_cast<const float4 *>(src), b = *reinterpret_cast<const float4 *>(src + 4);
  const float g[4] = {a.x, a.z, b.x, b.z}, u[4] = {a.y, a.w, b.y, b.w};
  uint16_t h[4];
#pragma unroll
  for (int k = 0; k < 4; k++) {
    const float sig = g[k] >= 0.0f ? 1.0f / (1.0f + expf(-g[k])) : expf(g[k]) / (1.0f + expf(g[k]));
    const float sv = g[k] == -INFINITY ? -0.0f : g[k] * sig;
    h[k] = to_half_bits(sv * u[k], BF16);
  }
  *reinterpret_cast<uint2 *>(act + (size_t)m * I + j) = make_uint2(h[0] | ((uint32_t)h[1] << 16), h[2] | ((uint32_t)h[3] << 16));
}

__global__ void set_position_kernel(int *state, int position) { state[0] = position; }

// dst[i][j] = widen/copy of src[rowmap[i]][col0 + j] (half -> half).  Packs a full (out,in) tensor
// into this rank's fused layout (paired q/k/v rows, interleaved gate/up rows, column shards).
__global__ void pack_rows_kernel(uint16_t *dst, const uint16_t *src, const uint32_t *rowmap, int rows, int cols,
                                 int src_cols, int col0) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < (size_t)rows * cols;
       i += (size_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / cols), c = (int)(i % cols);
    dst[i] = src[(size_t)rowmap[r] * src_cols + col0 + c];
  }
}

}  // namespace

namespace {

// Same generator as stb_fill_normal, addressed by (stream_i, logical_row_i * src_cols + col0 + j).
__global__ void fill_rows_kernel(void *dst, int dtype, const uint64_t *rowmap, int rows, int cols, int src_cols,
                                 int col0, uint64_t seed, double stddev) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < (size_t)rows * cols;
       i += (size_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / cols), c = (int)(i % cols);
    const uint64_t stream = rowmap[r] >> 32, lrow = rowmap[r] & 0xffffffffULL;
    const float v = __double2float_rn(
        __dmul_rn(stddev, rng_normal_dev(seed, stream, lrow * (uint64_t)src_cols + (uint64_t)(col0 + c))));
    if (dtype == STB_BF16) ((uint16_t *)dst)[i] = f32_to_bf16_rne(v);
    else ((__half *)dst)[i] = __float2half_rn(v);
  }
}

unsigned grid_for(size_t n) {
  size_t b = (n + 255) / 256;
  return (unsigned)(b > 148 * 32 ? 148 * 32 : (b ? b : 1));
}

// ---------------------------------------------------------------- layout maps

enum Which { W_EMBED = 0, W_FINAL = 1, W_HEAD = 2, W_IN = 3, W_POST = 4, W_Q = 5, W_K = 6, W_V = 7, W_O = 8,
             W_GATE = 9, W_UP = 10, W_DOWN = 11 };

uint64_t stream_of(int which, int layer) {
  return (which == W_EMBED || which == W_FINAL || which == W_HEAD) ? 4096ull + which : (uint64_t)layer * 16 + which;
}

// Physical row -> (logical tensor, logical row) for the paired QKV layout of this rank.
void qkv_rowmap(const stb_llama *m, std::vector<int> &which, std::vector<uint32_t> &lrow) {
  const int half = m->hd / 2;
  const int rows = (m->NH + 2 * m->KV) * m->hd;
  which.assign(rows, 0);
  lrow.assign(rows, 0);
  const int h0q = m->rank * m->NH, h0k = m->rank * m->KV;
  for (int pi = 0; pi < rows / 2; pi++) {
    int w, head, d;
    if (pi < m->NH * half) {
      w = W_Q; head = h0q + pi / half; d = pi % half;
    } else if (pi < (m->NH + m->KV) * half) {
      const int l = pi - m->NH * half;
      w = W_K; head = h0k + l / half; d = l % half;
    } else {
      const int l = pi - (m->NH + m->KV) * half;
      w = W_V; head = h0k + l / half; d = l % half;
    }
    which[2 * pi] = which[2 * pi + 1] = w;
    lrow[2 * pi] = (uint32_t)(head * m->hd + d);
    lrow[2 * pi + 1] = (uint32_t)(head * m->hd + d + half);
  }
}

void gu_rowmap(const stb_llama *m, std::vector<int> &which, std::vector<uint32_t> &lrow) {
  which.assign(2 * m->I, 0);
  lrow.assign(2 * m->I, 0);
  const int i0 = m->rank * m->I;
  for (int i = 0; i < m->I; i++) {
    which[2 * i] = W_GATE;
    which[2 * i + 1] = W_UP;
    lrow[2 * i] = lrow[2 * i + 1] = (uint32_t)(i0 + i);
  }
}

struct Target {
  uint64_t dst;
  int rows, cols, src_cols, col0;
  std::vector<int> which;
  std::vector<uint32_t> lrow;
};

// Where a named full tensor lands in this rank's resident layout.
Target target_of(stb_llama *m, int which, int layer) {
  Target t{};
  const int H = m->H;
  auto ident = [&](int rows, int row0) {
    t.which.assign(rows, which);
    t.lrow.resize(rows);
    for (int i = 0; i < rows; i++) t.lrow[i] = (uint32_t)(row0 + i);
  };
  switch (which) {
    case W_EMBED:
      t.dst = m->embed; t.rows = m->c.vocab_size; t.cols = H; t.src_cols = H; t.col0 = 0; ident(t.rows, 0);
      break;
    case W_HEAD:
      t.dst = m->lm_head; t.rows = m->V; t.cols = H; t.src_cols = H; t.col0 = 0; ident(t.rows, m->v0);
      break;
    case W_Q: case W_K: case W_V:
      t.dst = m->layers[layer].qkv; t.rows = (m->NH + 2 * m->KV) * m->hd; t.cols = H; t.src_cols = H; t.col0 = 0;
      qkv_rowmap(m, t.which, t.lrow);
      break;
    case W_O:
      t.dst = m->layers[layer].o; t.rows = H; t.cols = m->NH * m->hd; t.src_cols = m->c.hidden_size;
      t.col0 = m->rank * m->NH * m->hd; ident(H, 0);
      break;
    case W_GATE: case W_UP:
      t.dst = m->layers[layer].gu; t.rows = 2 * m->I; t.cols = H; t.src_cols = H; t.col0 = 0;
      gu_rowmap(m, t.which, t.lrow);
      break;
    case W_DOWN:
      t.dst = m->layers[layer].down; t.rows = H; t.cols = m->I; t.src_cols = m->c.intermediate_size;
      t.col0 = m->rank * m->I; ident(H, 0);
      break;
    default:
      throw Error(STB_ERR_INVALID, "not a matrix weight");
  }
  return t;
}

uint64_t logical_rows(const stb_llama *m, int which) {
  const auto &c = m->c;
  const int hd = c.hidden_size / c.num_attention_heads;
  switch (which) {
    case W_EMBED: case W_HEAD: return c.vocab_size;
    case W_Q: case W_O: case W_DOWN: case W_FINAL: case W_IN: case W_POST: return c.hidden_size;
    case W_K: case W_V: return (uint64_t)c.num_key_value_heads * hd;
    case W_GATE: case W_UP: return c.intermediate_size;
  }
  return 0;
}
uint64_t logical_cols(const stb_llama *m, int which) {
  const auto &c = m->c;
  if (which == W_FINAL || which == W_IN || which == W_POST) return 1;
  if (which == W_DOWN) return c.intermediate_size;
  return c.hidden_size;
}

// ---------------------------------------------------------------- cache scratch & steps

// Logit rows a cache keeps: every token row up to the reference's logits limit
// (LlamaLimits.maxLogitsElements = 16,777,216, LlamaModel.scala:10-12), at least one per batch row.
int logits_rows(const stb_llama_cache *c, int rows) {
  const long cap = std::max<long>(1, 16777216L / c->m->V);
  return (int)std::max<long>(c->batch, std::min<long>(rows, cap));
}

void ensure_rows(stb_llama_cache *c, int rows) {
  stb_llama *m = c->m;
  stb_session *s = m->s;
  if (rows <= c->rows) return;
  // grow: free old scratch (not the KV cache), drop the graph
  if (c->graph) {
    cudaGraphExecDestroy(c->graph);
    c->graph = nullptr;
  }
  const uint64_t kv = c->kv;
  std::vector<uint64_t> keep;
  for (uint64_t p : c->owned)
    if (p == kv) keep.push_back(p);
    else session_free(s, p);
  c->owned = keep;
  const int qw = m->NH * m->hd;
  c->hidden = alloc_owned(s, c->owned, (uint64_t)rows * m->H * 4);
  c->sum = alloc_owned(s, c->owned, (uint64_t)rows * m->H * 4);
  c->qbuf = alloc_owned(s, c->owned, (uint64_t)rows * qw * 4);
  c->att = alloc_owned(s, c->owned, (uint64_t)rows * qw * 4);
  c->act = alloc_owned(s, c->owned, (uint64_t)rows * m->I * 4);
  c->logits = alloc_owned(s, c->owned, (uint64_t)logits_rows(c, rows) * m->V * 4);
  c->best = alloc_owned(s, c->owned, (uint64_t)c->batch * 8);
  c->best_all = alloc_owned(s, c->owned, (uint64_t)c->batch * 8 * m->tp);
  STB_CUDA(cudaMemsetAsync((void *)c->best, 0, (size_t)c->batch * 8, s->stream));
  c->tokens = alloc_owned(s, c->owned, (uint64_t)rows * 8);
  c->state = alloc_owned(s, c->owned, (uint64_t)(2 + 2 * c->batch) * 4);
  c->xn = c->xh = c->qkvbuf = c->gubuf = 0;
  c->att_rows = c->batch;
  c->att_part = alloc_owned(s, c->owned,
                            std::max<size_t>({decode_attention_part_floats(c->batch, m->KV, c->capacity, m->hd),
                                              decode_attention_reg_part_floats(c->batch, m->KV, c->capacity, m->hd),
                                              decode_stream_part_floats(c->batch, m->KV, c->capacity)}) *
                                sizeof(float));
  c->att_count = alloc_owned(s, c->owned, (uint64_t)c->batch * m->KV * sizeof(int));
  STB_CUDA(cudaMemsetAsync((void *)c->att_count, 0, (size_t)c->batch * m->KV * sizeof(int), s->stream));
  c->skin = c->skin_bytes = c->skin_next = 0;
  {  // the largest scratch any projection of a chunk of up to min(rows, 64) rows takes
    const int sm = std::min(rows, 64);
    const int wdt = m->c.weight_dtype;
    const int qkv_n = (m->NH + 2 * m->KV) * m->hd;
    const int shapes[5][3] = {{sm, qkv_n, m->H}, {sm, m->H, qw}, {sm, 2 * m->I, m->H}, {sm, m->H, m->I},
                              {std::min(logits_rows(c, rows), 64), m->V, m->H}};
    uint64_t need = 0;
    for (const auto &sh : shapes)
      if (skinny_eligible(sh[0], sh[1], sh[2], wdt, (const void *)256))
        need = std::max(need, skinny_scratch_bytes(sh[0], sh[1], sh[2], s->device));
    if (need) {
      c->skin = alloc_owned(s, c->owned, need);
      c->skin_bytes = need;
      skinny_prepare(s->device);
      // terms [3][NT][K] of the widest K a fused fixup writes (hidden or intermediate)
      c->skin_next = alloc_owned(s, c->owned, (uint64_t)3 * skinny_nt(sm) * std::max(m->H, m->I) * 2);
    }
  }
  session_error_word(s);  // allocated now, not inside a graph capture
  if (rows >= m->tc_rows) {
    const uint64_t widest = std::max<uint64_t>(std::max<uint64_t>(m->H, qw), m->I);
    c->xn = alloc_owned(s, c->owned, (uint64_t)rows * m->H * 4);
    c->xh = alloc_owned(s, c->owned, (uint64_t)rows * widest * 2);
    c->qkvbuf = alloc_owned(s, c->owned, (uint64_t)rows * (m->NH + 2 * m->KV) * m->hd * 4);
    c->gubuf = alloc_owned(s, c->owned, (uint64_t)rows * 2 * m->I * 4);
  }
  c->rows = rows;
}

struct StepArgs {
  int rows, count;          // token rows in this chunk and tokens per batch row
  bool device_pos;          // read position from state[0] (graph) instead of c->used
  bool all_logits;          // logits for every row (decode API) or only each batch row's last token
  bool logits = true;       // false: a non-final prefill chunk (no lm_head, no pick)
  bool append = false;      // append picks to out_ids (generation)
  int advance = 0;          // position increment done on device
};

// Tensor-core form of one layer for a chunk of rows >= tc_rows: RMSNorm -> round -> tcgen05 GEMM
// -> RoPE/KV append; attention; round -> GEMM (+residual); RMSNorm -> round -> GEMM -> SiLU*up;
// round -> GEMM (+residual).  Row-split projections under TP write partial sums and reduce.
int enqueue_layer_tc(stb_llama_cache *c, size_t l, int rows, int count, const int *posd, float *kc, float *vc) {
  stb_llama *m = c->m;
  stb_session *s = m->s;
  cudaStream_t st = s->stream;
  const Layer &L = m->layers[l];
  const int H = m->H, qw = m->NH * m->hd, nqkv = (m->NH + 2 * m->KV) * m->hd, wdt = m->c.weight_dtype;
  const bool bf16 = wdt == STB_BF16;
  int *err = session_error_word(s);
  int launches = 0;
  uint16_t *xh = (uint16_t *)c->xh;  // the GEMM's activations, already in the weight type
  auto gemm_h = [&](int K, uint64_t w, int N, float *y, const float *residual) {
    gemm_tc_launch((const void *)xh, (const void *)w, wdt, nullptr, y, N, rows, N, K, err, s->device, st, residual,
                   residual ? N : 0);
    launches += 1;
  };
  auto row_split = [&](int K, uint64_t w) {  // o_proj / down_proj from xh
    if (m->tp == 1) {
      gemm_h(K, w, H, (float *)c->hidden, (const float *)c->hidden);
    } else {
      gemm_h(K, w, H, (float *)c->sum, m->rank == 0 ? (const float *)c->hidden : nullptr);
      allreduce_sum_f32(s, (void *)c->sum, (uint64_t)rows * H);
      std::swap(c->hidden, c->sum);
    }
  };
  // RMSNorm straight into the weight type when the row fits the register form, else Float32 + round
  auto norm = [&](uint64_t wnorm) {
    if (H <= 8192 && H % 4 == 0) {
      if (bf16)
        launch_kernel(rmsnorm_round_kernel<true>, dim3(rows), dim3(256), 0, st, false, (const float *)c->hidden,
                      (const float *)wnorm, m->c.rms_norm_eps, xh, H);
      else
        launch_kernel(rmsnorm_round_kernel<false>, dim3(rows), dim3(256), 0, st, false, (const float *)c->hidden,
                      (const float *)wnorm, m->c.rms_norm_eps, xh, H);
      launches += 1;
    } else {
      launch_kernel(rmsnorm_rows_kernel, dim3(rows), dim3(256), 0, st, false, (const float *)c->hidden,
                    (const float *)wnorm, m->c.rms_norm_eps, (float *)c->xn, H);
      round_activations((const float *)c->xn, xh, (size_t)rows * H, wdt, st);
      launches += 2;
    }
  };
  norm(L.in_norm);
  gemm_h(H, L.qkv, nqkv, (float *)c->qkvbuf, nullptr);
  const long pairs = (long)rows * (nqkv / 2);
  launch_kernel(rope_append_kernel, dim3((unsigned)((pairs + 255) / 256)), dim3(256), 0, st, false,
                (const float *)c->qkvbuf, nqkv, (const double2 *)m->rope, posd, c->used, count, m->NH, m->KV, m->hd,
                c->capacity, (float *)c->qbuf, qw, kc, vc, rows);
  launches += 1;
  // attention: the tensor-core kernel writes the o projection's operand in the weight type directly
  if (launch_flash_attention_tc((const float *)c->qbuf, qw, (const float *)kc, (const float *)vc, nullptr, qw, rows,
                                count, m->NH, m->KV, m->hd, c->capacity, posd, c->used, err, s->device, st, xh, wdt)) {
    launches += 1;
  } else {
    if (!launch_flash_attention((const float *)c->qbuf, qw, (const float *)kc, (const float *)vc, (float *)c->att,
                                qw, rows, count, m->NH, m->KV, m->hd, c->capacity, posd, c->used, s->device, st))
      launch_kernel(attention_kernel, dim3(rows * m->NH), dim3(ATT_THREADS), attention_smem(c->capacity, m->hd), st,
                    false, (const float *)c->qbuf, qw, (const float *)kc, (const float *)vc, (float *)c->att, qw,
                    rows, count, m->NH, m->KV, m->hd, c->capacity, posd, c->used, (const int *)nullptr);
    round_activations((const float *)c->att, xh, (size_t)rows * qw, wdt, st);
    launches += 2;
  }
  row_split(qw, L.o);
  norm(L.post_norm);
  gemm_h(H, L.gu, 2 * m->I, (float *)c->gubuf, nullptr);
  const long acts4 = (long)rows * m->I / 4;  // I % 8 == 0 (check_config)
  if (bf16)
    launch_kernel(silu_mul_round_kernel<true>, dim3((unsigned)((acts4 + 255) / 256)), dim3(256), 0, st, false,
                  (const float *)c->gubuf, xh, m->I, acts4);
  else
    launch_kernel(silu_mul_round_kernel<false>, dim3((unsigned)((acts4 + 255) / 256)), dim3(256), 0, st, false,
                  (const float *)c->gubuf, xh, m->I, acts4);
  launches += 1;
  row_split(m->I, L.down);
  return launches;
}

// One projection of a chunk: the tensor-core skinny form (three-term BF16 activations, FP32
// accurate) when it applies to the shape and the cache holds its scratch, else the vector GEMV.
// Returns the kernels launched.
bool projects_skinny(const stb_llama_cache *c, int M, int N, int K, int wdt, const void *w) {
  return c->skin && skinny_eligible(M, N, K, wdt, w) && skinny_scratch_bytes(M, N, K, c->m->s->device) <= c->skin_bytes;
}

// With x3_ready the skinny form's activation terms are already there (written by the previous
// kernel), and with next this projection's fixup writes the next one's: M <= 64, and the projection
// must take the skinny form.
template <int EPI>
int project(stb_llama_cache *c, const GemvParams &p, int wdt, GemvConfig cfg, cudaStream_t st,
            const uint16_t *x3_ready = nullptr, const SkinnyNext *next = nullptr, SkinnyParts *deferred = nullptr) {
  stb_session *s = c->m->s;
  if (projects_skinny(c, p.M, p.N, p.K, wdt, p.w))
    return skinny_launch<EPI>(p, (void *)c->skin, c->skin_bytes, session_error_word(s), s->device, st, x3_ready,
                              next, deferred);
  STB_REQUIRE(!x3_ready && !next && !deferred, "prepared activation terms need the skinny projection");
  launch_gemv<EPI>(p, wdt, cfg, st);
  return 1;
}

// Enqueues one forward chunk on the session stream.
int enqueue_step(stb_llama_cache *c, const StepArgs &a) {
  stb_llama *m = c->m;
  stb_session *s = m->s;
  cudaStream_t st = s->stream;
  const int H = m->H, rows = a.rows;
  const int *state = (const int *)c->state;
  // Once every row has stopped, finalize appends nothing and no longer advances the position, so
  // the remaining replays only recompute; the kernels themselves need not read the stop flag
  // (it would sit on each kernel's critical path).
  const int *stop = nullptr;
  const int *posd = a.device_pos ? state : nullptr;
  int launches = 0;
  const int wdt = m->c.weight_dtype;

  // The first kernel follows host copies (or the previous graph replay): a plain launch.  Every
  // later kernel is a programmatic dependent of its predecessor (see launch_kernel / pdl_wait).
  launch_kernel(embed_kernel, dim3((unsigned)((H / 8 + 127) / 128), rows), dim3(128), 0, st, false,
                (const int64_t *)c->tokens, (const uint16_t *)m->embed, wdt, H, m->c.vocab_size, (float *)c->hidden,
                rows, stop);
  launches++;
  const size_t kv_layer = (size_t)2 * c->batch * m->KV * c->capacity * m->hd;
  const size_t kv_half = kv_layer / 2;
  const int qw = m->NH * m->hd;
  const bool tensor_cores = rows >= m->tc_rows && c->xh != 0;
  // Chunks of up to 64 rows on the skinny form: the o, gate/up and down fixups (under tensor
  // parallelism: the gate/up fixup and the peer reduces) also write the next projection's activation
  // terms (RMSNorm and split, SiLU*up and split), whose prologue launch is then skipped.  `pending`
  // holds those terms for the next projection.
  static const int fuse_enabled = env_int("STB_FUSE_NEXT", 1);
  const bool fuse_next = fuse_enabled && c->skin_next && rows <= 64 && !tensor_cores;
  const bool fuse_norm = fuse_next && (m->tp == 1 ? skinny_norm_fusable(H) : peer_norm_fusable(H));
  const uint16_t *pending = nullptr;
  SkinnyNext next;
  next.x3 = (uint16_t *)c->skin_next;
  next.eps = m->c.rms_norm_eps;
  for (size_t l = 0; l < m->layers.size(); l++) {
    const Layer &L = m->layers[l];
    float *kc = (float *)c->kv + l * kv_layer;
    float *vc = kc + kv_half;
    if (tensor_cores) {
      launches += enqueue_layer_tc(c, l, rows, a.count, posd, kc, vc);
      continue;
    }
    // the streamed single-token attention leaves split records; the o projection's prologue merges them
    // -- or, for 5 to 8 query heads per KV head on the skinny QKV form, the attention itself adds the QKV
    // projection's pieces (RoPE + cache append) and merges its splits (two launches fewer)
    const bool stream_att = a.count == 1 && rows <= c->att_rows && c->kv_map_ok;
    const int qkv_n = (m->NH + 2 * m->KV) * m->hd;
    static const int fuse_att_enabled = env_int("STB_FUSE_ATT", 1);
    const bool fuse_att = fuse_att_enabled && stream_att && rows <= 64 && decode_stream_fusable(m->NH, m->KV) &&
                          projects_skinny(c, rows, qkv_n, H, wdt, (const void *)L.qkv) &&
                          projects_skinny(c, rows, H, qw, wdt, (const void *)L.o);
    SkinnyParts qkv_parts;
    {  // 1. QKV + RoPE + cache append
      GemvParams p;
      p.x = (const float *)c->hidden; p.ldx = H; p.w = (const void *)L.qkv;
      p.M = rows; p.N = (m->NH + 2 * m->KV) * m->hd; p.K = H;
      p.y = (float *)c->qbuf; p.ldy = qw;
      p.norm_w = pending ? nullptr : (const float *)L.in_norm; p.norm_eps = m->c.rms_norm_eps;
      p.rope = (const double2 *)m->rope; p.pos_dev = posd; p.pos0 = c->used; p.count = a.count;
      p.nh = m->NH; p.kvh = m->KV; p.hd = m->hd; p.capacity = c->capacity; p.k_cache = kc; p.v_cache = vc;
      p.stop = stop;
      p.pdl = true;
      launches += project<EPI_QKV>(c, p, wdt, choose_gemv(rows, p.N, p.K, true), st, pending, nullptr,
                                   fuse_att ? &qkv_parts : nullptr);
      pending = nullptr;
    }
    bool o_x3 = false;
    if (stream_att) {  // 2. attention (streamed form) and the merge: as the o projection's terms or Float32
      const DecodeStreamPlan plan = decode_stream_plan(rows, m->KV, c->capacity, s->device);
      o_x3 = rows <= 64 && projects_skinny(c, rows, H, qw, wdt, (const void *)L.o);
      if (fuse_att) {
        DecodeStreamFused fu;
        fu.part = qkv_parts.part; fu.kbs = qkv_parts.kbs; fu.T = qkv_parts.T; fu.G = qkv_parts.G;
        fu.pmax = qkv_parts.pmax; fu.M = qkv_parts.M;
        fu.rope = (const double2 *)m->rope;
        fu.counter = (int *)c->att_count;
        fu.x3 = (uint16_t *)c->skin;  // o takes the skinny form (a condition of fuse_att): o_x3
        fu.NT = skinny_nt(rows);
        launch_decode_attention_stream(c->kv_map, (long long)(l * kv_layer) / m->hd, (const float *)c->qbuf, qw, kc,
                                       vc, rows, 1, m->NH, m->KV, c->capacity, posd, c->used, plan,
                                       (float *)c->att_part, true, st, s->device, session_error_word(s), &fu);
        launches += 1;
      } else {
        launch_decode_attention_stream(c->kv_map, (long long)(l * kv_layer) / m->hd, (const float *)c->qbuf, qw, kc,
                                       vc, rows, 1, m->NH, m->KV, c->capacity, posd, c->used, plan,
                                       (float *)c->att_part, true, st, s->device, session_error_word(s));
        launch_attention_merge_split((const float *)c->att_part, plan, posd, c->used, rows, 1, m->NH, m->KV,
                                     skinny_nt(rows), o_x3 ? (uint16_t *)c->skin : nullptr,
                                     o_x3 ? nullptr : (float *)c->att, qw, st);
        launches += 2;
      }
    } else {  // 2. attention: split GQA kernel for single-token steps, tiled kernel for chunks
      bool done = false;
      if (a.count == 1 && rows <= c->att_rows)
        done = use_register_attention(rows, m->KV, m->hd, c->capacity, s->device)
                   ? launch_decode_attention_reg((const float *)c->qbuf, qw, (const float *)kc, (const float *)vc,
                                                 (float *)c->att, qw, rows, 1, m->NH, m->KV, m->hd, c->capacity, posd,
                                                 c->used, (float *)c->att_part, (int *)c->att_count, true, st)
                   : launch_decode_attention((const float *)c->qbuf, qw, (const float *)kc, (const float *)vc,
                                             (float *)c->att, qw, rows, 1, m->NH, m->KV, m->hd, c->capacity, posd,
                                             c->used, (float *)c->att_part, (int *)c->att_count, true, st, s->device,
                                             session_error_word(s));
      else if (a.count > 1)
        done = launch_flash_attention((const float *)c->qbuf, qw, (const float *)kc, (const float *)vc,
                                      (float *)c->att, qw, rows, a.count, m->NH, m->KV, m->hd, c->capacity, posd,
                                      c->used, s->device, st);
      if (!done) {
        const size_t smem = attention_smem(c->capacity, m->hd);
        launch_kernel(attention_kernel, dim3(rows * m->NH), dim3(ATT_THREADS), smem, st, true,
                      (const float *)c->qbuf, qw, (const float *)kc, (const float *)vc, (float *)c->att, qw, rows,
                      a.count, m->NH, m->KV, m->hd, c->capacity, posd, c->used, stop);
      }
      launches++;
    }
    const bool o_sk = projects_skinny(c, rows, H, qw, wdt, (const void *)L.o);
    const bool gu_sk = projects_skinny(c, rows, 2 * m->I, H, wdt, (const void *)L.gu);
    const bool down_sk = projects_skinny(c, rows, H, m->I, wdt, (const void *)L.down);
    const bool qkv_next_sk = l + 1 < m->layers.size() &&
                             projects_skinny(c, rows, (m->NH + 2 * m->KV) * m->hd, H, wdt,
                                             (const void *)m->layers[l + 1].qkv);
    for (int half = 0; half < 2; half++) {  // 3. O (+residual)   then   4./5. MLP (+residual)
      if (half == 1) {
        GemvParams p;
        p.x = (const float *)c->hidden; p.ldx = H; p.w = (const void *)L.gu;
        p.M = rows; p.N = 2 * m->I; p.K = H;
        p.y = (float *)c->act; p.ldy = m->I;
        p.norm_w = pending ? nullptr : (const float *)L.post_norm; p.norm_eps = m->c.rms_norm_eps;
        p.stop = stop;
        p.pdl = true;
        const bool fuse = fuse_next && gu_sk && down_sk;
        next.norm_w = nullptr;
        launches += project<EPI_SILU>(c, p, wdt, choose_gemv(rows, p.N, p.K, true), st, pending,
                                      fuse ? &next : nullptr);
        pending = fuse ? next.x3 : nullptr;
      }
      GemvParams p;
      p.x = (const float *)(half == 0 ? c->att : c->act);
      p.ldx = half == 0 ? qw : m->I;
      p.w = (const void *)(half == 0 ? L.o : L.down);
      p.M = rows; p.N = H; p.K = half == 0 ? qw : m->I;
      p.stop = stop;
      p.pdl = true;
      if (m->tp == 1) {
        p.y = (float *)c->hidden; p.ldy = H; p.residual = (const float *)c->hidden; p.ldr = H;
        const uint16_t *x3 = half == 0 ? (o_x3 ? (const uint16_t *)c->skin : nullptr) : pending;
        // o: the gate/up projection's RMSNorm prologue; down: the next layer's QKV RMSNorm prologue
        const bool fuse = fuse_norm && (half == 0 ? o_sk && gu_sk : down_sk && qkv_next_sk);
        next.norm_w = half == 0 ? (const float *)L.post_norm
                                : (l + 1 < m->layers.size() ? (const float *)m->layers[l + 1].in_norm : nullptr);
        launches += project<EPI_RESID>(c, p, wdt, choose_gemv(rows, p.N, p.K, false), st, x3, fuse ? &next : nullptr);
        pending = fuse ? next.x3 : nullptr;
      } else if (peer_usable(s, (uint64_t)rows * H)) {
        // fused row-split projection: partial sums stored into every rank's slots over NVLink,
        // then summed in rank order with the residual on each rank
        p.ldy = H;
        p.peer = peer_args(s, half);
        const GemvConfig cfg = choose_gemv(rows, p.N, p.K, false);
        const uint16_t *x3 = half == 0 ? (o_x3 ? (const uint16_t *)c->skin : nullptr) : pending;
        launches += project<EPI_PEER>(c, p, wdt, cfg, st, x3);
        // o: the reduce also does the gate/up projection's RMSNorm prologue; down: the next layer's
        const bool fuse = fuse_norm && (half == 0 ? o_sk && gu_sk : down_sk && qkv_next_sk);
        if (fuse) {
          const float *nw = half == 0 ? (const float *)L.post_norm : (const float *)m->layers[l + 1].in_norm;
          peer_reduce_norm_launch(s, half, rows, H, (const float *)c->hidden, (float *)c->hidden, nw,
                                  m->c.rms_norm_eps, next.x3, skinny_nt(rows));
        } else {
          peer_reduce_launch(s, half, (long)rows * H, (const float *)c->hidden, (float *)c->hidden);
        }
        pending = fuse ? next.x3 : nullptr;
        launches++;
      } else {
        p.y = (float *)c->sum; p.ldy = H;
        const uint16_t *x3 = half == 0 ? (o_x3 ? (const uint16_t *)c->skin : nullptr) : pending;
        if (m->rank == 0) {
          p.residual = (const float *)c->hidden; p.ldr = H;
          launches += project<EPI_RESID>(c, p, wdt, choose_gemv(rows, p.N, p.K, false), st, x3);
        } else {
          launches += project<EPI_PLAIN>(c, p, wdt, choose_gemv(rows, p.N, p.K, false), st, x3);
        }
        allreduce_sum_f32(s, (void *)c->sum, (uint64_t)rows * H);
        std::swap(c->hidden, c->sum);
        pending = nullptr;
      }
    }
  }
  // final norm + lm_head (+ greedy candidates)
  const int brows = a.all_logits ? rows : c->batch;
  if (a.logits) {
    GemvParams p;
    if (a.all_logits) {
      p.x = (const float *)c->hidden; p.ldx = H;
    } else {
      p.x = (const float *)c->hidden + (size_t)(a.count - 1) * H; p.ldx = a.count * H;
    }
    p.w = (const void *)m->lm_head;
    p.M = brows; p.N = m->V; p.K = H;
    p.y = (float *)c->logits; p.ldy = m->V;
    p.norm_w = (const float *)m->final_norm; p.norm_eps = m->c.rms_norm_eps;
    p.best = a.all_logits ? nullptr : (unsigned long long *)c->best;  // greedy candidates per batch row
    p.row_offset = m->v0;
    p.stop = stop;
    p.pdl = true;
    launches += project<EPI_LOGITS>(c, p, wdt, choose_gemv(brows, p.N, p.K, false), st);
    if (!a.all_logits) {
      const unsigned long long *all = (const unsigned long long *)c->best;
      if (m->tp > 1) {  // every rank's best over its vocabulary shard, [rank][batch]
        allgather_bytes(s, (const void *)c->best, (void *)c->best_all, (uint64_t)brows * 8);
        all = (const unsigned long long *)c->best_all;
      }
      launch_kernel(finalize_kernel, dim3(1), dim3(32), 0, st, m->tp == 1, all, (unsigned long long *)c->best, m->tp,
                    brows, a.count, (int64_t *)c->tokens, (int *)c->state,
                    a.append ? (int64_t *)c->out_ids : nullptr, c->out_stride, (const int64_t *)c->eos, c->eos_count,
                    a.advance);
      launches++;
    }
  }
  return launches;
}

void check_config(const stb_llama_config &c) {
  STB_REQUIRE(c.vocab_size > 0 && c.hidden_size > 0 && c.intermediate_size > 0 && c.num_layers > 0 &&
                  c.max_positions > 0,
              "invalid Llama dimensions");
  STB_REQUIRE(c.num_attention_heads > 0 && c.num_key_value_heads > 0 &&
                  c.hidden_size % c.num_attention_heads == 0 && c.num_attention_heads % c.num_key_value_heads == 0,
              "invalid Llama head dimensions");
  const int hd = c.hidden_size / c.num_attention_heads;
  STB_REQUIRE(hd % 2 == 0, "Llama rotary head width must be even");
  STB_REQUIRE(std::isfinite(c.rms_norm_eps) && c.rms_norm_eps > 0 && std::isfinite(c.rope_theta) && c.rope_theta > 0,
              "invalid Llama norm/rotary configuration");
  STB_REQUIRE(c.weight_dtype == STB_BF16 || c.weight_dtype == STB_F16, "Llama weights must be BF16 or F16");
  STB_REQUIRE(c.hidden_size % 8 == 0 && c.intermediate_size % 8 == 0 && hd % 8 == 0,
              "device Llama needs hidden, intermediate and head widths that are multiples of 8");
  const int tp = c.tp_size < 1 ? 1 : c.tp_size;
  STB_REQUIRE(c.tp_rank >= 0 && c.tp_rank < tp, "invalid tensor-parallel rank");
  STB_REQUIRE(c.num_attention_heads % tp == 0 && c.num_key_value_heads % tp == 0 &&
                  c.intermediate_size % tp == 0 && c.vocab_size % tp == 0 && (c.intermediate_size / tp) % 8 == 0,
              "heads, KV heads, intermediate size and vocabulary must split evenly over the tensor-parallel group");
}

}  // namespace

extern "C" {

int stb_llama_shard_plan(const stb_llama_config *config, int rank, int tp, int64_t out[14]) {
  return guarded([&] {
    STB_REQUIRE(config && out, "null argument");
    stb_llama_config c = *config;
    c.tp_rank = rank;
    c.tp_size = tp;
    STB_REQUIRE(tp >= 1, "invalid tensor-parallel size");
    check_config(c);
    const int64_t hd = c.hidden_size / c.num_attention_heads, H = c.hidden_size;
    const int64_t nh = c.num_attention_heads / tp, kv = c.num_key_value_heads / tp;
    const int64_t I = c.intermediate_size / tp, V = c.vocab_size / tp;
    const int64_t r = rank;
    const int64_t v[14] = {r * nh, (r + 1) * nh, r * kv, (r + 1) * kv, r * I, (r + 1) * I, r * V, (r + 1) * V,
                           r * nh * hd, (r + 1) * nh * hd, r * I, (r + 1) * I, 0, 0};
    for (int i = 0; i < 14; i++) out[i] = v[i];
    const int64_t layer = ((nh + 2 * kv) * hd * H + H * nh * hd + 2 * I * H + H * I) * 2;
    const bool head_is_embed = c.tie_word_embeddings && tp == 1;
    out[12] = layer * c.num_layers + (int64_t)c.vocab_size * H * 2 + (head_is_embed ? 0 : V * H * 2);
  });
}

int stb_llama_create(stb_session *s, const stb_llama_config *config, stb_llama **out) {
  return guarded([&] {
    enter(s);
    STB_REQUIRE(config && out, "null argument");
    *out = nullptr;
    check_config(*config);
    const int tp = config->tp_size < 1 ? 1 : config->tp_size;
    STB_REQUIRE(tp == s->tp_size, "tensor-parallel size differs from the session's communicator");
    STB_REQUIRE(config->tp_rank == s->tp_rank, "tensor-parallel rank differs from the session's communicator");
    auto *m = new stb_llama();
    m->s = s;
    m->c = *config;
    m->c.tp_size = tp;
    m->tp = tp;
    m->tc_rows = config->tc_prefill_rows == 0 ? 256 : (config->tc_prefill_rows < 0 ? INT_MAX : config->tc_prefill_rows);
    m->rank = config->tp_rank;
    m->H = config->hidden_size;
    m->hd = config->hidden_size / config->num_attention_heads;
    m->NH = config->num_attention_heads / tp;
    m->KV = config->num_key_value_heads / tp;
    m->I = config->intermediate_size / tp;
    m->V = config->vocab_size / tp;
    m->v0 = m->rank * m->V;
    try {
      const size_t hs = esize(config->weight_dtype);
      const uint64_t H = m->H;
      m->embed = alloc_owned(s, m->owned, (uint64_t)config->vocab_size * H * hs);
      m->final_norm = alloc_owned(s, m->owned, H * 4);
      if (config->tie_word_embeddings && tp == 1) {
        m->lm_head = m->embed;
        m->head_aliases_embed = true;
      } else {
        m->lm_head = alloc_owned(s, m->owned, (uint64_t)m->V * H * hs);
      }
      m->layers.resize(config->num_layers);
      for (auto &L : m->layers) {
        L.in_norm = alloc_owned(s, m->owned, H * 4);
        L.post_norm = alloc_owned(s, m->owned, H * 4);
        L.qkv = alloc_owned(s, m->owned, (uint64_t)(m->NH + 2 * m->KV) * m->hd * H * hs);
        L.o = alloc_owned(s, m->owned, H * (uint64_t)m->NH * m->hd * hs);
        L.gu = alloc_owned(s, m->owned, (uint64_t)2 * m->I * H * hs);
        L.down = alloc_owned(s, m->owned, H * (uint64_t)m->I * hs);
      }
      // Rotary coefficients of RotaryCoefficients.values (AttentionLayout.scala:23-34), in double.
      const int half = m->hd / 2;
      std::vector<double> cs((size_t)config->max_positions * half * 2);
      for (int t = 0; t < config->max_positions; t++)
        for (int d = 0; d < half; d++) {
          const double angle = (double)t * std::pow(config->rope_theta, -2.0 * d / m->hd);
          cs[((size_t)t * half + d) * 2] = std::cos(angle);
          cs[((size_t)t * half + d) * 2 + 1] = std::sin(angle);
        }
      m->rope = alloc_owned(s, m->owned, cs.size() * 8);
      upload(s, cs.data(), cs.size() * 8, m->rope);
      for (uint64_t p : m->owned) (void)p;
      m->weight_bytes = 0;
      for (uint64_t p : m->owned) m->weight_bytes += s->allocations[p];
    } catch (...) {
      free_owned(s, m->owned);
      delete m;
      throw;
    }
    *out = m;
  });
}

int stb_llama_destroy(stb_llama *m) {
  if (!m) return STB_OK;
  return guarded([&] {
    enter(m->s);
    if (m->gen) {
      stb_llama_cache_destroy(m->gen);
      m->gen = nullptr;
    }
    free_owned(m->s, m->owned);
    delete m;
  });
}

int stb_llama_weight_bytes(stb_llama *m, uint64_t *bytes) {
  return guarded([&] {
    STB_REQUIRE(m && bytes, "null argument");
    enter(m->s);
    *bytes = m->weight_bytes;
  });
}

int stb_llama_set_weight(stb_llama *m, int which, int layer, const void *host, uint64_t bytes, int dtype) {
  return guarded([&] {
    STB_REQUIRE(m, "null model");
    stb_session *s = m->s;
    enter(s);
    STB_REQUIRE(which >= W_EMBED && which <= W_DOWN, "unknown Llama weight");
    const bool global = which == W_EMBED || which == W_FINAL || which == W_HEAD;
    STB_REQUIRE(global || (layer >= 0 && layer < (int)m->layers.size()), "layer out of range");
    STB_REQUIRE(host || bytes == 0, "null payload");
    const uint64_t rows = logical_rows(m, which), cols = logical_cols(m, which);
    const uint64_t count = rows * cols;
    STB_REQUIRE(dtype == STB_F32 || dtype == STB_BF16 || dtype == STB_F16, "unsupported dtype");
    STB_REQUIRE(bytes == count * esize(dtype), "Llama weight metadata mismatch: payload size");
    if (which == W_FINAL || which == W_IN || which == W_POST) {
      std::vector<float> wide(count);
      const uint16_t *h = (const uint16_t *)host;
      for (uint64_t i = 0; i < count; i++) {
        if (dtype == STB_F32) std::memcpy(&wide[i], (const char *)host + 4 * i, 4);
        else if (dtype == STB_BF16) {
          uint32_t u = (uint32_t)h[i] << 16;
          std::memcpy(&wide[i], &u, 4);
        } else {
          wide[i] = __half2float(*reinterpret_cast<const __half *>(&h[i]));
        }
      }
      const uint64_t dst = which == W_FINAL ? m->final_norm
                                            : (which == W_IN ? m->layers[layer].in_norm : m->layers[layer].post_norm);
      upload(s, wide.data(), count * 4, dst);
      STB_CUDA(cudaStreamSynchronize(s->stream));
      return;
    }
    STB_REQUIRE(dtype == m->c.weight_dtype, "matrix payload dtype differs from the model's weight dtype");
    if (which == W_HEAD && m->head_aliases_embed) {
      // Tied head: LlamaModel.load requires a present lm_head to equal the embedding bitwise
      // (LlamaModel.scala:170-173); the resident copy is the embedding's.
      std::vector<uint16_t> emb(count);
      download(s, m->embed, emb.data(), count * 2);
      STB_REQUIRE(std::memcmp(emb.data(), host, count * 2) == 0, "conflicting tied lm_head weight");
      return;
    }
    Target t = target_of(m, which, layer);
    // stage the full tensor, then gather this rank's rows/columns into the fused layout
    uint64_t tmp = session_alloc(s, count * 2), map = 0;
    try {
      upload(s, host, count * 2, tmp);
      std::vector<uint32_t> rowmap;
      std::vector<uint32_t> dst_rows;
      for (int r = 0; r < t.rows; r++)
        if (t.which[r] == which) {
          dst_rows.push_back((uint32_t)r);
          rowmap.push_back(t.lrow[r]);
        }
      // pack rows of this tensor: dst row list scattered; do it row-list-wise via a compact map
      // (dst rows of one logical tensor are interleaved with the others' in paired layouts).
      map = session_alloc(s, rowmap.size() * 8);
      std::vector<uint32_t> both(rowmap.size() * 2);
      for (size_t i = 0; i < rowmap.size(); i++) {
        both[i] = rowmap[i];
        both[rowmap.size() + i] = dst_rows[i];
      }
      upload(s, both.data(), both.size() * 4, map);
      // one launch per destination row would be slow for big matrices; rows of one tensor are
      // gathered to consecutive temp rows first, then scattered with cudaMemcpy2D per run.
      uint64_t packed = session_alloc(s, (uint64_t)rowmap.size() * t.cols * 2);
      pack_rows_kernel<<<grid_for(rowmap.size() * (size_t)t.cols), 256, 0, s->stream>>>(
          (uint16_t *)packed, (const uint16_t *)tmp, (const uint32_t *)map, (int)rowmap.size(), t.cols, t.src_cols,
          t.col0);
      check_launch("pack_rows");
      count_launch(s);
      // scatter consecutive runs of destination rows
      size_t i = 0;
      while (i < dst_rows.size()) {
        size_t j = i + 1;
        uint32_t step = (j < dst_rows.size()) ? dst_rows[j] - dst_rows[i] : 1;
        while (j < dst_rows.size() && dst_rows[j] - dst_rows[j - 1] == step) j++;
        STB_CUDA(cudaMemcpy2DAsync((void *)(t.dst + (uint64_t)dst_rows[i] * t.cols * 2), (size_t)step * t.cols * 2,
                                   (const void *)(packed + (uint64_t)i * t.cols * 2), (size_t)t.cols * 2,
                                   (size_t)t.cols * 2, j - i, cudaMemcpyDeviceToDevice, s->stream));
        i = j;
      }
      STB_CUDA(cudaStreamSynchronize(s->stream));
      session_free(s, packed);
    } catch (...) {
      if (map) session_free(s, map);
      session_free(s, tmp);
      throw;
    }
    session_free(s, map);
    session_free(s, tmp);
  });
}

int stb_llama_init_random(stb_llama *m, uint64_t seed, double stddev) {
  return guarded([&] {
    STB_REQUIRE(m, "null model");
    stb_session *s = m->s;
    enter(s);
    const int wdt = m->c.weight_dtype;
    auto fill_target = [&](const Target &t, int layer) {
      std::vector<uint64_t> map(t.rows);
      for (int r = 0; r < t.rows; r++) map[r] = (stream_of(t.which[r], layer) << 32) | t.lrow[r];
      uint64_t dmap = session_alloc(s, map.size() * 8);
      try {
        upload(s, map.data(), map.size() * 8, dmap);
        fill_rows_kernel<<<grid_for((size_t)t.rows * t.cols), 256, 0, s->stream>>>(
            (void *)t.dst, wdt, (const uint64_t *)dmap, t.rows, t.cols, t.src_cols, t.col0, seed, stddev);
        check_launch("fill_rows");
        count_launch(s);
        STB_CUDA(cudaStreamSynchronize(s->stream));
      } catch (...) {
        session_free(s, dmap);
        throw;
      }
      session_free(s, dmap);
    };
    fill_target(target_of(m, W_EMBED, 0), 0);
    if (!m->head_aliases_embed) {
      // untied: its own stream; tied but sharded: the embedding's values
      Target t = target_of(m, W_HEAD, 0);
      if (m->c.tie_word_embeddings) std::fill(t.which.begin(), t.which.end(), (int)W_EMBED);
      fill_target(t, 0);
    }
    fill_value(s, m->final_norm, STB_F32, m->H, 1.0f);
    for (int l = 0; l < (int)m->layers.size(); l++) {
      fill_value(s, m->layers[l].in_norm, STB_F32, m->H, 1.0f);
      fill_value(s, m->layers[l].post_norm, STB_F32, m->H, 1.0f);
      fill_target(target_of(m, W_Q, l), l);
      fill_target(target_of(m, W_O, l), l);
      fill_target(target_of(m, W_GATE, l), l);
      fill_target(target_of(m, W_DOWN, l), l);
    }
    STB_CUDA(cudaStreamSynchronize(s->stream));
  });
}

int stb_llama_cache_create(stb_llama *m, int batch, int capacity, stb_llama_cache **out) {
  return guarded([&] {
    STB_REQUIRE(m && out, "null argument");
    enter(m->s);
    *out = nullptr;
    STB_REQUIRE(batch > 0 && capacity > 0 && capacity <= m->c.max_positions, "invalid model cache dimensions/budget");
    // attention keeps one row of double scores per block in shared memory
    STB_REQUIRE(capacity <= 26000, "model cache capacity exceeds the attention score workspace");
    STB_REQUIRE(m->hd <= ATT_THREADS, "head width exceeds the attention block");
    const size_t smem = attention_smem(capacity, m->hd);
    if (smem > 48 * 1024)
      STB_CUDA(cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    auto *c = new stb_llama_cache();
    c->m = m;
    c->batch = batch;
    c->capacity = capacity;
    try {
      const uint64_t bytes = (uint64_t)m->layers.size() * 2 * batch * m->KV * capacity * m->hd * 4;
      c->kv = alloc_owned(m->s, c->owned, bytes);
      if (decode_stream_applies(m->hd, m->NH, m->KV)) {
        c->kv_map = make_kv_map((const float *)c->kv, bytes / ((uint64_t)m->hd * 4));
        c->kv_map_ok = true;
      }
      ensure_rows(c, batch);
    } catch (...) {
      free_owned(m->s, c->owned);
      delete c;
      throw;
    }
    *out = c;
  });
}

int stb_llama_cache_destroy(stb_llama_cache *c) {
  if (!c) return STB_OK;
  return guarded([&] {
    enter(c->m->s);
    if (c->graph) cudaGraphExecDestroy(c->graph);
    free_owned(c->m->s, c->owned);
    delete c;
  });
}

int stb_llama_cache_position(stb_llama_cache *c, int *position) {
  return guarded([&] {
    STB_REQUIRE(c && position, "null argument");
    enter(c->m->s);
    *position = c->used;
  });
}

int stb_llama_cache_reset(stb_llama_cache *c) {
  return guarded([&] {
    STB_REQUIRE(c, "null cache");
    enter(c->m->s);
    c->used = 0;  // old tails are invisible and overwritten by the next append (LlamaCache.scala:50-54)
  });
}

int stb_llama_decode(stb_llama_cache *c, const int64_t *tokens, int batch, int count, float *logits,
                     int64_t *next_ids) {
  return guarded([&] {
    STB_REQUIRE(c, "null cache");
    stb_llama *m = c->m;
    stb_session *s = m->s;
    enter(s);
    STB_REQUIRE(tokens && batch == c->batch && count > 0, "cache tokens must match batch with positive chunk length");
    STB_REQUIRE((long)c->used + count <= c->capacity, "model cache capacity exceeded");
    const int rows = batch * count;
    // LlamaCache.decode's logits limit (LlamaLimits.maxLogitsElements, LlamaCache.scala:31-32)
    STB_REQUIRE((long)rows * m->c.vocab_size <= 16777216L, "cached logits allocation limit exceeded");
    for (int i = 0; i < rows; i++)
      STB_REQUIRE(tokens[i] >= 0 && tokens[i] < m->c.vocab_size, "embedding token ID out of bounds");
    ensure_rows(c, rows);
    if (m->tp > 1) peer_reset(s);  // collective, as every rank decodes the same chunk
    upload(s, tokens, (uint64_t)rows * 8, c->tokens);
    STB_CUDA(cudaMemsetAsync((void *)c->state, 0, (size_t)(2 + 2 * batch) * 4, s->stream));
    StepArgs a;
    a.rows = rows;
    a.count = count;
    a.device_pos = false;
    a.all_logits = true;
    a.append = false;
    a.advance = 0;
    int launches = enqueue_step(c, a);
    count_launch(s, launches);
    if (logits) {
      if (m->tp == 1) {
        download(s, c->logits, logits, (uint64_t)rows * m->V * 4);
      } else {
        // this rank holds vocabulary columns [v0, v0+V): gather all ranks' logits row blocks
        throw Error(STB_ERR_UNSUPPORTED, "full logits download under tensor parallelism; use next_ids");
      }
    }
    if (next_ids) {
      // greedy pick of each batch row's last token on the host, as BackendLlama samples the
      // downloaded logits (BackendLlama.scala:126-141; TokenSampler strict '>')
      STB_REQUIRE(m->tp == 1, "host-side greedy pick needs the full vocabulary on this rank");
      std::vector<float> last((size_t)batch * m->V);
      for (int b = 0; b < batch; b++) {
        const uint64_t src = c->logits + ((uint64_t)(b * count + count - 1) * m->V) * 4;
        download(s, src, last.data() + (size_t)b * m->V, (uint64_t)m->V * 4);
        int64_t best = 0;
        for (int i = 1; i < m->V; i++)
          if (last[(size_t)b * m->V + i] > last[(size_t)b * m->V + best]) best = i;
        next_ids[b] = best;
      }
    }
    STB_CUDA(cudaStreamSynchronize(s->stream));
    c->used += count;  // publish only after the whole chunk succeeded (BackendLlamaCache.scala:38-40)
  });
}

int stb_llama_generate(stb_llama *m, const int64_t *prompt, int batch, int prompt_len, int max_new,
                       const int64_t *eos, int eos_count, int64_t *out, int *generated, float *timings_ms) {
  return guarded([&] {
    STB_REQUIRE(m, "null model");
    stb_session *s = m->s;
    enter(s);
    STB_REQUIRE(prompt && out && batch > 0 && prompt_len > 0 && max_new >= 0 &&
                    (long)prompt_len + max_new <= m->c.max_positions,
                "invalid generation length");
    STB_REQUIRE(eos_count >= 0 && (eos_count == 0 || eos), "invalid EOS list");
    for (long i = 0; i < (long)batch * prompt_len; i++)
      STB_REQUIRE(prompt[i] >= 0 && prompt[i] < m->c.vocab_size, "generation token outside vocabulary");
    const int total = prompt_len + max_new;
    for (int b = 0; b < batch; b++)
      std::memcpy(out + (size_t)b * total, prompt + (size_t)b * prompt_len, (size_t)prompt_len * 8);
    if (generated)
      for (int b = 0; b < batch; b++) generated[b] = 0;
    if (timings_ms) timings_ms[0] = timings_ms[1] = 0.0f;
    if (max_new == 0) return;
    // The prompt is prefilled in chunks of at most STB_PREFILL_CHUNK_ROWS token rows (all batch
    // rows advance together), bounding the activation buffers for long or wide prompts.
    const char *env = std::getenv("STB_PREFILL_CHUNK_ROWS");
    const int chunk_rows = env && *env ? std::max(1, std::atoi(env)) : 4096;
    const int chunk = std::max(1, std::min(prompt_len, chunk_rows / batch));
    // A call of the same shape as the previous one reuses its cache, buffers and decode graph
    // (STB_GENERATE_REUSE=0: every call builds and frees its own).
    static const int reuse_enabled = env_int("STB_GENERATE_REUSE", 1);
    const int key[5] = {batch, total, max_new, eos_count, chunk};
    stb_llama_cache *c = nullptr;
    if (m->gen) {
      if (reuse_enabled && std::equal(key, key + 5, m->gen_key)) c = m->gen;
      else stb_llama_cache_destroy(m->gen);
      m->gen = nullptr;  // owned by this call until it completes
    }
    if (!c) {
      int rc = stb_llama_cache_create(m, batch, total, &c);
      if (rc != STB_OK) throw Error(rc, stb_last_error());
    }
    if (m->tp > 1) peer_reset(s);  // collective: every rank starts the exchange counters at zero
    cudaEvent_t ev[3] = {nullptr, nullptr, nullptr};
    try {
      for (auto &e : ev) STB_CUDA(cudaEventCreate(&e));
      ensure_rows(c, batch * chunk);
      c->used = 0;
      c->out_stride = max_new;
      if (!c->out_ids) c->out_ids = alloc_owned(s, c->owned, (uint64_t)batch * max_new * 8);
      if (eos_count) {
        if (!c->eos) c->eos = alloc_owned(s, c->owned, (uint64_t)eos_count * 8);
        upload(s, eos, (uint64_t)eos_count * 8, c->eos);
      }
      c->eos_count = eos_count;
      std::vector<int64_t> part((size_t)batch * chunk);
      STB_CUDA(cudaEventRecord(ev[0], s->stream));
      STB_CUDA(cudaMemsetAsync((void *)c->state, 0, (size_t)(2 + 2 * batch) * 4, s->stream));
      int last = 0;
      for (int t0 = 0; t0 < prompt_len; t0 += chunk) {
        const int count = std::min(chunk, prompt_len - t0);
        const bool final_chunk = t0 + count == prompt_len;
        for (int b = 0; b < batch; b++)
          std::memcpy(part.data() + (size_t)b * count, prompt + (size_t)b * prompt_len + t0, (size_t)count * 8);
        upload(s, part.data(), (uint64_t)batch * count * 8, c->tokens);
        StepArgs a;
        a.rows = batch * count;
        a.count = count;
        a.all_logits = false;
        if (final_chunk) {
          // the last chunk picks each row's first token; from here the position lives on the device
          launch_kernel(set_position_kernel, dim3(1), dim3(1), 0, s->stream, false, (int *)c->state, c->used);
          a.device_pos = true;
          a.append = true;
          a.advance = count;
        } else {
          a.device_pos = false;
          a.logits = false;
        }
        count_launch(s, enqueue_step(c, a));
        if (!final_chunk) c->used += count;
        last = count;
      }
      STB_CUDA(cudaEventRecord(ev[1], s->stream));
      if (max_new > 1) {
        // decode: tokens[b*count + count-1] was rewritten in place; compact them to rows 0..batch.  The
        // strided source and the packed destination overlap once batch > last - 1 (row 0's token sits
        // at index last - 1, which row last - 1's destination overwrites), and overlapping copies are
        // undefined: gather into best_all (batch * 8 bytes at least, rewritten before its next read)
        // and copy back.
        if (last > 1) {
          STB_CUDA(cudaMemcpy2DAsync((void *)c->best_all, 8, (const void *)(c->tokens + (uint64_t)(last - 1) * 8),
                                     (size_t)last * 8, 8, batch, cudaMemcpyDeviceToDevice, s->stream));
          STB_CUDA(cudaMemcpyAsync((void *)c->tokens, (const void *)c->best_all, (size_t)batch * 8,
                                   cudaMemcpyDeviceToDevice, s->stream));
        }
        StepArgs d;
        d.rows = batch;
        d.count = 1;
        d.device_pos = true;
        d.all_logits = false;
        d.append = true;
        d.advance = 1;
        if (!c->graph) {
          cudaGraph_t g = nullptr;
          STB_CUDA(cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal));
          int step_launches = 0;
          try {
            step_launches = enqueue_step(c, d);
          } catch (...) {
            cudaStreamEndCapture(s->stream, &g);
            if (g) cudaGraphDestroy(g);
            throw;
          }
          STB_CUDA(cudaStreamEndCapture(s->stream, &g));
          cudaGraphExec_t made = nullptr;
          cudaError_t e = cudaGraphInstantiate(&made, g, 0);
          cudaGraphDestroy(g);
          STB_CUDA(e);
          c->graph = made;
          c->graph_launches = step_launches;
        }
        cudaGraphExec_t exec = c->graph;
        const int step_launches = c->graph_launches;
        for (int i = 1; i < max_new; i++) STB_CUDA(cudaGraphLaunch(exec, s->stream));
        count_launch(s, (uint64_t)step_launches * (max_new - 1));
      }
      STB_CUDA(cudaEventRecord(ev[2], s->stream));
      std::vector<int64_t> picks((size_t)batch * max_new);
      std::vector<int> st(2 + 2 * batch);
      download(s, c->out_ids, picks.data(), picks.size() * 8);
      download(s, c->state, st.data(), st.size() * 4);
      for (int b = 0; b < batch; b++) {
        const int n = st[2 + batch + b];
        std::memcpy(out + (size_t)b * total + prompt_len, picks.data() + (size_t)b * max_new, (size_t)n * 8);
        if (generated) generated[b] = n;
      }
      if (timings_ms) {
        STB_CUDA(cudaEventElapsedTime(&timings_ms[0], ev[0], ev[1]));
        STB_CUDA(cudaEventElapsedTime(&timings_ms[1], ev[1], ev[2]));
      }
    } catch (...) {
      for (auto &e : ev)
        if (e) cudaEventDestroy(e);
      stb_llama_cache_destroy(c);
      throw;
    }
    for (auto &e : ev)
      if (e) cudaEventDestroy(e);
    if (reuse_enabled) {
      m->gen = c;
      std::copy(key, key + 5, m->gen_key);
    } else {
      int rc = stb_llama_cache_destroy(c);
      if (rc != STB_OK) throw Error(rc, stb_last_error());
    }
  });
}

}  // extern "C"
