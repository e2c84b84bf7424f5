// Decode-shaped Linear: y[M,N] = x[M,K] . W[N,K]^T for M <= 32 tokens (M-tiled beyond).
//
// The weight is the (out,in) half payload exactly as stored in the safetensors file
// (nn/src/main/scala/scalatorch/nn/Linear.scala:7, (out,in) layout).  K is the fastest axis of
// both x and W, so a row of W is one contiguous stream: lanes of a thread group walk it in
// 16-byte (8-element) chunks with L1-bypassing loads, widen the halves in registers
// (SafeTensors.scala:71-72 semantics, exact), and accumulate x.W with FP32 FMA.  Activations stay
// Float32.  One thread group = TPR consecutive threads covers the whole K range of ROWS rows and
// MT tokens; the group reduces with xor shuffles (and shared memory across warps when TPR > 32),
// so every output is produced by exactly one group in a fixed order: results are deterministic.
//
// Optional fused pieces for the Llama decode step:
//   * RMSNorm prologue (CpuFloatBackend.rmsNorm, cpu/.../CpuFloatBackend.scala:78-93): the block
//     computes each token row's inverse RMS in double and normalises x chunks as it loads them,
//     (float)((double)x * inverse * w), the reference's expression.
//   * epilogues: bias, residual add (LlamaBlock h = x + f(x), LlamaModel.scala:49-52), SiLU(gate)*up
//     on interleaved gate/up rows (LlamaMLP, LlamaModel.scala:39-43), RoPE + KV-cache append on
//     paired q/k/v rows (CpuAttention.rope + LlamaCache.Layer.append), and logits with a per-block
//     greedy argmax candidate (TokenSampler strict '>' ties to the lowest id).
#pragma once

#include "common.cuh"
#include "peer.cuh"

namespace stb {

// EPI_PEER: the partial sums of a row-split projection go to every tensor-parallel rank's receive
// slots (peer.cuh) instead of y.
enum GemvEpi { EPI_PLAIN = 0, EPI_RESID = 1, EPI_SILU = 2, EPI_QKV = 3, EPI_LOGITS = 4, EPI_PEER = 5 };

struct GemvParams {
  const float *x = nullptr;
  int ldx = 0;
  const void *w = nullptr;  // [N, K] half, rows 16-byte aligned (K % 8 == 0)
  int M = 0, N = 0, K = 0;
  float *y = nullptr;
  int ldy = 0;
  const float *bias = nullptr;      // EPI_PLAIN
  const float *residual = nullptr;  // EPI_RESID: y = residual + acc (may alias y)
  int ldr = 0;
  const float *norm_w = nullptr;  // RMSNorm weight over K, or null
  double norm_eps = 1e-6;
  // EPI_QKV
  const double2 *rope = nullptr;  // [positions][hd/2] (cos, sin) in double
  const int *pos_dev = nullptr;   // device position of token 0, or null -> pos0
  int pos0 = 0;
  int count = 1;  // tokens per batch row: row m = b*count + t
  int nh = 0, kvh = 0, hd = 0, capacity = 0;
  float *k_cache = nullptr, *v_cache = nullptr;  // [batch][kvh][capacity][hd] of this layer
  // EPI_LOGITS
  unsigned long long *best = nullptr;  // [M] greedy candidate keys (argmax_key), or null
  int row_offset = 0;                  // global index of row 0 (vocab shard offset)
  const int *stop = nullptr;  // device flag; nonzero makes the kernel a no-op
  bool pdl = false;           // launched as a programmatic dependent of the previous kernel
  PeerArgs peer{};            // EPI_PEER: receive slots of every rank (slot row stride = ldy)
};

struct GemvConfig {
  int mt, rows, tpr;
};

__device__ __forceinline__ double block_sum_double(double v, double *scratch) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  double total = 0.0;
  if (threadIdx.x == 0) {
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) total += scratch[i];
    scratch[0] = total;
  }
  __syncthreads();
  total = scratch[0];
  __syncthreads();
  return total;
}

// Greedy candidates as one 64-bit key: an order-preserving image of the logit in the high word
// (-0 folded onto +0, since the reference compares numerically) and the complement of the token
// id in the low word, so the unsigned maximum is the largest logit and, among equal logits, the
// lowest id -- TokenSampler's strict '>' scan (TokenSampler.scala:32-38).
__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
  if (v == 0.0f) v = 0.0f;
  const uint32_t b = __float_as_uint(v);
  const uint32_t ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)ord << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}
__device__ __forceinline__ int argmax_key_index(unsigned long long key) {
  return (int)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull));
}

// SiLU of CpuFloatBackend.silu (CpuFloatBackend.scala:70-77), in double.
__device__ __forceinline__ float silu_ref(float x) {
  double v = (double)x;
  double sigmoid;
  if (v >= 0.0) sigmoid = __ddiv_rn(1.0, __dadd_rn(1.0, exp(-v)));
  else {
    double e = exp(v);
    sigmoid = __ddiv_rn(e, __dadd_rn(1.0, e));
  }
  return (isinf(v) && v < 0.0) ? -0.0f : __double2float_rn(__dmul_rn(v, sigmoid));
}

// EPI_QKV for one pair of projection rows: pair pi enumerates q heads, then k heads, then v
// heads, each head contributing hd/2 pairs (d, d + hd/2).  q and k pairs are rotated
// (CpuAttention.rope: (a*c - b*s).toFloat, (b*c + a*s).toFloat in double, no contraction) and q
// goes to y, k to the key cache; v pairs go to the value cache unrotated.  Token row mm is batch
// row mm / count at position pos_base + mm % count.
__device__ __forceinline__ void qkv_store_pair(const GemvParams &p, int mm, int pi, float fa, float fb,
                                               int pos_base) {
  const int half = p.hd >> 1;
  const int qpairs = p.nh * half, kpairs = p.kvh * half;
  const int bb = mm / p.count, t = mm % p.count;
  const int pos = pos_base + t;
  if (pi < qpairs + kpairs) {
    const int local = pi < qpairs ? pi : pi - qpairs;
    const int h = local / half, d = local % half;
    const double2 cs = p.rope[(size_t)pos * half + d];
    const double a = (double)fa, b = (double)fb;
    const float oa = __double2float_rn(__dsub_rn(__dmul_rn(a, cs.x), __dmul_rn(b, cs.y)));
    const float ob = __double2float_rn(__dadd_rn(__dmul_rn(b, cs.x), __dmul_rn(a, cs.y)));
    if (pi < qpairs) {
      float *q = p.y + (size_t)mm * p.ldy + (size_t)h * p.hd;
      q[d] = oa;
      q[d + half] = ob;
    } else {
      float *kc = p.k_cache + (((size_t)bb * p.kvh + h) * p.capacity + pos) * p.hd;
      kc[d] = oa;
      kc[d + half] = ob;
    }
  } else {
    const int local = pi - qpairs - kpairs;
    const int h = local / half, d = local % half;
    float *vc = p.v_cache + (((size_t)bb * p.kvh + h) * p.capacity + pos) * p.hd;
    vc[d] = fa;
    vc[d + half] = fb;
  }
}

template <int MT, int ROWS, int TPR, typename WT, int EPI>
__global__ void __launch_bounds__(256) gemv_kernel(const GemvParams p, int mtiles, int items) {
  constexpr int G = 256 / TPR;
  constexpr int LW = TPR < 32 ? TPR : 32;
  __shared__ double s_inv[MT];
  __shared__ double s_scratch[8];
  __shared__ float s_out[G][ROWS][MT];
  __shared__ float s_red[TPR > 32 ? 8 : 1][ROWS * MT];
  __shared__ int s_inv_tile;  // m-tile whose inverse RMS s_inv holds

  const int tid = threadIdx.x;
  const int g = tid / TPR, lane = tid % TPR;
  if (tid == 0) s_inv_tile = -1;
  __syncthreads();
  // Grid-stride over (m-tile, row block) items: the grid holds at most what is resident at once,
  // so no partial last wave.  Each item is produced by one block in a fixed order.
  for (int item = blockIdx.x; item < items; item += gridDim.x) {
  const bool first = item == (int)blockIdx.x;
  const int mtile = item % mtiles, rblock = item / mtiles;
  const int m0 = mtile * MT;
  const int mcount = min(MT, p.M - m0);
  const int rowbase = (rblock * G + g) * ROWS;
  const int nchunk = p.K >> 3;

  // The weights never depend on the previous kernel.  Load this thread's first PRE chunks into
  // registers now and (under programmatic launch) pull the rest of the block's rows -- one
  // contiguous range -- into L2, all before waiting for the producer of x.
  constexpr int PRE = 2;  // the consumer loop below selects wpre[0] / wpre[1] with constant indices
  static_assert(PRE == 2, "preload depth");
  const uint16_t *W = (const uint16_t *)p.w;
  uint4 wpre[PRE][ROWS];
#pragma unroll
  for (int i = 0; i < PRE; i++) {
    const int c = lane + i * TPR;
#pragma unroll
    for (int r = 0; r < ROWS; r++) {
      const int row = rowbase + r;
      wpre[i][r] = (c < nchunk && row < p.N) ? ld_stream_u4(W + (size_t)row * p.K + (size_t)c * 8)
                                             : make_uint4(0, 0, 0, 0);
    }
  }
  if (p.pdl && first) {
    if (tid == 0 && mtile == 0 && nchunk > PRE * TPR) {
      const int r0 = rblock * G * ROWS;
      const int nrows = min(G * ROWS, p.N - r0);
      if (nrows > 0) {
        const char *base = (const char *)p.w + (size_t)r0 * p.K * 2;
        size_t bytes = (size_t)nrows * p.K * 2;
        for (size_t off = 0; off < bytes; off += 65536)
          prefetch_l2(base + off, (uint32_t)(bytes - off < 65536 ? bytes - off : 65536));
      }
    }
    pdl_wait();
  }
  if (p.stop && *p.stop) return;

  // The residual values this thread's epilogue adds, loaded now so the load overlaps the product
  // (epilogue item i = tid + 256 j covers (token m, row) = (i / (G*ROWS), i % (G*ROWS))).
  const int blockrow0 = rblock * G * ROWS;
  float resid_pre[2] = {0.0f, 0.0f};
  if constexpr (EPI == EPI_RESID) {
    static_assert(G * ROWS * MT <= 512, "residual prefetch covers two epilogue items per thread");
#pragma unroll
    for (int j = 0; j < 2; j++) {
      const int i = tid + 256 * j;
      const int m = i / (G * ROWS), row = blockrow0 + i % (G * ROWS);
      if (i < G * ROWS * MT && m < mcount && row < p.N) resid_pre[j] = p.residual[(size_t)(m0 + m) * p.ldr + row];
    }
  }

  if (p.norm_w && s_inv_tile != mtile) {
    __syncthreads();  // every thread has compared s_inv_tile before thread 0 updates it
    for (int m = 0; m < MT; m++) {
      double sq = 0.0;
      if (m < mcount) {
        const float *xr = p.x + (size_t)(m0 + m) * p.ldx;
        for (int k = tid; k < p.K; k += 256) {
          double v = (double)xr[k];
          sq = __dadd_rn(sq, __dmul_rn(v, v));
        }
      }
      double total = block_sum_double(sq, s_scratch);
      if (tid == 0) s_inv[m] = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(total, (double)p.K), p.norm_eps)));
    }
    if (tid == 0) s_inv_tile = mtile;
    __syncthreads();
  }

  float acc[ROWS][MT];
#pragma unroll
  for (int r = 0; r < ROWS; r++)
#pragma unroll
    for (int m = 0; m < MT; m++) acc[r][m] = 0.0f;

  // Chunks in increasing order; the weight loads run PRE chunk-steps ahead of the FMAs (the PRE
  // preloaded ones first), so each thread keeps (PRE + 1) x ROWS 16-byte loads in flight.
  uint4 cur[ROWS], nxt[ROWS];
#pragma unroll
  for (int r = 0; r < ROWS; r++) {
    cur[r] = wpre[0][r];
    nxt[r] = wpre[PRE - 1][r];
  }
  for (int c = lane; c < nchunk; c += TPR) {
    uint4 wv[ROWS], fut[ROWS];
    const int cf = c + PRE * TPR;
#pragma unroll
    for (int r = 0; r < ROWS; r++) {
      const int row = rowbase + r;
      fut[r] = (cf < nchunk && row < p.N) ? ld_stream_u4(W + (size_t)row * p.K + (size_t)cf * 8)
                                          : make_uint4(0, 0, 0, 0);
      wv[r] = cur[r];
      cur[r] = nxt[r];
      nxt[r] = fut[r];
    }
    float xv[MT][8];
#pragma unroll
    for (int m = 0; m < MT; m++) {
      if (m < mcount) {
        const float4 *xp = reinterpret_cast<const float4 *>(p.x + (size_t)(m0 + m) * p.ldx + (size_t)c * 8);
        float4 a = __ldg(xp), b = __ldg(xp + 1);
        xv[m][0] = a.x; xv[m][1] = a.y; xv[m][2] = a.z; xv[m][3] = a.w;
        xv[m][4] = b.x; xv[m][5] = b.y; xv[m][6] = b.z; xv[m][7] = b.w;
        if (p.norm_w) {
          const float4 *np = reinterpret_cast<const float4 *>(p.norm_w + (size_t)c * 8);
          float4 na = __ldg(np), nb = __ldg(np + 1);
          const float nw[8] = {na.x, na.y, na.z, na.w, nb.x, nb.y, nb.z, nb.w};
          const double inv = s_inv[m];
#pragma unroll
          for (int j = 0; j < 8; j++)
            xv[m][j] = __double2float_rn(__dmul_rn(__dmul_rn((double)xv[m][j], inv), (double)nw[j]));
        }
      } else {
#pragma unroll
        for (int j = 0; j < 8; j++) xv[m][j] = 0.0f;
      }
    }
#pragma unroll
    for (int r = 0; r < ROWS; r++) {
      const float2 w01 = widen2<WT>(wv[r].x), w23 = widen2<WT>(wv[r].y);
      const float2 w45 = widen2<WT>(wv[r].z), w67 = widen2<WT>(wv[r].w);
#pragma unroll
      for (int m = 0; m < MT; m++) {
        float a = acc[r][m];
        a = fmaf(w01.x, xv[m][0], a);
        a = fmaf(w01.y, xv[m][1], a);
        a = fmaf(w23.x, xv[m][2], a);
        a = fmaf(w23.y, xv[m][3], a);
        a = fmaf(w45.x, xv[m][4], a);
        a = fmaf(w45.y, xv[m][5], a);
        a = fmaf(w67.x, xv[m][6], a);
        a = fmaf(w67.y, xv[m][7], a);
        acc[r][m] = a;
      }
    }
  }

  if (p.pdl && first) pdl_trigger();  // the next kernel may start its own weight prefetch now

  // Group reduction in a fixed order.
#pragma unroll
  for (int r = 0; r < ROWS; r++)
#pragma unroll
    for (int m = 0; m < MT; m++)
#pragma unroll
      for (int off = LW / 2; off > 0; off >>= 1) acc[r][m] += __shfl_xor_sync(0xffffffffu, acc[r][m], off);
  if constexpr (TPR <= 32) {
    if (lane == 0) {
#pragma unroll
      for (int r = 0; r < ROWS; r++)
#pragma unroll
        for (int m = 0; m < MT; m++) s_out[g][r][m] = acc[r][m];
    }
  } else {
    const int warp = tid >> 5;
    if ((tid & 31) == 0) {
#pragma unroll
      for (int r = 0; r < ROWS; r++)
#pragma unroll
        for (int m = 0; m < MT; m++) s_red[warp][r * MT + m] = acc[r][m];
    }
    __syncthreads();
    constexpr int WPG = TPR / 32;
    for (int i = tid; i < G * ROWS * MT; i += 256) {
      const int gg = i / (ROWS * MT), rm = i % (ROWS * MT);
      float sum = 0.0f;
#pragma unroll
      for (int w = 0; w < WPG; w++) sum += s_red[gg * WPG + w][rm];
      s_out[gg][rm / MT][rm % MT] = sum;
    }
  }
  __syncthreads();

  if constexpr (EPI == EPI_PLAIN || EPI == EPI_RESID || EPI == EPI_LOGITS) {
    for (int i = tid, j = 0; i < G * ROWS * MT; i += 256, j++) {
      const int m = i / (G * ROWS), rr = i % (G * ROWS);
      const int row = blockrow0 + rr;
      if (m >= mcount || row >= p.N) continue;
      float v = s_out[rr / ROWS][rr % ROWS][m];
      const size_t mm = (size_t)(m0 + m);
      if constexpr (EPI == EPI_PLAIN) {
        if (p.bias) v = v + p.bias[row];
      } else if constexpr (EPI == EPI_RESID) {
        v = (j == 0 ? resid_pre[0] : resid_pre[1]) + v;
      }
      p.y[mm * p.ldy + row] = v;
    }
    if constexpr (EPI == EPI_LOGITS) {
      if (p.best && tid < mcount) {
        const int m = tid;
        float best = 0.0f;
        int besti = -1;
        for (int rr = 0; rr < G * ROWS; rr++) {
          const int row = blockrow0 + rr;
          if (row >= p.N) break;
          const float v = s_out[rr / ROWS][rr % ROWS][m];
          if (besti < 0 || v > best) {  // strict '>': the lowest row wins inside the block
            best = v;
            besti = row;
          }
        }
        if (besti >= 0) atomicMax(&p.best[m0 + m], argmax_key(best, besti + p.row_offset));
      }
    }
  } else if constexpr (EPI == EPI_PEER) {
    // one 8-byte (use, value) word per output to every rank, this rank's slot (peer.cuh)
    const uint32_t use = (uint32_t)(p.peer.my_epoch[p.peer.region] + 1ull);
    const size_t slot = ((size_t)p.peer.region * p.peer.tp + p.peer.rank) * p.peer.slot_elems;
    for (int i = tid; i < G * ROWS * MT; i += 256) {
      const int m = i / (G * ROWS), rr = i % (G * ROWS);
      const int row = blockrow0 + rr;
      if (m >= mcount || row >= p.N) continue;
      const unsigned long long w = peer_word(s_out[rr / ROWS][rr % ROWS][m], use);
      const size_t off = slot + (size_t)(m0 + m) * p.ldy + row;
      for (int r = 0; r < p.peer.tp; r++) peer_store(p.peer.slots[r] + off, w);
    }
  } else if constexpr (EPI == EPI_SILU) {
    // Rows are interleaved gate/up: row 2i = gate_i, row 2i+1 = up_i; output width N/2.
    constexpr int PAIRS = ROWS / 2;
    for (int i = tid; i < G * PAIRS * MT; i += 256) {
      const int m = i / (G * PAIRS), pr = i % (G * PAIRS);
      const int gg = pr / PAIRS, r = (pr % PAIRS) * 2;
      const int row = blockrow0 + gg * ROWS + r;
      if (m >= mcount || row >= p.N) continue;
      const float gate = s_out[gg][r][m], up = s_out[gg][r + 1][m];
      // LlamaMLP: multiply(silu(gate), up) -- Float32 product of the Float32 SiLU.
      p.y[(size_t)(m0 + m) * p.ldy + (row >> 1)] = silu_ref(gate) * up;
    }
  } else if constexpr (EPI == EPI_QKV) {
    // Rows are pairs (d, d + hd/2) of one head (qkv_store_pair).
    constexpr int PAIRS = ROWS / 2;
    const int pos_base = p.pos_dev ? *p.pos_dev : p.pos0;
    for (int i = tid; i < G * PAIRS * MT; i += 256) {
      const int m = i / (G * PAIRS), pr = i % (G * PAIRS);
      const int gg = pr / PAIRS, r = (pr % PAIRS) * 2;
      const int row = blockrow0 + gg * ROWS + r;
      if (m >= mcount || row >= p.N) continue;
      qkv_store_pair(p, m0 + m, row >> 1, s_out[gg][r][m], s_out[gg][r + 1][m], pos_base);
    }
  }
  __syncthreads();  // the shared arrays are reused by the block's next item
  }
}

// Generic fallback for layouts the vector kernel does not take (K % 8 != 0, unaligned x or W,
// ldx not a multiple of 4): one warp per output, scalar widening loads.  Plain epilogue only.
template <typename WT>
__global__ void gemv_scalar_kernel(const float *x, int ldx, const void *w, int w_f32, const float *bias,
                                   float *y, int ldy, int M, int N, int K) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= M * N) return;
  const int m = warp / N, n = warp % N;
  float acc = 0.0f;
  for (int k = lane; k < K; k += 32) {
    float wv;
    if (w_f32) wv = ((const float *)w)[(size_t)n * K + k];
    else wv = widen1<WT>(((const uint16_t *)w)[(size_t)n * K + k]);
    acc = fmaf(x[(size_t)m * ldx + k], wv, acc);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) y[(size_t)m * ldy + n] = bias ? acc + bias[n] : acc;
}

// Picks the thread-group shape for a problem.  paired = epilogue needs even ROWS.
GemvConfig choose_gemv(int M, int N, int K, bool paired);
// Launches the vector kernel for the configured epilogue.  Requires K % 8 == 0, 16-byte aligned
// W and x rows.  Returns the number of row blocks (the partial count for EPI_LOGITS).
template <int EPI>
int launch_gemv(const GemvParams &p, int w_dtype, GemvConfig cfg, cudaStream_t stream);
int gemv_row_blocks(int N, GemvConfig cfg);
// The launch shape launch_gemv<epi> really uses for a requested config.
GemvConfig normalize_gemv(GemvConfig cfg, int epi);
// Thread blocks one launch_gemv<epi> of (M, N) with cfg runs.
int gemv_grid_blocks(int M, int N, GemvConfig cfg, int epi);

// Tensor-core skinny form (gemm_skinny.cu) for BF16 weights, token rows in blocks of up to 64, the
// activations split into three BF16 terms (FP32-accurate), with the same prologue (RMSNorm) and
// epilogues as the vector kernel.  p.stop must be null.  skinny_eligible() says whether a
// problem takes it (STB_SKINNY=0 keeps the vector kernel; STB_SKINNY_MIN_ROWS / _MAX_ROWS bound
// M, default 1 .. unbounded); skinny_scratch_bytes() is the scratch one call of (M, N, K) needs.
bool skinny_eligible(int M, int N, int K, int w_dtype, const void *w);
uint64_t skinny_scratch_bytes(int M, int N, int K, int device);
// Sets the kernels' shared-memory limits on `device` (before a graph capture that launches them).
void skinny_prepare(int device);
// The next projection's prologue done by this projection's fixup (one 64-row block): its activation
// terms go to x3 [3][skinny_nt(M)][Kn] -- EPI_SILU: SiLU(gate) * up split for the down projection
// (Kn = N / 2, norm_w unused); EPI_RESID: the residual add, then RMSNorm with norm_w / eps and the split
// (Kn = N, skinny_norm_fusable(N)).  The buffer must not overlap the scratch.
struct SkinnyNext {
  uint16_t *x3 = nullptr;
  const float *norm_w = nullptr;
  double eps = 1e-6;
};
// The stream-K pieces of a skinny GEMM whose fixup is left to its consumer: output (m, n) is the sum
// over pieces c = first .. last of part[((t * pmax + c - first) * M + m) * 128 + n % 128], t = n / 128,
// first = skinny_cta_of(t * kbs, T, G), last = skinny_cta_of((t + 1) * kbs - 1, T, G), in piece order.
struct SkinnyParts {
  const float *part = nullptr;
  int kbs = 0;
  long long T = 0;
  int G = 0, pmax = 0, M = 0;
};

// The CTA whose stream-K range (CTA c covers iterations [floor(c T / G), floor((c + 1) T / G))) holds
// iteration i: the largest c with floor(c T / G) <= i, which is floor(((i + 1) G - 1) / T)
// (c T / G < i + 1  <=>  c T <= (i + 1) G - 1); in 32-bit arithmetic when T G fits (a 64-bit
// division is a long instruction sequence on the fixups' critical path).
__device__ __forceinline__ int skinny_cta_of(long long i, long long T, int G) {
  if ((unsigned long long)T * (unsigned)G <= 0xFFFFFFFFull)
    return (int)(((unsigned)(i + 1) * (unsigned)G - 1u) / (unsigned)T);
  return (int)(((unsigned long long)(i + 1) * (unsigned)G - 1ull) / (unsigned long long)T);
}

// Enqueues prologue -> stream-K GEMM -> fixup/epilogue per 64-row block (3 kernels each, all
// programmatic dependents except the first when !p.pdl).  With x3_ready (M <= 64, no RMSNorm) the
// previous kernel has already written the activation terms x3 [3][skinny_nt(M)][K] there (16-byte
// aligned; at the start of the scratch, or a SkinnyNext buffer) and the prologue is skipped.  With
// next, the fixup also writes the next projection's terms (SkinnyNext).  With deferred (M <= 64) no fixup
// is launched: the pieces stay in the scratch for the next kernel, described in *deferred.  Returns the
// number of kernels launched.
template <int EPI>
int skinny_launch(const GemvParams &p, void *scratch, uint64_t scratch_bytes, int *err, int device,
                  cudaStream_t stream, const uint16_t *x3_ready = nullptr, const SkinnyNext *next = nullptr,
                  SkinnyParts *deferred = nullptr);
// Token rows of the activation-term tile for a block of M <= 64 rows: 16, 32 or 64.
int skinny_nt(int M);
// Whether a residual projection of N outputs can do the next projection's RMSNorm prologue (SkinnyNext).
bool skinny_norm_fusable(int N);

}  // namespace stb
