// Decode GEMV dispatch and the stb_linear entry points (FloatBackend.matmul against an (out,in)
// half weight; nn.Linear.apply, nn/src/main/scala/scalatorch/nn/Linear.scala:11-17).
#include <cstdlib>
#include <mutex>

#include "gemv.cuh"

namespace stb {

int gemv_row_blocks(int N, GemvConfig cfg) {
  const int rows_per_block = (256 / cfg.tpr) * cfg.rows;
  return (N + rows_per_block - 1) / rows_per_block;
}

// K fixes the thread-group width (each lane walks at most ~8 chunks of 8 elements); then the
// number of rows per thread is the largest that still gives the grid enough blocks to cover
// every SM several times.  STB_GEMV_TPR / STB_GEMV_ROWS override for sweeps.
GemvConfig choose_gemv(int M, int N, int K, bool paired) {
  GemvConfig c;
  c.mt = M <= 1 ? 1 : (M <= 2 ? 2 : (M <= 4 ? 4 : 8));
  if (paired && c.mt != 1) c.mt = 8;
  const int nchunk = K / 8;
  int tpr = 16;
  while (tpr < 256 && (nchunk + tpr - 1) / tpr > 8) tpr *= 2;
  const int mtiles = (M + c.mt - 1) / c.mt;
  const int target_blocks = 148 * 4;
  int rows = paired ? 2 : 1;
  for (int cand : {4, 2}) {
    const int rpb = (256 / tpr) * cand;
    const long blocks = (long)((N + rpb - 1) / rpb) * mtiles;
    if (blocks >= target_blocks) {
      rows = cand;
      break;
    }
  }
  // Few rows: widen the group so more blocks share the work, while each lane keeps >= 1 chunk.
  while (tpr < 256 && 2 * tpr <= nchunk) {
    const int rpb = (256 / tpr) * rows;
    const long blocks = (long)((N + rpb - 1) / rpb) * mtiles;
    if (blocks >= 148) break;
    tpr *= 2;
  }
  c.tpr = env_int("STB_GEMV_TPR", tpr);
  c.rows = env_int("STB_GEMV_ROWS", rows);
  if (paired && (c.rows & 1)) c.rows = 2;
  return c;
}

template <int MT, int ROWS, int TPR, typename WT, int EPI>
static void launch_one(const GemvParams &p, cudaStream_t stream) {
  const int mtiles = (p.M + MT - 1) / MT;
  const int rpb = (256 / TPR) * ROWS;
  const long items = (long)((p.N + rpb - 1) / rpb) * mtiles;
  if (items > 0x7fffffffL) throw Error(STB_ERR_INVALID, "GEMV grid too large");
  // One block per item: the hardware starts a new block as soon as one retires, overlapping one
  // block's reduction with the next block's loads (a resident-capped grid-stride loop measured
  // slower on the 1 GB lm_head: 229 vs 211 us).
  const long blocks = items;
  launch_kernel(gemv_kernel<MT, ROWS, TPR, WT, EPI>, dim3((unsigned)blocks), dim3(256), 0, stream, p.pdl, p, mtiles,
                (int)items);
}

template <int MT, int ROWS, typename WT, int EPI>
static void dispatch_tpr(const GemvParams &p, int tpr, cudaStream_t stream) {
  switch (tpr) {
    case 16: launch_one<MT, ROWS, 16, WT, EPI>(p, stream); break;
    case 32: launch_one<MT, ROWS, 32, WT, EPI>(p, stream); break;
    case 64: launch_one<MT, ROWS, 64, WT, EPI>(p, stream); break;
    case 128: launch_one<MT, ROWS, 128, WT, EPI>(p, stream); break;
    case 256: launch_one<MT, ROWS, 256, WT, EPI>(p, stream); break;
    default: throw Error(STB_ERR_INVALID, "unsupported GEMV group width " + std::to_string(tpr));
  }
}

template <int MT, typename WT, int EPI>
static void dispatch_rows(const GemvParams &p, GemvConfig cfg, cudaStream_t stream) {
  if constexpr (EPI == EPI_SILU || EPI == EPI_QKV) {
    if (cfg.rows == 4) dispatch_tpr<MT, 4, WT, EPI>(p, cfg.tpr, stream);
    else dispatch_tpr<MT, 2, WT, EPI>(p, cfg.tpr, stream);
  } else if constexpr (EPI == EPI_PLAIN) {
    if (cfg.rows == 4) dispatch_tpr<MT, 4, WT, EPI>(p, cfg.tpr, stream);
    else if (cfg.rows == 2) dispatch_tpr<MT, 2, WT, EPI>(p, cfg.tpr, stream);
    else dispatch_tpr<MT, 1, WT, EPI>(p, cfg.tpr, stream);
  } else {
    if (cfg.rows >= 4) dispatch_tpr<MT, 4, WT, EPI>(p, cfg.tpr, stream);
    else dispatch_tpr<MT, 2, WT, EPI>(p, cfg.tpr, stream);
  }
}

template <typename WT, int EPI>
static void dispatch_mt(const GemvParams &p, GemvConfig cfg, cudaStream_t stream) {
  if constexpr (EPI == EPI_PLAIN) {
    switch (cfg.mt) {
      case 1: dispatch_rows<1, WT, EPI>(p, cfg, stream); break;
      case 2: dispatch_rows<2, WT, EPI>(p, cfg, stream); break;
      case 4: dispatch_rows<4, WT, EPI>(p, cfg, stream); break;
      default: dispatch_rows<8, WT, EPI>(p, cfg, stream); break;
    }
  } else {
    if (cfg.mt == 1) dispatch_rows<1, WT, EPI>(p, cfg, stream);
    else dispatch_rows<8, WT, EPI>(p, cfg, stream);
  }
}

// The shape actually instantiated for an epilogue: fused epilogues exist for MT in {1, 8} and
// ROWS in {2, 4}; the plain one for MT in {1, 2, 4, 8} and ROWS in {1, 2, 4}.  Row-block counts
// (the lm_head candidate slots) must be computed from this, not from the request.
GemvConfig normalize_gemv(GemvConfig cfg, int epi) {
  if (epi != EPI_PLAIN) {
    if (cfg.mt != 1) cfg.mt = 8;
    cfg.rows = cfg.rows >= 4 ? 4 : 2;
  } else {
    cfg.mt = cfg.mt <= 1 ? 1 : (cfg.mt <= 2 ? 2 : (cfg.mt <= 4 ? 4 : 8));
    cfg.rows = cfg.rows >= 4 ? 4 : (cfg.rows >= 2 ? 2 : 1);
  }
  return cfg;
}

template <int EPI>
int launch_gemv(const GemvParams &p, int w_dtype, GemvConfig cfg, cudaStream_t stream) {
  cfg = normalize_gemv(cfg, EPI);
  if (w_dtype == STB_BF16) dispatch_mt<__nv_bfloat16, EPI>(p, cfg, stream);
  else if (w_dtype == STB_F16) dispatch_mt<__half, EPI>(p, cfg, stream);
  else throw Error(STB_ERR_INVALID, "GEMV weight dtype must be BF16 or F16");
  check_launch("gemv");
  return gemv_row_blocks(p.N, cfg);
}

template int launch_gemv<EPI_PLAIN>(const GemvParams &, int, GemvConfig, cudaStream_t);
template int launch_gemv<EPI_RESID>(const GemvParams &, int, GemvConfig, cudaStream_t);
template int launch_gemv<EPI_SILU>(const GemvParams &, int, GemvConfig, cudaStream_t);
template int launch_gemv<EPI_QKV>(const GemvParams &, int, GemvConfig, cudaStream_t);
template int launch_gemv<EPI_LOGITS>(const GemvParams &, int, GemvConfig, cudaStream_t);
template int launch_gemv<EPI_PEER>(const GemvParams &, int, GemvConfig, cudaStream_t);

int gemv_grid_blocks(int M, int N, GemvConfig cfg, int epi) {
  cfg = normalize_gemv(cfg, epi);
  return gemv_row_blocks(N, cfg) * ((M + cfg.mt - 1) / cfg.mt);
}

__global__ void fill_bias_kernel(float *y, int ldy, const float *bias, int M, int N) {
  const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
  if (i >= (long)M * N) return;
  const int m = (int)(i / N), n = (int)(i % N);
  y[(size_t)m * ldy + n] = bias ? bias[n] : 0.0f;
}

void linear(stb_session *s, uint64_t x, int ldx, uint64_t w, int w_dtype, uint64_t bias, uint64_t y, int ldy,
            int M, int N, int K) {
  STB_REQUIRE(M >= 0 && N >= 0 && K >= 0, "Linear dimensions must be nonnegative");
  STB_REQUIRE(w_dtype == STB_F32 || w_dtype == STB_BF16 || w_dtype == STB_F16, "unsupported weight dtype");
  if (M == 0 || N == 0) return;
  STB_REQUIRE(y != 0, "Linear output is null");
  STB_REQUIRE(ldy >= N && (K == 0 || ldx >= K), "Linear leading dimensions too small");
  if (K == 0) {  // empty inner dimension: bias or zeros (BackendSuite.scala:34)
    const long total = (long)M * N;
    fill_bias_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s->stream>>>((float *)y, ldy, (const float *)bias,
                                                                            M, N);
    check_launch("linear(K=0)");
    count_launch(s);
    return;
  }
  STB_REQUIRE(x != 0 && w != 0, "Linear input or weight is null");
  const size_t esz = w_dtype == STB_F32 ? 4 : 2;
  const bool vec = w_dtype != STB_F32 && K % 8 == 0 && ldx % 4 == 0 && (x % 16) == 0 && (w % 16) == 0 &&
                   ((uint64_t)K * esz) % 16 == 0;
  if (!vec) {
    const long warps = (long)M * N;
    const long threads = warps * 32;
    STB_REQUIRE(threads / 256 < 0x7fffffffL, "Linear too large for the scalar path");
    if (w_dtype == STB_F16)
      gemv_scalar_kernel<__half><<<(unsigned)((threads + 255) / 256), 256, 0, s->stream>>>(
          (const float *)x, ldx, (const void *)w, 0, (const float *)bias, (float *)y, ldy, M, N, K);
    else
      gemv_scalar_kernel<__nv_bfloat16><<<(unsigned)((threads + 255) / 256), 256, 0, s->stream>>>(
          (const float *)x, ldx, (const void *)w, w_dtype == STB_F32, (const float *)bias, (float *)y, ldy, M, N,
          K);
    check_launch("gemv_scalar");
    count_launch(s);
    return;
  }
  GemvParams p;
  p.x = (const float *)x;
  p.ldx = ldx;
  p.w = (const void *)w;
  p.M = M;
  p.N = N;
  p.K = K;
  p.y = (float *)y;
  p.ldy = ldy;
  p.bias = (const float *)bias;
  if (skinny_eligible(M, N, K, w_dtype, (const void *)w)) {
    // 2+ token rows: tensor cores with the activations split into three BF16 terms, 64-row blocks
    const uint64_t bytes = skinny_scratch_bytes(M, N, K, s->device);
    void *scratch = (void *)session_scratch(s, bytes);
    count_launch(s, skinny_launch<EPI_PLAIN>(p, scratch, bytes, session_error_word(s), s->device, s->stream));
    return;
  }
  launch_gemv<EPI_PLAIN>(p, w_dtype, choose_gemv(M, N, K, false), s->stream);
  count_launch(s);
}

}  // namespace stb

using namespace stb;

extern "C" {

int stb_linear_ld(stb_session *s, uint64_t x, int ldx, uint64_t w, int w_dtype, uint64_t bias, uint64_t y,
                  int ldy, int M, int N, int K) {
  return guarded([&] {
    enter(s);
    linear(s, x, ldx, w, w_dtype, bias, y, ldy, M, N, K);
  });
}

int stb_linear(stb_session *s, uint64_t x, uint64_t w, int w_dtype, uint64_t bias, uint64_t y, int M, int N,
               int K) {
  return guarded([&] {
    enter(s);
    linear(s, x, K, w, w_dtype, bias, y, N, M, N, K);
  });
}

int stb_linear_host(stb_session *s, const float *x_host, uint64_t w, int w_dtype, uint64_t bias, float *y_host,
                    int M, int N, int K) {
  return guarded([&] {
    enter(s);
    STB_REQUIRE(M >= 0 && N >= 0 && K >= 0, "Linear dimensions must be nonnegative");
    const uint64_t xb = (uint64_t)M * K * 4, yb = (uint64_t)M * N * 4;
    const uint64_t xr = (xb + 255) & ~255ull;
    if (xr + yb <= (64ull << 20)) {
      // Small requests (every decode-sized call) reuse one grow-only device buffer, charged to the
      // session budget like any allocation: no allocation, free or extra synchronisation per call.
      if (s->io_bytes < xr + yb) {
        if (s->io_buf) session_free(s, s->io_buf);
        s->io_buf = 0;
        s->io_bytes = 0;
        s->io_buf = session_alloc(s, xr + yb);
        s->io_bytes = xr + yb;
      }
      upload(s, x_host, xb, s->io_buf);
      linear(s, s->io_buf, K, w, w_dtype, bias, s->io_buf + xr, N, M, N, K);
      download(s, s->io_buf + xr, y_host, yb);
      return;
    }
    uint64_t dx = 0, dy = 0;
    try {
      dx = session_alloc(s, xb);
      dy = session_alloc(s, yb);
      upload(s, x_host, xb, dx);
      linear(s, dx, K, w, w_dtype, bias, dy, N, M, N, K);
      download(s, dy, y_host, yb);
    } catch (...) {
      if (dy) session_free(s, dy);
      if (dx) session_free(s, dx);
      throw;
    }
    session_free(s, dy);
    session_free(s, dx);
  });
}

}  // extern "C"
