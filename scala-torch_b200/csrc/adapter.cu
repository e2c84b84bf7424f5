// Low-rank adapter terms of nn.Linear.apply (nn/src/main/scala/scalatorch/nn/Linear.scala:11-17):
// after the base product x.W^T (decode GEMV / skinny form), each adapter adds
// ((x.A^T).B^T) * scale (* multiplier for LinearAdapterScope entries), then the bias is added --
// the reference's operation order, every step rounded to Float32.  The adapters' rank is small
// (LoRA ranks 4-64), so the two thin products are two small kernels per term: the down
// projection t = x.A^T (one warp per (row, rank) output, FMA over K, xor reduction) and the up
// projection fused with the scale / multiplier / accumulate / bias epilogue (one thread per output,
// FMA over the rank in order).
#include <cmath>

#include "gemv.cuh"

namespace stb {

void linear(stb_session *s, uint64_t x, int ldx, uint64_t w, int w_dtype, uint64_t bias, uint64_t y, int ldy,
            int M, int N, int K);

namespace {

__global__ void adapter_down_kernel(const float *x, const float *a, float *t, int M, int r, int K) {
  const long warp = (blockIdx.x * (long)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= (long)M * r) return;
  const int m = (int)(warp / r), j = (int)(warp % r);
  const float *xr = x + (size_t)m * K, *ar = a + (size_t)j * K;
  float acc = 0.0f;
  for (int k = lane; k < K; k += 32) acc = fmaf(xr[k], ar[k], acc);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) t[(size_t)m * r + j] = acc;
}

__global__ void adapter_up_kernel(const float *t, const float *b, float *y, int M, int N, int r, float scale,
                                  int scoped, float multiplier, const float *bias) {
  const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
  if (i >= (long)M * N) return;
  const int m = (int)(i / N), n = (int)(i % N);
  const float *tr = t + (size_t)m * r, *br = b + (size_t)n * r;
  float u = 0.0f;
  for (int j = 0; j < r; j++) u = fmaf(tr[j], br[j], u);
  float v = u * scale;
  if (scoped) v = v * multiplier;
  float sum = y[i] + v;
  if (bias) sum = sum + bias[n];
  y[i] = sum;
}

}  // namespace
}  // namespace stb

using namespace stb;

extern "C" int stb_linear_adapted(stb_session *s, uint64_t x, uint64_t w, int w_dtype, uint64_t bias,
                                  const stb_adapter *adapters, int count, uint64_t y, int M, int N, int K) {
  return guarded([&] {
    enter(s);
    STB_REQUIRE(count >= 0 && (count == 0 || adapters), "adapter list is null");
    int max_rank = 0;
    for (int i = 0; i < count; i++) {
      const stb_adapter &ad = adapters[i];
      STB_REQUIRE(ad.a != 0 && ad.b != 0 && ad.rank > 0, "adapter factors must be non-null with rank > 0");
      STB_REQUIRE(std::isfinite(ad.scale) && ad.scale > 0.0f, "invalid adapter scale");
      STB_REQUIRE(std::isfinite(ad.multiplier), "adapter multiplier must be finite");
      STB_REQUIRE(ad.scoped == 1 || (ad.scoped == 0 && i == 0), "only the first term may be the Linear's own adapter");
      max_rank = std::max(max_rank, ad.rank);
    }
    if (count == 0 || M == 0 || N == 0) {
      linear(s, x, K, w, w_dtype, bias, y, N, M, N, K);
      return;
    }
    STB_REQUIRE(x != 0 || K == 0, "Linear input is null");
    linear(s, x, K, w, w_dtype, 0, y, N, M, N, K);
    float *t = (float *)session_scratch(s, (uint64_t)M * max_rank * sizeof(float));
    for (int i = 0; i < count; i++) {
      const stb_adapter &ad = adapters[i];
      const long warps = (long)M * ad.rank;
      adapter_down_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, s->stream>>>(
          (const float *)x, (const float *)ad.a, t, M, ad.rank, K);
      const long outs = (long)M * N;
      adapter_up_kernel<<<(unsigned)((outs + 255) / 256), 256, 0, s->stream>>>(
          t, (const float *)ad.b, (float *)y, M, N, ad.rank, ad.scale, ad.scoped, ad.multiplier,
          i == count - 1 ? (const float *)bias : nullptr);
      check_launch("adapter");
      count_launch(s, 2);
    }
  });
}
