// FloatBackend operator set (core/src/main/scala/scalatorch/FloatBackend.scala:7-31) on the B200.
//
// These are the per-op entry points the reference's generic BackendLlama drives
// (models/src/main/scala/scalatorch/models/BackendLlama.scala:41-111): embedding, transpose, add,
// multiply, scale, sum, expandScalar, silu, rmsNorm, rope, causalAttention and the attention
// cache's append.  Each is one kernel on the session stream with the arithmetic of the reference's
// CPU backend (cpu/src/main/scala/scalatorch/cpu/CpuFloatBackend.scala, CpuAttention.scala):
// Float32 elementwise ops, SiLU / RMSNorm / RoPE / attention in double, rounded once to Float32.
// They are the compatibility path (a model whose layers carry adapters, or any caller of the
// FloatBackend trait); the fused Llama runtime (llama.cu) is the fast path for whole-model decode.
//
// All of them are HBM-bound streaming kernels (attention: latency-bound per query row): grids are
// multiples of the SM count, loads and stores are coalesced, and 16-byte vector accesses are used
// where the buffers allow them.
#include <cmath>
#include <mutex>
#include <vector>

#include "gemv.cuh"

using namespace stb;

namespace {

constexpr int OP_THREADS = 256;

int sms(int device) {
  static int cached[64] = {};
  if (device >= 0 && device < 64 && cached[device]) return cached[device];
  int n = 0;
  STB_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device));
  if (device >= 0 && device < 64) cached[device] = n;
  return n;
}

// Grid of a grid-stride elementwise kernel over `units` work items: at most 8 blocks per SM.
unsigned ew_grid(stb_session *s, uint64_t units) {
  const uint64_t want = (units + OP_THREADS - 1) / OP_THREADS;
  const uint64_t cap = (uint64_t)sms(s->device) * 8;
  return (unsigned)std::max<uint64_t>(1, std::min(want, cap));
}

__device__ __forceinline__ double block_max_double(double v, double *scratch) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, off));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    double m = scratch[0];
    for (int i = 1; i < (int)(blockDim.x >> 5); i++) m = fmax(m, scratch[i]);
    scratch[0] = m;
  }
  __syncthreads();
  const double m = scratch[0];
  __syncthreads();
  return m;
}

bool aligned16(uint64_t p) { return p % 16 == 0; }

// ---- elementwise (CpuFloatBackend.add / multiply / scale: one Float32 operation per element)

template <int OP>  // 0: a + b, 1: a * b
__device__ __forceinline__ float binop(float a, float b) {
  return OP == 0 ? __fadd_rn(a, b) : __fmul_rn(a, b);
}

// vec: all three buffers 16-byte aligned; the first n / 4 * 4 elements move as float4, the rest
// one by one.
template <int OP>
__global__ void binary_kernel(const float *a, const float *b, float *y, uint64_t n, bool vec) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  const uint64_t g = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  uint64_t done = 0;
  if (vec) {
    const uint64_t n4 = n / 4;
    for (uint64_t j = g; j < n4; j += stride) {
      const float4 u = reinterpret_cast<const float4 *>(a)[j], v = reinterpret_cast<const float4 *>(b)[j];
      reinterpret_cast<float4 *>(y)[j] =
          make_float4(binop<OP>(u.x, v.x), binop<OP>(u.y, v.y), binop<OP>(u.z, v.z), binop<OP>(u.w, v.w));
    }
    done = n4 * 4;
  }
  for (uint64_t i = done + g; i < n; i += stride) y[i] = binop<OP>(a[i], b[i]);
}

__global__ void scale_kernel(const float *x, float *y, uint64_t n, float s) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    y[i] = __fmul_rn(x[i], s);
}

// CpuFloatBackend.silu (CpuFloatBackend.scala:70-77): double sigmoid, one rounding.
__global__ void silu_kernel(const float *x, float *y, uint64_t n) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    y[i] = silu_ref(x[i]);
}

__global__ void expand_kernel(const float *x, float *y, uint64_t n) {
  const float v = *x;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    y[i] = v;
}

// ---- sum (CpuFloatBackend.sum: a Double accumulation rounded once to Float32)

// Block b sums elements [b * chunk, (b + 1) * chunk) in double; a fixed tree, so the result is
// deterministic for a given element count.
__global__ void sum_partial_kernel(const float *x, uint64_t n, uint64_t chunk, double *part) {
  __shared__ double red[OP_THREADS / 32];
  const uint64_t b0 = blockIdx.x * chunk, b1 = min(n, b0 + chunk);
  double acc = 0.0;
  for (uint64_t i = b0 + threadIdx.x; i < b1; i += blockDim.x) acc = __dadd_rn(acc, (double)x[i]);
  acc = block_sum_double(acc, red);
  if (threadIdx.x == 0) part[blockIdx.x] = acc;
}

__global__ void sum_final_kernel(const double *part, int parts, float *y) {
  __shared__ double red[OP_THREADS / 32];
  double acc = 0.0;
  for (int i = threadIdx.x; i < parts; i += blockDim.x) acc = __dadd_rn(acc, part[i]);
  acc = block_sum_double(acc, red);
  if (threadIdx.x == 0) *y = __double2float_rn(acc);
}

// ---- rmsNorm over the last axis (CpuFloatBackend.rmsNorm, CpuFloatBackend.scala:78-93)

__global__ void rmsnorm_kernel(const float *x, const float *w, float *y, int width, double eps) {
  __shared__ double red[OP_THREADS / 32];
  const float *xr = x + (size_t)blockIdx.x * width;
  double sq = 0.0;
  for (int k = threadIdx.x; k < width; k += blockDim.x) {
    const double v = (double)xr[k];
    sq = __dadd_rn(sq, __dmul_rn(v, v));
  }
  const double total = block_sum_double(sq, red);
  const double inv = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(total, (double)width), eps)));
  for (int k = threadIdx.x; k < width; k += blockDim.x)
    y[(size_t)blockIdx.x * width + k] = __double2float_rn(__dmul_rn(__dmul_rn((double)xr[k], inv), (double)w[k]));
}

// ---- rope on (batch, heads, tokens, width) (CpuAttention.rope, CpuAttention.scala:6-18): the pair
// (d, d + width/2) of each row rotated by the host-computed (cos, sin) of its token, in double.
__global__ void rope_kernel(const float *x, float *y, const double2 *cs, uint64_t pairs, int tokens, int width) {
  const int half = width / 2;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < pairs;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t row = i / half;
    const int d = (int)(i % half);
    const double2 c = cs[(size_t)(row % tokens) * half + d];
    const double a = (double)x[row * width + d], b = (double)x[row * width + half + d];
    y[row * width + d] = __double2float_rn(__dsub_rn(__dmul_rn(a, c.x), __dmul_rn(b, c.y)));
    y[row * width + half + d] = __double2float_rn(__dadd_rn(__dmul_rn(b, c.x), __dmul_rn(a, c.y)));
  }
}

// ---- transpose of two axes of a packed tensor (rank <= 8): a copy, as CudaSession.transpose
constexpr int MAX_RANK = 8;
struct TransposeDims {
  int rank;
  int64_t out_dims[MAX_RANK];
  int64_t in_strides[MAX_RANK];  // input stride of each OUTPUT axis
};

__global__ void transpose_kernel(const float *x, float *y, uint64_t n, TransposeDims t) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    uint64_t rem = i, src = 0;
    for (int a = t.rank - 1; a >= 0; a--) {
      const uint64_t c = rem % (uint64_t)t.out_dims[a];
      rem /= (uint64_t)t.out_dims[a];
      src += c * (uint64_t)t.in_strides[a];
    }
    y[i] = x[src];
  }
}

// ---- embedding: rows of a Float32 / BF16 / F16 table (half rows widened exactly)
__global__ void embedding_kernel(const void *table, int dtype, const int64_t *ids, uint64_t count, int width,
                                 float *y) {
  const uint64_t n = count * (uint64_t)width;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t r = i / width, c = i % width;
    const uint64_t src = (uint64_t)ids[r] * width + c;
    float v;
    if (dtype == STB_F32) v = ((const float *)table)[src];
    else if (dtype == STB_BF16) v = widen1<__nv_bfloat16>(((const uint16_t *)table)[src]);
    else v = widen1<__half>(((const uint16_t *)table)[src]);
    y[i] = v;
  }
}

// ---- attention cache append: src (batch, heads, tokens, width) -> cache (batch, heads, capacity,
// width) at token `position` (CudaSession attentionCache's cache_append, CudaSession.scala:414-419)
__global__ void cache_append_kernel(const float *src, float *cache, uint64_t n, int heads, int tokens, int width,
                                    int capacity, int position) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t d = i % width, row = i / width;  // row = (b * heads + h) * tokens + t
    const uint64_t t = row % tokens, bh = row / tokens;
    cache[(bh * capacity + position + t) * width + d] = src[i];
  }
}

// ---- causal grouped-query attention (CpuAttention.causal, CpuAttention.scala:20-50), double
// throughout: one block per query row (b, h, t); scores of the visible keys j < min(keys, start +
// t + 1) in shared memory, softmax with the row maximum, weighted sum per output column with the
// keys in order.  q (batch, heads, tokens, width) packed; k / v (batch, kv_heads, key_stride,
// width / value_width), of which the first `keys` tokens are valid.
__global__ void __launch_bounds__(OP_THREADS) attention_op_kernel(const float *q, const float *k, const float *v,
                                                                  float *y, int heads, int tokens, int width,
                                                                  int kv_heads, int keys, int key_stride, int vw,
                                                                  int start) {
  extern __shared__ double p[];
  __shared__ double red[OP_THREADS / 32];
  const int row = blockIdx.x;  // (b * heads + h) * tokens + t
  const int t = row % tokens, bh = row / tokens, h = bh % heads, b = bh / heads;
  const int kvh = h / (heads / kv_heads);
  const size_t kv0 = ((size_t)b * kv_heads + kvh) * key_stride;
  const int visible = (int)min((long long)keys, (long long)start + t + 1);
  const float *qr = q + (size_t)row * width;
  const double scale = __ddiv_rn(1.0, __dsqrt_rn((double)width));
  double mx = -INFINITY;
  for (int j = threadIdx.x; j < visible; j += blockDim.x) {
    const float *kr = k + (kv0 + j) * width;
    double dot = 0.0;
    for (int d = 0; d < width; d++) dot = __dadd_rn(dot, __dmul_rn((double)qr[d], (double)kr[d]));
    const double sc = __dmul_rn(dot, scale);
    p[j] = sc;
    mx = fmax(mx, sc);
  }
  mx = block_max_double(mx, red);
  double den = 0.0;
  for (int j = threadIdx.x; j < visible; j += blockDim.x) {
    const double e = exp(__dsub_rn(p[j], mx));
    p[j] = e;
    den = __dadd_rn(den, e);
  }
  den = block_sum_double(den, red);
  for (int j = threadIdx.x; j < visible; j += blockDim.x) p[j] = __ddiv_rn(p[j], den);
  __syncthreads();
  for (int d = threadIdx.x; d < vw; d += blockDim.x) {
    double acc = 0.0;
    for (int j = 0; j < visible; j++) acc = __dadd_rn(acc, __dmul_rn(p[j], (double)v[(kv0 + j) * vw + d]));
    y[(size_t)row * vw + d] = __double2float_rn(acc);
  }
}

// Largest key count whose double scores fit the per-block shared memory this kernel may use.
constexpr int ATTN_MAX_KEYS = 24576;  // 192 KB

void require_f32(uint64_t p, const char *what) {
  STB_REQUIRE(p != 0 && p % 4 == 0, std::string(what) + ": null or misaligned Float32 buffer");
}

}  // namespace

namespace stb {
// (cos, sin) of RotaryCoefficients.values (core/src/main/scala/scalatorch/AttentionLayout.scala:23-34)
// for `tokens` positions from `start`: cs[t * (width/2) + d] = (cos a, sin a), a = (start + t) *
// theta^(-2d/width), computed in double on the host as the reference does.
std::vector<double> rotary_coefficients(int tokens, int width, int start, double theta) {
  const int half = width / 2;
  std::vector<double> cs((size_t)tokens * half * 2);
  for (int t = 0; t < tokens; t++)
    for (int d = 0; d < half; d++) {
      const double angle = (double)((long long)start + t) * std::pow(theta, -2.0 * d / width);
      if (!std::isfinite(angle)) throw Error(STB_ERR_INVALID, "rotary angle overflow");
      cs[((size_t)t * half + d) * 2] = std::cos(angle);
      cs[((size_t)t * half + d) * 2 + 1] = std::sin(angle);
    }
  return cs;
}
}  // namespace stb

extern "C" {

int stb_op_add(stb_session *s, uint64_t a, uint64_t b, uint64_t y, uint64_t count) {
  return guarded([&] {
    enter(s);
    if (!count) return;
    require_f32(a, "add");
    require_f32(b, "add");
    require_f32(y, "add");
    const bool vec = aligned16(a) && aligned16(b) && aligned16(y);
    launch_kernel(binary_kernel<0>, dim3(ew_grid(s, vec ? count / 4 : count)), dim3(OP_THREADS), 0, s->stream, false,
                  (const float *)a, (const float *)b, (float *)y, count, vec);
    count_launch(s);
  });
}

int stb_op_multiply(stb_session *s, uint64_t a, uint64_t b, uint64_t y, uint64_t count) {
  return guarded([&] {
    enter(s);
    if (!count) return;
    require_f32(a, "multiply");
    require_f32(b, "multiply");
    require_f32(y, "multiply");
    const bool vec = aligned16(a) && aligned16(b) && aligned16(y);
    launch_kernel(binary_kernel<1>, dim3(ew_grid(s, vec ? count / 4 : count)), dim3(OP_THREADS), 0, s->stream, false,
                  (const float *)a, (const float *)b, (float *)y, count, vec);
    count_launch(s);
  });
}

int stb_op_scale(stb_session *s, uint64_t x, uint64_t y, uint64_t count, float scalar) {
  return guarded([&] {
    enter(s);
    if (!count) return;
    require_f32(x, "scale");
    require_f32(y, "scale");
    launch_kernel(scale_kernel, dim3(ew_grid(s, count)), dim3(OP_THREADS), 0, s->stream, false, (const float *)x,
                  (float *)y, count, scalar);
    count_launch(s);
  });
}

int stb_op_silu(stb_session *s, uint64_t x, uint64_t y, uint64_t count) {
  return guarded([&] {
    enter(s);
    if (!count) return;
    require_f32(x, "silu");
    require_f32(y, "silu");
    launch_kernel(silu_kernel, dim3(ew_grid(s, count)), dim3(OP_THREADS), 0, s->stream, false, (const float *)x,
                  (float *)y, count);
    count_launch(s);
  });
}

int stb_op_expand_scalar(stb_session *s, uint64_t x, uint64_t y, uint64_t count) {
  return guarded([&] {
    enter(s);
    if (!count) return;
    require_f32(x, "expandScalar");
    require_f32(y, "expandScalar");
    launch_kernel(expand_kernel, dim3(ew_grid(s, count)), dim3(OP_THREADS), 0, s->stream, false, (const float *)x,
                  (float *)y, count);
    count_launch(s);
  });
}

int stb_op_sum(stb_session *s, uint64_t x, uint64_t count, uint64_t y) {
  return guarded([&] {
    enter(s);
    require_f32(y, "sum");
    if (!count) {
      fill_value(s, y, STB_F32, 1, 0.0f);
      return;
    }
    require_f32(x, "sum");
    const int parts = (int)std::min<uint64_t>((count + 4095) / 4096, (uint64_t)sms(s->device) * 4);
    const uint64_t chunk = (count + parts - 1) / parts;
    const uint64_t part = session_scratch(s, (uint64_t)parts * sizeof(double));
    launch_kernel(sum_partial_kernel, dim3(parts), dim3(OP_THREADS), 0, s->stream, false, (const float *)x, count,
                  chunk, (double *)part);
    launch_kernel(sum_final_kernel, dim3(1), dim3(OP_THREADS), 0, s->stream, false, (const double *)part, parts,
                  (float *)y);
    count_launch(s, 2);
  });
}

int stb_op_rmsnorm(stb_session *s, uint64_t x, uint64_t w, uint64_t y, uint64_t rows, int width, double eps) {
  return guarded([&] {
    enter(s);
    STB_REQUIRE(std::isfinite(eps) && eps > 0, "invalid RMSNorm epsilon");
    STB_REQUIRE(width > 0 && rows <= 0x7fffffffu, "invalid RMSNorm shapes");
    if (!rows) return;
    require_f32(x, "rmsNorm");
    require_f32(w, "rmsNorm");
    require_f32(y, "rmsNorm");
    launch_kernel(rmsnorm_kernel, dim3((unsigned)rows), dim3(OP_THREADS), 0, s->stream, false, (const float *)x,
                  (const float *)w, (float *)y, width, eps);
    count_launch(s);
  });
}

int stb_op_rope(stb_session *s, uint64_t x, uint64_t y, int batch, int heads, int tokens, int width, int start,
                double theta) {
  return guarded([&] {
    enter(s);
    STB_REQUIRE(batch >= 0 && heads >= 0 && tokens >= 0 && width > 0 && width % 2 == 0,
                "RoPE requires rank 4 and positive even width");
    STB_REQUIRE(start >= 0 && std::isfinite(theta) && theta > 0, "invalid rotary position or theta");
    const uint64_t n = (uint64_t)batch * heads * tokens * width;
    if (!n) return;
    require_f32(x, "rope");
    require_f32(y, "rope");
    const std::vector<double> cs = rotary_coefficients(tokens, width, start, theta);
    const uint64_t table = session_scratch(s, cs.size() * sizeof(double));
    upload(s, cs.data(), cs.size() * sizeof(double), table);
    launch_kernel(rope_kernel, dim3(ew_grid(s, n / 2)), dim3(OP_THREADS), 0, s->stream, false, (const float *)x,
                  (float *)y, (const double2 *)table, n / 2, tokens, width);
    count_launch(s);
  });
}

int stb_op_transpose(stb_session *s, uint64_t x, uint64_t y, int rank, const int64_t *dims, int dim0, int dim1) {
  return guarded([&] {
    enter(s);
    STB_REQUIRE(rank >= 1 && rank <= MAX_RANK && dims, "transpose supports ranks 1 to 8");
    STB_REQUIRE(dim0 >= 0 && dim0 < rank && dim1 >= 0 && dim1 < rank, "transpose dimension out of range");
    uint64_t n = 1;
    for (int a = 0; a < rank; a++) {
      STB_REQUIRE(dims[a] >= 0, "negative dimension");
      n *= (uint64_t)dims[a];
    }
    if (!n) return;
    require_f32(x, "transpose");
    require_f32(y, "transpose");
    TransposeDims t{};
    t.rank = rank;
    int64_t stride[MAX_RANK];
    stride[rank - 1] = 1;
    for (int a = rank - 2; a >= 0; a--) stride[a] = stride[a + 1] * dims[a + 1];
    for (int a = 0; a < rank; a++) {
      const int src = a == dim0 ? dim1 : (a == dim1 ? dim0 : a);
      t.out_dims[a] = dims[src];
      t.in_strides[a] = stride[src];
    }
    launch_kernel(transpose_kernel, dim3(ew_grid(s, n)), dim3(OP_THREADS), 0, s->stream, false, (const float *)x,
                  (float *)y, n, t);
    count_launch(s);
  });
}

int stb_op_embedding(stb_session *s, uint64_t table, int dtype, int64_t rows, int width, const int64_t *ids,
                     uint64_t count, uint64_t y) {
  return guarded([&] {
    enter(s);
    STB_REQUIRE(rows >= 0 && width > 0, "embedding requires a matrix with positive width");
    STB_REQUIRE(dtype == STB_F32 || dtype == STB_BF16 || dtype == STB_F16, "embedding table type");
    if (!count) return;
    STB_REQUIRE(ids, "null ids");
    for (uint64_t i = 0; i < count; i++) STB_REQUIRE(ids[i] >= 0 && ids[i] < rows, "embedding token ID out of bounds");
    STB_REQUIRE(table && y && y % 4 == 0, "null or misaligned buffer");
    const uint64_t dev_ids = session_scratch(s, count * 8);
    upload(s, ids, count * 8, dev_ids);
    launch_kernel(embedding_kernel, dim3(ew_grid(s, count * (uint64_t)width)), dim3(OP_THREADS), 0, s->stream, false,
                  (const void *)table, dtype, (const int64_t *)dev_ids, count, width, (float *)y);
    count_launch(s);
  });
}

int stb_op_cache_append(stb_session *s, uint64_t src, uint64_t cache, int batch, int heads, int tokens, int width,
                        int capacity, int position) {
  return guarded([&] {
    enter(s);
    STB_REQUIRE(batch > 0 && heads > 0 && width > 0 && capacity > 0 && tokens >= 0, "invalid cache dimensions");
    STB_REQUIRE(position >= 0 && (long long)position + tokens <= capacity, "cache append gap or capacity exceeded");
    const uint64_t n = (uint64_t)batch * heads * tokens * width;
    if (!n) return;
    require_f32(src, "cache append");
    require_f32(cache, "cache append");
    launch_kernel(cache_append_kernel, dim3(ew_grid(s, n)), dim3(OP_THREADS), 0, s->stream, false,
                  (const float *)src, (float *)cache, n, heads, tokens, width, capacity, position);
    count_launch(s);
  });
}

int stb_op_causal_attention(stb_session *s, uint64_t q, uint64_t k, uint64_t v, uint64_t y, int batch, int heads,
                            int tokens, int width, int kv_heads, int keys, int key_stride, int value_width,
                            int start) {
  return guarded([&] {
    enter(s);
    STB_REQUIRE(batch >= 0 && tokens >= 0 && start >= 0, "invalid attention offset or workspace limit");
    STB_REQUIRE(heads > 0 && kv_heads > 0 && heads % kv_heads == 0, "invalid grouped attention heads");
    STB_REQUIRE(width > 0 && value_width > 0 && keys >= 0 && key_stride >= keys, "attention width/token mismatch");
    const uint64_t rows = (uint64_t)batch * heads * tokens;
    if (!rows) return;
    STB_REQUIRE(keys > 0, "nonempty queries require keys");
    STB_REQUIRE(rows <= 0x7fffffffu, "attention output exceeds Int indexing");
    if (keys > ATTN_MAX_KEYS)
      throw Error(STB_ERR_UNSUPPORTED, "causal attention over more than 24576 keys per query row");
    require_f32(q, "attention");
    require_f32(k, "attention");
    require_f32(v, "attention");
    require_f32(y, "attention");
    const size_t smem = (size_t)keys * sizeof(double);
    {
      static std::mutex mu;
      static bool configured[64] = {};
      std::lock_guard<std::mutex> lock(mu);
      if (s->device < 0 || s->device >= 64 || !configured[s->device]) {
        STB_CUDA(cudaFuncSetAttribute(attention_op_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      ATTN_MAX_KEYS * (int)sizeof(double)));
        if (s->device >= 0 && s->device < 64) configured[s->device] = true;
      }
    }
    launch_kernel(attention_op_kernel, dim3((unsigned)rows), dim3(OP_THREADS), smem, s->stream, false,
                  (const float *)q, (const float *)k, (const float *)v, (float *)y, heads, tokens, width, kv_heads, keys,
                  key_stride, value_width, start);
    count_launch(s);
  });
}

}  // extern "C"
