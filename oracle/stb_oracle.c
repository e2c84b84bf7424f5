/*
 * stb_oracle.c -- CPU restatement of scala-torch's Float32 Linear / Llama decode arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY (the checker and the timed CPU baseline); see stb_oracle.h.
 * Build with -ffp-contract=off: the JVM never contracts a multiply and an add into an FMA, so
 * every product and every sum below is rounded separately, as the reference's are.
 */
#include "stb_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef __SSE2__
#include <emmintrin.h>
#endif
#ifdef _OPENMP
#include <omp.h>
#endif

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

int oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* ---------------------------------------------------------------- element conversions */

/* SafeTensors.scala:72: intBitsToFloat((bits & 0xffff) << 16) -- exact. */
float oracle_bf16_to_f32(uint16_t bits) { return u2f(((uint32_t)bits) << 16); }

/* SafeTensors.scala:71: java.lang.Float.float16ToFloat -- exact, NaN significand kept. */
float oracle_f16_to_f32(uint16_t h) {
  uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t man = h & 0x3ffu;
  if (exp == 0) {
    float mag = (float)man * 5.9604644775390625e-8f; /* man * 2^-24, exact */
    return u2f(f2u(mag) | sign);
  }
  if (exp == 31) return u2f(sign | 0x7f800000u | (man << 13));
  return u2f(sign | ((exp + 112u) << 23) | (man << 13));
}

/* SafeTensorsWriter.scala:58-61: NaN keeps its top bits and is quieted with 0x40; everything
 * else rounds to nearest even by adding 0x7fff plus the kept LSB. */
uint16_t oracle_f32_to_bf16(float value) {
  uint32_t bits = f2u(value);
  if ((bits & 0x7f800000u) == 0x7f800000u && (bits & 0x007fffffu) != 0)
    return (uint16_t)((bits >> 16) | 0x40u);
  return (uint16_t)((bits + 0x7fffu + ((bits >> 16) & 1u)) >> 16);
}

/* F32 -> F16 round to nearest even with overflow to infinity (IEEE 754 binary16). */
uint16_t oracle_f32_to_f16(float value) {
  uint32_t bits = f2u(value);
  uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
  uint32_t a = bits & 0x7fffffffu;
  if (a > 0x7f800000u) return (uint16_t)(sign | 0x7e00u | ((a >> 13) & 0x1ffu));
  if (a >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* >= 65520 rounds to infinity */
  if (a >= 0x38800000u) {                                   /* normal binary16 */
    a += 0xfffu + ((a >> 13) & 1u);
    return (uint16_t)(sign | ((a - 0x38000000u) >> 13));
  }
  if (a < 0x33000000u) return sign; /* below half the smallest subnormal */
  {
    int shift = 126 - (int)(a >> 23);
    uint32_t m = (a & 0x7fffffu) | 0x800000u;
    uint32_t q = m >> shift, rem = m & ((1u << shift) - 1u), halfway = 1u << (shift - 1);
    if (rem > halfway || (rem == halfway && (q & 1u))) q++;
    return (uint16_t)(sign | q);
  }
}

void oracle_widen(const void *src, int dtype, float *dst, size_t count) {
  size_t i;
  if (dtype == ORACLE_F32) { memcpy(dst, src, count * 4); return; }
  const uint16_t *h = (const uint16_t *)src;
  if (dtype == ORACLE_BF16)
    for (i = 0; i < count; i++) dst[i] = oracle_bf16_to_f32(h[i]);
  else
    for (i = 0; i < count; i++) dst[i] = oracle_f16_to_f32(h[i]);
}

void oracle_round_bf16(const float *src, uint16_t *dst, size_t count) {
  for (size_t i = 0; i < count; i++) dst[i] = oracle_f32_to_bf16(src[i]);
}
void oracle_round_f16(const float *src, uint16_t *dst, size_t count) {
  for (size_t i = 0; i < count; i++) dst[i] = oracle_f32_to_f16(src[i]);
}

/* ---------------------------------------------------------------- GEMM orders */

/* One output of the transposed-right product in numscala's documented order
 * (gemm.ptx:167-193): s[k & 3] += x[k] * w[k] over complete groups of four, the incomplete
 * tail into s0, then (s0 + s1) + (s2 + s3).  Each step rounds its multiply and its add. */
static float dot_numscala(const float *x, const float *w, int K) {
  int K4 = K & ~3, k;
  float s0, s1, s2, s3;
#ifdef __SSE2__
  __m128 acc = _mm_setzero_ps();
  for (k = 0; k < K4; k += 4)
    acc = _mm_add_ps(acc, _mm_mul_ps(_mm_loadu_ps(x + k), _mm_loadu_ps(w + k)));
  float s[4];
  _mm_storeu_ps(s, acc);
  s0 = s[0]; s1 = s[1]; s2 = s[2]; s3 = s[3];
#else
  s0 = s1 = s2 = s3 = 0.0f;
  for (k = 0; k < K4; k += 4) {
    float p0 = x[k] * w[k], p1 = x[k + 1] * w[k + 1], p2 = x[k + 2] * w[k + 2], p3 = x[k + 3] * w[k + 3];
    s0 = s0 + p0; s1 = s1 + p1; s2 = s2 + p2; s3 = s3 + p3;
  }
#endif
  for (k = K4; k < K; k++) {
    float p = x[k] * w[k];
    s0 = s0 + p;
  }
  float a = s0 + s1;
  float b = s2 + s3;
  return a + b;
}

void oracle_matmul_tr(const float *x, const float *w, float *y, int M, int N, int K, int threads) {
  long n;
  if (threads < 1) threads = 1;
#pragma omp parallel for schedule(static) num_threads(threads) if (threads > 1)
  for (n = 0; n < N; n++) {
    const float *wr = w + (size_t)n * K;
    for (int m = 0; m < M; m++) y[(size_t)m * N + n] = dot_numscala(x + (size_t)m * K, wr, K);
  }
}

/* Ops.scala:61-81: acc += a(i,p) * b(p,j), one Float32 accumulator, separately rounded. */
void oracle_matmul_seq(const float *a, const float *b, float *c, int M, int N, int K) {
  for (int i = 0; i < M; i++)
    for (int j = 0; j < N; j++) {
      float acc = 0.0f;
      for (int p = 0; p < K; p++) {
        float prod = a[(size_t)i * K + p] * b[(size_t)p * N + j];
        acc = acc + prod;
      }
      c[(size_t)i * N + j] = acc;
    }
}

void oracle_linear(const float *x, const void *w, int w_dtype, const float *bias, float *y,
                   int M, int N, int K, int order, int threads) {
  size_t count = (size_t)N * K;
  float *wf = (float *)malloc(count ? count * 4 : 4);
  oracle_widen(w, w_dtype, wf, count);
  if (order == ORACLE_ORDER_SEQUENTIAL) {
    /* Ops.matmul(x, W^T): b(p, j) = W[j, p]; pack W^T to reuse the logical-index loop. */
    float *wt = (float *)malloc(count ? count * 4 : 4);
    for (int n = 0; n < N; n++)
      for (int k = 0; k < K; k++) wt[(size_t)k * N + n] = wf[(size_t)n * K + k];
    oracle_matmul_seq(x, wt, y, M, N, K);
    free(wt);
  } else {
    oracle_matmul_tr(x, wf, y, M, N, K, threads);
  }
  free(wf);
  if (bias) /* Linear.scala:17: result + bias (Ops.add broadcast) */
    for (int m = 0; m < M; m++)
      for (int n = 0; n < N; n++) y[(size_t)m * N + n] = y[(size_t)m * N + n] + bias[n];
}

/* nn.Linear.apply with its low-rank adapter and the LinearAdapterScope adapters
 * (nn/src/main/scala/scalatorch/nn/Linear.scala:11-17; LowRankAdapter.scala:12-14):
 *   base = x.W^T;  attached (scoped == 0, first only): sum = base + ((x.A^T).B^T) * scale;
 *   each scoped entry: sum = sum + (((x.A^T).B^T) * scale) * multiplier;  then + bias.
 * A is [rank, K], B is [N, rank] (Float32 parameters); scale is LowRankAdapter.scale, (alpha / rank)
 * rounded to Float32.  Every product in numscala's transposed-right order, every elementwise
 * operation rounded to Float32 (Variable arithmetic). */
void oracle_linear_adapted(const float *x, const void *w, int w_dtype, const float *bias,
                           const float *const *a, const float *const *b, const int *rank,
                           const float *scale, const int *scoped, const float *multiplier, int count,
                           float *y, int M, int N, int K, int threads) {
  oracle_linear(x, w, w_dtype, NULL, y, M, N, K, ORACLE_ORDER_NUMSCALA, threads);
  for (int i = 0; i < count; i++) {
    int r = rank[i];
    float *t = (float *)malloc((size_t)M * r * 4 + 4);
    float *u = (float *)malloc((size_t)M * N * 4 + 4);
    oracle_matmul_tr(x, a[i], t, M, r, K, threads);   /* input.matmul(a.transpose(0, 1)) */
    oracle_matmul_tr(t, b[i], u, M, N, r, threads);   /* .matmul(b.transpose(0, 1)) */
    for (size_t e = 0; e < (size_t)M * N; e++) {
      float v = u[e] * scale[i];                       /* * scale */
      if (scoped[i]) v = v * multiplier[i];            /* adapter(input) * multiplier */
      y[e] = y[e] + v;
    }
    free(t);
    free(u);
  }
  if (bias)
    for (int m = 0; m < M; m++)
      for (int n = 0; n < N; n++) y[(size_t)m * N + n] = y[(size_t)m * N + n] + bias[n];
}

/* ---------------------------------------------------------------- decode-step ops */

void oracle_rmsnorm(const float *x, const float *w, float *y, int rows, int width, double eps) {
  for (int r = 0; r < rows; r++) {
    const float *xr = x + (size_t)r * width;
    double squares = 0.0;
    for (int j = 0; j < width; j++) squares += (double)xr[j] * xr[j];
    double inverse = 1.0 / sqrt(squares / width + eps);
    for (int j = 0; j < width; j++) y[(size_t)r * width + j] = (float)((double)xr[j] * inverse * w[j]);
  }
}

float oracle_silu(float x) {
  double v = x;
  double sigmoid;
  if (v >= 0) sigmoid = 1.0 / (1.0 + exp(-v));
  else { double e = exp(v); sigmoid = e / (1.0 + e); }
  return (float)(v == -INFINITY ? -0.0 : v * sigmoid);
}

void oracle_rope(const float *x, float *y, int batch, int heads, int tokens, int width, int start,
                 double theta) {
  int half = width / 2;
  long rows = (long)batch * heads * tokens;
  for (long row = 0; row < rows; row++) {
    int t = (int)(row % tokens);
    for (int d = 0; d < half; d++) {
      double angle = (double)((long)start + t) * pow(theta, -2.0 * d / width);
      double c = cos(angle), s = sin(angle);
      double a = x[row * width + d], b = x[row * width + half + d];
      y[row * width + d] = (float)(a * c - b * s);
      y[row * width + half + d] = (float)(b * c + a * s);
    }
  }
}

void oracle_causal_attention(const float *q, const float *k, const float *v, float *out,
                             int batch, int heads, int tokens, int width, int kv_heads,
                             int keys, int key_stride_tokens, int value_width, int start) {
  double *p = (double *)malloc((size_t)(keys > 0 ? keys : 1) * sizeof(double));
  double scale = 1.0 / sqrt((double)width);
  int group = heads / kv_heads;
  for (int b = 0; b < batch; b++)
    for (int h = 0; h < heads; h++)
      for (int t = 0; t < tokens; t++) {
        long row = ((long)b * heads + h) * tokens + t;
        long kv = ((long)b * kv_heads + h / group) * key_stride_tokens;
        long vis = (long)start + t + 1;
        int visible = (int)(vis < keys ? vis : keys);
        double maximum = -INFINITY;
        for (int j = 0; j < visible; j++) {
          double dot = 0.0;
          for (int d = 0; d < width; d++) dot += (double)q[row * width + d] * k[(kv + j) * width + d];
          p[j] = dot * scale;
          maximum = fmax(maximum, p[j]);
        }
        double denominator = 0.0;
        for (int j = 0; j < visible; j++) { p[j] = exp(p[j] - maximum); denominator += p[j]; }
        for (int j = 0; j < visible; j++) p[j] /= denominator;
        for (int d = 0; d < value_width; d++) {
          double sum = 0.0;
          for (int j = 0; j < visible; j++) sum += p[j] * v[(kv + j) * value_width + d];
          out[row * value_width + d] = (float)sum;
        }
      }
  free(p);
}

int64_t oracle_argmax(const float *logits, int64_t count) {
  int64_t best = 0;
  for (int64_t i = 1; i < count; i++)
    if (logits[i] > logits[best]) best = i;
  return best;
}

/* ---------------------------------------------------------------- counter-based RNG */

/* splitmix64 finaliser (Steele, Lea, Flood 2014; constants as published by S. Vigna). */
static inline uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
  return z ^ (z >> 31);
}

uint64_t oracle_rng_u64(uint64_t seed, uint64_t stream, uint64_t index) {
  uint64_t key = mix64(seed ^ (0x9e3779b97f4a7c15ULL * (stream + 1)));
  return mix64(key + 0x9e3779b97f4a7c15ULL * (index + 1));
}

/* Natural log for positive normal doubles: x = m * 2^e with m in (sqrt(1/2), sqrt(2)],
 * ln m = 2 atanh(t), t = (m-1)/(m+1), by the odd series sum t^(2i+1)/(2i+1) to i = 12
 * (|t| <= 0.1716, truncation < 1e-18).  Written with plain IEEE double operations only so a
 * device restatement with explicitly rounded intrinsics produces the same bits. */
double oracle_log(double x) {
  uint64_t b;
  memcpy(&b, &x, 8);
  int e = (int)((b >> 52) & 0x7ff) - 1023;
  b = (b & 0x000fffffffffffffULL) | 0x3ff0000000000000ULL;
  double m;
  memcpy(&m, &b, 8);
  if (m > 1.4142135623730951) { m = m * 0.5; e = e + 1; }
  double t = (m - 1.0) / (m + 1.0);
  double t2 = t * t;
  double p = 1.0 / 25.0;
  p = p * t2 + 1.0 / 23.0;
  p = p * t2 + 1.0 / 21.0;
  p = p * t2 + 1.0 / 19.0;
  p = p * t2 + 1.0 / 17.0;
  p = p * t2 + 1.0 / 15.0;
  p = p * t2 + 1.0 / 13.0;
  p = p * t2 + 1.0 / 11.0;
  p = p * t2 + 1.0 / 9.0;
  p = p * t2 + 1.0 / 7.0;
  p = p * t2 + 1.0 / 5.0;
  p = p * t2 + 1.0 / 3.0;
  p = p * t2 + 1.0;
  double tt = 2.0 * t;
  double lp = tt * p;
  double le = (double)e * 0x1.62e42fefa39efp-1; /* ln 2 rounded to double */
  return le + lp;
}

/* Marsaglia polar method: attempt j draws one 64-bit word keyed by (seed, stream, 64*index+j),
 * splits it into two uniforms in (-1,1) that are exact in double, rejects s >= 1. */
double oracle_rng_normal(uint64_t seed, uint64_t stream, uint64_t index) {
  for (uint64_t j = 0; j < 64; j++) {
    uint64_t r = oracle_rng_u64(seed, stream, index * 64 + j);
    double u = ((double)(r >> 32) + 0.5) * 0x1p-31 - 1.0;
    double v = ((double)(r & 0xffffffffULL) + 0.5) * 0x1p-31 - 1.0;
    double s = u * u + v * v;
    if (s >= 1.0 || s == 0.0) continue;
    double l = oracle_log(s);
    double q = -2.0 * l / s;
    return u * sqrt(q);
  }
  return 0.0;
}

void oracle_fill_normal_f32(float *dst, size_t count, uint64_t seed, uint64_t stream, double std,
                            int threads) {
  long i;
  if (threads < 1) threads = 1;
#pragma omp parallel for schedule(static) num_threads(threads) if (threads > 1)
  for (i = 0; i < (long)count; i++) dst[i] = (float)(std * oracle_rng_normal(seed, stream, (uint64_t)i));
}

void oracle_fill_normal_bf16(uint16_t *dst, size_t count, uint64_t seed, uint64_t stream,
                             double std, int threads) {
  long i;
  if (threads < 1) threads = 1;
#pragma omp parallel for schedule(static) num_threads(threads) if (threads > 1)
  for (i = 0; i < (long)count; i++)
    dst[i] = oracle_f32_to_bf16((float)(std * oracle_rng_normal(seed, stream, (uint64_t)i)));
}

/* ---------------------------------------------------------------- Llama decode */

struct oracle_llama_cache {
  int batch, capacity, layers, kv_heads, head_dim, used;
  float **keys, **values; /* per layer: (batch, kv_heads, capacity, head_dim) */
};

oracle_llama_cache *oracle_cache_create(const oracle_llama_config *c, int batch, int capacity) {
  oracle_llama_cache *cache = (oracle_llama_cache *)calloc(1, sizeof(*cache));
  int hd = c->hidden / c->heads;
  cache->batch = batch; cache->capacity = capacity; cache->layers = c->layers;
  cache->kv_heads = c->kv_heads; cache->head_dim = hd; cache->used = 0;
  cache->keys = (float **)calloc((size_t)c->layers, sizeof(float *));
  cache->values = (float **)calloc((size_t)c->layers, sizeof(float *));
  size_t per = (size_t)batch * c->kv_heads * capacity * hd;
  for (int l = 0; l < c->layers; l++) {
    cache->keys[l] = (float *)calloc(per, sizeof(float));
    cache->values[l] = (float *)calloc(per, sizeof(float));
  }
  return cache;
}

void oracle_cache_destroy(oracle_llama_cache *cache) {
  if (!cache) return;
  for (int l = 0; l < cache->layers; l++) { free(cache->keys[l]); free(cache->values[l]); }
  free(cache->keys); free(cache->values); free(cache);
}

int oracle_cache_position(const oracle_llama_cache *cache) { return cache->used; }

/* (rows, heads*hd) -> (batch, heads, tokens, hd): the reshape + transpose(1,2) of
 * LlamaAttention.heads (LlamaModel.scala:25-26). */
static void split_heads(const float *src, float *dst, int batch, int tokens, int heads, int hd) {
  for (int b = 0; b < batch; b++)
    for (int t = 0; t < tokens; t++)
      for (int h = 0; h < heads; h++)
        memcpy(dst + (((size_t)b * heads + h) * tokens + t) * hd,
               src + (((size_t)b * tokens + t) * heads + h) * hd, (size_t)hd * 4);
}
static void merge_heads(const float *src, float *dst, int batch, int tokens, int heads, int hd) {
  for (int b = 0; b < batch; b++)
    for (int t = 0; t < tokens; t++)
      for (int h = 0; h < heads; h++)
        memcpy(dst + (((size_t)b * tokens + t) * heads + h) * hd,
               src + (((size_t)b * heads + h) * tokens + t) * hd, (size_t)hd * 4);
}

int oracle_llama_decode(const oracle_llama_config *c, const oracle_llama_weights *w,
                        oracle_llama_cache *cache, const int64_t *tokens, int batch, int count,
                        float *logits, int threads) {
  if (batch != cache->batch || count <= 0 || cache->used + count > cache->capacity) return -1;
  int H = c->hidden, I = c->intermediate, NH = c->heads, KV = c->kv_heads, hd = H / NH;
  int KVD = KV * hd, rows = batch * count, pos = cache->used;
  size_t rh = (size_t)rows * H;
  float *hidden = (float *)malloc(rh * 4), *normed = (float *)malloc(rh * 4);
  float *q = (float *)malloc(rh * 4), *qh = (float *)malloc(rh * 4), *qr = (float *)malloc(rh * 4);
  float *k = (float *)malloc((size_t)rows * KVD * 4), *kh = (float *)malloc((size_t)rows * KVD * 4);
  float *kr = (float *)malloc((size_t)rows * KVD * 4);
  float *v = (float *)malloc((size_t)rows * KVD * 4), *vh = (float *)malloc((size_t)rows * KVD * 4);
  float *att = (float *)malloc(rh * 4), *attm = (float *)malloc(rh * 4), *proj = (float *)malloc(rh * 4);
  float *g = (float *)malloc((size_t)rows * I * 4), *u = (float *)malloc((size_t)rows * I * 4);
  for (int r = 0; r < rows; r++) { /* Embedding gather (CpuFloatBackend.embedding) */
    int64_t id = tokens[r];
    if (id < 0 || id >= c->vocab) return -2;
    memcpy(hidden + (size_t)r * H, w->embed + (size_t)id * H, (size_t)H * 4);
  }
  for (int l = 0; l < c->layers; l++) {
    /* LlamaBlock.cached (LlamaModel.scala:49-52): h = x + attention(norm(x)) */
    oracle_rmsnorm(hidden, w->in_norm[l], normed, rows, H, c->rms_eps);
    oracle_matmul_tr(normed, w->q[l], q, rows, H, H, threads);
    oracle_matmul_tr(normed, w->k[l], k, rows, KVD, H, threads);
    oracle_matmul_tr(normed, w->v[l], v, rows, KVD, H, threads);
    split_heads(q, qh, batch, count, NH, hd);
    split_heads(k, kh, batch, count, KV, hd);
    split_heads(v, vh, batch, count, KV, hd);
    oracle_rope(qh, qr, batch, NH, count, hd, pos, c->rope_theta);
    oracle_rope(kh, kr, batch, KV, count, hd, pos, c->rope_theta);
    /* LlamaCache.Layer.append (LlamaCache.scala:67-78) */
    for (int b = 0; b < batch; b++)
      for (int h = 0; h < KV; h++) {
        size_t from = ((size_t)b * KV + h) * count * hd;
        size_t to = (((size_t)b * KV + h) * cache->capacity + pos) * hd;
        memcpy(cache->keys[l] + to, kr + from, (size_t)count * hd * 4);
        memcpy(cache->values[l] + to, vh + from, (size_t)count * hd * 4);
      }
    oracle_causal_attention(qr, cache->keys[l], cache->values[l], att, batch, NH, count, hd, KV,
                            pos + count, cache->capacity, hd, pos);
    merge_heads(att, attm, batch, count, NH, hd);
    oracle_matmul_tr(attm, w->o[l], proj, rows, H, H, threads);
    for (size_t i = 0; i < rh; i++) hidden[i] = hidden[i] + proj[i];
    /* h + mlp(postNorm(h)); LlamaMLP: down(silu(gate(x)) * up(x)) (LlamaModel.scala:39-43) */
    oracle_rmsnorm(hidden, w->post_norm[l], normed, rows, H, c->rms_eps);
    oracle_matmul_tr(normed, w->gate[l], g, rows, I, H, threads);
    oracle_matmul_tr(normed, w->up[l], u, rows, I, H, threads);
    for (size_t i = 0; i < (size_t)rows * I; i++) g[i] = oracle_silu(g[i]) * u[i];
    oracle_matmul_tr(g, w->down[l], proj, rows, H, I, threads);
    for (size_t i = 0; i < rh; i++) hidden[i] = hidden[i] + proj[i];
  }
  oracle_rmsnorm(hidden, w->final_norm, normed, rows, H, c->rms_eps);
  oracle_matmul_tr(normed, w->lm_head, logits, rows, c->vocab, H, threads);
  cache->used = pos + count; /* LlamaCache.scala:45: publish only after success */
  free(hidden); free(normed); free(q); free(qh); free(qr); free(k); free(kh); free(kr);
  free(v); free(vh); free(att); free(attm); free(proj); free(g); free(u);
  return 0;
}

int oracle_llama_generate(const oracle_llama_config *c, const oracle_llama_weights *w,
                          const int64_t *prompt, int prompt_len, int max_new,
                          const int64_t *eos, int eos_count, int64_t *out, int threads) {
  memcpy(out, prompt, (size_t)prompt_len * 8);
  if (max_new == 0) return prompt_len;
  oracle_llama_cache *cache = oracle_cache_create(c, 1, prompt_len + max_new);
  float *logits = (float *)malloc((size_t)prompt_len * c->vocab * 4);
  int n = prompt_len;
  const int64_t *chunk = prompt;
  int chunk_len = prompt_len;
  for (int generated = 0; generated < max_new; generated++) {
    if (oracle_llama_decode(c, w, cache, chunk, 1, chunk_len, logits, threads) != 0) { n = -1; break; }
    int64_t next = oracle_argmax(logits + (size_t)(chunk_len - 1) * c->vocab, c->vocab);
    out[n++] = next;
    int stop = 0;
    for (int e = 0; e < eos_count; e++) stop |= (eos[e] == next);
    if (stop) break;
    chunk = out + n - 1;
    chunk_len = 1;
  }
  free(logits);
  oracle_cache_destroy(cache);
  return n;
}
