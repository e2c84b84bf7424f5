/*
 * stb_oracle.h -- CPU restatement of scala-torch's Float32 Linear / Llama decode arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (libstb200.so, the scalatorch Python
 * mirror) links, loads or calls this code.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py use it, and only as the checker or the
 * timed CPU baseline.
 *
 * Every function names the reference file:line whose arithmetic it restates.  Paths are
 * relative to the scala-torch project root.
 *
 * Parity pin: the element conversions (BF16/F16 widening, F32->BF16 RNE) and the small
 * integer GEMM answers are pinned against the reference's own known-answer tests (see
 * tests/golden/).  The numscala reduction order for non-integer data at K >= 5 lives in the
 * un-vendored artifact com.github.kmizu::numscala:0.5.0 and is restated from its documented
 * description (ffm/src/main/resources/scalatorch/gemm.ptx:180-193,
 * docs/research/float-backends.md:33); that order is "parity unpinned" and the tests compare
 * within tolerance against both restated orders.
 */
#ifndef STB_ORACLE_H
#define STB_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORACLE_F32 = 0, ORACLE_BF16 = 1, ORACLE_F16 = 2 };
enum { ORACLE_ORDER_NUMSCALA = 0, ORACLE_ORDER_SEQUENTIAL = 1 };

/* io/src/main/scala/scalatorch/io/SafeTensors.scala:72 */
float oracle_bf16_to_f32(uint16_t bits);
/* io/src/main/scala/scalatorch/io/SafeTensors.scala:71 (java.lang.Float.float16ToFloat) */
float oracle_f16_to_f32(uint16_t bits);
/* io/src/main/scala/scalatorch/io/SafeTensorsWriter.scala:58-61 */
uint16_t oracle_f32_to_bf16(float value);
/* F32 -> F16 round-to-nearest-even (java.lang.Float.floatToFloat16 semantics); used to make
 * F16 fixtures for the F16-weight variant. */
uint16_t oracle_f32_to_f16(float value);
/* SafeTensors.readFloat widening loop, SafeTensors.scala:63-77 */
void oracle_widen(const void *src, int dtype, float *dst, size_t count);
void oracle_round_bf16(const float *src, uint16_t *dst, size_t count);
void oracle_round_f16(const float *src, uint16_t *dst, size_t count);

/* y[M,N] = x[M,K] . W[N,K]^T as NumscalaBackend.matmul(x, W.transpose(0,1)) reaches
 * ScalarF32Kernels.gemmInto with Transpose.Yes (cpu/src/main/scala/scalatorch/cpu/
 * NumscalaBackend.scala:8-30).  Four Float32 partial sums selected by k mod 4, the tail of an
 * incomplete group into sum 0, separately rounded multiply and add, then (s0+s1)+(s2+s3)
 * (gemm.ptx:167-193).  threads <= 1: one thread; otherwise OpenMP over output rows. */
void oracle_matmul_tr(const float *x, const float *w, float *y, int M, int N, int K, int threads);
/* C[M,N] = A[M,K] . B[K,N] with one sequential Float32 accumulator (core/src/main/scala/
 * scalatorch/Ops.scala:61-81). */
void oracle_matmul_seq(const float *a, const float *b, float *c, int M, int N, int K);
/* nn.Linear.apply (nn/src/main/scala/scalatorch/nn/Linear.scala:11-17) for a half or F32
 * (out,in) weight that SafeTensors.readFloat widens first: y = x.W^T [+ bias]. */
void oracle_linear(const float *x, const void *w, int w_dtype, const float *bias, float *y,
                   int M, int N, int K, int order, int threads);
void oracle_linear_adapted(const float *x, const void *w, int w_dtype, const float *bias,
                           const float *const *a, const float *const *b, const int *rank,
                           const float *scale, const int *scoped, const float *multiplier, int count,
                           float *y, int M, int N, int K, int threads);

/* CpuFloatBackend.rmsNorm, cpu/src/main/scala/scalatorch/cpu/CpuFloatBackend.scala:78-93 */
void oracle_rmsnorm(const float *x, const float *w, float *y, int rows, int width, double eps);
/* CpuFloatBackend.silu, CpuFloatBackend.scala:70-77 */
float oracle_silu(float x);
/* CpuAttention.rope on (batch,heads,tokens,width), cpu/src/main/scala/scalatorch/cpu/
 * CpuAttention.scala:6-18 with RotaryCoefficients, core/src/main/scala/scalatorch/
 * AttentionLayout.scala:23-34 */
void oracle_rope(const float *x, float *y, int batch, int heads, int tokens, int width,
                 int start, double theta);
/* CpuAttention.causal, CpuAttention.scala:20-50.  q:(B,H,T,D) k:(B,KV,S,D) v:(B,KV,S,DV)
 * with explicit token strides for k/v (capacity-strided caches, CpuAttentionCache). */
void oracle_causal_attention(const float *q, const float *k, const float *v, float *out,
                             int batch, int heads, int tokens, int width, int kv_heads,
                             int keys, int key_stride_tokens, int value_width, int start);
/* TokenSampler greedy branch, models/src/main/scala/scalatorch/models/TokenSampler.scala:32-38:
 * strict '>' so the lowest index wins ties. */
int64_t oracle_argmax(const float *logits, int64_t count);

/* Counter-based synthetic weights: splitmix64 keyed by (seed, stream, index), Marsaglia polar
 * normal in IEEE double with a hand-written log, scaled by std, rounded to F32 and then to BF16
 * with SafeTensorsWriter.bfloat's RNE.  Bit-identical to the device generator. */
uint64_t oracle_rng_u64(uint64_t seed, uint64_t stream, uint64_t index);
double oracle_rng_normal(uint64_t seed, uint64_t stream, uint64_t index);
void oracle_fill_normal_bf16(uint16_t *dst, size_t count, uint64_t seed, uint64_t stream,
                             double std, int threads);
void oracle_fill_normal_f32(float *dst, size_t count, uint64_t seed, uint64_t stream, double std,
                            int threads);
double oracle_log(double x);

/* ---- Llama decode (LlamaModel / LlamaCache / BackendLlama on the CPU path) ---- */
typedef struct {
  int vocab, hidden, intermediate, layers, heads, kv_heads, max_positions, tie_embeddings;
  double rms_eps, rope_theta;
} oracle_llama_config;

/* Weights as F32 (already widened, the reference's in-memory form).  Layouts (out,in).
 * Per layer: in_norm[H], post_norm[H], q[H*H], k[KVD*H], v[KVD*H], o[H*H], gate[I*H], up[I*H],
 * down[H*I].  lm_head == embed when tied. */
typedef struct {
  const float *embed, *final_norm, *lm_head;
  const float **in_norm, **post_norm, **q, **k, **v, **o, **gate, **up, **down;
} oracle_llama_weights;

typedef struct oracle_llama_cache oracle_llama_cache;
oracle_llama_cache *oracle_cache_create(const oracle_llama_config *c, int batch, int capacity);
void oracle_cache_destroy(oracle_llama_cache *cache);
int oracle_cache_position(const oracle_llama_cache *cache);
/* LlamaCache.decode, models/src/main/scala/scalatorch/models/LlamaCache.scala:26-47:
 * tokens (batch,count) -> logits (batch,count,vocab); advances the cache position. */
int oracle_llama_decode(const oracle_llama_config *c, const oracle_llama_weights *w,
                        oracle_llama_cache *cache, const int64_t *tokens, int batch, int count,
                        float *logits, int threads);
/* LlamaModel.generateIds greedy with cache (LlamaModel.scala:68-90); eos_count may be 0.
 * Returns the number of ids written to out (prompt + generated). */
int oracle_llama_generate(const oracle_llama_config *c, const oracle_llama_weights *w,
                          const int64_t *prompt, int prompt_len, int max_new,
                          const int64_t *eos, int eos_count, int64_t *out, int threads);

int oracle_max_threads(void);

#ifdef __cplusplus
}
#endif
#endif
