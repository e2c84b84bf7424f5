/*
 * stb200.h -- C ABI of libstb200.so, the B200 (sm_100a) device backend for scala-torch's
 * half-precision-weight Linear path and the Llama decode runtime built on it.
 *
 * Conventions follow the reference's FFM downcall idiom (ffm/src/main/scala/scalatorch/ffm/
 * CudaDriver.scala:13-19): every entry point returns an int status, 0 = OK, and never lets a
 * C++ exception cross the boundary.  Device addresses travel as uint64_t (CUdeviceptr, bound as
 * JAVA_LONG), dimensions as int (JAVA_INT), handles as opaque pointers (ADDRESS).  On failure
 * stb_last_error() returns a message for the calling thread.
 *
 * Ordering: all device work of a session runs on the session's one non-blocking stream, in call
 * order.  Unlike CudaSession (which synchronises after every launch, CudaSession.scala:829-850)
 * calls return once the work is enqueued; stb_download and stb_sync complete it.
 * A session is thread-confined (CudaSession.scala:25,63-67): calls from another thread fail
 * with STB_ERR_THREAD.
 */
#ifndef STB200_H
#define STB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct stb_session stb_session;
typedef struct stb_llama stb_llama;
typedef struct stb_llama_cache stb_llama_cache;

enum stb_status {
  STB_OK = 0,
  STB_ERR_INVALID = 1,     /* bad shape / argument: IllegalArgumentException before launch */
  STB_ERR_BUDGET = 2,      /* session byte budget exceeded (CudaSession.scala:81-93) */
  STB_ERR_CUDA = 3,        /* CUDA runtime failure */
  STB_ERR_NCCL = 4,        /* NCCL failure */
  STB_ERR_THREAD = 5,      /* used from a thread other than the owner */
  STB_ERR_STATE = 6,       /* closed / stale handle: IllegalStateException */
  STB_ERR_UNSUPPORTED = 7, /* valid request this build does not implement */
};

/* Element types of weight payloads, as SafeTensors' SafeDType (io/.../SafeTensors.scala:9-16). */
enum stb_dtype { STB_F32 = 0, STB_BF16 = 1, STB_F16 = 2 };

/* ---------------------------------------------------------------- library / session */

/* ABI version (major*10000 + minor*100 + patch). */
int stb_version(void);
/* Message of the last failure on this thread ("" if none). */
const char *stb_last_error(void);

/* CudaSession.withDevice(deviceIndex, maxBytes), ffm/.../CudaSession.scala:886-891:
 * binds device `device`, creates the session stream, charges allocations against max_bytes. */
int stb_session_create(int device, uint64_t max_bytes, stb_session **out);
/* CudaSession close, CudaSession.scala:863-884: drains the stream, frees every allocation of the
 * session in reverse order.  Idempotent on NULL. */
int stb_session_destroy(stb_session *s);
/* CudaSession.allocatedBytes. */
int stb_session_allocated(stb_session *s, uint64_t *bytes);
/* cudaStream_t of the session (for callers that interleave their own work). */
int stb_session_stream(stb_session *s, void **stream);

/* CudaSession.allocate (CudaSession.scala:81-93): rejects with STB_ERR_BUDGET before allocating. */
int stb_alloc(stb_session *s, uint64_t bytes, uint64_t *dptr);
/* CudaSession.release (CudaSession.scala:852-861); releasing 0 is a no-op. */
int stb_release(stb_session *s, uint64_t dptr);
/* CudaSession.upload (CudaSession.scala:523-549) with any payload: `bytes` raw bytes from host
 * memory into device memory at dst, through pinned staging on the session stream.  Used for the
 * raw BF16/F16 safetensors payloads (no F32 expansion; replaces SafeTensors.readFloat +
 * upload of widened F32, SafeTensors.scala:63-77, BackendLlama.scala:153-174). */
int stb_upload(stb_session *s, const void *host, uint64_t bytes, uint64_t dst);
/* CudaSession.download (CudaSession.scala:551-559): completes all prior work, then copies. */
int stb_download(stb_session *s, uint64_t src, void *host, uint64_t bytes);
/* Device-to-device copy on the session stream. */
int stb_copy(stb_session *s, uint64_t dst, uint64_t src, uint64_t bytes);
/* cuStreamSynchronize on the session stream. */
int stb_sync(stb_session *s);
/* Pinned host memory for transfer buffers (cudaHostAlloc / cudaFreeHost). */
int stb_host_alloc(uint64_t bytes, void **host);
int stb_host_free(void *host);

/* ---------------------------------------------------------------- Linear */

/* nn.Linear.apply without adapters, nn/src/main/scala/scalatorch/nn/Linear.scala:11-17, as it
 * reaches FloatBackend.matmul(x, W^T) (core/.../FloatBackend.scala:16; CudaSession.matmul,
 * CudaSession.scala:561-571; NumscalaBackend.matmul, cpu/.../NumscalaBackend.scala:19-30):
 *   y[M,N] = x[M,K] . W[N,K]^T (+ bias[N])
 * x, y, bias: Float32 row-major device buffers; W: the (out,in) weight exactly as stored in the
 * safetensors payload (w_dtype STB_BF16 or STB_F16; STB_F32 is accepted too), widened in
 * registers.  FP32-accurate activations: the SIMT GEMV (FP32 FMA accumulation), or, for BF16 products
 * above 2^24 multiply-adds, the tcgen05 skinny form (activations split into three BF16 terms, FP32
 * accumulation); both within 1e-5 relative of the FP32 product.  M = 0 / N = 0 are no-ops; K = 0
 * writes bias or zeros.  bias may be 0. */
int stb_linear(stb_session *s, uint64_t x, uint64_t w, int w_dtype, uint64_t bias, uint64_t y,
               int M, int N, int K);
/* Same product with explicit leading dimensions (elements) for x and y. */
int stb_linear_ld(stb_session *s, uint64_t x, int ldx, uint64_t w, int w_dtype, uint64_t bias,
                  uint64_t y, int ldy, int M, int N, int K);
/* The prefill form of the same Linear (M >= 256 tokens): x is rounded to the weight's type
 * (BF16 or F16, round-to-nearest-even) and multiplied on the tcgen05 tensor cores with FP32
 * accumulation in TMEM.  The activation rounding is the stated tolerance source. */
int stb_linear_prefill(stb_session *s, uint64_t x, uint64_t w, int w_dtype, uint64_t bias,
                       uint64_t y, int M, int N, int K);
/* No counterpart in the reference.  The prefill Linear above without any device allocation, for
 * callers that may not allocate device memory themselves (a host framework that owns every device
 * allocation through its own allocator or budget; a serving loop that forbids allocation after
 * warm-up).  The rounded activations go to a fixed 16 MiB array compiled into the library instead
 * of the session's scratch, so M * K must not exceed 8,388,608 (larger requests are rejected with
 * STB_ERR_INVALID).  Runs on `stream` (a cudaStream_t, NULL for the legacy stream) of the current
 * device and returns after the product is complete.  All calls share the array: calls that
 * overlap on the GPU (other threads or streams) race.  The first call on a device is its set-up:
 * it loads the library's device code there (with CUDA's lazy module loading, that places the
 * 16 MiB + 256 byte array and the kernels in device memory) and looks up the array's address; make
 * it during warm-up, before any stream capture.  Later calls allocate nothing.  A cudaDeviceReset
 * while the library is loaded is not supported (the kept address would dangle). */
int stb_linear_prefill_static(void *stream, uint64_t x, uint64_t w, int w_dtype, uint64_t bias, uint64_t y,
                              int M, int N, int K);
/* One low-rank adapter term of nn.Linear.apply (nn/src/main/scala/scalatorch/nn/Linear.scala:11-17;
 * LowRankAdapter.apply, LowRankAdapter.scala:12-14; LinearAdapterScope.forWeight,
 * LinearAdapterScope.scala:14-21).  a: Float32 [rank, K] device buffer, b: Float32 [N, rank];
 * scale = LowRankAdapter.scale, (alpha / rank) rounded to Float32.  scoped = 0 is the Linear's own
 * adapter (`base + a(x)`), scoped = 1 a LinearAdapterScope entry (`sum + a(x) * multiplier`). */
typedef struct stb_adapter {
  uint64_t a;
  uint64_t b;
  int rank;
  float scale;
  int scoped;
  float multiplier;
} stb_adapter;

/* nn.Linear.apply with adapters (Linear.scala:11-17), each operation rounded to Float32 in the
 * reference's order: base = x.W^T; for each term in array order (the Linear's own adapter, if any,
 * first): t = x.A^T, u = t.B^T, v = u * scale (* multiplier when scoped), sum = sum + v; finally
 * sum + bias.  count = 0 is stb_linear.  Rejects (STB_ERR_INVALID) a null or non-positive factor,
 * a non-finite or non-positive scale, a non-finite multiplier, and an unscoped term that is not
 * first. */
int stb_linear_adapted(stb_session *s, uint64_t x, uint64_t w, int w_dtype, uint64_t bias,
                       const stb_adapter *adapters, int count, uint64_t y, int M, int N, int K);
/* Host-buffer form used for end-to-end measurement: copies x from host, runs stb_linear against
 * the resident weight, copies y back.  Synchronous.  Requests of up to 64 MiB of x and y keep one
 * grow-only device buffer in the session between calls (charged to its budget). */
int stb_linear_host(stb_session *s, const float *x_host, uint64_t w, int w_dtype, uint64_t bias,
                    float *y_host, int M, int N, int K);

/* ---------------------------------------------------------------- FloatBackend operator set
 *
 * The rest of trait FloatBackend (core/src/main/scala/scalatorch/FloatBackend.scala:7-31) as the
 * reference's generic BackendLlama drives it (models/src/main/scala/scalatorch/models/
 * BackendLlama.scala:41-111), one kernel each on the session stream.  Buffers are Float32 device
 * addresses, packed row-major; outputs are caller-allocated (stb_alloc) and may not alias inputs
 * unless stated.  Arithmetic is the reference CPU backend's (CpuFloatBackend.scala,
 * CpuAttention.scala): add / multiply / scale one Float32 operation per element; SiLU, RMSNorm,
 * RoPE and attention in double, rounded once.  Shape rules that the reference checks with
 * require(...) are checked by the host binding before the call; the calls themselves reject what
 * would be out of bounds (STB_ERR_INVALID).  reshape is a view (host-side: no call), fill is
 * stb_fill_value. */

/* FloatBackend.add / multiply (CpuFloatBackend.scala:61-67): y[i] = a[i] + b[i] / a[i] * b[i]. */
int stb_op_add(stb_session *s, uint64_t a, uint64_t b, uint64_t y, uint64_t count);
int stb_op_multiply(stb_session *s, uint64_t a, uint64_t b, uint64_t y, uint64_t count);
/* FloatBackend.scale (CpuFloatBackend.scala:68-69): y[i] = x[i] * scalar, IEEE nonfinite included. */
int stb_op_scale(stb_session *s, uint64_t x, uint64_t y, uint64_t count, float scalar);
/* FloatBackend.silu (CpuFloatBackend.scala:70-77): x * sigmoid(x) in double. */
int stb_op_silu(stb_session *s, uint64_t x, uint64_t y, uint64_t count);
/* FloatBackend.sum (CpuFloatBackend.scala:31-32): all elements into one Float32 at y, accumulated in
 * double (a fixed tree: deterministic for a given count). */
int stb_op_sum(stb_session *s, uint64_t x, uint64_t count, uint64_t y);
/* FloatBackend.expandScalar (CpuFloatBackend.scala:33-35): y[i] = *x, no host transfer. */
int stb_op_expand_scalar(stb_session *s, uint64_t x, uint64_t y, uint64_t count);
/* FloatBackend.rmsNorm (CpuFloatBackend.scala:78-93) over the last axis of `rows` rows of `width`:
 * squares summed in double, y = (float)(x * (1 / sqrt(sum / width + eps)) * w[j]). */
int stb_op_rmsnorm(stb_session *s, uint64_t x, uint64_t w, uint64_t y, uint64_t rows, int width, double eps);
/* FloatBackend.rope (CpuAttention.scala:6-18, RotaryCoefficients AttentionLayout.scala:23-34) on
 * (batch, heads, tokens, width): pairs (d, d + width/2) rotated by the host-computed double
 * coefficients of positions start .. start + tokens - 1. */
int stb_op_rope(stb_session *s, uint64_t x, uint64_t y, int batch, int heads, int tokens, int width, int start,
                double theta);
/* FloatBackend.transpose (CudaSession.scala:469-485): a packed copy with axes dim0 and dim1 of the
 * rank-`rank` (<= 8) input `dims` swapped. */
int stb_op_transpose(stb_session *s, uint64_t x, uint64_t y, int rank, const int64_t *dims, int dim0, int dim1);
/* FloatBackend.embedding (CpuFloatBackend.scala:49-59; CudaSession.scala:487-500): rows ids[0..count) of a (rows, width) table
 * in F32, BF16 or F16 (half rows widened exactly) into y (count, width).  ids are host int64 and
 * must lie in [0, rows). */
int stb_op_embedding(stb_session *s, uint64_t table, int dtype, int64_t rows, int width, const int64_t *ids,
                     uint64_t count, uint64_t y);
/* AttentionCache.attend's append (CudaSession.scala:414-419): src (batch, heads, tokens, width) into
 * the cache (batch, heads, capacity, width) at token `position`. */
int stb_op_cache_append(stb_session *s, uint64_t src, uint64_t cache, int batch, int heads, int tokens, int width,
                        int capacity, int position);
/* FloatBackend.causalAttention (CpuAttention.scala:20-50): q (batch, heads, tokens, width); k, v
 * (batch, kv_heads, key_stride, width / value_width) of which the first `keys` tokens are read;
 * query token t of the chunk sees keys j < min(keys, start + t + 1).  Scores, softmax and the
 * weighted sum in double.  keys <= 24576 (STB_ERR_UNSUPPORTED above). */
int stb_op_causal_attention(stb_session *s, uint64_t q, uint64_t k, uint64_t v, uint64_t y, int batch, int heads,
                            int tokens, int width, int kv_heads, int keys, int key_stride, int value_width,
                            int start);

/* ---------------------------------------------------------------- synthetic weights */

/* Counter-based N(0, std) weights rounded F32 -> half with RNE (SafeTensorsWriter.bfloat,
 * io/.../SafeTensorsWriter.scala:58-61); bit-identical to the CPU restatement keyed by the same
 * (seed, stream).  Stands in for LlamaModel.init's java.util.Random draw (LlamaModel.scala:148-156)
 * with a reproducible, sliceable stream. */
int stb_fill_normal(stb_session *s, uint64_t dst, int dtype, uint64_t count, uint64_t seed,
                    uint64_t stream, double std);
int stb_fill_value(stb_session *s, uint64_t dst, int dtype, uint64_t count, float value);

/* ---------------------------------------------------------------- Llama runtime */

/* LlamaConfig fields used by the runtime (models/.../LlamaConfig.scala:12-23). */
typedef struct {
  int vocab_size, hidden_size, intermediate_size, num_layers;
  int num_attention_heads, num_key_value_heads, max_positions, tie_word_embeddings;
  double rms_norm_eps, rope_theta;
  int weight_dtype; /* STB_BF16 or STB_F16 */
  int tp_rank, tp_size; /* tensor parallel coordinates; 0/1 for a single device */
  /* Chunks of at least this many token rows run their projections on the tcgen05 tensor cores
   * with activations rounded to the weight type (the prefill tolerance); smaller chunks -- every
   * decode step -- keep Float32 activations.  0 selects the default (256, the prefill threshold of the
   * Linear path); < 0 never. */
  int tc_prefill_rows;
} stb_llama_config;

/* Weight names, LlamaModel.namedWeights (LlamaModel.scala:91-105). */
enum stb_llama_weight {
  STB_W_EMBED = 0, STB_W_FINAL_NORM = 1, STB_W_LM_HEAD = 2, STB_W_IN_NORM = 3, STB_W_POST_NORM = 4,
  STB_W_Q = 5, STB_W_K = 6, STB_W_V = 7, STB_W_O = 8, STB_W_GATE = 9, STB_W_UP = 10, STB_W_DOWN = 11,
};

/* BackendLlama.prepare (models/.../BackendLlama.scala:153-174): validates the config, allocates
 * resident weights (half, never widened; tied lm_head stored once) in the session. */
int stb_llama_create(stb_session *s, const stb_llama_config *config, stb_llama **out);
int stb_llama_destroy(stb_llama *m);
/* Resident weight bytes of this rank. */
int stb_llama_weight_bytes(stb_llama *m, uint64_t *bytes);
/* Upload one named tensor's raw payload (the full, unsharded tensor as in the safetensors file;
 * this rank keeps its shard).  dtype must be the config's weight_dtype for matrices; norms may be
 * F32/BF16/F16 and are widened exactly.  layer is ignored for global tensors. */
int stb_llama_set_weight(stb_llama *m, int which, int layer, const void *host, uint64_t bytes,
                         int dtype);
/* LlamaModel.init analogue: every matrix ~ N(0, std) from the counter-based generator with
 * stream = layer*16 + which (global tensors: 4096 + which), norms = 1.  Generated on device. */
int stb_llama_init_random(stb_llama *m, uint64_t seed, double std);

/* BackendLlama.newCache / BackendLlamaCache (BackendLlamaCache.scala:8-49): Float32 K/V resident
 * in HBM, (batch, kv_heads, capacity, head_dim) per layer. */
int stb_llama_cache_create(stb_llama *m, int batch, int capacity, stb_llama_cache **out);
int stb_llama_cache_destroy(stb_llama_cache *c);
int stb_llama_cache_position(stb_llama_cache *c, int *position);
int stb_llama_cache_reset(stb_llama_cache *c);
/* BackendLlamaCache.decode (BackendLlamaCache.scala:31-41): tokens (batch, count) host int64 ->
 * logits (batch, count, vocab) host f32 (may be NULL) and greedy next ids per batch row host
 * int64 (may be NULL).  The position advances only after the whole chunk succeeded. */
int stb_llama_decode(stb_llama_cache *c, const int64_t *tokens, int batch, int count,
                     float *logits, int64_t *next_ids);
/* BackendLlama.generateIds with temperature 0 (BackendLlama.scala:126-141, TokenSampler greedy):
 * batch rows of prompt_len host ids; writes batch*(prompt_len+max_new) ids to out (row-major);
 * stops a row at any of eos[0..eos_count).  Decode steps run as one replayed CUDA graph with the
 * token feedback, position and stop flag kept on the device.  generated[b] receives the count of
 * generated ids per row (may be NULL).  timings_ms (may be NULL) receives {prefill, decode}. */
int stb_llama_generate(stb_llama *m, const int64_t *prompt, int batch, int prompt_len, int max_new,
                       const int64_t *eos, int eos_count, int64_t *out, int *generated,
                       float *timings_ms);

/* ---------------------------------------------------------------- tensor parallel (NCCL) */

/* The Megatron shard of `rank` in a tp-way split of config (host-only; no device is touched).
 * out[0..13] = query heads [begin, end), KV heads [begin, end), intermediate rows [begin, end),
 * vocabulary rows [begin, end), o_proj input columns [begin, end), down_proj input columns
 * [begin, end), and the resident half-weight bytes of that rank, and 0.  Fails like
 * stb_llama_create when the split is uneven.  No counterpart in the reference (it has no
 * distributed path, LlamaConfig.scala:91). */
int stb_llama_shard_plan(const stb_llama_config *config, int rank, int tp, int64_t out[14]);

/* ncclGetUniqueId: 128 bytes to broadcast from rank 0 to the group. */
int stb_nccl_unique_id(uint8_t id[128]);
/* ncclCommInitRank on the session's device; one communicator per session. */
int stb_session_init_tp(stb_session *s, int nranks, int rank, const uint8_t id[128]);
/* In-place Float32 sum allreduce on the session stream (the one exchange per row-split projection). */
int stb_allreduce_sum_f32(stb_session *s, uint64_t buf, uint64_t count);
/* Whether stb_session_init_tp mapped the group's NVLink receive buffers (CUDA IPC) that let the
 * decode step's row-split projections store their partial sums straight into every rank and reduce
 * them in rank order (set STB_TP_PEER=0 to keep NCCL); slot_elems = Float32 values one projection may
 * exchange per rank.  No counterpart in the reference. */
int stb_session_tp_peer(stb_session *s, int *enabled, uint64_t *slot_elems);
/* Failure detection without a fault: runs the device-side bounded wait used by the peer exchange on
 * a counter nothing increments, for wait_ns (<= 5 s), and returns the error code the kernel recorded
 * (99) -- the context stays usable.  No counterpart in the reference. */
int stb_check_bounded_wait(stb_session *s, uint64_t wait_ns, int *code);

/* ---------------------------------------------------------------- measurement */

/* Number of this library's kernel launches since the session was created (graph replays count
 * each kernel node once per replay). */
int stb_session_launches(stb_session *s, uint64_t *launches);

#ifdef __cplusplus
}
#endif
#endif
