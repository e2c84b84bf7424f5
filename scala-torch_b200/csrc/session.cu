// Session, memory and transfer entry points of libstb200.so, plus the synthetic weight generator.
// Mirrors the ownership model of the reference's CudaSession (ffm/src/main/scala/scalatorch/ffm/
// CudaSession.scala): a byte budget checked before every allocation, one stream, reverse-order
// release at close, thread confinement.
#include <cstring>
#include <vector>

#include "common.cuh"
#include "rng.cuh"

namespace stb {

static thread_local std::string g_last_error;
void set_last_error(const std::string &msg) { g_last_error = msg; }

void enter(stb_session *s) {
  if (!s) throw Error(STB_ERR_STATE, "session is null");
  if (s->closed) throw Error(STB_ERR_STATE, "session is closed");
  if (std::this_thread::get_id() != s->owner)
    throw Error(STB_ERR_THREAD, "session used from another thread");
  STB_CUDA(cudaSetDevice(s->device));
}

uint64_t session_alloc(stb_session *s, uint64_t bytes) {
  if (bytes > s->max_bytes || s->allocated > s->max_bytes - bytes)
    throw Error(STB_ERR_BUDGET, "CUDA session allocation budget exceeded: requested " +
                                    std::to_string(bytes) + " with " + std::to_string(s->allocated) +
                                    " of " + std::to_string(s->max_bytes) + " in use");
  void *p = nullptr;
  uint64_t rounded = bytes ? bytes : 1;
  cudaError_t e = cudaMalloc(&p, rounded);
  if (e != cudaSuccess) {
    cudaGetLastError();
    throw Error(STB_ERR_BUDGET, std::string("cudaMalloc failed: ") + cudaGetErrorString(e));
  }
  s->allocations[(uint64_t)p] = bytes;
  s->allocated += bytes;
  return (uint64_t)p;
}

void session_free(stb_session *s, uint64_t ptr) {
  if (!ptr) return;
  auto it = s->allocations.find(ptr);
  if (it == s->allocations.end()) throw Error(STB_ERR_STATE, "release of an address this session does not own");
  // Work already enqueued may still read the buffer: complete the stream before freeing.
  STB_CUDA(cudaStreamSynchronize(s->stream));
  STB_CUDA(cudaFree((void *)ptr));
  s->allocated -= it->second;
  s->allocations.erase(it);
}

uint64_t session_scratch(stb_session *s, uint64_t bytes) {
  if (bytes <= s->scratch_bytes && s->scratch) return s->scratch;
  if (s->scratch) {
    session_free(s, s->scratch);
    s->scratch = 0;
    s->scratch_bytes = 0;
  }
  const uint64_t want = bytes < (64ull << 20) ? (64ull << 20) : bytes;
  s->scratch = session_alloc(s, want);
  s->scratch_bytes = want;
  return s->scratch;
}

int *session_error_word(stb_session *s) {
  if (!s->err_word) {
    s->err_word = session_alloc(s, 256);
    STB_CUDA(cudaMemsetAsync((void *)s->err_word, 0, 256, s->stream));
  }
  return (int *)s->err_word;
}

// Enqueues the copy of the device error word into pinned host memory (before a stream sync).
static void enqueue_error_read(stb_session *s) {
  if (!s->err_word) return;
  if (!s->err_host) STB_CUDA(cudaHostAlloc((void **)&s->err_host, 64, cudaHostAllocDefault));
  STB_CUDA(cudaMemcpyAsync(s->err_host, (const void *)s->err_word, 4, cudaMemcpyDeviceToHost, s->stream));
}

// After the stream sync that followed enqueue_error_read: every staged upload has landed, and a
// nonzero error word is cleared and reported.
static void finish_error_read(stb_session *s) {
  s->staging_pending[0] = s->staging_pending[1] = false;
  if (!s->err_word || !*s->err_host) return;
  const int code = *s->err_host;
  *s->err_host = 0;
  STB_CUDA(cudaMemset((void *)s->err_word, 0, 4));
  throw Error(STB_ERR_CUDA, "a device-side wait expired (code " + std::to_string(code) + "); results are invalid");
}

void sync_and_check(stb_session *s) {
  enqueue_error_read(s);
  STB_CUDA(cudaStreamSynchronize(s->stream));
  finish_error_read(s);
}

void check_launch(const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw Error(STB_ERR_CUDA, std::string(what) + " launch failed: " + cudaGetErrorString(e));
}

static constexpr uint64_t kStagingChunk = 64ull << 20;  // two halves of 64 MiB

static void ensure_staging(stb_session *s) {
  if (s->staging) return;
  STB_CUDA(cudaHostAlloc(&s->staging, 2 * kStagingChunk, cudaHostAllocDefault));
  s->staging_bytes = 2 * kStagingChunk;
  for (auto &ev : s->staging_done) STB_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
}

static bool is_pinned(const void *host) {
  cudaPointerAttributes attr;
  cudaError_t e = cudaPointerGetAttributes(&attr, host);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return attr.type == cudaMemoryTypeHost;
}

// ---------------------------------------------------------------- synthetic weights

__global__ void fill_normal_kernel(void *dst, int dtype, uint64_t count, uint64_t seed, uint64_t stream,
                                   double stddev) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < count;
       i += (uint64_t)gridDim.x * blockDim.x) {
    float v = __double2float_rn(__dmul_rn(stddev, rng_normal_dev(seed, stream, i)));
    if (dtype == STB_F32) ((float *)dst)[i] = v;
    else if (dtype == STB_BF16) ((uint16_t *)dst)[i] = f32_to_bf16_rne(v);
    else ((__half *)dst)[i] = __float2half_rn(v);
  }
}

__global__ void fill_value_kernel(void *dst, int dtype, uint64_t count, float value) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < count;
       i += (uint64_t)gridDim.x * blockDim.x) {
    if (dtype == STB_F32) ((float *)dst)[i] = value;
    else if (dtype == STB_BF16) ((uint16_t *)dst)[i] = f32_to_bf16_rne(value);
    else ((__half *)dst)[i] = __float2half_rn(value);
  }
}

void fill_normal(stb_session *s, uint64_t dst, int dtype, uint64_t count, uint64_t seed, uint64_t stream,
                 double stddev) {
  if (!count) return;
  uint64_t blocks = (count + 255) / 256;
  if (blocks > 148ull * 64) blocks = 148ull * 64;
  fill_normal_kernel<<<(unsigned)blocks, 256, 0, s->stream>>>((void *)dst, dtype, count, seed, stream, stddev);
  check_launch("fill_normal");
  count_launch(s);
}

void fill_value(stb_session *s, uint64_t dst, int dtype, uint64_t count, float value) {
  if (!count) return;
  uint64_t blocks = (count + 255) / 256;
  if (blocks > 148ull * 64) blocks = 148ull * 64;
  fill_value_kernel<<<(unsigned)blocks, 256, 0, s->stream>>>((void *)dst, dtype, count, value);
  check_launch("fill_value");
  count_launch(s);
}

void upload(stb_session *s, const void *host, uint64_t bytes, uint64_t dst) {
  if (!bytes) return;
  STB_REQUIRE(host && dst, "upload requires host and device buffers");
  if (is_pinned(host)) {
    STB_CUDA(cudaMemcpyAsync((void *)dst, host, bytes, cudaMemcpyHostToDevice, s->stream));
    return;
  }
  // Pageable source: double-buffered pinned staging, ordered on the session stream, so the copy
  // never races a later kernel (the pageable-HtoD hazard of docs/research/backend-llama.md:40-42).
  // The caller's buffer is free again on return (its bytes are in the staging half); a half is
  // refilled only after its previous copy completed (its event, or a later stream sync).
  ensure_staging(s);
  uint64_t done = 0;
  int slot = 0;
  while (done < bytes) {
    uint64_t n = bytes - done < kStagingChunk ? bytes - done : kStagingChunk;
    char *stage = (char *)s->staging + slot * kStagingChunk;
    if (s->staging_pending[slot]) STB_CUDA(cudaEventSynchronize(s->staging_done[slot]));
    std::memcpy(stage, (const char *)host + done, n);
    STB_CUDA(cudaMemcpyAsync((char *)dst + done, stage, n, cudaMemcpyHostToDevice, s->stream));
    STB_CUDA(cudaEventRecord(s->staging_done[slot], s->stream));
    s->staging_pending[slot] = true;
    done += n;
    slot ^= 1;
  }
}

void download(stb_session *s, uint64_t src, void *host, uint64_t bytes) {
  if (!bytes) {
    sync_and_check(s);
    return;
  }
  STB_REQUIRE(host && src, "download requires host and device buffers");
  if (is_pinned(host)) {
    STB_CUDA(cudaMemcpyAsync(host, (const void *)src, bytes, cudaMemcpyDeviceToHost, s->stream));
    sync_and_check(s);
    return;
  }
  // Pageable destination through the staging buffer (stream order puts these copies after any
  // staged upload still reading it).  The error word rides with the first chunk's sync.
  ensure_staging(s);
  uint64_t done = 0;
  bool first = true;
  while (done < bytes) {
    uint64_t n = bytes - done < 2 * kStagingChunk ? bytes - done : 2 * kStagingChunk;
    STB_CUDA(cudaMemcpyAsync(s->staging, (const char *)src + done, n, cudaMemcpyDeviceToHost, s->stream));
    if (first) enqueue_error_read(s);
    STB_CUDA(cudaStreamSynchronize(s->stream));
    if (first) finish_error_read(s);
    first = false;
    std::memcpy((char *)host + done, s->staging, n);
    done += n;
  }
}

}  // namespace stb

using namespace stb;

extern "C" {

int stb_version(void) { return 100; }

const char *stb_last_error(void) { return g_last_error.c_str(); }

int stb_session_create(int device, uint64_t max_bytes, stb_session **out) {
  return guarded([&] {
    STB_REQUIRE(out, "output handle is null");
    *out = nullptr;
    int count = 0;
    STB_CUDA(cudaGetDeviceCount(&count));
    STB_REQUIRE(device >= 0 && device < count, "device index out of range");
    STB_CUDA(cudaSetDevice(device));
    auto *s = new stb_session();
    s->device = device;
    s->max_bytes = max_bytes;
    s->owner = std::this_thread::get_id();
    cudaError_t e = cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
      delete s;
      throw Error(STB_ERR_CUDA, std::string("cudaStreamCreate failed: ") + cudaGetErrorString(e));
    }
    *out = s;
  });
}

void stb_session_close_tp(stb_session *s);  // nccl.cu

int stb_session_destroy(stb_session *s) {
  if (!s) return STB_OK;
  return guarded([&] {
    enter(s);
    cudaError_t first = cudaStreamSynchronize(s->stream);
    stb_session_close_tp(s);
    // Reverse acquisition order (CudaSession.scala:863-884): highest address last allocated is
    // not guaranteed, so free in reverse map order deterministically.
    for (auto it = s->allocations.rbegin(); it != s->allocations.rend(); ++it) cudaFree((void *)it->first);
    s->allocations.clear();
    s->allocated = 0;
    for (auto &ev : s->staging_done)
      if (ev) cudaEventDestroy(ev);
    if (s->staging) cudaFreeHost(s->staging);
    if (s->err_host) cudaFreeHost(s->err_host);
    cudaStreamDestroy(s->stream);
    s->closed = true;
    delete s;
    if (first != cudaSuccess) throw Error(STB_ERR_CUDA, std::string("pending work failed: ") + cudaGetErrorString(first));
  });
}

int stb_session_allocated(stb_session *s, uint64_t *bytes) {
  return guarded([&] {
    enter(s);
    STB_REQUIRE(bytes, "output is null");
    *bytes = s->allocated;
  });
}

int stb_session_stream(stb_session *s, void **stream) {
  return guarded([&] {
    enter(s);
    STB_REQUIRE(stream, "output is null");
    *stream = (void *)s->stream;
  });
}

int stb_session_launches(stb_session *s, uint64_t *launches) {
  return guarded([&] {
    enter(s);
    STB_REQUIRE(launches, "output is null");
    *launches = s->launches.load();
  });
}

int stb_alloc(stb_session *s, uint64_t bytes, uint64_t *dptr) {
  return guarded([&] {
    enter(s);
    STB_REQUIRE(dptr, "output is null");
    *dptr = session_alloc(s, bytes);
  });
}

int stb_release(stb_session *s, uint64_t dptr) {
  return guarded([&] {
    enter(s);
    session_free(s, dptr);
  });
}

int stb_upload(stb_session *s, const void *host, uint64_t bytes, uint64_t dst) {
  return guarded([&] {
    enter(s);
    upload(s, host, bytes, dst);
  });
}

int stb_download(stb_session *s, uint64_t src, void *host, uint64_t bytes) {
  return guarded([&] {
    enter(s);
    download(s, src, host, bytes);
  });
}

int stb_copy(stb_session *s, uint64_t dst, uint64_t src, uint64_t bytes) {
  return guarded([&] {
    enter(s);
    if (bytes) STB_CUDA(cudaMemcpyAsync((void *)dst, (const void *)src, bytes, cudaMemcpyDeviceToDevice, s->stream));
  });
}

int stb_sync(stb_session *s) {
  return guarded([&] {
    enter(s);
    sync_and_check(s);
  });
}

int stb_host_alloc(uint64_t bytes, void **host) {
  return guarded([&] {
    STB_REQUIRE(host, "output is null");
    STB_CUDA(cudaHostAlloc(host, bytes ? bytes : 1, cudaHostAllocDefault));
  });
}

int stb_host_free(void *host) {
  return guarded([&] {
    if (host) STB_CUDA(cudaFreeHost(host));
  });
}

int stb_fill_normal(stb_session *s, uint64_t dst, int dtype, uint64_t count, uint64_t seed, uint64_t stream,
                    double stddev) {
  return guarded([&] {
    enter(s);
    STB_REQUIRE(dtype == STB_F32 || dtype == STB_BF16 || dtype == STB_F16, "unsupported dtype");
    STB_REQUIRE(count == 0 || dst, "null destination");
    fill_normal(s, dst, dtype, count, seed, stream, stddev);
  });
}

int stb_fill_value(stb_session *s, uint64_t dst, int dtype, uint64_t count, float value) {
  return guarded([&] {
    enter(s);
    STB_REQUIRE(dtype == STB_F32 || dtype == STB_BF16 || dtype == STB_F16, "unsupported dtype");
    STB_REQUIRE(count == 0 || dst, "null destination");
    fill_value(s, dst, dtype, count, value);
  });
}

}  // extern "C"
