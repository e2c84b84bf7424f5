// Shared internals of libstb200.so: status plumbing, the session object, small device helpers.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <map>
#include <stdexcept>
#include <string>
#include <thread>

#include "../../include/stb200.h"

namespace stb {

// Error carried to the C boundary as a status code plus a thread-local message.
struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string &m) : std::runtime_error(m), code(c) {}
};

void set_last_error(const std::string &msg);

#define STB_REQUIRE(cond, msg)                                      \
  do {                                                              \
    if (!(cond)) throw ::stb::Error(STB_ERR_INVALID, (msg));        \
  } while (0)

#define STB_CUDA(call)                                                                       \
  do {                                                                                       \
    cudaError_t e_ = (call);                                                                 \
    if (e_ != cudaSuccess)                                                                   \
      throw ::stb::Error(STB_ERR_CUDA, std::string(#call) + " failed: " + cudaGetErrorString(e_)); \
  } while (0)

// Runs `body` and maps every exception to a status; nothing escapes the C ABI.
template <typename F>
int guarded(F &&body) {
  try {
    body();
    set_last_error("");
    return STB_OK;
  } catch (const Error &e) {
    set_last_error(e.what());
    return e.code;
  } catch (const std::bad_alloc &) {
    set_last_error("host allocation failed");
    return STB_ERR_BUDGET;
  } catch (const std::exception &e) {
    set_last_error(e.what());
    return STB_ERR_CUDA;
  } catch (...) {
    set_last_error("unknown failure");
    return STB_ERR_CUDA;
  }
}

}  // namespace stb

struct stb_session {
  int device = 0;
  cudaStream_t stream = nullptr;
  uint64_t max_bytes = 0, allocated = 0;
  std::map<uint64_t, uint64_t> allocations;  // device address -> bytes
  std::thread::id owner;
  void *staging = nullptr;  // pinned host staging for pageable transfers
  uint64_t staging_bytes = 0;
  cudaEvent_t staging_done[2] = {nullptr, nullptr};
  bool staging_pending[2] = {false, false};  // an upload from that half may still be in flight
  int *err_host = nullptr;                   // pinned copy of the device error word, read at each sync
  uint64_t io_buf = 0, io_bytes = 0;         // grow-only device buffer of the host-buffer Linear
  void *nccl = nullptr;  // ncclComm_t
  void *peer = nullptr;  // PeerComm (peer.cu): IPC-mapped receive buffers of the TP group
  int tp_rank = 0, tp_size = 1;
  std::atomic<uint64_t> launches{0};
  uint64_t scratch = 0, scratch_bytes = 0;  // grow-only device scratch (charged to the budget)
  uint64_t err_word = 0;                    // device int: nonzero when a bounded device wait expired
  bool closed = false;
};

namespace stb {

// Validates a session handle, its owner thread, and makes its device current.
void enter(stb_session *s);
uint64_t session_alloc(stb_session *s, uint64_t bytes);
void session_free(stb_session *s, uint64_t ptr);
inline void count_launch(stb_session *s, uint64_t n = 1) { s->launches += n; }

// Integer tuning switch from the environment, or `fallback` when unset.
inline int env_int(const char *name, int fallback) {
  const char *v = std::getenv(name);
  return v && *v ? std::atoi(v) : fallback;
}
void check_launch(const char *what);
void upload(stb_session *s, const void *host, uint64_t bytes, uint64_t dst);
void download(stb_session *s, uint64_t src, void *host, uint64_t bytes);
void fill_normal(stb_session *s, uint64_t dst, int dtype, uint64_t count, uint64_t seed, uint64_t stream,
                 double stddev);
void fill_value(stb_session *s, uint64_t dst, int dtype, uint64_t count, float value);
// Grow-only scratch buffer of at least `bytes` (contents undefined).
uint64_t session_scratch(stb_session *s, uint64_t bytes);
// Device error word kernels write when a bounded wait expires (allocated and zeroed on first use).
int *session_error_word(stb_session *s);
// After a stream synchronisation: throws (and clears the word) if a kernel recorded an error.
// Completes the session stream and reports an expired device wait, reading the error word with
// the same synchronisation.
void sync_and_check(stb_session *s);

// ---------------------------------------------------------------- launch helpers

// Launches `kernel` on `stream`; with pdl the launch carries programmatic stream serialisation, so
// it may start while the previous kernel drains -- the kernel must call pdl_wait() before it
// touches anything the previous kernel writes.  Inside stream capture this becomes a
// programmatic graph edge.
template <typename... KArgs, typename... Args>
void launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl,
                   Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (e != cudaSuccess) throw Error(STB_ERR_CUDA, std::string("kernel launch failed: ") + cudaGetErrorString(e));
}

// ---------------------------------------------------------------- device helpers

// Programmatic dependent launch: wait for the prerequisite grid's completion and memory, and let
// the dependent grid begin launching.  Both are no-ops for launches without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// L2 prefetch of a byte range (16-byte aligned start, size a multiple of 16), issued by one thread.
__device__ __forceinline__ void prefetch_l2(const void *p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ uint4 ld_stream_u4(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Widen two packed half words (low half first in memory) to Float32, exactly.
template <typename WT>
__device__ __forceinline__ float2 widen2(uint32_t u);

template <>
__device__ __forceinline__ float2 widen2<__nv_bfloat16>(uint32_t u) {
  // SafeTensors.scala:72: bits << 16 is the Float32 with the same value.
  return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
}

template <>
__device__ __forceinline__ float2 widen2<__half>(uint32_t u) {
  __half2 h = *reinterpret_cast<__half2 *>(&u);
  return __half22float2(h);
}

template <typename WT>
__device__ __forceinline__ float widen1(uint16_t u);
template <>
__device__ __forceinline__ float widen1<__nv_bfloat16>(uint16_t u) {
  return __uint_as_float(((uint32_t)u) << 16);
}
template <>
__device__ __forceinline__ float widen1<__half>(uint16_t u) {
  return __half2float(__ushort_as_half(u));
}

__device__ __forceinline__ uint16_t f32_to_bf16_rne(float value) {
  // SafeTensorsWriter.scala:58-61.
  uint32_t bits = __float_as_uint(value);
  if ((bits & 0x7f800000u) == 0x7f800000u && (bits & 0x007fffffu) != 0)
    return (uint16_t)((bits >> 16) | 0x40u);
  return (uint16_t)((bits + 0x7fffu + ((bits >> 16) & 1u)) >> 16);
}

// f = x0 + x1 + x2 in three BF16 terms: x0 = rne(f), x1 = rne(f - x0), x2 = rne(f - x0 - x1) (both
// differences exact), which carry f's 24-bit significand.  A non-finite f keeps its class in x0 alone
// (Inf - Inf would make the lower terms NaN); a finite f that rounds past BF16's largest finite value
// (|f| > 0x1.fep127) takes the truncated first term instead, which stays finite and leaves an exact
// 16-bit remainder.
__device__ __forceinline__ void split3_bf16(float f, uint16_t &x0, uint16_t &x1, uint16_t &x2) {
  x0 = f32_to_bf16_rne(f);
  x1 = 0;
  x2 = 0;
  if (isfinite(f)) {
    if ((x0 & 0x7f80u) == 0x7f80u) x0 = (uint16_t)(__float_as_uint(f) >> 16);
    const float r1 = f - __uint_as_float((uint32_t)x0 << 16);  // exact
    x1 = f32_to_bf16_rne(r1);
    const float r2 = r1 - __uint_as_float((uint32_t)x1 << 16);  // exact
    x2 = f32_to_bf16_rne(r2);
  }
}

}  // namespace stb
