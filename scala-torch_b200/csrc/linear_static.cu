// Allocation-free form of the prefill Linear (stb_linear_prefill_static).
//
// stb_linear_prefill rounds the activations into the session's scratch buffer, which the session
// allocates (and grows) with cudaMalloc.  Some callers cannot allow that: a host framework that
// owns every device allocation through its own allocator or byte budget, or a serving loop that
// forbids device allocation after warm-up.  This entry point uses instead a fixed scratch array
// compiled into the library (a file-scope __device__ array, present on every GPU that loads the
// library until the process exits) and calls no allocating CUDA or library routine.
//
// Limits and sharing:
//   * the rounded activations must fit the array: M * K <= STB_PREFILL_STATIC_MAX_ELEMENTS;
//   * every call uses the same array, so calls that overlap on the GPU (other host threads or
//     streams) race on it; each call finishes its work before returning;
//   * the first call on a device is its set-up: it loads the library's device code on that device
//     (under CUDA's lazy module loading that is where the array, 16 MiB + 256 bytes, and the kernels
//     are placed in device memory) and looks up the array's device address (cudaGetSymbolAddress)
//     with that device current; make that first call during warm-up, before any stream capture.
//     Later calls allocate nothing;
//   * the address is kept per device for the life of the process: a cudaDeviceReset while the
//     library is loaded is not supported (the array is reloaded elsewhere, the kept address dangles).
#include <mutex>

#include "common.cuh"

namespace stb {
void gemm_tc_launch(const void *xh, const void *w, int dtype, const float *bias, float *y, int ldy, int M, int N,
                    int K, int *err, int device, cudaStream_t stream);
void round_activations(const float *x, uint16_t *out, size_t count, int dtype, cudaStream_t stream);
}  // namespace stb

using namespace stb;

namespace {

constexpr uint64_t kMaxElements = 8ull << 20;          // 8,388,608 half activations = 16 MiB
constexpr uint64_t kErrorOffset = kMaxElements * 2;    // then one int for bounded-wait failures
constexpr uint64_t kScratchBytes = kErrorOffset + 256;

static __device__ __align__(256) unsigned char g_prefill_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
void *g_scratch_addr[kMaxDevices] = {};

// Device address of the array on the current device (looked up once per device).
unsigned char *static_scratch(int device) {
  STB_REQUIRE(device >= 0 && device < kMaxDevices, "device index out of range for the static scratch table");
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (!g_scratch_addr[device]) {
    void *ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_prefill_scratch);
    if (e != cudaSuccess || !ptr)
      throw Error(STB_ERR_CUDA, std::string("cudaGetSymbolAddress(static prefill scratch) failed: ") +
                                    cudaGetErrorString(e));
    g_scratch_addr[device] = ptr;
  }
  return (unsigned char *)g_scratch_addr[device];
}

}  // namespace

extern "C" {

int stb_linear_prefill_static(void *stream, uint64_t x, uint64_t w, int w_dtype, uint64_t bias, uint64_t y, int M,
                              int N, int K) {
  return guarded([&] {
    STB_REQUIRE(M >= 0 && N >= 0 && K >= 0, "Linear dimensions must be nonnegative");
    STB_REQUIRE(w_dtype == STB_BF16 || w_dtype == STB_F16, "tensor-core Linear needs BF16 or F16 weights");
    if (M == 0 || N == 0) return;
    STB_REQUIRE(K > 0 && K % 8 == 0, "tensor-core Linear needs K a positive multiple of 8");
    STB_REQUIRE((uint64_t)M * (uint64_t)K <= kMaxElements,
                "M*K = " + std::to_string((uint64_t)M * (uint64_t)K) + " exceeds the static scratch limit of " +
                    std::to_string(kMaxElements) + " activations (16 MiB); use stb_linear_prefill");
    STB_REQUIRE(x && w && y, "null buffer");
    STB_REQUIRE(x % 16 == 0 && w % 16 == 0 && y % 16 == 0, "buffers must be 16-byte aligned");
    int device = 0;
    STB_CUDA(cudaGetDevice(&device));
    unsigned char *scratch = static_scratch(device);
    int *err = (int *)(scratch + kErrorOffset);
    cudaStream_t st = (cudaStream_t)stream;
    // The array keeps the previous call's contents: the error word must start at zero.
    STB_CUDA(cudaMemsetAsync(err, 0, sizeof(int), st));
    round_activations((const float *)x, (uint16_t *)scratch, (size_t)M * K, w_dtype, st);
    gemm_tc_launch(scratch, (const void *)w, w_dtype, (const float *)bias, (float *)y, N, M, N, K, err, device, st);
    // The error word comes back on the same stream, so the one synchronisation below waits for this
    // call's work only (no legacy-stream copy that would also wait for other streams' work).
    int code = 0;
    STB_CUDA(cudaMemcpyAsync(&code, err, sizeof(int), cudaMemcpyDeviceToHost, st));
    STB_CUDA(cudaStreamSynchronize(st));
    if (code) throw Error(STB_ERR_CUDA, "a device-side wait expired (code " + std::to_string(code) + ")");
  });
}

}  // extern "C"
