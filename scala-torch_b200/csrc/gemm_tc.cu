// Prefill Linear on the tcgen05 tensor cores (placeholder until the TMA/TMEM kernel lands).
#include "common.cuh"

using namespace stb;

extern "C" {

int stb_linear_prefill(stb_session *s, uint64_t x, uint64_t w, int w_dtype, uint64_t bias, uint64_t y, int M, int N,
                       int K) {
  return guarded([&] {
    enter(s);
    (void)x; (void)w; (void)w_dtype; (void)bias; (void)y; (void)M; (void)N; (void)K;
    throw Error(STB_ERR_UNSUPPORTED, "tensor-core prefill Linear is not built yet");
  });
}

}  // extern "C"
