// Whole-generation decode in one persistent launch for small single-GPU models (batch 1).
//
// Decode of a SmolLM2-sized model is latency-bound: a graph-replayed step is ~150 kernels of a few
// microseconds each, while its weights would stream in ~40 us.  decode_mega_kernel runs every
// decode step of a generation inside one cooperative launch (one block per SM), with grid-wide
// barriers between the data-dependent phases of a layer and L2 prefetches of the next phase's
// weights issued before each barrier.  Per layer:
//   A  RMSNorm (every block, the GEMV's expression) -> q/k/v row pairs of this block -> RoPE,
//      q to qbuf, k/v appended to the cache;
//   B  causal attention split over (query head, key range) blocks (FP32); the block holding a
//      head's first range waits for the head's other splits, merges them and multiplies by that
//      head's slice of the o projection, opart[h][n] = att_h . W_o[n, h*hd : h*hd + hd];
//   C  every block: hidden += sum over heads of opart (head order), post-attention RMSNorm,
//      gate/up row pairs of this block -> act = SiLU(gate) * up;
//   D  down rows of this block: hid[n] = hidden[n] + act . W_down[n].
// After the layers: final RMSNorm, lm_head rows of this block with a greedy candidate key
// (argmax_key) folded into one atomicMax, then block 0 runs the step's finalize (append, EOS,
// token feedback, position advance).  4 barriers per layer + 2 per step.  Each phase's weight slice
// is staged into shared memory by bulk copies issued right after the previous layer's use.
// Opt-in (STB_DECODE_PERSISTENT=1): on the SmolLM2-shaped workload the graph-replayed step is faster.
#pragma once

#include "common.cuh"

namespace stb {

struct MegaLayer {
  const uint16_t *qkv, *o, *gu, *down;  // fused BF16 layouts of the runtime (paired q/k/v, interleaved gate/up)
  const float *in_norm, *post_norm;
};

struct MegaArgs {
  const MegaLayer *layers;  // device array [L]
  int L, H, NH, KV, hd, I, V, capacity;
  double eps;
  const uint16_t *embed, *lm_head;
  const float *final_norm;
  const double2 *rope;
  float *kv;     // [L][2][1][KV][capacity][hd]
  float *qbuf;   // [NH * hd]
  float *opart;  // [NH][H]
  float *act;    // [I]
  float *hid;    // [H]
  float *apart;  // [NH][ceil(capacity / 64)][hd + 2] attention split records (max, sum, partial sums)
  int64_t *tokens;  // [1]
  int *state;       // [0] position, [1] all stopped, [2] stopped, [3] output count
  int64_t *out_ids;
  int out_stride;
  const int64_t *eos;
  int eos_count;
  unsigned long long *best;  // [1]
  unsigned *bar;             // [16 + NH]: [0] barrier count, [16 + h] head h's finished splits (zeroed before each launch)
  int *err;
  int steps;
};

// Whether a model / cache shape has the persistent form (see the conditions in decode_mega.cu).
bool mega_eligible(int H, int NH, int KV, int hd, int I, int V, int L, int capacity, int batch, int tp,
                   int w_dtype, int device);
// Launches the persistent decode (cooperative, one block per SM).  bar must be zero.
void mega_launch(const MegaArgs &a, int device, cudaStream_t st);

}  // namespace stb
