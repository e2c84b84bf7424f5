// Streamed single-token attention (head size 128) and its split merge fused into the o projection's
// prologue (attention_decode.cu).
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace stb {

// Keys per split (a multiple of 8, 32 .. 256) and the grid's split count for a cache capacity.
struct DecodeStreamPlan {
  int kps = 32, smax = 1;
};

// Whether the streamed form covers the shape (head size 128, at most 8 query heads per KV head, and
// STB_DECODE_STREAM not 0).
bool decode_stream_applies(int hd, int nh, int kvh);
DecodeStreamPlan decode_stream_plan(int rows, int kvh, int capacity, int device);
// Floats of split records for `rows` token rows at any plan of this capacity.
size_t decode_stream_part_floats(int rows, int kvh, int capacity);
// 2-D tensor map over a Float32 cache of `rows` rows of 128 values: 32 x 32 boxes, 128-byte swizzle.
CUtensorMap make_kv_map(const float *kv, uint64_t rows);
// The QKV projection's fixup and the split merge done by the attention itself (single-token steps of
// up to 64 rows, 5 to 8 query heads per KV head -- decode_stream_fusable): q, and the newest key's k
// (rotated) and v row (written to the cache), come from the skinny QKV projection's stream-K pieces
// (paired rows: q heads, k heads, v heads, rotary pairs (d, d + 64)), and the last split block of each
// (row, KV head) writes the merged output as the o projection's terms x3 [3][NT][nh x 128].
struct DecodeStreamFused {
  const float *part = nullptr;  // QKV pieces (SkinnyParts fields)
  int kbs = 0;
  long long T = 0;
  int G = 0, pmax = 0, M = 0;
  const double2 *rope = nullptr;  // [positions][64] (cos, sin) in double
  int *counter = nullptr;         // [rows][kvh] split arrivals, zero between launches
  uint16_t *x3 = nullptr;         // merged output as the o projection's terms
  int NT = 0;
};
bool decode_stream_fusable(int nh, int kvh);
// Split records of every (split, KV head, row) into `part`; krow0 is the map row of this layer's K
// cache (kc), vc the layer's V cache.  With fused (DecodeStreamFused) the QKV fixup and the merge are
// done here and no merge launch follows.
void launch_decode_attention_stream(const CUtensorMap &kmap, long long krow0, const float *q, int ldq, float *kc,
                                    float *vc, int rows, int count, int nh, int kvh, int capacity, const int *posd,
                                    int pos0, const DecodeStreamPlan &plan, float *part, bool pdl, cudaStream_t st,
                                    int device, int *err, const DecodeStreamFused *fused = nullptr);
// Merged attention output of `rows` token rows: as x3 [3][NT][nh x 128] BF16 terms (out null) or as
// Float32 rows of stride ldo (out set).
void launch_attention_merge_split(const float *part, const DecodeStreamPlan &plan, const int *posd, int pos0,
                                  int rows, int count, int nh, int kvh, int NT, uint16_t *x3, float *out, int ldo,
                                  cudaStream_t st);

}  // namespace stb
