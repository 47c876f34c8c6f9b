// attention.cuh -- paged-KV GQA attention launchers.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace hb {

struct AttnArgs {
  const __half* q;             // [T][Hq*d] (normed, RoPE applied)
  const __half* k_cache;       // this layer: [blocks][Hkv][16][d]
  const __half* v_cache;
  const int32_t* row_count;    // [R]
  const int32_t* row_first;    // [R]
  const int32_t* cu_seqlens;   // [R+1]
  const int32_t* seq_lens;     // [R]
  const int32_t* block_tables; // [R][max_blocks]
  const int32_t* cu_splits;    // [R+1] decode rows: ceil(ctx/split_tokens) splits, else 0
  const int32_t* cu_qtiles;    // [R+1] prefill rows: ceil(count/qtile_tokens) tiles, else 0
  int rows, hq, hkv, dim, max_blocks;
  int split_tokens;            // keys per decode split (multiple of 16)
  int qtile_tokens;            // query tokens per prefill tile
  float scale;                 // 1/sqrt(d)
  float* part_o;               // [splits][Hq][d]  unnormalised split outputs
  float* part_ml;              // [splits][Hq][2]  running max, denominator
  int* counters;               // [rows][Hkv] zero-initialised; returned to zero after use
  __half* out;                 // [T][ld_out]
  int ld_out;
  uint32_t* status;
};

// Query tokens per prefill tile for a GQA group size (64 query rows per CTA).
int attn_qtile_tokens(int group);

// Decode rows (one new token): split-K over the context; the splits of a row
// are merged by the last warp to finish (head sizes 64/128/256) or by a
// combine pass (other head sizes).
cudaError_t attn_decode_launch(const AttnArgs& a, int total_splits, cudaStream_t stream);
int attn_decode_launches(int dim);
// Prefill rows (several new tokens): causal tiles on the tensor cores.
cudaError_t attn_prefill_launch(const AttnArgs& a, int total_qtiles, cudaStream_t stream);

}  // namespace hb
