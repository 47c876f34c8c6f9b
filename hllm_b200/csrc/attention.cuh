// attention.cuh -- paged-KV GQA attention launchers.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace hb {

// TMA tensor maps of one layer's attention inputs: the query buffer (tcgen05
// prefill) and the K and V caches (tcgen05 prefill and the balanced decode
// pass), all with the 128-byte swizzle.
struct TcMaps {
  CUtensorMap q;  // [tokens][Hq][d] F16, box 64 dims x group heads x 128/group tokens
  CUtensorMap k;  // [blocks * Hkv * 16][d] F16, box 64 dims x one 16-key page
  CUtensorMap v;
};

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
  int decode_ctas;             // balanced decode grid (attn_decode_ctas), head sizes 64/128/256
  float* part_o;               // partial outputs: [splits][Hq][d] (combine path) or
                               // [pieces][Hq/Hkv][d] (balanced path)
  float* part_ml;              // matching running max, denominator pairs
  int* counters;               // [rows][Hkv] balanced decode: each stream's warp range,
                               // written by the decode pass for its merge pass
  int prefill_splits;          // key splits per prefill tile (attn_prefill_splits), >= 1
  float* pre_part;             // [qtiles][Hkv][splits] x 64 rows x (DP + 2): split rows, (m, l)
  int* pre_counters;           // [qtiles][Hkv] zero-initialised; returned to zero after use
  __half* out;                 // [T][ld_out]
  int ld_out;
  uint32_t* status;
};

// Query tokens per prefill tile for a GQA group size (64 query rows per CTA).
int attn_qtile_tokens(int group);

// Decode rows (one new token).  Head sizes 64/128/256: the decode rows' KV
// pages are split evenly over 4 * decode_ctas warps regardless of row
// lengths, each warp streaming its pages by TMA into its own ring; a second
// launch merges the pieces of each (row, kv head) split over several warps
// (split_tokens/cu_splits unused).  Other head sizes: split-K over
// split_tokens-key splits, one CTA per (kv head, split), then a combine pass.
// The balanced pass streams pages through maps.k / maps.v (attn_make_kv_maps).
cudaError_t attn_decode_launch(const AttnArgs& a, const TcMaps& maps, int total_splits,
                               cudaStream_t stream);
int attn_decode_launches(int dim);
bool attn_decode_balanced(int dim);
// CTAs of the balanced decode pass (GQA group size `group` = Hq/Hkv) for
// `pages` = sum over decode rows of
// ceil(ctx / 16) x Hkv: one wave of resident CTAs at most, about 8 pages per
// warp at least; 0 when the head size takes the combine path.
int attn_decode_ctas(int dim, int group, long long pages, int sm_count);
// Floats of part_o + part_ml that the balanced pass needs for `rows` rows.
size_t attn_decode_part_floats(int rows, int hq, int hkv, int dim, int ctas);
// Prefill rows (several new tokens): causal tiles on the tensor cores, each
// tile's keys split over prefill_splits CTAs whose results the last one merges.
constexpr int kPrefillMaxSplits = 4;
cudaError_t attn_prefill_launch(const AttnArgs& a, int total_qtiles, cudaStream_t stream);
// Key splits that keep one wave of resident CTAs busy (1..kPrefillMaxSplits);
// table_bytes = prefill_table_bytes of the launch (max_blocks x 4, rounded to 16).
int attn_prefill_splits(int dim, int hkv, int total_qtiles, int sm_count, size_t table_bytes);
size_t attn_prefill_part_floats(int dim, int hkv, int total_qtiles, int splits);
size_t prefill_table_bytes(const AttnArgs& a);

// Prefill rows on tcgen05 / TMEM (attention_tc.cu) for head sizes 64 and 128
// and GQA groups 1, 2, 4, 8.
bool attn_prefill_tc_supported(int dim, int group);
// The K and V maps only (head sizes 64, 128, 256).
bool attn_make_kv_maps(TcMaps* maps, int hkv, int dim, const void* k_cache, const void* v_cache,
                       long long kv_blocks);
// All three maps (head sizes 64 and 128, groups 1/2/4/8).
bool attn_tc_make_maps(TcMaps* maps, const void* q, long long q_tokens, int hq, int hkv, int dim,
                       const void* k_cache, const void* v_cache, long long kv_blocks);
// Key splits per tile for the tcgen05 kernel (one resident CTA per SM).
int attn_prefill_tc_splits(int hkv, int total_qtiles, int sm_count);
// Same contract as attn_prefill_launch (the same partial-tile workspace and
// counters for split tiles).
cudaError_t attn_prefill_tc_launch(const TcMaps& maps, const AttnArgs& a, int total_qtiles,
                                   cudaStream_t stream);

}  // namespace hb
