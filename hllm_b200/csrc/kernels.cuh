// kernels.cuh -- host launchers for the stage executor's non-GEMM kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "gemm.cuh"

namespace hb {

constexpr int kBlockTokens = 16;  // paged-KV block size (tokens)

// Per-step packed batch, device-resident.  Filled by pack_launch from the
// uploaded row descriptors (row_slot, row_first, row_count).
struct StepTensors {
  const int32_t* row_slot;
  const int32_t* row_first;
  const int32_t* row_count;
  int32_t* cu_seqlens;    // [R+1]
  int32_t* positions;     // [T]
  int32_t* slot_mapping;  // [T]
  int32_t* token_row;     // [T]
  int32_t* seq_lens;      // [R]
  int32_t* block_tables;  // [R][max_blocks]
  int32_t* cu_splits;     // [R+1] decode rows: ceil(ctx / split_tokens) context splits
  int32_t* cu_qtiles;     // [R+1] prefill rows: ceil(count / qtile_tokens) query tiles
  int rows;
  int tokens;
  int max_blocks;
  int split_tokens;
  int qtile_tokens;
};

// Ragged packer (cu_seqlens, positions, slot mapping, token->row map,
// sequence lengths, block tables, attention work prefixes) from the
// per-slot block lists [slots][max_blocks].  A row with one token is a decode
// row; a row with more is a prefill chunk.
cudaError_t pack_launch(const StepTensors& s, const int32_t* slot_blocks, uint32_t* status,
                        cudaStream_t stream);

// hidden[t][:] = F32(embedding[ids[t]][:]).
cudaError_t embed_launch(const int32_t* ids, int tokens, const __half* embedding, int vocab,
                         int hidden, int ld_embedding, float* out, uint32_t* status,
                         cudaStream_t stream);

// hidden[t][:] = F32(boundary[t][:]); non-finite input sets kDevNonFinite.
cudaError_t boundary_in_launch(const __half* in, int tokens, int hidden, float* out,
                               uint32_t* status, cudaStream_t stream);

// out[t][:] = F16(hidden[t][:]) (round to nearest even); a value that is not a
// finite F16 sets kDevNonFinite.
cudaError_t boundary_out_launch(const float* hidden, int tokens, int width, __half* out,
                                uint32_t* status, cudaStream_t stream);

// out[r][c] = F16(x[r][c] * inv_rms(x[r]) * w[c]) over `rows` rows; when
// `row_index` is non-null, row r reads x[row_index[r]] (last token of a row).
cudaError_t rmsnorm_launch(const float* x, int rows, int width, const float* w, float eps,
                           __half* out, int ld_out, const int32_t* row_index,
                           cudaStream_t stream);

// Per-token epilogue of the fused QKV projection: Qwen3 per-head q/k RMSNorm
// (optional), RoPE (half rotation) at the token's position, q to `q_out`
// [T][Hq*d] F16, k/v scattered to the paged cache at slot_mapping[t].
struct QkvPostArgs {
  const float* qkv;       // [T][ (Hq + 2 Hkv) d ] when the projection ran direct
  GemmSlots slots;        // its stream-K slots otherwise
  int from_slots;
  int tokens, hq, hkv, dim;
  const int32_t* positions;
  const int32_t* slot_mapping;
  const float* q_norm;    // [d] or null
  const float* k_norm;    // [d] or null
  float eps;
  const float* rope_pow;  // [d/2]: theta^(2i/d), computed on the host like the reference
  const float2* rope_table;  // [positions][d/2] (cos, sin) from the host, or null
  int rope_positions;
  __half* q_out;          // [T][Hq d]
  __half* k_cache;        // [blocks][Hkv][16][d] of this layer
  __half* v_cache;
};
cudaError_t qkv_post_launch(const QkvPostArgs& a, cudaStream_t stream);

// Fused residual add + RMSNorm (cpp/src/cpu/llama.cpp:268-272 and the next
// rms_norm): hidden[t] += the projection's stream-K slots (when `slots` is
// given; a direct projection already added itself), then, when `norm` is
// given, out[t] = F16(hidden[t] * inv_rms(hidden[t]) * norm).
cudaError_t residual_norm_launch(float* hidden, int tokens, int width, const GemmSlots* slots,
                                 const float* norm, float eps, __half* out, int ld_out,
                                 cudaStream_t stream);

// act[t][i] = F16(silu(g) * u) from a gate/up projection's stream-K slots.
cudaError_t swiglu_launch(const GemmSlots& slots, int tokens, __half* act, int ld_act,
                          cudaStream_t stream);

// Row indices of the last token of each sampling row: idx[i] = cu_seqlens[rows[i]+1]-1.
cudaError_t last_token_launch(const int32_t* cu_seqlens, const int32_t* sample_rows, int count,
                              int32_t* idx, cudaStream_t stream);

// Seeded synthetic weights (bit-identical with oracle_synth_*): an F16
// matrix [rows][cols] at row stride ld, or an F32 norm vector.
cudaError_t synth_matrix_launch(uint64_t seed, uint64_t tag, int rows, int cols, int ld,
                                float stddev, __half* out, cudaStream_t stream);
cudaError_t synth_norm_launch(uint64_t seed, uint64_t tag, int n, float spread, float* out,
                              cudaStream_t stream);

}  // namespace hb
