// gemm.cuh -- host interface of the tcgen05 projection GEMM.
//
// Y[n][m] = sum_k X[n][k] * W[m][k]  (the reference's `linear`,
// cpp/src/cpu/tensor.cpp:47-62: W row-major [out, in], F32 accumulate), run as
// D = W_tile * X_tile^T on the 5th-generation tensor cores: the 128 weight
// rows of a tile are the MMA's M dimension and the tokens are its N dimension,
// so one kernel serves GEMV-shaped decode (N = 16..64) and prefill chunks
// (N up to 256 per tile) while streaming each weight byte once.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace hb {

enum GemmEpilogue : int {
  kEpiStoreF32 = 0,   // out f32 [N][ldo] = acc
  kEpiStoreF16 = 1,   // out f16 [N][ldo] = acc
  kEpiResidual = 2,   // out f32 [N][ldo] += acc            (o_proj, down_proj)
  kEpiSwiGLU = 3,     // out f16 [N][ldo] = silu(acc0)*acc1 (gate/up pair)
};

constexpr int kGemmBlockK = 64;                 // one 128-byte swizzle atom of F16
constexpr int kGemmBlockM = 128;
constexpr int kGemmNumBn = 5;
constexpr int kGemmBn[kGemmNumBn] = {16, 32, 64, 128, 256};

// A weight operand: [rows_total][k_pad] F16, k_pad a multiple of 64.  With
// pair == 2 the matrix holds two row blocks (gate then up) of `m` rows each,
// the second starting at row `second_row`; one tile reads both.
struct GemmWeight {
  CUtensorMap map;
  const void* base;
  int m;            // output features
  int k_pad;        // padded inner dimension
  int pair;         // 1 or 2
  int second_row;   // row offset of the second block (pair == 2)
};

// A token operand: [rows_cap][k_pad] F16 activations, one map per tile width.
struct GemmInput {
  CUtensorMap maps[kGemmNumBn];
  const void* base;
  int rows_cap;
  int k_pad;
};

// Scratch shared by every GEMM on one stream: split-K partial tiles and one
// arrival counter per output tile.  Counters must start at zero; the kernel
// returns each one it uses to zero.
struct GemmScratch {
  float* partials;
  size_t partial_floats;
  unsigned* counters;
  size_t counter_count;
  uint32_t* status;
  int sm_count;
};

bool gemm_make_weight(GemmWeight* w, const void* base, int rows_total, int m, int k_pad, int pair,
                      int second_row);
bool gemm_make_input(GemmInput* x, const void* base, int rows_cap, int k_pad, int row_stride);
// Partial-tile floats the scratch needs for any call with these limits.
size_t gemm_partial_floats(int sm_count);
size_t gemm_counter_count(int max_m, int max_n);

// Launches Y = X W^T for the first n rows of X.  `grid_override` > 0 fixes
// the number of CTAs (tests); 0 picks one per SM.  Returns cudaSuccess or the
// launch error; cudaErrorInvalidValue for unsupported shapes.
cudaError_t gemm_run(const GemmWeight& w, const GemmInput& x, int n, int epilogue, void* out,
                     int ldo, const GemmScratch& scratch, cudaStream_t stream,
                     int bn_override = 0, int grid_override = 0);

}  // namespace hb
