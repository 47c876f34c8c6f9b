// gemm.cuh -- host interface of the tcgen05 projection GEMM.
//
// Y[n][m] = sum_k X[n][k] * W[m][k]  (the reference's `linear`,
// cpp/src/cpu/tensor.cpp:47-62: W row-major [out, in], F32 accumulate), run as
// D = W_tile * X_tile^T on the 5th-generation tensor cores: the 128 weight
// rows of a tile are the MMA's M dimension and the tokens are its N dimension,
// so one kernel serves GEMV-shaped decode (N = 16..64) and prefill chunks
// (N up to 256 per tile) while streaming each weight byte once.
//
// Two work splits:
//   direct   -- (at least two tiles per SM) each CTA owns whole tiles and
//               applies the epilogue itself;
//   stream-K -- (fewer tiles) the tiles' K blocks are dealt out evenly to one
//               CTA per SM; each CTA writes the F32 sums of its (at most three)
//               tile segments to its own slots and counts itself in at each
//               tile's counter.  Once a tile's CTAs have all counted in (they
//               are all resident: one CTA per SM), each adds its share of the
//               tile's columns over the tile's slots in CTA order -- a fixed
//               order, so results do not depend on timing -- and applies the
//               epilogue.  Waits are bounded.
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
constexpr int kGemmSlotsPerCta = 3;

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

struct GemmPlan {
  int bn_index = 0, bn = 16;
  int m_tiles = 0, n_tiles = 0, kb_count = 0;
  long long tiles = 0, units = 0;
  int grid = 0;
  bool stream_k = false;
};

// Stream-K bounds: segments per tile (the plan keeps each tile's CTAs below
// this) and tiles per plan (more tiles than this always run direct).
constexpr int kGemmMaxSegsPerTile = 16;
constexpr int kGemmMaxStreamKTiles = 512;
// Ints of per-tile counters (arrivals, departures) a stream-K launch needs
// (zero before the first launch; every launch leaves them zero).
constexpr size_t kGemmCounterInts = 2 * kGemmMaxStreamKTiles;

GemmPlan gemm_plan(const GemmWeight& w, int n, int sm_count, int bn_override = 0,
                   int grid_override = 0);
// Floats of slot storage a stream-K plan needs (0 for direct plans).
size_t gemm_slot_floats(const GemmPlan& plan, int pair);
size_t gemm_max_slot_floats(int sm_count);

bool gemm_make_weight(GemmWeight* w, const void* base, int rows_total, int m, int k_pad, int pair,
                      int second_row);
bool gemm_make_input(GemmInput* x, const void* base, int rows_cap, int k_pad, int row_stride);

// Runs the plan: out = epilogue(X W^T).  Stream-K plans also use `slots`
// (gemm_slot_floats of the plan) and `tile_counters` (kGemmCounterInts,
// zero-initialised).
cudaError_t gemm_launch(const GemmWeight& w, const GemmInput& x, int n, const GemmPlan& plan,
                        int epilogue, void* out, int ldo, float* slots, int* tile_counters,
                        uint32_t* status, cudaStream_t stream);

__host__ __device__ inline long long gemm_unit_begin(long long units, int grid, int c) {
  return units * c / grid;
}

}  // namespace hb
