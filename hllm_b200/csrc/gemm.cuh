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
//               tile segments to its own slots, and the kernel that consumes
//               the result adds the slots of each element in CTA order
//               (gemm_slot_sum) -- a fixed order, so results do not depend on
//               timing.  No CTA waits on another.
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

// Where a stream-K GEMM left its result: the consumer sums, for element
// (n, m) of accumulator `acc`, the slots of the CTAs that covered its tile, in
// CTA order.  Which CTAs those are, and which of each CTA's slots holds the
// tile, follow from the plan (units dealt U*c/G .. U*(c+1)/G to CTA c), so no
// index is stored: the consumer issues all slot loads at once.
constexpr int kGemmMaxSegsPerTile = 16;
constexpr int kGemmMaxStreamKTiles = 512;
struct GemmSlots {
  const float* slots;   // [grid * 3][pair][bn][128]
  long long units;      // tiles x K blocks
  int grid, kb_count;
  int bn, n_tiles, pair, m;
};

GemmPlan gemm_plan(const GemmWeight& w, int n, int sm_count, int bn_override = 0,
                   int grid_override = 0);
// Floats of slot storage a stream-K plan needs (0 for direct plans).
size_t gemm_slot_floats(const GemmPlan& plan, int pair);
size_t gemm_max_slot_floats(int sm_count);

bool gemm_make_weight(GemmWeight* w, const void* base, int rows_total, int m, int k_pad, int pair,
                      int second_row);
bool gemm_make_input(GemmInput* x, const void* base, int rows_cap, int k_pad, int row_stride);

// Runs the plan.  Direct plans apply `epilogue` into out/ldo; stream-K plans
// write `slots` and fill *result for the consumer.
cudaError_t gemm_launch(const GemmWeight& w, const GemmInput& x, int n, const GemmPlan& plan,
                        int epilogue, void* out, int ldo, float* slots, GemmSlots* result,
                        uint32_t* status, cudaStream_t stream);

// Generic consumer: out = epilogue(sum of slots) for every (n < rows, m).
cudaError_t gemm_finish_launch(const GemmSlots& s, int rows, int epilogue, void* out, int ldo,
                               cudaStream_t stream);

// ---------------------------------------------------------------- device side
__host__ __device__ inline long long gemm_unit_begin(long long units, int grid, int c) {
  return units * c / grid;
}

#ifdef __CUDACC__
// CTAs [c0, c1] that covered `tile`: c covers unit u iff U*c/G <= u < U*(c+1)/G.
// The plan keeps U*G below 2^31, so 32-bit arithmetic is exact.
__device__ __forceinline__ int2 gemm_tile_ctas(const GemmSlots& s, int tile) {
  const unsigned u0 = static_cast<unsigned>(tile) * static_cast<unsigned>(s.kb_count);
  const unsigned g = static_cast<unsigned>(s.grid), u = static_cast<unsigned>(s.units);
  return make_int2(static_cast<int>(((u0 + 1) * g - 1) / u),
                   static_cast<int>(((u0 + s.kb_count) * g - 1) / u));
}
// Slot of the first CTA c0 of `tile` (c0's units may start in an earlier
// tile).  Every later CTA of the tile starts inside it, so its slot is c * 3.
__device__ __forceinline__ int gemm_first_slot(const GemmSlots& s, int c0, int tile) {
  const unsigned begin = static_cast<unsigned>(s.units) * static_cast<unsigned>(c0) /
                         static_cast<unsigned>(s.grid);
  return c0 * kGemmSlotsPerCta + (tile - static_cast<int>(begin / static_cast<unsigned>(s.kb_count)));
}

// Sum of the slots holding element (n, m) of accumulator `acc`, in CTA order.
__device__ inline float gemm_slot_sum(const GemmSlots& s, int n, int m, int acc) {
  const int tile = (m >> 7) * s.n_tiles + n / s.bn;
  const int2 cs = gemm_tile_ctas(s, tile);
  const size_t within = static_cast<size_t>(acc) * s.bn * 128 +
                        static_cast<size_t>(n % s.bn) * 128 + (m & 127);
  const size_t slot_floats = static_cast<size_t>(s.pair) * s.bn * 128;
  float sum = __ldcg(s.slots + static_cast<size_t>(gemm_first_slot(s, cs.x, tile)) * slot_floats + within);
  for (int c = cs.x + 1; c <= cs.y; ++c)
    sum += __ldcg(s.slots + static_cast<size_t>(c) * kGemmSlotsPerCta * slot_floats + within);
  return sum;
}

// The same sum for four consecutive features m..m+3 (m % 4 == 0, one tile):
// slot loads go out CHUNK at a time (four registers each, so a consumer picks
// CHUNK against its occupancy) and are added in CTA order.
template <int CHUNK = 4>
__device__ inline float4 gemm_slot_sum4(const GemmSlots& s, int n, int m, int acc) {
  const int tile = (m >> 7) * s.n_tiles + n / s.bn;
  const int2 cs = gemm_tile_ctas(s, tile);
  const size_t within = static_cast<size_t>(acc) * s.bn * 128 +
                        static_cast<size_t>(n % s.bn) * 128 + (m & 127);
  const size_t slot_floats = static_cast<size_t>(s.pair) * s.bn * 128;
  const float* base = s.slots + within;
  const int first = gemm_first_slot(s, cs.x, tile);
  float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int c0 = cs.x; c0 <= cs.y; c0 += CHUNK) {
    float4 v[CHUNK];
#pragma unroll
    for (int j = 0; j < CHUNK; ++j) {
      const int c = c0 + j;
      const int slot = c == cs.x ? first : c * kGemmSlotsPerCta;
      v[j] = c <= cs.y ? __ldcg(reinterpret_cast<const float4*>(
                             base + static_cast<size_t>(slot) * slot_floats))
                       : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int j = 0; j < CHUNK; ++j) {
      if (c0 + j <= cs.y) {
        sum.x += v[j].x;
        sum.y += v[j].y;
        sum.z += v[j].z;
        sum.w += v[j].w;
      }
    }
  }
  return sum;
}
#endif

}  // namespace hb
