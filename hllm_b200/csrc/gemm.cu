// gemm.cu -- tcgen05 / TMEM projection GEMM (direct and stream-K work splits).
//
// Reference op: `linear` (cpp/src/cpu/tensor.cpp:47-62) as used for the q/k/v,
// o, gate/up, down and LM-head projections (cpp/src/cpu/llama.cpp:242-288);
// the reference CUDA worker issues these as cuBLAS GEMMs
// (cpp/src/cuda/stage.cpp:306-338, 415-419).
//
// Per CTA (192 threads, one CTA per SM):
//   warp 4: TMA producer -- 128B-swizzled weight tiles (L2 evict-first) and
//           token tiles (evict-last) into a STAGES-deep shared-memory ring;
//   warp 5: TMEM allocation and the single-thread tcgen05.mma issue loop into
//           double-buffered TMEM accumulators (when they fit 512 columns);
//   warps 0-3: epilogue, one TMEM lane (= one output feature) per thread.
// Work: a unit is one 64-wide K block of one output tile (128 weight rows x
// BN tokens), tiles token-tile-fastest.  Direct plans give each CTA whole
// tiles (c, c + G, ...) and apply the epilogue; stream-K plans give CTA c the
// units [U*c/G, U*(c+1)/G) and store each segment's F32 sums in the CTA's slot
// for that tile (see gemm.cuh).
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "gemm.cuh"

namespace hb {
namespace {

struct GemmParams {
  int m;             // output features
  int n;             // tokens
  int kb_count;      // K blocks
  int n_tiles;
  long long tiles;
  long long units;   // tiles * kb_count
  int stream_k;
  int second_row;
  int epilogue;
  void* out;
  int ldo;
  float* slots;
  uint32_t* status;
};

__host__ __device__ constexpr uint32_t pow2_at_least(uint32_t v) {
  uint32_t p = 32;
  while (p < v) p <<= 1;
  return p;
}

template <int BN, int NA>
struct GemmShape {
  static constexpr uint32_t kABytes = kGemmBlockM * kGemmBlockK * 2;  // 16 KB
  static constexpr uint32_t kBBytes = BN * kGemmBlockK * 2;
  static constexpr uint32_t kStageBytes = NA * kABytes + kBBytes;
  static constexpr int kStages = (200 * 1024) / kStageBytes < 8 ? (200 * 1024) / kStageBytes : 8;
  static constexpr int kAccBufs = (2 * NA * BN <= 512) ? 2 : 1;
  static constexpr uint32_t kTmemCols = pow2_at_least(kAccBufs * NA * BN);
  static constexpr uint32_t kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + 256;
};

__host__ __device__ __forceinline__ long long min_ll(long long a, long long b) {
  return a < b ? a : b;
}

// Segment j of this CTA's work: tile and K-block range.  Returns false past
// the last segment.
struct Segment {
  int tile, kb0, kb1;
  long long next;  // stream-K: first unit after this segment
};
__device__ __forceinline__ bool next_segment(const GemmParams& p, long long& cursor, long long end,
                                             int j, Segment& s) {
  if (!p.stream_k) {
    const long long tile = blockIdx.x + static_cast<long long>(j) * gridDim.x;
    if (tile >= p.tiles) return false;
    s.tile = static_cast<int>(tile);
    s.kb0 = 0;
    s.kb1 = p.kb_count;
    return true;
  }
  if (cursor >= end) return false;
  s.tile = static_cast<int>(cursor / p.kb_count);
  s.kb0 = static_cast<int>(cursor % p.kb_count);
  s.kb1 = static_cast<int>(min_ll(p.kb_count, s.kb0 + (end - cursor)));
  cursor += s.kb1 - s.kb0;
  return true;
}

__device__ __forceinline__ void apply_epilogue(const GemmParams& p, int n, int m, float a0,
                                               float a1) {
  const size_t idx = static_cast<size_t>(n) * p.ldo + m;
  switch (p.epilogue) {
    case kEpiStoreF32:
      static_cast<float*>(p.out)[idx] = a0;
      break;
    case kEpiStoreF16:
      static_cast<__half*>(p.out)[idx] = __float2half_rn(a0);
      break;
    case kEpiResidual:
      static_cast<float*>(p.out)[idx] += a0;
      break;
    default: {  // kEpiSwiGLU: (g / (1 + exp(-g))) * u, cpp/src/cpu/llama.cpp:274-280
      const float s = a0 / (1.0f + expf(-a0));
      static_cast<__half*>(p.out)[idx] = __float2half_rn(s * a1);
    }
  }
}

template <int BN, int NA>
__global__ void __launch_bounds__(192, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap map_a,
                   const __grid_constant__ CUtensorMap map_b, const GemmParams p) {
  using S = GemmShape<BN, NA>;
  constexpr int STAGES = S::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * S::kStageBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
    }
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, S::kTmemCols);
    tmem_relinquish();
  }
  if (warp == 4 && lane == 0) {
    prefetch_tensormap(&map_a);
    prefetch_tensormap(&map_b);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int grid = static_cast<int>(gridDim.x);
  const long long ub = p.stream_k ? gemm_unit_begin(p.units, grid, blockIdx.x) : 0;
  const long long ue = p.stream_k ? gemm_unit_begin(p.units, grid, blockIdx.x + 1) : 0;

  if (warp == 4) {
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      auto load_weights = [&](uint8_t* st, uint64_t* bar, int kb, int m_tile) {
        tma_load_2d_hint(st, &map_a, bar, kb * kGemmBlockK, m_tile * kGemmBlockM, pol_w);
        if (NA == 2)
          tma_load_2d_hint(st + S::kABytes, &map_a, bar, kb * kGemmBlockK,
                           p.second_row + m_tile * kGemmBlockM, pol_w);
      };
      // The weight tiles of the first STAGES K blocks go out before the wait
      // for the previous kernel: weights are fixed, only the token tiles are
      // that kernel's output.  (First use of each stage: no empty-wait.)
      uint32_t pre = 0;
      {
        long long cursor = ub;
        Segment sg;
        for (int j = 0; pre < STAGES && next_segment(p, cursor, ue, j, sg); ++j)
          for (int kb = sg.kb0; kb < sg.kb1 && pre < STAGES; ++kb, ++pre) {
            mbar_arrive_expect_tx(&full[pre], S::kStageBytes);
            load_weights(smem + pre * S::kStageBytes, &full[pre], kb, sg.tile / p.n_tiles);
          }
      }
      griddep_enter();
      uint32_t it = 0;
      long long cursor = ub;
      Segment sg;
      for (int j = 0; next_segment(p, cursor, ue, j, sg); ++j) {
        const int n_tile = sg.tile % p.n_tiles, m_tile = sg.tile / p.n_tiles;
        for (int kb = sg.kb0; kb < sg.kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          uint8_t* st = smem + s * S::kStageBytes;
          if (it >= pre) {
            if (!mbar_wait(&empty[s], ph ^ 1u, p.status)) goto producer_done;
            mbar_arrive_expect_tx(&full[s], S::kStageBytes);
            load_weights(st, &full[s], kb, m_tile);
          }
          tma_load_2d_hint(st + NA * S::kABytes, &map_b, &full[s], kb * kGemmBlockK,
                           n_tile * BN, pol_x);
        }
      }
    producer_done:;
    }
  } else if (warp == 5) {
    if (lane == 0) {
      uint32_t it = 0;
      long long cursor = ub;
      Segment sg;
      for (int j = 0; next_segment(p, cursor, ue, j, sg); ++j) {
        // The last token tile of a ragged N multiplies only its valid
        // columns, rounded up to the MMA's 16-column step.
        const int nv = min(BN, p.n - (sg.tile % p.n_tiles) * BN);
        const uint32_t idesc = umma_idesc(kGemmBlockM, min(BN, (nv + 15) & ~15), 0);
        const int b = j % S::kAccBufs;
        const uint32_t bph = (j / S::kAccBufs) & 1u;
        if (!mbar_wait(&tempty[b], bph ^ 1u, p.status)) goto mma_done;
        tc_fence_after();
        const uint32_t d = tmem_base + b * NA * BN;
        for (int kb = sg.kb0; kb < sg.kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!mbar_wait(&full[s], ph, p.status)) goto mma_done;
          tc_fence_after();
          const uint32_t a0 = smem_u32(smem + s * S::kStageBytes);
          const uint32_t b0 = a0 + NA * S::kABytes;
#pragma unroll
          for (int k = 0; k < kGemmBlockK / 16; ++k) {
            const uint32_t acc = (kb > sg.kb0 || k > 0) ? 1u : 0u;
            const uint64_t bd = sw128_desc(b0 + k * 32);
            umma_f16(d, sw128_desc(a0 + k * 32), bd, idesc, acc);
            if (NA == 2) umma_f16(d + BN, sw128_desc(a0 + S::kABytes + k * 32), bd, idesc, acc);
          }
          umma_commit(&empty[s]);
        }
        umma_commit(&tfull[b]);
      }
    mma_done:;
    }
  } else {
    // Epilogue: thread t owns TMEM lane t = output feature m_tile*128 + t.
    griddep_enter();  // it reads (residual) and writes buffers of earlier kernels
    const int t = threadIdx.x;
    long long cursor = ub;
    const int first_tile = static_cast<int>(ub / (p.kb_count > 0 ? p.kb_count : 1));
    Segment sg;
    for (int j = 0; next_segment(p, cursor, ue, j, sg); ++j) {
      const int n_tile = sg.tile % p.n_tiles, m_tile = sg.tile / p.n_tiles;
      const int b = j % S::kAccBufs;
      const uint32_t bph = (j / S::kAccBufs) & 1u;
      if (!mbar_wait(&tfull[b], bph, p.status)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(warp * 32) << 16) + b * NA * BN;
      const int m = m_tile * kGemmBlockM + t;
      const int n0 = n_tile * BN;
      const int nvalid = min(BN, p.n - n0);
      float* slot = nullptr;
      if (p.stream_k) {
        const int slot_id = static_cast<int>(blockIdx.x) * kGemmSlotsPerCta + (sg.tile - first_tile);
        slot = p.slots + static_cast<size_t>(slot_id) * NA * BN * 128;
      }
      for (int c = 0; c < BN / 16; ++c) {
        if (c * 16 >= nvalid) break;
        float v0[16], v1[16];
        tmem_ld16(taddr + c * 16, v0);
        if (NA == 2) tmem_ld16(taddr + BN + c * 16, v1);
        if (slot) {
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) {
            slot[(c * 16 + jj) * 128 + t] = v0[jj];
            if (NA == 2) slot[(BN + c * 16 + jj) * 128 + t] = v1[jj];
          }
        } else {
#pragma unroll
          for (int jj = 0; jj < 16; ++jj)
            if (c * 16 + jj < nvalid && m < p.m)
              apply_epilogue(p, n0 + c * 16 + jj, m, v0[jj], NA == 2 ? v1[jj] : 0.f);
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[b]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 5) tmem_dealloc(tmem_base, S::kTmemCols);
}

// ---------------------------------------------------------------- generic consumer
__global__ void gemm_finish_kernel(const GemmSlots s, int rows, int epilogue, void* out, int ldo) {
  griddep_enter();
  const int n = blockIdx.y;
  if (n >= rows) return;
  for (int m = blockIdx.x * blockDim.x + threadIdx.x; m < s.m; m += gridDim.x * blockDim.x) {
    const float a0 = gemm_slot_sum(s, n, m, 0);
    const size_t idx = static_cast<size_t>(n) * ldo + m;
    switch (epilogue) {
      case kEpiStoreF32: static_cast<float*>(out)[idx] = a0; break;
      case kEpiStoreF16: static_cast<__half*>(out)[idx] = __float2half_rn(a0); break;
      case kEpiResidual: static_cast<float*>(out)[idx] += a0; break;
      default: {
        const float a1 = gemm_slot_sum(s, n, m, 1);
        static_cast<__half*>(out)[idx] = __float2half_rn(a0 / (1.0f + expf(-a0)) * a1);
      }
    }
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

bool make_map(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows,
              uint64_t row_stride_elems, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {row_stride_elems * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kGemmBlockK), box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, int NA>
cudaError_t launch(const GemmWeight& w, const GemmInput& x, int bn_index, const GemmParams& p,
                   int grid, cudaStream_t stream) {
  using S = GemmShape<BN, NA>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<BN, NA>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(S::kSmemBytes));
    if (e != cudaSuccess) return e;
    configured = true;
  }
  return launch_dependent(gemm_tc_kernel<BN, NA>, dim3(grid), dim3(192), S::kSmemBytes, stream,
                          w.map, x.maps[bn_index], p);
}

}  // namespace

bool gemm_make_weight(GemmWeight* w, const void* base, int rows_total, int m, int k_pad, int pair,
                      int second_row) {
  if (k_pad % kGemmBlockK != 0 || (pair != 1 && pair != 2)) return false;
  w->base = base;
  w->m = m;
  w->k_pad = k_pad;
  w->pair = pair;
  w->second_row = second_row;
  return make_map(&w->map, base, k_pad, rows_total, k_pad, kGemmBlockM);
}

bool gemm_make_input(GemmInput* x, const void* base, int rows_cap, int k_pad, int row_stride) {
  if (k_pad % kGemmBlockK != 0 || row_stride < k_pad) return false;
  x->base = base;
  x->rows_cap = rows_cap;
  x->k_pad = k_pad;
  for (int i = 0; i < kGemmNumBn; ++i)
    if (!make_map(&x->maps[i], base, k_pad, rows_cap, row_stride, kGemmBn[i])) return false;
  return true;
}

GemmPlan gemm_plan(const GemmWeight& w, int n, int sm_count, int bn_override, int grid_override) {
  GemmPlan pl;
  int bi = 0;
  if (bn_override) {
    bi = -1;
    for (int i = 0; i < kGemmNumBn; ++i)
      if (kGemmBn[i] == bn_override) bi = i;
    if (bi < 0) bi = 0;
  } else {
    while (bi + 1 < kGemmNumBn && kGemmBn[bi] < n) ++bi;
  }
  if (w.pair == 2 && kGemmBn[bi] > 128) bi = 3;  // 2 accumulators x 128 x 2 buffers
  pl.bn_index = bi;
  pl.bn = kGemmBn[bi];
  pl.kb_count = w.k_pad / kGemmBlockK;
  pl.n_tiles = (n + pl.bn - 1) / pl.bn;
  pl.m_tiles = (w.m + kGemmBlockM - 1) / kGemmBlockM;
  pl.tiles = static_cast<long long>(pl.m_tiles) * pl.n_tiles;
  pl.units = pl.tiles * pl.kb_count;
  long long grid = grid_override > 0 ? grid_override : sm_count;
  // at least 4 K blocks per CTA when the units are split
  if (grid_override <= 0) grid = std::min<long long>(grid, std::max<long long>(1, pl.units / 4));
  grid = std::max<long long>(1, std::min<long long>(grid, pl.units));
  pl.stream_k = pl.tiles < 2 * grid;
  if (pl.stream_k) {
    // A tile is split over at most kGemmMaxSegsPerTile CTAs (bounding the
    // consumers' slot loads), and stream-K is kept to plans of few tiles.
    grid = std::min<long long>(grid, pl.tiles * (kGemmMaxSegsPerTile - 2));
    if (pl.tiles > kGemmMaxStreamKTiles) pl.stream_k = false;
    // the consumers locate slots with 32-bit arithmetic on units x grid
    if (pl.units * (grid + 1) >= (1LL << 31)) pl.stream_k = false;
  }
  if (!pl.stream_k) grid = std::min<long long>(grid, pl.tiles);
  pl.grid = static_cast<int>(grid);
  return pl;
}

size_t gemm_slot_floats(const GemmPlan& plan, int pair) {
  if (!plan.stream_k) return 0;
  return static_cast<size_t>(plan.grid) * kGemmSlotsPerCta * pair * plan.bn * 128;
}

size_t gemm_max_slot_floats(int sm_count) {
  // pair x bn is at most 2 x 128 or 1 x 256
  return static_cast<size_t>(sm_count) * kGemmSlotsPerCta * 256 * 128;
}

cudaError_t gemm_launch(const GemmWeight& w, const GemmInput& x, int n, const GemmPlan& pl,
                        int epilogue, void* out, int ldo, float* slots, GemmSlots* result,
                        uint32_t* status, cudaStream_t stream) {
  if (n <= 0 || n > x.rows_cap || w.k_pad != x.k_pad) return cudaErrorInvalidValue;
  if (pl.stream_k && (!slots || !result)) return cudaErrorInvalidValue;
  if (!pl.stream_k && (epilogue == kEpiSwiGLU) != (w.pair == 2)) return cudaErrorInvalidValue;
  GemmParams p{};
  p.m = w.m;
  p.n = n;
  p.kb_count = pl.kb_count;
  p.n_tiles = pl.n_tiles;
  p.tiles = pl.tiles;
  p.units = pl.units;
  p.stream_k = pl.stream_k ? 1 : 0;
  p.second_row = w.second_row;
  p.epilogue = epilogue;
  p.out = out;
  p.ldo = ldo;
  p.slots = slots;
  p.status = status;
  if (pl.stream_k) {
    result->slots = slots;
    result->units = pl.units;
    result->grid = pl.grid;
    result->kb_count = pl.kb_count;
    result->bn = pl.bn;
    result->n_tiles = pl.n_tiles;
    result->pair = w.pair;
    result->m = w.m;
  }
  const int g = pl.grid;
  const int bi = pl.bn_index;
  if (w.pair == 1) {
    switch (pl.bn) {
      case 16: return launch<16, 1>(w, x, bi, p, g, stream);
      case 32: return launch<32, 1>(w, x, bi, p, g, stream);
      case 64: return launch<64, 1>(w, x, bi, p, g, stream);
      case 128: return launch<128, 1>(w, x, bi, p, g, stream);
      default: return launch<256, 1>(w, x, bi, p, g, stream);
    }
  }
  switch (pl.bn) {
    case 16: return launch<16, 2>(w, x, bi, p, g, stream);
    case 32: return launch<32, 2>(w, x, bi, p, g, stream);
    case 64: return launch<64, 2>(w, x, bi, p, g, stream);
    default: return launch<128, 2>(w, x, bi, p, g, stream);
  }
}

cudaError_t gemm_finish_launch(const GemmSlots& s, int rows, int epilogue, void* out, int ldo,
                               cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  const dim3 grid(static_cast<unsigned>((s.m + 255) / 256), static_cast<unsigned>(rows));
  return launch_dependent(gemm_finish_kernel, grid, dim3(256), 0, stream, s, rows, epilogue, out,
                          ldo);
}

}  // namespace hb
