// gemm.cu -- tcgen05 / TMEM projection GEMM with stream-K work split.
//
// Reference op: `linear` (cpp/src/cpu/tensor.cpp:47-62) as used for the q/k/v,
// o, gate/up, down and LM-head projections (cpp/src/cpu/llama.cpp:242-288);
// the reference CUDA worker issues these as cuBLAS GEMMs
// (cpp/src/cuda/stage.cpp:306-338, 415-419).
//
// Design (one CTA per SM, persistent over a contiguous range of work units):
//   * a work unit is one 64-wide K block of one output tile (128 weight rows x
//     BN tokens); units are ordered tile-major, tiles token-tile-fastest, and
//     CTA c takes units [U*c/G, U*(c+1)/G).  Tiles that straddle CTAs leave
//     F32 partial tiles in scratch; the last CTA to finish a tile (arrival
//     counter) sums them in CTA order -- a fixed order, so results do not
//     depend on timing -- and applies the epilogue.  Nothing waits on another
//     CTA.
//   * warp 4: TMA producer (weights with L2 evict-first, tokens evict-last)
//     into a STAGES-deep ring of 128B-swizzled tiles;
//     warp 5: TMEM allocation and the single-thread tcgen05.mma issue loop,
//     double-buffered accumulators when they fit in 512 TMEM columns;
//     warps 0-3: epilogue, one TMEM lane (= one output feature) per thread,
//     fused residual add / SwiGLU / F16 store.
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
  long long units;   // tiles * kb_count
  int second_row;
  int epilogue;
  void* out;
  int ldo;
  float* partials;
  unsigned* counters;
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
  static constexpr int kStages = std::min<int>(8, (200 * 1024) / kStageBytes);
  static constexpr int kAccBufs = (2 * NA * BN <= 512) ? 2 : 1;
  static constexpr uint32_t kTmemCols = pow2_at_least(kAccBufs * NA * BN);
  static constexpr uint32_t kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + 256;
};

__host__ __device__ __forceinline__ long long min_ll(long long a, long long b) { return a < b ? a : b; }

__device__ __forceinline__ long long unit_begin(long long units, int grid, int c) {
  return units * c / grid;
}
// The CTA whose range holds unit u.
__device__ __forceinline__ int cta_of_unit(long long units, int grid, long long u) {
  int c = static_cast<int>((u * grid) / units);
  while (c + 1 < grid && unit_begin(units, grid, c + 1) <= u) ++c;
  while (c > 0 && unit_begin(units, grid, c) > u) --c;
  return c;
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
  volatile int* last_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

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
  const long long ub = unit_begin(p.units, grid, blockIdx.x);
  const long long ue = unit_begin(p.units, grid, blockIdx.x + 1);
  const int KB = p.kb_count;

  if (warp == 4) {
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      uint32_t it = 0;
      for (long long u = ub; u < ue;) {
        const int tile = static_cast<int>(u / KB);
        const int kb0 = static_cast<int>(u % KB);
        const int kb1 = static_cast<int>(min_ll(KB, kb0 + (ue - u)));
        const int n_tile = tile % p.n_tiles, m_tile = tile / p.n_tiles;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!mbar_wait(&empty[s], ph ^ 1u, p.status)) goto producer_done;
          mbar_arrive_expect_tx(&full[s], S::kStageBytes);
          uint8_t* st = smem + s * S::kStageBytes;
          tma_load_2d_hint(st, &map_a, &full[s], kb * kGemmBlockK, m_tile * kGemmBlockM, pol_w);
          if (NA == 2)
            tma_load_2d_hint(st + S::kABytes, &map_a, &full[s], kb * kGemmBlockK,
                             p.second_row + m_tile * kGemmBlockM, pol_w);
          tma_load_2d_hint(st + NA * S::kABytes, &map_b, &full[s], kb * kGemmBlockK,
                           n_tile * BN, pol_x);
        }
        u += kb1 - kb0;
      }
    producer_done:;
    }
  } else if (warp == 5) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc(kGemmBlockM, BN, 0);
      uint32_t it = 0, seg = 0;
      for (long long u = ub; u < ue; ++seg) {
        const int kb0 = static_cast<int>(u % KB);
        const int kb1 = static_cast<int>(min_ll(KB, kb0 + (ue - u)));
        const int b = seg % S::kAccBufs;
        const uint32_t bph = (seg / S::kAccBufs) & 1u;
        if (!mbar_wait(&tempty[b], bph ^ 1u, p.status)) goto mma_done;
        tc_fence_after();
        const uint32_t d = tmem_base + b * NA * BN;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!mbar_wait(&full[s], ph, p.status)) goto mma_done;
          tc_fence_after();
          const uint32_t a0 = smem_u32(smem + s * S::kStageBytes);
          const uint32_t b0 = a0 + NA * S::kABytes;
#pragma unroll
          for (int k = 0; k < kGemmBlockK / 16; ++k) {
            const uint32_t acc = (kb > kb0 || k > 0) ? 1u : 0u;
            const uint64_t bd = sw128_desc(b0 + k * 32);
            umma_f16(d, sw128_desc(a0 + k * 32), bd, idesc, acc);
            if (NA == 2) umma_f16(d + BN, sw128_desc(a0 + S::kABytes + k * 32), bd, idesc, acc);
          }
          umma_commit(&empty[s]);
        }
        umma_commit(&tfull[b]);
        u += kb1 - kb0;
      }
    mma_done:;
    }
  } else {
    // Epilogue: thread t owns TMEM lane t = output feature m_tile*128 + t.
    const int t = threadIdx.x;
    float red0[16], red1[16];
    uint32_t seg = 0;
    for (long long u = ub; u < ue; ++seg) {
      const int tile = static_cast<int>(u / KB);
      const int kb0 = static_cast<int>(u % KB);
      const int kb1 = static_cast<int>(min_ll(KB, kb0 + (ue - u)));
      const int n_tile = tile % p.n_tiles, m_tile = tile / p.n_tiles;
      const int b = seg % S::kAccBufs;
      const uint32_t bph = (seg / S::kAccBufs) & 1u;
      if (!mbar_wait(&tfull[b], bph, p.status)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(warp * 32) << 16) + b * NA * BN;
      const int m = m_tile * kGemmBlockM + t;
      const int n0 = n_tile * BN;
      const int nvalid = min(BN, p.n - n0);
      if (kb0 == 0 && kb1 == KB) {
        for (int c = 0; c < BN / 16; ++c) {
          if (c * 16 >= nvalid) break;
          float v0[16], v1[16];
          tmem_ld16(taddr + c * 16, v0);
          if (NA == 2) tmem_ld16(taddr + BN + c * 16, v1);
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (c * 16 + j < nvalid && m < p.m) apply_epilogue(p, n0 + c * 16 + j, m, v0[j], NA == 2 ? v1[j] : 0.f);
        }
        tc_fence_before();
        mbar_arrive(&tempty[b]);
      } else {
        const long long seg_start = u;
        const int slot = 2 * blockIdx.x + (seg_start == ub ? 0 : 1);
        float* dst = p.partials + static_cast<size_t>(slot) * NA * BN * 128;
        for (int c = 0; c < BN / 16; ++c) {
          if (c * 16 >= nvalid) break;
          float v0[16], v1[16];
          tmem_ld16(taddr + c * 16, v0);
          if (NA == 2) tmem_ld16(taddr + BN + c * 16, v1);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            dst[(c * 16 + j) * 128 + t] = v0[j];
            if (NA == 2) dst[(BN + c * 16 + j) * 128 + t] = v1[j];
          }
        }
        tc_fence_before();
        mbar_arrive(&tempty[b]);
        __threadfence();
        named_bar_sync(1, 128);
        const long long tile_u0 = static_cast<long long>(tile) * KB;
        const int c_first = cta_of_unit(p.units, grid, tile_u0);
        const int c_last = cta_of_unit(p.units, grid, tile_u0 + KB - 1);
        if (t == 0) {
          const unsigned prev = atomicAdd(&p.counters[tile], 1u);
          *last_flag = (prev == static_cast<unsigned>(c_last - c_first)) ? 1 : 0;
        }
        named_bar_sync(1, 128);
        if (*last_flag) {
          __threadfence();
          // Sum the tile's partials in CTA order.  Loads are issued in batches
          // (16 columns x up to 8 segments per accumulator) before any add, so
          // the reduction is bound by L2 bandwidth rather than load latency.
          constexpr int kCols = 16, kSegs = 8;
          for (int col0 = 0; col0 < nvalid; col0 += kCols) {
            for (int acc_i = 0; acc_i < NA; ++acc_i) {
              float sum[kCols];
#pragma unroll
              for (int j = 0; j < kCols; ++j) sum[j] = 0.f;
              for (int c0 = c_first; c0 <= c_last; c0 += kSegs) {
                float v[kSegs][kCols];
#pragma unroll
                for (int sidx = 0; sidx < kSegs; ++sidx) {
                  const int c = c0 + sidx;
                  if (c <= c_last) {
                    const int sl = 2 * c + (unit_begin(p.units, grid, c) >= tile_u0 ? 0 : 1);
                    const float* src = p.partials + static_cast<size_t>(sl) * NA * BN * 128 +
                                       static_cast<size_t>(acc_i * BN + col0) * 128 + t;
#pragma unroll
                    for (int j = 0; j < kCols; ++j)
                      v[sidx][j] = (col0 + j < nvalid) ? __ldcg(src + j * 128) : 0.f;
                  }
                }
#pragma unroll
                for (int sidx = 0; sidx < kSegs; ++sidx)
                  if (c0 + sidx <= c_last)
#pragma unroll
                    for (int j = 0; j < kCols; ++j) sum[j] += v[sidx][j];
              }
              if (acc_i == 0) {
#pragma unroll
                for (int j = 0; j < kCols; ++j) red0[j] = sum[j];
              } else {
#pragma unroll
                for (int j = 0; j < kCols; ++j) red1[j] = sum[j];
              }
            }
#pragma unroll
            for (int j = 0; j < kCols; ++j)
              if (col0 + j < nvalid && m < p.m)
                apply_epilogue(p, n0 + col0 + j, m, red0[j], NA == 2 ? red1[j] : 0.f);
          }
          if (t == 0) p.counters[tile] = 0u;
        }
      }
      u += kb1 - kb0;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 5) tmem_dealloc(tmem_base, S::kTmemCols);
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
  gemm_tc_kernel<BN, NA><<<grid, 192, S::kSmemBytes, stream>>>(w.map, x.maps[bn_index], p);
  return cudaGetLastError();
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

size_t gemm_partial_floats(int sm_count) {
  // Two partial slots per CTA, each up to 2 accumulators x 256 tokens x 128 rows.
  return static_cast<size_t>(sm_count) * 2 * 2 * 256 * 128;
}

size_t gemm_counter_count(int max_m, int max_n) {
  return static_cast<size_t>((max_m + kGemmBlockM - 1) / kGemmBlockM) *
         ((max_n + 15) / 16);
}

cudaError_t gemm_run(const GemmWeight& w, const GemmInput& x, int n, int epilogue, void* out,
                     int ldo, const GemmScratch& scratch, cudaStream_t stream, int bn_override,
                     int grid_override) {
  if (n <= 0 || n > x.rows_cap || w.k_pad != x.k_pad) return cudaErrorInvalidValue;
  if ((epilogue == kEpiSwiGLU) != (w.pair == 2)) return cudaErrorInvalidValue;
  int bn_index = 0;
  if (bn_override) {
    bn_index = -1;
    for (int i = 0; i < kGemmNumBn; ++i)
      if (kGemmBn[i] == bn_override) bn_index = i;
    if (bn_index < 0) return cudaErrorInvalidValue;
  } else {
    while (bn_index + 1 < kGemmNumBn && kGemmBn[bn_index] < n) ++bn_index;
  }
  if (w.pair == 2 && kGemmBn[bn_index] > 128) bn_index = 3;  // 2 accumulators x 128 x 2 buffers
  const int bn = kGemmBn[bn_index];
  GemmParams p{};
  p.m = w.m;
  p.n = n;
  p.kb_count = w.k_pad / kGemmBlockK;
  p.n_tiles = (n + bn - 1) / bn;
  const int m_tiles = (w.m + kGemmBlockM - 1) / kGemmBlockM;
  const long long tiles = static_cast<long long>(m_tiles) * p.n_tiles;
  if (static_cast<size_t>(tiles) > scratch.counter_count) return cudaErrorInvalidValue;
  p.units = tiles * p.kb_count;
  p.second_row = w.second_row;
  p.epilogue = epilogue;
  p.out = out;
  p.ldo = ldo;
  p.partials = scratch.partials;
  p.counters = scratch.counters;
  p.status = scratch.status;
  // One CTA per SM, but never fewer than 4 K blocks per CTA (pipeline fill).
  long long grid = grid_override > 0 ? grid_override : scratch.sm_count;
  if (grid_override <= 0) grid = std::min<long long>(grid, std::max<long long>(1, p.units / 4));
  grid = std::min<long long>(grid, p.units);
  const size_t need = static_cast<size_t>(grid) * 2 * w.pair * bn * 128;
  if (need > scratch.partial_floats) return cudaErrorInvalidValue;
  const int g = static_cast<int>(grid);
  if (w.pair == 1) {
    switch (bn) {
      case 16: return launch<16, 1>(w, x, bn_index, p, g, stream);
      case 32: return launch<32, 1>(w, x, bn_index, p, g, stream);
      case 64: return launch<64, 1>(w, x, bn_index, p, g, stream);
      case 128: return launch<128, 1>(w, x, bn_index, p, g, stream);
      default: return launch<256, 1>(w, x, bn_index, p, g, stream);
    }
  }
  switch (bn) {
    case 16: return launch<16, 2>(w, x, bn_index, p, g, stream);
    case 32: return launch<32, 2>(w, x, bn_index, p, g, stream);
    case 64: return launch<64, 2>(w, x, bn_index, p, g, stream);
    default: return launch<128, 2>(w, x, bn_index, p, g, stream);
  }
}

}  // namespace hb
