// attention_tc.cu -- prefill attention on the 5th-generation tensor cores.
//
// Reference op: `attention` (cpp/src/cpu/llama.cpp:67-112), causal GQA with
// scores scaled by 1/sqrt(d) and a max-subtracted softmax, for the prefill
// rows (several new tokens) of a packed batch, head sizes 64 and 128.
//
// One CTA per (kv head, query tile, key split), 192 threads:
//   warp 4   -- producer: the query tile (one 3-D TMA box per 64 dims: tokens x
//               the GQA group's heads), then for each 128-key tile its eight
//               16-key K and V pages, by block table, as 2-D TMA boxes with the
//               128-byte swizzle into a two-stage ring;
//   warp 5   -- TMEM owner and the single thread that issues tcgen05.mma:
//               S = Q K^T into one of two TMEM score buffers, then, once the
//               softmax has written P, O += P V into the TMEM output;
//   warps 0-3 -- softmax, one query row (TMEM lane) per thread: row maximum,
//               P = 2^(s * scale * log2 e - m) as F16 into shared memory in the
//               swizzled K-major layout the MMA reads, the running sum, and,
//               when a row's maximum passed its reference m by more than 2^8,
//               a new reference and the rescale of O in TMEM; at the end
//               O / l to the output, or, with several key splits, the split's
//               rows and (m, l) for the last split to merge in split order.
// The MMA for S on tile i+1 is issued before the PV of tile i, so it runs
// while the softmax works on tile i; the softmax of tile i waits for the PV of
// tile i - 2 (its P buffer) and only on a rescale for that of tile i - 1, so
// it overlaps the PV of tile i - 1.  The V tile is the PV MMA's B operand as
// it lies (MN-major: 64 dims per 128-byte row, one row per key), so no
// transpose is needed.  Scores of keys past a row's position or past the
// context are masked to p = 0; pages past the context are filled from a valid
// page so that no stale shared memory is multiplied in.  Every wait is bounded
// (common.cuh); every CTA issues its own TMA copies.
#include <cudaTypedefs.h>
#include <math.h>

#include <algorithm>
#include <mutex>

#include "attention.cuh"
#include "common.cuh"

namespace hb {
namespace {

constexpr int kTcRows = 128;     // query rows per CTA: tokens x heads of one GQA group
constexpr int kTcKeys = 128;     // keys per tile
constexpr int kTcThreads = 192;
constexpr int kTcPages = kTcKeys / 16;
constexpr float kTcLog2e = 1.4426950408889634f;

template <int DP>
struct TcShape {
  static constexpr uint32_t kAtom = 128 * 128;             // 128 rows x 64 F16: one swizzle column
  static constexpr uint32_t kQBytes = kTcRows * DP * 2;
  static constexpr uint32_t kKvBytes = kTcKeys * DP * 2;
  static constexpr uint32_t kPBytes = kTcRows * kTcKeys * 2;
  static constexpr uint32_t kQ = 0;
  static constexpr uint32_t kK = kQBytes;                  // two stages
  static constexpr uint32_t kV = kK + 2 * kKvBytes;        // two stages
  static constexpr uint32_t kP = kV + 2 * kKvBytes;        // two buffers
  static constexpr uint32_t kBar = kP + 2 * kPBytes;
  static constexpr uint32_t kSmem = kBar + 256 + 1024;     // barriers; 1024-byte alignment slack
  static constexpr uint32_t kTmemS = 0;                    // two 128-column score buffers
  static constexpr uint32_t kTmemO = 2 * kTcKeys;          // DP output columns
  static constexpr uint32_t kTmemCols = 512;
};

__device__ __forceinline__ int tile_row(const int32_t* cu, int rows, int idx) {
  int lo = 0, hi = rows;  // cu[lo] <= idx < cu[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (cu[mid] <= idx) lo = mid; else hi = mid;
  }
  return lo;
}

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t half2_bits(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

template <int DP>
__global__ void __launch_bounds__(kTcThreads, 1)
    prefill_attn_tc_kernel(const __grid_constant__ TcMaps maps, const AttnArgs a) {
  using S = TcShape<DP>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::kBar);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;    // [2]
  uint64_t* v_full = bars + 3;    // [2]
  uint64_t* kv_empty = bars + 5;  // [2]
  uint64_t* s_full = bars + 7;    // [2]
  uint64_t* s_empty = bars + 9;   // [2]
  uint64_t* p_full = bars + 11;   // [2] by tile parity
  uint64_t* o_done = bars + 13;   // [2] by tile parity: PV of that tile complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 15);
  int* last_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int G = a.hq / a.hkv;
  const int QT = kTcRows / G;
  const int kvh = blockIdx.x, tile = blockIdx.y;
  const int split = blockIdx.z, nsplit = gridDim.z;
  // The packer's tables are complete before this kernel starts.
  const int r = tile_row(a.cu_qtiles, a.rows, tile);
  const int count = a.row_count[r];
  if (count <= 1) return;  // the same for the whole CTA, before any set-up
  const int tok0 = (tile - a.cu_qtiles[r]) * QT;
  const int first = a.row_first[r];
  const int ntok = min(QT, count - tok0);
  const int ctx_hi = first + tok0 + ntok;  // keys [0, ctx_hi)
  const int n_kt = (ctx_hi + kTcKeys - 1) / kTcKeys;
  const int kt0 = n_kt * split / nsplit, kt1 = n_kt * (split + 1) / nsplit;
  const int n = kt1 - kt0;
  const int t_base = a.cu_seqlens[r];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&s_empty[s], 128);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&p_full[b], 128);
      mbar_init(&o_done[b], 1);
    }
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, S::kTmemCols);
    tmem_relinquish();
  }
  if (warp == 4 && lane == 0) {
    prefetch_tensormap(&maps.q);
    prefetch_tensormap(&maps.k);
    prefetch_tensormap(&maps.v);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_enter();  // q and this layer's K/V pages come from the previous kernels

  if (warp == 4) {
    // ---------------------------------------------------------------- producer
    const int32_t* table = a.block_tables + static_cast<size_t>(r) * a.max_blocks;
    const int npages = min((ctx_hi + 15) / 16, a.max_blocks);
    if (lane == 0 && n > 0) {
      mbar_arrive_expect_tx(q_full, S::kQBytes);
      for (int h = 0; h < DP / 64; ++h)
        tma_load_3d(smem + S::kQ + h * S::kAtom, &maps.q, q_full, h * 64, kvh * G, t_base + tok0);
    }
    int issued = 0;
    for (int i = 0; i < n; ++i) {
      const int s = i & 1;
      const int kt = kt0 + i;
      int bid = 0;
      if (lane < kTcPages) {
        // A page past the context is loaded from the row's first page: its
        // keys are masked to p = 0, and finite values keep 0 x v finite.
        const int pg = kt * kTcPages + lane < npages ? kt * kTcPages + lane : 0;
        bid = __ldg(table + pg);
        if (bid < 0) {
          atomicOr(a.status, kDevBadIndex);
          bid = 0;
        }
      }
      bool ok = true;
      if (lane == 0 && i >= 2) ok = mbar_wait(&kv_empty[s], ((i - 2) >> 1) & 1u, a.status);
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      if (lane == 0) {
        mbar_arrive_expect_tx(&k_full[s], S::kKvBytes);
        mbar_arrive_expect_tx(&v_full[s], S::kKvBytes);
      }
#pragma unroll
      for (int pp = 0; pp < kTcPages; ++pp) {
        const int b = __shfl_sync(0xffffffffu, bid, pp);
        if (lane == 0) {
          const int y = (b * a.hkv + kvh) * 16;
#pragma unroll
          for (int h = 0; h < DP / 64; ++h)
            tma_load_2d(smem + S::kK + s * S::kKvBytes + h * S::kAtom + pp * 2048, &maps.k,
                        &k_full[s], h * 64, y);
        }
      }
#pragma unroll
      for (int pp = 0; pp < kTcPages; ++pp) {
        const int b = __shfl_sync(0xffffffffu, bid, pp);
        if (lane == 0) {
          const int y = (b * a.hkv + kvh) * 16;
#pragma unroll
          for (int h = 0; h < DP / 64; ++h)
            tma_load_2d(smem + S::kV + s * S::kKvBytes + h * S::kAtom + pp * 2048, &maps.v,
                        &v_full[s], h * 64, y);
        }
      }
      issued = i + 1;
    }
    // Copies still in flight land before the CTA can exit (normally long
    // done; after a failed wait, bounded).
    if (lane == 0) {
      for (int i = max(0, issued - 2); i < issued; ++i) {
        mbar_wait(&k_full[i & 1], (i >> 1) & 1u, a.status);
        mbar_wait(&v_full[i & 1], (i >> 1) & 1u, a.status);
      }
      if (n > 0) mbar_wait(q_full, 0, a.status);
    }
  } else if (warp == 5) {
    // ---------------------------------------------------------------- MMA issue
    if (lane == 0 && n > 0) {
      constexpr uint32_t idesc_s = umma_idesc(kTcRows, kTcKeys, 0);
      constexpr uint32_t idesc_pv = umma_idesc(kTcRows, DP, 0) | (1u << 16);  // B MN-major
      const uint32_t q0 = smem_u32(smem + S::kQ);
      auto issue_s = [&](int i) -> bool {
        const int s = i & 1;
        if (i >= 2 && !mbar_wait(&s_empty[s], ((i - 2) >> 1) & 1u, a.status)) return false;
        if (!mbar_wait(&k_full[s], (i >> 1) & 1u, a.status)) return false;
        tc_fence_after();
        const uint32_t k0 = smem_u32(smem + S::kK + s * S::kKvBytes);
#pragma unroll
        for (int kk = 0; kk < DP / 16; ++kk) {
          const uint32_t off = (kk >> 2) * S::kAtom + (kk & 3) * 32;
          umma_f16(tmem + S::kTmemS + s * kTcKeys, sw128_desc(q0 + off), sw128_desc(k0 + off),
                   idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[s]);
        return true;
      };
      auto issue_pv = [&](int i) -> bool {
        const int s = i & 1;
        if (!mbar_wait(&p_full[i & 1], (i >> 1) & 1u, a.status)) return false;
        if (!mbar_wait(&v_full[s], (i >> 1) & 1u, a.status)) return false;
        tc_fence_after();
        const uint32_t p0 = smem_u32(smem + S::kP + s * S::kPBytes);
        const uint32_t v0 = smem_u32(smem + S::kV + s * S::kKvBytes);
#pragma unroll
        for (int ks = 0; ks < kTcKeys / 16; ++ks) {
          const uint32_t poff = (ks >> 2) * S::kAtom + (ks & 3) * 32;
          umma_f16(tmem + S::kTmemO, sw128_desc(p0 + poff),
                   sw128_desc_mn(v0 + ks * 2048, S::kAtom), idesc_pv,
                   (i > 0 || ks > 0) ? 1u : 0u);
        }
        umma_commit(&o_done[i & 1]);
        umma_commit(&kv_empty[s]);
        return true;
      };
      bool ok = mbar_wait(q_full, 0, a.status) && issue_s(0);
      for (int i = 0; ok && i < n; ++i) {
        if (i + 1 < n) ok = issue_s(i + 1);
        if (ok) ok = issue_pv(i);
      }
    }
  } else {
    // ---------------------------------------------------------------- softmax
    const int row = threadIdx.x;  // TMEM lane
    const int tl = row / G, g = row % G;
    const int pos = first + tok0 + tl;
    const float sl2 = a.scale * kTcLog2e;
    const uint32_t lanes = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    // m is the reference of this row's exponentials: raised only when a
    // tile's maximum exceeds it by more than kLazy (log2 units), so most
    // tiles need no rescale of O and P stays below 2^kLazy.
    constexpr float kLazy = 8.f;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int i = 0; i < n; ++i) {
      const int sb = i & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[sb], (i >> 1) & 1u, a.status));
      if (!ok) break;
      tc_fence_after();
      const int key0 = (kt0 + i) * kTcKeys;
      // Keys key0 + c are valid for this row while c <= lim.
      const int lim = min(pos, ctx_hi - 1) - key0;
      const uint32_t sa = lanes + S::kTmemS + sb * kTcKeys;
      float mx = -INFINITY;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t v0[32], v1[32];
        tmem_ld32_nowait(sa + h * 64, v0);
        tmem_ld32_nowait(sa + h * 64 + 32, v1);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          if (h * 64 + j <= lim) mx = fmaxf(mx, __uint_as_float(v0[j]));
          if (h * 64 + 32 + j <= lim) mx = fmaxf(mx, __uint_as_float(v1[j]));
        }
      }
      const float mt = mx * sl2;
      float alpha = 1.f;
      if (mt > m + kLazy || (m == -INFINITY && mt > -INFINITY)) {
        alpha = ex2f(m - mt);  // 0 while m is -inf
        m = mt;
      }
      // A row with no valid key yet keeps m = -inf; the reference point 0 then
      // makes every p exactly 0 (no inf - inf).
      const float ref = m == -INFINITY ? 0.f : m;
      // P goes to buffer i & 1, which the PV of tile i - 2 read.
      if (i >= 2) {
        ok = __all_sync(0xffffffffu, mbar_wait(&o_done[sb], ((i - 2) >> 1) & 1u, a.status));
        if (!ok) break;
      }
      uint8_t* prow = smem + S::kP + sb * S::kPBytes + row * 128;
      float rs = 0.f;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t v[2][32];
        tmem_ld32_nowait(sa + h * 64, v[0]);
        tmem_ld32_nowait(sa + h * 64 + 32, v[1]);
        tmem_ld_wait();
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int c = 2 * h + hh;
          uint32_t pk[16];
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            const float p0 =
                c * 32 + j <= lim ? ex2f(fmaf(__uint_as_float(v[hh][j]), sl2, -ref)) : 0.f;
            const float p1 =
                c * 32 + j + 1 <= lim ? ex2f(fmaf(__uint_as_float(v[hh][j + 1]), sl2, -ref)) : 0.f;
            rs += p0 + p1;
            pk[j >> 1] = half2_bits(p0, p1);
          }
          // Keys c*32 .. c*32+31 are 16-byte chunks kc = 4c .. 4c+3 of the row:
          // swizzle column kc / 8, chunk kc % 8 XOR the row (128-byte swizzle).
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int kc = c * 4 + q;
            uint8_t* dst = prow + (kc >> 3) * S::kAtom + (((kc & 7) ^ (row & 7)) << 4);
            *reinterpret_cast<uint4*>(dst) =
                make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&s_empty[sb]);
      l = l * alpha + rs;
      if (i > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
        // O holds the PV of the earlier tiles once tile i - 1's completed;
        // rescale it to the new reference.
        ok = __all_sync(0xffffffffu, mbar_wait(&o_done[(i - 1) & 1], ((i - 1) >> 1) & 1u, a.status));
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < DP / 32; ++c) {
          uint32_t v[32];
          tmem_ld32_nowait(lanes + S::kTmemO + c * 32, v);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) * alpha);
          tmem_st32(lanes + S::kTmemO + c * 32, v);
        }
        tmem_st_wait();
      }
      fence_proxy_async();  // P is read by the tensor cores (async proxy)
      tc_fence_before();
      mbar_arrive(&p_full[sb]);
    }
    if (ok && n > 0)
      ok = __all_sync(0xffffffffu,
                      mbar_wait(&o_done[(n - 1) & 1], ((n - 1) >> 1) & 1u, a.status));
    if (ok && n > 0) tc_fence_after();

    __half* out_row = tl < ntok ? a.out + static_cast<size_t>(t_base + tok0 + tl) * a.ld_out +
                                      static_cast<size_t>(kvh * G + g) * DP
                                : nullptr;
    if (nsplit == 1) {
      if (ok && n > 0) {
        const float inv = 1.0f / l;
#pragma unroll
        for (int c = 0; c < DP / 32; ++c) {
          uint32_t v[32];
          tmem_ld32_nowait(lanes + S::kTmemO + c * 32, v);
          tmem_ld_wait();
          if (out_row) {
            uint32_t hv[16];
#pragma unroll
            for (int j = 0; j < 32; j += 2)
              hv[j >> 1] = half2_bits(__uint_as_float(v[j]) * inv, __uint_as_float(v[j + 1]) * inv);
            uint4* dst = reinterpret_cast<uint4*>(out_row + c * 32);
#pragma unroll
            for (int q = 0; q < 4; ++q)
              dst[q] = make_uint4(hv[4 * q], hv[4 * q + 1], hv[4 * q + 2], hv[4 * q + 3]);
          }
        }
      }
    } else {
      // This split's unnormalised rows and (m, l), then the last split merges.
      const size_t cell = static_cast<size_t>(tile) * a.hkv + kvh;
      constexpr size_t kPiece = static_cast<size_t>(kTcRows) * (DP + 2);
      float* piece = a.pre_part + (cell * nsplit + split) * kPiece;
#pragma unroll
      for (int c = 0; c < DP / 32; ++c) {
        uint32_t v[32];
        if (ok && n > 0) {
          tmem_ld32_nowait(lanes + S::kTmemO + c * 32, v);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = 0u;
        }
        float4* dst = reinterpret_cast<float4*>(piece + row * DP + c * 32);
#pragma unroll
        for (int q = 0; q < 8; ++q)
          dst[q] = make_float4(__uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]),
                               __uint_as_float(v[4 * q + 2]), __uint_as_float(v[4 * q + 3]));
      }
      *reinterpret_cast<float2*>(piece + kTcRows * DP + row * 2) =
          make_float2(n > 0 ? m : -INFINITY, n > 0 ? l : 0.f);
      __threadfence();
      // All 128 softmax threads reach this barrier, ok or not.
      const bool all_ok = named_bar_all(1, 128, ok);
      if (row == 0) {
        int* counter = a.pre_counters + cell;
        const int last = atomicAdd(counter, 1) == nsplit - 1;
        if (last) *counter = 0;
        *last_flag = last;
      }
      named_bar_sync(1, 128);
      if (*last_flag && all_ok) {
        __threadfence();
        const float* pieces = a.pre_part + cell * nsplit * kPiece;
        float M = -INFINITY;
        for (int sp = 0; sp < nsplit; ++sp)
          M = fmaxf(M, __ldcg(pieces + sp * kPiece + kTcRows * DP + row * 2));
        float L = 0.f;
        for (int sp = 0; sp < nsplit; ++sp) {
          const float2 ml = __ldcg(
              reinterpret_cast<const float2*>(pieces + sp * kPiece + kTcRows * DP + row * 2));
          L += ml.y * exp2f(ml.x - M);  // 0 for a split with no key of this row
        }
        const float inv = 1.0f / L;
        for (int c4 = 0; c4 < DP && out_row; c4 += 4) {
          float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int sp = 0; sp < nsplit; ++sp) {
            const float* pc = pieces + sp * kPiece;
            const float w = exp2f(__ldcg(pc + kTcRows * DP + row * 2) - M);
            const float4 v = __ldcg(reinterpret_cast<const float4*>(pc + row * DP + c4));
            acc.x += v.x * w;
            acc.y += v.y * w;
            acc.z += v.z * w;
            acc.w += v.w * w;
          }
          *reinterpret_cast<uint2*>(out_row + c4) =
              make_uint2(half2_bits(acc.x * inv, acc.y * inv), half2_bits(acc.z * inv, acc.w * inv));
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 5) tmem_dealloc(tmem, S::kTmemCols);
}

PFN_cuTensorMapEncodeTiled_v12000 tc_encode_fn() {
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

template <int DP>
cudaError_t launch_tc(const TcMaps& maps, const AttnArgs& a, int total_qtiles, int splits,
                      cudaStream_t stream) {
  using S = TcShape<DP>;
  static bool configured = false;
  if (!configured) {
    const cudaError_t e = cudaFuncSetAttribute(prefill_attn_tc_kernel<DP>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(S::kSmem));
    if (e != cudaSuccess) return e;
    configured = true;
  }
  return launch_dependent(prefill_attn_tc_kernel<DP>, dim3(a.hkv, total_qtiles, splits),
                          dim3(kTcThreads), S::kSmem, stream, maps, a);
}

}  // namespace

bool attn_prefill_tc_supported(int dim, int group) {
  return (dim == 64 || dim == 128) && (group == 1 || group == 2 || group == 4 || group == 8);
}

bool attn_make_kv_maps(TcMaps* maps, int hkv, int dim, const void* k_cache, const void* v_cache,
                       long long kv_blocks) {
  auto fn = tc_encode_fn();
  if (!fn || dim % 64 != 0 || dim > 256 || kv_blocks <= 0) return false;
  // K and V caches [blocks][Hkv][16][d] as rows of d: box = 64 dims x one page.
  const cuuint32_t estr[2] = {1, 1};
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(dim),
                              static_cast<cuuint64_t>(kv_blocks) * hkv * 16};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(dim) * 2};
  const cuuint32_t box[2] = {64, 16};
  for (int which = 0; which < 2; ++which) {
    CUtensorMap* m = which == 0 ? &maps->k : &maps->v;
    const void* base = which == 0 ? k_cache : v_cache;
    if (fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return false;
  }
  return true;
}

bool attn_tc_make_maps(TcMaps* maps, const void* q, long long q_tokens, int hq, int hkv, int dim,
                       const void* k_cache, const void* v_cache, long long kv_blocks) {
  auto fn = tc_encode_fn();
  const int group = hq / hkv;
  if (!fn || !attn_prefill_tc_supported(dim, group) || q_tokens <= 0) return false;
  // q [tokens][Hq][d]: box = 64 dims x the group's heads x 128 / group tokens.
  const cuuint32_t estr[3] = {1, 1, 1};
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(dim), static_cast<cuuint64_t>(hq),
                              static_cast<cuuint64_t>(q_tokens)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(dim) * 2,
                                 static_cast<cuuint64_t>(hq) * dim * 2};
  const cuuint32_t box[3] = {64, static_cast<cuuint32_t>(group),
                             static_cast<cuuint32_t>(kTcRows / group)};
  if (fn(&maps->q, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(q), dims, strides, box,
         estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  return attn_make_kv_maps(maps, hkv, dim, k_cache, v_cache, kv_blocks);
}

int attn_prefill_tc_splits(int hkv, int total_qtiles, int sm_count) {
  if (total_qtiles <= 0) return 1;
  const long long base = static_cast<long long>(hkv) * total_qtiles;
  // One resident CTA per SM; as many key splits as still fit one wave.
  const long long s = static_cast<long long>(sm_count) / std::max<long long>(1, base);
  return static_cast<int>(std::max<long long>(1, std::min<long long>(s, kPrefillMaxSplits)));
}

cudaError_t attn_prefill_tc_launch(const TcMaps& maps, const AttnArgs& a, int total_qtiles,
                                   cudaStream_t stream) {
  if (total_qtiles <= 0) return cudaSuccess;
  if (!attn_prefill_tc_supported(a.dim, a.hq / a.hkv)) return cudaErrorInvalidValue;
  const int splits = a.prefill_splits > 0 ? a.prefill_splits : 1;
  if (splits > kPrefillMaxSplits || (splits > 1 && (!a.pre_part || !a.pre_counters)))
    return cudaErrorInvalidValue;
  return a.dim == 64 ? launch_tc<64>(maps, a, total_qtiles, splits, stream)
                     : launch_tc<128>(maps, a, total_qtiles, splits, stream);
}

}  // namespace hb
