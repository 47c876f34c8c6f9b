// attention.cu -- paged-KV GQA attention for mixed prefill-chunk + decode batches.
//
// Reference op: `attention` (cpp/src/cpu/llama.cpp:67-112): causal GQA (query
// head h reads kv head h / (Hq/Hkv)), scores scaled by 1/sqrt(d), softmax with
// the row maximum subtracted, over the per-sequence cache.  The reference CUDA
// worker materialises GQA-expanded F32 K/V and an [Hq, T, C] score matrix per
// sequence (cpp/src/cuda/stage.cpp:279-302, looped per batch member :326-333);
// here one launch covers the whole ragged batch, K/V stay F16 in 16-token
// pages, every query head of a GQA group shares one pass over its KV pages,
// and no score matrix is stored (online softmax).
//
//   decode rows:  head sizes 64/128/256 -- the batch's KV pages split evenly
//                 over one wave of warps (ranges cross row boundaries), QK^T
//                 and PV on the tensor cores (mma.sync), split streams' pieces
//                 merged by a second, small pass.  Other head sizes -- split-K
//                 with one CTA per (kv head, context split) streaming 16-token
//                 pages with cp.async.bulk (mbarrier completion, bounded
//                 waits), then a combine pass.
//   prefill rows: causal flash tiles on the tensor cores (mma.sync F16 -> F32),
//                 64 query rows per CTA = (tokens x heads of one GQA group),
//                 K/V pages gathered by block table with cp.async.
#include <math.h>

#include <algorithm>

#include "attention.cuh"
#include "common.cuh"

namespace hb {
namespace {

constexpr int kDecThreads = 128;
constexpr int kDecStages = 4;
constexpr int kMaxGroup = 8;
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ int find_row(const int32_t* cu, int rows, int idx) {
  int lo = 0, hi = rows;  // cu[lo] <= idx < cu[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (cu[mid] <= idx) lo = mid; else hi = mid;
  }
  return lo;
}

// ---------------------------------------------------------------- warp-level MMA helpers
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, "
      "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}


// ---------------------------------------------------------------- decode
__global__ void __launch_bounds__(kDecThreads)
    decode_attn_kernel(const AttnArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  griddep_enter();
  const int d = a.dim;
  const int G = a.hq / a.hkv;
  const int kvh = blockIdx.x;
  const int split = blockIdx.y;
  const int r = find_row(a.cu_splits, a.rows, split);
  if (a.row_count[r] != 1) return;
  const int local = split - a.cu_splits[r];
  const int ctx = a.seq_lens[r];
  const int key0 = local * a.split_tokens;
  const int key1 = min(ctx, key0 + a.split_tokens);
  const int kb0 = key0 / 16, kb1 = (key1 + 15) / 16;
  const int nblk = kb1 - kb0;
  const int t = a.cu_seqlens[r];

  const uint32_t page_bytes = 16u * d * 2u;
  __half* ring = reinterpret_cast<__half*>(smem);                       // [S][2][16][d]
  float* qs = reinterpret_cast<float*>(smem + kDecStages * 2 * page_bytes);  // [G][d]
  float* sc = qs + G * d;                                               // [G][16]
  float* pr = sc + G * 16;                                              // [G][16]
  float* st = pr + G * 16;                                              // m[G], l[G], alpha[G]
  uint64_t* full = reinterpret_cast<uint64_t*>(
      (reinterpret_cast<uintptr_t>(st + 3 * kMaxGroup) + 7) & ~static_cast<uintptr_t>(7));

  const int tid = threadIdx.x;
  if (tid == 0) {
    for (int s = 0; s < kDecStages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  for (int i = tid; i < G * d; i += kDecThreads)
    qs[i] = __half2float(a.q[static_cast<size_t>(t) * a.hq * d + (kvh * G) * d + i]);
  if (tid < G) {
    st[tid] = -INFINITY;
    st[kMaxGroup + tid] = 0.f;
  }
  __syncthreads();

  const int32_t* table = a.block_tables + static_cast<size_t>(r) * a.max_blocks;
  auto issue = [&](int i) {
    const int s = i % kDecStages;
    const int bid = table[kb0 + i];
    if (bid < 0) {  // no page: complete the phase without a copy and report it
      atomicOr(a.status, kDevBadIndex);
      mbar_arrive(&full[s]);
      return;
    }
    const size_t page = (static_cast<size_t>(bid) * a.hkv + kvh) * 16 * d;
    __half* dst = ring + static_cast<size_t>(s) * 2 * 16 * d;
    mbar_arrive_expect_tx(&full[s], 2 * page_bytes);
    bulk_load(dst, a.k_cache + page, page_bytes, &full[s]);
    bulk_load(dst + 16 * d, a.v_cache + page, page_bytes, &full[s]);
  };
  if (tid == 0)
    for (int i = 0; i < min(nblk, kDecStages); ++i) issue(i);

  // Per-thread PV accumulators: chunks of 4 dims, chunk c = tid + 128 k over G*d/4.
  const int chunks = G * d / 4;
  float acc[4][4];
#pragma unroll
  for (int k = 0; k < 4; ++k)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[k][e] = 0.f;

  const int grp = tid >> 3, sub = tid & 7;  // QK: 16 groups of 8 lanes, one key each
  bool ok = true;
  for (int i = 0; i < nblk; ++i) {
    const int s = i % kDecStages;
    if (!mbar_wait(&full[s], (i / kDecStages) & 1u, a.status)) { ok = false; }
    if (__syncthreads_or(!ok)) break;
    const __half* kp = ring + static_cast<size_t>(s) * 2 * 16 * d;
    const __half* vp = kp + 16 * d;
    // Phase 1: scores for key `grp` of this page, all G heads.
    {
      const int key = (kb0 + i) * 16 + grp;
      float part[kMaxGroup];
#pragma unroll
      for (int g = 0; g < kMaxGroup; ++g) part[g] = 0.f;
      for (int base = sub * 4; base < d; base += 32) {
        const uint2 raw = *reinterpret_cast<const uint2*>(kp + grp * d + base);
        const float2 k01 = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
        const float2 k23 = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
#pragma unroll
        for (int g = 0; g < kMaxGroup; ++g) {
          if (g < G) {
            const float* qg = qs + g * d + base;
            part[g] += qg[0] * k01.x + qg[1] * k01.y + qg[2] * k23.x + qg[3] * k23.y;
          }
        }
      }
#pragma unroll
      for (int g = 0; g < kMaxGroup; ++g) {
        if (g < G) {
          float v = part[g];
          v += __shfl_xor_sync(0xffffffffu, v, 1);
          v += __shfl_xor_sync(0xffffffffu, v, 2);
          v += __shfl_xor_sync(0xffffffffu, v, 4);
          if (sub == 0) sc[g * 16 + grp] = (key >= key0 && key < key1) ? v * a.scale : -INFINITY;
        }
      }
    }
    __syncthreads();
    // The previous page's slot is free now: refill it.
    if (tid == 0 && i >= 1 && i - 1 + kDecStages < nblk) issue(i - 1 + kDecStages);
    // Phase 2: online-softmax statistics per head.
    if (tid < G) {
      const float m_old = st[tid];
      float mx = m_old;
      for (int j = 0; j < 16; ++j) mx = fmaxf(mx, sc[tid * 16 + j]);
      const float alpha = expf(m_old - mx);
      float sum = 0.f;
      for (int j = 0; j < 16; ++j) {
        const float p = expf(sc[tid * 16 + j] - mx);
        pr[tid * 16 + j] = p;
        sum += p;
      }
      st[tid] = mx;
      st[kMaxGroup + tid] = st[kMaxGroup + tid] * alpha + sum;
      st[2 * kMaxGroup + tid] = alpha;
    }
    __syncthreads();
    // Phase 3: acc = acc * alpha + sum_j p_j V_j.
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int c = tid + k * kDecThreads;
      if (c < chunks) {
        const int g = c / (d / 4), i0 = (c % (d / 4)) * 4;
        const float alpha = st[2 * kMaxGroup + g];
        float o0 = acc[k][0] * alpha, o1 = acc[k][1] * alpha, o2 = acc[k][2] * alpha,
              o3 = acc[k][3] * alpha;
        for (int j = 0; j < 16; ++j) {
          const float p = pr[g * 16 + j];
          const uint2 raw = *reinterpret_cast<const uint2*>(vp + j * d + i0);
          const float2 v01 = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
          const float2 v23 = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
          o0 += p * v01.x;
          o1 += p * v01.y;
          o2 += p * v23.x;
          o3 += p * v23.y;
        }
        acc[k][0] = o0; acc[k][1] = o1; acc[k][2] = o2; acc[k][3] = o3;
      }
    }
  }
  // Write this split's unnormalised output and statistics.
  const int h0 = kvh * G;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int c = tid + k * kDecThreads;
    if (c < chunks) {
      const int g = c / (d / 4), i0 = (c % (d / 4)) * 4;
      float* dst = a.part_o + (static_cast<size_t>(split) * a.hq + h0 + g) * d + i0;
      *reinterpret_cast<float4*>(dst) = make_float4(acc[k][0], acc[k][1], acc[k][2], acc[k][3]);
    }
  }
  if (tid < G) {
    float* ml = a.part_ml + (static_cast<size_t>(split) * a.hq + h0 + tid) * 2;
    ml[0] = st[tid];
    ml[1] = st[kMaxGroup + tid];
  }
}

// ---------------------------------------------------------------- decode (tensor cores)
// Work is balanced over pages, not rows.  The decode rows' KV pages form one
// sequence ordered (row, kv head, page); each (row, kv head) is a "stream" of
// ceil(ctx / 16) pages.  Warp w of W takes the contiguous range
// [P w / W, P (w + 1) / W) of the P pages, whatever the rows' lengths, so one
// wave of warps finishes together.  A warp's range may cross streams; for each
// stream it touches it keeps a piece (m, l, unnormalised O of the G query
// heads).  A stream inside one warp is normalised and stored at once;
// otherwise its pieces go to part_o/part_ml at index (stream + warp) -- unique,
// since both grow along the sequence -- and the warp holding the stream's first
// page records the stream's warp range.  The merge pass (decode_merge_kernel)
// then combines each split stream's pieces in warp order (deterministic).
//
// Per warp: the G query heads of the kv head are the first G rows of an
// m16n8k16 tile (rows G..15 are zero), so QK^T and PV run on the tensor cores.
// K/V pages (16 keys x d) stream through a per-warp cp.async ring in an
// XOR-swizzled layout that ldmatrix reads without bank conflicts; a stream's
// query heads ride in the ring stage of its first page.  One lane of the warp
// fills the ring: each K and V page as 64-dimension TMA boxes of 16 keys with
// the 128-byte swizzle (d / 64 boxes per page), the query heads as one bulk
// copy, all completing on the stage's mbarrier; ldmatrix reads the swizzled
// pages without bank conflicts.  The ring runs ahead across stream
// boundaries, and block-table entries are fetched 32 pages at a time, so no
// global load sits between one page and the next.
// Ring depth: three stages (two pages in flight while one is computed); two
// for d = 256, whose stages would not fit three deep in shared memory.
template <int D>
__host__ __device__ constexpr int dec_stages() {
  return D >= 256 ? 2 : 3;
}

// Byte offset of 16-byte chunk `chunk` of key `row` in a page as the TMA boxes
// write it: box chunk / 8 (2 KB each), rows of 128 bytes, chunk % 8 XOR row % 8.
template <int D>
__device__ __forceinline__ uint32_t page_off(int row, int chunk) {
  return static_cast<uint32_t>(((chunk >> 3) << 11) + row * 128 + (((chunk & 7) ^ (row & 7)) << 4));
}

// Bytes of one ring stage: K page, V page, the group's query heads (1024-byte
// multiples, so every page starts on a swizzle-atom boundary).
__host__ __device__ constexpr uint32_t decode_stage_bytes(int d, int group) {
  return 2u * 16u * d * 2u + ((static_cast<uint32_t>(group) * d * 2u + 1023u) & ~1023u);
}

// Position in the page sequence: row, kv head, page within the stream, and
// the row's page count, context length and first packed token.
struct PageCursor {
  int r, kvh, q;
  int pages, ctx, t;
  long long cum;  // pages of the decode rows before r (one kv head)
};

__device__ __forceinline__ void cursor_load_row(const AttnArgs& a, PageCursor& c) {
  const int count = __ldg(a.row_count + c.r);
  c.ctx = __ldg(a.seq_lens + c.r);
  c.t = __ldg(a.cu_seqlens + c.r);
  c.pages = count == 1 ? (c.ctx + 15) >> 4 : 0;
}

__device__ __forceinline__ void cursor_next(const AttnArgs& a, PageCursor& c) {
  if (++c.q < c.pages) return;
  c.q = 0;
  if (++c.kvh < a.hkv) return;
  c.kvh = 0;
  c.cum += c.pages;
  while (++c.r < a.rows) {
    cursor_load_row(a, c);
    if (c.pages) return;
  }
  c.pages = 0;
}

__device__ __forceinline__ int warp_sum_int(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Decode pages of rows base + 32k + lane, k < 4 (0 past the end or for prefill
// rows); all eight loads are issued together.
__device__ __forceinline__ void load_row_pages(const AttnArgs& a, int base, int lane, int (&pg)[4]) {
  int cnt[4], len[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int r = base + 32 * k + lane;
    cnt[k] = r < a.rows ? __ldg(a.row_count + r) : 0;
    len[k] = r < a.rows ? __ldg(a.seq_lens + r) : 0;
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) pg[k] = cnt[k] == 1 ? (len[k] + 15) >> 4 : 0;
}

// Merges the ns pieces of one stream (pieces p0 + s * G + g, s < ns, g < G)
// in piece order and stores the G normalised head outputs at `out`.  Called
// by `warps` warps of a CTA: few pieces are merged by warp 0 in one round of
// loads; otherwise warp `warp` takes heads warp, warp + warps, ...
template <int D>
__device__ __noinline__ void decode_merge(const AttnArgs& a, size_t p0, int ns, int G,
                                          __half* out, int lane, int warp, int warps) {
  if (G * ns <= 32 && (G & (G - 1)) == 0) {
    if (warp != 0) return;
    // One (piece, head) per lane: j = s * G + g.  Lanes with equal g are the
    // lanes j ^ (multiples of G), so xor shuffles reduce per head.
    const int j = lane;
    float mj = -INFINITY, lj = 0.f;
    if (j < G * ns) {
      const float2 v = __ldcg(reinterpret_cast<const float2*>(a.part_ml + (p0 + j) * 2));
      mj = v.x;
      lj = v.y;
    }
    float M = mj;
    for (int o = G; o < 32; o <<= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    const float wj = j < G * ns ? expf(mj - M) : 0.f;
    float L = lj * wj;
    for (int o = G; o < 32; o <<= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
    // Output float4 f = lane + 32 k of the G x D block.
    constexpr int kMaxF = (8 * D / 4 + 31) / 32;
    const int nf4 = G * D / 4;
    float4 acc[kMaxF];
#pragma unroll
    for (int k = 0; k < kMaxF; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 2
    for (int s = 0; s < ns; ++s) {
#pragma unroll
      for (int k = 0; k < kMaxF; ++k) {
        const int f = lane + 32 * k;
        const int gg = min(f * 4 / D, G - 1);
        const float wt = __shfl_sync(0xffffffffu, wj, s * G + gg);
        if (f < nf4) {
          const float4 v = __ldcg(reinterpret_cast<const float4*>(
              a.part_o + (p0 + static_cast<size_t>(s) * G + gg) * D + (f * 4) % D));
          acc[k].x += wt * v.x;
          acc[k].y += wt * v.y;
          acc[k].z += wt * v.z;
          acc[k].w += wt * v.w;
        }
      }
    }
#pragma unroll
    for (int k = 0; k < kMaxF; ++k) {
      const int f = lane + 32 * k;
      const int gg = min(f * 4 / D, G - 1);
      const float inv = 1.0f / __shfl_sync(0xffffffffu, L, gg);
      if (f < nf4) {
        __half* dst = out + f * 4;  // head gg, element (f * 4) % D
        *reinterpret_cast<__half2*>(dst) = __floats2half2_rn(acc[k].x * inv, acc[k].y * inv);
        *reinterpret_cast<__half2*>(dst + 2) = __floats2half2_rn(acc[k].z * inv, acc[k].w * inv);
      }
    }
    return;
  }
  // Many pieces (or a group size that is not a power of two): a head per warp.
  for (int gg = warp; gg < G; gg += warps) {
    const float* ml = a.part_ml + (p0 + gg) * 2;
    const size_t mls = static_cast<size_t>(G) * 2;
    float mm = -INFINITY;
    for (int s = lane; s < ns; s += 32) mm = fmaxf(mm, __ldcg(ml + s * mls));
    mm = warp_max(mm);
    float ll = 0.f;
    for (int s = lane; s < ns; s += 32) ll += __ldcg(ml + s * mls + 1) * expf(__ldcg(ml + s * mls) - mm);
    ll = warp_sum(ll);
    const float inv = 1.0f / ll;
    const float* po = a.part_o + (p0 + gg) * D;
    const size_t pos = static_cast<size_t>(G) * D;
    for (int i0 = lane * 4; i0 < D; i0 += 128) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
      for (int s = 0; s < ns; ++s) {
        const float wt = expf(__ldcg(ml + s * mls) - mm);
        const float4 v = __ldcg(reinterpret_cast<const float4*>(po + s * pos + i0));
        acc.x += v.x * wt;
        acc.y += v.y * wt;
        acc.z += v.z * wt;
        acc.w += v.w * wt;
      }
      __half* dst = out + gg * D + i0;
      *reinterpret_cast<__half2*>(dst) = __floats2half2_rn(acc.x * inv, acc.y * inv);
      *reinterpret_cast<__half2*>(dst + 2) = __floats2half2_rn(acc.z * inv, acc.w * inv);
    }
  }
}

template <int D>
__global__ void __launch_bounds__(128)
    decode_attn_mma_kernel(const __grid_constant__ TcMaps maps, const AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  constexpr uint32_t kPage = 16 * D * 2;  // bytes of one K (or V) page
  constexpr int ST = dec_stages<D>();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int w = blockIdx.x * 4 + warp;
  const int hkv = a.hkv;
  const int G = a.hq / hkv;
  const uint32_t stage_bytes = decode_stage_bytes(D, G);

  // Total pages P (every warp computes it; the rows' counts are L2-resident).
  long long total = 0;
  for (int base = 0; base < a.rows; base += 128) {
    int pg[4];
    load_row_pages(a, base, lane, pg);
    total += warp_sum_int(pg[0] + pg[1] + pg[2] + pg[3]);
  }
  total *= hkv;
  // At most one warp per page, so that every warp in [0, W) owns at least one
  // page and each stream's pieces come from consecutive warps.
  const int W = static_cast<int>(min(static_cast<long long>(gridDim.x) * 4, total));
  if (w >= W) return;
  const long long p_begin = total * w / W, p_end = total * (w + 1) / W;

  // Locate p_begin: the row whose pages (x hkv) cover it.
  PageCursor c{};
  c.r = -1;
  {
    long long cum = 0;
    for (int base = 0; base < a.rows && c.r < 0; base += 128) {
      int pg[4];
      load_row_pages(a, base, lane, pg);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        int incl = pg[k];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int v = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += v;
        }
        const long long lo = (cum + incl - pg[k]) * hkv, hi = (cum + incl) * hkv;
        const unsigned hit =
            __ballot_sync(0xffffffffu, pg[k] > 0 && lo <= p_begin && p_begin < hi);
        if (c.r < 0 && hit) {
          const int src = __ffs(hit) - 1;
          c.r = base + 32 * k + src;
          c.cum = cum + __shfl_sync(0xffffffffu, incl - pg[k], src);
        }
        cum += __shfl_sync(0xffffffffu, incl, 31);
      }
    }
    if (c.r < 0) {  // unreachable for consistent row counts
      if (lane == 0) atomicOr(a.status, kDevBadIndex);
      return;
    }
    cursor_load_row(a, c);
    const long long off = p_begin - c.cum * hkv;
    c.kvh = static_cast<int>(off / c.pages);
    c.q = static_cast<int>(off % c.pages);
  }
  PageCursor ic = c;  // issue cursor, runs ahead of c
  const int n = static_cast<int>(p_end - p_begin);
  uint8_t* ring = smem + warp * (ST * stage_bytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + 4 * ST * stage_bytes) + warp * ST;
  const uint32_t q_bytes = static_cast<uint32_t>(G) * D * 2;
  if (lane == 0) {
    for (int s = 0; s < ST; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncwarp();

  // Block-table entries of the issue cursor's row, 32 pages per fetch.  The
  // first fetch, like everything above, reads only the packer's tables, so it
  // runs before the wait for the previous kernel (which writes q and the
  // current token's K/V).
  int tab_r = ic.r, tab_q0 = ic.q, tab_val = -1;
  {
    const int qq = ic.q + lane;
    tab_val = qq < ic.pages && qq < a.max_blocks
                  ? __ldg(a.block_tables + static_cast<size_t>(ic.r) * a.max_blocks + qq)
                  : -1;
  }
  griddep_enter();
  int issued = 0;
  auto issue = [&](int i) {
    uint8_t* kd = ring + (i % ST) * stage_bytes;
    if (ic.r != tab_r || ic.q < tab_q0 || ic.q >= tab_q0 + 32) {
      tab_r = ic.r;
      tab_q0 = ic.q;
      const int qq = ic.q + lane;
      tab_val = qq < ic.pages && qq < a.max_blocks
                    ? __ldg(a.block_tables + static_cast<size_t>(ic.r) * a.max_blocks + qq)
                    : -1;
    }
    const int bid_raw = __shfl_sync(0xffffffffu, tab_val, ic.q - tab_q0);
    // First page of a stream: its query heads ride along.
    const bool with_q = i == 0 || ic.q == 0;
    const __half* qs =
        a.q + static_cast<size_t>(ic.t) * a.hq * D + static_cast<size_t>(ic.kvh) * G * D;
    const int kvh = ic.kvh;
    cursor_next(a, ic);
    ++issued;
    if (lane == 0) {
      int bid = bid_raw;
      if (bid < 0) {  // a missing block: reported, and a valid page read in its place
        atomicOr(a.status, kDevBadIndex);
        bid = 0;
      }
      const int y = (bid * hkv + kvh) * 16;
      uint64_t* bar = &full[i % ST];
      mbar_arrive_expect_tx(bar, 2 * kPage + (with_q ? q_bytes : 0u));
#pragma unroll
      for (int h = 0; h < D / 64; ++h) {
        tma_load_2d(kd + h * 2048, &maps.k, bar, h * 64, y);
        tma_load_2d(kd + kPage + h * 2048, &maps.v, bar, h * 64, y);
      }
      if (with_q) bulk_load(kd + 2 * kPage, qs, q_bytes, bar);
    }
  };

  const int g = lane >> 2;
  const float sl2 = a.scale * kLog2e;
  uint32_t qa[D / 16][2];
  float o[D / 8][4];
  float m = -INFINITY, l = 0.f;

#pragma unroll
  for (int i = 0; i < ST - 1; ++i)
    if (i < n) issue(i);
  int i = 0;
  for (; i < n; ++i) {
    if (i + ST - 1 < n) issue(i + ST - 1);
    if (!__all_sync(0xffffffffu, mbar_wait(&full[i % ST], (i / ST) & 1u, a.status))) break;
    const uint8_t* stage = ring + (i % ST) * stage_bytes;
    if (i == 0 || c.q == 0) {
      // A new stream: its query heads as A fragments, fresh softmax state.
      const uint8_t* qrow = stage + 2 * kPage + g * D * 2;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const int col = kk * 16 + (lane & 3) * 2;
        qa[kk][0] = g < G ? *reinterpret_cast<const uint32_t*>(qrow + col * 2) : 0u;
        qa[kk][1] = g < G ? *reinterpret_cast<const uint32_t*>(qrow + (col + 8) * 2) : 0u;
      }
#pragma unroll
      for (int db = 0; db < D / 8; ++db)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[db][e] = 0.f;
      m = -INFINITY;
      l = 0.f;
    }
    const uint32_t kb = smem_u32(stage), vb = kb + kPage;
    float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t b0, b1, b2, b3;
      const int key = (lane & 7) + (lane >> 4) * 8;
      ldsm_x4(kb + page_off<D>(key, kk * 2 + ((lane >> 3) & 1)), b0, b1, b2, b3);
      mma16816(s[0], qa[kk][0], 0u, qa[kk][1], 0u, b0, b1);
      mma16816(s[1], qa[kk][0], 0u, qa[kk][1], 0u, b2, b3);
    }
    const int base = c.q * 16;
    float mx = m;
#pragma unroll
    for (int nb = 0; nb < 2; ++nb)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = base + nb * 8 + (lane & 3) * 2 + e;
        const float v = key < c.ctx ? s[nb][e] * sl2 : -INFINITY;
        s[nb][e] = v;
        mx = fmaxf(mx, v);
      }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float alpha = exp2f(m - mx);
    m = mx;
    const float p00 = exp2f(s[0][0] - m), p01 = exp2f(s[0][1] - m);
    const float p10 = exp2f(s[1][0] - m), p11 = exp2f(s[1][1] - m);
    l = l * alpha + (p00 + p01 + p10 + p11);
    const uint32_t pa0 = pack_half2(p00, p01), pa2 = pack_half2(p10, p11);
#pragma unroll
    for (int db = 0; db < D / 8; ++db) {
      o[db][0] *= alpha;
      o[db][1] *= alpha;
    }
#pragma unroll
    for (int db = 0; db < D / 8; db += 2) {
      uint32_t b0, b1, b2, b3;
      const int key = (lane & 7) + ((lane >> 3) & 1) * 8;
      ldsm_x4_t(vb + page_off<D>(key, db + (lane >> 4)), b0, b1, b2, b3);
      mma16816(o[db], pa0, 0u, pa2, 0u, b0, b1);
      mma16816(o[db + 1], pa0, 0u, pa2, 0u, b2, b3);
    }
    __syncwarp();  // every lane is done with this stage before it is refilled
    if (c.q == c.pages - 1 || i == n - 1) {
      // This warp's piece of the stream (c.r, c.kvh) is complete.
      float lt = l;
      lt += __shfl_xor_sync(0xffffffffu, lt, 1);
      lt += __shfl_xor_sync(0xffffffffu, lt, 2);
      const long long f0 = c.cum * hkv + static_cast<long long>(c.kvh) * c.pages;
      const int w0 = static_cast<int>(((f0 + 1) * W - 1) / total);
      const int w1 = static_cast<int>(((f0 + c.pages) * W - 1) / total);
      __half* out = a.out + static_cast<size_t>(c.t) * a.ld_out + static_cast<size_t>(c.kvh) * G * D;
      const int stream = c.r * hkv + c.kvh;
      // The warp that holds the stream's first page records which warps hold
      // its pieces, for the merge pass (every stream, every launch).
      if (w == w0 && lane == 0) a.counters[stream] = w0 | (w1 << 16);
      if (w0 == w1) {  // the whole stream in this warp: normalise and store
        if (g < G) {
          const float inv = 1.0f / lt;
#pragma unroll
          for (int db = 0; db < D / 8; ++db)
            *reinterpret_cast<__half2*>(out + g * D + db * 8 + (lane & 3) * 2) =
                __floats2half2_rn(o[db][0] * inv, o[db][1] * inv);
        }
      } else if (g < G) {  // one piece of a split stream; the merge pass combines them
          const size_t piece = static_cast<size_t>(stream + w) * G + g;
          float* dst = a.part_o + piece * D;
#pragma unroll
          for (int db = 0; db < D / 8; ++db)
            *reinterpret_cast<float2*>(dst + db * 8 + (lane & 3) * 2) =
                make_float2(o[db][0], o[db][1]);
          if ((lane & 3) == 0)
            *reinterpret_cast<float2*>(a.part_ml + piece * 2) =
                make_float2(m * 0.6931471805599453f, lt);  // natural-log domain
      }
    }
    cursor_next(a, c);
  }
  // Pages still in flight land before the warp exits (only after a failed
  // wait; bounded).
  for (; i < issued; ++i) mbar_wait(&full[i % ST], (i / ST) & 1u, a.status);
}

// The merge pass of the balanced decode kernel: one CTA per (decode row, kv
// head) stream whose pages were split over several warps combines the pieces
// in warp order and stores the normalised heads.  A separate pass keeps the
// decode warps free of fences and arrival counters, whose round trips held up
// the warps that end a split stream.
template <int D>
__global__ void __launch_bounds__(128) decode_merge_kernel(const AttnArgs a) {
  const int lane = threadIdx.x & 31;
  const int stream = blockIdx.x;
  const int r = stream / a.hkv, kvh = stream % a.hkv;
  if (r >= a.rows || __ldg(a.row_count + r) != 1) return;
  const int t = __ldg(a.cu_seqlens + r);
  const int G = a.hq / a.hkv;
  griddep_enter();
  const int rec = __ldcg(a.counters + stream);
  const int w0 = rec & 0xffff, w1 = rec >> 16;
  if (w1 <= w0) return;
  if (w1 >= a.decode_ctas * 4) {  // not a record of this pass's warps
    if (lane == 0) atomicOr(a.status, kDevBadIndex);
    return;
  }
  __half* out = a.out + static_cast<size_t>(t) * a.ld_out + static_cast<size_t>(kvh) * G * D;
  decode_merge<D>(a, static_cast<size_t>(stream + w0) * G, w1 - w0 + 1, G, out, lane,
                  threadIdx.x >> 5, 4);
}

// One CTA per (decode row, query head): merge the row's splits.
__global__ void decode_combine_kernel(const AttnArgs a) {
  griddep_enter();
  const int r = blockIdx.x, h = blockIdx.y;
  if (a.row_count[r] != 1) return;
  const int s0 = a.cu_splits[r], ns = a.cu_splits[r + 1] - s0;
  const int d = a.dim;
  constexpr int kMaxW = 1024;
  __shared__ float w[kMaxW];
  __shared__ float red[32];
  // max of the split maxima
  float m = -INFINITY;
  for (int s = threadIdx.x; s < ns; s += blockDim.x)
    m = fmaxf(m, a.part_ml[(static_cast<size_t>(s0 + s) * a.hq + h) * 2]);
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  m = red[0];
  for (int i = 1; i < static_cast<int>(blockDim.x >> 5); ++i) m = fmaxf(m, red[i]);
  __syncthreads();
  // split weights exp(m_s - m) and the merged denominator
  float l = 0.f;
  for (int s = threadIdx.x; s < ns; s += blockDim.x) {
    const float* ml = a.part_ml + (static_cast<size_t>(s0 + s) * a.hq + h) * 2;
    const float ws = expf(ml[0] - m);
    if (s < kMaxW) w[s] = ws;
    l += ml[1] * ws;
  }
  l = warp_sum(l);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = l;
  __syncthreads();
  l = 0.f;
  for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) l += red[i];
  const float inv = 1.0f / l;
  const int t = a.cu_seqlens[r];
  const float* po = a.part_o + (static_cast<size_t>(s0) * a.hq + h) * d;
  const size_t sstride = static_cast<size_t>(a.hq) * d;
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    float o = 0.f;
#pragma unroll 8
    for (int s = 0; s < ns; ++s) {
      const float ws =
          s < kMaxW ? w[s] : expf(a.part_ml[(static_cast<size_t>(s0 + s) * a.hq + h) * 2] - m);
      o += po[s * sstride + i] * ws;
    }
    a.out[static_cast<size_t>(t) * a.ld_out + h * d + i] = __float2half_rn(o * inv);
  }
}

// ---------------------------------------------------------------- prefill
// Byte offset of 16-byte chunk c of row `row` in a [rows][DP] F16 tile, with an
// XOR swizzle over the low three chunk bits so ldmatrix rows hit distinct banks.
template <int DP>
__device__ __forceinline__ uint32_t tile_off(int row, int c) {
  const int sc = DP >= 64 ? (c ^ (row & 7)) : c;
  return static_cast<uint32_t>(row * DP * 2 + sc * 16);
}

constexpr int kPreRows = 128;    // query rows per CTA = tokens x heads of one GQA group
constexpr int kPreThreads = 256; // 8 warps, 16 query rows each

template <int DP, int KT>
struct PrefillShape {
  static constexpr int kRows = kPreRows;
  static constexpr uint32_t kQBytes = kRows * DP * 2;
  static constexpr uint32_t kKvBytes = KT * DP * 2;
  static constexpr uint32_t kSmem = kQBytes + 4 * kKvBytes;  // Q + 2 x (K, V); block table after
  static constexpr int kMinBlocks = DP <= 128 ? 2 : 1;      // resident CTAs per SM aimed for
  static constexpr int kChunks = DP / 8;                     // 16-byte chunks per row
  static constexpr int kLoads = KT * kChunks / kPreThreads;  // K (or V) chunks per thread
};

// Loads `rows` rows of a [*][d] F16 source into a swizzled [rows][DP] tile;
// row_src(i) gives the source row pointer or null (zero row).
template <int DP, class RowSrc>
__device__ __forceinline__ void load_tile(uint8_t* tile, int rows, int d, RowSrc row_src) {
  const int chunks = DP / 8;
  const uint32_t base = smem_u32(tile);
  const bool vec = (d % 8) == 0;
  for (int idx = threadIdx.x; idx < rows * chunks; idx += blockDim.x) {
    const int rr = idx / chunks, c = idx % chunks;
    const __half* src = row_src(rr);
    const uint32_t off = tile_off<DP>(rr, c);
    if (src && vec && c * 8 < d) {
      cp_async16(base + off, src + c * 8);
    } else {
      __half tmp[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int dim = c * 8 + e;
        tmp[e] = (src && dim < d) ? src[dim] : __float2half(0.f);
      }
      *reinterpret_cast<uint4*>(tile + off) = *reinterpret_cast<uint4*>(tmp);
    }
  }
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Causal flash attention over one (kv head, query tile, key split): 128 query
// rows = (tokens x heads of one GQA group), 8 warps of 16 rows, key tiles
// [kt0, kt1) of the row's context.  With one split the tile is normalised and
// stored; with several, each split stores its unnormalised rows and (m, l) and
// the last split to arrive merges them in split order (deterministic).
// Per-tile work is kept to the MMAs where possible: the causal mask only on
// tiles that reach past the first query's position, the output rescale only
// when some row's running maximum moved, the softmax scale folded into one
// FMA before ex2, and each thread's copy slots fixed for the whole loop.
template <int DP, int KT>
__global__ void __launch_bounds__(kPreThreads, PrefillShape<DP, KT>::kMinBlocks)
    prefill_attn_kernel(const AttnArgs a) {
  using S = PrefillShape<DP, KT>;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* qs = smem;
  uint8_t* ks[2] = {smem + S::kQBytes, smem + S::kQBytes + S::kKvBytes};
  uint8_t* vs[2] = {smem + S::kQBytes + 2 * S::kKvBytes, smem + S::kQBytes + 3 * S::kKvBytes};
  int32_t* stab = reinterpret_cast<int32_t*>(smem + S::kSmem);

  const int d = a.dim;
  const int G = a.hq / a.hkv;
  const int QT = a.qtile_tokens;
  const int kvh = blockIdx.x;
  const int tile = blockIdx.y;
  const int split = blockIdx.z, nsplit = gridDim.z;
  // The packer's tables are complete before this kernel starts.
  const int r = find_row(a.cu_qtiles, a.rows, tile);
  const int count = a.row_count[r];
  if (count <= 1) return;
  const int tok0 = (tile - a.cu_qtiles[r]) * QT;  // first local token of this tile
  const int first = a.row_first[r];
  const int ntok = min(QT, count - tok0);
  const int ctx_hi = first + tok0 + ntok;  // keys [0, ctx_hi)
  const int n_kt = (ctx_hi + KT - 1) / KT;
  const int kt0 = n_kt * split / nsplit, kt1 = n_kt * (split + 1) / nsplit;
  // This split's block-table entries (pages [pg0, pg1)) into shared memory.
  const int pg0 = kt0 * KT / 16;
  const int pg1 = min(min((kt1 * KT + 15) / 16, (ctx_hi + 15) / 16), a.max_blocks);
  {
    const int32_t* table = a.block_tables + static_cast<size_t>(r) * a.max_blocks;
    for (int p = pg0 + threadIdx.x; p < pg1; p += blockDim.x) stab[p - pg0] = table[p];
  }
  griddep_enter();
  const int t_base = a.cu_seqlens[r];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = warp * 16 + (lane >> 2), row1 = row0 + 8;
  float o[DP / 8][4];
#pragma unroll
  for (int i = 0; i < DP / 8; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[i][e] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

  if (kt0 < kt1) {
    // Q tile: query row qr = (token qr / G, head qr % G of this group).
    load_tile<DP>(qs, S::kRows, d, [&](int qr) -> const __half* {
      const int tl = qr / G, g = qr % G;
      if (tl >= ntok) return nullptr;
      return a.q + static_cast<size_t>(t_base + tok0 + tl) * a.hq * d + (kvh * G + g) * d;
    });
    __syncthreads();  // the block table in shared memory
    // Copy slots: chunk c of rows row_j = tid / kChunks + j * (threads / kChunks).
    const bool fast = d == DP && S::kLoads >= 1;
    const int cslot = threadIdx.x % S::kChunks;
    const int rslot = threadIdx.x / S::kChunks;
    auto load_kv = [&](int kt, int buf) {
      if (fast) {
        const uint32_t kb = smem_u32(ks[buf]), vb = smem_u32(vs[buf]);
#pragma unroll
        for (int j = 0; j < S::kLoads; ++j) {
          const int row = rslot + j * (kPreThreads / S::kChunks);
          const int key = kt * KT + row;
          const int pg = key >> 4;
          const int bid = (key < ctx_hi && pg < pg1) ? stab[pg - pg0] : -1;
          const uint32_t off = tile_off<DP>(row, cslot);
          if (bid >= 0) {
            const size_t src = ((static_cast<size_t>(bid) * a.hkv + kvh) * 16 + (key & 15)) * DP +
                               cslot * 8;
            cp_async16(kb + off, a.k_cache + src);
            cp_async16(vb + off, a.v_cache + src);
          } else {  // past the context (or a missing block): zeros, never NaN
            *reinterpret_cast<uint4*>(ks[buf] + off) = make_uint4(0, 0, 0, 0);
            *reinterpret_cast<uint4*>(vs[buf] + off) = make_uint4(0, 0, 0, 0);
          }
        }
      } else {
        auto kv_src = [&](const __half* cache, int key) -> const __half* {
          if (key >= ctx_hi || (key >> 4) >= pg1) return nullptr;
          const int bid = stab[(key >> 4) - pg0];
          if (bid < 0) return nullptr;
          return cache + ((static_cast<size_t>(bid) * a.hkv + kvh) * 16 + (key & 15)) * d;
        };
        load_tile<DP>(ks[buf], KT, d, [&](int i) { return kv_src(a.k_cache, kt * KT + i); });
        load_tile<DP>(vs[buf], KT, d, [&](int i) { return kv_src(a.v_cache, kt * KT + i); });
      }
    };
    load_kv(kt0, 0);
    cp_async_commit();

    const int pos0 = first + tok0 + row0 / G, pos1 = first + tok0 + row1 / G;
    const int pos_min = first + tok0;  // the tile's first query position
    const float sl2 = a.scale * kLog2e;
    const uint32_t q_base = smem_u32(qs);

    for (int kt = kt0; kt < kt1; ++kt) {
      const int buf = (kt - kt0) & 1;
      if (kt + 1 < kt1) {
        load_kv(kt + 1, buf ^ 1);
        cp_async_commit();
        cp_async_wait<1>();
      } else {
        cp_async_wait<0>();
      }
      __syncthreads();
      const uint32_t k_base = smem_u32(ks[buf]);
      const uint32_t v_base = smem_u32(vs[buf]);

      float s[KT / 8][4];
#pragma unroll
      for (int i = 0; i < KT / 8; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) s[i][e] = 0.f;
#pragma unroll
      for (int kk = 0; kk < DP / 16; ++kk) {
        uint32_t a0, a1, a2, a3;
        {
          const int rr = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int c = kk * 2 + (lane >> 4);
          ldsm_x4(q_base + tile_off<DP>(rr, c), a0, a1, a2, a3);
        }
#pragma unroll
        for (int nb = 0; nb < KT / 8; nb += 2) {
          uint32_t b0, b1, b2, b3;
          const int key = nb * 8 + (lane & 7) + (lane >> 4) * 8;
          const int c = kk * 2 + ((lane >> 3) & 1);
          ldsm_x4(k_base + tile_off<DP>(key, c), b0, b1, b2, b3);
          mma16816(s[nb], a0, a1, a2, a3, b0, b1);
          mma16816(s[nb + 1], a0, a1, a2, a3, b2, b3);
        }
      }
      // Causal mask, only where the tile reaches past the first query.
      if (kt * KT + KT - 1 > pos_min || kt * KT + KT > ctx_hi) {
#pragma unroll
        for (int nb = 0; nb < KT / 8; ++nb)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int key = kt * KT + nb * 8 + (lane & 3) * 2 + (e & 1);
            const int pos = e < 2 ? pos0 : pos1;
            if (key > pos || key >= ctx_hi) s[nb][e] = -INFINITY;
          }
      }
      // Online softmax in base 2: p = 2^(s * scale * log2 e - m).
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int nb = 0; nb < KT / 8; ++nb) {
        mx0 = fmaxf(mx0, fmaxf(s[nb][0], s[nb][1]));
        mx1 = fmaxf(mx1, fmaxf(s[nb][2], s[nb][3]));
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float n0 = fmaxf(m0, mx0 * sl2), n1 = fmaxf(m1, mx1 * sl2);
      // A split that starts after a row's position sees no key of that row
      // yet: its maximum stays -inf and the reference point 0 keeps every
      // exponential at exactly 0 (no inf - inf).
      const float r0 = n0 == -INFINITY ? 0.f : n0, r1 = n1 == -INFINITY ? 0.f : n1;
      const float al0 = ex2_approx(m0 - r0), al1 = ex2_approx(m1 - r1);
      m0 = n0;
      m1 = n1;
      float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
      for (int nb = 0; nb < KT / 8; ++nb) {
        s[nb][0] = ex2_approx(fmaf(s[nb][0], sl2, -r0));
        s[nb][1] = ex2_approx(fmaf(s[nb][1], sl2, -r0));
        s[nb][2] = ex2_approx(fmaf(s[nb][2], sl2, -r1));
        s[nb][3] = ex2_approx(fmaf(s[nb][3], sl2, -r1));
        rs0 += s[nb][0] + s[nb][1];
        rs1 += s[nb][2] + s[nb][3];
      }
      l0 = l0 * al0 + rs0;
      l1 = l1 * al1 + rs1;
      if (!__all_sync(0xffffffffu, al0 == 1.f && al1 == 1.f)) {
#pragma unroll
        for (int i = 0; i < DP / 8; ++i) {
          o[i][0] *= al0;
          o[i][1] *= al0;
          o[i][2] *= al1;
          o[i][3] *= al1;
        }
      }
      // O += P V.
#pragma unroll
      for (int k2 = 0; k2 < KT / 16; ++k2) {
        const uint32_t p0 = pack_half2(s[2 * k2][0], s[2 * k2][1]);
        const uint32_t p1 = pack_half2(s[2 * k2][2], s[2 * k2][3]);
        const uint32_t p2 = pack_half2(s[2 * k2 + 1][0], s[2 * k2 + 1][1]);
        const uint32_t p3 = pack_half2(s[2 * k2 + 1][2], s[2 * k2 + 1][3]);
#pragma unroll
        for (int db = 0; db < DP / 8; db += 2) {
          uint32_t b0, b1, b2, b3;
          const int key = k2 * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int c = db + (lane >> 4);
          ldsm_x4_t(v_base + tile_off<DP>(key, c), b0, b1, b2, b3);
          mma16816(o[db], p0, p1, p2, p3, b0, b1);
          mma16816(o[db + 1], p0, p1, p2, p3, b2, b3);
        }
      }
      __syncthreads();
    }
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const int tl0 = row0 / G, g0 = row0 % G, tl1 = row1 / G, g1 = row1 % G;
  if (nsplit == 1) {
    const float inv0 = 1.0f / l0, inv1 = 1.0f / l1;
    __half* out0 = tl0 < ntok ? a.out + static_cast<size_t>(t_base + tok0 + tl0) * a.ld_out +
                                    (kvh * G + g0) * d
                              : nullptr;
    __half* out1 = tl1 < ntok ? a.out + static_cast<size_t>(t_base + tok0 + tl1) * a.ld_out +
                                    (kvh * G + g1) * d
                              : nullptr;
#pragma unroll
    for (int db = 0; db < DP / 8; ++db) {
      const int dim = db * 8 + (lane & 3) * 2;
      if (dim < d) {
        if (out0) {
          out0[dim] = __float2half_rn(o[db][0] * inv0);
          if (dim + 1 < d) out0[dim + 1] = __float2half_rn(o[db][1] * inv0);
        }
        if (out1) {
          out1[dim] = __float2half_rn(o[db][2] * inv1);
          if (dim + 1 < d) out1[dim + 1] = __float2half_rn(o[db][3] * inv1);
        }
      }
    }
    return;
  }
  // Several splits: store this split's rows [64][DP] and (m, l) [64][2].
  const size_t cell = static_cast<size_t>(tile) * a.hkv + kvh;
  constexpr size_t kPiece = static_cast<size_t>(S::kRows) * (DP + 2);
  float* piece = a.pre_part + (cell * nsplit + split) * kPiece;
#pragma unroll
  for (int db = 0; db < DP / 8; ++db) {
    const int dim = db * 8 + (lane & 3) * 2;
    *reinterpret_cast<float2*>(piece + row0 * DP + dim) = make_float2(o[db][0], o[db][1]);
    *reinterpret_cast<float2*>(piece + row1 * DP + dim) = make_float2(o[db][2], o[db][3]);
  }
  if ((lane & 3) == 0) {
    float* ml = piece + S::kRows * DP;
    *reinterpret_cast<float2*>(ml + row0 * 2) = make_float2(m0, l0);
    *reinterpret_cast<float2*>(ml + row1 * 2) = make_float2(m1, l1);
  }
  __threadfence();
  __syncthreads();
  __shared__ int s_last;
  if (threadIdx.x == 0) {
    int* counter = a.pre_counters + cell;
    const int last = atomicAdd(counter, 1) == nsplit - 1;
    if (last) *counter = 0;
    s_last = last;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // Merge the splits of this tile in split order.
  const float* pieces = a.pre_part + cell * nsplit * kPiece;
  for (int idx = threadIdx.x; idx < S::kRows * (DP / 4); idx += blockDim.x) {
    const int row = idx / (DP / 4), c4 = (idx % (DP / 4)) * 4;
    const int tl = row / G, g = row % G;
    if (tl >= ntok || c4 >= d) continue;
    float M = -INFINITY;
    for (int sp = 0; sp < nsplit; ++sp)
      M = fmaxf(M, __ldcg(pieces + sp * kPiece + S::kRows * DP + row * 2));
    float L = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int sp = 0; sp < nsplit; ++sp) {
      const float* p = pieces + sp * kPiece;
      const float2 ml = __ldcg(reinterpret_cast<const float2*>(p + S::kRows * DP + row * 2));
      const float w = exp2f(ml.x - M);  // 0 for a split with no key of this row
      const float4 v = __ldcg(reinterpret_cast<const float4*>(p + row * DP + c4));
      L += ml.y * w;
      acc.x += v.x * w;
      acc.y += v.y * w;
      acc.z += v.z * w;
      acc.w += v.w * w;
    }
    const float inv = 1.0f / L;
    __half* dst = a.out + static_cast<size_t>(t_base + tok0 + tl) * a.ld_out + (kvh * G + g) * d + c4;
    const float vals[4] = {acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv};
#pragma unroll
    for (int e = 0; e < 4; ++e)
      if (c4 + e < d) dst[e] = __float2half_rn(vals[e]);
  }
}

template <int DP, int KT>
int prefill_setup(size_t table_bytes) {
  using S = PrefillShape<DP, KT>;
  static int per_sm = 0;
  static size_t configured_bytes = 0;
  const size_t smem = S::kSmem + table_bytes;
  if (smem > configured_bytes) {
    if (cudaFuncSetAttribute(prefill_attn_kernel<DP, KT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return 0;
    configured_bytes = smem;
    per_sm = 0;
  }
  if (per_sm == 0) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, prefill_attn_kernel<DP, KT>, kPreThreads, smem) !=
        cudaSuccess)
      return 0;
    per_sm = n > 0 ? n : 1;
  }
  return per_sm;
}

template <int DP, int KT>
cudaError_t launch_prefill(const AttnArgs& a, int total_qtiles, cudaStream_t stream) {
  using S = PrefillShape<DP, KT>;
  const size_t table = prefill_table_bytes(a);
  if (prefill_setup<DP, KT>(table) == 0) return cudaErrorInvalidValue;
  const int splits = a.prefill_splits > 0 ? a.prefill_splits : 1;
  if (splits > 1 && (!a.pre_part || !a.pre_counters)) return cudaErrorInvalidValue;
  return launch_dependent(prefill_attn_kernel<DP, KT>, dim3(a.hkv, total_qtiles, splits),
                          dim3(kPreThreads), S::kSmem + table, stream, a);
}

// Four warps' rings, their stage barriers and 1024 bytes of alignment slack.
template <int D>
size_t decode_mma_smem(int group) {
  return static_cast<size_t>(4) * dec_stages<D>() * (decode_stage_bytes(D, group) + 8) + 1024;
}

// Sets the kernel's shared-memory limit once and returns its resident CTAs per
// SM for a GQA group size (1..kMaxGroup), 0 on failure.
template <int D>
int decode_mma_setup(int group) {
  static bool configured = false;
  static int per_sm[kMaxGroup + 1] = {};
  if (group < 1 || group > kMaxGroup) return 0;
  if (!configured) {
    if (cudaFuncSetAttribute(decode_attn_mma_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(decode_mma_smem<D>(kMaxGroup))) != cudaSuccess)
      return 0;
    configured = true;
  }
  if (per_sm[group] == 0) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_attn_mma_kernel<D>, 128,
                                                      decode_mma_smem<D>(group)) != cudaSuccess)
      return 0;
    per_sm[group] = n > 0 ? n : 1;
  }
  return per_sm[group];
}

template <int D>
cudaError_t launch_decode_mma(const AttnArgs& a, const TcMaps& maps, cudaStream_t stream) {
  const int group = a.hq / a.hkv;
  if (a.decode_ctas <= 0 || decode_mma_setup<D>(group) == 0) return cudaErrorInvalidValue;
  const cudaError_t e = launch_dependent(decode_attn_mma_kernel<D>, dim3(a.decode_ctas), dim3(128),
                                         decode_mma_smem<D>(group), stream, maps, a);
  if (e != cudaSuccess) return e;
  const unsigned streams = static_cast<unsigned>(a.rows) * static_cast<unsigned>(a.hkv);
  return launch_dependent(decode_merge_kernel<D>, dim3(streams), dim3(128), 0, stream, a);
}

}  // namespace

int attn_qtile_tokens(int group) { return kPreRows / group; }

bool attn_decode_balanced(int dim) { return dim == 64 || dim == 128 || dim == 256; }

int attn_decode_ctas(int dim, int group, long long pages, int sm_count) {
  if (!attn_decode_balanced(dim) || pages <= 0) return 0;
  const int per_sm = dim == 64 ? decode_mma_setup<64>(group)
                     : dim == 128 ? decode_mma_setup<128>(group)
                                  : decode_mma_setup<256>(group);
  if (per_sm == 0) return 0;
  // One wave of resident CTAs, but at least ~8 pages per warp.
  const long long want = (pages + 31) / 32;
  return static_cast<int>(std::max<long long>(1, std::min<long long>(want, 1LL * per_sm * sm_count)));
}

size_t attn_decode_part_floats(int rows, int hq, int hkv, int dim, int ctas) {
  const size_t pieces = static_cast<size_t>(rows) * hkv + 4 * static_cast<size_t>(ctas);
  return pieces * static_cast<size_t>(hq / hkv) * static_cast<size_t>(dim + 2);
}

cudaError_t attn_decode_launch(const AttnArgs& a, const TcMaps& maps, int total_splits,
                               cudaStream_t stream) {
  if (total_splits <= 0) return cudaSuccess;
  const int G = a.hq / a.hkv;
  if (G > kMaxGroup || a.dim % 4 != 0 || a.dim > 256 || G * a.dim / 4 > 4 * kDecThreads ||
      a.split_tokens % 16 != 0)
    return cudaErrorInvalidValue;
  cudaError_t e;
  if (attn_decode_balanced(a.dim)) {
    e = a.dim == 64    ? launch_decode_mma<64>(a, maps, stream)
        : a.dim == 128 ? launch_decode_mma<128>(a, maps, stream)
                       : launch_decode_mma<256>(a, maps, stream);
  } else {
    // Other head sizes (e.g. the tiny fixtures): one CTA per (kv head, split).
    const size_t smem = kDecStages * 2 * 16 * a.dim * 2 +
                        (G * a.dim + 2 * G * 16 + 3 * kMaxGroup) * sizeof(float) + 8 +
                        kDecStages * sizeof(uint64_t);
    static bool configured = false;
    if (!configured) {
      e = cudaFuncSetAttribute(decode_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               96 * 1024);
      if (e != cudaSuccess) return e;
      configured = true;
    }
    e = launch_dependent(decode_attn_kernel, dim3(a.hkv, total_splits), dim3(kDecThreads), smem,
                         stream, a);
    if (e != cudaSuccess) return e;
    e = launch_dependent(decode_combine_kernel, dim3(a.rows, a.hq), dim3(128), 0, stream, a);
  }
  return e;
}

int attn_decode_launches(int) { return 2; }  // the pass and its merge / combine

cudaError_t attn_prefill_launch(const AttnArgs& a, int total_qtiles, cudaStream_t stream) {
  if (total_qtiles <= 0) return cudaSuccess;
  const int G = a.hq / a.hkv;
  if (G > kPreRows) return cudaErrorInvalidValue;
  if (a.prefill_splits > kPrefillMaxSplits) return cudaErrorInvalidValue;
  if (a.dim <= 16) return launch_prefill<16, 64>(a, total_qtiles, stream);
  if (a.dim <= 64) return launch_prefill<64, 64>(a, total_qtiles, stream);
  if (a.dim <= 128) return launch_prefill<128, 64>(a, total_qtiles, stream);
  if (a.dim <= 256) return launch_prefill<256, 32>(a, total_qtiles, stream);
  return cudaErrorInvalidValue;
}

size_t prefill_table_bytes(const AttnArgs& a) {
  return (static_cast<size_t>(a.max_blocks) * 4 + 15) & ~static_cast<size_t>(15);
}

int attn_prefill_padded_dim(int dim) {
  return dim <= 16 ? 16 : dim <= 64 ? 64 : dim <= 128 ? 128 : 256;
}

int attn_prefill_splits(int dim, int hkv, int total_qtiles, int sm_count, size_t table_bytes) {
  if (total_qtiles <= 0 || dim > 256) return 1;
  const int per_sm = dim <= 16    ? prefill_setup<16, 64>(table_bytes)
                     : dim <= 64  ? prefill_setup<64, 64>(table_bytes)
                     : dim <= 128 ? prefill_setup<128, 64>(table_bytes)
                                  : prefill_setup<256, 32>(table_bytes);
  const long long base = static_cast<long long>(hkv) * total_qtiles;
  const long long resident = static_cast<long long>(per_sm > 0 ? per_sm : 1) * sm_count;
  // Whole waves only: as many splits as still fit in one wave of resident CTAs.
  const long long s = resident / std::max<long long>(1, base);
  return static_cast<int>(std::max<long long>(1, std::min<long long>(s, kPrefillMaxSplits)));
}

size_t attn_prefill_part_floats(int dim, int hkv, int total_qtiles, int splits) {
  if (splits <= 1) return 0;
  const size_t dp = static_cast<size_t>(attn_prefill_padded_dim(dim));
  return static_cast<size_t>(total_qtiles) * hkv * splits * kPreRows * (dp + 2);
}

}  // namespace hb
