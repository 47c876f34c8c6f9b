// kernels.cu -- packer, embedding, norms, q/k-norm + RoPE + paged-KV write,
// boundary conversion and synthetic initialisation for the stage executor.
#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "kernels.cuh"

namespace hb {
namespace {

// ---------------------------------------------------------------- packer
// One CTA per row.  The reference has no packer (it keeps one contiguous
// cache per sequence, cpp/src/cpu/llama.cpp:152-191, cpp/src/cuda/stage.cpp:72-83,
// and loops attention over batch members, cpp/src/cuda/stage.cpp:326-333);
// this kernel's contract is restated on the host by oracle_pack.
__global__ void pack_kernel(StepTensors s, const int32_t* __restrict__ slot_blocks,
                            uint32_t* status) {
  const int r = blockIdx.x;
  __shared__ int s_off, s_split;
  __shared__ int s_qt;
  if (threadIdx.x == 0) {
    int off = 0, sp = 0, qt = 0;
    for (int i = 0; i < r; ++i) {
      const int c = s.row_count[i];
      off += c;
      if (c == 1) sp += (s.row_first[i] + 1 + s.split_tokens - 1) / s.split_tokens;
      else qt += (c + s.qtile_tokens - 1) / s.qtile_tokens;
    }
    s_off = off;
    s_split = sp;
    s_qt = qt;
  }
  __syncthreads();
  const int first = s.row_first[r], count = s.row_count[r], slot = s.row_slot[r];
  const int ctx = first + count;
  const int need = (ctx + kBlockTokens - 1) / kBlockTokens;
  const int32_t* list = slot_blocks + static_cast<size_t>(slot) * s.max_blocks;
  if (threadIdx.x == 0) {
    s.cu_seqlens[r + 1] = s_off + count;
    if (r == 0) s.cu_seqlens[0] = 0;
    s.seq_lens[r] = ctx;
    const int splits = count == 1 ? (ctx + s.split_tokens - 1) / s.split_tokens : 0;
    const int qtiles = count == 1 ? 0 : (count + s.qtile_tokens - 1) / s.qtile_tokens;
    s.cu_splits[r + 1] = s_split + splits;
    s.cu_qtiles[r + 1] = s_qt + qtiles;
    if (r == 0) {
      s.cu_splits[0] = 0;
      s.cu_qtiles[0] = 0;
    }
    if (need > s.max_blocks) atomicOr(status, kDevBadIndex);
  }
  for (int b = threadIdx.x; b < s.max_blocks; b += blockDim.x) {
    const int v = b < need ? list[b] : -1;
    if (b < need && v < 0) atomicOr(status, kDevBadIndex);
    s.block_tables[static_cast<size_t>(r) * s.max_blocks + b] = v;
  }
  for (int i = threadIdx.x; i < count; i += blockDim.x) {
    const int t = s_off + i;
    const int pos = first + i;
    const int blk = pos / kBlockTokens < s.max_blocks ? list[pos / kBlockTokens] : -1;
    s.positions[t] = pos;
    s.slot_mapping[t] = blk < 0 ? -1 : blk * kBlockTokens + pos % kBlockTokens;
    s.token_row[t] = r;
  }
}

// ---------------------------------------------------------------- embedding
__global__ void embed_kernel(const int32_t* __restrict__ ids, const __half* __restrict__ emb,
                             int vocab, int hidden, int ld, float* __restrict__ out,
                             uint32_t* status) {
  griddep_enter();
  const int t = blockIdx.x;
  const int id = ids[t];
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0) atomicOr(status, kDevBadIndex);
    return;
  }
  const __half* row = emb + static_cast<size_t>(id) * ld;
  for (int c = threadIdx.x; c < hidden; c += blockDim.x)
    out[static_cast<size_t>(t) * hidden + c] = __half2float(row[c]);
}

__global__ void boundary_in_kernel(const __half* __restrict__ in, size_t n,
                                   float* __restrict__ out, uint32_t* status) {
  griddep_enter();
  bool bad = false;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const float v = __half2float(in[i]);
    bad |= !isfinite(v);
    out[i] = v;
  }
  if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) atomicOr(status, kDevNonFiniteInput);
}

__global__ void boundary_out_kernel(const float* __restrict__ in, size_t n,
                                    __half* __restrict__ out, uint32_t* status) {
  griddep_enter();
  bool bad = false;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const __half h = __float2half_rn(in[i]);
    bad |= !isfinite(__half2float(h));
    out[i] = h;
  }
  if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) atomicOr(status, kDevNonFinite);
}

// ---------------------------------------------------------------- RMSNorm
// cpp/src/cpu/llama.cpp:193-212: x * (1 / sqrt(mean(x^2) + eps)) * w.
__global__ void rmsnorm_kernel(const float* __restrict__ x, int width,
                               const float* __restrict__ w, float eps, __half* __restrict__ out,
                               int ld_out, const int32_t* __restrict__ row_index) {
  griddep_enter();
  const int r = blockIdx.x;
  const int src = row_index ? row_index[r] : r;
  const float* xr = x + static_cast<size_t>(src) * width;
  float ss = 0.f;
  for (int c = threadIdx.x; c < width; c += blockDim.x) ss += xr[c] * xr[c];
  __shared__ float red[32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float inv = 1.0f / sqrtf(red[0] / static_cast<float>(width) + eps);
  __half* o = out + static_cast<size_t>(r) * ld_out;
  for (int c = threadIdx.x; c < width; c += blockDim.x) o[c] = __float2half_rn(xr[c] * inv * w[c]);
}

// ---------------------------------------------------------------- q/k/v epilogue
// cpp/src/cpu/llama.cpp:255-264: optional per-head RMSNorm of q and k with one
// shared weight (normalize_heads, :114-130), then half-rotation RoPE
// (apply_rope, :214-240), then the K/V append (:264) -- here a scatter into
// 16-token blocks of the paged pool: element (slot, head, i) lives at
// ((slot/16 * Hkv + head) * 16 + slot%16) * d + i.
constexpr int kQkvWarps = 4;
constexpr int kMaxHeadDim = 256;

__global__ void __launch_bounds__(kQkvWarps * 32)
    qkv_post_kernel(QkvPostArgs a) {
  __shared__ __align__(16) float buf[kQkvWarps][kMaxHeadDim];
  constexpr int kPairs = kMaxHeadDim / 64;  // rotation pairs (i, i + d/2) per lane
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int d = a.dim, half = d / 2;
  const int heads = a.hq + 2 * a.hkv;
  const int h = blockIdx.y * kQkvWarps + warp;  // one head per warp
  const bool is_q = h < a.hq, is_k = !is_q && h < a.hq + a.hkv;
  // Up to the dependency wait only the packer's tables and fixed weights are
  // read: the position, the cache slot, this lane's rotation angles and norm
  // weights.
  const int ipos = a.positions[t];
  const int slot = a.slot_mapping[t];
  const float* nw = is_q ? a.q_norm : (is_k ? a.k_norm : nullptr);
  float rc[kPairs], rs[kPairs], w0[kPairs], w1[kPairs];
  if (h < heads && (is_q || is_k)) {
    const bool table = a.rope_table && ipos < a.rope_positions;
#pragma unroll
    for (int k = 0; k < kPairs; ++k) {
      const int i = lane + 32 * k;
      rc[k] = 1.f;
      rs[k] = 0.f;
      w0[k] = w1[k] = 1.f;
      if (i < half) {
        if (table) {
          const float2 cs = a.rope_table[static_cast<size_t>(ipos) * half + i];
          rc[k] = cs.x;
          rs[k] = cs.y;
        } else {
          const float angle = static_cast<float>(ipos) / a.rope_pow[i];
          rc[k] = cosf(angle);
          rs[k] = sinf(angle);
        }
        if (nw) {
          w0[k] = nw[i];
          w1[k] = nw[half + i];
        }
      }
    }
  }
  griddep_enter();
  if (h >= heads || slot < 0) return;  // a missing block: the packer has already flagged it
  const float* row = a.qkv + static_cast<size_t>(t) * heads * d;
  float* x = buf[warp];
  float ss = 0.f;
  for (int i = lane * 4; i < d; i += 128) {  // d % 4 == 0 (checked at stage creation)
    const float4 v = a.from_slots ? gemm_slot_sum4(a.slots, t, h * d + i, 0)
                                  : *reinterpret_cast<const float4*>(row + h * d + i);
    *reinterpret_cast<float4*>(x + i) = v;
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  ss = warp_sum(ss);
  __syncwarp();
  if (!is_q && !is_k) {  // value head: stored as projected
    const int kvh = h - a.hq - a.hkv;
    __half* dst = a.v_cache + ((static_cast<size_t>(slot / 16) * a.hkv + kvh) * 16 + slot % 16) * d;
    for (int i = lane * 2; i < d; i += 64)
      *reinterpret_cast<__half2*>(dst + i) = __floats2half2_rn(x[i], x[i + 1]);
    return;
  }
  const float inv = nw ? 1.0f / sqrtf(ss / static_cast<float>(d) + a.eps) : 1.f;
  __half* dst;
  if (is_q) {
    dst = a.q_out + static_cast<size_t>(t) * a.hq * d + static_cast<size_t>(h) * d;
  } else {
    const int kvh = h - a.hq;
    dst = a.k_cache + ((static_cast<size_t>(slot / 16) * a.hkv + kvh) * 16 + slot % 16) * d;
  }
#pragma unroll
  for (int k = 0; k < kPairs; ++k) {
    const int i = lane + 32 * k;
    if (i < half) {
      const float p0 = x[i] * (inv * w0[k]), p1 = x[half + i] * (inv * w1[k]);
      dst[i] = __float2half_rn(p0 * rc[k] - p1 * rs[k]);
      dst[half + i] = __float2half_rn(p1 * rc[k] + p0 * rs[k]);
    }
  }
}

// ---------------------------------------------------------------- residual + norm
// One CTA per token: add the projection's slots into the F32 residual stream,
// then RMSNorm the updated row into the next GEMM's F16 input.  EARLY_W is the
// decode-width form: a CTA of width/4 threads (one float4 of the row each)
// reads its norm weights before the dependency wait and keeps eight slot
// loads in flight -- a shorter chain for a few rows, at a register and thread
// cost that would lower occupancy when the rows take several waves.
template <bool EARLY_W>
__global__ void residual_norm_kernel(float* __restrict__ hidden, int width, GemmSlots slots,
                                     int has_slots, const float* __restrict__ w, float eps,
                                     __half* __restrict__ out, int ld_out) {
  const int t = blockIdx.x;
  float* xr = hidden + static_cast<size_t>(t) * width;
  __half* o = out + static_cast<size_t>(t) * ld_out;
  __shared__ float red[32];
  auto block_sum = [&](float v) {
    v = warp_sum(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x < 32) {
      float r = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
      r = warp_sum(r);
      if (threadIdx.x == 0) red[0] = r;
    }
    __syncthreads();
    return red[0];
  };
  constexpr int kVec = 4;  // float4 groups a thread keeps in registers
  if ((width & 3) == 0 && width <= static_cast<int>(blockDim.x) * 4 * kVec) {
    // A warp covers 128 consecutive features = one GEMM tile row; the row
    // stays in registers between the sum of squares and the output.
    float4 g[kVec];
    if (EARLY_W) {
#pragma unroll
      for (int k = 0; k < kVec; ++k) {
        const int c = (threadIdx.x + k * blockDim.x) * 4;
        g[k] = w && c < width ? *reinterpret_cast<const float4*>(w + c)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    griddep_enter();
    float4 v[kVec];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < kVec; ++k) {
      const int c = (threadIdx.x + k * blockDim.x) * 4;
      if (c < width) {
        v[k] = *reinterpret_cast<const float4*>(xr + c);
        if (has_slots) {
          const float4 a =
              EARLY_W ? gemm_slot_sum4<8>(slots, t, c, 0) : gemm_slot_sum4(slots, t, c, 0);
          v[k].x += a.x;
          v[k].y += a.y;
          v[k].z += a.z;
          v[k].w += a.w;
          *reinterpret_cast<float4*>(xr + c) = v[k];
        }
        ss += v[k].x * v[k].x + v[k].y * v[k].y + v[k].z * v[k].z + v[k].w * v[k].w;
      }
    }
    if (!w) return;
    const float inv = 1.0f / sqrtf(block_sum(ss) / static_cast<float>(width) + eps);
#pragma unroll
    for (int k = 0; k < kVec; ++k) {
      const int c = (threadIdx.x + k * blockDim.x) * 4;
      if (c < width) {
        if (!EARLY_W) g[k] = *reinterpret_cast<const float4*>(w + c);
        const __half2 lo = __floats2half2_rn(v[k].x * inv * g[k].x, v[k].y * inv * g[k].y);
        const __half2 hi = __floats2half2_rn(v[k].z * inv * g[k].z, v[k].w * inv * g[k].w);
        *reinterpret_cast<__half2*>(o + c) = lo;
        *reinterpret_cast<__half2*>(o + c + 2) = hi;
      }
    }
    return;
  }
  griddep_enter();
  float ss = 0.f;
  for (int c = threadIdx.x; c < width; c += blockDim.x) {
    float v = xr[c];
    if (has_slots) {
      v += gemm_slot_sum(slots, t, c, 0);
      xr[c] = v;
    }
    ss += v * v;
  }
  if (!w) return;
  const float inv = 1.0f / sqrtf(block_sum(ss) / static_cast<float>(width) + eps);
  for (int c = threadIdx.x; c < width; c += blockDim.x) o[c] = __float2half_rn(xr[c] * inv * w[c]);
}

// cpp/src/cpu/llama.cpp:274-280: (g / (1 + exp(-g))) * u.
__global__ void swiglu_kernel(GemmSlots slots, __half* __restrict__ act, int ld_act) {
  griddep_enter();
  const int t = blockIdx.y;
  __half* out = act + static_cast<size_t>(t) * ld_act;
  if ((slots.m & 3) == 0) {
    for (int i = (blockIdx.x * blockDim.x + threadIdx.x) * 4; i < slots.m;
         i += gridDim.x * blockDim.x * 4) {
      const float4 g = gemm_slot_sum4(slots, t, i, 0);
      const float4 u = gemm_slot_sum4(slots, t, i, 1);
      out[i] = __float2half_rn((g.x / (1.0f + expf(-g.x))) * u.x);
      out[i + 1] = __float2half_rn((g.y / (1.0f + expf(-g.y))) * u.y);
      out[i + 2] = __float2half_rn((g.z / (1.0f + expf(-g.z))) * u.z);
      out[i + 3] = __float2half_rn((g.w / (1.0f + expf(-g.w))) * u.w);
    }
    return;
  }
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < slots.m; i += gridDim.x * blockDim.x) {
    const float g = gemm_slot_sum(slots, t, i, 0);
    const float u = gemm_slot_sum(slots, t, i, 1);
    out[i] = __float2half_rn((g / (1.0f + expf(-g))) * u);
  }
}

__global__ void last_token_kernel(const int32_t* cu, const int32_t* rows, int count, int32_t* idx) {
  griddep_enter();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < count) idx[i] = cu[rows[i] + 1] - 1;
}

// ---------------------------------------------------------------- synthetic weights
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
  return z ^ (z >> 31);
}
__device__ __forceinline__ uint64_t synth_hash(uint64_t seed, uint64_t tag, uint64_t index) {
  return mix64(seed * 0xd1b54a32d192ed03ULL + tag * 0x9e3779b97f4a7c15ULL + index);
}

__global__ void synth_matrix_kernel(uint64_t seed, uint64_t tag, int rows, int cols, int ld,
                                    float unit, __half* out) {
  const size_t n = static_cast<size_t>(rows) * cols;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const uint64_t h = synth_hash(seed, tag, i);
    const int32_t s = static_cast<int32_t>((h & 0xffffu) + ((h >> 16) & 0xffffu) +
                                           ((h >> 32) & 0xffffu) + (h >> 48)) -
                      131070;
    const size_t r = i / cols, c = i % cols;
    out[r * ld + c] = __float2half_rn(__fmul_rn(static_cast<float>(s), unit));
  }
}

__global__ void synth_norm_kernel(uint64_t seed, uint64_t tag, int n, float unit, float* out) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const uint64_t h = synth_hash(seed, tag, static_cast<uint64_t>(i));
    const int32_t s = static_cast<int32_t>(h & 0xffffu) - 32768;
    const float v = __fadd_rn(1.0f, __fmul_rn(static_cast<float>(s), unit));
    out[i] = __half2float(__float2half_rn(v));
  }
}

int grid_for(size_t n, int threads) {
  const size_t g = (n + threads - 1) / threads;
  return static_cast<int>(g < 148 * 16 ? (g == 0 ? 1 : g) : 148 * 16);
}

}  // namespace

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("HLLM_B200_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

cudaError_t pack_launch(const StepTensors& s, const int32_t* slot_blocks, uint32_t* status,
                        cudaStream_t stream) {
  if (s.rows <= 0) return cudaErrorInvalidValue;
  pack_kernel<<<s.rows, 128, 0, stream>>>(s, slot_blocks, status);
  return cudaGetLastError();
}

cudaError_t embed_launch(const int32_t* ids, int tokens, const __half* embedding, int vocab,
                         int hidden, int ld_embedding, float* out, uint32_t* status,
                         cudaStream_t stream) {
  return launch_dependent(embed_kernel, dim3(tokens), dim3(256), 0, stream, ids, embedding, vocab,
                          hidden, ld_embedding, out, status);
}

cudaError_t boundary_in_launch(const __half* in, int tokens, int hidden, float* out,
                               uint32_t* status, cudaStream_t stream) {
  const size_t n = static_cast<size_t>(tokens) * hidden;
  return launch_dependent(boundary_in_kernel, dim3(grid_for(n, 256)), dim3(256), 0, stream, in, n,
                          out, status);
}

cudaError_t boundary_out_launch(const float* hidden, int tokens, int width, __half* out,
                                uint32_t* status, cudaStream_t stream) {
  const size_t n = static_cast<size_t>(tokens) * width;
  return launch_dependent(boundary_out_kernel, dim3(grid_for(n, 256)), dim3(256), 0, stream, hidden,
                          n, out, status);
}

cudaError_t rmsnorm_launch(const float* x, int rows, int width, const float* w, float eps,
                           __half* out, int ld_out, const int32_t* row_index,
                           cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  const int threads = width >= 1024 ? 512 : (width >= 256 ? 256 : 64);
  return launch_dependent(rmsnorm_kernel, dim3(rows), dim3(threads), 0, stream, x, width, w, eps,
                          out, ld_out, row_index);
}

cudaError_t qkv_post_launch(const QkvPostArgs& a, cudaStream_t stream) {
  if (a.dim > kMaxHeadDim || (a.dim & 1)) return cudaErrorInvalidValue;
  const int heads = a.hq + 2 * a.hkv;
  const dim3 grid(static_cast<unsigned>(a.tokens),
                  static_cast<unsigned>((heads + kQkvWarps - 1) / kQkvWarps));
  return launch_dependent(qkv_post_kernel, grid, dim3(kQkvWarps * 32), 0, stream, a);
}

cudaError_t residual_norm_launch(float* hidden, int tokens, int width, const GemmSlots* slots,
                                 const float* norm, float eps, __half* out, int ld_out,
                                 cudaStream_t stream) {
  if (tokens <= 0) return cudaSuccess;
  GemmSlots s{};
  if (slots) s = *slots;
  const int threads = tokens <= 128 && (width & 3) == 0 && width <= 4096
                          ? std::max(64, (width / 4 + 31) / 32 * 32)
                          : (width >= 1024 ? 512 : (width >= 256 ? 256 : 64));
  return launch_dependent(tokens <= 128 ? residual_norm_kernel<true> : residual_norm_kernel<false>,
                          dim3(tokens), dim3(threads), 0, stream, hidden,
                          width, s, slots ? 1 : 0, norm, eps, out, ld_out);
}

cudaError_t swiglu_launch(const GemmSlots& slots, int tokens, __half* act, int ld_act,
                          cudaStream_t stream) {
  if (tokens <= 0) return cudaSuccess;
  const int per_block = (slots.m & 3) == 0 ? 1024 : 256;
  const dim3 grid(static_cast<unsigned>((slots.m + per_block - 1) / per_block),
                  static_cast<unsigned>(tokens));
  return launch_dependent(swiglu_kernel, grid, dim3(256), 0, stream, slots, act, ld_act);
}

cudaError_t last_token_launch(const int32_t* cu_seqlens, const int32_t* sample_rows, int count,
                              int32_t* idx, cudaStream_t stream) {
  if (count <= 0) return cudaSuccess;
  return launch_dependent(last_token_kernel, dim3((count + 127) / 128), dim3(128), 0, stream,
                          cu_seqlens, sample_rows, count, idx);
}

cudaError_t synth_matrix_launch(uint64_t seed, uint64_t tag, int rows, int cols, int ld,
                                float stddev, __half* out, cudaStream_t stream) {
  const float unit = stddev / 37837.2f;
  synth_matrix_kernel<<<grid_for(static_cast<size_t>(rows) * cols, 256), 256, 0, stream>>>(
      seed, tag, rows, cols, ld, unit, out);
  return cudaGetLastError();
}

cudaError_t synth_norm_launch(uint64_t seed, uint64_t tag, int n, float spread, float* out,
                              cudaStream_t stream) {
  const float unit = spread / 32768.0f;
  synth_norm_kernel<<<grid_for(n, 256), 256, 0, stream>>>(seed, tag, n, unit, out);
  return cudaGetLastError();
}

}  // namespace hb
