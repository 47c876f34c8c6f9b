// sampler.cu -- greedy / temperature / top-k / top-p sampling with logprobs.
//
// Reference: sample_logits / sample_token (cpp/src/sampling.cpp:19-90) and the
// greedy fast path greedy_sample_last (cpp/src/cpu/llama.cpp:290-308).
//
//   * greedy: first maximum wins (std::max_element); any non-finite logit is
//     refused (the row's status is set, the host raises an internal error).
//   * temperature > 0: the reference computes p_i = exp((l_i - max)/T) in
//     double, stable-sorts descending (ties: lower token id), truncates to
//     top-k, keeps the shortest prefix whose mass reaches top_p * total
//     (do-while, at least one), draws u in [0,1) from SplitMix64(seed +
//     phi*(index+1)) and scans the prefix subtracting p_i until the target
//     goes negative.  No sort is done here: p is monotone in the logit, so the
//     sorted order is the order of the 64-bit key (order-preserving logit bits
//     << 32 | ~index), and each cut (k-th element, top-p prefix end, drawn
//     element) is found by an 8-bit radix select over those keys that
//     accumulates probability mass per digit bucket.
//   * logprobs: l - max - log(sum exp(l - max)) in double; the top-n list is
//     ordered by (logprob desc, id asc).
// Mass sums run in a different order than the reference's sequential sums, so
// results can differ from it only when a cut falls within rounding error of a
// bucket boundary (probability ~1e-16 per draw).
#include <math.h>

#include "common.cuh"
#include "sampler.cuh"

namespace hb {
namespace {

constexpr int kThreads = 1024;

__device__ __forceinline__ uint64_t sort_key(float v, int i) {
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);  // order-preserving for finite floats
  return (static_cast<uint64_t>(b) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(i));
}
__device__ __forceinline__ int key_index(uint64_t k) {
  return static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(k & 0xFFFFFFFFu));
}

__device__ double block_sum_d(double v, double* sh) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    double w = sh[threadIdx.x];
    for (int o = 16; o > 0; o >>= 1) w += __shfl_xor_sync(0xffffffffu, w, o);
    if (threadIdx.x == 0) sh[0] = w;
  }
  __syncthreads();
  const double r = sh[0];
  __syncthreads();
  return r;
}

__device__ uint64_t block_max_u64(uint64_t v, uint64_t* sh) {
  for (int o = 16; o > 0; o >>= 1) {
    const uint64_t w = __shfl_xor_sync(0xffffffffu, v, o);
    v = w > v ? w : v;
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    uint64_t w = sh[threadIdx.x];
    for (int o = 16; o > 0; o >>= 1) {
      const uint64_t x = __shfl_xor_sync(0xffffffffu, w, o);
      w = x > w ? x : w;
    }
    if (threadIdx.x == 0) sh[0] = w;
  }
  __syncthreads();
  const uint64_t r = sh[0];
  __syncthreads();
  return r;
}

struct SelectShared {
  double mass[256];
  unsigned count[256];
  uint64_t prefix, mask, found;
  double above;
  unsigned long long count_above;
  int sel_count, fallback;
};

// Among elements with key >= floor_key, walking keys in descending order,
// returns the key of the first element at which the running total reaches the
// target: mode 0 -> count >= k; mode 1 -> mass >= thr; mode 2 -> mass > thr.
// If the total never reaches it, returns the smallest key >= floor_key.
// *mass_through receives the running mass including the returned element.
__device__ uint64_t radix_select(const float* lg, const double* p, int n, uint64_t floor_key,
                                 int mode, double thr, unsigned long long k, SelectShared& s,
                                 double* mass_through) {
  if (threadIdx.x == 0) {
    s.prefix = 0;
    s.mask = 0;
    s.above = 0.0;
    s.count_above = 0;
    s.fallback = 0;
    s.found = 0;
  }
  __syncthreads();
  for (int shift = 56; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) {
      s.mass[i] = 0.0;
      s.count[i] = 0;
    }
    __syncthreads();
    const uint64_t prefix = s.prefix, mask = s.mask;
    // Whole warps walk the row (trip counts equal across a warp).  Keys of
    // nearby logits share their high digits, so most of a warp's lanes often
    // hit one bucket: the lanes that agree with the warp's first live lane
    // add their mass through one shuffle reduction and one shared atomic.
    const int lane = static_cast<int>(threadIdx.x & 31);
    for (int base = static_cast<int>(threadIdx.x) - lane; base < n;
         base += static_cast<int>(blockDim.x)) {
      const int i = base + lane;
      int digit = -1;
      double pm = 0.0;
      if (i < n) {
        const uint64_t key = sort_key(lg[i], i);
        if (key >= floor_key && (key & mask) == prefix) {
          digit = static_cast<int>((key >> shift) & 255u);
          pm = p[i];
        }
      }
      const unsigned live = __ballot_sync(0xffffffffu, digit >= 0);
      if (live == 0) continue;
      const int d0 = __shfl_sync(0xffffffffu, digit, __ffs(live) - 1);
      const unsigned same = __ballot_sync(0xffffffffu, digit == d0);
      double agg = digit == d0 ? pm : 0.0;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) agg += __shfl_xor_sync(0xffffffffu, agg, o);
      if (lane == __ffs(same) - 1) {
        atomicAdd(&s.mass[d0], agg);
        atomicAdd(&s.count[d0], static_cast<unsigned>(__popc(same)));
      }
      if (digit >= 0 && digit != d0) {
        atomicAdd(&s.mass[digit], pm);
        atomicAdd(&s.count[digit], 1u);
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int sel = -1, lowest = -1;
      double above = s.above;
      unsigned long long ca = s.count_above;
      for (int dg = 255; dg >= 0; --dg) {
        const unsigned c = s.count[dg];
        if (c == 0) continue;
        lowest = dg;
        if (!s.fallback) {
          const double m = s.mass[dg];
          const bool hit = mode == 0 ? (ca + c >= k) : mode == 1 ? (above + m >= thr) : (above + m > thr);
          if (hit) { sel = dg; break; }
          above += m;
          ca += c;
        }
      }
      if (sel < 0) {  // never reached: continue toward the smallest key
        sel = lowest;
        s.fallback = 1;
        above = s.above;
        for (int dg = 255; dg > sel; --dg) above += s.mass[dg];
      }
      s.above = above;
      s.count_above = ca;
      s.prefix |= static_cast<uint64_t>(sel) << shift;
      s.mask |= static_cast<uint64_t>(255u) << shift;
      s.sel_count = static_cast<int>(s.count[sel]);
    }
    __syncthreads();
    if (s.sel_count == 1 || shift == 0) break;
  }
  // The bucket now holds exactly one element (or shift reached 0: the key is exact).
  {
    const uint64_t prefix = s.prefix, mask = s.mask;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const uint64_t key = sort_key(lg[i], i);
      if (key >= floor_key && (key & mask) == prefix) s.found = key;
    }
  }
  __syncthreads();
  const uint64_t key = s.found;
  *mass_through = s.above + p[key_index(key)];
  __syncthreads();
  return key;
}

__global__ void __launch_bounds__(kThreads)
    sample_kernel(const float* __restrict__ logits, int vocab, int ld,
                  const SampleParams* __restrict__ params, double* __restrict__ scratch,
                  SampleResult* __restrict__ out, uint32_t* status) {
  griddep_enter();
  __shared__ SelectShared sel;
  __shared__ double dsh[32];
  __shared__ uint64_t ush[32];
  __shared__ int bad_flag;
  const int r = blockIdx.x;
  const float* lg = logits + static_cast<size_t>(r) * ld;
  double* p = scratch + static_cast<size_t>(r) * vocab;
  const SampleParams P = params[r];
  SampleResult res{};
  if (threadIdx.x == 0) bad_flag = 0;
  __syncthreads();

  // Maximum key == (largest logit, lowest index among equals): the first maximum.
  uint64_t best = 0;
  bool bad = false;
  for (int i = threadIdx.x; i < vocab; i += blockDim.x) {
    const float v = lg[i];
    if (!isfinite(v)) bad = true;
    const uint64_t k = sort_key(v, i);
    best = k > best ? k : best;
  }
  if (bad) bad_flag = 1;
  best = block_max_u64(best, ush);
  if (bad_flag) {
    if (threadIdx.x == 0) {
      res.status = kDevNonFinite;
      out[r] = res;
      atomicOr(status, kDevNonFinite);
    }
    return;
  }
  const int argmax = key_index(best);
  const double mx = static_cast<double>(lg[argmax]);
  int64_t token = argmax;

  if (P.temperature != 0.0) {
    for (int i = threadIdx.x; i < vocab; i += blockDim.x)
      p[i] = exp((static_cast<double>(lg[i]) - mx) / P.temperature);
    __syncthreads();
    // Top-k: keep keys >= the k-th largest.
    uint64_t floor_key = 0;
    double dummy;
    if (P.top_k != 0 && P.top_k < static_cast<uint64_t>(vocab))
      floor_key = radix_select(lg, p, vocab, 0, 0, 0.0, P.top_k, sel, &dummy);
    double local = 0.0;
    for (int i = threadIdx.x; i < vocab; i += blockDim.x)
      if (sort_key(lg[i], i) >= floor_key) local += p[i];
    const double total = block_sum_d(local, dsh);
    const double threshold = total * P.top_p;
    double retained;
    const uint64_t cut = radix_select(lg, p, vocab, floor_key, 1, threshold, 0, sel, &retained);
    // SplitMix64 draw (cpp/src/sampling.cpp:52-57).
    uint64_t bits = P.seed + 0x9e3779b97f4a7c15ULL * (P.generated_index + 1u);
    bits = (bits ^ (bits >> 30)) * 0xbf58476d1ce4e5b9ULL;
    bits = (bits ^ (bits >> 27)) * 0x94d049bb133111ebULL;
    bits ^= bits >> 31;
    const double target = static_cast<double>(bits >> 11) * 0x1.0p-53 * retained;
    double through;
    const uint64_t drawn = radix_select(lg, p, vocab, cut, 2, target, 0, sel, &through);
    token = key_index(drawn);
  }

  if (P.return_logprobs) {
    double local = 0.0;
    for (int i = threadIdx.x; i < vocab; i += blockDim.x)
      local += exp(static_cast<double>(lg[i]) - mx);
    const double log_sum = log(block_sum_d(local, dsh));
    res.logprob = static_cast<double>(lg[token]) - mx - log_sum;
    const int n_top = static_cast<int>(P.top_logprobs < static_cast<uint32_t>(vocab)
                                           ? P.top_logprobs : static_cast<uint32_t>(vocab));
    uint64_t ceiling = ~0ull;
    for (int j = 0; j < n_top; ++j) {
      uint64_t b = 0;
      for (int i = threadIdx.x; i < vocab; i += blockDim.x) {
        const uint64_t k = sort_key(lg[i], i);
        if (k < ceiling && k > b) b = k;
      }
      b = block_max_u64(b, ush);
      const int id = key_index(b);
      res.top_ids[j] = id;
      res.top_logprobs[j] = static_cast<double>(lg[id]) - mx - log_sum;
      ceiling = b;
    }
    res.n_top = n_top;
  }
  if (threadIdx.x == 0) {
    res.token = token;
    out[r] = res;
  }
}

}  // namespace

cudaError_t sample_launch(const float* logits, int rows, int vocab, int ld,
                          const SampleParams* params, double* scratch, SampleResult* out,
                          uint32_t* status, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  return launch_dependent(sample_kernel, dim3(rows), dim3(kThreads), 0, stream, logits, vocab, ld,
                          params, scratch, out, status);
}

}  // namespace hb
