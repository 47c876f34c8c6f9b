// capi_kernels.cu -- device-pointer C entry points of the individual kernels
// (include/hllm_b200.h, "kernel entry points"): used by the parity tests and
// the per-operator benchmarks.  They launch exactly the kernels the stage
// executor launches.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "attention.cuh"
#include "common.cuh"
#include "gemm.cuh"
#include "hllm_b200.h"
#include "kernels.cuh"
#include "sampler.cuh"

namespace hb {
void set_last_error(const std::string& message);  // stage.cu
}

namespace {

void set_error(const std::string& m) { hb::set_last_error(m); }

hllm_b200_status cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return HLLM_B200_OK;
  set_error(cudaGetErrorString(e));
  return e == cudaErrorInvalidValue ? HLLM_B200_INVALID_REQUEST : HLLM_B200_INTERNAL;
}

// GEMM slot storage owned by the library, one per device, allocated on first
// use and kept until the process exits.
struct DeviceScratch {
  float* slots = nullptr;
  uint32_t* status = nullptr;
  int sm_count = 0;
};
std::mutex g_scratch_mutex;
std::map<int, DeviceScratch> g_scratch;

hllm_b200_status scratch_for_device(DeviceScratch* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  std::scoped_lock lock(g_scratch_mutex);
  DeviceScratch& s = g_scratch[dev];
  if (!s.slots) {
    e = cudaDeviceGetAttribute(&s.sm_count, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess)
      e = cudaMalloc(&s.slots, hb::gemm_max_slot_floats(s.sm_count) * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&s.status, 256);
    if (e == cudaSuccess) e = cudaMemset(s.status, 0, 256);
    if (e != cudaSuccess) {
      s.slots = nullptr;
      return cuda_status(e);
    }
  }
  *out = s;
  return HLLM_B200_OK;
}

}  // namespace

extern "C" {

hllm_b200_status hllm_b200_gemm(const void* w, uint64_t m, uint64_t k_pad, uint32_t pair,
                                uint64_t second_row, const void* x, uint64_t n, uint32_t epilogue,
                                void* y, uint64_t ldy, uint32_t bn, uint32_t grid, void* stream) {
  if (!w || !x || !y || m == 0 || n == 0 || k_pad == 0 || k_pad % 64 != 0 || epilogue > 3 ||
      (pair != 1 && pair != 2) || (pair == 2) != (epilogue == 3))
    return HLLM_B200_INVALID_REQUEST;
  hb::GemmWeight gw{};
  const int rows_total = pair == 2 ? static_cast<int>(second_row + m) : static_cast<int>(m);
  if (!hb::gemm_make_weight(&gw, w, rows_total, static_cast<int>(m), static_cast<int>(k_pad),
                            static_cast<int>(pair), static_cast<int>(second_row)))
    return HLLM_B200_INTERNAL;
  hb::GemmInput gx{};
  if (!hb::gemm_make_input(&gx, x, static_cast<int>(n), static_cast<int>(k_pad),
                           static_cast<int>(k_pad)))
    return HLLM_B200_INTERNAL;
  DeviceScratch sc;
  const hllm_b200_status st = scratch_for_device(&sc);
  if (st != HLLM_B200_OK) return st;
  const hb::GemmPlan plan = hb::gemm_plan(gw, static_cast<int>(n), sc.sm_count,
                                          static_cast<int>(bn), static_cast<int>(grid));
  // The scratch holds the partial sums of one CTA per SM; a grid override
  // larger than that would write past it.
  const size_t need = hb::gemm_slot_floats(plan, static_cast<int>(pair));
  if (need > hb::gemm_max_slot_floats(sc.sm_count)) {
    set_error("GEMM split needs " + std::to_string(need * 4) + " bytes of partial sums; the " +
              "library's scratch holds " + std::to_string(hb::gemm_max_slot_floats(sc.sm_count) * 4) +
              " (use at most one CTA per SM)");
    return HLLM_B200_RESOURCE_EXHAUSTED;
  }
  hb::GemmSlots slots{};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = hb::gemm_launch(gw, gx, static_cast<int>(n), plan, static_cast<int>(epilogue), y,
                                  static_cast<int>(ldy), sc.slots, &slots, sc.status,
                                  s);
  if (e == cudaSuccess && plan.stream_k)
    e = hb::gemm_finish_launch(slots, static_cast<int>(n), static_cast<int>(epilogue), y,
                               static_cast<int>(ldy), s);
  return cuda_status(e);
}

hllm_b200_status hllm_b200_rmsnorm(const float* x, uint64_t rows, uint64_t width, const float* w,
                                   float eps, uint16_t* out, uint64_t ld_out, void* stream) {
  return cuda_status(hb::rmsnorm_launch(x, static_cast<int>(rows), static_cast<int>(width), w, eps,
                                        reinterpret_cast<__half*>(out), static_cast<int>(ld_out),
                                        nullptr, static_cast<cudaStream_t>(stream)));
}

hllm_b200_status hllm_b200_pack(const int32_t* row_slot, const int32_t* row_first,
                                const int32_t* row_count, uint32_t rows, uint32_t tokens,
                                const int32_t* slot_blocks, uint32_t max_blocks,
                                uint32_t split_tokens, uint32_t qtile_tokens, int32_t* cu_seqlens,
                                int32_t* positions, int32_t* slot_mapping, int32_t* token_row,
                                int32_t* seq_lens, int32_t* block_tables, int32_t* cu_splits,
                                int32_t* cu_qtiles, uint32_t* status, void* stream) {
  if (split_tokens == 0 || qtile_tokens == 0) return HLLM_B200_INVALID_REQUEST;
  hb::StepTensors s{};
  s.row_slot = row_slot;
  s.row_first = row_first;
  s.row_count = row_count;
  s.cu_seqlens = cu_seqlens;
  s.positions = positions;
  s.slot_mapping = slot_mapping;
  s.token_row = token_row;
  s.seq_lens = seq_lens;
  s.block_tables = block_tables;
  s.cu_splits = cu_splits;
  s.cu_qtiles = cu_qtiles;
  s.rows = static_cast<int>(rows);
  s.tokens = static_cast<int>(tokens);
  s.max_blocks = static_cast<int>(max_blocks);
  s.split_tokens = static_cast<int>(split_tokens);
  s.qtile_tokens = static_cast<int>(qtile_tokens);
  return cuda_status(hb::pack_launch(s, slot_blocks, status, static_cast<cudaStream_t>(stream)));
}

uint32_t hllm_b200_attention_qtile_tokens(uint32_t group) {
  return group ? static_cast<uint32_t>(hb::attn_qtile_tokens(static_cast<int>(group))) : 0u;
}

hllm_b200_status hllm_b200_attention(const uint16_t* q, const uint16_t* k_cache,
                                     const uint16_t* v_cache, const int32_t* row_first,
                                     const int32_t* row_count, const int32_t* cu_seqlens,
                                     const int32_t* seq_lens, const int32_t* block_tables,
                                     const int32_t* cu_splits, const int32_t* cu_qtiles,
                                     uint32_t rows, uint32_t total_splits, uint32_t total_qtiles,
                                     uint32_t hq, uint32_t hkv, uint32_t dim, uint32_t max_blocks,
                                     uint32_t split_tokens, uint16_t* out, uint64_t ld_out,
                                     uint64_t q_tokens, uint64_t kv_blocks, uint32_t* status,
                                     void* stream) {
  if (hkv == 0 || hq % hkv != 0 || dim == 0) return HLLM_B200_INVALID_REQUEST;
  hb::AttnArgs a{};
  a.q = reinterpret_cast<const __half*>(q);
  a.k_cache = reinterpret_cast<const __half*>(k_cache);
  a.v_cache = reinterpret_cast<const __half*>(v_cache);
  a.row_count = row_count;
  a.row_first = row_first;
  a.cu_seqlens = cu_seqlens;
  a.seq_lens = seq_lens;
  a.block_tables = block_tables;
  a.cu_splits = cu_splits;
  a.cu_qtiles = cu_qtiles;
  a.rows = static_cast<int>(rows);
  a.hq = static_cast<int>(hq);
  a.hkv = static_cast<int>(hkv);
  a.dim = static_cast<int>(dim);
  a.max_blocks = static_cast<int>(max_blocks);
  a.split_tokens = static_cast<int>(split_tokens);
  a.qtile_tokens = hb::attn_qtile_tokens(static_cast<int>(hq / hkv));
  a.scale = 1.0f / std::sqrt(static_cast<float>(dim));
  a.out = reinterpret_cast<__half*>(out);
  a.ld_out = static_cast<int>(ld_out);
  a.status = status;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int dev = 0, sm_count = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return cuda_status(e);
  // Decode: the balanced pass (head sizes 64/128/256) sizes its grid from the
  // pages the splits cover (an upper bound of the decode rows' pages).
  size_t part_floats = 0;
  if (total_splits) {
    const long long pages = static_cast<long long>(total_splits) *
                            ((split_tokens + 15) / 16) * static_cast<long long>(hkv);
    a.decode_ctas = hb::attn_decode_ctas(static_cast<int>(dim), static_cast<int>(hq / hkv), pages,
                                         sm_count);
    part_floats = std::max(static_cast<size_t>(total_splits) * hq * (dim + 2),
                           hb::attn_decode_part_floats(static_cast<int>(rows), static_cast<int>(hq),
                                                       static_cast<int>(hkv),
                                                       static_cast<int>(dim), a.decode_ctas));
  }
  // Prefill: tcgen05 tiles where the stage uses them (head sizes 64/128, and
  // HLLM_B200_TC_PREFILL not 0), else the mma.sync kernel; key splits per
  // tile, merged by the last split of each tile.
  const char* env = std::getenv("HLLM_B200_TC_PREFILL");
  const bool tc = total_qtiles && q_tokens && kv_blocks &&
                  hb::attn_prefill_tc_supported(static_cast<int>(dim), static_cast<int>(hq / hkv)) &&
                  !(env && env[0] == '0');
  hb::TcMaps maps{};
  // The balanced decode pass reads its pages through TMA maps of the caches.
  if (total_splits && hb::attn_decode_balanced(static_cast<int>(dim))) {
    if (!kv_blocks) {
      set_error("decode attention needs kv_blocks (the caches' extent)");
      return HLLM_B200_INVALID_REQUEST;
    }
    if (!hb::attn_make_kv_maps(&maps, static_cast<int>(hkv), static_cast<int>(dim), k_cache,
                               v_cache, static_cast<long long>(kv_blocks))) {
      set_error("tensor map creation failed");
      return HLLM_B200_INTERNAL;
    }
  }
  if (tc && !hb::attn_tc_make_maps(&maps, q, static_cast<long long>(q_tokens), static_cast<int>(hq),
                                   static_cast<int>(hkv), static_cast<int>(dim), k_cache, v_cache,
                                   static_cast<long long>(kv_blocks))) {
    set_error("tensor map creation failed");
    return HLLM_B200_INTERNAL;
  }
  a.prefill_splits = !total_qtiles ? 1
                     : tc          ? hb::attn_prefill_tc_splits(static_cast<int>(hkv),
                                                                static_cast<int>(total_qtiles),
                                                                sm_count)
                                   : hb::attn_prefill_splits(static_cast<int>(dim),
                                                             static_cast<int>(hkv),
                                                             static_cast<int>(total_qtiles),
                                                             sm_count, hb::prefill_table_bytes(a));
  const size_t pre_floats = hb::attn_prefill_part_floats(
      static_cast<int>(dim), static_cast<int>(hkv), static_cast<int>(total_qtiles), a.prefill_splits);
  if (part_floats || pre_floats) {
    // Split outputs live in a grow-only buffer per device, kept for the
    // process: a fixed block of ints at its head (decode: one warp-range record
    // per (row, kv head) in the first half, written by each decode pass;
    // prefill: one arrival counter per (tile, kv head) in the second half,
    // zeroed on allocation and returned to zero by the kernels), then the
    // decode pieces, then the prefill pieces.
    static std::mutex mu;
    static std::map<int, std::pair<float*, size_t>> buffers;
    constexpr size_t kCounters = 1 << 16;
    if (static_cast<size_t>(rows) * hkv > kCounters / 2 ||
        static_cast<size_t>(total_qtiles) * hkv > kCounters / 2)
      return HLLM_B200_INVALID_REQUEST;
    const size_t need = kCounters + part_floats + pre_floats;
    float* base = nullptr;
    {
      std::scoped_lock lock(mu);
      auto& buf = buffers[dev];
      if (buf.second < need) {
        if (buf.first) {
          cudaStreamSynchronize(st);
          cudaFree(buf.first);
        }
        buf = {nullptr, 0};
        e = cudaMalloc(&buf.first, need * sizeof(float));
        if (e == cudaSuccess) e = cudaMemset(buf.first, 0, need * sizeof(float));
        if (e != cudaSuccess) return cuda_status(e);
        buf.second = need;
      }
      base = buf.first;
    }
    a.counters = reinterpret_cast<int*>(base);
    a.pre_counters = reinterpret_cast<int*>(base) + kCounters / 2;
    a.part_o = base + kCounters;
    // part_ml after the larger of the two decode layouts' part_o extents.
    a.part_ml = a.part_o + part_floats / (dim + 2) * dim;
    a.pre_part = base + kCounters + part_floats;
  }
  if (total_splits) {
    e = hb::attn_decode_launch(a, maps, static_cast<int>(total_splits), st);
    if (e != cudaSuccess) return cuda_status(e);
  }
  return cuda_status(tc ? hb::attn_prefill_tc_launch(maps, a, static_cast<int>(total_qtiles), st)
                        : hb::attn_prefill_launch(a, static_cast<int>(total_qtiles), st));
}

hllm_b200_status hllm_b200_qkv_post(const float* qkv, uint64_t tokens, uint32_t hq, uint32_t hkv,
                                    uint32_t dim, const int32_t* positions,
                                    const int32_t* slot_mapping, const float* q_norm,
                                    const float* k_norm, float eps, const float* rope_pow,
                                    uint16_t* q_out, uint16_t* k_cache, uint16_t* v_cache,
                                    void* stream) {
  hb::QkvPostArgs a{};
  a.qkv = qkv;
  a.tokens = static_cast<int>(tokens);
  a.hq = static_cast<int>(hq);
  a.hkv = static_cast<int>(hkv);
  a.dim = static_cast<int>(dim);
  a.positions = positions;
  a.slot_mapping = slot_mapping;
  a.q_norm = q_norm;
  a.k_norm = k_norm;
  a.eps = eps;
  a.rope_pow = rope_pow;
  a.q_out = reinterpret_cast<__half*>(q_out);
  a.k_cache = reinterpret_cast<__half*>(k_cache);
  a.v_cache = reinterpret_cast<__half*>(v_cache);
  return cuda_status(hb::qkv_post_launch(a, static_cast<cudaStream_t>(stream)));
}

hllm_b200_status hllm_b200_sample(const float* logits, uint32_t rows, uint64_t vocab, uint64_t ld,
                                  const hllm_b200_sampling* options,
                                  const uint64_t* generated_index, hllm_b200_sampled* out,
                                  void* stream) {
  if (!logits || !options || !out || rows == 0 || vocab == 0 || ld < vocab)
    return HLLM_B200_INVALID_REQUEST;
  for (uint32_t i = 0; i < rows; ++i) {
    const auto& o = options[i];
    if (!std::isfinite(o.temperature) || o.temperature < 0.0 || o.temperature > 100.0 ||
        !std::isfinite(o.top_p) || o.top_p <= 0.0 || o.top_p > 1.0 || o.top_logprobs > 5U ||
        (!o.return_logprobs && o.top_logprobs != 0U)) {
      set_error("invalid sampling parameters");
      return HLLM_B200_INVALID_REQUEST;
    }
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  std::vector<hb::SampleParams> params(rows);
  for (uint32_t i = 0; i < rows; ++i)
    params[i] = hb::SampleParams{options[i].temperature, options[i].top_p, options[i].top_k,
                                 options[i].seed, generated_index ? generated_index[i] : 0,
                                 options[i].return_logprobs, options[i].top_logprobs};
  hb::SampleParams* dp = nullptr;
  hb::SampleResult* dr = nullptr;
  double* scratch = nullptr;
  uint32_t* status = nullptr;
  cudaError_t e = cudaMalloc(&dp, rows * sizeof(hb::SampleParams));
  if (e == cudaSuccess) e = cudaMalloc(&dr, rows * sizeof(hb::SampleResult));
  if (e == cudaSuccess) e = cudaMalloc(&scratch, static_cast<size_t>(rows) * vocab * sizeof(double));
  if (e == cudaSuccess) e = cudaMalloc(&status, 4);
  if (e == cudaSuccess) e = cudaMemsetAsync(status, 0, 4, st);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(dp, params.data(), rows * sizeof(hb::SampleParams), cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess)
    e = hb::sample_launch(logits, static_cast<int>(rows), static_cast<int>(vocab),
                          static_cast<int>(ld), dp, scratch, dr, status, st);
  std::vector<hb::SampleResult> res(rows);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(res.data(), dr, rows * sizeof(hb::SampleResult), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  cudaFree(dp);
  cudaFree(dr);
  cudaFree(scratch);
  cudaFree(status);
  if (e != cudaSuccess) return cuda_status(e);
  hllm_b200_status code = HLLM_B200_OK;
  for (uint32_t i = 0; i < rows; ++i) {
    out[i].token_id = static_cast<uint64_t>(res[i].token);
    out[i].logprob = res[i].logprob;
    out[i].has_logprob = options[i].return_logprobs ? 1u : 0u;
    out[i].n_top = static_cast<uint32_t>(res[i].n_top);
    for (int k = 0; k < 5; ++k) {
      out[i].top_ids[k] = static_cast<uint64_t>(res[i].top_ids[k]);
      out[i].top_logprobs[k] = res[i].top_logprobs[k];
    }
    if (res[i].status != 0) {
      set_error("cannot sample nonfinite logits");
      code = HLLM_B200_INTERNAL;
    }
  }
  return code;
}

hllm_b200_status hllm_b200_synth_matrix(uint64_t seed, uint64_t tag, uint64_t rows, uint64_t cols,
                                        uint64_t ld, float stddev, uint16_t* out, void* stream) {
  return cuda_status(hb::synth_matrix_launch(seed, tag, static_cast<int>(rows),
                                             static_cast<int>(cols), static_cast<int>(ld), stddev,
                                             reinterpret_cast<__half*>(out),
                                             static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
