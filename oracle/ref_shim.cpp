// ref_shim.cpp -- a C entry layer over the reference's own CPU math.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together with
// the reference sources where they lie (cpp/src/cpu/llama.cpp, cpp/src/cpu/tensor.cpp,
// cpp/src/half.cpp, cpp/src/sampling.cpp, cpp/src/decode_batch.cpp) into
// oracle/_ref/libhllm_ref.so.  Tests use it to pin the C restatement in
// oracle/hllm_oracle.c, and bench.py's reference arm times it as the CPU
// baseline.  No reference source is copied: only its public headers are
// included and its functions called.
//
// Wrapped functions:
//   hllm::cpu::transformer_layer   cpp/src/cpu/llama.cpp:242
//   hllm::cpu::final_logits        cpp/src/cpu/llama.cpp:284
//   hllm::cpu::greedy_sample_last  cpp/src/cpu/llama.cpp:290
//   hllm::cpu::rms_norm / apply_rope / linear
//   hllm::runtime::sample_token    cpp/src/sampling.cpp:65
//   hllm::runtime::float_to_float16 / float16_to_float  cpp/src/half.cpp
//   hllm::runtime::combine_decode_inputs  cpp/src/decode_batch.cpp:8
//   hllm::runtime::validate_tensor_envelope, SequenceTracker  cpp/src/tensor_envelope.cpp
//
// cpp/src/safetensors.cpp (which also defines data_type_bytes) needs
// nlohmann/json and is not compiled; this file defines data_type_bytes with
// the element sizes of safetensors.hpp's DataType (the same table as
// safetensors.cpp:118-138) so that tensor_envelope.cpp links.
#include <cstdint>
#include <cstring>
#include <exception>
#include <memory>
#include <vector>

#include "hllm/cpu/llama.hpp"
#include "hllm/cpu/tensor.hpp"
#include "hllm/runtime/error.hpp"
#include "hllm/runtime/half.hpp"
#include "hllm/runtime/sampling.hpp"
#include "hllm/runtime/stage_backend.hpp"
#include "hllm/runtime/tensor_envelope.hpp"

namespace hllm::runtime {
std::size_t data_type_bytes(const DataType dtype) noexcept {
  switch (dtype) {
    case DataType::kBool: case DataType::kU8: case DataType::kI8: return 1U;
    case DataType::kI16: case DataType::kU16: case DataType::kF16: case DataType::kBF16: return 2U;
    case DataType::kI32: case DataType::kU32: case DataType::kF32: return 4U;
    case DataType::kI64: case DataType::kU64: case DataType::kF64: return 8U;
  }
  return 0U;
}
}  // namespace hllm::runtime

namespace {
using hllm::cpu::LayerKvCache;
using hllm::cpu::LayerWeights;
using hllm::cpu::LlamaConfig;
using hllm::cpu::Matrix;

struct RefConfig {
  std::uint64_t hidden_size, intermediate_size, attention_heads, key_value_heads,
      head_dimension, maximum_sequence_length;
  float rms_norm_epsilon, rope_theta;
  std::uint32_t query_key_norm;
};
struct RefLayer {
  const float *input_norm, *query, *key, *value, *attention_output, *post_attention_norm;
  const float *gate, *up, *down, *query_norm, *key_norm;
};
struct RefSampling {
  double temperature, top_p;
  std::uint64_t top_k, seed;
  std::uint32_t return_logprobs, top_logprobs;
};
struct RefSampled {
  std::uint64_t token_id;
  double logprob;
  std::uint32_t has_logprob, n_top;
  std::uint64_t top_ids[5];
  double top_logprobs[5];
};

LlamaConfig config(const RefConfig& c) {
  return {c.hidden_size, c.intermediate_size, c.attention_heads, c.key_value_heads,
          c.head_dimension, c.maximum_sequence_length, c.rms_norm_epsilon, c.rope_theta,
          c.query_key_norm != 0U};
}
Matrix matrix(const float* p, std::size_t rows, std::size_t cols) {
  return Matrix(rows, cols, std::vector<float>(p, p + rows * cols));
}
std::vector<float> vec(const float* p, std::size_t n) { return std::vector<float>(p, p + n); }

int status_of(const std::exception& e) {
  if (const auto* err = dynamic_cast<const hllm::runtime::Error*>(&e)) {
    return 1 + static_cast<int>(err->code());
  }
  return 100;
}
}  // namespace

extern "C" {

void* ref_cache_new(std::uint64_t capacity, std::uint64_t heads, std::uint64_t dim) {
  try {
    return new LayerKvCache(capacity, heads, dim);
  } catch (...) {
    return nullptr;
  }
}
void ref_cache_free(void* cache) { delete static_cast<LayerKvCache*>(cache); }
std::uint64_t ref_cache_length(void* cache) { return static_cast<LayerKvCache*>(cache)->length(); }
// Appends `rows` positions of keys and values ([rows][heads * dim] each) at the
// cache's end through the reference's own LayerKvCache::append; 0 on success.
int ref_cache_append(void* cache, std::uint64_t rows, const float* keys, const float* values) {
  try {
    auto* c = static_cast<LayerKvCache*>(cache);
    const std::size_t width = c->heads() * c->head_dimension();
    c->append(c->length(), matrix(keys, rows, width), matrix(values, rows, width));
    return 0;
  } catch (const std::exception& e) {
    return status_of(e);
  }
}
// Reads the cache as [length][heads][dim].
void ref_cache_read(void* cache, float* keys, float* values) {
  auto* c = static_cast<LayerKvCache*>(cache);
  std::size_t i = 0;
  for (std::size_t p = 0; p < c->length(); ++p)
    for (std::size_t h = 0; h < c->heads(); ++h)
      for (std::size_t d = 0; d < c->head_dimension(); ++d, ++i) {
        keys[i] = c->key(p, h, d);
        values[i] = c->value(p, h, d);
      }
}

int ref_transformer_layer(const float* input, std::uint64_t rows, const RefLayer* w,
                          const RefConfig* cfg, std::uint64_t first_position, void* cache,
                          float* output) {
  try {
    const auto c = config(*cfg);
    const auto h = c.hidden_size, I = c.intermediate_size;
    const auto qw = c.attention_heads * c.head_dimension;
    const auto kw = c.key_value_heads * c.head_dimension;
    LayerWeights weights{vec(w->input_norm, h),
                         matrix(w->query, qw, h),
                         matrix(w->key, kw, h),
                         matrix(w->value, kw, h),
                         matrix(w->attention_output, h, qw),
                         vec(w->post_attention_norm, h),
                         matrix(w->gate, I, h),
                         matrix(w->up, I, h),
                         matrix(w->down, h, I),
                         c.query_key_norm ? vec(w->query_norm, c.head_dimension)
                                          : std::vector<float>{},
                         c.query_key_norm ? vec(w->key_norm, c.head_dimension)
                                          : std::vector<float>{}};
    const auto out = hllm::cpu::transformer_layer(matrix(input, rows, h), weights, c,
                                                  first_position,
                                                  *static_cast<LayerKvCache*>(cache));
    std::memcpy(output, out.values().data(), sizeof(float) * out.size());
    return 0;
  } catch (const std::exception& e) {
    return status_of(e);
  }
}

// Persistent forms: the layer weights / LM head are converted into the
// reference's Matrix objects once, so that timing a call measures the
// reference's math rather than the shim's copies.
struct RefLayerHandle {
  LlamaConfig config;
  LayerWeights weights;
};
void* ref_layer_new(const RefLayer* w, const RefConfig* cfg) {
  try {
    const auto c = config(*cfg);
    const auto h = c.hidden_size, I = c.intermediate_size;
    const auto qw = c.attention_heads * c.head_dimension;
    const auto kw = c.key_value_heads * c.head_dimension;
    return new RefLayerHandle{
        c,
        LayerWeights{vec(w->input_norm, h), matrix(w->query, qw, h), matrix(w->key, kw, h),
                     matrix(w->value, kw, h), matrix(w->attention_output, h, qw),
                     vec(w->post_attention_norm, h), matrix(w->gate, I, h), matrix(w->up, I, h),
                     matrix(w->down, h, I),
                     c.query_key_norm ? vec(w->query_norm, c.head_dimension) : std::vector<float>{},
                     c.query_key_norm ? vec(w->key_norm, c.head_dimension) : std::vector<float>{}}};
  } catch (...) {
    return nullptr;
  }
}
void ref_layer_free(void* handle) { delete static_cast<RefLayerHandle*>(handle); }
int ref_layer_forward(void* handle, const float* input, std::uint64_t rows,
                      std::uint64_t first_position, void* cache, float* output) {
  try {
    auto* L = static_cast<RefLayerHandle*>(handle);
    const auto out = hllm::cpu::transformer_layer(matrix(input, rows, L->config.hidden_size),
                                                  L->weights, L->config, first_position,
                                                  *static_cast<LayerKvCache*>(cache));
    std::memcpy(output, out.values().data(), sizeof(float) * out.size());
    return 0;
  } catch (const std::exception& e) {
    return status_of(e);
  }
}
struct RefHeadHandle {
  std::vector<float> norm;
  Matrix head;
};
void* ref_head_new(const float* norm, const float* head, std::uint64_t vocab, std::uint64_t h) {
  try {
    return new RefHeadHandle{vec(norm, h), matrix(head, vocab, h)};
  } catch (...) {
    return nullptr;
  }
}
void ref_head_free(void* handle) { delete static_cast<RefHeadHandle*>(handle); }
int ref_head_logits(void* handle, const float* hidden, std::uint64_t rows, float eps,
                    float* logits) {
  try {
    auto* H = static_cast<RefHeadHandle*>(handle);
    const auto out = hllm::cpu::final_logits(matrix(hidden, rows, H->norm.size()), H->norm,
                                             H->head, eps);
    std::memcpy(logits, out.values().data(), sizeof(float) * out.size());
    return 0;
  } catch (const std::exception& e) {
    return status_of(e);
  }
}

int ref_final_logits(const float* hidden, std::uint64_t rows, std::uint64_t h,
                     const float* norm, const float* head, std::uint64_t vocab, float eps,
                     float* logits) {
  try {
    const auto out = hllm::cpu::final_logits(matrix(hidden, rows, h), vec(norm, h),
                                             matrix(head, vocab, h), eps);
    std::memcpy(logits, out.values().data(), sizeof(float) * out.size());
    return 0;
  } catch (const std::exception& e) {
    return status_of(e);
  }
}

long long ref_greedy_sample_last(const float* logits, std::uint64_t rows, std::uint64_t cols) {
  try {
    return static_cast<long long>(hllm::cpu::greedy_sample_last(matrix(logits, rows, cols)));
  } catch (...) {
    return -1;
  }
}

int ref_rms_norm(const float* in, const float* w, std::uint64_t rows, std::uint64_t cols,
                 float eps, float* out) {
  try {
    const auto r = hllm::cpu::rms_norm(matrix(in, rows, cols), vec(w, cols), eps);
    std::memcpy(out, r.values().data(), sizeof(float) * r.size());
    return 0;
  } catch (const std::exception& e) {
    return status_of(e);
  }
}

int ref_apply_rope(float* values, std::uint64_t rows, std::uint64_t heads, std::uint64_t dim,
                   std::uint64_t first_position, float theta) {
  try {
    auto m = matrix(values, rows, heads * dim);
    hllm::cpu::apply_rope(m, heads, dim, first_position, theta);
    std::memcpy(values, m.values().data(), sizeof(float) * m.size());
    return 0;
  } catch (const std::exception& e) {
    return status_of(e);
  }
}

int ref_linear(const float* x, std::uint64_t rows, std::uint64_t in, const float* w,
               std::uint64_t out, float* y) {
  try {
    const auto r = hllm::cpu::linear(matrix(x, rows, in), matrix(w, out, in));
    std::memcpy(y, r.values().data(), sizeof(float) * r.size());
    return 0;
  } catch (const std::exception& e) {
    return status_of(e);
  }
}

int ref_sample_token(const float* logits, std::uint64_t n, const RefSampling* o,
                     std::uint64_t generated_index, RefSampled* out) {
  std::memset(out, 0, sizeof(*out));
  try {
    hllm::runtime::SamplingOptions options{o->temperature, o->top_p, o->top_k, o->seed,
                                           o->return_logprobs != 0U, o->top_logprobs};
    const auto t = hllm::runtime::sample_token(std::span<const float>(logits, n), options,
                                               generated_index);
    out->token_id = t.id;
    if (t.logprob) {
      out->has_logprob = 1;
      out->logprob = *t.logprob;
    }
    out->n_top = static_cast<std::uint32_t>(t.top_logprobs.size());
    for (std::size_t i = 0; i < t.top_logprobs.size() && i < 5; ++i) {
      out->top_ids[i] = t.top_logprobs[i].token_id;
      out->top_logprobs[i] = t.top_logprobs[i].logprob;
    }
    return 0;
  } catch (const std::exception& e) {
    return status_of(e);
  }
}

std::uint16_t ref_float_to_float16(float v) { return hllm::runtime::float_to_float16(v); }
float ref_float16_to_float(std::uint16_t v) { return hllm::runtime::float16_to_float(v); }

// combine_decode_inputs over token inputs: `positions[i]`, `prefilling[i]`,
// `prefill_only[i]`, `same[i]` (index of a sequence shared with an earlier item,
// or -1).  Returns 0 and writes the combined ids, or the error status.
int ref_combine_decode_tokens(const std::uint64_t* ids, const std::uint64_t* counts,
                              const std::uint64_t* positions, const std::uint8_t* prefilling,
                              const std::uint8_t* prefill_only, const std::int32_t* same,
                              std::uint64_t n, std::uint64_t* out) {
  try {
    std::vector<std::unique_ptr<hllm::runtime::SequenceState>> states;
    std::atomic_bool cancelled{false};
    std::vector<hllm::runtime::DecodeBatchItem> items;
    std::size_t offset = 0;
    for (std::size_t i = 0; i < n; ++i) {
      hllm::runtime::SequenceState* state;
      if (same[i] >= 0) {
        state = states.at(static_cast<std::size_t>(same[i])).get();
        states.push_back(nullptr);
      } else {
        states.push_back(std::make_unique<hllm::runtime::SequenceState>());
        state = states.back().get();
        state->prefilling = prefilling[i] != 0U;
        state->prefill_only = prefill_only[i] != 0U;
      }
      hllm::runtime::TokenInput input{
          std::vector<std::uint64_t>(ids + offset, ids + offset + counts[i])};
      offset += counts[i];
      items.push_back({std::move(input), positions[i], state, &cancelled});
    }
    const auto combined = hllm::runtime::combine_decode_inputs(items);
    const auto& tokens = std::get<hllm::runtime::TokenInput>(combined);
    std::memcpy(out, tokens.ids.data(), sizeof(std::uint64_t) * tokens.ids.size());
    return 0;
  } catch (const std::exception& e) {
    return status_of(e);
  }
}

// runtime::validate_tensor_envelope on the metadata decode_tensor builds
// (F16, dense row-major; phase 0 prefill, 1 decode).  Returns 0 or the error
// status, and the exception message in `message`.
int ref_validate_envelope(std::uint32_t protocol_version, const char* deployment_id,
                          std::uint64_t deployment_version, const char* request_id,
                          std::uint64_t microbatch_id, std::uint64_t sequence_number,
                          std::uint32_t decode, std::uint64_t first_position,
                          const std::uint64_t* lengths, std::uint64_t n_lengths,
                          const std::uint64_t* slots, std::uint64_t n_slots,
                          const std::uint64_t* shape, std::uint64_t n_shape,
                          std::uint64_t payload_length, std::uint64_t received,
                          std::uint64_t maximum_batch, std::uint64_t maximum_sequence_length,
                          std::uint64_t hidden_size, std::uint64_t maximum_payload_bytes,
                          char* message, std::uint64_t message_size) {
  try {
    hllm::runtime::TensorEnvelopeMetadata m{
        protocol_version, deployment_id, deployment_version, request_id, microbatch_id,
        sequence_number,
        decode ? hllm::runtime::ExecutionPhase::kDecode : hllm::runtime::ExecutionPhase::kPrefill,
        first_position,
        std::vector<std::uint64_t>(lengths, lengths + n_lengths),
        std::vector<std::uint64_t>(slots, slots + n_slots),
        std::vector<std::uint64_t>(shape, shape + n_shape),
        hllm::runtime::DataType::kF16,
        hllm::runtime::TensorLayout::kDenseRowMajorLittleEndian,
        payload_length};
    hllm::runtime::TensorEnvelopeLimits limits{};
    limits.maximum_batch = maximum_batch;
    limits.maximum_sequence_length = maximum_sequence_length;
    limits.hidden_size = hidden_size;
    limits.maximum_payload_bytes = maximum_payload_bytes;
    hllm::runtime::validate_tensor_envelope(m, received, limits);
    return 0;
  } catch (const std::exception& e) {
    if (message && message_size) {
      std::strncpy(message, e.what(), message_size - 1);
      message[message_size - 1] = 0;
    }
    return status_of(e);
  }
}

// runtime::SequenceTracker: feeds `n` numbers; returns how many were accepted
// before the first rejection (n when all were).
std::uint64_t ref_sequence_tracker(const std::uint64_t* numbers, std::uint64_t n) {
  hllm::runtime::SequenceTracker tracker;
  for (std::uint64_t i = 0; i < n; ++i) {
    try {
      tracker.accept(numbers[i]);
    } catch (const std::exception&) {
      return i;
    }
  }
  return n;
}

}  // extern "C"
