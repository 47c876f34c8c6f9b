// b200_stage_backend.cpp -- see b200_stage_backend.hpp.
#include "b200_stage_backend.hpp"

#include <chrono>
#include <cstring>
#include <stdexcept>
#include <string>
#include <variant>

#include "hllm/runtime/error.hpp"

namespace hllm::b200 {
namespace {

std::string last_error() {
  char buffer[1024];
  hllm_b200_last_error(buffer, sizeof(buffer));
  return buffer;
}

hllm_b200_sampling to_abi(const runtime::SamplingOptions& o) {
  return {o.temperature, o.top_p, o.top_k, o.seed, o.return_logprobs ? 1U : 0U, o.top_logprobs};
}

runtime::SampledToken from_abi(const hllm_b200_sampled& s, bool logprobs) {
  runtime::SampledToken token{s.token_id};
  if (logprobs) {
    token.logprob = s.logprob;
    for (std::uint32_t i = 0; i < s.n_top; ++i)
      token.top_logprobs.push_back({s.top_ids[i], s.top_logprobs[i]});
  }
  return token;
}

}  // namespace

void throw_status(hllm_b200_status status) {
  const auto message = last_error();
  switch (status) {
    case HLLM_B200_INVALID_REQUEST: throw runtime::Error::invalid_request(message);
    case HLLM_B200_INCOMPATIBLE_WORKER: throw runtime::Error::incompatible_worker(message);
    case HLLM_B200_RESOURCE_EXHAUSTED: throw runtime::Error::resource_exhausted(message);
    case HLLM_B200_DEADLINE_EXCEEDED: throw runtime::Error::deadline_exceeded(message);
    case HLLM_B200_CANCELLED: throw runtime::Error::cancelled(message);
    default: throw runtime::Error::internal(message);
  }
}

B200Sequence::~B200Sequence() {
  if (stage && handle) hllm_b200_seq_free(stage, handle);
}

B200StageBackend::B200StageBackend(hllm_b200_stage* stage, bool first, bool final)
    : stage_(stage), first_(first), final_(final) {
  std::uint64_t weights = 0, hidden = 0, vocab = 0, max_tokens = 0;
  check(hllm_b200_stage_info(stage_, &weights, &hidden, &vocab, &max_tokens));
  hidden_ = hidden;
  vocab_ = vocab;
  max_tokens_ = max_tokens;
}

B200StageBackend::~B200StageBackend() { hllm_b200_stage_destroy(stage_); }

runtime::MemoryAmounts B200StageBackend::weight_memory() const {
  std::uint64_t weights = 0;
  check(hllm_b200_stage_info(stage_, &weights, nullptr, nullptr, nullptr));
  return {0U, weights, 0U, 0U};
}

runtime::SequenceMemory B200StageBackend::sequence_memory(std::size_t tokens,
                                                          std::size_t maximum_query_tokens) const {
  std::uint64_t cache = 0, workspace = 0;
  check(hllm_b200_sequence_memory(stage_, tokens, maximum_query_tokens, &cache, &workspace));
  // The device KV blocks live with the request; the step workspace is shared.
  const auto transport = runtime::request_transport_bytes(
      tokens, runtime::query_rows(tokens, maximum_query_tokens), hidden_);
  return {{transport, cache, 0U, 0U}, {0U, workspace, 0U, 0U}};
}

std::unique_ptr<runtime::SequenceState> B200StageBackend::allocate_sequence(
    std::size_t tokens) const {
  auto state = std::make_unique<B200Sequence>();
  state->stage = stage_;
  check(hllm_b200_seq_alloc(stage_, tokens, &state->handle));
  return state;
}

std::vector<runtime::StageOutput> B200StageBackend::run(
    std::vector<runtime::DecodeBatchItem>& items) const {
  std::scoped_lock lock(mutex_);
  std::vector<hllm_b200_row> rows(items.size());
  std::size_t samples = 0, tokens = 0;
  for (std::size_t i = 0; i < items.size(); ++i) {
    auto* seq = dynamic_cast<B200Sequence*>(items[i].sequence);
    if (!seq || seq->stage != stage_) {
      throw runtime::Error::invalid_request("sequence state does not belong to this stage");
    }
    auto& row = rows[i];
    row.sequence = seq->handle;
    row.first_position = items[i].position;
    if (const auto* t = std::get_if<runtime::TokenInput>(&items[i].input)) {
      if (!first_) throw runtime::Error::invalid_request("only stage zero accepts tokens");
      row.tokens = t->ids.size();
      row.token_ids = t->ids.data();
    } else {
      if (first_) throw runtime::Error::invalid_request("stage zero requires tokens");
      const auto& b = std::get<runtime::BoundaryActivation>(items[i].input);
      if (b.width != hidden_ || b.payload.size() != b.tokens * b.width * 2U) {
        throw runtime::Error::invalid_request("invalid boundary activation");
      }
      row.tokens = b.tokens;
      row.activations = reinterpret_cast<const std::uint16_t*>(b.payload.data());
    }
    row.sample = final_ && !seq->prefill_only ? 1U : 0U;
    row.sampling = to_abi(seq->sampling);
    row.generated_index = seq->generated_index;
    samples += row.sample;
    tokens += row.tokens;
  }
  std::vector<hllm_b200_sampled> sampled(samples ? samples : 1U);
  std::vector<std::uint16_t> boundary(final_ ? 0U : tokens * hidden_);
  check(hllm_b200_step(stage_, rows.data(), static_cast<std::uint32_t>(rows.size()),
                       sampled.data(), boundary.data()));
  std::vector<runtime::StageOutput> outputs;
  std::size_t k = 0, offset = 0;
  for (std::size_t i = 0; i < items.size(); ++i) {
    auto* seq = static_cast<B200Sequence*>(items[i].sequence);
    if (final_) {
      if (!rows[i].sample) {
        outputs.emplace_back(runtime::PrefillProgress{});
        continue;
      }
      const auto& o = seq->sampling;
      outputs.emplace_back(from_abi(sampled[k++], o.return_logprobs));
      // The greedy fast path consumes no draw (cpp/src/cpu/stage.cpp:165-166).
      if (!(o.temperature == 0.0 && !o.return_logprobs)) ++seq->generated_index;
    } else {
      runtime::BoundaryActivation out{rows[i].tokens, hidden_,
                                      std::vector<std::byte>(rows[i].tokens * hidden_ * 2U)};
      std::memcpy(out.payload.data(), boundary.data() + offset * hidden_, out.payload.size());
      offset += rows[i].tokens;
      outputs.emplace_back(std::move(out));
    }
  }
  return outputs;
}

runtime::StageOutput B200StageBackend::execute(runtime::StageInput input,
                                               std::size_t first_position,
                                               runtime::SequenceState& state,
                                               const std::atomic_bool& cancelled) const {
  if (cancelled.load()) throw runtime::Error::cancelled("request cancelled");
  std::vector<runtime::DecodeBatchItem> items;
  items.push_back({std::move(input), first_position, &state, &cancelled});
  auto outputs = run(items);
  if (cancelled.load()) throw runtime::Error::cancelled("request cancelled");
  return std::move(outputs.front());
}

std::vector<runtime::StageOutput> B200StageBackend::execute_decode_batch(
    std::vector<runtime::DecodeBatchItem> items) const {
  // The reference's batch rules (cpp/src/decode_batch.cpp:8-38) validate the
  // members; the combined input itself is not needed, the executor takes rows.
  static_cast<void>(runtime::combine_decode_inputs(items));
  return run(items);
}

std::vector<runtime::StageOutput> B200StageBackend::execute_mixed_batch(
    std::vector<runtime::DecodeBatchItem> items) const {
  return run(items);
}

runtime::StageOutput B200StageBackend::execute_profiled(runtime::StageInput input,
                                                        std::size_t first_position,
                                                        runtime::SequenceState& state,
                                                        const std::atomic_bool& cancelled,
                                                        runtime::ExecutionTiming& timing) const {
  // The reference's components (cpp/src/cuda/stage.cpp:394-454): input,
  // one "layer" per owned layer, then final norm / LM head / sampling or the
  // boundary output, timed with CUDA events on the stage stream.
  timing = {};
  check(hllm_b200_stage_component_timing(stage_, 1U));
  runtime::StageOutput output;
  try {
    output = execute(std::move(input), first_position, state, cancelled);
  } catch (...) {
    hllm_b200_stage_component_timing(stage_, 0U);
    throw;
  }
  std::uint32_t count = 0;
  check(hllm_b200_stage_components(stage_, nullptr, 0, &count));
  std::vector<hllm_b200_component_timing> parts(count);
  check(hllm_b200_stage_components(stage_, parts.data(), count, &count));
  check(hllm_b200_stage_component_timing(stage_, 0U));
  for (const auto& c : parts)
    timing.components.push_back(
        {c.component,
         c.layer_index >= 0 ? std::optional<std::size_t>(static_cast<std::size_t>(c.layer_index))
                            : std::nullopt,
         c.milliseconds});
  return output;
}

}  // namespace hllm::b200
