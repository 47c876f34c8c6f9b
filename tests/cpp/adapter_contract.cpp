// adapter_contract.cpp -- the B200 stage behind hLLM's own runtime types.
//
// Built by tests/cpp/Makefile against the reference headers and sources
// (runtime/stage_backend.hpp, decode_batch.cpp, worker/scheduler.cpp) and
// libhllm_b200.so; run by tests/test_gpu_adapter.py on a B200.
//
//  1. The decode-batch contract of tests/cpp/decode_batch_contract.hpp:8-47 in
//     the reference: a ragged batch (lengths 7, 2, 4, 1) run through
//     execute_decode_batch equals serial execute: same tokens, logprobs within
//     0.02, same generated_index; greedy and seeded sampling.
//  2. The reference's StageScheduler (cpp/src/worker/scheduler.cpp) driving the
//     backend from concurrent request threads: every request's tokens equal a
//     serial run's, and the scheduler formed decode batches of at most 8.
//  3. (`adapter_contract mixed`) MixedStageScheduler
//     (hllm_b200/adapter/mixed_scheduler.cpp) driving the backend from
//     concurrent requests with chunked prompts: mixed prefill + decode passes
//     form, and every request's greedy tokens equal a serial run's up to the
//     first near-tie (top-2 logprob gap below 1e-2).
//  4. (`adapter_contract reference`) The reference's own contract headers,
//     compiled from the reference tree with gtest_shim/ for GoogleTest's
//     assertion macros: decode_batch_contract (tests/cpp/decode_batch_contract.hpp)
//     on the two-layer stage, and paired_timing_contract
//     (tests/cpp/profiling_contract.hpp) on a first stage (layer 0) and a final
//     stage (layer 1): execute_profiled outputs equal execute's, components run
//     from "embedding" to "to-wire" and from "from-wire" to "sampling", with
//     the right layer indices.
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <latch>
#include <memory>
#include <string>
#include <thread>
#include <variant>
#include <vector>

#include "b200_stage_backend.hpp"
#include "hllm/worker/scheduler.hpp"
#include "mixed_scheduler.hpp"
#include "decode_batch_contract.hpp"
#include "profiling_contract.hpp"

using namespace hllm;

namespace {
int failures = 0;
#define EXPECT(cond, ...)                        \
  do {                                           \
    if (!(cond)) {                               \
      ++failures;                                \
      std::printf("FAIL %s:%d ", __FILE__, __LINE__); \
      std::printf(__VA_ARGS__);                  \
      std::printf("\n");                         \
    }                                            \
  } while (0)

std::unique_ptr<b200::B200StageBackend> make_stage(std::uint64_t seed, std::uint64_t start = 0,
                                                   std::uint64_t end = 2, bool first = true,
                                                   bool final = true) {
  hllm_b200_stage_desc d{};
  d.hidden_size = 256;
  d.intermediate_size = 688;
  d.attention_heads = 4;
  d.key_value_heads = 2;
  d.head_dimension = 64;
  d.maximum_sequence_length = 256;
  d.rms_norm_epsilon = 1e-6F;
  d.rope_theta = 1e6F;
  d.query_key_norm = 1;
  d.vocabulary_size = 4096;
  d.layer_start = start;
  d.layer_end = end;
  d.first = first ? 1 : 0;
  d.final = final ? 1 : 0;
  d.tied_head = 1;
  d.device_id = 0;
  d.kv_pool_tokens = 8192;
  d.max_step_tokens = 512;
  d.max_step_rows = 64;
  d.max_sequences = 64;
  hllm_b200_stage* stage = nullptr;
  b200::check(hllm_b200_stage_create(&d, &stage));
  b200::check(hllm_b200_stage_init_synthetic(stage, seed));
  b200::check(hllm_b200_stage_finalize(stage));
  return std::make_unique<b200::B200StageBackend>(stage, first, final);
}

void decode_batch_case(runtime::StageBackend& stage, double temperature) {
  std::atomic_bool cancelled{false};
  std::vector<std::unique_ptr<runtime::SequenceState>> reference, batched;
  const std::vector<std::size_t> lengths{7, 2, 4, 1};
  std::vector<runtime::SampledToken> expected;
  for (std::size_t i = 0; i < lengths.size(); ++i) {
    reference.push_back(stage.allocate_sequence(lengths[i] + 1U));
    batched.push_back(stage.allocate_sequence(lengths[i] + 1U));
    for (auto* state : {reference.back().get(), batched.back().get()}) {
      state->sampling = {temperature, 0.95, 8, i + 42U, true, 3};
      static_cast<void>(stage.execute(
          runtime::TokenInput{std::vector<std::uint64_t>(lengths[i], 1U)}, 0U, *state, cancelled));
    }
    expected.push_back(std::get<runtime::SampledToken>(
        stage.execute(runtime::TokenInput{{4U}}, lengths[i], *reference.back(), cancelled)));
  }
  std::vector<runtime::DecodeBatchItem> items;
  for (std::size_t i = 0; i < lengths.size(); ++i)
    items.push_back({runtime::TokenInput{{4U}}, lengths[i], batched[i].get(), &cancelled});
  const auto actual = stage.execute_decode_batch(std::move(items));
  EXPECT(actual.size() == expected.size(), "batch size");
  for (std::size_t i = 0; i < expected.size() && i < actual.size(); ++i) {
    const auto& token = std::get<runtime::SampledToken>(actual[i]);
    EXPECT(token.id == expected[i].id, "token %zu: %llu vs %llu", i,
           static_cast<unsigned long long>(token.id),
           static_cast<unsigned long long>(expected[i].id));
    EXPECT(token.logprob && expected[i].logprob &&
               std::abs(*token.logprob - *expected[i].logprob) < 0.02,
           "logprob %zu", i);
    EXPECT(token.top_logprobs.size() == 3U, "top logprobs %zu", i);
    EXPECT(batched[i]->generated_index == reference[i]->generated_index, "generated_index %zu", i);
  }
}

std::vector<std::uint64_t> run_request(runtime::StageBackend& stage,
                                       worker::StageScheduler* scheduler,
                                       const std::vector<std::uint64_t>& prompt, int steps) {
  std::atomic_bool cancelled{false};
  auto state = stage.allocate_sequence(prompt.size() + steps);
  std::vector<std::uint64_t> out;
  std::vector<std::uint64_t> input = prompt;
  std::size_t position = 0;
  const auto deadline = std::chrono::system_clock::now() + std::chrono::minutes(5);
  for (int s = 0; s < steps; ++s) {
    runtime::StageOutput result =
        scheduler ? scheduler->execute(stage, runtime::TokenInput{input}, position, *state,
                                       cancelled, deadline)
                  : stage.execute(runtime::TokenInput{input}, position, *state, cancelled);
    const auto token = std::get<runtime::SampledToken>(result).id;
    out.push_back(token);
    position += input.size();
    input = {token};
  }
  return out;
}
}  // namespace

// Concurrent requests with chunked prompts through MixedStageScheduler against
// the same requests run serially.  Greedy, with the top two logprobs: where a
// concurrent token differs from the serial one, the serial top-2 gap must be
// below 1e-2 (batch-dependent rounding decides near-ties), and the request is
// compared no further.
struct Run {
  std::vector<std::uint64_t> tokens;
  std::vector<double> gaps;
};

Run run_chunked(runtime::StageBackend& stage, b200::MixedStageScheduler* scheduler,
                std::unique_ptr<runtime::SequenceState> state,
                const std::vector<std::uint64_t>& prompt, std::size_t chunk, int steps) {
  std::atomic_bool cancelled{false};
  state->sampling = {0.0, 1.0, 0, 0, true, 2};
  const auto deadline = std::chrono::system_clock::now() + std::chrono::minutes(5);
  Run run;
  std::size_t position = 0;
  std::vector<std::uint64_t> input;
  auto pass = [&](std::vector<std::uint64_t> ids) {
    return scheduler ? scheduler->execute(stage, runtime::TokenInput{std::move(ids)}, position,
                                          *state, cancelled, deadline)
                     : stage.execute(runtime::TokenInput{std::move(ids)}, position, *state,
                                     cancelled);
  };
  while (position < prompt.size()) {
    const std::size_t n = std::min(chunk, prompt.size() - position);
    state->prefilling = position > 0;
    state->prefill_only = position + n < prompt.size();
    auto out = pass({prompt.begin() + static_cast<std::ptrdiff_t>(position),
                     prompt.begin() + static_cast<std::ptrdiff_t>(position + n)});
    position += n;
    if (!state->prefill_only) input = {std::get<runtime::SampledToken>(out).id};
    if (!state->prefill_only) {
      const auto& t = std::get<runtime::SampledToken>(out);
      run.tokens.push_back(t.id);
      run.gaps.push_back(t.top_logprobs.size() == 2
                             ? t.top_logprobs[0].logprob - t.top_logprobs[1].logprob
                             : 1.0);
    }
  }
  state->prefilling = false;
  state->prefill_only = false;
  for (int s = 0; s < steps; ++s) {
    auto out = pass(input);
    const auto& t = std::get<runtime::SampledToken>(out);
    run.tokens.push_back(t.id);
    run.gaps.push_back(t.top_logprobs.size() == 2
                           ? t.top_logprobs[0].logprob - t.top_logprobs[1].logprob
                           : 1.0);
    position += 1;
    input = {t.id};
  }
  return run;
}

int mixed_scheduler_contract() {
  auto stage = make_stage(13);
  const int requests = 8, steps = 12;
  const std::size_t chunk = 64;
  std::vector<std::vector<std::uint64_t>> prompts;
  for (int r = 0; r < requests; ++r) {
    std::vector<std::uint64_t> p;
    for (int i = 0; i < 5 + 23 * r; ++i)
      p.push_back(static_cast<std::uint64_t>((r * 977 + i * 31) % 4096));
    prompts.push_back(p);
  }
  std::vector<Run> serial;
  for (int r = 0; r < requests; ++r)
    serial.push_back(run_chunked(*stage, nullptr, stage->allocate_sequence(prompts[r].size() + steps),
                                 prompts[r], chunk, steps));
  b200::MixedStageScheduler scheduler;
  scheduler.configure(16, 128);
  // Every sequence is allocated before any request starts: allocation takes
  // the stage's lock, which a thread running passes back to back would hold
  // against it.  Then all requests start together from one latch.
  std::vector<std::unique_ptr<runtime::SequenceState>> states;
  for (int r = 0; r < requests; ++r) states.push_back(stage->allocate_sequence(prompts[r].size() + steps));
  std::vector<Run> concurrent(requests);
  std::latch start(requests);
  std::vector<std::thread> threads;
  for (int r = 0; r < requests; ++r)
    threads.emplace_back([&, r] {
      start.arrive_and_wait();
      concurrent[r] = run_chunked(*stage, &scheduler, std::move(states[r]), prompts[r], chunk, steps);
    });
  for (auto& t : threads) t.join();
  int compared = 0;
  for (int r = 0; r < requests; ++r) {
    const auto& a = serial[r].tokens;
    const auto& b = concurrent[r].tokens;
    EXPECT(a.size() == b.size(), "request %d token count", r);
    for (std::size_t i = 0; i < a.size() && i < b.size(); ++i) {
      if (a[i] != b[i]) {
        EXPECT(serial[r].gaps[i] < 1e-2, "request %d step %zu: tokens differ with top-2 gap %g",
               r, i, serial[r].gaps[i]);
        break;
      }
      ++compared;
    }
  }
  const auto m = scheduler.metrics();
  EXPECT(m.completed_steps > 0 && m.mixed_batches > 0, "no mixed pass formed");
  EXPECT(m.decode_batches > 0 && m.largest_decode_batch >= 4, "passes of several tickets %zu, largest %zu",
         m.decode_batches, m.largest_decode_batch);
  std::printf("mixed: tokens compared=%d steps=%zu passes_with_several=%zu mixed=%zu largest=%zu "
              "gather=%.2f ms\n",
              compared, m.completed_steps, m.decode_batches, m.mixed_batches, m.largest_decode_batch,
              m.gather_wait_ms);
  std::printf(failures ? "mixed scheduler contract: %d failures\n"
                       : "mixed scheduler contract: ok\n",
              failures);
  return failures ? 1 : 0;
}

// The reference's own contracts: decode batches on the two-layer stage, then
// component timing on a two-stage split (layer 0 | layer 1).
int reference_contracts() {
  {
    auto stage = make_stage(11);
    test::decode_batch_contract(*stage);
  }
  const int batch = gtest_shim::failures();
  std::printf("decode batch contract: %s\n", batch ? "failed" : "ok");
  {
    auto first = make_stage(7, 0, 1, true, false);
    auto last = make_stage(7, 1, 2, false, true);
    test::paired_timing_contract(*first, *last);
  }
  const int timing = gtest_shim::failures() - batch;
  std::printf("paired timing contract: %s\n", timing ? "failed" : "ok");
  std::printf(batch + timing ? "reference contracts: %d failures\n" : "reference contracts: ok\n",
              batch + timing);
  return batch + timing ? 1 : 0;
}

int main(int argc, char** argv) {
  if (argc > 1 && std::string(argv[1]) == "reference") return reference_contracts();
  if (argc > 1 && std::string(argv[1]) == "mixed") return mixed_scheduler_contract();
  auto stage = make_stage(7);
  decode_batch_case(*stage, 0.0);
  decode_batch_case(*stage, 0.8);

  // Concurrent requests through the reference scheduler vs serial execution.
  const int requests = 6, steps = 10;
  std::vector<std::vector<std::uint64_t>> prompts;
  for (int r = 0; r < requests; ++r) {
    std::vector<std::uint64_t> p;
    for (int i = 0; i < 5 + 3 * r; ++i) p.push_back(static_cast<std::uint64_t>((r * 977 + i * 31) % 4096));
    prompts.push_back(p);
  }
  std::vector<std::vector<std::uint64_t>> serial;
  for (int r = 0; r < requests; ++r) serial.push_back(run_request(*stage, nullptr, prompts[r], steps));
  worker::StageScheduler scheduler;
  scheduler.configure(8);
  std::vector<std::vector<std::uint64_t>> concurrent(requests);
  std::vector<std::thread> threads;
  for (int r = 0; r < requests; ++r)
    threads.emplace_back([&, r] { concurrent[r] = run_request(*stage, &scheduler, prompts[r], steps); });
  for (auto& t : threads) t.join();
  for (int r = 0; r < requests; ++r)
    EXPECT(concurrent[r] == serial[r], "request %d tokens differ under the scheduler", r);
  const auto metrics = scheduler.metrics();
  EXPECT(metrics.completed_steps == static_cast<std::size_t>(requests * steps), "completed %zu",
         metrics.completed_steps);
  EXPECT(metrics.largest_decode_batch <= 8U, "largest batch %zu", metrics.largest_decode_batch);
  std::printf("decode_batches=%zu largest_decode_batch=%zu completed_steps=%zu\n",
              metrics.decode_batches, metrics.largest_decode_batch, metrics.completed_steps);
  std::printf(failures ? "adapter contract: %d failures\n" : "adapter contract: ok\n", failures);
  return failures ? 1 : 0;
}
