// mixed_scheduler_test.cpp -- MixedStageScheduler on fake backends (no GPU).
//
// Built by tests/cpp/Makefile against the reference's runtime headers and run
// by tests/test_mixed_scheduler.py.  Request threads drive prefill chunks and
// decode steps through the scheduler, as the worker's RPC handlers drive the
// reference's StageScheduler (cpp/src/worker/execution_service.cpp); the fake
// backends record every pass and return outputs derived from (sequence,
// position), so each request can check that it got its own results.  A fake
// pass busy-waits 20-100 us, the length of a small stage's pass on a B200:
// nothing sleeps, so passes form only through the scheduler's own logic.
// Every sequence is allocated before the request threads start, and the
// threads are released together from one latch.
//
//  1. A mixing backend: passes carry decode tickets and prefill chunks
//     together, never more decodes than configured, never more prefill tokens
//     than the budget (except a single chunk), distinct sequences per pass;
//     mixed passes form and returning callers regroup into multi-ticket passes.
//  2. A backend without the capability: the reference's policy (prefills
//     alone, decode batches of at most 8, no mixed pass).
//  3. Cancellation and deadlines before a ticket is claimed, and an exception
//     from the backend reaching every member of its pass.
#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdio>
#include <latch>
#include <memory>
#include <mutex>
#include <set>
#include <string>
#include <thread>
#include <variant>
#include <vector>

#include "hllm/runtime/error.hpp"
#include "mixed_scheduler.hpp"

using namespace hllm;
using Clock = std::chrono::system_clock;

namespace {
std::atomic<int> failures{0};
#define EXPECT(cond, ...)                                   \
  do {                                                      \
    if (!(cond)) {                                          \
      ++failures;                                           \
      std::printf("FAIL %s:%d ", __FILE__, __LINE__);       \
      std::printf(__VA_ARGS__);                             \
      std::printf("\n");                                    \
    }                                                       \
  } while (0)

struct FakeSequence final : runtime::SequenceState {
  int id = 0;
};

struct Pass {
  std::size_t prefills = 0, decodes = 0, prefill_tokens = 0;
  bool distinct = true;
};

// Output of a row: a token id that encodes (sequence, position) so a request
// can check it received its own row's result.
std::uint64_t token_of(const runtime::SequenceState* s, std::size_t position) {
  return static_cast<std::uint64_t>(static_cast<const FakeSequence*>(s)->id) * 100000U + position;
}

class FakeBackend : public runtime::StageBackend {
 public:
  mutable std::mutex mutex;
  mutable std::vector<Pass> passes;
  std::chrono::microseconds delay{50};
  mutable std::atomic<int> fail_next{0};

  runtime::MemoryAmounts weight_memory() const override { return {}; }
  std::size_t hidden_size() const override { return 8; }
  std::size_t vocabulary_size() const override { return 1U << 30; }
  std::size_t maximum_tokens() const override { return 4096; }
  using runtime::StageBackend::sequence_memory;
  runtime::SequenceMemory sequence_memory(std::size_t, std::size_t) const override { return {}; }
  std::unique_ptr<runtime::SequenceState> allocate_sequence(std::size_t) const override {
    return std::make_unique<FakeSequence>();
  }
  runtime::StageOutput execute(runtime::StageInput input, std::size_t position,
                               runtime::SequenceState& state,
                               const std::atomic_bool&) const override {
    std::vector<runtime::DecodeBatchItem> one;
    static const std::atomic_bool no{false};
    one.push_back({std::move(input), position, &state, &no});
    return pass(one).front();
  }
  bool supports_decode_batch() const override { return true; }
  std::vector<runtime::StageOutput> execute_decode_batch(
      std::vector<runtime::DecodeBatchItem> items) const override {
    for (const auto& it : items)
      if (it.position == 0 || it.sequence->prefilling)
        throw runtime::Error::invalid_request("decode batch requires decode sequences");
    return pass(items);
  }

 protected:
  std::vector<runtime::StageOutput> pass(const std::vector<runtime::DecodeBatchItem>& items) const {
    const auto until = std::chrono::steady_clock::now() + delay;
    while (std::chrono::steady_clock::now() < until) {
    }
    if (fail_next.exchange(0)) throw runtime::Error::internal("injected backend failure");
    Pass p;
    std::set<const runtime::SequenceState*> seen;
    std::vector<runtime::StageOutput> out;
    for (const auto& it : items) {
      const auto n = std::get<runtime::TokenInput>(it.input).ids.size();
      const bool prefill = it.position == 0 || it.sequence->prefilling;
      if (prefill) {
        ++p.prefills;
        p.prefill_tokens += n;
      } else {
        ++p.decodes;
      }
      p.distinct = p.distinct && seen.insert(it.sequence).second;
      if (it.sequence->prefill_only)
        out.push_back(runtime::PrefillProgress{});
      else
        out.push_back(runtime::SampledToken{token_of(it.sequence, it.position + n - 1)});
    }
    std::scoped_lock lock(mutex);
    passes.push_back(p);
    return out;
  }
};

class FakeMixingBackend final : public FakeBackend, public b200::MixedBatchBackend {
 public:
  std::vector<runtime::StageOutput> execute_mixed_batch(
      std::vector<runtime::DecodeBatchItem> items) const override {
    return pass(items);
  }
};

// One request: prompt in chunks of `chunk` tokens, then `steps` decode tokens.
void run_request(const runtime::StageBackend& backend, b200::MixedStageScheduler& scheduler,
                 runtime::SequenceState& state, int id, std::size_t prompt, std::size_t chunk,
                 int steps) {
  std::atomic_bool cancelled{false};
  const auto deadline = Clock::now() + std::chrono::minutes(5);
  std::size_t position = 0;
  while (position < prompt) {
    const std::size_t n = std::min(chunk, prompt - position);
    state.prefilling = position > 0;
    state.prefill_only = position + n < prompt;
    auto out = scheduler.execute(backend, runtime::TokenInput{std::vector<std::uint64_t>(n, 1)},
                                 position, state, cancelled, deadline);
    if (state.prefill_only) {
      EXPECT(std::holds_alternative<runtime::PrefillProgress>(out), "request %d chunk", id);
    } else {
      EXPECT(std::holds_alternative<runtime::SampledToken>(out) &&
                 std::get<runtime::SampledToken>(out).id == token_of(&state, position + n - 1),
             "request %d first token", id);
    }
    position += n;
  }
  state.prefilling = false;
  state.prefill_only = false;
  for (int s = 0; s < steps; ++s) {
    auto out = scheduler.execute(backend, runtime::TokenInput{{7}}, position, state, cancelled,
                                 deadline);
    EXPECT(std::holds_alternative<runtime::SampledToken>(out) &&
               std::get<runtime::SampledToken>(out).id == token_of(&state, position),
           "request %d step %d", id, s);
    ++position;
  }
}

// `requests` requests with prompts of 100 + 37 r tokens in 64-token chunks and
// 12 decode steps each; sequences first, then every thread from one latch.
void run_many(const FakeBackend& backend, b200::MixedStageScheduler& scheduler, int requests) {
  std::vector<std::unique_ptr<runtime::SequenceState>> states;
  for (int r = 0; r < requests; ++r) {
    states.push_back(backend.allocate_sequence(1024));
    static_cast<FakeSequence*>(states.back().get())->id = r + 1;
  }
  std::latch start(requests);
  std::vector<std::thread> threads;
  for (int r = 0; r < requests; ++r)
    threads.emplace_back([&, r] {
      start.arrive_and_wait();
      run_request(backend, scheduler, *states[r], r + 1, 100 + 37 * r, 64, 12);
    });
  for (auto& t : threads) t.join();
}

void mixing_case() {
  FakeMixingBackend backend;
  b200::MixedStageScheduler scheduler;
  scheduler.configure(16, 128);
  run_many(backend, scheduler, 24);
  std::size_t mixed = 0, rows = 0;
  for (const auto& p : backend.passes) {
    EXPECT(p.distinct, "a pass repeated a sequence");
    EXPECT(p.decodes <= 16, "pass with %zu decodes", p.decodes);
    EXPECT(p.prefills <= 1 || p.prefill_tokens <= 128, "pass with %zu prefill tokens",
           p.prefill_tokens);
    mixed += p.prefills && p.decodes;
    rows += p.prefills + p.decodes;
  }
  const auto m = scheduler.metrics();
  EXPECT(mixed > 0 && m.mixed_batches == mixed, "mixed passes %zu (metrics %zu)", mixed,
         m.mixed_batches);
  EXPECT(m.completed_steps == rows, "completed %zu rows %zu", m.completed_steps, rows);
  EXPECT(m.queued_prefills == 0 && m.queued_decodes == 0 && m.executing == 0, "queues drained");
  // 24 callers that all come back after each pass: most passes carry several.
  EXPECT(m.decode_batches * 2 > backend.passes.size(), "multi-ticket passes %zu of %zu",
         m.decode_batches, backend.passes.size());
  // 16 decodes and two 64-token chunks at most: 18 tickets.
  EXPECT(m.largest_decode_batch >= 10, "largest pass %zu", m.largest_decode_batch);
  std::printf("mixing: passes=%zu mixed=%zu largest=%zu rows=%zu gather=%.2f ms\n",
              backend.passes.size(), mixed, m.largest_decode_batch, rows, m.gather_wait_ms);
}

void reference_policy_case() {
  FakeBackend backend;  // no mixing capability
  b200::MixedStageScheduler scheduler;
  scheduler.configure(16, 128);  // capped at the reference's 8 without mixing
  run_many(backend, scheduler, 16);
  std::size_t largest = 0;
  for (const auto& p : backend.passes) {
    EXPECT(!(p.prefills && p.decodes), "a mixed pass without the capability");
    EXPECT(p.prefills <= 1, "%zu prefills in one pass", p.prefills);
    largest = std::max(largest, p.decodes);
  }
  EXPECT(largest <= 8, "decode batch of %zu", largest);
  EXPECT(scheduler.metrics().mixed_batches == 0, "mixed metric");
  std::printf("reference policy: passes=%zu largest decode batch=%zu\n", backend.passes.size(),
              largest);
}

void failure_cases() {
  FakeMixingBackend backend;
  backend.delay = std::chrono::microseconds(100000);
  b200::MixedStageScheduler scheduler;
  scheduler.configure(8, 64);
  // A long pass holds the scheduler while tickets queue behind it.
  std::atomic_bool no{false};
  auto blocker = backend.allocate_sequence(8);
  std::thread lead([&] {
    static_cast<void>(scheduler.execute(backend, runtime::TokenInput{{1, 2}}, 0, *blocker, no,
                                        Clock::now() + std::chrono::minutes(1)));
  });
  std::this_thread::sleep_for(std::chrono::milliseconds(5));
  auto a = backend.allocate_sequence(8);
  auto b = backend.allocate_sequence(8);
  std::atomic_bool cancel_a{false};
  int code_a = -1, code_b = -1;
  std::thread ta([&] {
    try {
      static_cast<void>(scheduler.execute(backend, runtime::TokenInput{{3}}, 0, *a, cancel_a,
                                          Clock::now() + std::chrono::minutes(1)));
    } catch (const runtime::Error& e) {
      code_a = static_cast<int>(e.code());
    }
  });
  std::thread tb([&] {
    try {
      static_cast<void>(scheduler.execute(backend, runtime::TokenInput{{4}}, 0, *b, no,
                                          Clock::now() + std::chrono::milliseconds(2)));
    } catch (const runtime::Error& e) {
      code_b = static_cast<int>(e.code());
    }
  });
  std::this_thread::sleep_for(std::chrono::milliseconds(4));
  cancel_a = true;
  lead.join();
  ta.join();
  tb.join();
  EXPECT(code_a == static_cast<int>(runtime::ErrorCode::kCancelled), "cancelled: %d", code_a);
  EXPECT(code_b == static_cast<int>(runtime::ErrorCode::kDeadlineExceeded), "deadline: %d",
         code_b);
  // A failing pass: every member sees the backend's error.
  backend.delay = std::chrono::microseconds(5000);
  std::vector<std::unique_ptr<runtime::SequenceState>> states;
  for (int i = 0; i < 4; ++i) {
    states.push_back(backend.allocate_sequence(8));
    states.back()->prefill_only = false;
  }
  // Prefill them first (one at a time), then fail one decode pass.
  for (auto& s : states)
    static_cast<void>(scheduler.execute(backend, runtime::TokenInput{{5}}, 0, *s, no,
                                        Clock::now() + std::chrono::minutes(1)));
  std::atomic<int> internal{0}, ok{0};
  backend.fail_next = 1;  // the next pass fails
  std::vector<std::thread> ts;
  for (auto& s : states)
    ts.emplace_back([&, st = s.get()] {
      try {
        static_cast<void>(scheduler.execute(backend, runtime::TokenInput{{8}}, 1, *st, no,
                                            Clock::now() + std::chrono::minutes(1)));
        ++ok;
      } catch (const runtime::Error& e) {
        if (e.code() == runtime::ErrorCode::kInternal) ++internal;
      }
    });
  for (auto& t : ts) t.join();
  EXPECT(internal + ok == 4 && internal >= 1, "failing pass: internal %d ok %d", internal.load(),
         ok.load());
  // configure() validates and refuses while active
  bool refused = false;
  try {
    scheduler.configure(0);
  } catch (const runtime::Error&) {
    refused = true;
  }
  EXPECT(refused, "configure(0) accepted");
  std::printf("failures: cancelled=%d deadline=%d internal=%d\n", code_a, code_b,
              internal.load());
}
}  // namespace

int main() {
  mixing_case();
  reference_policy_case();
  failure_cases();
  const int n = failures.load();
  std::printf(n ? "mixed scheduler: %d failures\n" : "mixed scheduler: ok\n", n);
  return n ? 1 : 0;
}
