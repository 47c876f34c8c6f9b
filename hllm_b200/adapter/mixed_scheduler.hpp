// mixed_scheduler.hpp -- a StageScheduler that mixes prefill chunks into decode
// batches.
//
// The reference's worker::StageScheduler (cpp/include/hllm/worker/scheduler.hpp,
// cpp/src/worker/scheduler.cpp:27-140) serialises a stage's passes: each pass
// is one prefill ticket alone or up to 8 decode tickets, and prefills wait for
// a streak of 8 decode passes.  On a B200 one pass costs the same whether it
// carries 1 or 64 decode rows plus a prefill chunk (the step streams every
// weight once), so MixedStageScheduler puts them in the same pass: the leader
// claims up to `maximum_decode_batch` ready decode tickets and, after them,
// prefill tickets in arrival order up to `prefill_token_budget` tokens (at
// least one), and runs them as one execute_mixed_batch.  Backends without
// that capability get the reference's policy unchanged.
//
// Same contract as the reference scheduler: RPC callers own their tickets and
// sequences until compute completes; one caller leads each dispatch and the
// others wait for their own result; a ticket cancelled or past its deadline
// before it is claimed fails with CANCELLED or DEADLINE_EXCEEDED; an exception
// from the backend reaches every member of the dispatch.
#pragma once

#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstddef>
#include <deque>
#include <exception>
#include <mutex>
#include <optional>
#include <vector>

#include "hllm/runtime/stage_backend.hpp"

namespace hllm::b200 {

// The optional StageBackend capability a mixed pass needs.  In the reference
// it would be two more virtuals of runtime::StageBackend
// (cpp/include/hllm/runtime/stage_backend.hpp:69-107); B200StageBackend
// implements this interface instead, so the reference header stays unchanged.
class MixedBatchBackend {
 public:
  virtual ~MixedBatchBackend() = default;
  // One pass over rows that may mix prefill chunks and decode tokens of
  // distinct sequences; one output per row, in order.
  virtual std::vector<runtime::StageOutput> execute_mixed_batch(
      std::vector<runtime::DecodeBatchItem> items) const = 0;
};

struct MixedSchedulerMetrics {
  std::size_t queued_prefills{};
  std::size_t queued_decodes{};
  std::size_t executing{};
  std::size_t completed_steps{};
  double queue_wait_ms{};
  std::size_t decode_batches{};       // passes of more than one ticket
  std::size_t largest_decode_batch{};  // most tickets in one pass
  std::size_t mixed_batches{};        // passes with both prefill and decode tickets
};

class MixedStageScheduler final {
 public:
  static constexpr std::size_t kMaximumBatch = 64;   // decode tickets per pass
  static constexpr std::size_t kReferenceBatch = 8;  // the reference's cap without mixing
  static constexpr std::size_t kReferenceStreak = 8;

  // maximum_decode_batch in [1, 64] (capped at 8 for backends that cannot
  // mix); prefill_token_budget > 0.
  void configure(std::size_t maximum_decode_batch, std::size_t prefill_token_budget = 512);
  runtime::StageOutput execute(const runtime::StageBackend& backend, runtime::StageInput input,
                               std::size_t position, runtime::SequenceState& sequence,
                               const std::atomic_bool& cancelled,
                               std::chrono::system_clock::time_point deadline);
  MixedSchedulerMetrics metrics() const;

 private:
  struct Ticket {
    runtime::DecodeBatchItem item;
    std::chrono::system_clock::time_point deadline;
    std::chrono::steady_clock::time_point queued;
    bool prefill{false};
    bool claimed{false}, done{false};
    std::optional<runtime::StageOutput> result;
    std::exception_ptr error;
  };
  static constexpr std::size_t kMaximumDispatch = 2 * kMaximumBatch;
  Ticket* next(bool mixing) const;
  // Pops the front ticket of `queue` and claims it.  A ticket cancelled or
  // past its deadline fails there and is not added to the dispatch.
  void claim(std::deque<Ticket*>& queue, Ticket** dispatch, std::size_t& count);

  mutable std::mutex mutex_;
  std::condition_variable ready_;
  std::deque<Ticket*> prefills_, decodes_;
  std::size_t maximum_decode_batch_{1};
  std::size_t prefill_token_budget_{512};
  std::size_t executing_{0};
  std::size_t decode_streak_{0};
  std::size_t completed_steps_{0};
  double queue_wait_ms_{0};
  std::size_t decode_batches_{0}, largest_decode_batch_{0}, mixed_batches_{0};
};

}  // namespace hllm::b200
