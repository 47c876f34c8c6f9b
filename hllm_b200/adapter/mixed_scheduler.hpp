// mixed_scheduler.hpp -- forms stage passes that carry prefill chunks and
// decode tokens together.
//
// On a B200 a stage pass streams every weight of its layers once, so a pass
// with 64 decode rows and a 512-token prefill chunk costs little more than a
// pass with one decode row.  The reference worker's StageScheduler
// (cpp/src/worker/scheduler.cpp:27-140) never mixes the two kinds: a pass is
// one prefill, or up to 8 decodes, with prefills admitted after a streak of 8
// decode tickets.  This scheduler is a drop-in for it in the worker's RPC
// handlers (same execute() signature, same error codes and messages, the same
// metrics plus two), with its own pass former:
//
//  * Tickets wait in one arrival-ordered list threaded through the callers'
//    own stack frames, so queueing allocates nothing.
//  * Any waiting caller that finds the stage idle forms the next pass, whether
//    or not its own ticket ends up in it, runs it, and hands each member its
//    result.  Members sleep until their ticket is finished.
//  * Gather window: the callers of the last pass usually come straight back
//    with their next step.  The former waits, at most `gather`, until as many
//    tickets are queued as the last pass had members, so a pass is not started
//    by whichever caller happened to return first.
//  * Backends that implement MixedBatchBackend get mixed passes: up to
//    `decode_rows` decode tickets and, in arrival order, prefill chunks up to
//    `prefill_tokens` tokens (the oldest chunk always fits).  Other backends
//    get the reference's policy, cap of 8 and decode streak included.
//
// Contract kept from the reference: callers own their tickets and sequences
// until their call returns; a ticket cancelled or past its deadline before a
// pass takes it fails with CANCELLED / DEADLINE_EXCEEDED and the reference's
// messages; an exception from the backend reaches every member of the pass.
#pragma once

#include <array>
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstddef>
#include <exception>
#include <mutex>
#include <optional>
#include <vector>

#include "hllm/runtime/stage_backend.hpp"

namespace hllm::b200 {

// The optional StageBackend capability a mixed pass needs.  In the reference
// it would be one more virtual of runtime::StageBackend
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

// The reference's SchedulerMetrics (cpp/include/hllm/worker/scheduler.hpp:16-24)
// plus mixed_batches and gather_wait_ms.
struct MixedSchedulerMetrics {
  std::size_t queued_prefills{};
  std::size_t queued_decodes{};
  std::size_t executing{};
  std::size_t completed_steps{};
  double queue_wait_ms{};
  std::size_t decode_batches{};        // passes of more than one ticket
  std::size_t largest_decode_batch{};  // most tickets in one pass
  std::size_t mixed_batches{};         // passes with prefill and decode tickets
  double gather_wait_ms{};             // time formers spent in the gather window
};

struct MixedSchedulerOptions {
  std::size_t decode_rows{64};       // decode tickets per pass, 1..64
  std::size_t prefill_tokens{512};   // prefill chunk tokens per pass, > 0
  std::chrono::microseconds gather{300};
};

class MixedStageScheduler final {
 public:
  static constexpr std::size_t kMaximumBatch = 64;   // decode tickets per pass
  static constexpr std::size_t kReferenceBatch = 8;  // the reference's cap without mixing
  static constexpr std::size_t kReferenceStreak = 8;

  // maximum_decode_batch in [1, 64] (8 at most is used for a backend that
  // cannot mix); prefill_token_budget > 0.  Refused while tickets are queued
  // or a pass runs.
  void configure(std::size_t maximum_decode_batch, std::size_t prefill_token_budget = 512);
  void configure(const MixedSchedulerOptions& options);

  runtime::StageOutput execute(const runtime::StageBackend& backend, runtime::StageInput input,
                               std::size_t position, runtime::SequenceState& sequence,
                               const std::atomic_bool& cancelled,
                               std::chrono::system_clock::time_point deadline);
  MixedSchedulerMetrics metrics() const;

 private:
  static constexpr std::size_t kPrefillTickets = 64;  // prefill chunks per pass
  static constexpr std::size_t kPassSize = kMaximumBatch + kPrefillTickets;

  enum class Phase { kQueued, kRunning, kFinished };
  struct Ticket {
    runtime::DecodeBatchItem item;
    std::chrono::system_clock::time_point deadline;
    std::chrono::steady_clock::time_point arrived;
    std::size_t tokens{};
    bool prefill{};
    Phase phase{Phase::kQueued};
    Ticket* next{nullptr};
    std::optional<runtime::StageOutput> output;
    std::exception_ptr error;
  };
  struct Pass {
    std::array<Ticket*, kPassSize> members{};
    std::size_t size{0};
    std::size_t prefills{0};
  };

  // All private members run with mutex_ held.
  void append(Ticket* ticket);
  void unlink(Ticket* ticket);
  std::size_t queued() const { return queued_prefills_ + queued_decodes_; }
  // Fails a queued ticket whose caller gave up; true if it did.
  bool drop_if_abandoned(Ticket* ticket);
  void take(Pass& pass, Ticket* ticket);
  void choose_mixed(Pass& pass);
  void choose_reference(Pass& pass, bool batching);
  // Forms one pass (after the gather window) and runs it.  Returns with the
  // lock held.
  void lead(std::unique_lock<std::mutex>& lock, const runtime::StageBackend& backend,
            const MixedBatchBackend* mixer);

  mutable std::mutex mutex_;
  std::condition_variable changed_;
  Ticket* head_{nullptr};
  Ticket* tail_{nullptr};
  std::size_t queued_prefills_{0}, queued_decodes_{0};
  bool forming_{false};
  std::size_t running_{0};    // members of the pass in the backend
  std::size_t returning_{0};  // members of the last finished pass
  std::size_t decode_run_{0}; // decode tickets since the last prefill (reference policy)
  // Unconfigured: one decode ticket per pass, as the reference's scheduler.
  MixedSchedulerOptions options_{1, 512, std::chrono::microseconds(300)};
  std::size_t completed_steps_{0}, multi_passes_{0}, largest_pass_{0}, mixed_passes_{0};
  double queue_wait_ms_{0}, gather_wait_ms_{0};
};

}  // namespace hllm::b200
