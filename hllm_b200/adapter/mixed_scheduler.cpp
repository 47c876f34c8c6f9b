// mixed_scheduler.cpp -- see mixed_scheduler.hpp.
#include "mixed_scheduler.hpp"

#include <algorithm>
#include <type_traits>
#include <variant>

#include "hllm/runtime/error.hpp"

namespace hllm::b200 {
namespace {
using std::chrono::steady_clock;
using std::chrono::system_clock;

// A finished pass moves each output into its member's empty optional after the
// backend returned; that step has no way to report a failure.
static_assert(std::is_nothrow_move_constructible_v<runtime::StageOutput>);

std::size_t rows_of(const runtime::StageInput& input) {
  if (const auto* tokens = std::get_if<runtime::TokenInput>(&input)) return tokens->ids.size();
  return std::get<runtime::BoundaryActivation>(input).tokens;
}

bool past(system_clock::time_point deadline) { return system_clock::now() >= deadline; }

double milliseconds_since(steady_clock::time_point start) {
  return std::chrono::duration<double, std::milli>(steady_clock::now() - start).count();
}

// The errors and messages the reference's queue gives a ticket that leaves
// unserved (cpp/src/worker/scheduler.cpp:53-58), so RPC status mapping is
// unchanged.
[[noreturn]] void throw_unserved(bool expired) {
  if (expired) throw runtime::Error::deadline_exceeded("deadline expired in native queue");
  throw runtime::Error::cancelled("request cancelled in native queue");
}
}  // namespace

void MixedStageScheduler::configure(std::size_t maximum_decode_batch,
                                    std::size_t prefill_token_budget) {
  std::chrono::microseconds gather{};
  {
    std::scoped_lock lock(mutex_);
    gather = options_.gather;
  }
  configure(MixedSchedulerOptions{maximum_decode_batch, prefill_token_budget, gather});
}

void MixedStageScheduler::configure(const MixedSchedulerOptions& options) {
  if (options.decode_rows == 0 || options.decode_rows > kMaximumBatch)
    throw runtime::Error::invalid_request("decode batch size must be between 1 and 64");
  if (options.prefill_tokens == 0)
    throw runtime::Error::invalid_request("prefill token budget must be positive");
  if (options.gather.count() < 0 || options.gather > std::chrono::seconds(1))
    throw runtime::Error::invalid_request("gather window must be between 0 and 1 s");
  std::scoped_lock lock(mutex_);
  if (running_ || forming_ || head_)
    throw runtime::Error::internal("cannot reconfigure an active scheduler");
  options_ = options;
}

void MixedStageScheduler::append(Ticket* ticket) {
  ticket->next = nullptr;
  (tail_ ? tail_->next : head_) = ticket;
  tail_ = ticket;
  ++(ticket->prefill ? queued_prefills_ : queued_decodes_);
}

void MixedStageScheduler::unlink(Ticket* ticket) {
  Ticket* before = nullptr;
  for (Ticket** link = &head_; *link; link = &(*link)->next) {
    if (*link != ticket) {
      before = *link;
      continue;
    }
    *link = ticket->next;
    if (tail_ == ticket) tail_ = before;
    ticket->next = nullptr;
    --(ticket->prefill ? queued_prefills_ : queued_decodes_);
    return;
  }
}

bool MixedStageScheduler::drop_if_abandoned(Ticket* ticket) {
  const bool expired = past(ticket->deadline);
  if (!expired && !ticket->item.cancelled->load()) return false;
  unlink(ticket);
  // Building the exception may itself fail (bad_alloc); either way the owner
  // gets an error rather than a hang.
  try {
    throw_unserved(expired);
  } catch (...) {
    ticket->error = std::current_exception();
  }
  ticket->phase = Phase::kFinished;
  return true;
}

void MixedStageScheduler::take(Pass& pass, Ticket* ticket) {
  unlink(ticket);
  ticket->phase = Phase::kRunning;
  pass.members[pass.size++] = ticket;
  if (ticket->prefill) ++pass.prefills;
  queue_wait_ms_ += milliseconds_since(ticket->arrived);
}

// Every queued decode ticket up to decode_rows, then prefill chunks in arrival
// order while they fit the token budget.  The oldest chunk is always taken;
// once one does not fit, no later chunk overtakes it.
void MixedStageScheduler::choose_mixed(Pass& pass) {
  std::size_t decodes = 0, prefill_tokens = 0;
  bool prefills_closed = false;
  for (Ticket* ticket = head_; ticket && pass.size < kPassSize;) {
    Ticket* after = ticket->next;
    if (!drop_if_abandoned(ticket)) {
      if (!ticket->prefill) {
        if (decodes < options_.decode_rows) {
          take(pass, ticket);
          ++decodes;
        }
      } else if (!prefills_closed) {
        const bool fits = pass.prefills == 0 ||
                          prefill_tokens + ticket->tokens <= options_.prefill_tokens;
        if (fits && pass.prefills < kPrefillTickets) {
          take(pass, ticket);
          prefill_tokens += ticket->tokens;
        } else {
          prefills_closed = true;
        }
      }
    }
    ticket = after;
  }
}

// The reference's policy for a backend that cannot mix
// (cpp/src/worker/scheduler.cpp:27-32 and 60-67): a prefill runs alone, and
// leads whenever no decode waits or 8 decode tickets ran since the last
// prefill; decode passes take at most 8 tickets (one without batch support),
// and no more than the streak has left while a prefill waits.
void MixedStageScheduler::choose_reference(Pass& pass, bool batching) {
  const bool prefill_turn =
      queued_prefills_ && (!queued_decodes_ || decode_run_ >= kReferenceStreak);
  std::size_t limit = 1;
  if (!prefill_turn) {
    if (batching) limit = std::min(options_.decode_rows, kReferenceBatch);
    if (queued_prefills_) limit = std::min(limit, kReferenceStreak - decode_run_);
  }
  for (Ticket* ticket = head_; ticket && pass.size < limit;) {
    Ticket* after = ticket->next;
    if (ticket->prefill == prefill_turn && !drop_if_abandoned(ticket)) take(pass, ticket);
    ticket = after;
  }
  if (pass.size == 0) return;
  decode_run_ = prefill_turn ? 0 : std::min(decode_run_ + pass.size, kReferenceStreak);
}

void MixedStageScheduler::lead(std::unique_lock<std::mutex>& lock,
                               const runtime::StageBackend& backend,
                               const MixedBatchBackend* mixer) {
  forming_ = true;
  const bool batching = mixer != nullptr || backend.supports_decode_batch();
  if (batching && options_.gather.count() > 0 && queued() < returning_) {
    const auto start = steady_clock::now();
    changed_.wait_until(lock, start + options_.gather,
                        [this] { return queued() >= returning_; });
    gather_wait_ms_ += milliseconds_since(start);
  }
  Pass pass;
  if (mixer)
    choose_mixed(pass);
  else
    choose_reference(pass, backend.supports_decode_batch());
  forming_ = false;
  if (pass.size == 0) {
    changed_.notify_all();
    return;
  }
  running_ = pass.size;
  lock.unlock();

  std::vector<runtime::StageOutput> outputs;
  std::exception_ptr error;
  try {
    if (pass.size == 1) {
      auto& item = pass.members[0]->item;
      outputs.push_back(
          backend.execute(std::move(item.input), item.position, *item.sequence, *item.cancelled));
    } else {
      std::vector<runtime::DecodeBatchItem> items;
      items.reserve(pass.size);
      for (std::size_t i = 0; i < pass.size; ++i) items.push_back(std::move(pass.members[i]->item));
      outputs = pass.prefills ? mixer->execute_mixed_batch(std::move(items))
                              : backend.execute_decode_batch(std::move(items));
      if (outputs.size() != pass.size) throw runtime::Error::internal("batch output count mismatch");
    }
  } catch (...) {
    error = std::current_exception();
  }

  lock.lock();
  for (std::size_t i = 0; i < pass.size; ++i) {
    Ticket* member = pass.members[i];
    if (error)
      member->error = error;
    else
      member->output.emplace(std::move(outputs[i]));
    member->phase = Phase::kFinished;
  }
  completed_steps_ += pass.size;
  if (pass.size > 1) {
    ++multi_passes_;
    largest_pass_ = std::max(largest_pass_, pass.size);
  }
  if (pass.prefills && pass.prefills < pass.size) ++mixed_passes_;
  running_ = 0;
  returning_ = pass.size;
  changed_.notify_all();
}

runtime::StageOutput MixedStageScheduler::execute(const runtime::StageBackend& backend,
                                                  runtime::StageInput input,
                                                  std::size_t position,
                                                  runtime::SequenceState& sequence,
                                                  const std::atomic_bool& cancelled,
                                                  system_clock::time_point deadline) {
  Ticket self{{std::move(input), position, &sequence, &cancelled}, deadline, steady_clock::now()};
  self.tokens = rows_of(self.item.input);
  self.prefill = position == 0 || sequence.prefilling;
  const auto* mixer = dynamic_cast<const MixedBatchBackend*>(&backend);

  std::unique_lock lock(mutex_);
  append(&self);
  changed_.notify_all();  // a former in its gather window counts arrivals
  while (self.phase != Phase::kFinished) {
    if (self.phase == Phase::kQueued) {
      const bool expired = past(deadline);
      if (expired || cancelled.load()) {
        unlink(&self);
        changed_.notify_all();
        throw_unserved(expired);
      }
      if (!forming_ && running_ == 0) {
        lead(lock, backend, mixer);
        continue;
      }
    }
    // Cancellation and deadlines are polled: nothing notifies on them.
    changed_.wait_for(lock, std::chrono::milliseconds(5));
  }
  if (self.error) std::rethrow_exception(self.error);
  return std::move(*self.output);
}

MixedSchedulerMetrics MixedStageScheduler::metrics() const {
  std::scoped_lock lock(mutex_);
  return {queued_prefills_, queued_decodes_, running_,      completed_steps_, queue_wait_ms_,
          multi_passes_,    largest_pass_,   mixed_passes_, gather_wait_ms_};
}

}  // namespace hllm::b200
