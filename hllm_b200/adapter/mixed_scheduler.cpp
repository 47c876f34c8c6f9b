// mixed_scheduler.cpp -- see mixed_scheduler.hpp.
#include "mixed_scheduler.hpp"

#include <algorithm>
#include <array>
#include <type_traits>
#include <variant>

#include "hllm/runtime/error.hpp"

namespace hllm::b200 {
namespace {
// Delivery into an empty optional must not fail after ownership is transferred.
static_assert(std::is_nothrow_move_constructible_v<runtime::StageOutput>);

std::size_t input_tokens(const runtime::StageInput& input) {
  if (const auto* t = std::get_if<runtime::TokenInput>(&input)) return t->ids.size();
  return std::get<runtime::BoundaryActivation>(input).tokens;
}

bool expired(std::chrono::system_clock::time_point deadline) {
  return std::chrono::system_clock::now() >= deadline;
}
}  // namespace

void MixedStageScheduler::configure(std::size_t maximum_decode_batch,
                                    std::size_t prefill_token_budget) {
  if (maximum_decode_batch == 0 || maximum_decode_batch > kMaximumBatch)
    throw runtime::Error::invalid_request("decode batch size must be between 1 and 64");
  if (prefill_token_budget == 0)
    throw runtime::Error::invalid_request("prefill token budget must be positive");
  std::scoped_lock lock(mutex_);
  if (executing_ || !prefills_.empty() || !decodes_.empty())
    throw runtime::Error::internal("cannot reconfigure an active scheduler");
  maximum_decode_batch_ = maximum_decode_batch;
  prefill_token_budget_ = prefill_token_budget;
}

// Without mixing: the reference's order (cpp/src/worker/scheduler.cpp:27-32),
// prefills first unless decodes are waiting and the decode streak is short.
// With mixing every pass carries both kinds, so any queue front may lead.
MixedStageScheduler::Ticket* MixedStageScheduler::next(bool mixing) const {
  if (mixing) {
    if (!decodes_.empty()) return decodes_.front();
    return prefills_.empty() ? nullptr : prefills_.front();
  }
  if (!prefills_.empty() && (decodes_.empty() || decode_streak_ >= kReferenceStreak))
    return prefills_.front();
  if (!decodes_.empty()) return decodes_.front();
  return nullptr;
}

void MixedStageScheduler::claim(std::deque<Ticket*>& queue, Ticket** dispatch,
                                std::size_t& count) {
  auto* member = queue.front();
  queue.pop_front();
  member->claimed = true;
  if (member->item.cancelled->load() || expired(member->deadline)) {
    // Even constructing an error message can fail under memory pressure.
    try {
      if (expired(member->deadline))
        throw runtime::Error::deadline_exceeded("deadline expired in native queue");
      throw runtime::Error::cancelled("request cancelled in native queue");
    } catch (...) {
      member->error = std::current_exception();
    }
    member->done = true;
    return;
  }
  dispatch[count++] = member;
  queue_wait_ms_ +=
      std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - member->queued)
          .count();
}

runtime::StageOutput MixedStageScheduler::execute(const runtime::StageBackend& backend,
                                                  runtime::StageInput input,
                                                  std::size_t position,
                                                  runtime::SequenceState& sequence,
                                                  const std::atomic_bool& cancelled,
                                                  std::chrono::system_clock::time_point deadline) {
  const bool prefill = position == 0 || sequence.prefilling;
  Ticket ticket{{std::move(input), position, &sequence, &cancelled},
                deadline, std::chrono::steady_clock::now(), prefill, false, false, {}, {}};
  const auto* mixer = dynamic_cast<const MixedBatchBackend*>(&backend);
  const bool batch_supported = backend.supports_decode_batch();
  std::unique_lock lock(mutex_);
  auto& queue = prefill ? prefills_ : decodes_;
  queue.push_back(&ticket);
  while (!ticket.done) {
    if (!ticket.claimed && (cancelled.load() || expired(deadline))) {
      queue.erase(std::find(queue.begin(), queue.end(), &ticket));
      ready_.notify_all();
      if (expired(deadline)) throw runtime::Error::deadline_exceeded("deadline expired in native queue");
      throw runtime::Error::cancelled("request cancelled in native queue");
    }
    if (ticket.claimed || executing_ || next(mixer != nullptr) != &ticket) {
      ready_.wait_for(lock, std::chrono::milliseconds(5));
      continue;
    }
    // Claiming tickets must not allocate: callers cannot abandon claimed work.
    std::array<Ticket*, kMaximumDispatch> storage{};
    std::size_t count = 0, prefills = 0;
    if (mixer) {
      while (!decodes_.empty() && count < maximum_decode_batch_) claim(decodes_, storage.data(), count);
      std::size_t tokens = 0;
      while (!prefills_.empty() && count < kMaximumDispatch) {
        const std::size_t t = input_tokens(prefills_.front()->item.input);
        if (prefills && tokens + t > prefill_token_budget_) break;
        const std::size_t before = count;
        claim(prefills_, storage.data(), count);
        if (count > before) {
          ++prefills;
          tokens += t;
        }
      }
    } else {
      // The reference's dispatch (cpp/src/worker/scheduler.cpp:58-72).
      auto limit = prefill || !batch_supported ? std::size_t{1}
                                               : std::min(maximum_decode_batch_, kReferenceBatch);
      if (!prefill && !prefills_.empty())
        limit = std::min(limit, kReferenceStreak - decode_streak_);
      while (!queue.empty() && count < limit) claim(queue, storage.data(), count);
      if (prefill) prefills = count;
    }
    if (count == 0) {
      ready_.notify_all();
      continue;
    }
    executing_ = count;
    const std::size_t decodes = count - prefills;
    if (!mixer)
      decode_streak_ = prefill ? 0U : std::min(decode_streak_ + count, kReferenceStreak);
    lock.unlock();
    std::vector<runtime::StageOutput> outputs;
    std::exception_ptr error;
    try {
      if (count == 1) {
        auto& item = storage[0]->item;
        outputs.push_back(
            backend.execute(std::move(item.input), item.position, *item.sequence, *item.cancelled));
      } else {
        std::vector<runtime::DecodeBatchItem> items;
        items.reserve(count);
        for (std::size_t i = 0; i < count; ++i) items.push_back(std::move(storage[i]->item));
        outputs = prefills ? mixer->execute_mixed_batch(std::move(items))
                           : backend.execute_decode_batch(std::move(items));
        if (outputs.size() != count) throw runtime::Error::internal("batch output count mismatch");
      }
    } catch (...) {
      error = std::current_exception();
    }
    lock.lock();
    for (std::size_t i = 0; i < count; ++i) {
      auto* member = storage[i];
      member->error = error;
      if (!error) member->result.emplace(std::move(outputs[i]));
      member->done = true;
    }
    completed_steps_ += count;
    if (count > 1) {
      ++decode_batches_;
      largest_decode_batch_ = std::max(largest_decode_batch_, count);
    }
    if (prefills && decodes) ++mixed_batches_;
    executing_ = 0;
    ready_.notify_all();
  }
  if (ticket.error) std::rethrow_exception(ticket.error);
  return std::move(*ticket.result);
}

MixedSchedulerMetrics MixedStageScheduler::metrics() const {
  std::scoped_lock lock(mutex_);
  return {prefills_.size(), decodes_.size(), executing_,           completed_steps_,
          queue_wait_ms_,   decode_batches_, largest_decode_batch_, mixed_batches_};
}

}  // namespace hllm::b200
