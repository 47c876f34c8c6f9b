// b200_stage_backend.hpp -- hLLM runtime::StageBackend over the B200 C ABI.
//
// The drop-in class a maintainer links into the reference's native worker in
// place of the ATen CUDA stage (cpp/src/cuda/stage.cpp:85).  It implements
// every virtual of runtime::StageBackend
// (cpp/include/hllm/runtime/stage_backend.hpp:69-107) by calling
// libhllm_b200.so through include/hllm_b200.h, and translates
// hllm_b200_status codes into runtime::Error (cpp/include/hllm/runtime/error.hpp).
// Build it against the reference headers: -I<reference>/cpp/include.
#pragma once

#include <atomic>
#include <cstdint>
#include <memory>
#include <mutex>
#include <vector>

#include "hllm/runtime/stage_backend.hpp"
#include "hllm_b200.h"
#include "mixed_scheduler.hpp"

namespace hllm::b200 {

// Throws the runtime::Error matching a failed C-ABI call.
[[noreturn]] void throw_status(hllm_b200_status status);
inline void check(hllm_b200_status status) {
  if (status != HLLM_B200_OK) throw_status(status);
}

// Per-request state: the reference's SequenceState plus the paged-KV sequence.
struct B200Sequence final : runtime::SequenceState {
  hllm_b200_stage* stage{nullptr};
  hllm_b200_seq* handle{nullptr};
  ~B200Sequence() override;
};

class B200StageBackend final : public runtime::StageBackend, public MixedBatchBackend {
 public:
  // Takes ownership of a finalized stage (hllm_b200_stage_create + weights +
  // hllm_b200_stage_finalize).
  B200StageBackend(hllm_b200_stage* stage, bool first, bool final);
  ~B200StageBackend() override;

  [[nodiscard]] runtime::MemoryAmounts weight_memory() const override;
  [[nodiscard]] std::size_t hidden_size() const override { return hidden_; }
  [[nodiscard]] std::size_t vocabulary_size() const override { return vocab_; }
  [[nodiscard]] std::size_t maximum_tokens() const override { return max_tokens_; }
  using runtime::StageBackend::sequence_memory;
  [[nodiscard]] runtime::SequenceMemory sequence_memory(
      std::size_t tokens, std::size_t maximum_query_tokens) const override;
  [[nodiscard]] std::unique_ptr<runtime::SequenceState> allocate_sequence(
      std::size_t tokens) const override;
  [[nodiscard]] runtime::StageOutput execute(runtime::StageInput input, std::size_t first_position,
                                             runtime::SequenceState& state,
                                             const std::atomic_bool& cancelled) const override;
  bool supports_decode_batch() const override { return true; }
  std::vector<runtime::StageOutput> execute_decode_batch(
      std::vector<runtime::DecodeBatchItem> items) const override;
  [[nodiscard]] runtime::StageOutput execute_profiled(runtime::StageInput input,
                                                      std::size_t first_position,
                                                      runtime::SequenceState& state,
                                                      const std::atomic_bool& cancelled,
                                                      runtime::ExecutionTiming& timing) const override;

  // One pass over rows that may mix prefill chunks and decode tokens (the
  // reference scheduler never forms such batches; MixedStageScheduler does).
  std::vector<runtime::StageOutput> execute_mixed_batch(
      std::vector<runtime::DecodeBatchItem> items) const override;

 private:
  std::vector<runtime::StageOutput> run(std::vector<runtime::DecodeBatchItem>& items) const;

  hllm_b200_stage* stage_;
  bool first_, final_;
  std::size_t hidden_{}, vocab_{}, max_tokens_{};
  mutable std::mutex mutex_;
};

}  // namespace hllm::b200
