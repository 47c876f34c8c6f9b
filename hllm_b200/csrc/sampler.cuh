// sampler.cuh -- GPU token sampler.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace hb {

struct SampleParams {   // one per sampling row (validated on the host)
  double temperature;
  double top_p;
  uint64_t top_k;
  uint64_t seed;
  uint64_t generated_index;
  uint32_t return_logprobs;
  uint32_t top_logprobs;
};

struct SampleResult {
  int64_t token;
  double logprob;
  int32_t n_top;
  int32_t status;        // 0 ok, else DeviceStatus bits (non-finite logits)
  int64_t top_ids[5];
  double top_logprobs[5];
};

// One CTA per row: logits [rows][ld] F32 (vocab valid columns).  `scratch`
// holds rows * vocab doubles (the unnormalised probabilities).
cudaError_t sample_launch(const float* logits, int rows, int vocab, int ld,
                          const SampleParams* params, double* scratch, SampleResult* out,
                          uint32_t* status, cudaStream_t stream);

}  // namespace hb
