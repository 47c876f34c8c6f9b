/*
 * hllm_b200.h -- C ABI of the B200 stage executor (libhllm_b200.so).
 *
 * The executor runs one contiguous layer range of a Llama / Qwen3 decoder
 * (a hLLM "stage") on one B200.  It is the drop-in for hLLM's per-step hot path
 * behind runtime::StageBackend / runtime::BackendFactory
 * (cpp/include/hllm/runtime/stage_backend.hpp:69-107,
 *  cpp/include/hllm/runtime/backend_factory.hpp:28-47); the C++ adapter in
 * hllm_b200/adapter/ implements those classes over this ABI.
 *
 * Conventions: plain C types, caller-owned host pointers valid for the call,
 * device state owned by the stage.  No exception crosses the ABI; every call
 * returns an hllm_b200_status and hllm_b200_last_error() describes the last
 * failure on the calling thread.  One caller at a time per stage (the
 * reference scheduler serialises passes, cpp/src/worker/scheduler.cpp:60-63).
 */
#ifndef HLLM_B200_H_
#define HLLM_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Mirrors runtime::ErrorCode (cpp/include/hllm/runtime/error.hpp:10-17). */
typedef enum {
  HLLM_B200_OK = 0,
  HLLM_B200_INVALID_REQUEST = 1,
  HLLM_B200_INCOMPATIBLE_WORKER = 2,
  HLLM_B200_RESOURCE_EXHAUSTED = 3,
  HLLM_B200_DEADLINE_EXCEEDED = 4,
  HLLM_B200_CANCELLED = 5,
  HLLM_B200_INTERNAL = 6
} hllm_b200_status;

/* Source tensor types accepted by hllm_b200_stage_load_tensor
 * (runtime::DataType kF32 / kF16 / kBF16, cpp/include/hllm/runtime/safetensors.hpp:15-29). */
typedef enum { HLLM_B200_F32 = 0, HLLM_B200_F16 = 1, HLLM_B200_BF16 = 2 } hllm_b200_dtype;

typedef struct hllm_b200_stage hllm_b200_stage;
typedef struct hllm_b200_seq hllm_b200_seq;

/* Stage description: model::DenseConfig (cpp/include/hllm/model/dense_source.hpp:15-25)
 * plus the fields of model::DenseSource that select the layer range
 * (:35-45), plus executor capacities. */
typedef struct {
  uint64_t hidden_size;
  uint64_t intermediate_size;
  uint64_t attention_heads;
  uint64_t key_value_heads;
  uint64_t head_dimension;
  uint64_t maximum_sequence_length;
  float rms_norm_epsilon;
  float rope_theta;
  uint32_t query_key_norm;     /* Qwen3 per-head q/k RMSNorm */
  uint64_t vocabulary_size;
  uint64_t layer_start;        /* [layer_start, layer_end) of the model */
  uint64_t layer_end;
  uint32_t first;              /* stage embeds token ids */
  uint32_t final;              /* stage owns final norm + LM head and samples */
  uint32_t tied_head;          /* LM head is the embedding matrix */
  int32_t device_id;
  uint64_t kv_pool_tokens;     /* paged-KV capacity in tokens (16-token blocks) */
  uint32_t max_step_tokens;    /* most tokens in one step (all rows) */
  uint32_t max_step_rows;      /* most rows (sequences) in one step */
  uint32_t max_sequences;      /* most live sequences */
} hllm_b200_stage_desc;

/* runtime::SamplingOptions (cpp/include/hllm/runtime/sampling.hpp:10-17). */
typedef struct {
  double temperature;
  double top_p;
  uint64_t top_k;
  uint64_t seed;
  uint32_t return_logprobs;
  uint32_t top_logprobs;
} hllm_b200_sampling;

/* One row of a step: one sequence's input for this pass.  Replaces
 * StageBackend::execute's (input, first_position, state) triple and one
 * runtime::DecodeBatchItem (stage_backend.hpp:52-58, 90-92). */
typedef struct {
  hllm_b200_seq* sequence;
  uint64_t first_position;     /* must equal the sequence's current length */
  uint64_t tokens;             /* rows of input (prefill chunk) or 1 (decode) */
  const uint64_t* token_ids;   /* first stage: `tokens` ids */
  const uint16_t* activations; /* other stages: F16 [tokens][hidden] little-endian */
  uint32_t sample;             /* final stage: produce a SampledToken from the last row */
  hllm_b200_sampling sampling;
  uint64_t generated_index;    /* counter of the request's seeded draws */
} hllm_b200_row;

/* runtime::SampledToken (cpp/include/hllm/runtime/sampling.hpp:22-27). */
typedef struct {
  uint64_t token_id;
  double logprob;
  uint32_t has_logprob;
  uint32_t n_top;
  uint64_t top_ids[5];
  double top_logprobs[5];
} hllm_b200_sampled;

/* ---------------------------------------------------------------- errors */
/* Copies the calling thread's last error message (NUL-terminated, truncated). */
size_t hllm_b200_last_error(char* buffer, size_t size);

/* ------------------------------------------------------------ stage life */
/* Replaces BackendFactory::load (backend_factory.hpp:44-46) and the CUDA stage
 * constructor (cpp/src/cuda/stage.cpp:87-143): allocates device weights, the
 * paged KV pool and step workspaces.  Weights are then supplied tensor by
 * tensor (load_tensor) or generated (init_synthetic); finalize checks that
 * every tensor of the range is present. */
hllm_b200_status hllm_b200_stage_create(const hllm_b200_stage_desc* desc, hllm_b200_stage** out);
void hllm_b200_stage_destroy(hllm_b200_stage* stage);

/* One named Safetensors tensor (names as in cpp/src/cpu/stage.cpp:236-259),
 * row-major, converted to F16 on upload.  A value not representable as a
 * finite F16 is rejected (cpp/src/cuda/stage.cpp:127-133). */
hllm_b200_status hllm_b200_stage_load_tensor(hllm_b200_stage* stage, const char* name,
                                             hllm_b200_dtype dtype, const void* data,
                                             const uint64_t* shape, uint32_t rank);
/* Fills every tensor of the stage with the seeded synthetic weights of this
 * executor (bit-identical with the CPU oracle's generator).  No reference
 * counterpart: used for benchmarks on random-init models. */
hllm_b200_status hllm_b200_stage_init_synthetic(hllm_b200_stage* stage, uint64_t seed);
hllm_b200_status hllm_b200_stage_finalize(hllm_b200_stage* stage);

/* StageBackend::weight_memory / hidden_size / vocabulary_size / maximum_tokens
 * (stage_backend.hpp:72-75). */
hllm_b200_status hllm_b200_stage_info(const hllm_b200_stage* stage, uint64_t* weight_device_bytes,
                                      uint64_t* hidden_size, uint64_t* vocabulary_size,
                                      uint64_t* maximum_tokens);

/* Device bytes of the stage, for BackendFactory::allocator_metrics
 * (cpp/include/hllm/runtime/backend_factory.hpp:24-26, 33-35): weights, the
 * step workspace, the paged KV pool, the pool bytes held by live sequences
 * now, and the most they ever held.  All device memory is allocated when the
 * stage is created; nothing is cached or freed during steps. */
hllm_b200_status hllm_b200_stage_memory(hllm_b200_stage* stage, uint64_t* weights,
                                        uint64_t* workspace, uint64_t* kv_pool,
                                        uint64_t* kv_in_use, uint64_t* kv_peak);

/* StageBackend::sequence_memory (stage_backend.hpp:80-81; SequenceMemory
 * memory.hpp:46-49): device bytes a sequence of `tokens` positions holds for
 * its life (whole 16-token KV blocks over this stage's layers), and the shared
 * per-pass workspace, for prefill inputs of at most `maximum_query_tokens`
 * rows. */
hllm_b200_status hllm_b200_sequence_memory(const hllm_b200_stage* stage, uint64_t tokens,
                                           uint64_t maximum_query_tokens,
                                           uint64_t* cache_device_bytes,
                                           uint64_t* workspace_device_bytes);

/* StageBackend::allocate_sequence (stage_backend.hpp:84-85): reserves the KV
 * blocks for `tokens` positions from the paged pool (RESOURCE_EXHAUSTED when
 * the pool cannot hold them). */
hllm_b200_status hllm_b200_seq_alloc(hllm_b200_stage* stage, uint64_t tokens, hllm_b200_seq** out);
/* Returns the sequence's blocks to the pool (the reference frees a request's
 * KV when release() resets its state, cpp/src/worker/control_service.cpp:509-515). */
void hllm_b200_seq_free(hllm_b200_stage* stage, hllm_b200_seq* seq);
/* Current length and capacity; failed != 0 once a pass that included it failed
 * (cpp/src/cuda/stage.cpp:463-468 poisons such sequences). */
hllm_b200_status hllm_b200_seq_info(const hllm_b200_seq* seq, uint64_t* length, uint64_t* capacity,
                                    uint32_t* failed);

/* ------------------------------------------------------------------ step */
/* One pass over a ragged batch: StageBackend::execute for one row and
 * execute_decode_batch for many (stage_backend.hpp:90-97; CUDA
 * cpp/src/cuda/stage.cpp:204-232, 340-470).  Rows may mix prefill chunks and
 * decode tokens.  Rows must name distinct sequences.
 *   final stage: sampled[i] is written for every row with sample != 0;
 *   other stages: boundary receives F16 [sum of tokens][hidden], rows in order.
 * Host outputs are ready when the call returns.  On failure every sequence of
 * the step is marked failed. */
hllm_b200_status hllm_b200_step(hllm_b200_stage* stage, const hllm_b200_row* rows, uint32_t n_rows,
                                hllm_b200_sampled* sampled, uint16_t* boundary);

/* Enqueue-only variant for device-resident inputs: token ids (or F16
 * activations) are read from device memory `device_input` (ids as int32, or
 * F16 [tokens][hidden]) in row order; nothing is copied back and the call does
 * not wait.  Results stay on the device (hllm_b200_stage_results reads them).
 * hllm_b200_stage_sync waits and returns the first failure since the last
 * sync.  No reference counterpart: used to time the hot path with inputs
 * resident in HBM. */
hllm_b200_status hllm_b200_step_async(hllm_b200_stage* stage, const hllm_b200_row* rows,
                                      uint32_t n_rows, const void* device_input);
hllm_b200_status hllm_b200_stage_sync(hllm_b200_stage* stage);
/* Copies the last step's sampled results (one per sampling row, in order). */
hllm_b200_status hllm_b200_stage_results(hllm_b200_stage* stage, hllm_b200_sampled* sampled,
                                         uint32_t count);

/* The stage's CUDA stream (cudaStream_t) and device, for callers that time or
 * order work around steps. */
void* hllm_b200_stage_stream(hllm_b200_stage* stage);
int32_t hllm_b200_stage_device(const hllm_b200_stage* stage);
/* Kernel launches of the last step (for launch accounting). */
uint32_t hllm_b200_stage_last_launches(const hllm_b200_stage* stage);
/* Device address of the stage's F16 boundary output, [tokens][hidden] of the
 * last step (non-final stages), valid until the next step is enqueued; work
 * that reads it must be ordered after the step on the stage stream.  No
 * reference counterpart: pipeline ranks send it to the next stage's GPU
 * device to device instead of through the host. */
const void* hllm_b200_stage_boundary(const hllm_b200_stage* stage);
/* ------------------------------------------------------------------------
 * The F16 boundary on the wire between workers: a serialized
 * hllm.v1.StageMessage whose `tensor` member is a TensorEnvelope
 * (proto/execution.proto:48-65, 115-123).  The bytes are the reference
 * worker's own: encode produces what worker::encode_tensor serializes, decode
 * accepts what worker::decode_tensor accepts, with its checks and messages. */

/* worker::BoundaryIdentity (cpp/include/hllm/worker/boundary_codec.hpp:7-13):
 * the active sequence's deployment and request, its token budget and the
 * model width.  Strings are NUL-terminated UTF-8. */
typedef struct hllm_b200_boundary_identity {
  const char* deployment_id;
  uint64_t deployment_version;
  const char* request_id;
  uint64_t maximum_tokens;
  uint64_t hidden_size;
} hllm_b200_boundary_identity;

/* worker::encode_tensor (cpp/src/worker/boundary_codec.cpp:68-108): the
 * serialized StageMessage for `tokens` F16 rows of `width` (`payload_bytes`
 * bytes at `payload`, host memory) as step `sequence` at `position`; the phase
 * is prefill when sequence == 0 or `prefill`.  With out == NULL only the
 * message size goes to *written.  RESOURCE_EXHAUSTED for a payload above
 * 8 MiB, INTERNAL for a bad shape or a non-finite value (the reference's
 * errors), INVALID_REQUEST when `capacity` is below the size. */
hllm_b200_status hllm_b200_envelope_encode(const hllm_b200_boundary_identity* identity,
                                           uint64_t sequence, uint64_t position, uint32_t prefill,
                                           const uint16_t* payload, uint64_t payload_bytes,
                                           uint64_t tokens, uint64_t width, uint8_t* out,
                                           uint64_t capacity, uint64_t* written);

/* worker::decode_tensor (cpp/src/worker/boundary_codec.cpp:15-66, with
 * runtime::validate_tensor_envelope, cpp/src/tensor_envelope.cpp:26-83) on a
 * received serialized StageMessage: on OK the F16 rows are the
 * *tokens x hidden_size values at message + *payload_offset -- no copy; pass
 * that address as hllm_b200_row.activations.  INVALID_REQUEST with the
 * reference's message otherwise (and "malformed stage message" for bytes
 * that do not parse). */
hllm_b200_status hllm_b200_envelope_decode(const uint8_t* message, uint64_t bytes,
                                           const hllm_b200_boundary_identity* identity,
                                           uint64_t sequence, uint64_t position, uint32_t prefill,
                                           uint64_t* payload_offset, uint64_t* tokens);

/* The envelope of boundary rows [first_token, first_token + tokens) of the
 * stage's last step (a non-final stage), built straight from device memory
 * (no reference counterpart; it replaces the host copy that precedes
 * encode_tensor): the message frame is written on the host and the payload is
 * copied device->host into its place in `out` on a copy stream, ordered after
 * the last step.  The call does not wait: `out` (pinned memory for an
 * asynchronous copy) must stay valid until hllm_b200_stage_envelope_wait.
 * Steps enqueued meanwhile run alongside the copy; only a later step's write
 * of the boundary buffer waits for it.  The last step must have succeeded
 * (its own completion reports a failure). */
hllm_b200_status hllm_b200_stage_envelope(hllm_b200_stage* stage, uint64_t first_token,
                                          uint64_t tokens,
                                          const hllm_b200_boundary_identity* identity,
                                          uint64_t sequence, uint64_t position, uint32_t prefill,
                                          uint8_t* out, uint64_t capacity, uint64_t* written);
/* One row range of the last step's boundary to encode, for
 * hllm_b200_stage_envelopes. */
typedef struct hllm_b200_envelope_row {
  uint64_t first_token;
  uint64_t tokens;
  hllm_b200_boundary_identity identity;
  uint64_t sequence;
  uint64_t position;
  uint32_t prefill;
} hllm_b200_envelope_row;

/* The envelopes of `n` row ranges at once, e.g. one per request of a decode
 * batch (no reference counterpart; each message is what encode_tensor makes
 * for its row).  Messages are written back to back into `out`; message i
 * occupies [offsets[i], offsets[i + 1]) (offsets has n + 1 entries; with
 * out == NULL only offsets are filled).  The rows' payloads go device->host in
 * one copy into pinned staging and are placed into the messages by
 * hllm_b200_stage_envelope_wait; `out` must stay valid until then.  A second
 * call finishes the previous batch first. */
hllm_b200_status hllm_b200_stage_envelopes(hllm_b200_stage* stage,
                                           const hllm_b200_envelope_row* rows, uint32_t n,
                                           uint8_t* out, uint64_t capacity, uint64_t* offsets);
/* Waits for the envelope copies issued since the last wait, places batched
 * payloads into their messages, then applies encode_tensor's finite check to
 * every payload (INTERNAL if one fails). */
hllm_b200_status hllm_b200_stage_envelope_wait(hllm_b200_stage* stage);

/* Host->device and device->host bytes the last step copied. */
hllm_b200_status hllm_b200_stage_last_transfer(const hllm_b200_stage* stage, uint64_t* h2d_bytes,
                                               uint64_t* d2h_bytes);

/* Per-launch timing of the stage's kernels, for benchmarks.  enable != 0
 * resets the counters and brackets every later launch with CUDA events on the
 * stage stream; 0 stops.  Kernel classes: 0 projection GEMMs at decode width
 * (<= 128 tokens), 1 projection GEMMs at prefill width, 2 decode attention
 * (split + combine), 3 prefill attention, 4 packer / embedding / boundary,
 * 5 RMSNorm and residual-add consumers, 6 q/k-norm + RoPE + KV write,
 * 7 SwiGLU / split-sum consumers, 8 sampler.  profile_read
 * waits for the stream and returns a class's summed device milliseconds,
 * launch count, and algorithmic bytes and FLOPs.  No reference counterpart;
 * the reference times components with a host clock after a device
 * synchronize (cpp/include/hllm/runtime/timing.hpp:26-47). */
hllm_b200_status hllm_b200_stage_profile(hllm_b200_stage* stage, uint32_t enable);
hllm_b200_status hllm_b200_stage_profile_read(hllm_b200_stage* stage, uint32_t kind, double* ms,
                                              uint64_t* launches, double* bytes, double* flops);

/* Component timing of a step in the reference's taxonomy
 * (runtime::ExecutionTiming, cpp/include/hllm/runtime/timing.hpp:10-17, as
 * cpp/src/cuda/stage.cpp:394-454 marks it): "embedding" or "from-wire", then
 * "layer" for each owned layer (layer_index = its model index), then
 * "final_norm", "lm_head", "sampling" on a final stage that samples, or
 * "to-wire" on a non-final stage.  Each is the device time from the previous
 * mark (the first from the start of the step, host->device input included),
 * taken with CUDA events on the stage stream rather than host clocks after a
 * synchronize.  enable != 0 records marks on every step; components() returns
 * those of the last hllm_b200_step (the blocking call records the last mark
 * after its device->host copies), *count = their number, at most `capacity`
 * written.  Backs StageBackend::execute_profiled (stage_backend.hpp:103-106). */
typedef struct hllm_b200_component_timing {
  char component[16];
  int64_t layer_index; /* -1: none */
  double milliseconds;
} hllm_b200_component_timing;
hllm_b200_status hllm_b200_stage_component_timing(hllm_b200_stage* stage, uint32_t enable);
hllm_b200_status hllm_b200_stage_components(hllm_b200_stage* stage,
                                            hllm_b200_component_timing* out, uint32_t capacity,
                                            uint32_t* count);

/* Reads back one layer's K or V for positions [0, length) of a sequence as
 * F16 [length][kv_heads][head_dim] (the reference's contiguous cache layout,
 * cpp/src/cpu/llama.cpp:152-158), gathering the paged blocks.  Test trace;
 * the reference's CUDA execute_traced snapshots the same
 * (cpp/include/hllm/cuda/stage.hpp:8-21). */
hllm_b200_status hllm_b200_seq_read_kv(hllm_b200_stage* stage, const hllm_b200_seq* seq,
                                       uint64_t layer, uint32_t values, uint16_t* out);
/* Copies the stage's F32 hidden state of the last step, [tokens][hidden]. */
hllm_b200_status hllm_b200_stage_read_hidden(hllm_b200_stage* stage, float* out, uint64_t tokens);
/* Copies the last step's F32 logits of the sampling rows, [rows][vocab]. */
hllm_b200_status hllm_b200_stage_read_logits(hllm_b200_stage* stage, float* out, uint64_t rows);

/* ------------------------------------------------------ kernel entry points */
/* Device-pointer entry points of the individual kernels, for parity tests and
 * benchmarks of one operator.  All pointers are device memory; `stream` is a
 * cudaStream_t (0 = legacy default stream).  Each call is asynchronous. */

/* Y[n][m] = sum_k X[n][k] W[m][k] on tcgen05 (reference `linear`,
 * cpp/src/cpu/tensor.cpp:47-62).  W: F16 [m][k_pad] (pair == 2: [2*second_row..]
 * gate rows then up rows), X: F16 [n][k_pad] with zero padding columns,
 * k_pad % 64 == 0.  epilogue: 0 store F32, 1 store F16, 2 add into F32 Y,
 * 3 SwiGLU of the pair into F16 Y.  Uses a scratch area owned by the library
 * (allocated on first use per device) that holds one CTA per SM: a split with
 * a larger grid is refused with HLLM_B200_RESOURCE_EXHAUSTED.  A device wait
 * inside the kernel that runs out (2 s) ends the kernel early; this
 * asynchronous entry point does not report it (hllm_b200_step does). */
hllm_b200_status hllm_b200_gemm(const void* w, uint64_t m, uint64_t k_pad, uint32_t pair,
                                uint64_t second_row, const void* x, uint64_t n, uint32_t epilogue,
                                void* y, uint64_t ldy, uint32_t bn, uint32_t grid, void* stream);

/* The same GEMM without allocating anything.  No counterpart in the reference:
 * it exists for callers that cannot let a library allocate device memory --
 * a serving process that fixes its device budget at start-up and admits
 * requests against it, or a host that owns all of a plugin's device memory.
 * Its split-K scratch is a static device array of 32 MiB of partial sums, plus
 * a 256-byte status word, that every GPU loading the library holds until the
 * process exits.
 * Splits that need more partial-sum storage than that are rejected with
 * HLLM_B200_RESOURCE_EXHAUSTED and a message; plans that need none always run.
 * The first call on a device, with that device current, resolves the array's
 * device address (cudaGetSymbolAddress); make that first call before any
 * stream capture.  All calls on a device share the array: calls whose GPU
 * work overlaps (e.g. on two streams) race and must not be issued.  Calls no
 * cudaMalloc/cudaFree.  As for hllm_b200_gemm, a device wait that runs out is
 * not reported by this asynchronous call. */
hllm_b200_status hllm_b200_gemm_noalloc(const void* w, uint64_t m, uint64_t k_pad, uint32_t pair,
                                        uint64_t second_row, const void* x, uint64_t n,
                                        uint32_t epilogue, void* y, uint64_t ldy, uint32_t bn,
                                        uint32_t grid, void* stream);

/* RMSNorm of rows of F32 x into F16 out (cpp/src/cpu/llama.cpp:193-212). */
hllm_b200_status hllm_b200_rmsnorm(const float* x, uint64_t rows, uint64_t width, const float* w,
                                   float eps, uint16_t* out, uint64_t ld_out, void* stream);

/* The ragged packer (no reference counterpart; oracle_pack restates it):
 * from row_slot/row_first/row_count [rows] and slot_blocks [slots][max_blocks]
 * writes cu_seqlens [rows+1], positions, slot_mapping, token_row [tokens],
 * seq_lens [rows], block_tables [rows][max_blocks], cu_splits and cu_qtiles
 * [rows+1].  status (device u32) receives error bits. */
hllm_b200_status hllm_b200_pack(const int32_t* row_slot, const int32_t* row_first,
                                const int32_t* row_count, uint32_t rows, uint32_t tokens,
                                const int32_t* slot_blocks, uint32_t max_blocks,
                                uint32_t split_tokens, uint32_t qtile_tokens, int32_t* cu_seqlens,
                                int32_t* positions, int32_t* slot_mapping, int32_t* token_row,
                                int32_t* seq_lens, int32_t* block_tables, int32_t* cu_splits,
                                int32_t* cu_qtiles, uint32_t* status, void* stream);

/* Paged GQA attention over a packed batch (reference `attention`,
 * cpp/src/cpu/llama.cpp:67-112).  q F16 [q_tokens][Hq*d]; caches F16
 * [kv_blocks][Hkv][16][d]; packer outputs as above; out F16 [tokens][ld_out].
 * Decode rows (one token): for head sizes 64/128/256 the decode rows' KV
 * pages are split evenly over one wave of warps, each streaming its pages by
 * TMA (kv_blocks bounds the maps and is required), and a second launch
 * merges the pieces of each (row, kv head) split across warps (cu_splits
 * and split_tokens only bound the work); other head sizes use split-K over
 * `split_tokens`-key splits.  Prefill rows: causal tiles of hllm_b200_attention_qtile_tokens(
 * Hq/Hkv) tokens, each tile's keys split over CTAs that fill one wave; for
 * head sizes 64 and 128 (GQA groups 1/2/4/8) on tcgen05 with S and O in TMEM
 * and TMA-fed K/V pages (q_tokens and kv_blocks bound the TMA maps; 0 selects
 * the mma.sync tiles, as HLLM_B200_TC_PREFILL=0 does).  Split outputs, the
 * decode streams' warp ranges and the prefill arrival counters live in a
 * per-device workspace that the first call allocates. */
hllm_b200_status hllm_b200_attention(const uint16_t* q, const uint16_t* k_cache,
                                     const uint16_t* v_cache, const int32_t* row_first,
                                     const int32_t* row_count, const int32_t* cu_seqlens,
                                     const int32_t* seq_lens, const int32_t* block_tables,
                                     const int32_t* cu_splits, const int32_t* cu_qtiles,
                                     uint32_t rows, uint32_t total_splits, uint32_t total_qtiles,
                                     uint32_t hq, uint32_t hkv, uint32_t dim, uint32_t max_blocks,
                                     uint32_t split_tokens, uint16_t* out, uint64_t ld_out,
                                     uint64_t q_tokens, uint64_t kv_blocks, uint32_t* status,
                                     void* stream);
/* Query tokens per prefill tile for a GQA group size (128 query rows per
 * tile: 128 / group tokens). */
uint32_t hllm_b200_attention_qtile_tokens(uint32_t group);

/* q/k RMSNorm + RoPE + paged K/V write for a packed batch (reference
 * cpp/src/cpu/llama.cpp:255-264).  qkv F32 [tokens][(Hq+2Hkv)d];
 * rope_pow [d/2] = theta^(2i/d) as the reference computes it. */
hllm_b200_status hllm_b200_qkv_post(const float* qkv, uint64_t tokens, uint32_t hq, uint32_t hkv,
                                    uint32_t dim, const int32_t* positions,
                                    const int32_t* slot_mapping, const float* q_norm,
                                    const float* k_norm, float eps, const float* rope_pow,
                                    uint16_t* q_out, uint16_t* k_cache, uint16_t* v_cache,
                                    void* stream);

/* Sampler (reference sample_token, cpp/src/sampling.cpp:19-90): logits F32
 * [rows][ld] on the device, options per row on the host; results to host. */
hllm_b200_status hllm_b200_sample(const float* logits, uint32_t rows, uint64_t vocab, uint64_t ld,
                                  const hllm_b200_sampling* options,
                                  const uint64_t* generated_index, hllm_b200_sampled* out,
                                  void* stream);

/* Seeded synthetic F16 matrix [rows][cols] at row stride ld (device). */
hllm_b200_status hllm_b200_synth_matrix(uint64_t seed, uint64_t tag, uint64_t rows, uint64_t cols,
                                        uint64_t ld, float stddev, uint16_t* out, void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* HLLM_B200_H_ */
