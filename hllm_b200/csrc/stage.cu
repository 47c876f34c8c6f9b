// stage.cu -- the B200 stage executor behind the C ABI in include/hllm_b200.h.
//
// Host side of one hLLM stage: weight upload and seeded initialisation, the
// paged KV pool and its block allocator, per-sequence block lists, and the
// per-step launch sequence
//
//   H2D(row descriptors, ids) -> pack -> embed | boundary-in
//   per layer: rmsnorm -> QKV GEMM -> q/k-norm+RoPE+KV write -> attention
//              -> O GEMM (+residual) -> rmsnorm -> gate/up GEMM (SwiGLU)
//              -> down GEMM (+residual)
//   final stage: last-row gather + final norm -> LM-head GEMM -> sampler
//   other stages: F16 boundary
//   D2H(status, sampled tokens | boundary)
//
// which restates, in one ragged pass, what the reference CUDA stage does per
// sequence (cpp/src/cuda/stage.cpp:340-470) and the CPU oracle defines
// (cpp/src/cpu/stage.cpp:129-191, cpp/src/cpu/llama.cpp:242-308).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <new>
#include <set>
#include <string>
#include <vector>

#include "attention.cuh"
#include "common.cuh"
#include "envelope.cuh"
#include "gemm.cuh"
#include "hllm_b200.h"
#include "kernels.cuh"
#include "sampler.cuh"

namespace {

thread_local std::string g_last_error;

struct Fail {
  hllm_b200_status code;
  std::string message;
};
[[noreturn]] void fail(hllm_b200_status code, const std::string& message) {
  throw Fail{code, message};
}
void check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    if (e == cudaErrorMemoryAllocation)
      fail(HLLM_B200_RESOURCE_EXHAUSTED, std::string(what) + ": device memory exhausted");
    fail(HLLM_B200_INTERNAL, std::string(what) + ": " + cudaGetErrorString(e));
  }
}
template <class F>
hllm_b200_status guarded(F&& f) {
  try {
    f();
    return HLLM_B200_OK;
  } catch (const Fail& e) {
    g_last_error = e.message;
    return e.code;
  } catch (const std::bad_alloc&) {
    g_last_error = "host allocation failed";
    return HLLM_B200_RESOURCE_EXHAUSTED;
  } catch (const std::exception& e) {
    g_last_error = e.what();
    return HLLM_B200_INTERNAL;
  }
}

size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

constexpr uint32_t kInputNonFinite = hb::kDevNonFiniteInput;

struct DeviceBuffer {
  void* ptr = nullptr;
  size_t bytes = 0;
  DeviceBuffer() = default;
  DeviceBuffer(const DeviceBuffer&) = delete;
  DeviceBuffer& operator=(const DeviceBuffer&) = delete;
  ~DeviceBuffer() {
    if (ptr) cudaFree(ptr);
  }
};

struct Layer {
  __half* qkv = nullptr;      // [Hq d + 2 Hkv d][h_pad]
  __half* o = nullptr;        // [h][qw_pad]
  __half* gate_up = nullptr;  // [2I][h_pad]: gate rows then up rows
  __half* down = nullptr;     // [h][I_pad]
  float* in_norm = nullptr;
  float* post_norm = nullptr;
  float* q_norm = nullptr;
  float* k_norm = nullptr;
  hb::GemmWeight g_qkv{}, g_o{}, g_gu{}, g_down{};
};

// Where a named tensor lands on the device.
struct Target {
  enum Kind { kMatrix, kNorm } kind;
  __half* matrix = nullptr;  // base of the destination matrix
  size_t row_offset = 0;     // first destination row
  size_t ld = 0;             // destination row stride (elements)
  float* norm = nullptr;
  size_t rows = 0, cols = 0;  // expected source shape
  uint64_t tag = 0;           // synthetic-weight tag
};

}  // namespace

namespace hb {
void set_last_error(const std::string& message) { g_last_error = message; }
}  // namespace hb

struct hllm_b200_seq {
  hllm_b200_stage* owner = nullptr;
  int slot = -1;
  std::vector<int32_t> blocks;
  uint64_t capacity = 0;
  uint64_t length = 0;
  bool failed = false;
};

struct hllm_b200_stage {
  hllm_b200_stage_desc desc{};
  int device = 0;
  int sm_count = 0;
  cudaStream_t stream = nullptr;
  size_t h = 0, I = 0, hq = 0, hkv = 0, dim = 0, qw = 0, kw = 0, qkvw = 0, V = 0;
  size_t h_pad = 0, qw_pad = 0, I_pad = 0;
  size_t n_layers = 0;
  size_t max_blocks = 0, num_blocks = 0;
  size_t T_max = 0, R_max = 0, max_seqs = 0, max_splits = 0;
  size_t weight_bytes = 0, workspace_bytes = 0;
  std::vector<std::unique_ptr<DeviceBuffer>> owned;

  __half* embed = nullptr;
  __half* head = nullptr;
  float* final_norm = nullptr;
  std::vector<Layer> layers;
  hb::GemmWeight g_head{};
  __half* kv = nullptr;  // [layers][2][blocks][Hkv][16][d]
  size_t kv_layer_elems = 0;
  size_t kv_peak_blocks = 0;  // most pool blocks ever held by live sequences
  float* rope_pow = nullptr;
  float2* rope_table = nullptr;  // [max positions][d/2] (cos, sin)
  int rope_positions = 0;

  // per-step device tensors
  int32_t* up = nullptr;  // row_slot | row_first | row_count | sample_rows | ids
  hb::SampleParams* d_params = nullptr;
  size_t up_bytes = 0;
  int32_t *row_slot = nullptr, *row_first = nullptr, *row_count = nullptr, *sample_rows = nullptr,
          *ids = nullptr;
  int32_t *cu_seqlens = nullptr, *positions = nullptr, *slot_mapping = nullptr,
          *token_row = nullptr, *seq_lens = nullptr, *block_tables = nullptr,
          *cu_splits = nullptr, *cu_qtiles = nullptr, *last_idx = nullptr;
  int32_t* slot_blocks = nullptr;  // [max_seqs][max_blocks]
  uint8_t* down = nullptr;         // status (8 bytes) | SampleResult[R_max]
  uint32_t* status = nullptr;
  hb::SampleResult* results = nullptr;
  float* hidden = nullptr;
  __half *xn = nullptr, *q = nullptr, *attn = nullptr, *act = nullptr, *xs = nullptr,
         *bin = nullptr, *bout = nullptr;
  float* qkv = nullptr;
  float* logits = nullptr;
  double* sample_scratch = nullptr;
  float *part_o = nullptr, *part_ml = nullptr;
  int* attn_counters = nullptr;  // [R_max][Hkv] decode streams' warp ranges (per launch)
  size_t attn_counter_ints = 0;
  float* pre_part = nullptr;     // prefill key-split pieces
  int* pre_counters = nullptr;   // [max qtiles][Hkv] split arrival counters (self-resetting)
  size_t pre_counter_ints = 0;
  int max_qtiles = 0;
  hb::GemmInput in_xn{}, in_attn{}, in_act{}, in_xs{};
  // Prefill attention on tcgen05 (head sizes 64/128): per-layer TMA maps of
  // the query buffer and the layer's K/V caches.  HLLM_B200_TC_PREFILL=0
  // selects the mma.sync kernel instead (for comparisons).
  bool tc_prefill = false;
  std::vector<hb::TcMaps> tc_maps;
  float* slots = nullptr;  // stream-K GEMM slots, consumed by the next kernel

  // pinned host staging
  // Descriptor uploads go through a ring of pinned buffers so that enqueue-only
  // steps never overwrite a buffer whose copy has not run; each slot's event
  // marks its copy as consumed.
  static constexpr int kUpRing = 8;
  uint8_t* h_up_ring[kUpRing] = {};
  cudaEvent_t up_done[kUpRing] = {};
  int up_next = 0;
  uint8_t* h_up = nullptr;  // the ring slot of the step being built
  uint8_t* h_down = nullptr;
  int32_t* h_slot_rows = nullptr;             // pinned [max_seqs][max_blocks] block-list staging
  std::vector<cudaEvent_t> slot_copy_done;    // per slot: its last staging copy has run
  __half* h_act = nullptr;  // boundary in/out staging [T_max][h]
  // Envelope copies (hllm_b200_stage_envelope): boundary rows go device->host
  // on their own stream after the step that wrote them; a later step's
  // boundary write waits for env_done.  Payloads are checked at the next wait.
  cudaStream_t copy_stream = nullptr;
  cudaEvent_t step_done = nullptr, env_done = nullptr;
  bool env_pending = false;
  std::vector<std::pair<const uint8_t*, uint64_t>> env_payloads;
  // Batched envelopes (hllm_b200_stage_envelopes): one device->host copy of the
  // rows into pinned staging, placed into the messages at the next wait.
  uint8_t* h_env = nullptr;
  struct EnvPlace {
    uint8_t* dst;
    uint64_t src, bytes;  // offset into h_env, length
  };
  std::vector<EnvPlace> env_places;

  std::map<std::string, Target> targets;
  std::set<std::string> loaded;
  bool finalized = false;
  std::vector<int32_t> free_blocks;
  std::vector<int> free_slots;
  std::set<hllm_b200_seq*> live;
  uint32_t launches = 0;
  uint64_t last_h2d = 0, last_d2h = 0;  // host<->device bytes of the last step
  uint32_t last_samples = 0;
  uint64_t last_tokens = 0;
  std::vector<hllm_b200_seq*> pending;  // sequences of steps enqueued since the last sync
  std::mutex mutex;

  // Optional per-launch timing (hllm_b200_stage_profile): CUDA events around
  // every launch, grouped by kernel class, with each launch's algorithmic
  // bytes and FLOPs.
  struct ProfEvent {
    int kind;
    double bytes, flops;
    cudaEvent_t a, b;
  };
  static constexpr int kProfKinds = 9;
  bool profiling = false;
  std::vector<ProfEvent> prof_pending;
  std::vector<cudaEvent_t> event_pool;
  double prof_ms[kProfKinds] = {}, prof_bytes[kProfKinds] = {}, prof_flops[kProfKinds] = {};
  uint64_t prof_n[kProfKinds] = {};
  cudaEvent_t prof_open = nullptr;

  // Component timing (hllm_b200_stage_component_timing): CUDA events at the
  // reference's phase boundaries of a step -- input, each layer, final norm,
  // LM head, sampling or boundary output (cpp/src/cuda/stage.cpp:394-454).
  struct Mark {
    const char* name;
    int64_t layer;
    cudaEvent_t ev;
  };
  bool comp_timing = false;
  std::vector<Mark> marks;  // the last step's
  std::vector<cudaEvent_t> mark_pool;
  cudaEvent_t mark_start = nullptr;

  void mark_begin() {
    if (!comp_timing) return;
    marks.clear();
    if (!mark_start) check_cuda(cudaEventCreate(&mark_start), "cudaEventCreate");
    check_cuda(cudaEventRecord(mark_start, stream), "component timing");
  }
  void mark(const char* name, int64_t layer = -1) {
    if (!comp_timing) return;
    if (marks.size() == mark_pool.size()) {
      cudaEvent_t e;
      check_cuda(cudaEventCreate(&e), "cudaEventCreate");
      mark_pool.push_back(e);
    }
    cudaEvent_t e = mark_pool[marks.size()];
    check_cuda(cudaEventRecord(e, stream), "component timing");
    marks.push_back({name, layer, e});
  }

  ~hllm_b200_stage() {
    if (copy_stream) {
      cudaStreamSynchronize(copy_stream);
      cudaStreamDestroy(copy_stream);
    }
    if (step_done) cudaEventDestroy(step_done);
    if (env_done) cudaEventDestroy(env_done);
    if (h_env) cudaFreeHost(h_env);
    if (stream) {
      cudaStreamSynchronize(stream);
      cudaStreamDestroy(stream);
    }
    for (int i = 0; i < kUpRing; ++i) {
      if (h_up_ring[i]) cudaFreeHost(h_up_ring[i]);
      if (up_done[i]) cudaEventDestroy(up_done[i]);
    }
    if (h_down) cudaFreeHost(h_down);
    if (h_act) cudaFreeHost(h_act);
    if (h_slot_rows) cudaFreeHost(h_slot_rows);
    for (auto e : slot_copy_done) cudaEventDestroy(e);
    for (auto* s : live) delete s;
    for (auto& e : prof_pending) {
      cudaEventDestroy(e.a);
      cudaEventDestroy(e.b);
    }
    for (auto e : event_pool) cudaEventDestroy(e);
    for (auto e : mark_pool) cudaEventDestroy(e);
    if (mark_start) cudaEventDestroy(mark_start);
  }

  cudaEvent_t take_event() {
    if (event_pool.empty()) {
      cudaEvent_t e;
      check_cuda(cudaEventCreate(&e), "cudaEventCreate");
      return e;
    }
    cudaEvent_t e = event_pool.back();
    event_pool.pop_back();
    return e;
  }
  void prof_begin() {
    if (!profiling) return;
    prof_open = take_event();
    check_cuda(cudaEventRecord(prof_open, stream), "cudaEventRecord");
  }
  void prof_end(int kind, double bytes, double flops) {
    if (!profiling) return;
    cudaEvent_t b = take_event();
    check_cuda(cudaEventRecord(b, stream), "cudaEventRecord");
    prof_pending.push_back({kind, bytes, flops, prof_open, b});
    prof_open = nullptr;
  }
  // Call after the stream has drained the recorded events.
  void prof_collect() {
    for (auto& e : prof_pending) {
      float ms = 0.f;
      if (cudaEventElapsedTime(&ms, e.a, e.b) == cudaSuccess) {
        prof_ms[e.kind] += ms;
        prof_bytes[e.kind] += e.bytes;
        prof_flops[e.kind] += e.flops;
        prof_n[e.kind] += 1;
      }
      event_pool.push_back(e.a);
      event_pool.push_back(e.b);
    }
    prof_pending.clear();
  }

  template <class T>
  T* alloc(size_t count, bool track_weight = false) {
    auto b = std::make_unique<DeviceBuffer>();
    b->bytes = std::max<size_t>(count * sizeof(T), 256);
    check_cuda(cudaMalloc(&b->ptr, b->bytes), "cudaMalloc");
    check_cuda(cudaMemsetAsync(b->ptr, 0, b->bytes, stream), "cudaMemset");
    if (track_weight) weight_bytes += b->bytes;
    else workspace_bytes += b->bytes;
    T* p = static_cast<T*>(b->ptr);
    owned.push_back(std::move(b));
    return p;
  }
};

namespace {

constexpr uint64_t kTagEmbed = 0xE0000, kTagHead = 0xE0001, kTagFinalNorm = 0xE0002;
constexpr float kWeightStd = 0.02f, kNormSpread = 0.1f;

void add_matrix(hllm_b200_stage* s, const std::string& name, __half* base, size_t row_offset,
                size_t ld, size_t rows, size_t cols, uint64_t tag) {
  Target t{Target::kMatrix};
  t.matrix = base;
  t.row_offset = row_offset;
  t.ld = ld;
  t.rows = rows;
  t.cols = cols;
  t.tag = tag;
  s->targets[name] = t;
}
void add_norm(hllm_b200_stage* s, const std::string& name, float* dst, size_t n, uint64_t tag) {
  Target t{Target::kNorm};
  t.norm = dst;
  t.rows = n;
  t.cols = 1;
  t.tag = tag;
  s->targets[name] = t;
}

void build_stage(hllm_b200_stage* s, const hllm_b200_stage_desc& d) {
  s->desc = d;
  if (d.hidden_size == 0 || d.intermediate_size == 0 || d.attention_heads == 0 ||
      d.key_value_heads == 0 || d.head_dimension == 0 || d.maximum_sequence_length == 0 ||
      d.vocabulary_size == 0 || !(d.rms_norm_epsilon > 0.f) || !(d.rope_theta > 0.f) ||
      !std::isfinite(d.rms_norm_epsilon) || !std::isfinite(d.rope_theta))
    fail(HLLM_B200_INVALID_REQUEST, "stage configuration values must be positive");
  if (d.attention_heads % d.key_value_heads != 0 || d.head_dimension % 4 != 0 ||
      d.head_dimension > 256 || d.attention_heads / d.key_value_heads > 8)
    fail(HLLM_B200_INCOMPATIBLE_WORKER,
         "attention geometry unsupported (head_dim % 4, head_dim <= 256, group <= 8)");
  if (d.layer_end < d.layer_start) fail(HLLM_B200_INVALID_REQUEST, "invalid layer range");
  if (d.hidden_size > (1u << 20) || d.vocabulary_size > (1u << 30) ||
      d.maximum_sequence_length > (1u << 24))
    fail(HLLM_B200_INCOMPATIBLE_WORKER, "stage dimensions exceed executor limits");
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess) count = 0;
  if (d.device_id < 0 || d.device_id >= count)
    fail(HLLM_B200_INCOMPATIBLE_WORKER, "no such CUDA device");
  s->device = d.device_id;
  check_cuda(cudaSetDevice(s->device), "cudaSetDevice");
  cudaDeviceProp prop{};
  check_cuda(cudaGetDeviceProperties(&prop, s->device), "cudaGetDeviceProperties");
  if (prop.major != 10)
    fail(HLLM_B200_INCOMPATIBLE_WORKER, "the B200 executor needs an sm_100 device");
  s->sm_count = prop.multiProcessorCount;
  check_cuda(cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking), "cudaStreamCreate");

  s->h = d.hidden_size;
  s->I = d.intermediate_size;
  s->hq = d.attention_heads;
  s->hkv = d.key_value_heads;
  s->dim = d.head_dimension;
  s->qw = s->hq * s->dim;
  s->kw = s->hkv * s->dim;
  s->qkvw = s->qw + 2 * s->kw;
  s->V = d.vocabulary_size;
  s->h_pad = round_up(s->h, 64);
  s->qw_pad = round_up(s->qw, 64);
  s->I_pad = round_up(s->I, 64);
  s->n_layers = d.layer_end - d.layer_start;
  s->max_blocks = (d.maximum_sequence_length + hb::kBlockTokens - 1) / hb::kBlockTokens;
  s->num_blocks = std::max<uint64_t>(1, (d.kv_pool_tokens + hb::kBlockTokens - 1) / hb::kBlockTokens);
  s->T_max = d.max_step_tokens ? d.max_step_tokens : 2048;
  s->R_max = d.max_step_rows ? d.max_step_rows : 256;
  s->max_seqs = d.max_sequences ? d.max_sequences : 512;
  s->max_splits = std::max<size_t>(4096, 2 * s->R_max);
  if (s->R_max > s->T_max) s->R_max = s->T_max;

  // ---- weights
  if (d.first || (d.final && d.tied_head)) {
    s->embed = s->alloc<__half>(s->V * s->h_pad, true);
    add_matrix(s, "model.embed_tokens.weight", s->embed, 0, s->h_pad, s->V, s->h, kTagEmbed);
  }
  if (d.final) {
    s->final_norm = s->alloc<float>(s->h, true);
    add_norm(s, "model.norm.weight", s->final_norm, s->h, kTagFinalNorm);
    if (!d.tied_head) {
      s->head = s->alloc<__half>(s->V * s->h_pad, true);
      add_matrix(s, "lm_head.weight", s->head, 0, s->h_pad, s->V, s->h, kTagHead);
    }
  }
  s->layers.resize(s->n_layers);
  for (size_t li = 0; li < s->n_layers; ++li) {
    const size_t gl = d.layer_start + li;
    Layer& L = s->layers[li];
    const std::string p = "model.layers." + std::to_string(gl) + ".";
    const uint64_t tb = gl * 16;
    L.in_norm = s->alloc<float>(s->h, true);
    L.post_norm = s->alloc<float>(s->h, true);
    L.qkv = s->alloc<__half>(s->qkvw * s->h_pad, true);
    L.o = s->alloc<__half>(s->h * s->qw_pad, true);
    L.gate_up = s->alloc<__half>(2 * s->I * s->h_pad, true);
    L.down = s->alloc<__half>(s->h * s->I_pad, true);
    add_norm(s, p + "input_layernorm.weight", L.in_norm, s->h, tb + 0);
    add_matrix(s, p + "self_attn.q_proj.weight", L.qkv, 0, s->h_pad, s->qw, s->h, tb + 1);
    add_matrix(s, p + "self_attn.k_proj.weight", L.qkv, s->qw, s->h_pad, s->kw, s->h, tb + 2);
    add_matrix(s, p + "self_attn.v_proj.weight", L.qkv, s->qw + s->kw, s->h_pad, s->kw, s->h,
               tb + 3);
    add_matrix(s, p + "self_attn.o_proj.weight", L.o, 0, s->qw_pad, s->h, s->qw, tb + 4);
    add_norm(s, p + "post_attention_layernorm.weight", L.post_norm, s->h, tb + 5);
    add_matrix(s, p + "mlp.gate_proj.weight", L.gate_up, 0, s->h_pad, s->I, s->h, tb + 6);
    add_matrix(s, p + "mlp.up_proj.weight", L.gate_up, s->I, s->h_pad, s->I, s->h, tb + 7);
    add_matrix(s, p + "mlp.down_proj.weight", L.down, 0, s->I_pad, s->h, s->I, tb + 8);
    if (d.query_key_norm) {
      L.q_norm = s->alloc<float>(s->dim, true);
      L.k_norm = s->alloc<float>(s->dim, true);
      add_norm(s, p + "self_attn.q_norm.weight", L.q_norm, s->dim, tb + 9);
      add_norm(s, p + "self_attn.k_norm.weight", L.k_norm, s->dim, tb + 10);
    }
    if (!hb::gemm_make_weight(&L.g_qkv, L.qkv, static_cast<int>(s->qkvw), static_cast<int>(s->qkvw),
                              static_cast<int>(s->h_pad), 1, 0) ||
        !hb::gemm_make_weight(&L.g_o, L.o, static_cast<int>(s->h), static_cast<int>(s->h),
                              static_cast<int>(s->qw_pad), 1, 0) ||
        !hb::gemm_make_weight(&L.g_gu, L.gate_up, static_cast<int>(2 * s->I),
                              static_cast<int>(s->I), static_cast<int>(s->h_pad), 2,
                              static_cast<int>(s->I)) ||
        !hb::gemm_make_weight(&L.g_down, L.down, static_cast<int>(s->h), static_cast<int>(s->h),
                              static_cast<int>(s->I_pad), 1, 0))
      fail(HLLM_B200_INTERNAL, "tensor map creation failed");
  }
  if (d.final) {
    const __half* hm = d.tied_head ? s->embed : s->head;
    if (!hb::gemm_make_weight(&s->g_head, hm, static_cast<int>(s->V), static_cast<int>(s->V),
                              static_cast<int>(s->h_pad), 1, 0))
      fail(HLLM_B200_INTERNAL, "tensor map creation failed");
  }

  // ---- KV pool and sequence tables
  s->kv_layer_elems = 2 * s->num_blocks * s->hkv * hb::kBlockTokens * s->dim;
  s->kv = s->alloc<__half>(std::max<size_t>(1, s->n_layers) * s->kv_layer_elems);
  s->slot_blocks = s->alloc<int32_t>(s->max_seqs * s->max_blocks);
  for (size_t b = s->num_blocks; b-- > 0;) s->free_blocks.push_back(static_cast<int32_t>(b));
  for (size_t i = s->max_seqs; i-- > 0;) s->free_slots.push_back(static_cast<int>(i));

  // RoPE divisors theta^(2i/d), computed on the host with the reference's
  // F32 expression (cpp/src/cpu/llama.cpp:225-228).
  std::vector<float> pw(s->dim / 2);
  for (size_t i = 0; i < pw.size(); ++i)
    pw[i] = std::pow(d.rope_theta,
                     static_cast<float>(2U * i) / static_cast<float>(s->dim));
  s->rope_pow = s->alloc<float>(pw.size());
  check_cuda(cudaMemcpyAsync(s->rope_pow, pw.data(), pw.size() * sizeof(float),
                             cudaMemcpyHostToDevice, s->stream), "rope upload");
  // (cos, sin) of position / theta^(2i/d) for every position, from the same
  // F32 expressions (cpp/src/cpu/llama.cpp:222-231), so that the rotation
  // matches the reference's values exactly.
  {
    const size_t positions = d.maximum_sequence_length, half = s->dim / 2;
    std::vector<float2> table(positions * half);
    for (size_t pos = 0; pos < positions; ++pos) {
      const float position = static_cast<float>(pos);
      for (size_t i = 0; i < half; ++i) {
        const float angle = position / pw[i];
        table[pos * half + i] = make_float2(std::cos(angle), std::sin(angle));
      }
    }
    s->rope_table = s->alloc<float2>(table.size());
    s->rope_positions = static_cast<int>(positions);
    check_cuda(cudaMemcpy(s->rope_table, table.data(), table.size() * sizeof(float2),
                          cudaMemcpyHostToDevice), "rope table upload");
  }

  // ---- step workspaces
  const size_t R = s->R_max, T = s->T_max;
  s->up_bytes = (4 * R + T) * sizeof(int32_t);
  s->up_bytes = round_up(s->up_bytes, 16) + R * sizeof(hb::SampleParams);
  s->up = s->alloc<int32_t>(s->up_bytes / sizeof(int32_t) + 4);
  s->row_slot = s->up;
  s->row_first = s->up + R;
  s->row_count = s->up + 2 * R;
  s->sample_rows = s->up + 3 * R;
  s->ids = s->up + 4 * R;
  s->d_params = reinterpret_cast<hb::SampleParams*>(
      reinterpret_cast<uint8_t*>(s->up) + round_up((4 * R + T) * sizeof(int32_t), 16));
  s->cu_seqlens = s->alloc<int32_t>(R + 1);
  s->positions = s->alloc<int32_t>(T);
  s->slot_mapping = s->alloc<int32_t>(T);
  s->token_row = s->alloc<int32_t>(T);
  s->seq_lens = s->alloc<int32_t>(R);
  s->block_tables = s->alloc<int32_t>(R * s->max_blocks);
  s->cu_splits = s->alloc<int32_t>(R + 1);
  s->cu_qtiles = s->alloc<int32_t>(R + 1);
  s->last_idx = s->alloc<int32_t>(R);
  s->down = s->alloc<uint8_t>(8 + R * sizeof(hb::SampleResult));
  s->status = reinterpret_cast<uint32_t*>(s->down);
  s->results = reinterpret_cast<hb::SampleResult*>(s->down + 8);
  s->hidden = s->alloc<float>(T * s->h);
  s->xn = s->alloc<__half>(T * s->h_pad);
  s->qkv = s->alloc<float>(T * s->qkvw);
  s->q = s->alloc<__half>(T * s->qw);
  s->attn = s->alloc<__half>(T * s->qw_pad);
  s->act = s->alloc<__half>(T * s->I_pad);
  s->bin = s->alloc<__half>(T * s->h);
  s->bout = s->alloc<__half>(T * s->h);
  if (d.final) {
    s->xs = s->alloc<__half>(R * s->h_pad);
    s->logits = s->alloc<float>(R * s->V);
    s->sample_scratch = s->alloc<double>(R * s->V);
  }
  {
    // Partial decode outputs: split-K splits (combine path) or the balanced
    // pass's pieces, whichever needs more.
    const int max_ctas = hb::attn_decode_ctas(static_cast<int>(s->dim), static_cast<int>(s->hq / s->hkv),
                                              1LL << 40, s->sm_count);
    const size_t pieces = R * s->hkv + 4 * static_cast<size_t>(max_ctas);
    const size_t group = s->hq / s->hkv;
    s->part_o = s->alloc<float>(std::max(s->max_splits * s->hq, pieces * group) * s->dim);
    s->part_ml = s->alloc<float>(std::max(s->max_splits * s->hq, pieces * group) * 2);
  }
  s->attn_counter_ints = R * s->hkv;
  s->attn_counters = s->alloc<int>(s->attn_counter_ints);
  {
    // Prefill tiles: at most one partial tile per row beyond T / qtile_tokens.
    const int qt = hb::attn_qtile_tokens(static_cast<int>(s->hq / s->hkv));
    s->max_qtiles = static_cast<int>((T + qt - 1) / qt + R);
    s->pre_part = s->alloc<float>(std::max<size_t>(
        1, hb::attn_prefill_part_floats(static_cast<int>(s->dim), static_cast<int>(s->hkv),
                                        s->max_qtiles, hb::kPrefillMaxSplits)));
    s->pre_counter_ints = static_cast<size_t>(s->max_qtiles) * s->hkv;
    s->pre_counters = s->alloc<int>(s->pre_counter_ints);
  }
  s->slots = s->alloc<float>(hb::gemm_max_slot_floats(s->sm_count));
  {
    // TMA maps per layer: K and V for the balanced decode pass (head sizes
    // 64/128/256) and, with the query buffer, for the tcgen05 prefill.
    const char* env = std::getenv("HLLM_B200_TC_PREFILL");
    s->tc_prefill = hb::attn_prefill_tc_supported(static_cast<int>(s->dim),
                                                  static_cast<int>(s->hq / s->hkv)) &&
                    !(env && env[0] == '0');
    if (s->tc_prefill || hb::attn_decode_balanced(static_cast<int>(s->dim))) {
      s->tc_maps.resize(std::max<size_t>(1, s->n_layers));
      for (size_t li = 0; li < s->n_layers; ++li) {
        const __half* kc = s->kv + li * s->kv_layer_elems;
        const __half* vc = kc + s->kv_layer_elems / 2;
        const bool ok =
            s->tc_prefill
                ? hb::attn_tc_make_maps(&s->tc_maps[li], s->q, static_cast<long long>(T),
                                        static_cast<int>(s->hq), static_cast<int>(s->hkv),
                                        static_cast<int>(s->dim), kc, vc,
                                        static_cast<long long>(s->num_blocks))
                : hb::attn_make_kv_maps(&s->tc_maps[li], static_cast<int>(s->hkv),
                                        static_cast<int>(s->dim), kc, vc,
                                        static_cast<long long>(s->num_blocks));
        if (!ok) fail(HLLM_B200_INTERNAL, "tensor map creation failed");
      }
    }
  }
  if (!hb::gemm_make_input(&s->in_xn, s->xn, static_cast<int>(T), static_cast<int>(s->h_pad),
                           static_cast<int>(s->h_pad)) ||
      !hb::gemm_make_input(&s->in_attn, s->attn, static_cast<int>(T), static_cast<int>(s->qw_pad),
                           static_cast<int>(s->qw_pad)) ||
      !hb::gemm_make_input(&s->in_act, s->act, static_cast<int>(T), static_cast<int>(s->I_pad),
                           static_cast<int>(s->I_pad)) ||
      (d.final && !hb::gemm_make_input(&s->in_xs, s->xs, static_cast<int>(R),
                                       static_cast<int>(s->h_pad), static_cast<int>(s->h_pad))))
    fail(HLLM_B200_INTERNAL, "tensor map creation failed");

  for (int i = 0; i < hllm_b200_stage::kUpRing; ++i) {
    check_cuda(cudaMallocHost(&s->h_up_ring[i], s->up_bytes), "cudaMallocHost");
    check_cuda(cudaEventCreateWithFlags(&s->up_done[i], cudaEventDisableTiming), "cudaEventCreate");
  }
  check_cuda(cudaMallocHost(&s->h_down, 8 + R * sizeof(hb::SampleResult)), "cudaMallocHost");
  check_cuda(cudaMallocHost(&s->h_act, T * s->h * sizeof(__half)), "cudaMallocHost");
  check_cuda(cudaMallocHost(&s->h_slot_rows, s->max_seqs * s->max_blocks * sizeof(int32_t)),
             "cudaMallocHost");
  s->slot_copy_done.resize(s->max_seqs);
  for (auto& e : s->slot_copy_done)
    check_cuda(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
  check_cuda(cudaStreamSynchronize(s->stream), "stage setup");
}

void check_finite_f16(const std::vector<__half>& v, const std::string& name) {
  for (const auto x : v)
    if ((__half_as_ushort(x) & 0x7c00u) == 0x7c00u)
      fail(HLLM_B200_INCOMPATIBLE_WORKER, "weight is not representable as finite F16: " + name);
}

float source_float(hllm_b200_dtype dt, const void* data, size_t i) {
  switch (dt) {
    case HLLM_B200_F32: return static_cast<const float*>(data)[i];
    case HLLM_B200_F16: return __half2float(__ushort_as_half(static_cast<const uint16_t*>(data)[i]));
    default: {
      const uint32_t b = static_cast<uint32_t>(static_cast<const uint16_t*>(data)[i]) << 16;
      float f;
      std::memcpy(&f, &b, 4);
      return f;
    }
  }
}

void load_tensor(hllm_b200_stage* s, const char* name, hllm_b200_dtype dt, const void* data,
                 const uint64_t* shape, uint32_t rank) {
  if (s->finalized) fail(HLLM_B200_INVALID_REQUEST, "stage already finalized");
  if (!name || !data || !shape) fail(HLLM_B200_INVALID_REQUEST, "null tensor argument");
  const auto it = s->targets.find(name);
  if (it == s->targets.end())
    fail(HLLM_B200_INVALID_REQUEST, std::string("tensor is not part of this stage: ") + name);
  const Target& t = it->second;
  const bool ok_shape = t.kind == Target::kNorm ? (rank == 1 && shape[0] == t.rows)
                                                : (rank == 2 && shape[0] == t.rows && shape[1] == t.cols);
  if (!ok_shape) fail(HLLM_B200_INVALID_REQUEST, std::string("tensor shape mismatch: ") + name);
  if (dt != HLLM_B200_F32 && dt != HLLM_B200_F16 && dt != HLLM_B200_BF16)
    fail(HLLM_B200_INCOMPATIBLE_WORKER, "unsupported tensor dtype");
  check_cuda(cudaSetDevice(s->device), "cudaSetDevice");
  if (t.kind == Target::kNorm) {
    std::vector<float> v(t.rows);
    for (size_t i = 0; i < t.rows; ++i) v[i] = source_float(dt, data, i);
    std::vector<__half> hv(t.rows);
    for (size_t i = 0; i < t.rows; ++i) hv[i] = __float2half_rn(v[i]);
    check_finite_f16(hv, name);
    check_cuda(cudaMemcpy(t.norm, v.data(), v.size() * sizeof(float), cudaMemcpyHostToDevice),
               "norm upload");
  } else {
    const size_t n = t.rows * t.cols;
    std::vector<__half> hv(n);
    if (dt == HLLM_B200_F16) std::memcpy(hv.data(), data, n * sizeof(__half));
    else
      for (size_t i = 0; i < n; ++i) hv[i] = __float2half_rn(source_float(dt, data, i));
    check_finite_f16(hv, name);
    check_cuda(cudaMemcpy2D(t.matrix + t.row_offset * t.ld, t.ld * sizeof(__half), hv.data(),
                            t.cols * sizeof(__half), t.cols * sizeof(__half), t.rows,
                            cudaMemcpyHostToDevice),
               "weight upload");
  }
  s->loaded.insert(name);
}

void init_synthetic(hllm_b200_stage* s, uint64_t seed) {
  if (s->finalized) fail(HLLM_B200_INVALID_REQUEST, "stage already finalized");
  check_cuda(cudaSetDevice(s->device), "cudaSetDevice");
  for (const auto& [name, t] : s->targets) {
    if (t.kind == Target::kNorm) {
      check_cuda(hb::synth_norm_launch(seed, t.tag, static_cast<int>(t.rows), kNormSpread, t.norm,
                                       s->stream), "synth");
    } else {
      check_cuda(hb::synth_matrix_launch(seed, t.tag, static_cast<int>(t.rows),
                                         static_cast<int>(t.cols), static_cast<int>(t.ld),
                                         kWeightStd, t.matrix + t.row_offset * t.ld, s->stream),
                 "synth");
    }
    s->loaded.insert(name);
  }
  check_cuda(cudaStreamSynchronize(s->stream), "synthetic init");
}

// ------------------------------------------------------------------ step
struct StepPlan {
  uint32_t rows = 0;
  uint64_t tokens = 0;
  uint32_t samples = 0;
  int split_tokens = 16;
  int total_splits = 0;
  int total_qtiles = 0;
  int qtile_tokens = 0;
  int decode_ctas = 0;     // balanced decode attention grid
  int prefill_splits = 1;  // key splits per prefill tile
  double attn_dec_bytes = 0, attn_dec_flops = 0;  // algorithmic, per layer
  double attn_pre_bytes = 0, attn_pre_flops = 0;
};

void validate_sampling(const hllm_b200_sampling& o) {
  if (!std::isfinite(o.temperature) || o.temperature < 0.0 || o.temperature > 100.0 ||
      !std::isfinite(o.top_p) || o.top_p <= 0.0 || o.top_p > 1.0 || o.top_logprobs > 5U ||
      (!o.return_logprobs && o.top_logprobs != 0U))
    fail(HLLM_B200_INVALID_REQUEST, "invalid sampling parameters");
}

StepPlan plan_step(hllm_b200_stage* s, const hllm_b200_row* rows, uint32_t n, bool device_input) {
  if (!s->finalized) fail(HLLM_B200_INVALID_REQUEST, "stage weights are not finalized");
  if (n == 0 || !rows) fail(HLLM_B200_INVALID_REQUEST, "empty step");
  if (n > s->R_max) fail(HLLM_B200_RESOURCE_EXHAUSTED, "step has more rows than max_step_rows");
  StepPlan p;
  p.rows = n;
  std::set<const hllm_b200_seq*> seen;
  uint64_t decode_keys = 0, decode_pages = 0;
  int decode_rows = 0;
  for (uint32_t i = 0; i < n; ++i) {
    const auto& r = rows[i];
    const hllm_b200_seq* q = r.sequence;
    if (!q || q->owner != s || !s->live.count(const_cast<hllm_b200_seq*>(q)) || q->failed ||
        r.first_position != q->length)
      fail(HLLM_B200_INVALID_REQUEST, "sequence state or position is invalid");
    if (!seen.insert(q).second)
      fail(HLLM_B200_INVALID_REQUEST, "a step requires distinct sequences");
    if (r.tokens == 0 || r.first_position > q->capacity || r.tokens > q->capacity - r.first_position)
      fail(HLLM_B200_INVALID_REQUEST, "invalid stage input or context capacity");
    if (!device_input) {
      if (s->desc.first && !r.token_ids)
        fail(HLLM_B200_INVALID_REQUEST, "stage zero requires tokens");
      if (!s->desc.first && !r.activations)
        fail(HLLM_B200_INVALID_REQUEST, "only stage zero accepts tokens");
      if (s->desc.first)
        for (uint64_t k = 0; k < r.tokens; ++k)
          if (r.token_ids[k] >= s->V) fail(HLLM_B200_INVALID_REQUEST, "token ID exceeds vocabulary");
    }
    if (r.sample && s->desc.final) {
      validate_sampling(r.sampling);
      ++p.samples;
    }
    p.tokens += r.tokens;
    if (r.tokens == 1) {
      decode_keys += r.first_position + 1;
      decode_pages += (r.first_position + 1 + hb::kBlockTokens - 1) / hb::kBlockTokens;
      ++decode_rows;
    }
  }
  if (p.tokens > s->T_max) fail(HLLM_B200_RESOURCE_EXHAUSTED, "step exceeds max_step_tokens");
  // Decode split size: one warp handles one (row, kv head, split); aim for
  // about 16 such items per SM so that rows of very different lengths still
  // balance, with at least 64 keys per split, within the split workspace.
  const uint64_t target = std::max<uint64_t>(1, (16ull * s->sm_count) / s->hkv);
  uint64_t split = std::max<uint64_t>(64, round_up((decode_keys + target - 1) / target, 16));
  auto count_splits = [&](uint64_t sp) {
    uint64_t total = 0;
    for (uint32_t i = 0; i < n; ++i)
      if (rows[i].tokens == 1) total += (rows[i].first_position + 1 + sp - 1) / sp;
    return total;
  };
  while (count_splits(split) > s->max_splits) split *= 2;
  p.split_tokens = static_cast<int>(std::min<uint64_t>(split, 1u << 30));
  p.total_splits = static_cast<int>(count_splits(split));
  p.decode_ctas = hb::attn_decode_ctas(static_cast<int>(s->dim), static_cast<int>(s->hq / s->hkv),
                                       static_cast<long long>(decode_pages * s->hkv), s->sm_count);
  p.qtile_tokens = hb::attn_qtile_tokens(static_cast<int>(s->hq / s->hkv));
  for (uint32_t i = 0; i < n; ++i)
    if (rows[i].tokens > 1)
      p.total_qtiles += static_cast<int>((rows[i].tokens + p.qtile_tokens - 1) / p.qtile_tokens);
  if (p.total_qtiles > s->max_qtiles) fail(HLLM_B200_INTERNAL, "prefill tiles exceed the workspace");
  if (s->tc_prefill) {
    p.prefill_splits = hb::attn_prefill_tc_splits(static_cast<int>(s->hkv), p.total_qtiles,
                                                  s->sm_count);
  } else {
    hb::AttnArgs probe{};
    probe.max_blocks = static_cast<int>(s->max_blocks);
    p.prefill_splits = hb::attn_prefill_splits(static_cast<int>(s->dim), static_cast<int>(s->hkv),
                                               p.total_qtiles, s->sm_count,
                                               hb::prefill_table_bytes(probe));
  }
  // Algorithmic attention work per layer: K and V of every context position
  // read once per kv head, q read and output written once; causal FLOPs
  // 4 * Hq * d per (query, key) pair.
  const double kvb = 2.0 * s->hkv * s->dim * 2.0, qb = 2.0 * s->hq * s->dim * 2.0;
  for (uint32_t i = 0; i < n; ++i) {
    const double ctx = static_cast<double>(rows[i].first_position + rows[i].tokens);
    const double cnt = static_cast<double>(rows[i].tokens);
    const double pairs = cnt * static_cast<double>(rows[i].first_position) + cnt * (cnt + 1) / 2;
    if (rows[i].tokens == 1) {
      p.attn_dec_bytes += ctx * kvb + qb;
      p.attn_dec_flops += 4.0 * s->hq * s->dim * ctx;
    } else {
      p.attn_pre_bytes += ctx * kvb + cnt * qb;
      p.attn_pre_flops += 4.0 * s->hq * s->dim * pairs;
    }
  }
  (void)decode_rows;
  return p;
}

#define LAUNCH(expr)                                    \
  do {                                                  \
    check_cuda((expr), #expr);                          \
    ++s->launches;                                      \
  } while (0)

// Kernel classes of the profile: projection GEMMs at decode width (n <= 128)
// and prefill width, decode attention (split + combine), prefill attention,
// everything else (norms, q/k epilogue, packer, embedding, sampler, boundary).
enum ProfKind { kProfGemmDecode = 0, kProfGemmPrefill = 1, kProfAttnDecode = 2,
                kProfAttnPrefill = 3, kProfOther = 4, kProfNorm = 5, kProfQkv = 6,
                kProfSwiglu = 7, kProfSample = 8 };

#define PLAUNCH(kind, bytes, flops, expr)               \
  do {                                                  \
    s->prof_begin();                                    \
    check_cuda((expr), #expr);                          \
    s->prof_end((kind), (bytes), (flops));              \
    ++s->launches;                                      \
  } while (0)

// Algorithmic traffic and work of one projection GEMM: weights once, tokens
// once, outputs (read + write for the residual add).
double gemm_bytes(double m, double n, double k, int pair, int epilogue) {
  const double out = epilogue == hb::kEpiResidual ? 8.0 : (epilogue == hb::kEpiStoreF32 ? 4.0 : 2.0);
  return pair * m * k * 2.0 + n * k * 2.0 + n * m * out;
}
double gemm_flops(double m, double n, double k, int pair) { return 2.0 * pair * m * n * k; }

void enqueue_step(hllm_b200_stage* s, const hllm_b200_row* rows, const StepPlan& p,
                  const void* device_input) {
  const size_t R = s->R_max;
  const int T = static_cast<int>(p.tokens);
  s->launches = 0;
  s->mark_begin();
  // ---- upload row descriptors (and ids / activations)
  const int ring = s->up_next;
  s->up_next = (s->up_next + 1) % hllm_b200_stage::kUpRing;
  check_cuda(cudaEventSynchronize(s->up_done[ring]), "upload staging");
  s->h_up = s->h_up_ring[ring];
  int32_t* hu = reinterpret_cast<int32_t*>(s->h_up);
  int t = 0;
  uint32_t si = 0;
  auto* hp = reinterpret_cast<hb::SampleParams*>(
      s->h_up + round_up((4 * R + s->T_max) * sizeof(int32_t), 16));
  for (uint32_t i = 0; i < p.rows; ++i) {
    const auto& r = rows[i];
    hu[i] = r.sequence->slot;
    hu[R + i] = static_cast<int32_t>(r.first_position);
    hu[2 * R + i] = static_cast<int32_t>(r.tokens);
    if (r.sample && s->desc.final) {
      hu[3 * R + si] = static_cast<int32_t>(i);
      hp[si] = hb::SampleParams{r.sampling.temperature, r.sampling.top_p, r.sampling.top_k,
                                r.sampling.seed, r.generated_index, r.sampling.return_logprobs,
                                r.sampling.top_logprobs};
      ++si;
    }
    if (!device_input) {
      if (s->desc.first) {
        for (uint64_t k = 0; k < r.tokens; ++k) hu[4 * R + t + k] = static_cast<int32_t>(r.token_ids[k]);
      } else {
        std::memcpy(s->h_act + static_cast<size_t>(t) * s->h, r.activations,
                    r.tokens * s->h * sizeof(__half));
      }
    }
    t += static_cast<int>(r.tokens);
  }
  check_cuda(cudaMemcpyAsync(s->up, s->h_up, s->up_bytes, cudaMemcpyHostToDevice, s->stream),
             "descriptor upload");
  check_cuda(cudaEventRecord(s->up_done[ring], s->stream), "upload staging");
  s->last_h2d = s->up_bytes + ((!s->desc.first && !device_input)
                                   ? static_cast<uint64_t>(T) * s->h * sizeof(__half) : 0);
  s->last_d2h = 0;
  if (s->desc.first && device_input)
    check_cuda(cudaMemcpyAsync(s->ids, device_input, T * sizeof(int32_t),
                               cudaMemcpyDeviceToDevice, s->stream), "id copy");
  if (!s->desc.first)
    check_cuda(cudaMemcpyAsync(s->bin, device_input ? device_input : s->h_act,
                               static_cast<size_t>(T) * s->h * sizeof(__half),
                               device_input ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                               s->stream), "activation upload");

  // ---- pack
  hb::StepTensors st{};
  st.row_slot = s->row_slot;
  st.row_first = s->row_first;
  st.row_count = s->row_count;
  st.cu_seqlens = s->cu_seqlens;
  st.positions = s->positions;
  st.slot_mapping = s->slot_mapping;
  st.token_row = s->token_row;
  st.seq_lens = s->seq_lens;
  st.block_tables = s->block_tables;
  st.cu_splits = s->cu_splits;
  st.cu_qtiles = s->cu_qtiles;
  st.rows = static_cast<int>(p.rows);
  st.tokens = T;
  st.max_blocks = static_cast<int>(s->max_blocks);
  st.split_tokens = p.split_tokens;
  st.qtile_tokens = p.qtile_tokens;
  PLAUNCH(kProfOther, 0, 0, hb::pack_launch(st, s->slot_blocks, s->status, s->stream));

  // ---- input
  if (s->desc.first) {
    PLAUNCH(kProfOther, 0, 0, hb::embed_launch(s->ids, T, s->embed, static_cast<int>(s->V), static_cast<int>(s->h),
                            static_cast<int>(s->h_pad), s->hidden, s->status, s->stream));
  } else {
    PLAUNCH(kProfOther, 0, 0, hb::boundary_in_launch(s->bin, T, static_cast<int>(s->h), s->hidden, s->status,
                                  s->stream));
  }
  s->mark(s->desc.first ? "embedding" : "from-wire");

  // ---- layers
  const float eps = s->desc.rms_norm_epsilon;
  const int h = static_cast<int>(s->h);
  const int gk = T <= 128 ? kProfGemmDecode : kProfGemmPrefill;
  for (size_t li = 0; li < s->n_layers; ++li) {
    const Layer& L = s->layers[li];
    __half* kc = s->kv + li * s->kv_layer_elems;
    __half* vc = kc + s->kv_layer_elems / 2;
    // Layer 0's input norm runs alone; every later one is fused into the
    // previous layer's residual consumer.
    if (li == 0)
      PLAUNCH(kProfNorm, 0, 0, hb::rmsnorm_launch(s->hidden, T, h, L.in_norm, eps, s->xn,
                                                   static_cast<int>(s->h_pad), nullptr, s->stream));
    const hb::GemmPlan pq = hb::gemm_plan(L.g_qkv, T, s->sm_count);
    hb::GemmSlots qslots{};
    PLAUNCH(gk, gemm_bytes(s->qkvw, T, s->h, 1, hb::kEpiStoreF32), gemm_flops(s->qkvw, T, s->h, 1),
            hb::gemm_launch(L.g_qkv, s->in_xn, T, pq, hb::kEpiStoreF32, s->qkv,
                            static_cast<int>(s->qkvw), s->slots, &qslots, s->status, s->stream));
    hb::QkvPostArgs qa{};
    qa.qkv = s->qkv;
    qa.slots = qslots;
    qa.from_slots = pq.stream_k ? 1 : 0;
    qa.tokens = T;
    qa.hq = static_cast<int>(s->hq);
    qa.hkv = static_cast<int>(s->hkv);
    qa.dim = static_cast<int>(s->dim);
    qa.positions = s->positions;
    qa.slot_mapping = s->slot_mapping;
    qa.q_norm = L.q_norm;
    qa.k_norm = L.k_norm;
    qa.eps = eps;
    qa.rope_pow = s->rope_pow;
    qa.rope_table = s->rope_table;
    qa.rope_positions = s->rope_positions;
    qa.q_out = s->q;
    qa.k_cache = kc;
    qa.v_cache = vc;
    PLAUNCH(kProfQkv, 0, 0, hb::qkv_post_launch(qa, s->stream));
    hb::AttnArgs aa{};
    aa.q = s->q;
    aa.k_cache = kc;
    aa.v_cache = vc;
    aa.row_count = s->row_count;
    aa.row_first = s->row_first;
    aa.cu_seqlens = s->cu_seqlens;
    aa.seq_lens = s->seq_lens;
    aa.block_tables = s->block_tables;
    aa.cu_splits = s->cu_splits;
    aa.cu_qtiles = s->cu_qtiles;
    aa.rows = static_cast<int>(p.rows);
    aa.hq = static_cast<int>(s->hq);
    aa.hkv = static_cast<int>(s->hkv);
    aa.dim = static_cast<int>(s->dim);
    aa.max_blocks = static_cast<int>(s->max_blocks);
    aa.split_tokens = p.split_tokens;
    aa.qtile_tokens = p.qtile_tokens;
    aa.decode_ctas = p.decode_ctas;
    aa.prefill_splits = p.prefill_splits;
    aa.pre_part = s->pre_part;
    aa.pre_counters = s->pre_counters;
    aa.scale = 1.0f / std::sqrt(static_cast<float>(s->dim));
    aa.part_o = s->part_o;
    aa.part_ml = s->part_ml;
    aa.counters = s->attn_counters;
    aa.out = s->attn;
    aa.ld_out = static_cast<int>(s->qw_pad);
    aa.status = s->status;
    if (p.total_splits) {
      PLAUNCH(kProfAttnDecode, p.attn_dec_bytes, p.attn_dec_flops,
              hb::attn_decode_launch(aa, s->tc_maps.empty() ? hb::TcMaps{} : s->tc_maps[li],
                                     p.total_splits, s->stream));
      s->launches += hb::attn_decode_launches(static_cast<int>(s->dim)) - 1;  // combine pass
    }
    if (p.total_qtiles)
      PLAUNCH(kProfAttnPrefill, p.attn_pre_bytes, p.attn_pre_flops,
              s->tc_prefill ? hb::attn_prefill_tc_launch(s->tc_maps[li], aa, p.total_qtiles, s->stream)
                            : hb::attn_prefill_launch(aa, p.total_qtiles, s->stream));
    // o_proj, then the fused residual add + post-attention RMSNorm.
    const hb::GemmPlan po = hb::gemm_plan(L.g_o, T, s->sm_count);
    hb::GemmSlots oslots{};
    PLAUNCH(gk, gemm_bytes(s->h, T, s->qw, 1, hb::kEpiResidual), gemm_flops(s->h, T, s->qw, 1),
            hb::gemm_launch(L.g_o, s->in_attn, T, po, hb::kEpiResidual, s->hidden, h, s->slots,
                            &oslots, s->status, s->stream));
    PLAUNCH(kProfNorm, 0, 0,
            hb::residual_norm_launch(s->hidden, T, h, po.stream_k ? &oslots : nullptr,
                                     L.post_norm, eps, s->xn, static_cast<int>(s->h_pad),
                                     s->stream));
    // gate/up with SwiGLU: in the GEMM epilogue, or from the stream-K slots.
    const hb::GemmPlan pg = hb::gemm_plan(L.g_gu, T, s->sm_count);
    hb::GemmSlots gslots{};
    PLAUNCH(gk, gemm_bytes(s->I, T, s->h, 2, hb::kEpiSwiGLU), gemm_flops(s->I, T, s->h, 2),
            hb::gemm_launch(L.g_gu, s->in_xn, T, pg, hb::kEpiSwiGLU, s->act,
                            static_cast<int>(s->I_pad), s->slots, &gslots, s->status, s->stream));
    if (pg.stream_k)
      PLAUNCH(kProfSwiglu, 0, 0,
              hb::swiglu_launch(gslots, T, s->act, static_cast<int>(s->I_pad), s->stream));
    // down_proj, then the residual add fused with the next layer's input norm.
    const hb::GemmPlan pd = hb::gemm_plan(L.g_down, T, s->sm_count);
    hb::GemmSlots dslots{};
    PLAUNCH(gk, gemm_bytes(s->h, T, s->I, 1, hb::kEpiResidual), gemm_flops(s->h, T, s->I, 1),
            hb::gemm_launch(L.g_down, s->in_act, T, pd, hb::kEpiResidual, s->hidden, h, s->slots,
                            &dslots, s->status, s->stream));
    const float* next_norm = li + 1 < s->n_layers ? s->layers[li + 1].in_norm : nullptr;
    if (pd.stream_k || next_norm)
      PLAUNCH(kProfNorm, 0, 0,
              hb::residual_norm_launch(s->hidden, T, h, pd.stream_k ? &dslots : nullptr,
                                       next_norm, eps, s->xn, static_cast<int>(s->h_pad),
                                       s->stream));
    s->mark("layer", static_cast<int64_t>(s->desc.layer_start + li));
  }

  // ---- output
  if (s->desc.final) {
    if (p.samples) {
      const int S = static_cast<int>(p.samples);
      PLAUNCH(kProfOther, 0, 0, hb::last_token_launch(s->cu_seqlens, s->sample_rows, S, s->last_idx, s->stream));
      PLAUNCH(kProfNorm, 0, 0, hb::rmsnorm_launch(s->hidden, S, h, s->final_norm, eps, s->xs,
                                static_cast<int>(s->h_pad), s->last_idx, s->stream));
      s->mark("final_norm");
      const hb::GemmPlan ph = hb::gemm_plan(s->g_head, S, s->sm_count);
      hb::GemmSlots hslots{};
      PLAUNCH(S <= 128 ? kProfGemmDecode : kProfGemmPrefill,
              gemm_bytes(s->V, S, s->h, 1, hb::kEpiStoreF32), gemm_flops(s->V, S, s->h, 1),
              hb::gemm_launch(s->g_head, s->in_xs, S, ph, hb::kEpiStoreF32, s->logits,
                              static_cast<int>(s->V), s->slots, &hslots, s->status, s->stream));
      if (ph.stream_k)
        PLAUNCH(kProfSwiglu, 0, 0,
                hb::gemm_finish_launch(hslots, S, hb::kEpiStoreF32, s->logits,
                                       static_cast<int>(s->V), s->stream));
      s->mark("lm_head");
      PLAUNCH(kProfSample, 0, 0, hb::sample_launch(s->logits, S, static_cast<int>(s->V), static_cast<int>(s->V),
                               s->d_params, s->sample_scratch, s->results, s->status, s->stream));
    }
  } else {
    if (s->env_pending)  // an envelope copy may still be reading the boundary buffer
      check_cuda(cudaStreamWaitEvent(s->stream, s->env_done, 0), "envelope order");
    PLAUNCH(kProfOther, 0, 0, hb::boundary_out_launch(s->hidden, T, h, s->bout, s->status, s->stream));
  }
  s->last_samples = p.samples;
  s->last_tokens = p.tokens;
}

// Prefill attention returns its arrival counters to zero when it finishes; a
// kernel that ended early on a failed wait may leave one behind, so a failed
// step clears them (and the decode streams' warp-range records).
void reset_counters(hllm_b200_stage* s) {
  check_cuda(cudaMemsetAsync(s->attn_counters, 0, s->attn_counter_ints * sizeof(int), s->stream),
             "counter reset");
  check_cuda(cudaMemsetAsync(s->pre_counters, 0, s->pre_counter_ints * sizeof(int), s->stream),
             "counter reset");
}

hllm_b200_status status_to_code(uint32_t bits, std::string* msg) {
  if (bits == 0) return HLLM_B200_OK;
  if (bits & kInputNonFinite) {
    *msg = "non-finite activation";
    return HLLM_B200_INVALID_REQUEST;
  }
  if (bits & hb::kDevWaitTimeout) *msg = "a device wait ran past its time limit";
  else if (bits & hb::kDevBadIndex) *msg = "a device index was out of range";
  else if (bits & hb::kDevNonFinite) *msg = "non-finite CUDA tensor";
  else *msg = "device error";
  return HLLM_B200_INTERNAL;
}

void mark_failed(const hllm_b200_row* rows, uint32_t n) {
  for (uint32_t i = 0; i < n; ++i)
    if (rows[i].sequence) rows[i].sequence->failed = true;
}

void copy_sampled(const hb::SampleResult& r, hllm_b200_sampled* o) {
  o->token_id = static_cast<uint64_t>(r.token);
  o->has_logprob = 0;
  o->logprob = 0;
  o->n_top = 0;
  o->has_logprob = 0;
  for (int k = 0; k < 5; ++k) {
    o->top_ids[k] = static_cast<uint64_t>(r.top_ids[k]);
    o->top_logprobs[k] = r.top_logprobs[k];
  }
  o->logprob = r.logprob;
  o->n_top = static_cast<uint32_t>(r.n_top);
}

}  // namespace

// =================================================================== C ABI
extern "C" {

size_t hllm_b200_last_error(char* buffer, size_t size) {
  if (buffer && size) {
    const size_t n = std::min(size - 1, g_last_error.size());
    std::memcpy(buffer, g_last_error.data(), n);
    buffer[n] = 0;
  }
  return g_last_error.size();
}

hllm_b200_status hllm_b200_stage_create(const hllm_b200_stage_desc* desc, hllm_b200_stage** out) {
  return guarded([&] {
    if (!desc || !out) fail(HLLM_B200_INVALID_REQUEST, "null argument");
    *out = nullptr;
    auto s = std::make_unique<hllm_b200_stage>();
    build_stage(s.get(), *desc);
    *out = s.release();
  });
}

void hllm_b200_stage_destroy(hllm_b200_stage* stage) {
  if (!stage) return;
  cudaSetDevice(stage->device);
  delete stage;
}

hllm_b200_status hllm_b200_stage_load_tensor(hllm_b200_stage* stage, const char* name,
                                             hllm_b200_dtype dtype, const void* data,
                                             const uint64_t* shape, uint32_t rank) {
  return guarded([&] {
    if (!stage) fail(HLLM_B200_INVALID_REQUEST, "null stage");
    std::scoped_lock lock(stage->mutex);
    load_tensor(stage, name, dtype, data, shape, rank);
  });
}

hllm_b200_status hllm_b200_stage_init_synthetic(hllm_b200_stage* stage, uint64_t seed) {
  return guarded([&] {
    if (!stage) fail(HLLM_B200_INVALID_REQUEST, "null stage");
    std::scoped_lock lock(stage->mutex);
    init_synthetic(stage, seed);
  });
}

hllm_b200_status hllm_b200_stage_finalize(hllm_b200_stage* stage) {
  return guarded([&] {
    if (!stage) fail(HLLM_B200_INVALID_REQUEST, "null stage");
    std::scoped_lock lock(stage->mutex);
    for (const auto& [name, t] : stage->targets)
      if (!stage->loaded.count(name))
        fail(HLLM_B200_INVALID_REQUEST, "missing tensor for stage: " + name);
    check_cuda(cudaSetDevice(stage->device), "cudaSetDevice");
    check_cuda(cudaDeviceSynchronize(), "finalize");
    stage->finalized = true;
  });
}

hllm_b200_status hllm_b200_stage_info(const hllm_b200_stage* stage, uint64_t* weight_device_bytes,
                                      uint64_t* hidden_size, uint64_t* vocabulary_size,
                                      uint64_t* maximum_tokens) {
  return guarded([&] {
    if (!stage) fail(HLLM_B200_INVALID_REQUEST, "null stage");
    if (weight_device_bytes) *weight_device_bytes = stage->weight_bytes;
    if (hidden_size) *hidden_size = stage->h;
    if (vocabulary_size) *vocabulary_size = stage->V;
    if (maximum_tokens) *maximum_tokens = stage->desc.maximum_sequence_length;
  });
}

hllm_b200_status hllm_b200_stage_memory(hllm_b200_stage* stage, uint64_t* weights,
                                        uint64_t* workspace, uint64_t* kv_pool,
                                        uint64_t* kv_in_use, uint64_t* kv_peak) {
  return guarded([&] {
    if (!stage) fail(HLLM_B200_INVALID_REQUEST, "null stage");
    std::scoped_lock lock(stage->mutex);
    const uint64_t block = static_cast<uint64_t>(std::max<size_t>(1, stage->n_layers)) * 2 *
                           stage->hkv * hb::kBlockTokens * stage->dim * sizeof(__half);
    const uint64_t used = stage->num_blocks - stage->free_blocks.size();
    if (weights) *weights = stage->weight_bytes;
    if (workspace) *workspace = stage->workspace_bytes - stage->num_blocks * block;
    if (kv_pool) *kv_pool = stage->num_blocks * block;
    if (kv_in_use) *kv_in_use = used * block;
    if (kv_peak) *kv_peak = stage->kv_peak_blocks * block;
  });
}

hllm_b200_status hllm_b200_sequence_memory(const hllm_b200_stage* stage, uint64_t tokens,
                                           uint64_t maximum_query_tokens,
                                           uint64_t* cache_device_bytes,
                                           uint64_t* workspace_device_bytes) {
  return guarded([&] {
    if (!stage) fail(HLLM_B200_INVALID_REQUEST, "null stage");
    if (tokens == 0 || tokens > stage->desc.maximum_sequence_length)
      fail(HLLM_B200_INVALID_REQUEST, "request exceeds model context capacity");
    const uint64_t rows = (maximum_query_tokens == 0 || maximum_query_tokens > tokens)
                              ? tokens : maximum_query_tokens;
    if (rows > stage->T_max)
      fail(HLLM_B200_RESOURCE_EXHAUSTED, "prefill rows exceed max_step_tokens");
    const uint64_t blocks = (tokens + hb::kBlockTokens - 1) / hb::kBlockTokens;
    if (cache_device_bytes)
      *cache_device_bytes = blocks * hb::kBlockTokens * stage->n_layers * stage->hkv *
                            stage->dim * 2 * sizeof(__half);
    if (workspace_device_bytes) *workspace_device_bytes = stage->workspace_bytes;
  });
}

hllm_b200_status hllm_b200_seq_alloc(hllm_b200_stage* stage, uint64_t tokens, hllm_b200_seq** out) {
  return guarded([&] {
    if (!stage || !out) fail(HLLM_B200_INVALID_REQUEST, "null argument");
    std::scoped_lock lock(stage->mutex);
    *out = nullptr;
    if (tokens == 0 || tokens > stage->desc.maximum_sequence_length)
      fail(HLLM_B200_INVALID_REQUEST, "request exceeds model context capacity");
    const size_t need = (tokens + hb::kBlockTokens - 1) / hb::kBlockTokens;
    if (stage->free_slots.empty()) fail(HLLM_B200_RESOURCE_EXHAUSTED, "no free sequence slot");
    if (stage->free_blocks.size() < need)
      fail(HLLM_B200_RESOURCE_EXHAUSTED, "paged KV pool exhausted");
    auto seq = std::make_unique<hllm_b200_seq>();
    seq->owner = stage;
    seq->capacity = tokens;
    seq->slot = stage->free_slots.back();
    seq->blocks.assign(stage->free_blocks.end() - static_cast<std::ptrdiff_t>(need),
                       stage->free_blocks.end());
    std::reverse(seq->blocks.begin(), seq->blocks.end());
    // The block list goes through the slot's own pinned staging row, copied in
    // stream order ahead of any step that uses the sequence; the slot's event
    // guards the staging row against reuse before its previous copy ran.
    check_cuda(cudaSetDevice(stage->device), "cudaSetDevice");
    cudaEvent_t done = stage->slot_copy_done[seq->slot];
    check_cuda(cudaEventSynchronize(done), "slot staging");
    int32_t* row = stage->h_slot_rows + static_cast<size_t>(seq->slot) * stage->max_blocks;
    std::fill(row, row + stage->max_blocks, -1);
    std::copy(seq->blocks.begin(), seq->blocks.end(), row);
    check_cuda(cudaMemcpyAsync(stage->slot_blocks + static_cast<size_t>(seq->slot) * stage->max_blocks,
                               row, stage->max_blocks * sizeof(int32_t), cudaMemcpyHostToDevice,
                               stage->stream),
               "block table upload");
    check_cuda(cudaEventRecord(done, stage->stream), "slot staging");
    stage->free_slots.pop_back();
    stage->free_blocks.resize(stage->free_blocks.size() - need);
    stage->kv_peak_blocks = std::max(stage->kv_peak_blocks,
                                     stage->num_blocks - stage->free_blocks.size());
    stage->live.insert(seq.get());
    *out = seq.release();
  });
}

void hllm_b200_seq_free(hllm_b200_stage* stage, hllm_b200_seq* seq) {
  if (!stage || !seq || seq->owner != stage) return;
  std::scoped_lock lock(stage->mutex);
  if (!stage->live.erase(seq)) return;
  for (auto it = seq->blocks.rbegin(); it != seq->blocks.rend(); ++it)
    stage->free_blocks.push_back(*it);
  stage->free_slots.push_back(seq->slot);
  delete seq;
}

hllm_b200_status hllm_b200_seq_info(const hllm_b200_seq* seq, uint64_t* length, uint64_t* capacity,
                                    uint32_t* failed) {
  return guarded([&] {
    if (!seq) fail(HLLM_B200_INVALID_REQUEST, "null sequence");
    if (length) *length = seq->length;
    if (capacity) *capacity = seq->capacity;
    if (failed) *failed = seq->failed ? 1u : 0u;
  });
}

hllm_b200_status hllm_b200_step(hllm_b200_stage* stage, const hllm_b200_row* rows, uint32_t n_rows,
                                hllm_b200_sampled* sampled, uint16_t* boundary) {
  bool enqueued = false;
  const hllm_b200_status st = guarded([&] {
    if (!stage) fail(HLLM_B200_INVALID_REQUEST, "null stage");
    std::scoped_lock lock(stage->mutex);
    check_cuda(cudaSetDevice(stage->device), "cudaSetDevice");
    const StepPlan p = plan_step(stage, rows, n_rows, false);
    if (stage->desc.final && p.samples && !sampled)
      fail(HLLM_B200_INVALID_REQUEST, "sampled output buffer required");
    if (!stage->desc.final && !boundary)
      fail(HLLM_B200_INVALID_REQUEST, "boundary output buffer required");
    check_cuda(cudaMemsetAsync(stage->status, 0, sizeof(uint32_t), stage->stream), "status reset");
    enqueued = true;
    enqueue_step(stage, rows, p, nullptr);
    const size_t down_bytes = 8 + p.samples * sizeof(hb::SampleResult);
    stage->last_d2h = down_bytes + (stage->desc.final ? 0 : p.tokens * stage->h * sizeof(__half));
    check_cuda(cudaMemcpyAsync(stage->h_down, stage->down, down_bytes, cudaMemcpyDeviceToHost,
                               stage->stream), "result download");
    if (!stage->desc.final)
      check_cuda(cudaMemcpyAsync(stage->h_act, stage->bout, p.tokens * stage->h * sizeof(__half),
                                 cudaMemcpyDeviceToHost, stage->stream), "boundary download");
    if (!stage->desc.final)
      stage->mark("to-wire");
    else if (p.samples)
      stage->mark("sampling");
    check_cuda(cudaStreamSynchronize(stage->stream), "step");
    stage->prof_collect();
    uint32_t bits;
    std::memcpy(&bits, stage->h_down, sizeof(bits));
    std::string msg;
    const hllm_b200_status code = status_to_code(bits, &msg);
    if (code != HLLM_B200_OK) {
      reset_counters(stage);
      fail(code, msg);
    }
    if (stage->desc.final) {
      const auto* res = reinterpret_cast<const hb::SampleResult*>(stage->h_down + 8);
      for (uint32_t i = 0; i < p.samples; ++i) copy_sampled(res[i], &sampled[i]);
    } else {
      std::memcpy(boundary, stage->h_act, p.tokens * stage->h * sizeof(__half));
    }
    for (uint32_t i = 0; i < n_rows; ++i) rows[i].sequence->length += rows[i].tokens;
  });
  if (st != HLLM_B200_OK && enqueued) mark_failed(rows, n_rows);
  return st;
}

hllm_b200_status hllm_b200_step_async(hllm_b200_stage* stage, const hllm_b200_row* rows,
                                      uint32_t n_rows, const void* device_input) {
  bool enqueued = false;
  const hllm_b200_status st = guarded([&] {
    if (!stage || !device_input) fail(HLLM_B200_INVALID_REQUEST, "null argument");
    std::scoped_lock lock(stage->mutex);
    check_cuda(cudaSetDevice(stage->device), "cudaSetDevice");
    const StepPlan p = plan_step(stage, rows, n_rows, true);
    enqueued = true;
    enqueue_step(stage, rows, p, device_input);
    for (uint32_t i = 0; i < n_rows; ++i) {
      rows[i].sequence->length += rows[i].tokens;
      stage->pending.push_back(rows[i].sequence);
    }
  });
  if (st != HLLM_B200_OK && enqueued) mark_failed(rows, n_rows);
  return st;
}

hllm_b200_status hllm_b200_stage_sync(hllm_b200_stage* stage) {
  return guarded([&] {
    if (!stage) fail(HLLM_B200_INVALID_REQUEST, "null stage");
    std::scoped_lock lock(stage->mutex);
    check_cuda(cudaSetDevice(stage->device), "cudaSetDevice");
    uint32_t bits = 0;
    check_cuda(cudaMemcpyAsync(&bits, stage->status, sizeof(bits), cudaMemcpyDeviceToHost,
                               stage->stream), "status download");
    check_cuda(cudaStreamSynchronize(stage->stream), "sync");
    stage->prof_collect();
    check_cuda(cudaMemsetAsync(stage->status, 0, sizeof(uint32_t), stage->stream), "status reset");
    std::string msg;
    const hllm_b200_status code = status_to_code(bits, &msg);
    if (code != HLLM_B200_OK) {
      reset_counters(stage);
      for (auto* q : stage->pending)
        if (stage->live.count(q)) q->failed = true;
      stage->pending.clear();
      fail(code, msg);
    }
    stage->pending.clear();
  });
}

hllm_b200_status hllm_b200_stage_results(hllm_b200_stage* stage, hllm_b200_sampled* sampled,
                                         uint32_t count) {
  return guarded([&] {
    if (!stage || (count && !sampled)) fail(HLLM_B200_INVALID_REQUEST, "null argument");
    std::scoped_lock lock(stage->mutex);
    if (count > stage->last_samples) fail(HLLM_B200_INVALID_REQUEST, "more results than samples");
    std::vector<hb::SampleResult> res(count);
    check_cuda(cudaMemcpyAsync(res.data(), stage->results, count * sizeof(hb::SampleResult),
                               cudaMemcpyDeviceToHost, stage->stream), "results");
    check_cuda(cudaStreamSynchronize(stage->stream), "results");
    for (uint32_t i = 0; i < count; ++i) copy_sampled(res[i], &sampled[i]);
  });
}

hllm_b200_status hllm_b200_stage_profile(hllm_b200_stage* stage, uint32_t enable) {
  return guarded([&] {
    if (!stage) fail(HLLM_B200_INVALID_REQUEST, "null stage");
    std::scoped_lock lock(stage->mutex);
    check_cuda(cudaSetDevice(stage->device), "cudaSetDevice");
    check_cuda(cudaStreamSynchronize(stage->stream), "profile");
    stage->prof_collect();
    for (int k = 0; k < hllm_b200_stage::kProfKinds; ++k) {
      stage->prof_ms[k] = stage->prof_bytes[k] = stage->prof_flops[k] = 0;
      stage->prof_n[k] = 0;
    }
    stage->profiling = enable != 0;
  });
}

hllm_b200_status hllm_b200_stage_profile_read(hllm_b200_stage* stage, uint32_t kind, double* ms,
                                              uint64_t* launches, double* bytes, double* flops) {
  return guarded([&] {
    if (!stage || kind >= static_cast<uint32_t>(hllm_b200_stage::kProfKinds))
      fail(HLLM_B200_INVALID_REQUEST, "bad argument");
    std::scoped_lock lock(stage->mutex);
    check_cuda(cudaSetDevice(stage->device), "cudaSetDevice");
    check_cuda(cudaStreamSynchronize(stage->stream), "profile");
    stage->prof_collect();
    if (ms) *ms = stage->prof_ms[kind];
    if (launches) *launches = stage->prof_n[kind];
    if (bytes) *bytes = stage->prof_bytes[kind];
    if (flops) *flops = stage->prof_flops[kind];
  });
}

void* hllm_b200_stage_stream(hllm_b200_stage* stage) { return stage ? stage->stream : nullptr; }
int32_t hllm_b200_stage_device(const hllm_b200_stage* stage) { return stage ? stage->device : -1; }
uint32_t hllm_b200_stage_last_launches(const hllm_b200_stage* stage) {
  return stage ? stage->launches : 0;
}

const void* hllm_b200_stage_boundary(const hllm_b200_stage* stage) {
  return stage && !stage->desc.final ? static_cast<const void*>(stage->bout) : nullptr;
}

hllm_b200_status hllm_b200_stage_component_timing(hllm_b200_stage* stage, uint32_t enable) {
  return guarded([&] {
    if (!stage) fail(HLLM_B200_INVALID_REQUEST, "null stage");
    std::scoped_lock lock(stage->mutex);
    check_cuda(cudaSetDevice(stage->device), "cudaSetDevice");
    stage->comp_timing = enable != 0;
    stage->marks.clear();
  });
}

hllm_b200_status hllm_b200_stage_components(hllm_b200_stage* stage,
                                            hllm_b200_component_timing* out, uint32_t capacity,
                                            uint32_t* count) {
  return guarded([&] {
    if (!stage || !count || (capacity && !out)) fail(HLLM_B200_INVALID_REQUEST, "null argument");
    std::scoped_lock lock(stage->mutex);
    check_cuda(cudaSetDevice(stage->device), "cudaSetDevice");
    *count = static_cast<uint32_t>(stage->marks.size());
    if (stage->marks.empty()) return;
    check_cuda(cudaEventSynchronize(stage->marks.back().ev), "component timing");
    cudaEvent_t prev = stage->mark_start;
    for (size_t i = 0; i < stage->marks.size(); ++i) {
      const auto& m = stage->marks[i];
      float ms = 0.f;
      check_cuda(cudaEventElapsedTime(&ms, prev, m.ev), "component timing");
      prev = m.ev;
      if (i >= capacity) continue;
      hllm_b200_component_timing& o = out[i];
      std::memset(&o, 0, sizeof(o));
      std::strncpy(o.component, m.name, sizeof(o.component) - 1);
      o.layer_index = m.layer;
      o.milliseconds = ms;
    }
  });
}

namespace {
hb::EnvelopeIdentity envelope_identity(const hllm_b200_boundary_identity& c) {
  if (!c.deployment_id || !c.request_id) fail(HLLM_B200_INVALID_REQUEST, "null argument");
  hb::EnvelopeIdentity id;
  id.deployment_id = c.deployment_id;
  id.deployment_version = c.deployment_version;
  id.request_id = c.request_id;
  id.maximum_tokens = c.maximum_tokens;
  id.hidden_size = c.hidden_size;
  return id;
}

void envelope_streams(hllm_b200_stage* s) {
  if (s->copy_stream) return;
  check_cuda(cudaStreamCreateWithFlags(&s->copy_stream, cudaStreamNonBlocking), "cudaStreamCreate");
  check_cuda(cudaEventCreateWithFlags(&s->step_done, cudaEventDisableTiming), "cudaEventCreate");
  check_cuda(cudaEventCreateWithFlags(&s->env_done, cudaEventDisableTiming), "cudaEventCreate");
}

// Waits for the envelope copies in flight, places staged payloads into their
// messages, and applies encode_tensor's finite check to every payload
// (cpp/src/worker/boundary_codec.cpp:96-100).  Caller holds the mutex.
void envelope_finish(hllm_b200_stage* s) {
  if (!s->env_pending) return;
  check_cuda(cudaSetDevice(s->device), "cudaSetDevice");
  check_cuda(cudaEventSynchronize(s->env_done), "envelope copy");
  std::vector<std::pair<const uint8_t*, uint64_t>> payloads;
  payloads.swap(s->env_payloads);
  std::vector<hllm_b200_stage::EnvPlace> places;
  places.swap(s->env_places);
  s->env_pending = false;
  for (const auto& pl : places) {
    std::memcpy(pl.dst, s->h_env + pl.src, pl.bytes);
    payloads.emplace_back(pl.dst, pl.bytes);
  }
  for (const auto& [p, n] : payloads)
    if (!hb::f16_payload_finite(p, n))
      fail(HLLM_B200_INTERNAL, "backend returned a non-finite boundary activation");
}
}  // namespace

hllm_b200_status hllm_b200_stage_envelopes(hllm_b200_stage* stage,
                                           const hllm_b200_envelope_row* rows, uint32_t n,
                                           uint8_t* out, uint64_t capacity, uint64_t* offsets) {
  return guarded([&] {
    if (!stage || !rows || !n || !offsets) fail(HLLM_B200_INVALID_REQUEST, "null argument");
    std::scoped_lock lock(stage->mutex);
    if (stage->desc.final) fail(HLLM_B200_INVALID_REQUEST, "a final stage has no boundary output");
    const size_t row_bytes = stage->h * sizeof(__half);
    std::vector<hb::EnvelopeLayout> layouts(n);
    uint64_t total = 0, lo = UINT64_MAX, hi = 0;
    for (uint32_t i = 0; i < n; ++i) {
      const auto& r = rows[i];
      if (r.tokens == 0 || r.first_token > stage->last_tokens ||
          r.tokens > stage->last_tokens - r.first_token)
        fail(HLLM_B200_INVALID_REQUEST, "rows outside the last step's boundary");
      std::string why;
      const hllm_b200_status st =
          hb::envelope_plan(envelope_identity(r.identity), r.sequence, r.position, r.prefill != 0,
                            r.tokens * row_bytes, r.tokens, stage->h, &layouts[i], &why);
      if (st != HLLM_B200_OK) fail(st, why);
      offsets[i] = total;
      total += layouts[i].total;
      lo = std::min<uint64_t>(lo, r.first_token);
      hi = std::max<uint64_t>(hi, r.first_token + r.tokens);
    }
    offsets[n] = total;
    if (!out) return;  // size query
    if (capacity < total) fail(HLLM_B200_INVALID_REQUEST, "output buffer too small");
    // The staging holds one batch: finish the previous one first.
    envelope_finish(stage);
    check_cuda(cudaSetDevice(stage->device), "cudaSetDevice");
    envelope_streams(stage);
    if (!stage->h_env)
      check_cuda(cudaMallocHost(&stage->h_env, stage->T_max * row_bytes), "cudaMallocHost");
    for (uint32_t i = 0; i < n; ++i) {
      const auto& r = rows[i];
      hb::envelope_write_frame(envelope_identity(r.identity), r.sequence, r.position,
                               r.prefill != 0, r.tokens, stage->h, out + offsets[i]);
    }
    check_cuda(cudaEventRecord(stage->step_done, stage->stream), "envelope order");
    check_cuda(cudaStreamWaitEvent(stage->copy_stream, stage->step_done, 0), "envelope order");
    check_cuda(cudaMemcpyAsync(stage->h_env + lo * row_bytes, stage->bout + lo * stage->h,
                               (hi - lo) * row_bytes, cudaMemcpyDeviceToHost, stage->copy_stream),
               "envelope copy");
    check_cuda(cudaEventRecord(stage->env_done, stage->copy_stream), "envelope order");
    stage->env_pending = true;
    for (uint32_t i = 0; i < n; ++i)
      stage->env_places.push_back({out + offsets[i] + layouts[i].payload_offset,
                                   rows[i].first_token * row_bytes, rows[i].tokens * row_bytes});
  });
}

hllm_b200_status hllm_b200_stage_envelope(hllm_b200_stage* stage, uint64_t first_token,
                                          uint64_t tokens,
                                          const hllm_b200_boundary_identity* identity,
                                          uint64_t sequence, uint64_t position, uint32_t prefill,
                                          uint8_t* out, uint64_t capacity, uint64_t* written) {
  return guarded([&] {
    if (!stage || !identity || !written) fail(HLLM_B200_INVALID_REQUEST, "null argument");
    std::scoped_lock lock(stage->mutex);
    if (stage->desc.final) fail(HLLM_B200_INVALID_REQUEST, "a final stage has no boundary output");
    if (tokens == 0 || first_token > stage->last_tokens || tokens > stage->last_tokens - first_token)
      fail(HLLM_B200_INVALID_REQUEST, "rows outside the last step's boundary");
    const hb::EnvelopeIdentity id = envelope_identity(*identity);
    const uint64_t bytes = tokens * stage->h * sizeof(__half);
    hb::EnvelopeLayout layout;
    std::string why;
    const hllm_b200_status st = hb::envelope_plan(id, sequence, position, prefill != 0, bytes,
                                                  tokens, stage->h, &layout, &why);
    if (st != HLLM_B200_OK) fail(st, why);
    *written = layout.total;
    if (!out) return;  // size query
    if (capacity < layout.total) fail(HLLM_B200_INVALID_REQUEST, "output buffer too small");
    check_cuda(cudaSetDevice(stage->device), "cudaSetDevice");
    envelope_streams(stage);
    hb::envelope_write_frame(id, sequence, position, prefill != 0, tokens, stage->h, out);
    check_cuda(cudaEventRecord(stage->step_done, stage->stream), "envelope order");
    check_cuda(cudaStreamWaitEvent(stage->copy_stream, stage->step_done, 0), "envelope order");
    check_cuda(cudaMemcpyAsync(out + layout.payload_offset, stage->bout + first_token * stage->h,
                               bytes, cudaMemcpyDeviceToHost, stage->copy_stream),
               "envelope copy");
    check_cuda(cudaEventRecord(stage->env_done, stage->copy_stream), "envelope order");
    stage->env_pending = true;
    stage->env_payloads.emplace_back(out + layout.payload_offset, bytes);
  });
}

hllm_b200_status hllm_b200_stage_envelope_wait(hllm_b200_stage* stage) {
  return guarded([&] {
    if (!stage) fail(HLLM_B200_INVALID_REQUEST, "null stage");
    std::scoped_lock lock(stage->mutex);
    envelope_finish(stage);
  });
}

hllm_b200_status hllm_b200_stage_last_transfer(const hllm_b200_stage* stage, uint64_t* h2d_bytes,
                                               uint64_t* d2h_bytes) {
  return guarded([&] {
    if (!stage) fail(HLLM_B200_INVALID_REQUEST, "null stage");
    if (h2d_bytes) *h2d_bytes = stage->last_h2d;
    if (d2h_bytes) *d2h_bytes = stage->last_d2h;
  });
}

hllm_b200_status hllm_b200_seq_read_kv(hllm_b200_stage* stage, const hllm_b200_seq* seq,
                                       uint64_t layer, uint32_t values, uint16_t* out) {
  return guarded([&] {
    if (!stage || !seq || !out || seq->owner != stage) fail(HLLM_B200_INVALID_REQUEST, "bad argument");
    if (layer < stage->desc.layer_start || layer >= stage->desc.layer_end)
      fail(HLLM_B200_INVALID_REQUEST, "layer not owned by this stage");
    std::scoped_lock lock(stage->mutex);
    check_cuda(cudaSetDevice(stage->device), "cudaSetDevice");
    const size_t li = layer - stage->desc.layer_start;
    const __half* base = stage->kv + li * stage->kv_layer_elems + (values ? stage->kv_layer_elems / 2 : 0);
    const size_t d = stage->dim, hkv = stage->hkv;
    for (uint64_t pos = 0; pos < seq->length; ++pos) {
      const int32_t blk = seq->blocks[pos / hb::kBlockTokens];
      for (size_t hh = 0; hh < hkv; ++hh) {
        const __half* src = base + ((static_cast<size_t>(blk) * hkv + hh) * hb::kBlockTokens +
                                    pos % hb::kBlockTokens) * d;
        check_cuda(cudaMemcpyAsync(out + (pos * hkv + hh) * d, src, d * sizeof(__half),
                                   cudaMemcpyDeviceToHost, stage->stream), "kv read");
      }
    }
    check_cuda(cudaStreamSynchronize(stage->stream), "kv read");
  });
}

hllm_b200_status hllm_b200_stage_read_hidden(hllm_b200_stage* stage, float* out, uint64_t tokens) {
  return guarded([&] {
    if (!stage || !out || tokens > stage->T_max) fail(HLLM_B200_INVALID_REQUEST, "bad argument");
    std::scoped_lock lock(stage->mutex);
    check_cuda(cudaSetDevice(stage->device), "cudaSetDevice");
    check_cuda(cudaMemcpyAsync(out, stage->hidden, tokens * stage->h * sizeof(float),
                               cudaMemcpyDeviceToHost, stage->stream), "hidden read");
    check_cuda(cudaStreamSynchronize(stage->stream), "hidden read");
  });
}

hllm_b200_status hllm_b200_stage_read_logits(hllm_b200_stage* stage, float* out, uint64_t rows) {
  return guarded([&] {
    if (!stage || !out || !stage->logits || rows > stage->R_max)
      fail(HLLM_B200_INVALID_REQUEST, "bad argument");
    std::scoped_lock lock(stage->mutex);
    check_cuda(cudaSetDevice(stage->device), "cudaSetDevice");
    check_cuda(cudaMemcpyAsync(out, stage->logits, rows * stage->V * sizeof(float),
                               cudaMemcpyDeviceToHost, stage->stream), "logits read");
    check_cuda(cudaStreamSynchronize(stage->stream), "logits read");
  });
}

}  // extern "C"
