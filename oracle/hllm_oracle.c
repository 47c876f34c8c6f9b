/*
 * hllm_oracle.c -- CPU restatement of hLLM's F32 reference math.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the B200
 * stage executor: it is built into oracle/liboracle.so and may be loaded only
 * by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg.  The
 * product library (hllm_b200/libhllm_b200.so) never links or calls it.
 *
 * Every function restates one function of the reference C++ CPU backend,
 * keeping its order of floating-point operations so that results agree with
 * the reference bit for bit (checked against oracle/_ref, which is the
 * reference's own code compiled from its sources):
 *
 *   oracle_f16_to_f32 / oracle_f32_to_f16   cpp/src/half.cpp:8-88
 *   oracle_rms_norm                         cpp/src/cpu/llama.cpp:193-212
 *   oracle_normalize_heads                  cpp/src/cpu/llama.cpp:114-130
 *   oracle_apply_rope                       cpp/src/cpu/llama.cpp:214-240
 *   oracle_attention                        cpp/src/cpu/llama.cpp:67-112
 *   oracle_linear                           cpp/src/cpu/tensor.cpp:47-62
 *   oracle_transformer_layer                cpp/src/cpu/llama.cpp:242-282
 *   oracle_final_logits                     cpp/src/cpu/llama.cpp:284-288
 *   oracle_greedy_sample_last               cpp/src/cpu/llama.cpp:290-308
 *   oracle_sample_logits / _sample_token    cpp/src/sampling.cpp:10-90
 *
 * Two more functions have no reference counterpart and state this build's
 * own contracts: oracle_pack (the ragged batch packer: cu_seqlens, positions,
 * slot mapping and block tables for paged KV) and oracle_synth_* (the seeded
 * synthetic weight generator that the device initialiser reproduces exactly).
 *
 * Threading: loops are split across OpenMP threads only over independent
 * output elements; each element is computed in the reference's order, so the
 * thread count never changes a result.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define ORACLE_OK 0
#define ORACLE_INVALID 1
#define ORACLE_INTERNAL 6

/* ----------------------------------------------------------------------- */
/* half.cpp:8-88 -- F16 <-> F32, round to nearest even                      */
/* ----------------------------------------------------------------------- */
static uint32_t f_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float f_from(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

float oracle_f16_to_f32(uint16_t value) {
  uint32_t sign = (uint32_t)(value & 0x8000u) << 16;
  uint32_t exponent = (value >> 10) & 0x1fu;
  uint32_t mantissa = value & 0x03ffu;
  uint32_t bits;
  if (exponent == 0u) {
    if (mantissa == 0u) {
      bits = sign;
    } else {
      int e = -14;
      while ((mantissa & 0x0400u) == 0u) { mantissa <<= 1; --e; }
      mantissa &= 0x03ffu;
      bits = sign | ((uint32_t)(e + 127) << 23) | (mantissa << 13);
    }
  } else if (exponent == 0x1fu) {
    bits = sign | 0x7f800000u | (mantissa << 13);
  } else {
    bits = sign | ((exponent + 112u) << 23) | (mantissa << 13);
  }
  return f_from(bits);
}

uint16_t oracle_f32_to_f16(float value) {
  uint32_t bits = f_bits(value);
  uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
  uint32_t exponent = (bits >> 23) & 0xffu;
  uint32_t mantissa = bits & 0x007fffffu;
  if (exponent == 0xffu) {
    if (mantissa == 0u) return (uint16_t)(sign | 0x7c00u);
    return (uint16_t)(sign | 0x7c00u | (uint16_t)(mantissa >> 13) | 1u);
  }
  int he = (int)exponent - 127 + 15;
  if (he >= 31) return (uint16_t)(sign | 0x7c00u);
  if (he <= 0) {
    if (he < -10) return sign;
    uint32_t normalized = mantissa | 0x00800000u;
    uint32_t shift = (uint32_t)(14 - he);
    uint32_t rounded = normalized >> shift;
    uint32_t rem = normalized & ((1u << shift) - 1u);
    uint32_t halfway = 1u << (shift - 1u);
    if (rem > halfway || (rem == halfway && (rounded & 1u))) ++rounded;
    return (uint16_t)(sign | rounded);
  }
  uint32_t rm = mantissa >> 13;
  uint32_t rem = mantissa & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (rm & 1u))) {
    ++rm;
    if (rm == 0x0400u) {
      if (he + 1 >= 31) return (uint16_t)(sign | 0x7c00u);
      return (uint16_t)(sign | (uint16_t)((he + 1) << 10));
    }
  }
  return (uint16_t)(sign | (uint16_t)(he << 10) | (uint16_t)rm);
}

void oracle_f32_to_f16_array(const float* in, uint16_t* out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = oracle_f32_to_f16(in[i]);
}
void oracle_f16_to_f32_array(const uint16_t* in, float* out, size_t n) {
#pragma omp parallel for schedule(static) if (n > (1u << 20))
  for (size_t i = 0; i < n; ++i) out[i] = oracle_f16_to_f32(in[i]);
}

/* ----------------------------------------------------------------------- */
/* Dense layer math                                                          */
/* ----------------------------------------------------------------------- */

/* llama.cpp:193-212.  out = x * (1/sqrt(mean(x^2)+eps)) * w, per row. */
void oracle_rms_norm(const float* in, const float* w, size_t rows, size_t cols, float eps,
                     float* out) {
  for (size_t r = 0; r < rows; ++r) {
    const float* x = in + r * cols;
    float ss = 0.0f;
    for (size_t c = 0; c < cols; ++c) ss += x[c] * x[c];
    float inv = 1.0f / sqrtf(ss / (float)cols + eps);
    for (size_t c = 0; c < cols; ++c) out[r * cols + c] = x[c] * inv * w[c];
  }
}

/* llama.cpp:114-130.  One shared weight vector of length `width`; every
 * consecutive `width` values (one head) is normalised separately. */
void oracle_normalize_heads(float* v, size_t n, const float* w, size_t width, float eps) {
  for (size_t off = 0; off < n; off += width) {
    float ss = 0.0f;
    for (size_t d = 0; d < width; ++d) ss += v[off + d] * v[off + d];
    float inv = 1.0f / sqrtf(ss / (float)width + eps);
    for (size_t d = 0; d < width; ++d) v[off + d] *= inv * w[d];
  }
}

/* llama.cpp:214-240.  Half rotation: pairs (i, i + d/2), angle =
 * position / theta^(2i/d), all in F32. */
void oracle_apply_rope(float* v, size_t rows, size_t heads, size_t d, size_t first_pos,
                       float theta) {
  size_t half = d / 2;
  size_t width = heads * d;
  for (size_t t = 0; t < rows; ++t) {
    float position = (float)(first_pos + t);
    for (size_t h = 0; h < heads; ++h) {
      float* x = v + t * width + h * d;
      for (size_t i = 0; i < half; ++i) {
        float exponent = (float)(2u * i) / (float)d;
        float angle = position / powf(theta, exponent);
        float c = cosf(angle), s = sinf(angle);
        float a = x[i], b = x[half + i];
        x[i] = a * c - b * s;
        x[half + i] = b * c + a * s;
      }
    }
  }
}

/* tensor.cpp:47-62.  y[r][o] = sum_i x[r][i] * W[o][i], sequential over i. */
void oracle_linear(const float* x, size_t rows, size_t in, const float* W, size_t out,
                   float* y) {
  long long total = (long long)rows * (long long)out;
#pragma omp parallel for schedule(static)
  for (long long idx = 0; idx < total; ++idx) {
    size_t r = (size_t)(idx / (long long)out), o = (size_t)(idx % (long long)out);
    const float* xr = x + r * in;
    const float* wr = W + o * in;
    float sum = 0.0f;
    for (size_t i = 0; i < in; ++i) sum += xr[i] * wr[i];
    y[r * out + o] = sum;
  }
}

typedef struct {
  uint64_t hidden_size, intermediate_size, attention_heads, key_value_heads, head_dimension,
      maximum_sequence_length;
  float rms_norm_epsilon, rope_theta;
  uint32_t query_key_norm;
} oracle_config;

typedef struct {
  const float *input_norm, *query, *key, *value, *attention_output, *post_attention_norm;
  const float *gate, *up, *down, *query_norm, *key_norm;
} oracle_layer;

/* llama.cpp:28-52,152-191: contiguous per-sequence cache, index
 * (position * kv_heads + head) * head_dim + dim. */
typedef struct {
  uint64_t capacity, heads, dim, length;
  float* keys;
  float* values;
} oracle_kv;

/* llama.cpp:67-112.  Causal GQA: query head h reads kv head h / (Hq/Hkv);
 * scores scaled by 1/sqrt(d) after the dot product, softmax with the row
 * maximum subtracted, probabilities divided before the value product. */
void oracle_attention(const float* q, size_t rows, const oracle_config* cfg, size_t first_pos,
                      const oracle_kv* cache, float* out) {
  size_t Hq = cfg->attention_heads, Hkv = cfg->key_value_heads, d = cfg->head_dimension;
  size_t group = Hq / Hkv;
  float scale = 1.0f / sqrtf((float)d);
  long long total = (long long)rows * (long long)Hq;
#pragma omp parallel
  {
    float* scores = (float*)malloc(sizeof(float) * (first_pos + rows + 1));
#pragma omp for schedule(dynamic, 1)
    for (long long idx = 0; idx < total; ++idx) {
      size_t t = (size_t)(idx / (long long)Hq), h = (size_t)(idx % (long long)Hq);
      size_t kvh = h / group;
      size_t maxp = first_pos + t;
      const float* qr = q + t * Hq * d + h * d;
      float m = -INFINITY;
      for (size_t p = 0; p <= maxp; ++p) {
        const float* k = cache->keys + (p * Hkv + kvh) * d;
        float s = 0.0f;
        for (size_t i = 0; i < d; ++i) s += qr[i] * k[i];
        s *= scale;
        scores[p] = s;
        if (m < s) m = s; /* std::max(m, s) */
      }
      float den = 0.0f;
      for (size_t p = 0; p <= maxp; ++p) {
        scores[p] = expf(scores[p] - m);
        den += scores[p];
      }
      for (size_t i = 0; i < d; ++i) {
        float r = 0.0f;
        for (size_t p = 0; p <= maxp; ++p)
          r += (scores[p] / den) * cache->values[(p * Hkv + kvh) * d + i];
        out[t * Hq * d + h * d + i] = r;
      }
    }
    free(scores);
  }
}

/* llama.cpp:242-282.  One transformer layer over `rows` new tokens starting
 * at `first_pos`; appends K/V to the cache (position must equal its length). */
int oracle_transformer_layer(const float* input, size_t rows, const oracle_layer* w,
                             const oracle_config* cfg, size_t first_pos, oracle_kv* cache,
                             float* output) {
  size_t h = cfg->hidden_size, I = cfg->intermediate_size, d = cfg->head_dimension;
  size_t qw = cfg->attention_heads * d, kw = cfg->key_value_heads * d;
  if (rows == 0 || first_pos != cache->length || first_pos + rows > cache->capacity ||
      cache->heads != cfg->key_value_heads || cache->dim != d)
    return ORACLE_INVALID;
  float* normed = (float*)malloc(sizeof(float) * rows * h);
  float* q = (float*)malloc(sizeof(float) * rows * qw);
  float* k = (float*)malloc(sizeof(float) * rows * kw);
  float* v = (float*)malloc(sizeof(float) * rows * kw);
  float* att = (float*)malloc(sizeof(float) * rows * qw);
  float* hid = (float*)malloc(sizeof(float) * rows * h);
  float* g = (float*)malloc(sizeof(float) * rows * I);
  float* u = (float*)malloc(sizeof(float) * rows * I);
  oracle_rms_norm(input, w->input_norm, rows, h, cfg->rms_norm_epsilon, normed);
  oracle_linear(normed, rows, h, w->query, qw, q);
  oracle_linear(normed, rows, h, w->key, kw, k);
  oracle_linear(normed, rows, h, w->value, kw, v);
  if (cfg->query_key_norm) {
    oracle_normalize_heads(q, rows * qw, w->query_norm, d, cfg->rms_norm_epsilon);
    oracle_normalize_heads(k, rows * kw, w->key_norm, d, cfg->rms_norm_epsilon);
  }
  oracle_apply_rope(q, rows, cfg->attention_heads, d, first_pos, cfg->rope_theta);
  oracle_apply_rope(k, rows, cfg->key_value_heads, d, first_pos, cfg->rope_theta);
  memcpy(cache->keys + cache->length * kw, k, sizeof(float) * rows * kw);
  memcpy(cache->values + cache->length * kw, v, sizeof(float) * rows * kw);
  cache->length += rows;
  oracle_attention(q, rows, cfg, first_pos, cache, att);
  oracle_linear(att, rows, qw, w->attention_output, h, hid);
  for (size_t i = 0; i < rows * h; ++i) hid[i] += input[i];
  oracle_rms_norm(hid, w->post_attention_norm, rows, h, cfg->rms_norm_epsilon, normed);
  oracle_linear(normed, rows, h, w->gate, I, g);
  oracle_linear(normed, rows, h, w->up, I, u);
  for (size_t i = 0; i < rows * I; ++i) {
    float x = g[i];
    g[i] = (x / (1.0f + expf(-x))) * u[i];
  }
  oracle_linear(g, rows, I, w->down, h, output);
  for (size_t i = 0; i < rows * h; ++i) output[i] += hid[i];
  free(normed); free(q); free(k); free(v); free(att); free(hid); free(g); free(u);
  return ORACLE_OK;
}

/* llama.cpp:284-288. */
void oracle_final_logits(const float* hidden, size_t rows, size_t h, const float* norm_w,
                         const float* head, size_t vocab, float eps, float* logits) {
  float* normed = (float*)malloc(sizeof(float) * rows * h);
  oracle_rms_norm(hidden, norm_w, rows, h, eps, normed);
  oracle_linear(normed, rows, h, head, vocab, logits);
  free(normed);
}

/* llama.cpp:290-308.  First maximum wins; any non-finite logit is refused.
 * Returns the index, or -1 for a refusal. */
long long oracle_greedy_sample_last(const float* logits, size_t rows, size_t cols) {
  if (rows == 0 || cols == 0) return -1;
  const float* row = logits + (rows - 1) * cols;
  for (size_t i = 0; i < cols; ++i)
    if (!isfinite(row[i])) return -1;
  size_t sel = 0;
  for (size_t i = 1; i < cols; ++i)
    if (row[i] > row[sel]) sel = i;
  return (long long)sel;
}

/* ----------------------------------------------------------------------- */
/* sampling.cpp:10-90                                                        */
/* ----------------------------------------------------------------------- */
typedef struct {
  double temperature, top_p;
  uint64_t top_k, seed;
  uint32_t return_logprobs, top_logprobs;
} oracle_sampling;

typedef struct {
  double probability;
  uint64_t token;
} oracle_candidate;

static int cand_cmp(const void* pa, const void* pb) {
  const oracle_candidate* a = (const oracle_candidate*)pa;
  const oracle_candidate* b = (const oracle_candidate*)pb;
  /* Descending probability, then ascending token: a strict total order. */
  if (a->probability == b->probability) return a->token < b->token ? -1 : (a->token > b->token);
  return a->probability > b->probability ? -1 : 1;
}

/* sampling.cpp:10-17. */
int oracle_validate_sampling(const oracle_sampling* o) {
  if (!isfinite(o->temperature) || o->temperature < 0.0 || o->temperature > 100.0 ||
      !isfinite(o->top_p) || o->top_p <= 0.0 || o->top_p > 1.0 || o->top_logprobs > 5u ||
      (!o->return_logprobs && o->top_logprobs != 0u))
    return ORACLE_INVALID;
  return ORACLE_OK;
}

/* The 53-bit uniform draw of sampling.cpp:52-57 (SplitMix64 finaliser of
 * seed + golden-ratio * (index + 1)). */
double oracle_uniform(uint64_t seed, uint64_t generated_index) {
  uint64_t bits = seed + 0x9e3779b97f4a7c15ULL * (generated_index + 1u);
  bits = (bits ^ (bits >> 30)) * 0xbf58476d1ce4e5b9ULL;
  bits = (bits ^ (bits >> 27)) * 0x94d049bb133111ebULL;
  bits ^= bits >> 31;
  return (double)(bits >> 11) * 0x1.0p-53;
}

/* sampling.cpp:19-63.  Writes the token to *out; returns a status. */
int oracle_sample_logits(const float* logits, size_t n, const oracle_sampling* o,
                         uint64_t generated_index, uint64_t* out) {
  if (oracle_validate_sampling(o) != ORACLE_OK) return ORACLE_INVALID;
  if (n == 0) return ORACLE_INTERNAL;
  for (size_t i = 0; i < n; ++i)
    if (!isfinite(logits[i])) return ORACLE_INTERNAL;
  size_t best = 0;
  for (size_t i = 1; i < n; ++i)
    if (logits[i] > logits[best]) best = i;
  if (o->temperature == 0.0) { *out = best; return ORACLE_OK; }
  oracle_candidate* c = (oracle_candidate*)malloc(sizeof(oracle_candidate) * n);
  for (size_t i = 0; i < n; ++i) {
    c[i].probability = exp(((double)logits[i] - logits[best]) / o->temperature);
    c[i].token = i;
  }
  qsort(c, n, sizeof(oracle_candidate), cand_cmp);
  size_t size = n;
  if (o->top_k != 0 && o->top_k < size) size = (size_t)o->top_k;
  double total = 0.0;
  for (size_t i = 0; i < size; ++i) total += c[i].probability;
  double threshold = total * o->top_p;
  double retained = 0.0;
  size_t count = 0;
  do {
    retained += c[count++].probability;
  } while (retained < threshold && count < size);
  double target = oracle_uniform(o->seed, generated_index) * retained;
  uint64_t token = c[count - 1].token;
  for (size_t i = 0; i + 1 < count; ++i) {
    target -= c[i].probability;
    if (target < 0.0) { token = c[i].token; break; }
  }
  free(c);
  *out = token;
  return ORACLE_OK;
}

typedef struct {
  uint64_t token_id;
  double logprob;
  uint32_t has_logprob, n_top;
  uint64_t top_ids[5];
  double top_logprobs[5];
} oracle_sampled;

/* sampling.cpp:65-90. */
int oracle_sample_token(const float* logits, size_t n, const oracle_sampling* o,
                        uint64_t generated_index, oracle_sampled* out) {
  memset(out, 0, sizeof(*out));
  int st = oracle_sample_logits(logits, n, o, generated_index, &out->token_id);
  if (st != ORACLE_OK || !o->return_logprobs) return st;
  double maximum = logits[0];
  for (size_t i = 1; i < n; ++i)
    if ((double)logits[i] > maximum) maximum = logits[i];
  double sum = 0.0;
  for (size_t i = 0; i < n; ++i) sum += exp((double)logits[i] - maximum);
  double log_sum = log(sum);
  out->has_logprob = 1;
  out->logprob = (double)logits[out->token_id] - maximum - log_sum;
  size_t count = o->top_logprobs < n ? o->top_logprobs : n;
  /* partial_sort by (logprob desc, token asc): repeated selection. */
  for (size_t k = 0; k < count; ++k) {
    long long pick = -1;
    double pl = 0.0;
    for (size_t i = 0; i < n; ++i) {
      int used = 0;
      for (size_t j = 0; j < k; ++j) used |= out->top_ids[j] == i;
      if (used) continue;
      double lp = (double)logits[i] - maximum - log_sum;
      if (pick < 0 || lp > pl) { pick = (long long)i; pl = lp; }
    }
    out->top_ids[k] = (uint64_t)pick;
    out->top_logprobs[k] = pl;
  }
  out->n_top = (uint32_t)count;
  return ORACLE_OK;
}

/* ----------------------------------------------------------------------- */
/* Ragged batch packer (this build's contract; no reference counterpart:    */
/* the reference keeps one contiguous cache per sequence).                  */
/*                                                                          */
/* Inputs: R rows of (sequence slot, first position, token count) and the   */
/* per-slot block lists [slots][max_blocks].  Outputs, for T = sum of the   */
/* token counts:                                                            */
/*   cu_seqlens[R+1]  prefix sums of token counts                           */
/*   positions[T]     first_position + offset within the row                */
/*   slot_mapping[T]  block_list[slot][pos / B] * B + pos % B               */
/*   token_row[T]     row index of each token                               */
/*   seq_lens[R]      first_position + token count (context after the step) */
/*   block_tables[R][max_blocks]  the slot's block list, -1 past the blocks */
/*                    the context needs                                     */
/* Returns ORACLE_INVALID when a row needs a block its slot does not own.   */
/* ----------------------------------------------------------------------- */
int oracle_pack(const int32_t* row_slot, const int32_t* row_first, const int32_t* row_count,
                int32_t rows, const int32_t* slot_blocks, int32_t max_blocks, int32_t block,
                int32_t* cu_seqlens, int32_t* positions, int32_t* slot_mapping,
                int32_t* token_row, int32_t* seq_lens, int32_t* block_tables) {
  int32_t t = 0;
  cu_seqlens[0] = 0;
  for (int32_t r = 0; r < rows; ++r) {
    const int32_t* list = slot_blocks + (size_t)row_slot[r] * max_blocks;
    int32_t ctx = row_first[r] + row_count[r];
    int32_t need = (ctx + block - 1) / block;
    if (need > max_blocks) return ORACLE_INVALID;
    for (int32_t b = 0; b < need; ++b)
      if (list[b] < 0) return ORACLE_INVALID;
    for (int32_t i = 0; i < row_count[r]; ++i, ++t) {
      int32_t pos = row_first[r] + i;
      positions[t] = pos;
      slot_mapping[t] = list[pos / block] * block + pos % block;
      token_row[t] = r;
    }
    cu_seqlens[r + 1] = t;
    seq_lens[r] = ctx;
    for (int32_t b = 0; b < max_blocks; ++b)
      block_tables[(size_t)r * max_blocks + b] = b < need ? list[b] : -1;
  }
  return ORACLE_OK;
}

/* ----------------------------------------------------------------------- */
/* Seeded synthetic weights (this build's contract, shared bit for bit with */
/* the device initialiser in hllm_b200/csrc/synth.cu).                       */
/*                                                                          */
/* h = mix64(seed * K1 + tag * K2 + index) with the SplitMix64 finaliser.   */
/* Matrices: the sum of the four 16-bit fields of h (an Irwin-Hall(4)       */
/* variate, mean 131070, standard deviation 37837.2) centred and scaled to  */
/* the requested standard deviation; integer-to-float is exact and the one  */
/* F32 multiply rounds the same way on any IEEE machine.  Norm vectors:     */
/* 1 + spread * u with u uniform in [-1, 1).  Values are then rounded to    */
/* F16 (round to nearest even).                                             */
/* ----------------------------------------------------------------------- */
static uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
  return z ^ (z >> 31);
}

static uint64_t synth_hash(uint64_t seed, uint64_t tag, uint64_t index) {
  return mix64(seed * 0xd1b54a32d192ed03ULL + tag * 0x9e3779b97f4a7c15ULL + index);
}

void oracle_synth_matrix_f16(uint64_t seed, uint64_t tag, uint64_t n, float stddev,
                             uint16_t* out) {
  float unit = stddev / 37837.2f;
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < (long long)n; ++i) {
    uint64_t h = synth_hash(seed, tag, (uint64_t)i);
    int32_t s = (int32_t)((h & 0xffffu) + ((h >> 16) & 0xffffu) + ((h >> 32) & 0xffffu) +
                          (h >> 48)) - 131070;
    out[i] = oracle_f32_to_f16((float)s * unit);
  }
}

void oracle_synth_norm_f16(uint64_t seed, uint64_t tag, uint64_t n, float spread,
                           uint16_t* out) {
  float unit = spread / 32768.0f;
  for (uint64_t i = 0; i < n; ++i) {
    uint64_t h = synth_hash(seed, tag, i);
    int32_t s = (int32_t)(h & 0xffffu) - 32768;
    out[i] = oracle_f32_to_f16(1.0f + (float)s * unit);
  }
}

int oracle_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
