// envelope.cu -- the F16 boundary wire message (StageMessage{TensorEnvelope}).
//
// Encoding follows worker::encode_tensor (cpp/src/worker/boundary_codec.cpp:68-108):
// the fields it sets, serialized the way protobuf's proto3 serializers do --
// field-number order, zero scalars and empty strings left out, repeated
// scalars packed -- so the bytes equal the reference worker's.  The payload is
// the last field but one (field 15; deployment_version, field 16, follows), so
// a caller can place the payload itself: from host memory here, or by a
// device-to-host copy straight into the message (hllm_b200_stage_envelope).
//
// Decoding parses any valid encoding (packed or unpacked repeated fields,
// repeated and unknown fields, split or interleaved oneof members), then checks
// the message exactly as worker::decode_tensor (boundary_codec.cpp:15-66) and
// runtime::validate_tensor_envelope (cpp/src/tensor_envelope.cpp:26-83) do, with
// their messages, and returns where the payload lies in the received bytes.
#include <cstring>
#include <vector>

#include "envelope.cuh"

namespace hb {
void set_last_error(const std::string& message);  // stage.cu

namespace {

constexpr uint64_t kMaximumRpcBytes = 16ull * 1024 * 1024;  // boundary_codec.hpp:6
constexpr uint64_t kMaximumPayload = kMaximumRpcBytes / 2;
constexpr int kPhasePrefill = 1, kPhaseDecode = 2;            // execution.proto:7-11
constexpr int kDataTypeF16 = 10;                              // common.proto:23
constexpr std::string_view kLayout = "dense_row_major_le";
constexpr int kMaxGroupDepth = 64;

int varint_size(uint64_t v) {
  int n = 1;
  while (v >= 0x80) {
    v >>= 7;
    ++n;
  }
  return n;
}

uint8_t* put_varint(uint8_t* p, uint64_t v) {
  while (v >= 0x80) {
    *p++ = static_cast<uint8_t>(v) | 0x80;
    v >>= 7;
  }
  *p++ = static_cast<uint8_t>(v);
  return p;
}

uint8_t* put_bytes(uint8_t* p, uint8_t key, std::string_view s) {
  *p++ = key;
  p = put_varint(p, s.size());
  std::memcpy(p, s.data(), s.size());
  return p + s.size();
}

// Size of the TensorEnvelope fields before field 15's value, and after it.
struct EnvelopeSizes {
  uint64_t head, tail;
};
EnvelopeSizes envelope_sizes(const EnvelopeIdentity& id, uint64_t sequence, uint64_t position,
                             uint64_t tokens, uint64_t width, uint64_t payload) {
  uint64_t head = 2;  // protocol_version = 1
  if (!id.deployment_id.empty())
    head += 1 + varint_size(id.deployment_id.size()) + id.deployment_id.size();
  if (!id.request_id.empty()) head += 1 + varint_size(id.request_id.size()) + id.request_id.size();
  if (sequence) head += 1 + varint_size(sequence);
  head += 2;  // phase
  if (position) head += 1 + varint_size(position);
  head += 2 + varint_size(tokens);                          // sequence_lengths [tokens]
  head += 3;                                                // cache_slot_ids [0]
  head += 2 + 1 + varint_size(tokens) + varint_size(width);  // shape [1, tokens, width]
  head += 2;                                                // dtype
  head += 2 + kLayout.size();                               // layout
  head += 1 + varint_size(payload);                         // payload_length
  head += 1 + varint_size(payload);                         // payload key and length
  const uint64_t tail = id.deployment_version ? 2 + varint_size(id.deployment_version) : 0;
  return {head, tail};
}

// ------------------------------------------------------------------ parsing
struct Reader {
  const uint8_t* p;
  const uint8_t* end;
  bool bad = false;

  bool varint(uint64_t* v) {
    uint64_t x = 0;
    for (int i = 0; i < 10; ++i) {
      if (p >= end) return fail();
      const uint8_t b = *p++;
      x |= static_cast<uint64_t>(b & 0x7F) << (7 * i);  // bits past 64 drop
      if (!(b & 0x80)) {
        *v = x;
        return true;
      }
    }
    return fail();
  }
  bool key(uint32_t* field, int* wire) {
    uint64_t k;
    if (!varint(&k)) return false;
    if (k > 0xFFFFFFFFull || (k >> 3) == 0 || (k & 7) > 5) return fail();
    *field = static_cast<uint32_t>(k >> 3);
    *wire = static_cast<int>(k & 7);
    return true;
  }
  bool bytes(std::string_view* out) {
    uint64_t n;
    if (!varint(&n)) return false;
    if (n > static_cast<uint64_t>(end - p)) return fail();
    *out = std::string_view(reinterpret_cast<const char*>(p), n);
    p += n;
    return true;
  }
  // Skips the value of an unknown field; a group is skipped to its end tag.
  bool skip(uint32_t field, int wire, int depth = 0) {
    uint64_t v;
    std::string_view s;
    switch (wire) {
      case 0: return varint(&v);
      case 1:
      case 5: {
        const int n = wire == 1 ? 8 : 4;
        if (end - p < n) return fail();
        p += n;
        return true;
      }
      case 2: return bytes(&s);
      case 3: {
        if (depth >= kMaxGroupDepth) return fail();
        for (;;) {
          if (p >= end) return fail();
          uint32_t f;
          int w;
          if (!key(&f, &w)) return false;
          if (w == 4) return f == field ? true : fail();
          if (!skip(f, w, depth + 1)) return false;
        }
      }
      default: return fail();  // an end-group tag with no group open
    }
  }
  bool fail() {
    bad = true;
    return false;
  }
};

// Strict UTF-8 (no overlong forms, surrogates or code points past U+10FFFF):
// proto3 strings that are not valid UTF-8 do not parse.
bool valid_utf8(std::string_view s) {
  const auto* p = reinterpret_cast<const uint8_t*>(s.data());
  const auto* e = p + s.size();
  while (p < e) {
    const uint8_t c = *p;
    if (c < 0x80) {
      ++p;
      continue;
    }
    int n;
    uint32_t cp, min;
    if ((c & 0xE0) == 0xC0) {
      n = 1, cp = c & 0x1F, min = 0x80;
    } else if ((c & 0xF0) == 0xE0) {
      n = 2, cp = c & 0x0F, min = 0x800;
    } else if ((c & 0xF8) == 0xF0) {
      n = 3, cp = c & 0x07, min = 0x10000;
    } else {
      return false;
    }
    if (e - p <= n) return false;
    for (int k = 1; k <= n; ++k) {
      if ((p[k] & 0xC0) != 0x80) return false;
      cp = (cp << 6) | (p[k] & 0x3F);
    }
    if (cp < min || cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF)) return false;
    p += n + 1;
  }
  return true;
}

struct Envelope {
  uint32_t protocol_version = 0;
  std::string_view deployment_id, request_id, layout, checksum, payload;
  uint64_t microbatch_id = 0, sequence_number = 0, first_position = 0, payload_length = 0;
  uint64_t deployment_version = 0;
  int32_t phase = 0, dtype = 0;
  std::vector<uint64_t> sequence_lengths, cache_slot_ids, shape;

  std::vector<uint64_t>* repeated(uint32_t f) {
    return f == 8 ? &sequence_lengths : f == 9 ? &cache_slot_ids : f == 10 ? &shape : nullptr;
  }
};

// Merges one serialized TensorEnvelope into *e (scalars last-wins, repeated
// fields appended, a known field with another wire type kept as unknown).
bool merge_envelope(std::string_view body, Envelope* e) {
  Reader r{reinterpret_cast<const uint8_t*>(body.data()),
           reinterpret_cast<const uint8_t*>(body.data()) + body.size()};
  while (r.p < r.end) {
    uint32_t f;
    int w;
    if (!r.key(&f, &w)) return false;
    uint64_t v;
    std::string_view s;
    const bool scalar = f == 1 || (f >= 4 && f <= 7) || f == 11 || f == 13 || f == 16;
    if (w == 0 && scalar) {
      if (!r.varint(&v)) return false;
      switch (f) {
        case 1: e->protocol_version = static_cast<uint32_t>(v); break;
        case 4: e->microbatch_id = v; break;
        case 5: e->sequence_number = v; break;
        case 6: e->phase = static_cast<int32_t>(static_cast<uint32_t>(v)); break;
        case 7: e->first_position = v; break;
        case 11: e->dtype = static_cast<int32_t>(static_cast<uint32_t>(v)); break;
        case 13: e->payload_length = v; break;
        default: e->deployment_version = v;
      }
    } else if (w == 0 && e->repeated(f)) {
      if (!r.varint(&v)) return false;
      e->repeated(f)->push_back(v);
    } else if (w == 2 && (f == 2 || f == 3 || f == 12 || f == 14 || f == 15 || e->repeated(f))) {
      if (!r.bytes(&s)) return false;
      if (auto* rep = e->repeated(f)) {
        Reader q{reinterpret_cast<const uint8_t*>(s.data()),
                 reinterpret_cast<const uint8_t*>(s.data()) + s.size()};
        while (q.p < q.end) {
          if (!q.varint(&v)) return false;
          rep->push_back(v);
        }
      } else if (f == 14) {
        e->checksum = s;
      } else if (f == 15) {
        e->payload = s;
      } else {
        if (!valid_utf8(s)) return false;
        (f == 2 ? e->deployment_id : f == 3 ? e->request_id : e->layout) = s;
      }
    } else if (!r.skip(f, w)) {
      return false;
    }
  }
  return true;
}

// The StageMessage's body: 0 none, 2 tensor (into *e), another member's number.
bool parse_stage_message(const uint8_t* msg, uint64_t n, Envelope* e, int* body) {
  Reader r{msg, msg + n};
  *body = 0;
  while (r.p < r.end) {
    uint32_t f;
    int w;
    if (!r.key(&f, &w)) return false;
    if (w != 2 || f < 1 || f > 6) {
      if (!r.skip(f, w)) return false;
      continue;
    }
    std::string_view s;
    if (!r.bytes(&s)) return false;
    if (f == 2) {
      if (*body != 2) *e = Envelope{};
      if (!merge_envelope(s, e)) return false;
    }
    *body = static_cast<int>(f);
  }
  return true;
}

}  // namespace

hllm_b200_status envelope_plan(const EnvelopeIdentity& id, uint64_t sequence, uint64_t position,
                               bool prefill, uint64_t payload_bytes, uint64_t tokens,
                               uint64_t width, EnvelopeLayout* layout, std::string* why) {
  (void)prefill;
  if (payload_bytes > kMaximumPayload) {  // boundary_codec.cpp:71-73
    *why = "prefill activation exceeds transport limit";
    return HLLM_B200_RESOURCE_EXHAUSTED;
  }
  if (width == 0 || width != id.hidden_size || tokens == 0 ||  // :90-95
      tokens > (kMaximumRpcBytes / 4) / width || payload_bytes != tokens * width * 2) {
    *why = "backend returned an invalid boundary shape";
    return HLLM_B200_INTERNAL;
  }
  const EnvelopeSizes z = envelope_sizes(id, sequence, position, tokens, width, payload_bytes);
  const uint64_t env = z.head + payload_bytes + z.tail;
  layout->payload_offset = 1 + varint_size(env) + z.head;
  layout->total = 1 + varint_size(env) + env;
  return HLLM_B200_OK;
}

void envelope_write_frame(const EnvelopeIdentity& id, uint64_t sequence, uint64_t position,
                          bool prefill, uint64_t tokens, uint64_t width, uint8_t* out) {
  const uint64_t payload = tokens * width * 2;
  const EnvelopeSizes z = envelope_sizes(id, sequence, position, tokens, width, payload);
  uint8_t* p = out;
  *p++ = 0x12;  // StageMessage.tensor (field 2, length-delimited)
  p = put_varint(p, z.head + payload + z.tail);
  *p++ = 0x08;  // protocol_version
  *p++ = 0x01;
  if (!id.deployment_id.empty()) p = put_bytes(p, 0x12, id.deployment_id);
  if (!id.request_id.empty()) p = put_bytes(p, 0x1A, id.request_id);
  if (sequence) {
    *p++ = 0x28;
    p = put_varint(p, sequence);
  }
  *p++ = 0x30;  // phase
  *p++ = (sequence == 0 || prefill) ? kPhasePrefill : kPhaseDecode;
  if (position) {
    *p++ = 0x38;
    p = put_varint(p, position);
  }
  *p++ = 0x42;  // sequence_lengths, packed
  *p++ = static_cast<uint8_t>(varint_size(tokens));
  p = put_varint(p, tokens);
  *p++ = 0x4A;  // cache_slot_ids [0], packed
  *p++ = 0x01;
  *p++ = 0x00;
  *p++ = 0x52;  // shape [1, tokens, width], packed
  *p++ = static_cast<uint8_t>(1 + varint_size(tokens) + varint_size(width));
  *p++ = 0x01;
  p = put_varint(p, tokens);
  p = put_varint(p, width);
  *p++ = 0x58;  // dtype F16
  *p++ = kDataTypeF16;
  p = put_bytes(p, 0x62, kLayout);
  *p++ = 0x68;  // payload_length
  p = put_varint(p, payload);
  *p++ = 0x7A;  // payload
  p = put_varint(p, payload);
  p += payload;
  if (id.deployment_version) {
    *p++ = 0x80;  // field 16, varint
    *p++ = 0x01;
    p = put_varint(p, id.deployment_version);
  }
}

bool f16_payload_finite(const uint8_t* payload, uint64_t bytes) {
  uint8_t any = 0;  // a plain loop: the compiler vectorises it
  for (uint64_t i = 1; i < bytes; i += 2) any |= ((payload[i] & 0x7C) == 0x7C);
  return !any;
}

hllm_b200_status envelope_decode(const uint8_t* message, uint64_t bytes,
                                 const EnvelopeIdentity& id, uint64_t sequence,
                                 uint64_t position, bool prefill, uint64_t* payload_offset,
                                 uint64_t* tokens, std::string* why) {
  auto invalid = [&](const char* m) {
    *why = m;
    return HLLM_B200_INVALID_REQUEST;
  };
  Envelope e;
  int body = 0;
  if (!parse_stage_message(message, bytes, &e, &body)) return invalid("malformed stage message");
  if (body != 2) return invalid("stage message does not carry a tensor");
  if (e.deployment_id != id.deployment_id || e.deployment_version != id.deployment_version ||
      e.request_id != id.request_id || e.microbatch_id != 0)  // boundary_codec.cpp:8-13
    return invalid("message identity does not match the active sequence");
  const int phase = (sequence == 0 || prefill) ? kPhasePrefill : kPhaseDecode;
  if (e.sequence_number != sequence || e.first_position != position || e.phase != phase ||
      e.dtype != kDataTypeF16 || e.layout != kLayout || !e.checksum.empty())  // :20-27
    return invalid("invalid tensor order, phase, encoding or unsupported checksum");
  // runtime::validate_tensor_envelope with decode_tensor's limits (:43-47):
  // batch 1, the request's tokens, the model width, half the RPC limit.
  const uint64_t max_seq = id.maximum_tokens, hidden_limit = id.hidden_size;
  if (e.protocol_version != 1) return invalid("unsupported tensor protocol version");
  if (e.deployment_id.empty() || e.deployment_version == 0 || e.request_id.empty())
    return invalid("tensor envelope is missing deployment or request identity");
  if (max_seq == 0 || hidden_limit == 0) return invalid("tensor envelope limits are invalid");
  if (e.shape.size() != 3) return invalid("tensor boundary shape must be [batch, sequence, hidden]");
  const uint64_t batch = e.shape[0], seq = e.shape[1], hidden = e.shape[2];
  if (batch == 0 || batch > 1 || seq == 0 || hidden != hidden_limit ||
      e.sequence_lengths.size() != batch || e.cache_slot_ids.size() != batch)
    return invalid("tensor boundary dimensions or batch metadata are invalid");
  if (phase == kPhaseDecode && seq != 1)
    return invalid("decode tensor must have a singleton sequence dimension");
  for (const uint64_t length : e.sequence_lengths)
    if (length == 0 || length != seq || e.first_position > max_seq ||
        length > max_seq - e.first_position)
      return invalid("tensor sequence metadata exceeds configured capacity");
  uint64_t expected = batch;
  for (const uint64_t factor : {seq, hidden, uint64_t{2}}) {
    if (expected != 0 && factor > UINT64_MAX / expected)
      return invalid("tensor payload size overflows native size limits");
    expected *= factor;
  }
  if (expected != e.payload_length || e.payload_length != e.payload.size() ||
      e.payload_length > kMaximumPayload)
    return invalid("tensor payload length does not match its shape or limits");
  if (e.cache_slot_ids.size() != 1 || e.cache_slot_ids[0] != 0)  // boundary_codec.cpp:48-50
    return invalid("single-sequence execution requires cache slot zero");
  const auto* payload = reinterpret_cast<const uint8_t*>(e.payload.data());
  if (!f16_payload_finite(payload, e.payload.size()))  // :55-60
    return invalid("non-finite boundary activation");
  *payload_offset = static_cast<uint64_t>(payload - message);
  *tokens = seq;
  return HLLM_B200_OK;
}

namespace {
bool identity_of(const hllm_b200_boundary_identity* in, EnvelopeIdentity* out) {
  if (!in || !in->deployment_id || !in->request_id) return false;
  out->deployment_id = in->deployment_id;
  out->request_id = in->request_id;
  out->deployment_version = in->deployment_version;
  out->maximum_tokens = in->maximum_tokens;
  out->hidden_size = in->hidden_size;
  return true;
}

hllm_b200_status report(hllm_b200_status code, const std::string& message) {
  set_last_error(message);
  return code;
}
}  // namespace

}  // namespace hb

extern "C" hllm_b200_status hllm_b200_envelope_encode(
    const hllm_b200_boundary_identity* identity, uint64_t sequence, uint64_t position,
    uint32_t prefill, const uint16_t* payload, uint64_t payload_bytes, uint64_t tokens,
    uint64_t width, uint8_t* out, uint64_t capacity, uint64_t* written) {
  hb::EnvelopeIdentity id;
  if (!hb::identity_of(identity, &id) || !written)
    return hb::report(HLLM_B200_INVALID_REQUEST, "null argument");
  hb::EnvelopeLayout layout;
  std::string why;
  const hllm_b200_status st = hb::envelope_plan(id, sequence, position, prefill != 0,
                                                payload_bytes, tokens, width, &layout, &why);
  if (st != HLLM_B200_OK) return hb::report(st, why);
  *written = layout.total;
  if (!out) return HLLM_B200_OK;  // size query
  if (capacity < layout.total) return hb::report(HLLM_B200_INVALID_REQUEST, "output buffer too small");
  if (!payload) return hb::report(HLLM_B200_INVALID_REQUEST, "null payload");
  const auto* bytes = reinterpret_cast<const uint8_t*>(payload);
  if (!hb::f16_payload_finite(bytes, payload_bytes))
    return hb::report(HLLM_B200_INTERNAL, "backend returned a non-finite boundary activation");
  hb::envelope_write_frame(id, sequence, position, prefill != 0, tokens, width, out);
  std::memcpy(out + layout.payload_offset, bytes, payload_bytes);
  return HLLM_B200_OK;
}

extern "C" hllm_b200_status hllm_b200_envelope_decode(
    const uint8_t* message, uint64_t bytes, const hllm_b200_boundary_identity* identity,
    uint64_t sequence, uint64_t position, uint32_t prefill, uint64_t* payload_offset,
    uint64_t* tokens) {
  hb::EnvelopeIdentity id;
  if (!hb::identity_of(identity, &id) || (!message && bytes) || !payload_offset || !tokens)
    return hb::report(HLLM_B200_INVALID_REQUEST, "null argument");
  std::string why;
  const hllm_b200_status st = hb::envelope_decode(message, bytes, id, sequence, position,
                                                  prefill != 0, payload_offset, tokens, &why);
  if (st != HLLM_B200_OK) return hb::report(st, why);
  return HLLM_B200_OK;
}
