// envelope.cuh -- hLLM's F16 boundary wire message, host side.
//
// A stage boundary crosses workers as a serialized hllm.v1.StageMessage whose
// `tensor` member is a TensorEnvelope (proto/execution.proto:48-65, 115-123),
// built by worker::encode_tensor and checked by worker::decode_tensor
// (cpp/src/worker/boundary_codec.cpp:15-108) with runtime::validate_tensor_envelope
// (cpp/src/tensor_envelope.cpp:26-83).  This codec writes and reads those bytes
// itself (protobuf wire format, proto3 rules), so that the F16 payload can be
// copied straight from device memory into its final place in the message and
// read by the stage straight out of a received message.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <string>
#include <string_view>

#include "hllm_b200.h"

namespace hb {

// worker::BoundaryIdentity (cpp/include/hllm/worker/boundary_codec.hpp:7-13).
struct EnvelopeIdentity {
  std::string_view deployment_id;
  uint64_t deployment_version = 0;
  std::string_view request_id;
  uint64_t maximum_tokens = 0;
  uint64_t hidden_size = 0;
};

// Where the payload sits in an encoded message, and the message's size.
struct EnvelopeLayout {
  uint64_t payload_offset = 0;
  uint64_t total = 0;
};

// The checks encode_tensor makes before it serializes (boundary_codec.cpp:71-73,
// 90-95), then the layout of the message.  Non-OK with *why on failure.
hllm_b200_status envelope_plan(const EnvelopeIdentity& id, uint64_t sequence, uint64_t position,
                               bool prefill, uint64_t payload_bytes, uint64_t tokens,
                               uint64_t width, EnvelopeLayout* layout, std::string* why);

// Writes the message around its payload: every byte of [0, total) except
// [payload_offset, payload_offset + tokens * width * 2).
void envelope_write_frame(const EnvelopeIdentity& id, uint64_t sequence, uint64_t position,
                          bool prefill, uint64_t tokens, uint64_t width, uint8_t* out);

// encode_tensor's finite check (boundary_codec.cpp:96-100): no F16 value in
// `payload` has an all-ones exponent.
bool f16_payload_finite(const uint8_t* payload, uint64_t bytes);

// decode_tensor on a serialized StageMessage: parses it, checks it like
// boundary_codec.cpp:15-66 and tensor_envelope.cpp:26-83, and locates the F16
// rows inside `message` (no copy).
hllm_b200_status envelope_decode(const uint8_t* message, uint64_t bytes,
                                 const EnvelopeIdentity& id, uint64_t sequence,
                                 uint64_t position, bool prefill, uint64_t* payload_offset,
                                 uint64_t* tokens, std::string* why);

}  // namespace hb
