"""CPU restatement of hLLM's F16 boundary wire codec (TEST INFRASTRUCTURE ONLY).

Imported by tests/ alone; the product package never imports it.  It restates,
function by function:

* ``worker::encode_tensor``  cpp/src/worker/boundary_codec.cpp:68-108
* ``worker::decode_tensor``  cpp/src/worker/boundary_codec.cpp:15-66
* ``runtime::validate_tensor_envelope``  cpp/src/tensor_envelope.cpp:26-83
* ``runtime::SequenceTracker::accept``  cpp/src/tensor_envelope.cpp:85-93

and the protobuf wire format of ``hllm.v1.StageMessage`` / ``TensorEnvelope``
(proto/execution.proto:48-65, 115-123) as protobuf's proto3 serializers write
it: fields in field-number order, default scalars and empty strings omitted,
repeated scalars packed.  The restatement is pinned by
tests/golden/envelope_cases.json (messages serialized by the reference's own
generated execution_pb2) and, for the metadata rules, by the reference's
validate_tensor_envelope compiled into oracle/_ref.

Errors are returned as (status, message) with the statuses of
include/hllm_b200.h (INVALID_REQUEST 1, RESOURCE_EXHAUSTED 3, INTERNAL 6)
and the reference's exception messages.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Tuple

INVALID_REQUEST, RESOURCE_EXHAUSTED, INTERNAL = 1, 3, 6
MAXIMUM_RPC_BYTES = 16 * 1024 * 1024          # boundary_codec.hpp:6
PHASE_PREFILL, PHASE_DECODE = 1, 2            # execution.proto:7-11
DATA_TYPE_F16 = 10                            # common.proto:23
LAYOUT = b"dense_row_major_le"
U64 = (1 << 64) - 1


class EnvelopeFailure(Exception):
    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status
        self.message = message


@dataclass
class Identity:
    """worker::BoundaryIdentity (boundary_codec.hpp:7-13)."""
    deployment_id: bytes
    deployment_version: int
    request_id: bytes
    maximum_tokens: int
    hidden_size: int


# ----------------------------------------------------------------------------- wire
def varint(v: int) -> bytes:
    out = bytearray()
    v &= U64
    while True:
        b = v & 0x7F
        v >>= 7
        if v:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _key(field: int, wire: int) -> bytes:
    return varint((field << 3) | wire)


def _len_field(field: int, data: bytes) -> bytes:
    return _key(field, 2) + varint(len(data)) + data


def _packed(field: int, values: List[int]) -> bytes:
    if not values:
        return b""
    return _len_field(field, b"".join(varint(v) for v in values))


def envelope_bytes(protocol_version=0, deployment_id=b"", request_id=b"", microbatch_id=0,
                   sequence_number=0, phase=0, first_position=0, sequence_lengths=(),
                   cache_slot_ids=(), shape=(), dtype=0, layout=b"", payload_length=0,
                   checksum=b"", payload=b"", deployment_version=0) -> bytes:
    """A serialized TensorEnvelope (execution.proto:48-65), proto3 rules."""
    out = bytearray()
    if protocol_version:
        out += _key(1, 0) + varint(protocol_version & 0xFFFFFFFF)
    if deployment_id:
        out += _len_field(2, deployment_id)
    if request_id:
        out += _len_field(3, request_id)
    for field, v in ((4, microbatch_id), (5, sequence_number), (6, phase), (7, first_position)):
        if v:
            out += _key(field, 0) + varint(v)
    out += _packed(8, list(sequence_lengths))
    out += _packed(9, list(cache_slot_ids))
    out += _packed(10, list(shape))
    if dtype:
        out += _key(11, 0) + varint(dtype)
    if layout:
        out += _len_field(12, layout)
    if payload_length:
        out += _key(13, 0) + varint(payload_length)
    if checksum:
        out += _len_field(14, checksum)
    if payload:
        out += _len_field(15, payload)
    if deployment_version:
        out += _key(16, 0) + varint(deployment_version)
    return bytes(out)


def stage_message(envelope: bytes) -> bytes:
    """StageMessage{tensor = envelope} (execution.proto:115-123, field 2)."""
    return _len_field(2, envelope)


class _Malformed(Exception):
    pass


def _read_varint(buf: bytes, i: int) -> Tuple[int, int]:
    """At most 10 bytes; the value wraps modulo 2^64 (bits past 64 are dropped)."""
    v, shift = 0, 0
    for _ in range(10):
        if i >= len(buf):
            raise _Malformed()
        b = buf[i]
        i += 1
        v |= (b & 0x7F) << shift
        shift += 7
        if not b & 0x80:
            return v & U64, i
    raise _Malformed()


def _read_key(buf: bytes, i: int) -> Tuple[int, int, int]:
    """(field, wire type, next index): a tag wider than 32 bits, field 0 or the
    wire types 6 and 7 do not parse."""
    key, i = _read_varint(buf, i)
    field, wire = key >> 3, key & 7
    if key > 0xFFFFFFFF or field == 0 or wire > 5:
        raise _Malformed()
    return field, wire, i


def _skip(buf: bytes, i: int, field: int, wire: int, depth: int = 0) -> int:
    """Index after the value of an unknown field (groups skipped to their end
    tag, nested at most 64 deep)."""
    if wire == 0:
        return _read_varint(buf, i)[1]
    if wire == 1 or wire == 5:
        i += 8 if wire == 1 else 4
        if i > len(buf):
            raise _Malformed()
        return i
    if wire == 2:
        n, i = _read_varint(buf, i)
        if n > len(buf) - i:
            raise _Malformed()
        return i + n
    if wire == 3:
        if depth >= 64:
            raise _Malformed()
        while True:
            if i >= len(buf):
                raise _Malformed()
            f, w, i = _read_key(buf, i)
            if w == 4:
                if f != field:
                    raise _Malformed()
                return i
            i = _skip(buf, i, f, w, depth + 1)
    raise _Malformed()  # an end-group tag with no group open


def _utf8(b: bytes) -> bytes:
    b.decode("utf-8")  # proto3 strings must be valid UTF-8
    return b


class Envelope:
    """Parsed TensorEnvelope fields (proto3 defaults)."""

    def __init__(self):
        self.protocol_version = 0
        self.deployment_id = b""
        self.request_id = b""
        self.microbatch_id = 0
        self.sequence_number = 0
        self.phase = 0
        self.first_position = 0
        self.sequence_lengths: List[int] = []
        self.cache_slot_ids: List[int] = []
        self.shape: List[int] = []
        self.dtype = 0
        self.layout = b""
        self.payload_length = 0
        self.checksum = b""
        self.payload = b""
        self.payload_offset = 0  # where the payload bytes sit in the parsed message
        self.deployment_version = 0


def parse_stage_message(msg: bytes) -> Optional[Envelope]:
    """The TensorEnvelope a StageMessage carries (None when its body is
    another member).  Raises EnvelopeFailure on bytes that do not parse."""
    env, case = None, 0
    try:
        i = 0
        while i < len(msg):
            field, wire, i = _read_key(msg, i)
            if wire != 2 or not 1 <= field <= 6:
                i = _skip(msg, i, field, wire)
                continue
            n, i = _read_varint(msg, i)
            if n > len(msg) - i:
                raise _Malformed()
            body = msg[i:i + n]
            if field == 2:
                if case != 2:
                    env = Envelope()
                _merge_envelope(env, body, i)
                case = 2
            else:  # another member of the oneof body (its contents are not checked)
                case, env = field, None
            i += n
    except (_Malformed, UnicodeDecodeError):
        raise EnvelopeFailure(INVALID_REQUEST, "malformed stage message")
    return env if case == 2 else None


def _merge_envelope(env: Envelope, buf: bytes, base: int) -> None:
    """Merges one serialized TensorEnvelope (at offset `base` of the message)
    into env: scalars and strings last-wins, repeated fields appended (packed
    or not), a known field with another wire type kept as unknown."""
    scalars = {1: "protocol_version", 4: "microbatch_id", 5: "sequence_number", 6: "phase",
               7: "first_position", 11: "dtype", 13: "payload_length", 16: "deployment_version"}
    strings = {2: "deployment_id", 3: "request_id", 12: "layout"}
    repeated = {8: "sequence_lengths", 9: "cache_slot_ids", 10: "shape"}
    i = 0
    while i < len(buf):
        field, wire, i = _read_key(buf, i)
        if wire == 0 and field in scalars:
            v, i = _read_varint(buf, i)
            if field == 1:                    # uint32
                v &= 0xFFFFFFFF
            elif field in (6, 11):            # enums are int32
                v &= 0xFFFFFFFF
                if v >= 1 << 31:
                    v -= 1 << 32
            setattr(env, scalars[field], v)
        elif wire == 0 and field in repeated:
            v, i = _read_varint(buf, i)
            getattr(env, repeated[field]).append(v)
        elif wire == 2 and (field in strings or field in repeated or field in (14, 15)):
            n, i = _read_varint(buf, i)
            if n > len(buf) - i:
                raise _Malformed()
            v = buf[i:i + n]
            if field in strings:
                setattr(env, strings[field], _utf8(bytes(v)))
            elif field in repeated:
                j, vals = 0, getattr(env, repeated[field])
                while j < len(v):
                    x, j = _read_varint(v, j)
                    vals.append(x)
            elif field == 14:
                env.checksum = bytes(v)
            else:
                env.payload = bytes(v)
                env.payload_offset = base + i
            i += n
        else:
            i = _skip(buf, i, field, wire)


# ----------------------------------------------------------------------------- codec
def encode_tensor(payload: bytes, tokens: int, width: int, identity: Identity, sequence: int,
                  position: int, prefill: bool = False) -> bytes:
    """boundary_codec.cpp:68-108: the serialized StageMessage, or EnvelopeFailure."""
    if len(payload) > MAXIMUM_RPC_BYTES // 2:                                   # :71-73
        raise EnvelopeFailure(RESOURCE_EXHAUSTED, "prefill activation exceeds transport limit")
    if (width == 0 or width != identity.hidden_size or tokens == 0                # :90-95
            or tokens > (MAXIMUM_RPC_BYTES // 4) // width or len(payload) != tokens * width * 2):
        raise EnvelopeFailure(INTERNAL, "backend returned an invalid boundary shape")
    for i in range(1, len(payload), 2):                                          # :96-100
        if payload[i] & 0x7C == 0x7C:
            raise EnvelopeFailure(INTERNAL, "backend returned a non-finite boundary activation")
    env = envelope_bytes(                                                        # :74-89, 101-102
        protocol_version=1, deployment_id=identity.deployment_id,
        request_id=identity.request_id, sequence_number=sequence,
        phase=PHASE_PREFILL if (sequence == 0 or prefill) else PHASE_DECODE,
        first_position=position, sequence_lengths=[tokens], cache_slot_ids=[0],
        shape=[1, tokens, width], dtype=DATA_TYPE_F16, layout=LAYOUT,
        payload_length=len(payload), payload=payload,
        deployment_version=identity.deployment_version)
    return stage_message(env)


def validate_tensor_envelope(env: Envelope, phase: int, received: int, maximum_batch: int,
                             maximum_sequence_length: int, hidden_size: int,
                             maximum_payload_bytes: int, protocol_version: int = 1) -> None:
    """tensor_envelope.cpp:26-83 on the metadata decode_tensor builds (its phase
    is the expected one; dtype and layout already matched)."""
    def bad(msg):
        raise EnvelopeFailure(INVALID_REQUEST, msg)
    if env.protocol_version != protocol_version:                                 # :29-31
        bad("unsupported tensor protocol version")
    if not env.deployment_id or env.deployment_version == 0 or not env.request_id:
        bad("tensor envelope is missing deployment or request identity")        # :32-35
    if (maximum_batch == 0 or maximum_sequence_length == 0 or hidden_size == 0
            or maximum_payload_bytes == 0):
        bad("tensor envelope limits are invalid")                                # :36-39
    if len(env.shape) != 3:                                                      # :44-46
        bad("tensor boundary shape must be [batch, sequence, hidden]")
    batch, sequence, hidden = env.shape
    if (batch == 0 or batch > maximum_batch or sequence == 0 or hidden != hidden_size
            or len(env.sequence_lengths) != batch or len(env.cache_slot_ids) != batch):
        bad("tensor boundary dimensions or batch metadata are invalid")          # :51-55
    if phase == PHASE_DECODE and sequence != 1:                                  # :56-58
        bad("decode tensor must have a singleton sequence dimension")
    for length in env.sequence_lengths:                                          # :60-67
        if (length == 0 or length != sequence or env.first_position > maximum_sequence_length
                or length > maximum_sequence_length - env.first_position):
            bad("tensor sequence metadata exceeds configured capacity")
    expected = batch                                                             # :69-71
    for factor in (sequence, hidden, 2):
        if expected != 0 and factor > U64 // expected:
            bad("tensor payload size overflows native size limits")
        expected *= factor
    declared = env.payload_length                                                # :72-77
    if expected != declared or declared != received or declared > maximum_payload_bytes:
        bad("tensor payload length does not match its shape or limits")


def decode_tensor(message: bytes, identity: Identity, sequence: int, position: int,
                  prefill: bool = False) -> Tuple[int, int]:
    """boundary_codec.cpp:15-66 on a serialized StageMessage: returns
    (payload offset in `message`, tokens), or raises EnvelopeFailure."""
    env = parse_stage_message(message)
    if env is None:
        raise EnvelopeFailure(INVALID_REQUEST, "stage message does not carry a tensor")
    if (env.deployment_id != identity.deployment_id                             # :8-13
            or env.deployment_version != identity.deployment_version
            or env.request_id != identity.request_id or env.microbatch_id != 0):
        raise EnvelopeFailure(INVALID_REQUEST,
                              "message identity does not match the active sequence")
    phase = PHASE_PREFILL if (sequence == 0 or prefill) else PHASE_DECODE
    if (env.sequence_number != sequence or env.first_position != position       # :20-27
            or env.phase != phase or env.dtype != DATA_TYPE_F16 or env.layout != LAYOUT
            or env.checksum):
        raise EnvelopeFailure(INVALID_REQUEST,
                              "invalid tensor order, phase, encoding or unsupported checksum")
    validate_tensor_envelope(env, phase, len(env.payload), 1, identity.maximum_tokens,
                             identity.hidden_size, MAXIMUM_RPC_BYTES // 2)       # :43-47
    if len(env.cache_slot_ids) != 1 or env.cache_slot_ids[0] != 0:              # :48-50
        raise EnvelopeFailure(INVALID_REQUEST, "single-sequence execution requires cache slot zero")
    for i in range(0, len(env.payload), 2):                                      # :55-60
        if env.payload[i + 1] & 0x7C == 0x7C:
            raise EnvelopeFailure(INVALID_REQUEST, "non-finite boundary activation")
    return env.payload_offset, env.shape[1]


class SequenceTracker:
    """runtime::SequenceTracker (tensor_envelope.hpp:52-60, tensor_envelope.cpp:85-93)."""

    def __init__(self):
        self.expected = 0

    def accept(self, number: int) -> None:
        if number != self.expected:
            raise EnvelopeFailure(INVALID_REQUEST, "stage message arrived out of order")
        if self.expected == U64:
            raise EnvelopeFailure(INVALID_REQUEST, "stage sequence number exhausted")
        self.expected += 1
