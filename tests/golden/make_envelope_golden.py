"""Regenerates tests/golden/envelope_cases.json: boundary wire messages made and
parsed by the reference's own generated protobuf code.

Run in a container that has the reference tree (read-only):

    python tests/golden/make_envelope_golden.py /path/to/reference

It imports ``hllm_control.proto.execution_pb2`` from the reference's python/
folder (generated from proto/execution.proto) and records:

* ``encode``: StageMessage{tensor} messages built field by field the way
  ``worker::encode_tensor`` fills them (cpp/src/worker/boundary_codec.cpp:74-102)
  and serialized by execution_pb2 -- the bytes (hex) for small payloads, the
  length and SHA-256 for large ones.  Payloads come from ``payload_for``.
* ``parse``: hand-built byte strings (packed and unpacked repeated fields,
  repeated scalars, unknown fields, split and interleaved oneof members,
  truncations, invalid UTF-8) with what execution_pb2 parses from them: the
  body member, every TensorEnvelope field, or that the bytes do not parse.

Nothing under the reference tree is read at test time.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "envelope_cases.json")
INLINE_LIMIT = 4096  # payload bytes stored inline (hex); larger ones by digest

# (deployment id, version, request id, maximum tokens, hidden, sequence, position,
#  prefill, tokens, seed) -- identities as in the reference tests, long and
# non-ASCII ids, large varints, prefill and decode phases.
ENCODE_CASES = [
    ("plan-1", 1, "request-1", 16, 8, 0, 0, False, 4, 1),
    ("plan-1", 1, "request-1", 16, 8, 1, 4, False, 1, 2),
    ("plan-1", 1, "request-1", 16, 8, 2, 5, True, 3, 3),
    ("deployment-ü-東京", 2, "req-é", 4096, 64, 7, 127, False, 1, 4),
    ("d" * 200, (1 << 40) + 3, "r" * 130, 1 << 20, 16, 128, 300, True, 130, 5),
    ("x", (1 << 64) - 1, "y", 4608, 2560, (1 << 35) + 1, 4095, False, 1, 6),
    ("qwen3-4b-plan", 3, "capture", 4608, 2560, 0, 0, False, 64, 7),
    ("qwen3-4b-plan", 3, "capture", 4608, 2560, 0, 0, True, 512, 8),
]


def payload_for(seed: int, tokens: int, width: int) -> bytes:
    """Seeded finite F16 activations, [tokens][width] little-endian."""
    x = np.random.default_rng(seed).standard_normal(tokens * width) * 4.0
    return x.astype("<f2").tobytes()


def _env_fields(t) -> dict:
    return {
        "protocol_version": t.protocol_version, "deployment_id": t.deployment_id.encode().hex(),
        "request_id": t.request_id.encode().hex(), "microbatch_id": t.microbatch_id,
        "sequence_number": t.sequence_number, "phase": int(t.phase),
        "first_position": t.first_position, "sequence_lengths": list(t.sequence_lengths),
        "cache_slot_ids": list(t.cache_slot_ids), "shape": list(t.shape),
        "dtype": int(t.dtype), "layout": t.layout.encode().hex(),
        "payload_length": t.payload_length, "checksum": t.checksum.hex(),
        "payload": t.payload.hex(), "deployment_version": t.deployment_version,
    }


def _varint(v: int) -> bytes:
    out = bytearray()
    while True:
        b = v & 0x7F
        v >>= 7
        out.append(b | (0x80 if v else 0))
        if not v:
            return bytes(out)


def _key(field, wire):
    return _varint((field << 3) | wire)


def _ld(field, data):
    return _key(field, 2) + _varint(len(data)) + data


def _parse_inputs(pb):
    """Byte strings whose parse by execution_pb2 is recorded."""
    good = pb.StageMessage()
    t = good.tensor
    t.protocol_version = 1
    t.deployment_id = "plan-1"
    t.deployment_version = 1
    t.request_id = "request-1"
    t.sequence_number = 2
    t.phase = pb.EXECUTION_PHASE_DECODE
    t.first_position = 9
    t.sequence_lengths.append(1)
    t.cache_slot_ids.append(0)
    t.shape.extend([1, 1, 8])
    t.dtype = 10
    t.layout = "dense_row_major_le"
    t.payload = payload_for(11, 1, 8)
    t.payload_length = len(t.payload)
    base = good.SerializeToString()
    env = t.SerializeToString()
    cases = {"valid": base}
    # repeated scalars written unpacked, and packed fields split in two
    unpacked = (_key(1, 0) + b"\x01" + _ld(2, b"plan-1") + _ld(3, b"request-1")
                + _key(5, 0) + b"\x02" + _key(6, 0) + b"\x02" + _key(7, 0) + b"\x09"
                + _key(8, 0) + b"\x01" + _key(9, 0) + b"\x00"
                + _key(10, 0) + b"\x01" + _ld(10, b"\x01\x08")
                + _key(11, 0) + b"\x0a" + _ld(12, b"dense_row_major_le")
                + _key(13, 0) + b"\x10" + _ld(15, payload_for(11, 1, 8)) + _key(16, 0) + b"\x01")
    cases["unpacked_and_split_repeated"] = _ld(2, unpacked)
    # scalars repeated (last wins), fields out of order, unknown fields of every wire type
    extra = (_key(5, 0) + b"\x07" + _key(99, 0) + b"\x05" + _key(98, 1) + b"\x00" * 8
             + _key(97, 5) + b"\x00" * 4 + _ld(96, b"abc") + _key(5, 0) + b"\x02"
             + _key(1, 2) + b"\x00")  # field 1 with the wrong wire type: unknown
    cases["repeated_scalars_unknown_fields"] = _ld(2, extra + env)
    # the tensor member split in two (merged), and top-level unknown fields
    a = pb.TensorEnvelope()
    a.CopyFrom(t)
    a.ClearField("payload")
    b = pb.TensorEnvelope()
    b.payload = t.payload
    cases["tensor_member_merged"] = (_ld(2, a.SerializeToString()) + _key(77, 0) + b"\x01"
                                     + _ld(2, b.SerializeToString()))
    # another oneof member after the tensor, and a tensor after another member
    cases["other_member_last"] = base + _ld(1, b"")
    cases["tensor_after_other_member"] = _ld(6, b"") + base
    cases["tensor_then_other_then_tensor"] = (_ld(2, a.SerializeToString()) + _ld(3, b"")
                                              + _ld(2, b.SerializeToString()))
    cases["empty_message"] = b""
    cases["empty_tensor"] = _ld(2, b"")
    # large varints, enum values outside the enum, a negative enum
    big = (_key(1, 0) + _varint(5_000_000_000) + _key(6, 0) + _varint(7)
           + _key(11, 0) + _varint((1 << 64) - 1) + _key(7, 0) + _varint((1 << 64) - 1))
    cases["wide_varints_and_open_enums"] = _ld(2, big)
    # bytes that do not parse
    cases["truncated_length"] = base[:-3]
    cases["truncated_varint"] = _ld(2, _key(5, 0) + b"\xff")
    cases["length_beyond_end"] = b"\x12\x7f\x08\x01"
    cases["field_zero"] = _ld(2, b"\x00\x01")
    cases["invalid_utf8_string"] = _ld(2, _ld(2, b"\xff\xfe"))
    cases["invalid_utf8_layout"] = _ld(2, _ld(12, b"dense\xc3"))
    cases["overlong_varint"] = _ld(2, _key(5, 0) + b"\xff" * 10 + b"\x01")
    cases["tenth_varint_byte_wraps"] = _ld(2, _key(5, 0) + b"\xff" * 9 + b"\x02")
    cases["tag_beyond_32_bits"] = _ld(2, _varint(1 << 32) + b"\x01")
    cases["wire_type_6"] = _ld(2, _key(20, 6))
    cases["wire_type_7"] = _ld(2, _key(20, 7))
    # unknown groups are skipped (nested, with fields inside, at the top level,
    # and a known field number written as a group)
    cases["nested_groups"] = _ld(2, _key(20, 3) + _key(21, 3) + _key(21, 4) + _key(20, 4)
                                 + _key(5, 0) + b"\x03")
    cases["group_with_fields"] = _ld(2, _key(20, 3) + _key(5, 0) + b"\x09" + _ld(6, b"xy")
                                     + _key(20, 4) + _key(5, 0) + b"\x03")
    cases["top_level_group"] = _key(20, 3) + _key(20, 4) + _ld(2, _key(5, 0) + b"\x04")
    cases["known_field_as_group"] = _ld(2, _key(5, 3) + _key(5, 4) + _key(7, 0) + b"\x01")
    cases["end_group_alone"] = _ld(2, _key(20, 4))
    cases["group_end_mismatch"] = _ld(2, _key(20, 3) + _key(21, 4))
    cases["unterminated_group"] = _ld(2, _key(20, 3))
    cases["packed_truncated"] = _ld(2, _ld(8, b"\xff"))
    cases["packed_empty"] = _ld(2, _ld(8, b"") + _key(5, 0) + b"\x01")
    cases["uint32_and_enum_truncation"] = _ld(2, _key(1, 0) + _varint((1 << 32) + 5)
                                              + _key(6, 0) + _varint((1 << 32) + 1))
    cases["negative_enum"] = _ld(2, _key(11, 0) + _varint((1 << 64) - 3))
    cases["wrong_wire_types_are_unknown"] = _ld(2, _key(2, 0) + b"\x05" + _ld(6, b"\x01")
                                                + _key(5, 0) + b"\x06")
    cases["member_as_varint"] = _key(2, 0) + b"\x01"
    cases["fixed64_truncated"] = _ld(2, _key(30, 1) + b"\x00" * 3)
    return cases


def main(ref_root: str) -> None:
    sys.path.insert(0, os.path.join(ref_root, "python"))
    from hllm_control.proto import execution_pb2 as pb

    out = {"encode": [], "parse": []}
    for dep, ver, req, max_tok, hidden, seq, pos, prefill, tokens, seed in ENCODE_CASES:
        payload = payload_for(seed, tokens, hidden)
        m = pb.StageMessage()
        t = m.tensor
        t.protocol_version = 1
        t.deployment_id = dep
        t.deployment_version = ver
        t.request_id = req
        t.sequence_number = seq
        t.phase = (pb.EXECUTION_PHASE_PREFILL if (seq == 0 or prefill)
                   else pb.EXECUTION_PHASE_DECODE)
        t.first_position = pos
        t.sequence_lengths.append(tokens)
        t.cache_slot_ids.append(0)
        t.shape.extend([1, tokens, hidden])
        t.dtype = pb.DATA_TYPE_F16 if hasattr(pb, "DATA_TYPE_F16") else 10
        t.layout = "dense_row_major_le"
        t.payload = payload
        t.payload_length = len(payload)
        wire = m.SerializeToString()
        case = {"deployment_id": dep.encode().hex(), "deployment_version": ver,
                "request_id": req.encode().hex(), "maximum_tokens": max_tok, "hidden": hidden,
                "sequence": seq, "position": pos, "prefill": prefill, "tokens": tokens,
                "seed": seed, "bytes": len(wire), "sha256": hashlib.sha256(wire).hexdigest()}
        if len(payload) <= INLINE_LIMIT:
            case["message"] = wire.hex()
        out["encode"].append(case)
    for name, data in _parse_inputs(pb).items():
        rec = {"name": name, "message": data.hex()}
        try:
            m = pb.StageMessage.FromString(data)
            body = m.WhichOneof("body")
            rec["parses"] = True
            rec["body"] = body
            if body == "tensor":
                rec["tensor"] = _env_fields(m.tensor)
        except Exception as e:  # google.protobuf.message.DecodeError and friends
            rec["parses"] = False
            rec["error"] = type(e).__name__
        out["parse"].append(rec)
    with open(OUT, "w") as f:
        json.dump(out, f, indent=1)
    print(f"wrote {OUT}: {len(out['encode'])} encode cases, {len(out['parse'])} parse cases")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_envelope_golden.py <reference tree>")
    main(sys.argv[1])
