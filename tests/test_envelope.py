"""The F16 boundary wire codec between workers, on the CPU.

Pins, in order:
* the CPU restatement (oracle/envelope.py) against messages serialized and
  parsed by the reference's own generated protobuf code
  (tests/golden/envelope_cases.json, made by make_envelope_golden.py) and
  against the reference's validate_tensor_envelope / SequenceTracker compiled
  from its sources into oracle/_ref;
* the product codec in libhllm_b200 (hllm_b200_envelope_encode / _decode,
  through hllm_b200.wire) against the golden bytes and against the
  restatement: equal bytes, and for every input the same status, message,
  payload offset and token count -- on the reference's own test cases
  (tests/cpp/tensor_envelope_test.cpp), on every single-field change of a
  valid message, and on seeded truncations and byte flips.
No GPU is needed: the codec is host code.
"""
import ctypes as C
import hashlib
import json
import os
import random
import struct

import numpy as np
import pytest

import oracle
from oracle import envelope as O
from hllm_b200 import _lib
from hllm_b200.backend import BoundaryActivation, StageError
from hllm_b200.wire import BoundaryIdentity, SequenceTracker, decode_tensor, encode_tensor
from tests.golden.make_envelope_golden import payload_for

GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "envelope_cases.json")))


def _oid(c) -> O.Identity:
    return O.Identity(bytes.fromhex(c["deployment_id"]), c["deployment_version"],
                      bytes.fromhex(c["request_id"]), c["maximum_tokens"], c["hidden"])


def _pid(i: O.Identity) -> BoundaryIdentity:
    return BoundaryIdentity(i.deployment_id.decode(), i.deployment_version, i.request_id.decode(),
                            i.maximum_tokens, i.hidden_size)


# ----------------------------------------------------------------------------- pinning
def test_oracle_encoding_equals_reference_protobuf_bytes():
    for c in GOLD["encode"]:
        payload = payload_for(c["seed"], c["tokens"], c["hidden"])
        got = O.encode_tensor(payload, c["tokens"], c["hidden"], _oid(c), c["sequence"],
                              c["position"], c["prefill"])
        assert len(got) == c["bytes"]
        assert hashlib.sha256(got).hexdigest() == c["sha256"]
        if "message" in c:
            assert got.hex() == c["message"]


def test_oracle_parse_equals_reference_protobuf_parse():
    for rec in GOLD["parse"]:
        msg = bytes.fromhex(rec["message"])
        if not rec["parses"]:
            with pytest.raises(O.EnvelopeFailure) as e:
                O.parse_stage_message(msg)
            assert e.value.message == "malformed stage message", rec["name"]
            continue
        env = O.parse_stage_message(msg)
        if rec["body"] != "tensor":
            assert env is None, rec["name"]
            continue
        t = rec["tensor"]
        assert env is not None, rec["name"]
        for k in ("protocol_version", "microbatch_id", "sequence_number", "phase",
                  "first_position", "sequence_lengths", "cache_slot_ids", "shape", "dtype",
                  "payload_length", "deployment_version"):
            assert getattr(env, k) == t[k], (rec["name"], k)
        for k in ("deployment_id", "request_id", "layout", "checksum", "payload"):
            assert getattr(env, k).hex() == t[k], (rec["name"], k)
        if env.payload:
            assert msg[env.payload_offset:env.payload_offset + len(env.payload)] == env.payload


def _ref():
    r = oracle.ref()
    if r is None or not hasattr(r, "ref_validate_envelope"):
        pytest.skip("oracle/_ref not built from the reference sources")
    r.ref_validate_envelope.restype = C.c_int
    return r


def _ref_validate(r, env: O.Envelope, phase, received, limits):
    def arr(v):
        return (C.c_uint64 * max(1, len(v)))(*v), len(v)
    lengths, nl = arr(env.sequence_lengths)
    slots, ns = arr(env.cache_slot_ids)
    shape, nsh = arr(env.shape)
    msg = C.create_string_buffer(256)
    st = r.ref_validate_envelope(
        C.c_uint32(env.protocol_version), env.deployment_id, C.c_uint64(env.deployment_version),
        env.request_id, C.c_uint64(env.microbatch_id), C.c_uint64(env.sequence_number),
        C.c_uint32(1 if phase == O.PHASE_DECODE else 0), C.c_uint64(env.first_position),
        lengths, C.c_uint64(nl), slots, C.c_uint64(ns), shape, C.c_uint64(nsh),
        C.c_uint64(env.payload_length), C.c_uint64(received), C.c_uint64(limits[0]),
        C.c_uint64(limits[1]), C.c_uint64(limits[2]), C.c_uint64(limits[3]), msg,
        C.c_uint64(256))
    return st, msg.value.decode()


def _oracle_validate(env, phase, received, limits):
    try:
        O.validate_tensor_envelope(env, phase, received, *limits)
        return 0, ""
    except O.EnvelopeFailure as e:
        return e.status, e.message


def _metadata(**kw) -> O.Envelope:
    """tests/cpp/tensor_envelope_test.cpp:10-27's valid envelope, with changes."""
    e = O.Envelope()
    e.protocol_version, e.deployment_id, e.deployment_version = 1, b"plan-1", 1
    e.request_id, e.microbatch_id, e.sequence_number = b"request-1", 0, 0
    e.first_position, e.sequence_lengths, e.cache_slot_ids = 0, [4], [0]
    e.shape, e.payload_length = [1, 4, 8], 64
    for k, v in kw.items():
        setattr(e, k, v)
    return e


LIMITS = (1, 16, 8, 256)  # tensor_envelope_test.cpp:29-36: batch, sequence, hidden, payload


def test_oracle_validation_equals_reference_validate_tensor_envelope():
    r = _ref()
    cases = [  # the reference's own tests first
        (_metadata(), O.PHASE_PREFILL, 64, LIMITS, 0),
        (_metadata(payload_length=63), O.PHASE_PREFILL, 63, LIMITS, 1),
        (_metadata(), O.PHASE_DECODE, 64, LIMITS, 1),
        (_metadata(first_position=20), O.PHASE_PREFILL, 64, LIMITS, 1),
    ]
    rng = random.Random(7)
    fields = [("protocol_version", [0, 1, 2]), ("deployment_id", [b"", b"plan-1"]),
              ("deployment_version", [0, 1, 1 << 63]), ("request_id", [b"", b"r"]),
              ("first_position", [0, 1, 12, 15, 16, 17, (1 << 64) - 1]),
              ("sequence_lengths", [[], [4], [1], [0], [4, 4], [5]]),
              ("cache_slot_ids", [[], [0], [3], [0, 0]]),
              ("shape", [[], [1, 4], [1, 4, 8], [2, 4, 8], [0, 4, 8], [1, 0, 8], [1, 4, 7],
                         [1, 1, 8], [1, (1 << 62), 8], [1, 4, 8, 1]]),
              ("payload_length", [0, 16, 63, 64, 65, 512, (1 << 64) - 1])]
    for _ in range(400):
        kw = {k: rng.choice(v) for k, v in rng.sample(fields, rng.randint(1, 4))}
        phase = rng.choice([O.PHASE_PREFILL, O.PHASE_DECODE])
        received = rng.choice([0, 16, 63, 64, 512])
        limits = rng.choice([LIMITS, (1, 4, 8, 64), (1, 16, 8, 32), (0, 16, 8, 256),
                             (1, 0, 8, 256), (1, 16, 0, 256), (1, 16, 8, 0), (2, 16, 8, 256)])
        cases.append((_metadata(**kw), phase, received, limits, None))
    for env, phase, received, limits, want in cases:
        got_ref = _ref_validate(r, env, phase, received, limits)
        got = _oracle_validate(env, phase, received, limits)
        assert got == got_ref, (vars(env), phase, received, limits)
        if want is not None:
            assert got[0] == want


def test_sequence_tracker_equals_reference():
    r = _ref()
    r.ref_sequence_tracker.restype = C.c_uint64
    for seq in ([0, 1, 2], [0, 1, 3, 4], [1], [0, 0], [], list(range(50)) + [49]):
        arr = (C.c_uint64 * max(1, len(seq)))(*seq)
        accepted = r.ref_sequence_tracker(arr, C.c_uint64(len(seq)))
        for tracker in (O.SequenceTracker(), SequenceTracker()):
            n = 0
            for x in seq:
                try:
                    tracker.accept(x)
                except (O.EnvelopeFailure, StageError):
                    break
                n += 1
            assert n == accepted, seq


# ----------------------------------------------------------------------------- product
def test_product_encoding_equals_reference_protobuf_bytes():
    for c in GOLD["encode"]:
        payload = payload_for(c["seed"], c["tokens"], c["hidden"])
        got = encode_tensor(BoundaryActivation(c["tokens"], c["hidden"], payload),
                            _pid(_oid(c)), c["sequence"], c["position"], c["prefill"])
        assert hashlib.sha256(got).hexdigest() == c["sha256"]
        back = decode_tensor(got, _pid(_oid(c)), c["sequence"], c["position"], c["prefill"])
        assert (back.tokens, back.width, back.payload) == (c["tokens"], c["hidden"], payload)


def _product_encode(payload, tokens, width, ident: O.Identity, seq, pos, prefill):
    try:
        return 0, encode_tensor(BoundaryActivation(tokens, width, payload), _pid(ident), seq, pos,
                                prefill)
    except StageError as e:
        return e.code, e.message


def _oracle_encode(payload, tokens, width, ident, seq, pos, prefill):
    try:
        return 0, O.encode_tensor(payload, tokens, width, ident, seq, pos, prefill)
    except O.EnvelopeFailure as e:
        return e.status, e.message


def test_product_encoding_equals_restatement_including_errors():
    rng = random.Random(11)
    f16 = lambda n, s: payload_for(s, 1, n)  # noqa: E731
    cases = []
    for k in range(300):
        width = rng.choice([1, 8, 64, 2560, 3072])
        tokens = rng.choice([1, 2, 7, 64, 300, 1638, 1639])
        ident = O.Identity(rng.choice([b"", b"p", b"plan-\xc3\xbc" * rng.randint(1, 40)]),
                           rng.choice([0, 1, 127, 128, (1 << 64) - 1]),
                           rng.choice([b"", b"r", b"req" * 50]), 4096,
                           rng.choice([width, width, width + 1]))
        n = tokens * width
        if n * 2 > 9 * (1 << 20):
            payload = bytes(n * 2)
        else:
            payload = f16(n, k)
        if rng.random() < 0.1:
            payload = payload[:-2]  # size disagrees with the shape
        if rng.random() < 0.1 and len(payload) >= 2:
            j = rng.randrange(len(payload) // 2)
            payload = payload[:2 * j] + rng.choice([b"\x00\x7c", b"\x00\xfc", b"\x01\x7e"]) \
                + payload[2 * j + 2:]
        cases.append((payload, tokens, width, ident, rng.choice([0, 1, 300, 1 << 40]),
                      rng.choice([0, 1, 4095, 1 << 33]), rng.random() < 0.5))
    cases.append((bytes(8 * 1024 * 1024 + 2), 1, 4 * 1024 * 1024 + 1,
                  O.Identity(b"p", 1, b"r", 1, 4 * 1024 * 1024 + 1), 0, 0, False))
    cases.append((b"", 0, 8, O.Identity(b"p", 1, b"r", 16, 8), 0, 0, False))
    statuses = set()
    for c in cases:
        got, want = _product_encode(*c), _oracle_encode(*c)
        assert got == want, (c[1:3], c[3], c[4:], got[1] if got[0] else len(got[1]))
        statuses.add(got[0])
    assert statuses == {0, O.RESOURCE_EXHAUSTED, O.INTERNAL}


def _decode_both(msg, ident, seq, pos, prefill):
    try:
        want = (0,) + O.decode_tensor(msg, ident, seq, pos, prefill)
    except O.EnvelopeFailure as e:
        want = (e.status, e.message)
    c_ident = _pid(ident).c()
    off, tok = C.c_uint64(), C.c_uint64()
    st = _lib.lib().hllm_b200_envelope_decode(msg, len(msg), C.byref(c_ident), seq, pos,
                                              int(prefill), C.byref(off), C.byref(tok))
    got = (0, off.value, tok.value) if st == 0 else (st, _lib.last_error())
    return got, want


def _valid(ident: O.Identity, seq=2, pos=9, tokens=1, prefill=False, seed=3, **kw):
    args = dict(protocol_version=1, deployment_id=ident.deployment_id,
                request_id=ident.request_id, sequence_number=seq,
                phase=O.PHASE_PREFILL if (seq == 0 or prefill) else O.PHASE_DECODE,
                first_position=pos, sequence_lengths=[tokens], cache_slot_ids=[0],
                shape=[1, tokens, ident.hidden_size], dtype=O.DATA_TYPE_F16, layout=O.LAYOUT,
                payload=payload_for(seed, tokens, ident.hidden_size),
                deployment_version=ident.deployment_version)
    args["payload_length"] = len(args["payload"])
    args.update(kw)
    return O.stage_message(O.envelope_bytes(**args))


def test_reference_envelope_tests_through_the_product_decoder():
    """tests/cpp/tensor_envelope_test.cpp:38-58 as wire messages."""
    ident = O.Identity(b"plan-1", 1, b"request-1", 16, 8)
    ok = _valid(ident, seq=0, pos=0, tokens=4)
    got, want = _decode_both(ok, ident, 0, 0, False)
    assert got == want and got[0] == 0 and got[2] == 4
    short = _valid(ident, seq=0, pos=0, tokens=4, payload_length=63)
    got, want = _decode_both(short, ident, 0, 0, False)
    assert got == want == (1, "tensor payload length does not match its shape or limits")
    multi = _valid(ident, seq=1, pos=0, tokens=4)
    got, want = _decode_both(multi, ident, 1, 0, False)
    assert got == want == (1, "decode tensor must have a singleton sequence dimension")
    beyond = _valid(ident, seq=0, pos=20, tokens=4)
    got, want = _decode_both(beyond, ident, 0, 20, False)
    assert got == want == (1, "tensor sequence metadata exceeds configured capacity")


MUTATIONS = {
    "protocol_version": [0, 2, (1 << 32) + 1], "deployment_id": [b"", b"plan-2", b"plan-1x"],
    "request_id": [b"", b"request-2"], "microbatch_id": [1], "sequence_number": [0, 1, 3],
    "phase": [0, 1, 2, 3, -1], "first_position": [0, 8, 10, 4096, (1 << 64) - 1],
    "sequence_lengths": [[], [0], [2], [1, 1]], "cache_slot_ids": [[], [1], [0, 0]],
    "shape": [[], [1, 1], [1, 1, 8, 1], [0, 1, 8], [2, 1, 8], [1, 0, 8], [1, 2, 8], [1, 1, 9],
              [1, 1, 7], [1, (1 << 63), 8]],
    "dtype": [0, 9, 11, -1], "layout": [b"", b"dense_row_major_be", b"Dense_row_major_le"],
    "payload_length": [0, 15, 17, 1 << 40], "checksum": [b"\x00", b"sha"],
    "payload": [b"", b"\x00" * 15, b"\x00" * 18, b"\x00\x3c" * 7 + b"\x00\x7c",
                b"\x00\x3c" * 7 + b"\xff\xff", b"\x00\x3c" * 7 + b"\x00\xfc"],
    "deployment_version": [0, 2, (1 << 64) - 1],
}


def test_product_decoder_equals_restatement_on_field_changes():
    ident = O.Identity(b"plan-1", 1, b"request-1", 16, 8)
    n = 0
    for field, values in MUTATIONS.items():
        for v in values:
            for seq, pos, prefill in ((2, 9, False), (2, 9, True), (0, 9, False)):
                msg = _valid(ident, seq=seq, pos=pos, prefill=prefill, **{field: v})
                for expect in ((seq, pos, prefill), (seq + 1, pos, prefill), (seq, pos, not prefill)):
                    got, want = _decode_both(msg, ident, *expect)
                    assert got == want, (field, v, seq, pos, prefill, expect)
                    n += 1
    # identities with other limits and widths
    for ident2 in (O.Identity(b"plan-1", 1, b"request-1", 9, 8),
                   O.Identity(b"plan-1", 1, b"request-1", 10, 8),
                   O.Identity(b"plan-1", 1, b"request-1", 0, 8),
                   O.Identity(b"plan-1", 1, b"request-1", 16, 0),
                   O.Identity(b"plan-1", 0, b"request-1", 16, 8),
                   O.Identity(b"", 1, b"request-1", 16, 8)):
        msg = _valid(O.Identity(ident2.deployment_id, ident2.deployment_version, ident2.request_id,
                                16, 8))
        got, want = _decode_both(msg, ident2, 2, 9, False)
        assert got == want, vars(ident2)
    assert n > 300


def test_product_decoder_equals_restatement_on_parse_cases_and_fuzz():
    ident = O.Identity(b"plan-1", 1, b"request-1", 4608, 8)
    msgs = [bytes.fromhex(r["message"]) for r in GOLD["parse"]]
    rng = random.Random(5)
    base = _valid(ident)
    for _ in range(1500):
        m = bytearray(rng.choice(msgs + [base] * 4))
        op = rng.random()
        if op < 0.3 and m:
            del m[rng.randrange(len(m)):]
        elif op < 0.7 and m:
            for _ in range(rng.randint(1, 3)):
                m[rng.randrange(len(m))] = rng.randrange(256)
        elif op < 0.85:
            m += bytes(rng.randrange(256) for _ in range(rng.randint(1, 6)))
        else:
            j = rng.randrange(len(m) + 1)
            m[j:j] = bytes(rng.randrange(256) for _ in range(rng.randint(1, 4)))
        msgs.append(bytes(m))
    outcomes = set()
    for m in msgs:
        for seq, pos in ((2, 9), (0, 0)):
            got, want = _decode_both(m, ident, seq, pos, False)
            assert got == want, m.hex()
            outcomes.add(got[1] if got[0] else "ok")
    assert "ok" in outcomes and "malformed stage message" in outcomes
    assert len(outcomes) >= 4


def test_wire_mirror_round_trip_and_errors():
    ident = BoundaryIdentity("plan-1", 1, "request-1", 4608, 64)
    x = (np.random.default_rng(0).standard_normal((5, 64)) * 3).astype("<f2")
    act = BoundaryActivation(5, 64, x.tobytes())
    msg = encode_tensor(act, ident, 0, 0)
    back = decode_tensor(msg, ident, 0, 0)
    assert (back.tokens, back.width, back.payload) == (5, 64, x.tobytes())
    with pytest.raises(StageError) as e:
        decode_tensor(msg, ident, 1, 0)
    assert e.value.code == _lib.INVALID_REQUEST
    bad = x.copy()
    bad[2, 3] = np.inf
    with pytest.raises(StageError) as e:
        encode_tensor(BoundaryActivation(5, 64, bad.tobytes()), ident, 0, 0)
    assert e.value.code == _lib.INTERNAL
    assert e.value.message == "backend returned a non-finite boundary activation"
    with pytest.raises(StageError) as e:
        encode_tensor(BoundaryActivation(1, 4 * 1024 * 1024 + 1, bytes(8 * 1024 * 1024 + 2)),
                      BoundaryIdentity("p", 1, "r", 4, 4 * 1024 * 1024 + 1), 0, 0)
    assert e.value.code == _lib.RESOURCE_EXHAUSTED
    # a StageMessage whose body is another member
    with pytest.raises(StageError) as e:
        decode_tensor(b"\x0a\x00", ident, 0, 0)
    assert e.value.message == "stage message does not carry a tensor"
    t = SequenceTracker()
    t.accept(0)
    t.accept(1)
    assert t.expected == 2
    with pytest.raises(StageError):
        t.accept(3)
    assert t.expected == 2


def test_decode_locates_the_payload_in_place():
    ident = BoundaryIdentity("plan-1", 7, "r", 4608, 2560)
    x = (np.random.default_rng(1).standard_normal((3, 2560))).astype("<f2")
    msg = encode_tensor(BoundaryActivation(3, 2560, x.tobytes()), ident, 4, 100, prefill=True)
    c_ident = ident.c()
    off, tok = C.c_uint64(), C.c_uint64()
    _lib.check(_lib.lib().hllm_b200_envelope_decode(msg, len(msg), C.byref(c_ident), 4, 100, 1,
                                                    C.byref(off), C.byref(tok)))
    assert tok.value == 3
    assert msg[off.value:off.value + x.nbytes] == x.tobytes()
    assert struct.unpack_from("<e", msg, off.value)[0] == float(x[0, 0])
