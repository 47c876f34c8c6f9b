"""hLLM's F16 stage boundary on the wire between workers.

Mirrors the reference worker's boundary codec (cpp/include/hllm/worker/boundary_codec.hpp:6-19,
cpp/src/worker/boundary_codec.cpp) and runtime::SequenceTracker
(cpp/include/hllm/runtime/tensor_envelope.hpp:52-60): a boundary activation
travels as a serialized hllm.v1.StageMessage whose `tensor` member is a
TensorEnvelope (proto/execution.proto:48-65).  The bytes are produced and
checked by libhllm_b200 (hllm_b200_envelope_encode / _decode), equal to the
reference worker's; ``B200Stage.encode_boundary`` builds them straight from
the stage's device boundary buffer.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

from . import _lib
from ._lib import StageError, check, lib

__all__ = ["BoundaryIdentity", "MAXIMUM_RPC_BYTES", "SequenceTracker", "decode_tensor",
           "encode_tensor"]

MAXIMUM_RPC_BYTES = 16 * 1024 * 1024  # worker::kMaximumRpcBytes (boundary_codec.hpp:6)


@dataclass
class BoundaryIdentity:
    """worker::BoundaryIdentity (boundary_codec.hpp:7-13)."""
    deployment_id: str
    deployment_version: int
    request_id: str
    maximum_tokens: int
    hidden_size: int

    def c(self) -> _lib.BoundaryIdentity:
        return _lib.BoundaryIdentity(self.deployment_id.encode(), self.deployment_version,
                                     self.request_id.encode(), self.maximum_tokens,
                                     self.hidden_size)


def encode_tensor(hidden, identity: BoundaryIdentity, sequence: int, position: int,
                  prefill: bool = False) -> bytes:
    """worker::encode_tensor (boundary_codec.cpp:68-108): the serialized
    StageMessage carrying `hidden` (a BoundaryActivation) as step `sequence`."""
    payload = bytes(hidden.payload)
    ident = identity.c()
    n = C.c_uint64()
    args = (C.byref(ident), sequence, position, int(prefill), payload, len(payload),
            hidden.tokens, hidden.width)
    check(lib().hllm_b200_envelope_encode(*args, None, 0, C.byref(n)))
    out = C.create_string_buffer(n.value)
    check(lib().hllm_b200_envelope_encode(*args, out, n.value, C.byref(n)))
    return out.raw[:n.value]


def decode_tensor(message: bytes, identity: BoundaryIdentity, sequence: int, position: int,
                  prefill: bool = False):
    """worker::decode_tensor (boundary_codec.cpp:15-66) on a serialized
    StageMessage: the BoundaryActivation it carries, or StageError."""
    from .backend import BoundaryActivation
    message = bytes(message)
    ident = identity.c()
    off, tokens = C.c_uint64(), C.c_uint64()
    check(lib().hllm_b200_envelope_decode(message, len(message), C.byref(ident), sequence,
                                          position, int(prefill), C.byref(off),
                                          C.byref(tokens)))
    n = tokens.value * identity.hidden_size * 2
    return BoundaryActivation(tokens.value, identity.hidden_size,
                              message[off.value:off.value + n])


class SequenceTracker:
    """runtime::SequenceTracker (cpp/src/tensor_envelope.cpp:85-93): stage
    messages of a sequence must arrive numbered 0, 1, 2, ..."""

    def __init__(self):
        self._expected = 0

    @property
    def expected(self) -> int:
        return self._expected

    def accept(self, number: int) -> None:
        if number != self._expected:
            raise StageError(_lib.INVALID_REQUEST, "stage message arrived out of order")
        if self._expected == (1 << 64) - 1:
            raise StageError(_lib.INVALID_REQUEST, "stage sequence number exhausted")
        self._expected += 1
