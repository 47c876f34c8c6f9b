"""Host-side mirror of hLLM's StageBackend over the B200 C ABI.

Mirrors ``runtime::StageBackend`` (cpp/include/hllm/runtime/stage_backend.hpp:69-107)
method for method -- ``weight_memory``, ``hidden_size``, ``vocabulary_size``,
``maximum_tokens``, ``sequence_memory``, ``allocate_sequence``, ``execute``,
``supports_decode_batch``, ``execute_decode_batch`` -- with the same argument
meaning and error behaviour, plus ``execute_mixed_batch`` (one pass over
prefill chunks and decode tokens together, which the reference scheduler never
forms).  Every computation runs in libhllm_b200.so on the GPU.
"""
from __future__ import annotations

import ctypes as C
import itertools
import threading
from dataclasses import dataclass, field
from typing import Optional, Sequence, Union

import numpy as np

from . import _lib
from ._lib import StageError, check, lib

__all__ = ["ModelConfig", "TokenInput", "BoundaryActivation", "PrefillProgress", "SampledToken",
           "SamplingOptions", "SequenceState", "DecodeBatchItem", "B200Stage", "StageError"]


@dataclass(frozen=True)
class ModelConfig:
    """model::DenseConfig (cpp/include/hllm/model/dense_source.hpp:15-25) + vocabulary."""
    hidden_size: int
    intermediate_size: int
    attention_heads: int
    key_value_heads: int
    head_dimension: int
    maximum_sequence_length: int
    rms_norm_epsilon: float
    rope_theta: float
    query_key_norm: bool
    vocabulary_size: int
    layers: int
    tied: bool


@dataclass
class TokenInput:
    ids: list


@dataclass
class BoundaryActivation:
    """Row-major little-endian F16 [tokens, width] (stage_backend.hpp:18-24)."""
    tokens: int
    width: int
    payload: bytes


class PrefillProgress:
    def __eq__(self, other):
        return isinstance(other, PrefillProgress)


@dataclass
class SampledToken:
    id: int
    logprob: Optional[float] = None
    top_logprobs: list = field(default_factory=list)


@dataclass
class SamplingOptions:
    temperature: float = 0.0
    top_p: float = 1.0
    top_k: int = 0
    seed: int = 0
    return_logprobs: bool = False
    top_logprobs: int = 0


def _dtype_of(ctype):
    """numpy dtype with the memory layout of a ctypes scalar, pointer or
    Structure (field offsets and size taken from the ctypes mirror)."""
    if isinstance(ctype, type) and issubclass(ctype, C.Structure):
        names = [f for f, _ in ctype._fields_]
        return np.dtype({"names": names,
                         "formats": [_dtype_of(t) for _, t in ctype._fields_],
                         "offsets": [getattr(ctype, f).offset for f in names],
                         "itemsize": C.sizeof(ctype)})
    if ctype is C.c_void_p or (isinstance(ctype, type) and issubclass(ctype, C._Pointer)):
        return np.dtype(np.uintp)
    return np.dtype(ctype)


_ROW = _dtype_of(_lib.Row)
_SAMPLING = _dtype_of(_lib.Sampling)
_SAMPLED = _dtype_of(_lib.Sampled)


@dataclass
class SequenceState:
    """runtime::SequenceState (stage_backend.hpp:44-50) plus the device handle."""
    handle: int
    capacity: int
    sampling: SamplingOptions = field(default_factory=SamplingOptions)
    prefilling: bool = False
    prefill_only: bool = False
    generated_index: int = 0
    owner: object = None


@dataclass
class DecodeBatchItem:
    input: Union[TokenInput, BoundaryActivation]
    position: int
    sequence: SequenceState
    cancelled: object = None  # threading.Event, a callable, or None


StageInput = Union[TokenInput, BoundaryActivation]


def _is_cancelled(flag) -> bool:
    if flag is None:
        return False
    if isinstance(flag, threading.Event):
        return flag.is_set()
    if callable(flag):
        return bool(flag())
    return bool(flag)


class B200Stage:
    """One hLLM stage (contiguous layer range) on one B200."""

    def __init__(self, config: ModelConfig, layer_start: int = 0, layer_end: Optional[int] = None,
                 first: bool = True, final: bool = True, device: int = 0,
                 kv_pool_tokens: int = 1 << 16, max_step_tokens: int = 2048,
                 max_step_rows: int = 256, max_sequences: int = 512):
        self.config = config
        self.layer_start = layer_start
        self.layer_end = config.layers if layer_end is None else layer_end
        self.first = first
        self.final = final
        d = _lib.StageDesc(
            config.hidden_size, config.intermediate_size, config.attention_heads,
            config.key_value_heads, config.head_dimension, config.maximum_sequence_length,
            config.rms_norm_epsilon, config.rope_theta, int(config.query_key_norm),
            config.vocabulary_size, layer_start, self.layer_end, int(first), int(final),
            int(config.tied), device, kv_pool_tokens, max_step_tokens, max_step_rows,
            max_sequences)
        handle = C.c_void_p()
        check(lib().hllm_b200_stage_create(C.byref(d), C.byref(handle)))
        self._h = handle
        self._lock = threading.Lock()

    # ------------------------------------------------------------ lifetime
    def encode_boundary(self, first_token: int, tokens: int, identity, sequence: int,
                        position: int, prefill: bool = False) -> bytes:
        """The serialized StageMessage (worker::encode_tensor,
        cpp/src/worker/boundary_codec.cpp:68-108) of boundary rows
        [first_token, first_token + tokens) of this non-final stage's last
        step, built from device memory (hllm_b200_stage_envelope, then
        hllm_b200_stage_envelope_wait).  `identity` is a wire.BoundaryIdentity."""
        ident = identity.c()
        n = C.c_uint64()
        args = (self._h, first_token, tokens, C.byref(ident), sequence, position, int(prefill))
        with self._lock:
            check(lib().hllm_b200_stage_envelope(*args, None, 0, C.byref(n)))
            out = C.create_string_buffer(n.value)
            check(lib().hllm_b200_stage_envelope(*args, out, n.value, C.byref(n)))
            check(lib().hllm_b200_stage_envelope_wait(self._h))
        return out.raw[:n.value]

    def memory(self) -> dict:
        """Device bytes (hllm_b200_stage_memory): weights, workspace, kv_pool,
        kv_in_use, kv_peak -- what BackendFactory::allocator_metrics reports."""
        v = [C.c_uint64() for _ in range(5)]
        check(lib().hllm_b200_stage_memory(self._h, *[C.byref(x) for x in v]))
        return dict(zip(("weights", "workspace", "kv_pool", "kv_in_use", "kv_peak"),
                        (x.value for x in v)))

    def encode_boundaries(self, rows) -> list:
        """Envelopes of several row ranges of the last step's boundary at once
        (hllm_b200_stage_envelopes, one device->host copy): `rows` holds
        (first_token, tokens, identity, sequence, position, prefill) tuples;
        returns one serialized StageMessage per row range, in order."""
        n = len(rows)
        arr = (_lib.EnvelopeRow * max(1, n))()
        keep = []
        for i, (first, tokens, identity, sequence, position, prefill) in enumerate(rows):
            ident = identity.c()
            keep.append(ident)
            arr[i] = _lib.EnvelopeRow(first, tokens, ident, sequence, position, int(prefill))
        offsets = (C.c_uint64 * (n + 1))()
        with self._lock:
            check(lib().hllm_b200_stage_envelopes(self._h, arr, n, None, 0, offsets))
            out = C.create_string_buffer(max(1, offsets[n]))
            check(lib().hllm_b200_stage_envelopes(self._h, arr, n, out, offsets[n], offsets))
            check(lib().hllm_b200_stage_envelope_wait(self._h))
        raw = out.raw
        return [raw[offsets[i]:offsets[i + 1]] for i in range(n)]

    def close(self):
        if self._h:
            lib().hllm_b200_stage_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def handle(self):
        return self._h

    def load_tensor(self, name: str, array: np.ndarray) -> None:
        a = np.ascontiguousarray(array)
        if a.dtype == np.float32:
            dt = _lib.F32
        elif a.dtype == np.float16:
            dt = _lib.F16
            a = a.view(np.uint16)
        elif a.dtype == np.uint16:
            dt = _lib.F16
        else:
            raise StageError(_lib.INCOMPATIBLE_WORKER, f"unsupported dtype {a.dtype}")
        shape = (C.c_uint64 * a.ndim)(*a.shape)
        check(lib().hllm_b200_stage_load_tensor(self._h, name.encode(), dt,
                                                a.ctypes.data_as(C.c_void_p), shape, a.ndim))

    def load_weights(self, weights: dict) -> None:
        """Loads every tensor of this stage's range from a name -> array mapping and
        finalises (the reference loads via DenseSource, cpp/src/cpu/stage.cpp:207-260)."""
        names = self.expected_tensors()
        for name in names:
            if name not in weights:
                raise StageError(_lib.INVALID_REQUEST, f"missing tensor {name}")
            self.load_tensor(name, weights[name])
        self.finalize()

    def init_synthetic(self, seed: int) -> None:
        check(lib().hllm_b200_stage_init_synthetic(self._h, seed))
        self.finalize()

    def finalize(self) -> None:
        check(lib().hllm_b200_stage_finalize(self._h))

    def expected_tensors(self) -> list:
        c = self.config
        out = []
        if self.first or (self.final and c.tied):
            out.append("model.embed_tokens.weight")
        if self.final:
            out.append("model.norm.weight")
            if not c.tied:
                out.append("lm_head.weight")
        for i in range(self.layer_start, self.layer_end):
            p = f"model.layers.{i}."
            out += [p + n + ".weight" for n in (
                "input_layernorm", "self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj",
                "self_attn.o_proj", "post_attention_layernorm", "mlp.gate_proj", "mlp.up_proj",
                "mlp.down_proj")]
            if c.query_key_norm:
                out += [p + "self_attn.q_norm.weight", p + "self_attn.k_norm.weight"]
        return out

    # ------------------------------------------------- StageBackend surface
    def _info(self):
        v = [C.c_uint64() for _ in range(4)]
        check(lib().hllm_b200_stage_info(self._h, *[C.byref(x) for x in v]))
        return [x.value for x in v]

    def weight_memory(self) -> dict:
        return {"host_bytes": 0, "device_bytes": self._info()[0], "pinned_host_bytes": 0,
                "unified_bytes": 0}

    def hidden_size(self) -> int:
        return self.config.hidden_size

    def vocabulary_size(self) -> int:
        return self.config.vocabulary_size

    def maximum_tokens(self) -> int:
        return self.config.maximum_sequence_length

    def sequence_memory(self, tokens: int, maximum_query_tokens: Optional[int] = None) -> dict:
        if maximum_query_tokens is None:
            maximum_query_tokens = tokens
        cache, work = C.c_uint64(), C.c_uint64()
        check(lib().hllm_b200_sequence_memory(self._h, tokens, maximum_query_tokens,
                                              C.byref(cache), C.byref(work)))
        return {"cache": {"device_bytes": cache.value}, "workspace": {"device_bytes": work.value}}

    def allocate_sequence(self, tokens: int) -> SequenceState:
        h = C.c_void_p()
        check(lib().hllm_b200_seq_alloc(self._h, tokens, C.byref(h)))
        return SequenceState(handle=h.value, capacity=tokens, owner=self)

    def release(self, state: SequenceState) -> None:
        """Frees the sequence's KV blocks (control_service.cpp:509-515 resets it on release)."""
        if state.handle and state.owner is self:
            lib().hllm_b200_seq_free(self._h, C.c_void_p(state.handle))
            state.handle = 0

    def sequence_info(self, state: SequenceState):
        n, cap, failed = C.c_uint64(), C.c_uint64(), C.c_uint32()
        check(lib().hllm_b200_seq_info(C.c_void_p(state.handle), C.byref(n), C.byref(cap),
                                       C.byref(failed)))
        return n.value, cap.value, bool(failed.value)

    def supports_decode_batch(self) -> bool:
        return True

    def execute(self, input: StageInput, first_position: int, state: SequenceState,
                cancelled=None):
        """One pass for one sequence (stage_backend.hpp:90-92)."""
        return self.execute_mixed_batch([DecodeBatchItem(input, first_position, state, cancelled)],
                                        _check_cancel_all=True)[0]

    def execute_profiled(self, input: StageInput, first_position: int, state: SequenceState,
                         cancelled=None):
        """execute() plus its component timing (stage_backend.hpp:103-106):
        (output, [(component, layer index or None, milliseconds), ...]) with the
        reference's components -- "embedding" / "from-wire", one "layer" per
        owned layer, then "final_norm", "lm_head", "sampling" or "to-wire"."""
        with self._lock:
            check(lib().hllm_b200_stage_component_timing(self._h, 1))
        try:
            output = self.execute(input, first_position, state, cancelled)
            n = C.c_uint32()
            with self._lock:
                check(lib().hllm_b200_stage_components(self._h, None, 0, C.byref(n)))
                parts = (_lib.ComponentTiming * max(1, n.value))()
                check(lib().hllm_b200_stage_components(self._h, parts, n.value, C.byref(n)))
        finally:
            with self._lock:
                lib().hllm_b200_stage_component_timing(self._h, 0)
        timing = [(p.component.decode(), p.layer_index if p.layer_index >= 0 else None,
                   p.milliseconds) for p in parts[:n.value]]
        return output, timing

    def execute_decode_batch(self, items: Sequence[DecodeBatchItem]):
        """combine_decode_inputs rules (cpp/src/decode_batch.cpp:8-38) then one pass.
        An in-flight batch is not pre-empted by one member's cancellation
        (cpp/src/cuda/stage.cpp:218-220)."""
        if not items or len(items) > 64:
            raise StageError(_lib.INVALID_REQUEST, "invalid decode batch size")
        tokens = isinstance(items[0].input, TokenInput)
        seen = set()
        for it in items:
            s = it.sequence
            if (s is None or it.position == 0 or s.prefilling or s.prefill_only or id(s) in seen
                    or tokens != isinstance(it.input, TokenInput)):
                raise StageError(_lib.INVALID_REQUEST,
                                 "decode batch requires independent, ready decode sequences")
            seen.add(id(s))
            if tokens and len(it.input.ids) != 1:
                raise StageError(_lib.INVALID_REQUEST, "decode batch requires one token per sequence")
            if not tokens and it.input.tokens != 1:
                raise StageError(_lib.INVALID_REQUEST, "invalid decode batch boundary")
        return self.execute_mixed_batch(items)

    def execute_mixed_batch(self, items: Sequence[DecodeBatchItem], _check_cancel_all=False):
        """One pass over rows that may mix prefill chunks and decode tokens.
        Returns one output per item, in order."""
        if _check_cancel_all:
            for it in items:
                if _is_cancelled(it.cancelled):
                    raise StageError(_lib.CANCELLED, "request cancelled")
        n = len(items)
        rows, keep, tokens = self._build_rows(items)
        total = int(tokens.sum())
        samples = rows["sample"]
        n_samples = int(samples.sum())
        sampled = np.zeros(max(1, n_samples), _SAMPLED)
        boundary = None
        if not self.final:
            boundary = np.empty(total * self.config.hidden_size, np.uint16)
        with self._lock:
            check(lib().hllm_b200_step(
                self._h, rows.ctypes.data_as(C.POINTER(_lib.Row)), n,
                sampled.ctypes.data_as(C.POINTER(_lib.Sampled)),
                boundary.ctypes.data_as(C.POINTER(C.c_uint16)) if boundary is not None else None))
        outputs = []
        if self.final:
            ids = sampled["token_id"].tolist()
            k = 0
            for i, it in enumerate(items):
                if not samples[i]:
                    outputs.append(PrefillProgress())
                    continue
                o = it.sequence.sampling
                tok = SampledToken(ids[k])
                if o.return_logprobs:
                    res = sampled[k]
                    tok.logprob = float(res["logprob"])
                    tok.top_logprobs = [(int(res["top_ids"][j]), float(res["top_logprobs"][j]))
                                        for j in range(int(res["n_top"]))]
                k += 1
                # The greedy fast path does not consume a draw (cpp/src/cpu/stage.cpp:165-166).
                if not (o.temperature == 0.0 and not o.return_logprobs):
                    it.sequence.generated_index += 1
                outputs.append(tok)
        else:
            off = 0
            h = self.config.hidden_size
            for t in tokens.tolist():
                outputs.append(BoundaryActivation(t, h, boundary[off * h:(off + t) * h].tobytes()))
                off += t
        for it in items:
            if _check_cancel_all and _is_cancelled(it.cancelled):
                raise StageError(_lib.CANCELLED, "request cancelled")
        return outputs

    def _build_rows(self, items):
        """The step's hllm_b200_row array (numpy, the C struct's layout), the
        host buffers its pointers reference, and each row's token count.  One
        Python pass reads the items; columns are then filled at once."""
        n = len(items)
        first, final = self.first, self.final
        handles, positions, counts, samples, draws, options = [], [], [], [], [], []
        id_lists, id_rows, acts = [], [], []
        for i, it in enumerate(items):
            s = it.sequence
            if s is None or s.owner is not self or not s.handle:
                raise StageError(_lib.INVALID_REQUEST, "sequence state or position is invalid")
            inp = it.input
            if isinstance(inp, TokenInput):
                if not first:
                    raise StageError(_lib.INVALID_REQUEST, "only stage zero accepts tokens")
                k = len(inp.ids)
                if k == 0:
                    raise StageError(_lib.INVALID_REQUEST, "invalid stage input")
                id_lists.append(inp.ids)
                id_rows.append(i)
            else:
                if first:
                    raise StageError(_lib.INVALID_REQUEST, "stage zero requires tokens")
                if (inp.width != self.config.hidden_size or inp.tokens == 0
                        or len(inp.payload) != inp.tokens * inp.width * 2):
                    raise StageError(_lib.INVALID_REQUEST, "invalid boundary activation")
                k = inp.tokens
                acts.append((i, np.frombuffer(inp.payload, dtype=np.uint16)))
            handles.append(s.handle)
            positions.append(it.position)
            counts.append(k)
            samples.append(final and not s.prefill_only)
            o = s.sampling
            options.append((o.temperature, o.top_p, o.top_k, o.seed, int(o.return_logprobs),
                            o.top_logprobs))
            draws.append(s.generated_index)
        rows = np.zeros(n, _ROW)
        tokens = np.asarray(counts, np.uint64)
        rows["sequence"] = handles
        rows["first_position"] = positions
        rows["tokens"] = tokens
        rows["sample"] = samples
        rows["sampling"] = np.array(options, _SAMPLING)
        rows["generated_index"] = draws
        keep = []
        if id_lists:
            sizes = tokens[id_rows]
            flat = np.fromiter(itertools.chain.from_iterable(id_lists), np.uint64,
                               count=int(sizes.sum()))
            starts = np.concatenate(([0], np.cumsum(sizes)[:-1])).astype(np.uint64)
            rows["token_ids"][id_rows] = flat.ctypes.data + 8 * starts
            keep.append(flat)
        for i, a in acts:
            rows["activations"][i] = a.ctypes.data
            keep.append(a)
        return rows, keep, tokens

    # ----------------------------------------------------------- test trace
    def read_kv(self, state: SequenceState, layer: int, values: bool) -> np.ndarray:
        n, _, _ = self.sequence_info(state)
        out = np.empty((n, self.config.key_value_heads, self.config.head_dimension), np.uint16)
        check(lib().hllm_b200_seq_read_kv(self._h, C.c_void_p(state.handle), layer, int(values),
                                          out.ctypes.data_as(C.POINTER(C.c_uint16))))
        return out

    def read_hidden(self, tokens: int) -> np.ndarray:
        out = np.empty((tokens, self.config.hidden_size), np.float32)
        check(lib().hllm_b200_stage_read_hidden(self._h, out.ctypes.data_as(C.POINTER(C.c_float)),
                                                tokens))
        return out

    def read_logits(self, rows: int) -> np.ndarray:
        out = np.empty((rows, self.config.vocabulary_size), np.float32)
        check(lib().hllm_b200_stage_read_logits(self._h, out.ctypes.data_as(C.POINTER(C.c_float)),
                                                rows))
        return out

    def last_launches(self) -> int:
        return int(lib().hllm_b200_stage_last_launches(self._h))
