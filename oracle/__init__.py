"""CPU parity checkers for the B200 stage executor.

TEST INFRASTRUCTURE ONLY: imported by tests/, ``__graft_entry__.smoke()`` and
the CPU-baseline leg of ``bench.py``.  The product package ``hllm_b200`` never
imports this module.

Two libraries sit behind this module:

* ``liboracle.so`` -- ``hllm_oracle.c``, a plain-C restatement of the
  reference's F32 CPU math (cpp/src/cpu/llama.cpp, cpp/src/cpu/tensor.cpp,
  cpp/src/sampling.cpp, cpp/src/half.cpp) plus this build's packer and
  synthetic-weight contracts.
* ``_ref/libhllm_ref.so`` -- the reference's own CPU sources compiled by
  ``oracle/Makefile`` with ``ref_shim.cpp`` (present wherever the reference
  tree was available at build time).

``oracle.envelope`` (pure Python) restates the boundary wire codec
(cpp/src/worker/boundary_codec.cpp, cpp/src/tensor_envelope.cpp).

``OracleModel`` composes the layer functions the way the reference's
``DenseStage::run`` does (cpp/src/cpu/stage.cpp:129-191): embed, layers,
last-row final norm + LM head, sampling; F16 boundary rounding between stages.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from dataclasses import dataclass, field

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_F = C.POINTER(C.c_float)
_U16 = C.POINTER(C.c_uint16)
_I32 = C.POINTER(C.c_int32)
_U64 = C.POINTER(C.c_uint64)


class Config(C.Structure):
    _fields_ = [("hidden_size", C.c_uint64), ("intermediate_size", C.c_uint64),
                ("attention_heads", C.c_uint64), ("key_value_heads", C.c_uint64),
                ("head_dimension", C.c_uint64), ("maximum_sequence_length", C.c_uint64),
                ("rms_norm_epsilon", C.c_float), ("rope_theta", C.c_float),
                ("query_key_norm", C.c_uint32)]


class Layer(C.Structure):
    _fields_ = [(n, _F) for n in ("input_norm", "query", "key", "value", "attention_output",
                                  "post_attention_norm", "gate", "up", "down", "query_norm",
                                  "key_norm")]


class KV(C.Structure):
    _fields_ = [("capacity", C.c_uint64), ("heads", C.c_uint64), ("dim", C.c_uint64),
                ("length", C.c_uint64), ("keys", _F), ("values", _F)]


class Sampling(C.Structure):
    _fields_ = [("temperature", C.c_double), ("top_p", C.c_double), ("top_k", C.c_uint64),
                ("seed", C.c_uint64), ("return_logprobs", C.c_uint32),
                ("top_logprobs", C.c_uint32)]


class Sampled(C.Structure):
    _fields_ = [("token_id", C.c_uint64), ("logprob", C.c_double), ("has_logprob", C.c_uint32),
                ("n_top", C.c_uint32), ("top_ids", C.c_uint64 * 5),
                ("top_logprobs", C.c_double * 5)]


def build(force: bool = False) -> None:
    """Compile liboracle.so (and _ref when the reference tree is present)."""
    if force or not os.path.exists(os.path.join(HERE, "liboracle.so")):
        subprocess.run(["make", "-s", "-C", HERE], check=True)


def _load(path):
    lib = C.CDLL(path)
    return lib


_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        _lib = _load(path)
        _lib.oracle_f32_to_f16.restype = C.c_uint16
        _lib.oracle_f32_to_f16.argtypes = [C.c_float]
        _lib.oracle_f16_to_f32.restype = C.c_float
        _lib.oracle_f16_to_f32.argtypes = [C.c_uint16]
        _lib.oracle_rms_norm.argtypes = [_F, _F, C.c_size_t, C.c_size_t, C.c_float, _F]
        _lib.oracle_normalize_heads.argtypes = [_F, C.c_size_t, _F, C.c_size_t, C.c_float]
        _lib.oracle_apply_rope.argtypes = [_F, C.c_size_t, C.c_size_t, C.c_size_t, C.c_size_t,
                                           C.c_float]
        _lib.oracle_linear.argtypes = [_F, C.c_size_t, C.c_size_t, _F, C.c_size_t, _F]
        _lib.oracle_attention.argtypes = [_F, C.c_size_t, C.POINTER(Config), C.c_size_t,
                                          C.POINTER(KV), _F]
        _lib.oracle_transformer_layer.argtypes = [_F, C.c_size_t, C.POINTER(Layer),
                                                  C.POINTER(Config), C.c_size_t, C.POINTER(KV),
                                                  _F]
        _lib.oracle_final_logits.argtypes = [_F, C.c_size_t, C.c_size_t, _F, _F, C.c_size_t,
                                             C.c_float, _F]
        _lib.oracle_greedy_sample_last.restype = C.c_longlong
        _lib.oracle_greedy_sample_last.argtypes = [_F, C.c_size_t, C.c_size_t]
        _lib.oracle_sample_logits.argtypes = [_F, C.c_size_t, C.POINTER(Sampling), C.c_uint64,
                                              _U64]
        _lib.oracle_sample_token.argtypes = [_F, C.c_size_t, C.POINTER(Sampling), C.c_uint64,
                                             C.POINTER(Sampled)]
        _lib.oracle_uniform.restype = C.c_double
        _lib.oracle_uniform.argtypes = [C.c_uint64, C.c_uint64]
        _lib.oracle_pack.argtypes = [_I32, _I32, _I32, C.c_int32, _I32, C.c_int32, C.c_int32,
                                     _I32, _I32, _I32, _I32, _I32, _I32]
        _lib.oracle_synth_matrix_f16.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64, C.c_float,
                                                 _U16]
        _lib.oracle_synth_norm_f16.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64, C.c_float,
                                               _U16]
        _lib.oracle_f32_to_f16_array.argtypes = [_F, _U16, C.c_size_t]
        _lib.oracle_f16_to_f32_array.argtypes = [_U16, _F, C.c_size_t]
        _lib.oracle_num_threads.restype = C.c_int
    return _lib


def ref_path() -> str:
    return os.path.join(HERE, "_ref", "libhllm_ref.so")


def ref():
    """The reference's own CPU math (None when oracle/_ref was never built)."""
    global _ref
    if _ref is None:
        if not os.path.exists(ref_path()):
            return None
        r = _load(ref_path())
        r.ref_cache_new.restype = C.c_void_p
        r.ref_cache_new.argtypes = [C.c_uint64] * 3
        r.ref_cache_free.argtypes = [C.c_void_p]
        r.ref_cache_length.restype = C.c_uint64
        r.ref_cache_length.argtypes = [C.c_void_p]
        r.ref_cache_read.argtypes = [C.c_void_p, _F, _F]
        r.ref_cache_append.argtypes = [C.c_void_p, C.c_uint64, _F, _F]
        r.ref_transformer_layer.argtypes = [_F, C.c_uint64, C.POINTER(Layer), C.POINTER(Config),
                                            C.c_uint64, C.c_void_p, _F]
        r.ref_final_logits.argtypes = [_F, C.c_uint64, C.c_uint64, _F, _F, C.c_uint64,
                                       C.c_float, _F]
        r.ref_greedy_sample_last.restype = C.c_longlong
        r.ref_greedy_sample_last.argtypes = [_F, C.c_uint64, C.c_uint64]
        r.ref_rms_norm.argtypes = [_F, _F, C.c_uint64, C.c_uint64, C.c_float, _F]
        r.ref_apply_rope.argtypes = [_F, C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint64,
                                     C.c_float]
        r.ref_linear.argtypes = [_F, C.c_uint64, C.c_uint64, _F, C.c_uint64, _F]
        r.ref_sample_token.argtypes = [_F, C.c_uint64, C.POINTER(Sampling), C.c_uint64,
                                       C.POINTER(Sampled)]
        r.ref_float_to_float16.restype = C.c_uint16
        r.ref_float_to_float16.argtypes = [C.c_float]
        r.ref_float16_to_float.restype = C.c_float
        r.ref_float16_to_float.argtypes = [C.c_uint16]
        r.ref_combine_decode_tokens.argtypes = [_U64, _U64, _U64, C.POINTER(C.c_uint8),
                                                C.POINTER(C.c_uint8), _I32, C.c_uint64, _U64]
        r.ref_layer_new.restype = C.c_void_p
        r.ref_layer_new.argtypes = [C.POINTER(Layer), C.POINTER(Config)]
        r.ref_layer_free.argtypes = [C.c_void_p]
        r.ref_layer_forward.argtypes = [C.c_void_p, _F, C.c_uint64, C.c_uint64, C.c_void_p, _F]
        r.ref_head_new.restype = C.c_void_p
        r.ref_head_new.argtypes = [_F, _F, C.c_uint64, C.c_uint64]
        r.ref_head_free.argtypes = [C.c_void_p]
        r.ref_head_logits.argtypes = [C.c_void_p, _F, C.c_uint64, C.c_float, _F]
        _ref = r
    return _ref


def fp(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_F)


def ip(a: np.ndarray):
    assert a.dtype == np.int32 and a.flags.c_contiguous
    return a.ctypes.data_as(_I32)


# --------------------------------------------------------------------------
# numpy front ends
# --------------------------------------------------------------------------

def f16_round(x: np.ndarray) -> np.ndarray:
    """F32 -> F16 (round to nearest even, half.cpp rules) -> F32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    bits = np.empty(x.shape, dtype=np.uint16)
    lib().oracle_f32_to_f16_array(fp(x), bits.ctypes.data_as(_U16), x.size)
    return f16_decode(bits)


def f16_encode(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    bits = np.empty(x.shape, dtype=np.uint16)
    lib().oracle_f32_to_f16_array(fp(x), bits.ctypes.data_as(_U16), x.size)
    return bits


def f16_decode(bits: np.ndarray) -> np.ndarray:
    bits = np.ascontiguousarray(bits, dtype=np.uint16)
    out = np.empty(bits.shape, dtype=np.float32)
    lib().oracle_f16_to_f32_array(bits.ctypes.data_as(_U16), fp(out), bits.size)
    return out


def rms_norm(x, w, eps):
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.empty_like(x)
    lib().oracle_rms_norm(fp(x), fp(w), x.shape[0], x.shape[1], eps, fp(out))
    return out


def linear(x, W):
    x = np.ascontiguousarray(x, np.float32)
    W = np.ascontiguousarray(W, np.float32)
    y = np.empty((x.shape[0], W.shape[0]), np.float32)
    lib().oracle_linear(fp(x), x.shape[0], x.shape[1], fp(W), W.shape[0], fp(y))
    return y


def normalize_heads(x, w, eps):
    x = np.array(x, np.float32, order="C", copy=True)
    w = np.ascontiguousarray(w, np.float32)
    lib().oracle_normalize_heads(fp(x), x.size, fp(w), w.size, eps)
    return x


def apply_rope(x, heads, dim, first_position, theta):
    x = np.array(x, np.float32, order="C", copy=True)
    lib().oracle_apply_rope(fp(x), x.shape[0], heads, dim, first_position, theta)
    return x


def sampling(temperature=0.0, top_p=1.0, top_k=0, seed=0, return_logprobs=False,
             top_logprobs=0) -> Sampling:
    return Sampling(temperature, top_p, top_k, seed, int(return_logprobs), top_logprobs)


def sample_token(logits, opts: Sampling, generated_index: int):
    """Returns (status, Sampled) exactly as sampling.cpp:65-90 would."""
    logits = np.ascontiguousarray(logits, np.float32)
    out = Sampled()
    st = lib().oracle_sample_token(fp(logits), logits.size, C.byref(opts), generated_index,
                                   C.byref(out))
    return st, out


def greedy(logits) -> int:
    logits = np.ascontiguousarray(np.atleast_2d(logits), np.float32)
    return int(lib().oracle_greedy_sample_last(fp(logits), logits.shape[0], logits.shape[1]))


def pack(row_slot, row_first, row_count, slot_blocks, block=16):
    """Host restatement of the ragged packer; returns a dict of int32 arrays
    (or None when a row needs a block its slot does not own)."""
    row_slot = np.ascontiguousarray(row_slot, np.int32)
    row_first = np.ascontiguousarray(row_first, np.int32)
    row_count = np.ascontiguousarray(row_count, np.int32)
    slot_blocks = np.ascontiguousarray(slot_blocks, np.int32)
    R = row_slot.size
    T = int(row_count.sum())
    mb = slot_blocks.shape[1]
    out = dict(cu_seqlens=np.zeros(R + 1, np.int32), positions=np.zeros(T, np.int32),
               slot_mapping=np.zeros(T, np.int32), token_row=np.zeros(T, np.int32),
               seq_lens=np.zeros(R, np.int32), block_tables=np.zeros((R, mb), np.int32))
    st = lib().oracle_pack(ip(row_slot), ip(row_first), ip(row_count), R, ip(slot_blocks), mb,
                           block, ip(out["cu_seqlens"]), ip(out["positions"]),
                           ip(out["slot_mapping"]), ip(out["token_row"]), ip(out["seq_lens"]),
                           ip(out["block_tables"]))
    return out if st == 0 else None


# --------------------------------------------------------------------------
# Synthetic weights (bit-identical to the device initialiser)
# --------------------------------------------------------------------------
KIND = dict(input_norm=0, query=1, key=2, value=3, attention_output=4, post_attention_norm=5,
            gate=6, up=7, down=8, query_norm=9, key_norm=10)
TAG_EMBED, TAG_HEAD, TAG_FINAL_NORM = 0xE0000, 0xE0001, 0xE0002
WEIGHT_STD = 0.02
NORM_SPREAD = 0.1


def synth_matrix(seed, tag, shape, std=WEIGHT_STD) -> np.ndarray:
    n = int(np.prod(shape))
    out = np.empty(n, np.uint16)
    lib().oracle_synth_matrix_f16(seed, tag, n, std, out.ctypes.data_as(_U16))
    return out.reshape(shape)


def synth_norm(seed, tag, n, spread=NORM_SPREAD) -> np.ndarray:
    out = np.empty(n, np.uint16)
    lib().oracle_synth_norm_f16(seed, tag, n, spread, out.ctypes.data_as(_U16))
    return out


# --------------------------------------------------------------------------
# Model-level oracle
# --------------------------------------------------------------------------
@dataclass
class ModelSpec:
    """Geometry of one decoder (the reference's DenseConfig plus vocabulary)."""
    hidden_size: int
    intermediate_size: int
    attention_heads: int
    key_value_heads: int
    head_dimension: int
    layers: int
    vocabulary_size: int
    maximum_sequence_length: int
    rms_norm_epsilon: float
    rope_theta: float
    query_key_norm: bool
    tied: bool

    def config(self) -> Config:
        return Config(self.hidden_size, self.intermediate_size, self.attention_heads,
                      self.key_value_heads, self.head_dimension, self.maximum_sequence_length,
                      self.rms_norm_epsilon, self.rope_theta, int(self.query_key_norm))


def layer_shapes(spec: ModelSpec):
    h, I, d = spec.hidden_size, spec.intermediate_size, spec.head_dimension
    qw, kw = spec.attention_heads * d, spec.key_value_heads * d
    shapes = dict(input_norm=(h,), query=(qw, h), key=(kw, h), value=(kw, h),
                  attention_output=(h, qw), post_attention_norm=(h,), gate=(I, h), up=(I, h),
                  down=(h, I))
    if spec.query_key_norm:
        shapes.update(query_norm=(d,), key_norm=(d,))
    return shapes


def synth_head_weights(spec: ModelSpec, seed: int):
    """The embedding, final norm and (untied) LM head of the seeded synthetic
    model, as F16 bit patterns named like the reference's Safetensors tensors."""
    h = spec.hidden_size
    out = {"model.embed_tokens.weight": synth_matrix(seed, TAG_EMBED, (spec.vocabulary_size, h))}
    if not spec.tied:
        out["lm_head.weight"] = synth_matrix(seed, TAG_HEAD, (spec.vocabulary_size, h))
    out["model.norm.weight"] = synth_norm(seed, TAG_FINAL_NORM, h)
    return out


def synth_layer_weights(spec: ModelSpec, seed: int, i: int):
    """Layer i's tensors of the seeded synthetic model (F16 bit patterns)."""
    out = {}
    for kind, shape in layer_shapes(spec).items():
        tag = i * 16 + KIND[kind]
        arr = synth_norm(seed, tag, shape[0]) if len(shape) == 1 else synth_matrix(seed, tag, shape)
        out[f"model.layers.{i}.{LAYER_NAMES[kind]}.weight"] = arr
    return out


def synth_weights(spec: ModelSpec, seed: int, layers=None):
    """F16 bit patterns of the seeded synthetic model: {name: uint16 array}, named
    like the reference's Safetensors tensors (cpp/src/cpu/stage.cpp:246-259)."""
    out = synth_head_weights(spec, seed)
    for i in (range(spec.layers) if layers is None else layers):
        out.update(synth_layer_weights(spec, seed, i))
    return out


LAYER_NAMES = dict(input_norm="input_layernorm", query="self_attn.q_proj",
                   key="self_attn.k_proj", value="self_attn.v_proj",
                   attention_output="self_attn.o_proj",
                   post_attention_norm="post_attention_layernorm", gate="mlp.gate_proj",
                   up="mlp.up_proj", down="mlp.down_proj", query_norm="self_attn.q_norm",
                   key_norm="self_attn.k_norm")


@dataclass
class OracleSequence:
    caches: list
    keep: list = field(default_factory=list)
    length: int = 0
    generated_index: int = 0


class OracleModel:
    """The reference's F32 pipeline over one contiguous layer range.

    ``weights`` maps tensor names to float32 arrays (F16 storage decoded to F32,
    as the reference's dense source does for an F16 checkpoint)."""

    def __init__(self, spec: ModelSpec, weights: dict, layer_start=0, layer_end=None,
                 use_ref=False):
        self.spec = spec
        self.cfg = spec.config()
        self.start = layer_start
        self.end = spec.layers if layer_end is None else layer_end
        self.use_ref = use_ref
        f32 = {k: (f16_decode(v) if v.dtype == np.uint16 else np.ascontiguousarray(v, np.float32))
               for k, v in weights.items()}
        self.w = f32
        self.layers = []
        for i in range(self.start, self.end):
            arrs = {}
            for kind in LAYER_NAMES:
                name = f"model.layers.{i}.{LAYER_NAMES[kind]}.weight"
                if name in f32:
                    arrs[kind] = np.ascontiguousarray(f32[name], np.float32)
            lw = Layer(**{k: fp(v) for k, v in arrs.items()})
            self.layers.append((lw, arrs))
        self._ref_layers = []
        self._ref_head = None
        if use_ref:
            for lw, _ in self.layers:
                handle = ref().ref_layer_new(C.byref(lw), C.byref(self.cfg))
                if not handle:
                    raise MemoryError("reference layer construction failed")
                self._ref_layers.append(handle)

    def __del__(self):
        r = _ref
        if r is None:
            return
        for h in getattr(self, "_ref_layers", []):
            r.ref_layer_free(h)
        if getattr(self, "_ref_head", None):
            r.ref_head_free(self._ref_head)

    def new_sequence(self, capacity: int) -> OracleSequence:
        s = self.spec
        caches, keep = [], []
        for _ in range(self.start, self.end):
            if self.use_ref:
                caches.append(ref().ref_cache_new(capacity, s.key_value_heads, s.head_dimension))
            else:
                k = np.zeros((capacity, s.key_value_heads, s.head_dimension), np.float32)
                v = np.zeros_like(k)
                keep.append((k, v))
                caches.append(KV(capacity, s.key_value_heads, s.head_dimension, 0, fp(k), fp(v)))
        return OracleSequence(caches, keep)

    def fill_context(self, seq: OracleSequence, length: int, seed: int = 0):
        """Sets every owned layer's cache of a fresh sequence to `length`
        positions of seeded synthetic keys and values (N(0, 1) scaled by
        1/sqrt(d)), as if that much context had been processed: the cost of
        later steps depends on the context length, not on its values."""
        s = self.spec
        rng = np.random.default_rng(seed)
        width = s.key_value_heads * s.head_dimension
        for li in range(len(seq.caches)):
            k = (rng.standard_normal((length, width)) / np.sqrt(s.head_dimension)).astype(np.float32)
            v = (rng.standard_normal((length, width)) / np.sqrt(s.head_dimension)).astype(np.float32)
            if self.use_ref:
                if ref().ref_cache_append(seq.caches[li], length, fp(k), fp(v)) != 0:
                    raise ValueError("reference cache rejected the context")
            else:
                kk, vv = seq.keep[li]
                kk[:length] = k.reshape(length, s.key_value_heads, s.head_dimension)
                vv[:length] = v.reshape(length, s.key_value_heads, s.head_dimension)
                seq.caches[li].length = length
        seq.length = length

    def free_sequence(self, seq: OracleSequence):
        if self.use_ref:
            for c in seq.caches:
                ref().ref_cache_free(c)
        seq.caches = []

    def embed(self, ids) -> np.ndarray:
        E = self.w["model.embed_tokens.weight"]
        return np.ascontiguousarray(E[np.asarray(ids, np.int64)], np.float32)

    def forward(self, hidden: np.ndarray, position: int, seq: OracleSequence, trace=None):
        hidden = np.ascontiguousarray(hidden, np.float32)
        rows = hidden.shape[0]
        for li, ((lw, _), cache) in enumerate(zip(self.layers, seq.caches)):
            out = np.empty_like(hidden)
            if self.use_ref:
                st = ref().ref_layer_forward(self._ref_layers[li], fp(hidden), rows, position, cache,
                                             fp(out))
            else:
                st = lib().oracle_transformer_layer(fp(hidden), rows, C.byref(lw),
                                                    C.byref(self.cfg), position, C.byref(cache),
                                                    fp(out))
            if st != 0:
                raise ValueError(f"oracle layer rejected input (status {st})")
            hidden = out
            if trace is not None:
                trace.append(hidden.copy())
        seq.length = position + rows
        return hidden

    def head_matrix(self):
        return self.w["model.embed_tokens.weight"] if self.spec.tied else self.w["lm_head.weight"]

    def logits(self, hidden_rows: np.ndarray) -> np.ndarray:
        hidden_rows = np.ascontiguousarray(hidden_rows, np.float32)
        head = np.ascontiguousarray(self.head_matrix(), np.float32)
        norm = np.ascontiguousarray(self.w["model.norm.weight"], np.float32)
        out = np.empty((hidden_rows.shape[0], head.shape[0]), np.float32)
        if self.use_ref:
            if self._ref_head is None:
                self._ref_head = ref().ref_head_new(fp(norm), fp(head), head.shape[0], head.shape[1])
            st = ref().ref_head_logits(self._ref_head, fp(hidden_rows), hidden_rows.shape[0],
                                       self.spec.rms_norm_epsilon, fp(out))
            if st != 0:
                raise ValueError(f"reference head rejected input (status {st})")
            return out
        lib().oracle_final_logits(fp(hidden_rows), hidden_rows.shape[0], hidden_rows.shape[1],
                                  fp(norm), fp(head), head.shape[0], self.spec.rms_norm_epsilon,
                                  fp(out))
        return out

    def kv(self, seq: OracleSequence, layer: int):
        """(keys, values) of one owned layer as [length, kv_heads, dim]."""
        s = self.spec
        li = layer - self.start
        if self.use_ref:
            n = int(ref().ref_cache_length(seq.caches[li]))
            k = np.empty((n, s.key_value_heads, s.head_dimension), np.float32)
            v = np.empty_like(k)
            ref().ref_cache_read(seq.caches[li], fp(k), fp(v))
            return k, v
        n = seq.caches[li].length
        k, v = seq.keep[li]
        return k[:n].copy(), v[:n].copy()
