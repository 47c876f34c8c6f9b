"""ctypes binding of libhllm_b200.so (declarations in include/hllm_b200.h).

The library is the only compute path: importing this module on a machine
without the built library, or calling into it without a CUDA device, raises --
there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB_PATH = os.path.join(HERE, "libhllm_b200.so")
HEADER = os.path.join(ROOT, "include", "hllm_b200.h")

OK, INVALID_REQUEST, INCOMPATIBLE_WORKER, RESOURCE_EXHAUSTED, DEADLINE_EXCEEDED, CANCELLED, \
    INTERNAL = range(7)
CODE_NAMES = {0: "ok", 1: "invalid_request", 2: "incompatible_worker", 3: "resource_exhausted",
              4: "deadline_exceeded", 5: "cancelled", 6: "internal"}
F32, F16, BF16 = 0, 1, 2


class StageError(RuntimeError):
    """A failed call; ``code`` mirrors runtime::ErrorCode (cpp/include/hllm/runtime/error.hpp)."""

    def __init__(self, code: int, message: str):
        super().__init__(f"{CODE_NAMES.get(code, code)}: {message}")
        self.code = code
        self.message = message


class StageDesc(C.Structure):
    _fields_ = [("hidden_size", C.c_uint64), ("intermediate_size", C.c_uint64),
                ("attention_heads", C.c_uint64), ("key_value_heads", C.c_uint64),
                ("head_dimension", C.c_uint64), ("maximum_sequence_length", C.c_uint64),
                ("rms_norm_epsilon", C.c_float), ("rope_theta", C.c_float),
                ("query_key_norm", C.c_uint32), ("vocabulary_size", C.c_uint64),
                ("layer_start", C.c_uint64), ("layer_end", C.c_uint64), ("first", C.c_uint32),
                ("final", C.c_uint32), ("tied_head", C.c_uint32), ("device_id", C.c_int32),
                ("kv_pool_tokens", C.c_uint64), ("max_step_tokens", C.c_uint32),
                ("max_step_rows", C.c_uint32), ("max_sequences", C.c_uint32)]


class Sampling(C.Structure):
    _fields_ = [("temperature", C.c_double), ("top_p", C.c_double), ("top_k", C.c_uint64),
                ("seed", C.c_uint64), ("return_logprobs", C.c_uint32),
                ("top_logprobs", C.c_uint32)]


class Row(C.Structure):
    _fields_ = [("sequence", C.c_void_p), ("first_position", C.c_uint64), ("tokens", C.c_uint64),
                ("token_ids", C.POINTER(C.c_uint64)), ("activations", C.POINTER(C.c_uint16)),
                ("sample", C.c_uint32), ("sampling", Sampling), ("generated_index", C.c_uint64)]


class BoundaryIdentity(C.Structure):
    _fields_ = [("deployment_id", C.c_char_p), ("deployment_version", C.c_uint64),
                ("request_id", C.c_char_p), ("maximum_tokens", C.c_uint64),
                ("hidden_size", C.c_uint64)]


class EnvelopeRow(C.Structure):
    _fields_ = [("first_token", C.c_uint64), ("tokens", C.c_uint64),
                ("identity", BoundaryIdentity), ("sequence", C.c_uint64),
                ("position", C.c_uint64), ("prefill", C.c_uint32)]


class ComponentTiming(C.Structure):
    _fields_ = [("component", C.c_char * 16), ("layer_index", C.c_int64),
                ("milliseconds", C.c_double)]


class Sampled(C.Structure):
    _fields_ = [("token_id", C.c_uint64), ("logprob", C.c_double), ("has_logprob", C.c_uint32),
                ("n_top", C.c_uint32), ("top_ids", C.c_uint64 * 5),
                ("top_logprobs", C.c_double * 5)]


_lib = None
vp = C.c_void_p
u32, u64, i32, f32 = C.c_uint32, C.c_uint64, C.c_int32, C.c_float


def header_functions() -> list[str]:
    """Names of every function include/hllm_b200.h declares."""
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(hllm_b200_\w+)\s*\(", text)))


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is not built; run `python -m hllm_b200.build` "
                          "(the B200 executor has no CPU fallback)")
    L = C.CDLL(LIB_PATH)
    sig = {
        "hllm_b200_last_error": (C.c_size_t, [C.c_char_p, C.c_size_t]),
        "hllm_b200_stage_create": (C.c_int, [C.POINTER(StageDesc), C.POINTER(vp)]),
        "hllm_b200_stage_destroy": (None, [vp]),
        "hllm_b200_stage_load_tensor": (C.c_int, [vp, C.c_char_p, C.c_int, vp, C.POINTER(u64), u32]),
        "hllm_b200_stage_init_synthetic": (C.c_int, [vp, u64]),
        "hllm_b200_stage_finalize": (C.c_int, [vp]),
        "hllm_b200_stage_info": (C.c_int, [vp] + [C.POINTER(u64)] * 4),
        "hllm_b200_sequence_memory": (C.c_int, [vp, u64, u64, C.POINTER(u64), C.POINTER(u64)]),
        "hllm_b200_seq_alloc": (C.c_int, [vp, u64, C.POINTER(vp)]),
        "hllm_b200_seq_free": (None, [vp, vp]),
        "hllm_b200_seq_info": (C.c_int, [vp, C.POINTER(u64), C.POINTER(u64), C.POINTER(u32)]),
        "hllm_b200_step": (C.c_int, [vp, C.POINTER(Row), u32, C.POINTER(Sampled),
                                     C.POINTER(C.c_uint16)]),
        "hllm_b200_step_async": (C.c_int, [vp, C.POINTER(Row), u32, vp]),
        "hllm_b200_stage_sync": (C.c_int, [vp]),
        "hllm_b200_stage_results": (C.c_int, [vp, C.POINTER(Sampled), u32]),
        "hllm_b200_stage_profile": (C.c_int, [vp, u32]),
        "hllm_b200_stage_profile_read": (C.c_int, [vp, u32, C.POINTER(C.c_double), C.POINTER(u64),
                                                   C.POINTER(C.c_double), C.POINTER(C.c_double)]),
        "hllm_b200_stage_stream": (vp, [vp]),
        "hllm_b200_stage_device": (i32, [vp]),
        "hllm_b200_stage_last_launches": (u32, [vp]),
        "hllm_b200_stage_boundary": (vp, [vp]),
        "hllm_b200_stage_last_transfer": (C.c_int, [vp, C.POINTER(u64), C.POINTER(u64)]),
        "hllm_b200_envelope_encode": (C.c_int, [C.POINTER(BoundaryIdentity), u64, u64, u32, vp,
                                                u64, u64, u64, vp, u64, C.POINTER(u64)]),
        "hllm_b200_envelope_decode": (C.c_int, [vp, u64, C.POINTER(BoundaryIdentity), u64, u64,
                                                u32, C.POINTER(u64), C.POINTER(u64)]),
        "hllm_b200_stage_envelope": (C.c_int, [vp, u64, u64, C.POINTER(BoundaryIdentity), u64,
                                               u64, u32, vp, u64, C.POINTER(u64)]),
        "hllm_b200_stage_envelope_wait": (C.c_int, [vp]),
        "hllm_b200_stage_envelopes": (C.c_int, [vp, C.POINTER(EnvelopeRow), u32, vp, u64,
                                                C.POINTER(u64)]),
        "hllm_b200_stage_component_timing": (C.c_int, [vp, u32]),
        "hllm_b200_stage_memory": (C.c_int, [vp] + [C.POINTER(u64)] * 5),
        "hllm_b200_stage_components": (C.c_int, [vp, C.POINTER(ComponentTiming), u32,
                                                 C.POINTER(u32)]),
        "hllm_b200_seq_read_kv": (C.c_int, [vp, vp, u64, u32, C.POINTER(C.c_uint16)]),
        "hllm_b200_stage_read_hidden": (C.c_int, [vp, C.POINTER(C.c_float), u64]),
        "hllm_b200_stage_read_logits": (C.c_int, [vp, C.POINTER(C.c_float), u64]),
        "hllm_b200_gemm": (C.c_int, [vp, u64, u64, u32, u64, vp, u64, u32, vp, u64, u32, u32, vp]),
        "hllm_b200_gemm_noalloc": (C.c_int, [vp, u64, u64, u32, u64, vp, u64, u32, vp, u64, u32,
                                             u32, vp]),
        "hllm_b200_rmsnorm": (C.c_int, [vp, u64, u64, vp, f32, vp, u64, vp]),
        "hllm_b200_pack": (C.c_int, [vp, vp, vp, u32, u32, vp, u32, u32, u32] + [vp] * 9 + [vp]),
        "hllm_b200_attention": (C.c_int, [vp] * 10 + [u32] * 8 + [vp, u64, u64, u64, vp, vp]),
        "hllm_b200_attention_qtile_tokens": (u32, [u32]),
        "hllm_b200_qkv_post": (C.c_int, [vp, u64, u32, u32, u32, vp, vp, vp, vp, f32, vp, vp, vp,
                                         vp, vp]),
        "hllm_b200_sample": (C.c_int, [vp, u32, u64, u64, C.POINTER(Sampling), C.POINTER(u64),
                                       C.POINTER(Sampled), vp]),
        "hllm_b200_synth_matrix": (C.c_int, [u64, u64, u64, u64, u64, f32, vp, vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def last_error() -> str:
    buf = C.create_string_buffer(4096)
    lib().hllm_b200_last_error(buf, 4096)
    return buf.value.decode(errors="replace")


def check(status: int) -> None:
    if status != OK:
        raise StageError(status, last_error())
