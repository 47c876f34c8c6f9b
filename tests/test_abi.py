"""CPU checks of the drop-in boundary: the C-ABI library loads, exports every
function include/hllm_b200.h declares, and refuses to run without a B200
(there is no CPU fallback)."""
import ctypes as C
import subprocess

import pytest

from hllm_b200 import _lib
from hllm_b200.backend import (B200Stage, DecodeBatchItem, ModelConfig, SamplingOptions,
                               SequenceState, StageError, TokenInput)


def test_library_exports_every_header_function():
    lib = _lib.lib()
    names = _lib.header_functions()
    assert len(names) >= 25
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert set(names) <= exported


def test_header_compiles_as_c():
    r = subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", "-fsyntax-only", "-x", "c",
                        _lib.HEADER], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_status_codes_mirror_reference_error_codes():
    # runtime::ErrorCode order (cpp/include/hllm/runtime/error.hpp:10-17), shifted by OK = 0.
    assert (_lib.INVALID_REQUEST, _lib.INCOMPATIBLE_WORKER, _lib.RESOURCE_EXHAUSTED,
            _lib.DEADLINE_EXCEEDED, _lib.CANCELLED, _lib.INTERNAL) == (1, 2, 3, 4, 5, 6)


def test_structs_match_header_layout(tmp_path):
    """The ctypes mirrors have the C header's sizes and field offsets (gcc)."""
    structs = {"hllm_b200_sampling": _lib.Sampling, "hllm_b200_sampled": _lib.Sampled,
               "hllm_b200_row": _lib.Row, "hllm_b200_stage_desc": _lib.StageDesc,
               "hllm_b200_boundary_identity": _lib.BoundaryIdentity,
               "hllm_b200_envelope_row": _lib.EnvelopeRow,
               "hllm_b200_component_timing": _lib.ComponentTiming}
    lines = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{_lib.HEADER}"',
             'int main(void) {']
    for cname, cls in structs.items():
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for field, _ in cls._fields_:
            lines.append(f'  printf("{cname} {field} %zu\\n", offsetof({cname}, {field}));')
    lines += ['  return 0;', '}']
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    r = subprocess.run(["gcc", "-std=c11", str(src), "-o", str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    got = {tuple(line.split()[:2]): int(line.split()[2]) for line in out if line}
    for cname, cls in structs.items():
        assert got[(cname, "size")] == C.sizeof(cls), cname
        for field, _ in cls._fields_:
            assert got[(cname, field)] == getattr(cls, field).offset, (cname, field)


def test_no_cpu_fallback_without_gpu():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    cfg = ModelConfig(6, 10, 4, 2, 4, 32, 1e-6, 1e6, True, 11, 2, True)
    with pytest.raises(StageError) as e:
        B200Stage(cfg)
    assert e.value.code == _lib.INCOMPATIBLE_WORKER


def test_last_error_is_reported():
    st = _lib.lib().hllm_b200_stage_create(None, None)
    assert st == _lib.INVALID_REQUEST
    assert "null" in _lib.last_error()


def test_decode_batch_rules_checked_before_any_device_call():
    """combine_decode_inputs rules (cpp/src/decode_batch.cpp:8-38) run on the
    host: each violation is an invalid request."""
    stage = B200Stage.__new__(B200Stage)  # host-side validation only; no device stage
    stage.first, stage.final = True, True
    ready = SequenceState(handle=1, capacity=8, owner=stage)
    other = SequenceState(handle=2, capacity=8, owner=stage)
    bad_cases = [
        [],
        [DecodeBatchItem(TokenInput([1]), 0, ready)],                        # position 0
        [DecodeBatchItem(TokenInput([1, 2]), 3, ready)],                     # two tokens
        [DecodeBatchItem(TokenInput([1]), 3, ready), DecodeBatchItem(TokenInput([1]), 3, ready)],
    ]
    prefilling = SequenceState(handle=3, capacity=8, owner=stage, prefilling=True)
    bad_cases.append([DecodeBatchItem(TokenInput([1]), 3, prefilling)])
    only = SequenceState(handle=4, capacity=8, owner=stage, prefill_only=True)
    bad_cases.append([DecodeBatchItem(TokenInput([1]), 3, only)])
    bad_cases.append([DecodeBatchItem(TokenInput([1]), 3, other)] * 65)
    for items in bad_cases:
        with pytest.raises(StageError) as e:
            stage.execute_decode_batch(items)
        assert e.value.code == _lib.INVALID_REQUEST
    assert SamplingOptions().temperature == 0.0
