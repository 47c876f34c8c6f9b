"""The Python mirror's step rows (B200Stage._build_rows) against the same rows
filled field by field through the ctypes mirror of hllm_b200_row: equal bytes
in every field, equal data behind the id and activation pointers, and the
same errors.  Host only: no stage is created."""
import ctypes as C
import random

import numpy as np
import pytest

from hllm_b200 import _lib
from hllm_b200.backend import (B200Stage, BoundaryActivation, DecodeBatchItem, ModelConfig,
                               SamplingOptions, SequenceState, StageError, TokenInput)

CFG = ModelConfig(64, 128, 4, 2, 16, 4096, 1e-6, 1e6, True, 1000, 2, True)


def _stage(first=True, final=True):
    st = B200Stage.__new__(B200Stage)  # host-side row building only; no device stage
    st.first, st.final, st.config = first, final, CFG
    return st


def _ctypes_rows(st, items):
    """hllm_b200_row filled one field at a time through ctypes."""
    rows = (_lib.Row * len(items))()
    for i, it in enumerate(items):
        s, r = it.sequence, rows[i]
        r.sequence = s.handle
        r.first_position = it.position
        r.tokens = len(it.input.ids) if isinstance(it.input, TokenInput) else it.input.tokens
        r.sample = int(st.final and not s.prefill_only)
        o = s.sampling
        r.sampling = _lib.Sampling(o.temperature, o.top_p, o.top_k, o.seed,
                                   int(o.return_logprobs), o.top_logprobs)
        r.generated_index = s.generated_index
    return rows


def _items(st, rng, n, boundary=False):
    out = []
    for i in range(n):
        s = SequenceState(handle=rng.randrange(1, 1 << 40), capacity=4096, owner=st,
                          prefill_only=rng.random() < 0.3,
                          generated_index=rng.randrange(0, 1 << 20))
        s.sampling = SamplingOptions(rng.choice([0.0, 0.7, 1.3]), rng.choice([1.0, 0.9]),
                                     rng.choice([0, 8]), rng.randrange(0, 1 << 62),
                                     rng.random() < 0.5, rng.choice([0, 3, 5]))
        k = rng.choice([1, 1, 1, 3, 77])
        if boundary:
            payload = np.random.default_rng(i).integers(0, 1 << 15, k * CFG.hidden_size,
                                                        dtype=np.uint16).tobytes()
            inp = BoundaryActivation(k, CFG.hidden_size, payload)
        else:
            inp = TokenInput([rng.randrange(0, 1000) for _ in range(k)])
        out.append(DecodeBatchItem(inp, rng.randrange(0, 3000), s))
    return out


@pytest.mark.parametrize("boundary", [False, True])
def test_rows_equal_the_ctypes_fill(boundary):
    rng = random.Random(3 + boundary)
    for n in (1, 2, 7, 65):
        st = _stage(first=not boundary, final=rng.random() < 0.7)
        items = _items(st, rng, n, boundary)
        rows, keep, tokens = st._build_rows(items)
        ref = _ctypes_rows(st, items)
        got = (_lib.Row * n).from_buffer_copy(rows.tobytes())
        assert rows.itemsize == C.sizeof(_lib.Row)
        for i, it in enumerate(items):
            for f, _ in _lib.Row._fields_:
                if f in ("token_ids", "activations"):
                    continue
                a, b = getattr(got[i], f), getattr(ref[i], f)
                if f == "sampling":
                    a, b = bytes(a), bytes(b)
                assert a == b, (n, i, f)
            k = int(tokens[i])
            if boundary:
                assert not got[i].token_ids
                data = C.string_at(got[i].activations, k * CFG.hidden_size * 2)
                assert data == it.input.payload
            else:
                assert not got[i].activations
                assert list(got[i].token_ids[:k]) == list(it.input.ids)


def test_row_errors_match():
    st = _stage()
    s = SequenceState(handle=1, capacity=8, owner=st)
    other = SequenceState(handle=2, capacity=8, owner=object())
    for bad in ([DecodeBatchItem(TokenInput([]), 0, s)],
                [DecodeBatchItem(TokenInput([1]), 0, other)],
                [DecodeBatchItem(BoundaryActivation(1, CFG.hidden_size, bytes(128)), 0, s)]):
        with pytest.raises(StageError) as e:
            st._build_rows(bad)
        assert e.value.code == _lib.INVALID_REQUEST
    st2 = _stage(first=False)
    with pytest.raises(StageError):
        st2._build_rows([DecodeBatchItem(TokenInput([1]), 0, s)])
    with pytest.raises(StageError):  # payload size disagrees with the shape
        st2._build_rows([DecodeBatchItem(BoundaryActivation(2, CFG.hidden_size, bytes(128)), 0,
                                         SequenceState(handle=3, capacity=8, owner=st2))])


class _FakeLib:
    """Stands in for libhllm_b200's step call: checks the rows it receives and
    writes known results, as the library does."""

    def __init__(self):
        self.calls = []

    def hllm_b200_step(self, handle, rows_ptr, n, sampled_ptr, boundary_ptr):
        rows = C.cast(rows_ptr, C.POINTER(_lib.Row))
        k = 0
        total = 0
        for i in range(n):
            r = rows[i]
            total += r.tokens
            if r.sample:
                res = C.cast(sampled_ptr, C.POINTER(_lib.Sampled))[k]
                res.token_id = 1000 + i
                res.logprob = -0.25 * (i + 1)
                res.has_logprob = 1
                res.n_top = 3
                for j in range(3):
                    res.top_ids[j] = 10 * i + j
                    res.top_logprobs[j] = -float(j)
                k += 1
        if boundary_ptr:
            buf = C.cast(boundary_ptr, C.POINTER(C.c_uint16))
            for e in range(total * CFG.hidden_size):
                buf[e] = e % 65000
        self.calls.append((n, k, total))
        return 0


def test_outputs_read_back_from_the_step(monkeypatch):
    import threading
    from hllm_b200 import backend
    fake = _FakeLib()
    monkeypatch.setattr(backend, "lib", lambda: fake)
    st = _stage()
    st._lock, st._h = threading.Lock(), C.c_void_p(1)
    greedy = SequenceState(handle=1, capacity=64, owner=st)
    hot = SequenceState(handle=2, capacity=64, owner=st)
    hot.sampling = SamplingOptions(0.7, 0.9, 0, 5, True, 3)
    mid = SequenceState(handle=3, capacity=64, owner=st, prefill_only=True)
    outs = st.execute_mixed_batch([DecodeBatchItem(TokenInput([1]), 4, greedy),
                                   DecodeBatchItem(TokenInput([2, 3]), 0, mid),
                                   DecodeBatchItem(TokenInput([7]), 9, hot)])
    assert fake.calls == [(3, 2, 4)]
    assert outs[0].id == 1000 and outs[0].logprob is None
    assert outs[1] == backend.PrefillProgress()
    assert outs[2].id == 1002 and outs[2].logprob == -0.75
    assert outs[2].top_logprobs == [(20, 0.0), (21, -1.0), (22, -2.0)]
    assert (greedy.generated_index, hot.generated_index, mid.generated_index) == (0, 1, 0)
    # a non-final stage returns each row's slice of the boundary
    st2 = _stage(first=True, final=False)
    st2._lock, st2._h = threading.Lock(), C.c_void_p(1)
    a = SequenceState(handle=4, capacity=64, owner=st2)
    b = SequenceState(handle=5, capacity=64, owner=st2)
    outs = st2.execute_mixed_batch([DecodeBatchItem(TokenInput([1, 2]), 0, a),
                                    DecodeBatchItem(TokenInput([3]), 0, b)])
    h = CFG.hidden_size
    flat = (np.arange(3 * h) % 65000).astype(np.uint16)
    assert outs[0].tokens == 2 and outs[0].payload == flat[:2 * h].tobytes()
    assert outs[1].tokens == 1 and outs[1].payload == flat[2 * h:].tobytes()
