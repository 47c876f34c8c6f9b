"""The boundary envelope built from device memory (hllm_b200_stage_envelope)
against the host codec on the same rows, and its ordering against later steps.

A tiny Qwen3 model runs as stage 0 (layer 0, embeds) and stage 1 (layer 1,
samples).  The bar: the envelope of each row of stage 0's last boundary,
copied device->host into the message, equals hllm_b200_envelope_encode of the
boundary that hllm_b200_step returned for that row, byte for byte; decoding it
and feeding stage 1 gives the token that the boundary itself gives; and an
envelope issued before the next step still holds the earlier step's rows."""
import ctypes as C

import pytest

from hllm_b200 import DecodeBatchItem, TokenInput, _lib
from hllm_b200.wire import BoundaryIdentity, decode_tensor, encode_tensor
from tests.test_gpu_stage import make_stage, tiny_qwen

pytestmark = pytest.mark.gpu


def _stages():
    cfg, weights, _ = tiny_qwen()
    s0 = make_stage(cfg, weights, layer_start=0, layer_end=1, first=True, final=False,
                    kv_pool_tokens=256)
    s1 = make_stage(cfg, weights, layer_start=1, layer_end=2, first=False, final=True,
                    kv_pool_tokens=256)
    return cfg, s0, s1


def test_device_envelopes_equal_host_encoding_and_feed_the_next_stage():
    cfg, s0, s1 = _stages()
    ident = BoundaryIdentity("plan-1", 1, "request-1", 64, cfg.hidden_size)
    prompts = [[1, 4, 2, 8, 3], [5, 6], [7]]
    q0 = [s0.allocate_sequence(16) for _ in prompts]
    q1 = [s1.allocate_sequence(16) for _ in prompts]
    outs = s0.execute_mixed_batch([DecodeBatchItem(TokenInput(p), 0, q)
                                   for p, q in zip(prompts, q0)])
    off = 0
    direct, via_wire = [], []
    for p, o, q in zip(prompts, outs, q1):
        dev = s0.encode_boundary(off, len(p), ident, 0, 0)
        assert dev == encode_tensor(o, ident, 0, 0)
        back = decode_tensor(dev, ident, 0, 0)
        assert back.payload == o.payload
        via_wire.append(DecodeBatchItem(back, 0, q))
        off += len(p)
    direct = [r.id for r in s1.execute_mixed_batch(via_wire)]
    q2 = [s1.allocate_sequence(16) for _ in prompts]
    again = [r.id for r in s1.execute_mixed_batch([DecodeBatchItem(o, 0, q)
                                                   for o, q in zip(outs, q2)])]
    assert direct == again
    with pytest.raises(_lib.StageError):  # rows past the last step's boundary
        s0.encode_boundary(off - 1, 2, ident, 0, 0)
    with pytest.raises(_lib.StageError):  # a final stage has no boundary
        s1.encode_boundary(0, 1, ident, 0, 0)
    s0.close()
    s1.close()


def test_envelope_issued_before_the_next_step_keeps_its_rows():
    torch = pytest.importorskip("torch")
    cfg, s0, s1 = _stages()
    ident = BoundaryIdentity("plan-1", 1, "request-1", 64, cfg.hidden_size)
    q = s0.allocate_sequence(16)
    first = s0.execute_mixed_batch([DecodeBatchItem(TokenInput([1, 4, 2, 8, 3]), 0, q)])[0]
    c_ident = ident.c()
    n = C.c_uint64()
    L = _lib.lib()
    _lib.check(L.hllm_b200_stage_envelope(s0.handle, 0, 5, C.byref(c_ident), 0, 0, 0, None, 0,
                                          C.byref(n)))
    out = torch.empty(n.value, dtype=torch.uint8, pin_memory=True)
    _lib.check(L.hllm_b200_stage_envelope(s0.handle, 0, 5, C.byref(c_ident), 0, 0, 0,
                                          out.data_ptr(), n.value, C.byref(n)))
    # the next steps overwrite the boundary buffer after the copy has read it
    second = s0.execute_mixed_batch([DecodeBatchItem(TokenInput([9]), 5, q)])[0]
    s0.execute_mixed_batch([DecodeBatchItem(TokenInput([2]), 6, q)])
    _lib.check(L.hllm_b200_stage_envelope_wait(s0.handle))
    got = bytes(out.numpy())
    assert got == encode_tensor(first, ident, 0, 0)
    assert second.payload != first.payload[:len(second.payload)]
    s0.close()
    s1.close()
