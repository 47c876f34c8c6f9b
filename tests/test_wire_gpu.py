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


def test_b200_worker_to_cpu_worker_over_the_wire():
    """Configuration 1 split as a B200 worker (layers 0-1) and a CPU worker
    (layers 2-3, the reference's CPU math as restated by the oracle), with the
    boundary carried as wire bytes: the B200 stage's device envelope, parsed and
    checked by the CPU side's decode_tensor restatement.  The greedy tokens are
    the reference's two-stage golden up to the first step whose top-2 logit gap
    is below 1e-2."""
    import numpy as np
    import os
    import oracle
    from oracle import envelope as O
    from tests.test_gpu_stage import GAP, GOLD, c1_spec, cfg_of, top2_gap
    from hllm_b200 import B200Stage
    from tests.gpu_util import torch_cuda

    torch_cuda()
    spec, seed = c1_spec()
    g = np.load(os.path.join(GOLD, "tiny_llama_pipeline.npz"))
    s0 = B200Stage(cfg_of(spec), 0, 2, first=True, final=False, kv_pool_tokens=4096)
    s0.init_synthetic(seed)
    cpu = oracle.OracleModel(spec, oracle.synth_weights(spec, seed), 2, 4)
    lens = g["prompt_lengths"]
    offs = np.concatenate([[0], np.cumsum(lens)])
    for r in range(4):
        prompt = [int(x) for x in g["prompt_ids"][offs[r]:offs[r + 1]]]
        ident = BoundaryIdentity("c1-plan", 1, f"request-{r}", len(prompt) + 32, spec.hidden_size)
        o_ident = O.Identity(b"c1-plan", 1, f"request-{r}".encode(), len(prompt) + 32,
                             spec.hidden_size)
        a = s0.allocate_sequence(len(prompt) + 32)
        b = cpu.new_sequence(len(prompt) + 32)
        inp, pos, agree = prompt, 0, True
        for step in range(32):
            s0.execute(TokenInput(inp), pos, a)
            wire = s0.encode_boundary(0, len(inp), ident, step, pos)
            off, tokens = O.decode_tensor(wire, o_ident, step, pos)
            assert tokens == len(inp)
            bits = np.frombuffer(wire, np.uint16, count=tokens * spec.hidden_size, offset=off)
            h = oracle.f16_decode(bits.reshape(tokens, spec.hidden_size))
            logits = cpu.logits(cpu.forward(h, pos, b)[-1:])[0]
            tok = int(np.argmax(logits))
            if agree:
                if top2_gap(logits) < GAP:
                    agree = False
                else:
                    assert tok == int(g["tokens"][r, step]), (r, step)
            pos += len(inp)
            inp = [tok]
        s0.release(a)
    s0.close()


def test_batched_envelopes_equal_per_row_host_encodings():
    """hllm_b200_stage_envelopes: one device->host copy for all rows of a
    decode batch, each message equal to encode_tensor of its row."""
    cfg, s0, s1 = _stages()
    prompts = [[1, 4, 2, 8, 3], [5, 6], [7], [9, 9, 9]]
    seqs = [s0.allocate_sequence(16) for _ in prompts]
    outs = s0.execute_mixed_batch([DecodeBatchItem(TokenInput(p), 0, q)
                                   for p, q in zip(prompts, seqs)])
    idents = [BoundaryIdentity("plan-1", 1, f"request-{i}" * (i + 1), 64, cfg.hidden_size)
              for i in range(len(prompts))]
    rows, off = [], 0
    for p, ident in zip(prompts, idents):
        rows.append((off, len(p), ident, 0, 0, False))
        off += len(p)
    got = s0.encode_boundaries(rows)
    assert got == [encode_tensor(o, ident, 0, 0) for o, ident in zip(outs, idents)]
    # one decode step later: sequence number 1, decode phase, one row each
    outs = s0.execute_mixed_batch([DecodeBatchItem(TokenInput([3]), len(p), q)
                                   for p, q in zip(prompts, seqs)])
    got = s0.encode_boundaries([(i, 1, ident, 1, len(p), False)
                                for i, (p, ident) in enumerate(zip(prompts, idents))])
    assert got == [encode_tensor(o, ident, 1, len(p))
                   for o, ident, p in zip(outs, idents, prompts)]
    s0.close()
    s1.close()
