"""Stage workloads at the other BASELINE configurations' shapes, component
timing, and the reference's profiling contract over the C++ adapter.

* Configuration 2 (Qwen3-0.6B geometry) as a two-stage split with chunked
  prefill and batched decode in the same mixed steps.
* Configuration 4 (Falcon3-3B geometry: d = 256, G = 3, untied head) with
  per-request seeded sampling and cancellation mid-decode that frees KV blocks
  and sequence slots for new requests.
* execute_profiled's components in the reference's taxonomy
  (cpp/src/cuda/stage.cpp:394-454) through the Python mirror, and the C++
  adapter under the reference's own contract headers (tests/cpp/
  decode_batch_contract.hpp and profiling_contract.hpp in the reference tree).

Bars as in test_gpu_stage.py: logits within 2e-2 of the F32 oracle on the
GPU's own token path, greedy tokens by the top-2 gap rule, sampled tokens
equal to the reference sampler's draw on the GPU's logits row.
"""
import os
import subprocess

import numpy as np
import pytest

import oracle
from hllm_b200 import (B200Stage, DecodeBatchItem, PrefillProgress, SamplingOptions, StageError,
                       TokenInput)
from hllm_b200 import _lib
from tests.gpu_util import torch_cuda
from tests.test_gpu_stage import GAP, LOGIT_TOL, cfg_of, make_stage, tiny_qwen, top2_gap

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ADAPTER = os.path.join(ROOT, "_build", "adapter_contract")


def test_execute_profiled_components_follow_the_reference_taxonomy():
    """execute_profiled (stage_backend.hpp:103-106) reports the components of
    cpp/src/cuda/stage.cpp:394-454 -- input, one "layer" per owned layer with
    its model index, then final norm / LM head / sampling or the boundary
    output -- and returns what execute returns."""
    cfg, weights, _ = tiny_qwen()
    s0 = make_stage(cfg, weights, layer_start=0, layer_end=1, first=True, final=False,
                    kv_pool_tokens=256)
    s1 = make_stage(cfg, weights, layer_start=1, layer_end=2, first=False, final=True,
                    kv_pool_tokens=256)
    a, b = s0.allocate_sequence(16), s0.allocate_sequence(16)
    c, d = s1.allocate_sequence(16), s1.allocate_sequence(16)
    ids = [1, 4, 2, 8, 3]
    for pos in (0, 3, 4):
        inp = TokenInput(ids[pos:pos + (3 if pos == 0 else 1)])
        plain = s0.execute(inp, pos, a)
        timed, parts = s0.execute_profiled(inp, pos, b)
        assert plain.payload == timed.payload
        assert [p[0] for p in parts] == ["embedding", "layer", "to-wire"]
        assert parts[1][1] == 0 and parts[0][1] is None
        assert all(np.isfinite(p[2]) and p[2] >= 0 for p in parts)
        out_plain = s1.execute(plain, pos, c)
        out_timed, parts = s1.execute_profiled(timed, pos, d)
        assert out_plain.id == out_timed.id
        assert [p[0] for p in parts] == ["from-wire", "layer", "final_norm", "lm_head",
                                          "sampling"]
        assert parts[1][1] == 1
    # timing is off again: a plain step records nothing new
    s0.execute(TokenInput([5]), 5, a)
    s0.close()
    s1.close()


FALCON3_3B = oracle.ModelSpec(hidden_size=3072, intermediate_size=9216, attention_heads=12,
                              key_value_heads=4, head_dimension=256, layers=22,
                              vocabulary_size=131072, maximum_sequence_length=2304,
                              rms_norm_epsilon=1e-6, rope_theta=1e6, query_key_norm=False,
                              tied=False)


def test_falcon3_geometry_seeded_sampling_with_cancellation_and_slot_reuse():
    """Configuration 4's shapes (h3072, 12q/4kv, d256, I9216, V131072, untied
    LM head), two layers, seeded synthetic weights.  Eight requests with their
    own seeds (temperature 0.7, top-p 0.9) prefill and then decode as one
    batch; after the third decode step a quarter of them are cancelled and
    released, and two new requests are admitted.  The pool and the sequence
    slots hold exactly eight requests, so the new ones run only in the freed
    KV blocks and slots.  Bars: every live row's logits at every step within
    2e-2 of the F32 oracle on the GPU's own token path (stale K/V in a reused
    block would break this), and every sampled token equal to the reference
    sampler's draw on the GPU's logits row with the request's seed and draw
    counter (sampling.cpp:65-90)."""
    spec = FALCON3_3B
    seed = 3303
    cap = 128
    torch_cuda()
    stage = B200Stage(cfg_of(spec), 0, 2, first=True, final=True, kv_pool_tokens=8 * cap,
                      max_sequences=8)
    stage.init_synthetic(seed)
    orc = oracle.OracleModel(spec, oracle.synth_weights(spec, seed, layers=range(2)), 0, 2)
    rng = np.random.default_rng(44)

    class Req:
        def __init__(self, rid):
            self.rid = rid
            self.prompt = [int(x) for x in rng.integers(0, spec.vocabulary_size,
                                                       int(rng.integers(16, 97)))]
            self.seq = stage.allocate_sequence(cap)
            self.seq.sampling = SamplingOptions(0.7, 0.9, 0, 1000 + rid, False, 0)
            self.oseq = orc.new_sequence(cap)
            self.pos = 0
            self.next = self.prompt

    live = [Req(r) for r in range(8)]
    with pytest.raises(StageError) as e:  # the pool is full
        stage.allocate_sequence(cap)
    assert e.value.code == _lib.RESOURCE_EXHAUSTED
    draws = 0
    for step in range(8):
        if step == 4:  # cancel a quarter mid-decode; their blocks and slots go back
            for r in (live[1], live[5]):
                stage.release(r.seq)
            live = [r for i, r in enumerate(live) if i not in (1, 5)]
            live += [Req(100), Req(101)]
        items = [DecodeBatchItem(TokenInput(r.next), r.pos, r.seq) for r in live]
        counters = [r.seq.generated_index for r in live]
        outs = stage.execute_mixed_batch(items)
        gpu = stage.read_logits(len(live))
        for i, (r, out) in enumerate(zip(live, outs)):
            ol = orc.logits(orc.forward(orc.embed(r.next), r.pos, r.oseq)[-1:])[0]
            err = float(np.max(np.abs(gpu[i] - ol)))
            assert err < LOGIT_TOL, (step, r.rid, err)
            opts = oracle.Sampling(0.7, 0.9, 0, 1000 + r.rid, 0, 0)
            st, want = oracle.sample_token(gpu[i], opts, counters[i])
            assert st == 0 and out.id == want.token_id, (step, r.rid)
            assert r.seq.generated_index == counters[i] + 1
            draws += 1
            r.pos += len(r.next)
            r.next = [out.id]
    assert draws == 8 * 8
    stage.close()


QWEN3_06B = oracle.ModelSpec(hidden_size=1024, intermediate_size=3072, attention_heads=16,
                             key_value_heads=8, head_dimension=128, layers=28,
                             vocabulary_size=151936, maximum_sequence_length=2048,
                             rms_norm_epsilon=1e-6, rope_theta=1e6, query_key_norm=True,
                             tied=True)


def test_qwen3_06b_geometry_two_stage_split_chunked_prefill_and_batched_decode():
    """Configuration 2's shapes (h1024, 16q/8kv, d128, I3072, V151936, tied,
    q/k-norm) as a two-stage split (layer 0 | layer 1, F16 boundary between the
    stages, as 14 | 14 splits the model).  Sixteen requests with prompts
    U[64, 1024) prefill in chunks of at most 256 tokens, all sixteen rows in
    one mixed step per tick; rows still inside their prompt do not sample, and
    requests past their prompt decode in the same steps."""
    spec = QWEN3_06B
    seed = 606
    chunk = 256
    torch_cuda()
    cfg = cfg_of(spec)
    s0 = B200Stage(cfg, 0, 1, first=True, final=False, kv_pool_tokens=16 * 1088,
                   max_step_tokens=16 * chunk)
    s1 = B200Stage(cfg, 1, 2, first=False, final=True, kv_pool_tokens=16 * 1088,
                   max_step_tokens=16 * chunk)
    s0.init_synthetic(seed)
    s1.init_synthetic(seed)
    weights = oracle.synth_weights(spec, seed, layers=range(2))
    o0 = oracle.OracleModel(spec, weights, 0, 1)
    o1 = oracle.OracleModel(spec, weights, 1, 2)
    rng = np.random.default_rng(66)
    reqs = []
    for _ in range(16):
        prompt = [int(x) for x in rng.integers(0, spec.vocabulary_size, int(rng.integers(64, 1024)))]
        cap = len(prompt) + 8
        reqs.append(dict(prompt=prompt, pos=0, next=None, agree=True,
                         a=s0.allocate_sequence(cap), b=s1.allocate_sequence(cap),
                         oa=o0.new_sequence(cap), ob=o1.new_sequence(cap)))
    sampled = 0
    for step in range(8):
        rows = []
        for q in reqs:
            if q["pos"] < len(q["prompt"]):
                inp = q["prompt"][q["pos"]:q["pos"] + chunk]
                samples = q["pos"] + len(inp) == len(q["prompt"])
            else:
                inp, samples = [q["next"]], True
            q["b"].prefill_only = not samples
            rows.append((q, inp, samples))
        bounds = s0.execute_mixed_batch([DecodeBatchItem(TokenInput(inp), q["pos"], q["a"])
                                         for q, inp, _ in rows])
        outs = s1.execute_mixed_batch([DecodeBatchItem(bd, q["pos"], q["b"])
                                       for bd, (q, _, _) in zip(bounds, rows)])
        gpu = s1.read_logits(sum(1 for r in rows if r[2]))
        k = 0
        for (q, inp, samples), out in zip(rows, outs):
            h = oracle.f16_round(o0.forward(o0.embed(inp), q["pos"], q["oa"]))
            last = o1.forward(h, q["pos"], q["ob"])[-1:]
            q["pos"] += len(inp)
            if not samples:
                assert out == PrefillProgress(), step
                continue
            ol = o1.logits(last)[0]
            err = float(np.max(np.abs(gpu[k] - ol)))
            assert err < LOGIT_TOL, (step, k, err)
            k += 1
            sampled += 1
            if q["agree"]:
                if top2_gap(ol) < GAP:
                    q["agree"] = False
                else:
                    assert out.id == int(np.argmax(ol)), step
            q["next"] = out.id
    assert sampled >= 16 * 4  # every request finished its prompt and decoded
    s0.close()
    s1.close()


def test_reference_contract_headers_over_the_adapter():
    """The reference's decode_batch_contract and paired_timing_contract,
    compiled from its tests/cpp headers into adapter_contract."""
    torch_cuda()
    if not os.path.exists(ADAPTER):
        pytest.skip("adapter contract not built (needs the reference tree at build time)")
    r = subprocess.run([ADAPTER, "reference"], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "reference contracts: ok" in r.stdout


def test_mixed_scheduler_over_the_adapter():
    """MixedStageScheduler (hllm_b200/adapter/mixed_scheduler.cpp) driving the
    C++ adapter from concurrent requests with chunked prompts: mixed passes
    form, and tokens equal serial runs up to the first near-tie."""
    torch_cuda()
    if not os.path.exists(ADAPTER):
        pytest.skip("adapter contract not built (needs the reference tree at build time)")
    r = subprocess.run([ADAPTER, "mixed"], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "mixed scheduler contract: ok" in r.stdout


def test_stage_memory_tracks_kv_blocks():
    """hllm_b200_stage_memory (BackendFactory::allocator_metrics): the KV bytes
    held by live sequences follow allocation and release in whole 16-token
    blocks, and the peak stays."""
    cfg, weights, _ = tiny_qwen()
    s = make_stage(cfg, weights, kv_pool_tokens=256)
    m0 = s.memory()
    assert m0["weights"] > 0 and m0["workspace"] > 0 and m0["kv_in_use"] == 0
    block = m0["kv_pool"] // (256 // 16)
    # The fixture's context is 32 tokens: at most two blocks per sequence.
    a = s.allocate_sequence(30)  # 2 blocks
    b = s.allocate_sequence(16)  # 1 block
    m1 = s.memory()
    assert m1["kv_in_use"] == 3 * block and m1["kv_peak"] == 3 * block
    s.release(a)
    m2 = s.memory()
    assert m2["kv_in_use"] == block and m2["kv_peak"] == 3 * block
    assert m2["weights"] == m0["weights"] and m2["kv_pool"] == m0["kv_pool"]
    s.release(b)
    s.close()
