"""bench.py's per-phase roofline arithmetic (decode-only steps against HBM,
steps carrying a prefill chunk against the tensor roof), on the CPU, against
the Qwen3-4B figures: 201.85 MB of F16 weights per layer, a 777.9 MB head,
147,456 bytes of K/V per token over 36 layers, 7.267 GFLOP per token."""
import pytest

import bench


def test_step_work_matches_the_configuration_3_formulas():
    layer, head = bench.qwen_stage_bytes()
    assert layer == pytest.approx(201.85e6, rel=1e-3) and head == pytest.approx(777.9e6, rel=1e-3)
    dec = [(999, 1, True)] * 64  # 64 decode rows with 1,000 keys each
    nbytes, flops = bench.step_work(dec)
    ctx = 64 * 1000
    expect = 36 * layer + head + 147456 * ctx + 64 * 147456 + 64 * 2560 * 4
    assert nbytes == pytest.approx(expect, rel=1e-9)
    expect_flops = 64 * 7.267e9 + 4 * 32 * 128 * 36 * ctx + 64 * 2 * 151936 * 2560
    assert flops == pytest.approx(expect_flops, rel=2e-3)
    # a 512-token chunk at position 0: 512 * 513 / 2 causal pairs
    _, f = bench.step_work([(0, 512, True)])
    assert f == pytest.approx(512 * 7.267e9 + 4 * 32 * 128 * 36 * (512 * 513 // 2)
                              + 2 * 151936 * 2560, rel=2e-3)


def test_phase_summary_splits_decode_and_prefill_steps():
    dec = [(999, 1, True)] * 64
    pre = [(999, 1, True)] * 63 + [(0, 512, True)]
    out = bench.phase_summary([(dec, True), (pre, False), (dec, True)], [5.0, 10.0, 6.0],
                              6650.0, 1400.0)
    assert out["decode"]["steps"] == 2 and out["prefill"]["steps"] == 1
    assert out["decode"]["ms_per_step"] == 5.5 and out["decode"]["bound"] == "hbm"
    b = bench.step_work(dec)[0]
    assert out["decode"]["achieved"] == pytest.approx(2 * b / 11e-3 / 1e9, rel=1e-3)
    assert out["prefill"]["bound"] == "tensor"
    assert out["prefill"]["tokens_per_s"] == pytest.approx(575 / 10e-3, rel=1e-3)
    assert bench.phase_summary([(dec, True)], [5.0], 6650.0, 1400.0).keys() == {"decode"}


def test_pipeline_split_is_the_measured_one_and_fits():
    """bench.py's N-GPU split comes from the planner (Qwen3-4B geometry, the
    configuration-3 workload, one B200's budget per rank).  Its most-loaded rank
    streams what the uniform-layer split's does (LM head = V*h bytes on the
    last rank); at the scaling run's 1, 2, 4 and 8 GPUs the ranges are the
    same ones, so the measured configurations are unchanged.  (At 6 and 7 the
    planner also counts the first rank's embedding rows and breaks a tie the
    other way.)  Every rank fits its memory."""
    from hllm_b200.pipeline import partition_layers, stage_bytes
    layer, head = bench.qwen_stage_bytes()
    for world in range(1, 9):
        plan = bench.pipeline_plan(world)
        ours, uniform = bench.pipeline_ranges(world), partition_layers(36, world, layer, head)
        assert max(stage_bytes(ours, layer, head)) == max(stage_bytes(uniform, layer, head))
        if world in (1, 2, 4, 8):
            assert ours == uniform
        assert plan["feasible"] and len(plan["gpus"]) == world
        assert all(0 < g["memory"]["pressure"] < 1 for g in plan["gpus"])
    assert bench.pipeline_ranges(8)[-1] == (35, 36)


def test_geometry_shape_equals_the_prepared_manifest():
    """shape_from_geometry(Qwen3-4B) gives the reference prepare_model's tensor
    bytes per stage (tests/golden/planner_cases.json, Qwen3-4B manifest)."""
    import json
    import os
    from hllm_b200 import planner as P
    from hllm_b200.workload import QWEN3_4B
    path = os.path.join(os.path.dirname(__file__), "golden", "planner_cases.json")
    with open(path, encoding="utf-8") as f:
        gold = json.load(f)
    ref = P.ModelShape.from_manifest(gold["models"]["qwen3_4b"])
    ours = P.shape_from_geometry(**QWEN3_4B)
    assert (ours.num_layers, ours.hidden_size, ours.num_kv_heads, ours.head_dim,
            ours.vocabulary_size, ours.tied_embeddings) == \
        (ref.num_layers, ref.hidden_size, ref.num_kv_heads, ref.head_dim, ref.vocabulary_size,
         ref.tied_embeddings)
    for s, e in ((0, 1), (0, 36), (5, 17), (35, 36)):
        for first in (False, True):
            for final in (False, True):
                assert P.stage_weight_bytes(ours, start=s, end=e, is_first=first,
                                            is_final=final) == \
                    P.stage_weight_bytes(ref, start=s, end=e, is_first=first, is_final=final)
