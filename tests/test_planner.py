"""hllm_b200.planner against the reference planner's own numbers.

tests/golden/planner_cases.json holds, for Qwen3-4B, Falcon3-3B and the
reference tests' tiny Llama (tied and untied) on three worker profiles and two
workloads, the reference's _stage_memory (python/hllm_control/planner/
planner.py:73-129) for every two-way split and for the whole model, and the
split its create_plan (planner.py:246) selects for two identical workers
(written by tests/golden/make_planner_golden.py).
"""
from __future__ import annotations

import itertools
import json
import os
import random

import pytest

from hllm_b200 import planner as P
from hllm_b200.pipeline import partition_layers

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "planner_cases.json")


@pytest.fixture(scope="module")
def gold():
    with open(GOLD, encoding="utf-8") as f:
        return json.load(f)


def shape_of(gold, name):
    return P.ModelShape.from_manifest(gold["models"][name])


def case(gold, model, worker, workload):
    return next(c for c in gold["cases"] if c["model"] == model and
                c["worker"]["worker_id"] == worker and c["workload"]["workload_id"] == workload)


def test_stage_memory_equals_the_reference_on_every_split(gold):
    checked = 0
    for c in gold["cases"]:
        shape = shape_of(gold, c["model"])
        L = shape.num_layers
        for k, (first, final) in c["splits"].items():
            k = int(k)
            assert P.stage_memory(shape, c["worker"], c["workload"], start=0, end=k,
                                  is_first=True, is_final=False) == first
            assert P.stage_memory(shape, c["worker"], c["workload"], start=k, end=L,
                                  is_first=False, is_final=True) == final
            assert P.stage_weight_bytes(shape, start=0, end=k, is_first=True,
                                        is_final=False) == first["weight_bytes"]
            checked += 2
        assert P.stage_memory(shape, c["worker"], c["workload"], start=0, end=L,
                              is_first=True, is_final=True) == c["whole"]
    assert checked > 200


def test_pressure_split_on_two_gpus_is_the_reference_selection(gold):
    for c in gold["cases"]:
        shape = shape_of(gold, c["model"])
        if c["selected"] is None:
            with pytest.raises(P.NoFeasibleSplit):
                P.split_stage(shape, c["worker"], c["workload"], 2, objective="pressure")
            continue
        k = c["selected"]["split_layer"]
        assert P.split_stage(shape, c["worker"], c["workload"], 2, objective="pressure") == \
            [(0, k), (k, shape.num_layers)]
        plan = P.plan_worker(shape, c["worker"], c["workload"], 2, objective="pressure")
        ref = c["splits"][str(k)]
        assert [g["memory"]["required_bytes"] for g in plan["gpus"]] == \
            [s["required_bytes"] for s in ref]
        assert plan["max_pressure"] == max(s["pressure"] for s in ref)


def test_infeasible_worker_reports_the_reference_reason_per_gpu(gold):
    c = case(gold, "qwen3_4b", "rtx-3060-ti", "interactive-512-256")
    shape = shape_of(gold, "qwen3_4b")
    one = P.plan_worker(shape, c["worker"], c["workload"], 1)
    assert not one["feasible"]
    assert one["rejection_reasons"] == ["DEVICE_MEMORY_EXCEEDED:rtx-3060-ti/gpu0"]
    assert one["gpus"][0]["memory"] == {**c["whole"], "worker_id": "rtx-3060-ti/gpu0"}
    # Enough GPUs of the same kind hold it.
    fits = [g for g in range(1, 9)
            if P.plan_worker(shape, c["worker"], c["workload"], g)["feasible"]]
    assert fits and fits == list(range(fits[0], 9))


def test_qwen3_4b_on_b200_gpus(gold):
    c = case(gold, "qwen3_4b", "b200", "batch-64")
    shape = shape_of(gold, "qwen3_4b")
    h, V = shape.hidden_size, shape.vocabulary_size
    layer_bytes = P.stage_weight_bytes(shape, start=0, end=1, is_first=False, is_final=False)
    periods = []
    for g in (1, 2, 4, 8):
        plan = P.plan_worker(shape, c["worker"], c["workload"], g)
        assert plan["feasible"] and plan["rejection_reasons"] == []
        gpus = plan["gpus"]
        assert [x["gpu"] for x in gpus] == list(range(g))
        assert gpus[0]["layer_start"] == 0 and gpus[-1]["layer_end"] == 36
        assert all(a["layer_end"] == b["layer_start"] for a, b in zip(gpus, gpus[1:]))
        assert [x["owns_token_embedding"] for x in gpus] == [True] + [False] * (g - 1)
        for flag in ("owns_final_norm", "owns_lm_head", "owns_sampling"):
            assert [x[flag] for x in gpus] == [False] * (g - 1) + [True]
        # Tied embeddings: resident on the first GPU and again on the last.
        total = sum(x["memory"]["weight_bytes"] for x in gpus)
        whole = c["whole"]["weight_bytes"]
        assert total == whole + (V * h * 2 if g > 1 else 0)
        periods.append(plan["period_bytes"])
        # Weights alone (no KV term): the split the pipeline bench runs.
        weights_only = P.plan_worker(shape, c["worker"], c["workload"], g, kv_tokens=0)
        assert P.ranges_of(weights_only) == partition_layers(36, g, layer_bytes, V * h * 2)
    assert periods == sorted(periods, reverse=True)


def test_a_reference_stage_assignment_splits_inside_its_range(gold):
    c = case(gold, "falcon3_3b", "b200", "batch-64")
    shape = shape_of(gold, "falcon3_3b")
    k = c["selected"]["split_layer"]
    second = {"stage_index": 1, "worker_id": "b200", "layer_start": k, "layer_end": 22,
              "owns_token_embedding": False, "owns_final_norm": True, "owns_lm_head": True,
              "owns_sampling": True}
    plan = P.plan_worker(shape, c["worker"], c["workload"], 3, assignment=second)
    assert plan["stage_index"] == 1 and plan["layer_start"] == k and plan["layer_end"] == 22
    gpus = plan["gpus"]
    assert gpus[0]["layer_start"] == k and gpus[-1]["layer_end"] == 22
    assert not any(x["owns_token_embedding"] for x in gpus)
    assert [x["owns_lm_head"] for x in gpus] == [False, False, True]
    for x in gpus:
        final = x["gpu"] == 2
        want = P.stage_memory(shape, c["worker"], c["workload"], start=x["layer_start"],
                              end=x["layer_end"], is_first=False, is_final=final,
                              worker_id=f"b200/gpu{x['gpu']}")
        assert x["memory"] == want
    # One GPU for the stage: the reference's own record for that stage.
    one = P.plan_worker(shape, c["worker"], c["workload"], 1, assignment=second)
    assert one["gpus"][0]["memory"] == {**c["splits"][str(k)][1], "worker_id": "b200/gpu0"}


def test_split_costs_is_the_most_even_least_maximum():
    rng = random.Random(7)
    for _ in range(300):
        n = rng.randint(1, 9)
        parts = rng.randint(1, n)
        w = [rng.choice([1.0, 2.0, 3.0, rng.random() * 4]) for _ in range(n)]
        tail = rng.choice([0.0, 1.5, 5.0])
        cost = lambda g, s, e: sum(w[s:e]) + (tail if g == parts - 1 else 0.0)  # noqa: E731
        got = P.split_costs(0, n, parts, cost)
        assert got[0][0] == 0 and got[-1][1] == n and len(got) == parts
        assert all(e > s for s, e in got)
        best = None
        for cuts in itertools.combinations(range(1, n), parts - 1):
            edges = (0,) + cuts + (n,)
            cs = [cost(g, edges[g], edges[g + 1]) for g in range(parts)]
            key = (max(cs), sum(x * x for x in cs))
            best = key if best is None or key < best else best
        cs = [cost(g, s, e) for g, (s, e) in enumerate(got)]
        assert max(cs) == pytest.approx(best[0], rel=1e-12)
        assert sum(x * x for x in cs) == pytest.approx(best[1], rel=1e-9)


def test_split_costs_never_uses_a_forbidden_range():
    # Part 0 may hold at most two layers; part 1 at most four.
    cost = lambda g, s, e: float("inf") if (e - s) > (2 if g == 0 else 4) else 1.0  # noqa: E731
    assert P.split_costs(0, 6, 2, cost) == [(0, 2), (2, 6)]
    with pytest.raises(P.PlanningError):
        P.split_costs(0, 7, 2, cost)


def test_planner_input_errors(gold):
    c = case(gold, "tiny", "b200", "interactive-512-256")
    shape = shape_of(gold, "tiny")
    with pytest.raises(P.PlanningError):
        P.plan_worker(shape, c["worker"], c["workload"], 0)
    with pytest.raises(P.PlanningError):
        P.plan_worker(shape, c["worker"], c["workload"], 5)  # 4 layers
    with pytest.raises(P.PlanningError):
        P.plan_worker(shape, c["worker"], c["workload"], 1,
                      assignment={"stage_index": 0, "layer_start": 3, "layer_end": 9,
                                  "owns_token_embedding": False, "owns_final_norm": True,
                                  "owns_lm_head": True, "owns_sampling": True})
    with pytest.raises(P.PlanningError):
        P.split_stage(shape, c["worker"], c["workload"], 2, objective="latency")
    with pytest.raises(P.PlanningError):
        P.plan_worker(shape, c["worker"], c["workload"], 2, objective="latency")
    homeless = {**c["worker"], "primary_memory_domain": "UNIFIED"}
    with pytest.raises(P.PlanningError):
        P.stage_memory(shape, homeless, c["workload"], start=0, end=4, is_first=True,
                       is_final=True)


def test_manifest_json_form_reads_like_the_compact_one(gold):
    compact = gold["models"]["tiny_tied"]
    full = {"config": dict(compact["config"], intermediate_size=16, num_attention_heads=4),
            "tensors": [{"name": f"t{i}", "role": role, "layer_index": layer,
                         "shape": [n], "dtype": "F16"}
                        for i, (role, layer, n) in enumerate(compact["tensors"])]}
    assert P.ModelShape.from_manifest(full) == P.ModelShape.from_manifest(compact)


def test_object_inputs_read_like_dicts(gold):
    """The reference's pydantic models (ModelManifest, WorkerProfile,
    WorkloadProfile, StageAssignment) are read by attribute, their StrEnum
    fields by value: the same plan as from the JSON forms."""
    from types import SimpleNamespace as NS

    class Role:  # a StrEnum member stand-in: compared by .value
        def __init__(self, v):
            self.value = v

    compact = gold["models"]["falcon3_3b"]
    manifest = NS(config=NS(**compact["config"]),
                  tensors=[NS(role=Role(r), layer_index=li, num_elements=n)
                           for r, li, n in compact["tensors"]])
    c = case(gold, "falcon3_3b", "b200", "batch-64")
    worker = NS(**{**c["worker"], "primary_memory_domain": Role("DEVICE"),
                   "memory_budgets": [NS(**{**b, "domain": Role(b["domain"])})
                                      for b in c["worker"]["memory_budgets"]]})
    workload = NS(**{**c["workload"], "kv_dtype": Role("F16"), "activation_dtype": Role("F16")})
    stage = NS(stage_index=1, worker_id="b200", layer_start=11, layer_end=22,
               owns_token_embedding=False, owns_final_norm=True, owns_lm_head=True,
               owns_sampling=True)
    shape = P.ModelShape.from_manifest(manifest)
    assert shape == shape_of(gold, "falcon3_3b")
    a = P.plan_worker(shape, worker, workload, 2, assignment=stage)
    b = P.plan_worker(shape, c["worker"], c["workload"], 2, assignment=vars(stage))
    assert a == b and a["feasible"]
