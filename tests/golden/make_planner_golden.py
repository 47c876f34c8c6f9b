"""Writes tests/golden/planner_cases.json from the reference planner.

Run in a checkout that has the reference project next to it:

    python tests/golden/make_planner_golden.py <reference root>

For each model shape (Qwen3-4B, Falcon3-3B and the reference tests' tiny
Llama, tied and untied) it writes a sparse Safetensors file, prepares the
manifest with the reference's prepare_model
(python/hllm_control/prepare/manifest.py:99), and records
  * the manifest's tensor records as (role, layer index, elements) and the
    config fields the planner reads;
  * the reference's per-stage memory (_stage_memory, planner.py:73-129) for
    every contiguous two-way split and for the whole model on one stage, for
    each (worker, workload) pair below;
  * the candidate the reference's create_plan (planner.py:246) selects for
    two identical workers in feasibility mode, with its score.
tests/test_planner.py checks hllm_b200.planner against these numbers.  The
reference imports its gRPC stubs at import time; the control stub is replaced
by an empty module here because the planner never calls it.
"""
from __future__ import annotations

import json
import struct
import sys
import tempfile
import types
from pathlib import Path

OUT = Path(__file__).with_name("planner_cases.json")

GIB = 1024 ** 3


def write_sparse_safetensors(path: Path, tensors: dict, dtype_bytes: dict) -> None:
    offset = 0
    header: dict = {"__metadata__": {"format": "pt"}}
    for name, (dtype, shape) in tensors.items():
        n = 1
        for dim in shape:
            n *= dim
        length = n * dtype_bytes[dtype]
        header[name] = {"dtype": dtype, "shape": list(shape),
                        "data_offsets": [offset, offset + length]}
        offset += length
    raw = json.dumps(header, separators=(",", ":")).encode()
    raw += b" " * (-len(raw) % 8)
    prefix = struct.pack("<Q", len(raw)) + raw
    with path.open("wb") as f:
        f.write(prefix)
        if offset:
            f.seek(len(prefix) + offset - 1)
            f.write(b"\0")


def llama_tensors(dtype, layers, h, inter, hq, hkv, d, vocab, tied, qk_norm):
    t = {"model.embed_tokens.weight": (dtype, (vocab, h)),
         "model.norm.weight": (dtype, (h,))}
    if not tied:
        t["lm_head.weight"] = (dtype, (vocab, h))
    for i in range(layers):
        p = f"model.layers.{i}"
        t.update({
            f"{p}.input_layernorm.weight": (dtype, (h,)),
            f"{p}.post_attention_layernorm.weight": (dtype, (h,)),
            f"{p}.self_attn.q_proj.weight": (dtype, (hq * d, h)),
            f"{p}.self_attn.k_proj.weight": (dtype, (hkv * d, h)),
            f"{p}.self_attn.v_proj.weight": (dtype, (hkv * d, h)),
            f"{p}.self_attn.o_proj.weight": (dtype, (h, hq * d)),
            f"{p}.mlp.gate_proj.weight": (dtype, (inter, h)),
            f"{p}.mlp.up_proj.weight": (dtype, (inter, h)),
            f"{p}.mlp.down_proj.weight": (dtype, (h, inter)),
        })
        if qk_norm:
            t[f"{p}.self_attn.q_norm.weight"] = (dtype, (d,))
            t[f"{p}.self_attn.k_norm.weight"] = (dtype, (d,))
    return dict(sorted(t.items()))


MODELS = {
    "qwen3_4b": dict(
        config={"architectures": ["Qwen3ForCausalLM"], "model_type": "qwen3",
                "hidden_size": 2560, "intermediate_size": 9728, "num_hidden_layers": 36,
                "num_attention_heads": 32, "num_key_value_heads": 8, "head_dim": 128,
                "vocab_size": 151936, "max_position_embeddings": 40960,
                "tie_word_embeddings": True, "rms_norm_eps": 1e-6,
                "rope_theta": 1000000.0, "eos_token_id": 151645},
        tensors=lambda: llama_tensors("F16", 36, 2560, 9728, 32, 8, 128, 151936, True, True)),
    "falcon3_3b": dict(
        config={"architectures": ["LlamaForCausalLM"], "model_type": "llama",
                "hidden_size": 3072, "intermediate_size": 9216, "num_hidden_layers": 22,
                "num_attention_heads": 12, "num_key_value_heads": 4, "head_dim": 256,
                "vocab_size": 131072, "max_position_embeddings": 32768,
                "tie_word_embeddings": False},
        tensors=lambda: llama_tensors("BF16", 22, 3072, 9216, 12, 4, 256, 131072, False, False)),
    "tiny": dict(
        config={"architectures": ["LlamaForCausalLM"], "model_type": "llama",
                "hidden_size": 8, "intermediate_size": 16, "num_hidden_layers": 4,
                "num_attention_heads": 4, "num_key_value_heads": 2, "head_dim": 2,
                "vocab_size": 16, "max_position_embeddings": 128,
                "tie_word_embeddings": False, "rms_norm_eps": 1e-5,
                "rope_theta": 500000.0, "eos_token_id": [2, 3]},
        tensors=lambda: llama_tensors("F16", 4, 8, 16, 4, 2, 2, 16, False, False)),
    "tiny_tied": dict(
        config={"architectures": ["LlamaForCausalLM"], "model_type": "llama",
                "hidden_size": 8, "intermediate_size": 16, "num_hidden_layers": 4,
                "num_attention_heads": 4, "num_key_value_heads": 2, "head_dim": 2,
                "vocab_size": 16, "max_position_embeddings": 128,
                "tie_word_embeddings": True, "rms_norm_eps": 1e-5,
                "rope_theta": 500000.0, "eos_token_id": [2, 3]},
        tensors=lambda: llama_tensors("F16", 4, 8, 16, 4, 2, 2, 16, True, False)),
}

# Worker profiles (field names of the reference WorkerProfile, models.py:222).
WORKERS = {
    # One B200: 183,359 MiB of HBM3e, 2 GiB kept for the driver and context.
    "b200": dict(worker_id="b200", endpoint="b200-host:50051", backend="cuda",
                 primary_memory_domain="DEVICE",
                 supported_architectures=["llama.v1", "qwen3.v1"],
                 supported_execution_dtypes=["F16", "F32"],
                 memory_budgets=[dict(domain="DEVICE", capacity_bytes=183359 * 1024 * 1024,
                                      runtime_reserve_bytes=2 * GIB, safety_fraction=0.05)],
                 fixed_workspace_bytes=4 * GIB, activation_buffer_count=2,
                 allocator_allowance_fraction=0.05, host_transport_buffer_bytes=64 * 1024 * 1024),
    # The reference's own example CUDA worker (examples/profiles/workers-m3pro-3060ti.yaml).
    "rtx3060ti": dict(worker_id="rtx-3060-ti", endpoint="cuda-host:50051", backend="cuda",
                      primary_memory_domain="DEVICE",
                      supported_architectures=["llama.v1", "qwen3.v1"],
                      supported_execution_dtypes=["F16"],
                      memory_budgets=[dict(domain="DEVICE", capacity_bytes=8 * GIB,
                                           runtime_reserve_bytes=805306368, safety_fraction=0.10),
                                      dict(domain="HOST", capacity_bytes=16 * GIB,
                                           runtime_reserve_bytes=4 * GIB, safety_fraction=0.10)],
                      fixed_workspace_bytes=512 * 1024 * 1024, activation_buffer_count=2,
                      allocator_allowance_fraction=0.05, host_transport_buffer_bytes=64 * 1024 * 1024),
    # A unified-memory worker: transport buffers count against the stage's budget.
    "unified": dict(worker_id="mac", endpoint="mac-host:50051", backend="mlx",
                    primary_memory_domain="UNIFIED",
                    supported_architectures=["llama.v1", "qwen3.v1"],
                    supported_execution_dtypes=["F16"],
                    memory_budgets=[dict(domain="UNIFIED", capacity_bytes=18 * GIB,
                                         runtime_reserve_bytes=4 * GIB, safety_fraction=0.10)],
                    fixed_workspace_bytes=512 * 1024 * 1024, activation_buffer_count=2,
                    allocator_allowance_fraction=0.05, host_transport_buffer_bytes=64 * 1024 * 1024),
}

WORKLOADS = {
    # examples/workloads/interactive.yaml
    "interactive": dict(workload_id="interactive-512-256", prompt_tokens=512, output_tokens=256,
                        concurrency=1, total_cached_tokens=32768, kv_overhead_factor=1.10,
                        kv_dtype="F16", activation_dtype="F16"),
    # 64 concurrent requests with prompts up to 4,096 and outputs up to 512 tokens.
    "batch64": dict(workload_id="batch-64", prompt_tokens=512, output_tokens=512,
                    concurrency=64, total_cached_tokens=64 * 4608, kv_overhead_factor=1.10,
                    kv_dtype="F16", activation_dtype="F16", prefill_chunk_tokens=256),
}

PAIRS = [("qwen3_4b", "b200", "interactive"), ("qwen3_4b", "b200", "batch64"),
         ("qwen3_4b", "rtx3060ti", "interactive"), ("qwen3_4b", "unified", "interactive"),
         ("falcon3_3b", "b200", "batch64"), ("falcon3_3b", "rtx3060ti", "interactive"),
         ("tiny", "b200", "interactive"), ("tiny_tied", "unified", "batch64")]


def main(reference: Path) -> None:
    sys.path.insert(0, str(reference / "python"))
    sys.modules["hllm_control.proto.control_pb2_grpc"] = types.ModuleType("control_pb2_grpc")
    from hllm_control.models import (DTYPE_BYTES, PlannerSettings, WorkerProfile,
                                     WorkloadProfile)
    from hllm_control.planner import planner as P
    from hllm_control.prepare.manifest import prepare_model

    dtype_bytes = {d.value: n for d, n in DTYPE_BYTES.items()}
    out = {"models": {}, "cases": []}
    manifests = {}
    with tempfile.TemporaryDirectory() as tmp:
        for name, spec in MODELS.items():
            path = Path(tmp) / name
            path.mkdir()
            (path / "config.json").write_text(json.dumps(spec["config"]), encoding="utf-8")
            write_sparse_safetensors(path / "model.safetensors", spec["tensors"](), dtype_bytes)
            m = prepare_model(path, model_id=f"{name}-shape-fixture")
            manifests[name] = m
            c = m.config
            out["models"][name] = {
                "config": {"num_layers": c.num_layers, "hidden_size": c.hidden_size,
                           "num_kv_heads": c.num_kv_heads, "head_dim": c.head_dim,
                           "vocabulary_size": c.vocabulary_size,
                           "tied_embeddings": c.tied_embeddings},
                "tensors": [[t.role.value, t.layer_index, t.num_elements] for t in m.tensors],
            }

    settings = PlannerSettings()
    for model, wname, lname in PAIRS:
        m = manifests[model]
        worker = WorkerProfile(**WORKERS[wname])
        workload = WorkloadProfile(**WORKLOADS[lname])
        L = m.config.num_layers

        def mem(start, end, first, final):
            s = P._stage_memory(m, worker, workload, settings, start=start, end=end,
                                is_first=first, is_final=final)
            return s.model_dump(mode="json")

        splits = {str(k): [mem(0, k, True, False), mem(k, L, False, True)] for k in range(1, L)}
        whole = mem(0, L, True, True)
        twin = worker.model_copy(update={"worker_id": worker.worker_id + "-b"})
        report = P.create_plan(m, (worker, twin), (), workload, settings)
        chosen = None
        if report.plan is not None:
            sel = next(c for c in report.candidates if c.candidate_id == report.selected_candidate_id)
            chosen = {"split_layer": sel.split_layer, "score": sel.score,
                      "stage_zero_worker_id": sel.stage_zero_worker_id}
        out["cases"].append({"model": model, "worker": WORKERS[wname], "workload": WORKLOADS[lname],
                             "splits": splits, "whole": whole, "selected": chosen,
                             "feasible_candidates": sum(c.feasible for c in report.candidates)})
    OUT.write_text(json.dumps(out, sort_keys=True, separators=(",", ":")) + "\n",
                   encoding="utf-8")
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(out['cases'])} cases)")


if __name__ == "__main__":
    main(Path(sys.argv[1]) if len(sys.argv) > 1 else Path("../reference"))
