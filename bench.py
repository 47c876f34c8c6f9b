#!/usr/bin/env python
"""Benchmark of the B200 stage executor on hLLM's Qwen3-4B configuration.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (configuration 3): Qwen3-4B architecture (36 layers, h2560, 32q/8kv,
d128, I9728, V151936, tied, q/k-norm, theta 1e6), seeded random-init F16
weights, continuous batching of 64 concurrent requests, prompt lengths
log-normal(median 512, sigma 1) in [32, 4096], output lengths U[64, 512],
512-token prefill chunks mixed into the decode batch, greedy decoding (see
hllm_b200/workload.py).  A step is one pass of the stage executor over one
mixed batch (every running sequence's decode token plus up to 512 prefill
tokens).  Before warm-up the trace is fast-forwarded (untimed) past the
start-up ramp to the steady state.

Arms and numbers:
  value  -- tokens (prefill + decode) per second with the step inputs already
            in HBM: all steps' token ids are uploaded before the timed region
            and steps are enqueued back to back (hllm_b200_step_async); CUDA
            events on the executor's stream around exactly K steps.
  e2e    -- the same steps through the public call (hllm_b200_step via
            B200Stage.execute_mixed_batch): per step the row descriptors and
            token ids go host->device from pinned memory and the sampled
            tokens come back device->host and feed the next step.
  --impl reference -- the reference's own CPU math (oracle/_ref, compiled
            from the reference sources; the C restatement when absent) on the
            host: each step is one decode token through one Qwen3-4B layer,
            extrapolated to the model (36 layers + LM head share).
Multi-GPU (torchrun, N > 1): every rank runs the workload on its own GPU
(replicas; no collective in the data path); value = all ranks' tokens / max
time over ranks.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Qwen3-4B F16 ragged-batch tokens/s at 1/2/4/8 B200; p50 TTFT; HBM GB/s"
SEED = 20261201
MAX_ACTIVE = 64
CHUNK = 512
GEN_FRACTION = 288.0 / 1128.0  # generated share of processed tokens in the trace (sets LM-head work)


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d["bf16_tflops_sustained"]), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


# ---------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples during the timed region (clocks and throttle reasons)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.device), "-lms", "200"], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except FileNotFoundError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        sm, mx, reasons = [], None, set()
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown",
                                  "sw_power_cap"), parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------- schedule
def plan_schedule(n_steps: int, seed: int = SEED):
    """Host-only simulation of the mixed planner: per step the admitted
    requests, the rows, and the finished requests."""
    from hllm_b200.workload import MixedPlanner, make_trace
    trace = make_trace(seed)
    planner = MixedPlanner(trace, max_active=MAX_ACTIVE, prefill_budget=CHUNK)
    steps = []
    for _ in range(n_steps):
        admits = []
        planner.admit(on_admit=admits.append)
        rows = planner.plan()
        row_info = [(r.req.rid, r.first_position, r.tokens, r.sample, r.decode) for r in rows]
        fin = planner.commit(rows)
        steps.append((list(admits), row_info, [r.rid for r in fin]))
    return trace, steps


def prompt_ids(rid: int, n: int, vocab: int) -> np.ndarray:
    return np.random.default_rng((SEED, rid)).integers(0, vocab, n, dtype=np.int64)


# ---------------------------------------------------------------------------- our arm
def make_stage(device: int):
    from hllm_b200 import B200Stage, ModelConfig
    from hllm_b200.workload import QWEN3_4B as Q
    cfg = ModelConfig(Q["hidden_size"], Q["intermediate_size"], Q["attention_heads"],
                      Q["key_value_heads"], Q["head_dimension"], Q["maximum_sequence_length"],
                      Q["rms_norm_epsilon"], Q["rope_theta"], Q["query_key_norm"],
                      Q["vocabulary_size"], Q["layers"], Q["tied"])
    stage = B200Stage(cfg, 0, Q["layers"], first=True, final=True, device=device,
                      kv_pool_tokens=MAX_ACTIVE * Q["maximum_sequence_length"] + 4096,
                      max_step_tokens=MAX_ACTIVE + CHUNK + 64, max_step_rows=MAX_ACTIVE + 16,
                      max_sequences=MAX_ACTIVE + 16)
    stage.init_synthetic(SEED)
    return stage, cfg


def run_device_phase(stage, cfg, trace, steps, first_timed, K, profile=False, clocks=None,
                     profiler_range=False):
    """Steps [0, first_timed + K) with device-resident ids; times the last K.

    With profiler_range the timed steps are bracketed by cudaProfilerStart/Stop, so
    that `ncu --profile-from-start off` lists exactly their launches."""
    import torch
    from hllm_b200 import _lib
    L = _lib.lib()
    V = cfg.vocabulary_size
    # All steps' ids (prefill: the prompt; decode: a token id per position),
    # uploaded before anything is timed.
    offsets, chunks, off = [], [], 0
    for admits, rows, _ in steps:
        offsets.append(off)
        for rid, first, count, sample, decode in rows:
            if decode:
                ids = np.asarray([(rid * 7919 + first) % V], np.int32)
            else:
                ids = prompt_ids(rid, trace[rid].prompt_len, V)[first:first + count].astype(np.int32)
            chunks.append(ids)
            off += count
    all_ids = torch.from_numpy(np.concatenate(chunks)).cuda()
    base = all_ids.data_ptr()
    seqs = {}
    stream = torch.cuda.ExternalStream(L.hllm_b200_stage_stream(stage.handle))
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    greedy = _lib.Sampling(0.0, 1.0, 0, 0, 0, 0)
    tokens = launches = 0
    for i, (admits, rows, fin) in enumerate(steps):
        if i == first_timed:
            _lib.check(L.hllm_b200_stage_sync(stage.handle))
            if profile:
                _lib.check(L.hllm_b200_stage_profile(stage.handle, 1))
            if clocks:
                clocks.start()
            torch.cuda.synchronize()
            if profiler_range:
                torch.cuda.profiler.start()
            start.record(stream)
        for r in admits:
            seqs[r.rid] = stage.allocate_sequence(r.capacity)
        arr = (_lib.Row * len(rows))()
        for j, (rid, first, count, sample, decode) in enumerate(rows):
            arr[j].sequence = seqs[rid].handle
            arr[j].first_position = first
            arr[j].tokens = count
            arr[j].sample = int(sample)
            arr[j].sampling = greedy
        _lib.check(L.hllm_b200_step_async(stage.handle, arr, len(rows), base + 4 * offsets[i]))
        if i >= first_timed:
            tokens += sum(r[2] for r in rows)
            launches += int(L.hllm_b200_stage_last_launches(stage.handle))
        for rid in fin:
            stage.release(seqs.pop(rid))
    end.record(stream)
    _lib.check(L.hllm_b200_stage_sync(stage.handle))
    torch.cuda.synchronize()
    if profiler_range:
        torch.cuda.profiler.stop()
    ms = start.elapsed_time(end)
    clock_info = clocks.stop() if clocks else None
    prof = None
    if profile:
        prof = {}
        for kind, name in enumerate(("gemm_decode", "gemm_prefill", "attn_decode", "attn_prefill",
                                     "misc", "norm", "qkv_rope", "swiglu", "sampler")):
            v = [C.c_double(), C.c_uint64(), C.c_double(), C.c_double()]
            _lib.check(L.hllm_b200_stage_profile_read(stage.handle, kind, C.byref(v[0]),
                                                      C.byref(v[1]), C.byref(v[2]), C.byref(v[3])))
            prof[name] = dict(ms=v[0].value, launches=v[1].value, bytes=v[2].value,
                              flops=v[3].value)
        _lib.check(L.hllm_b200_stage_profile(stage.handle, 0))
    for s in seqs.values():
        stage.release(s)
    return ms, tokens, launches, prof, clock_info


def run_host_phase(stage, cfg, trace, steps, first_timed, K):
    """The same steps through the public API with host buffers and token feedback."""
    import torch
    from hllm_b200 import DecodeBatchItem, TokenInput, _lib
    L = _lib.lib()
    V = cfg.vocabulary_size
    stream = torch.cuda.ExternalStream(L.hllm_b200_stage_stream(stage.handle))
    seqs, last_tok, admit_t, ttft = {}, {}, {}, []
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    tokens = h2d = d2h = 0
    generated = 0
    for i, (admits, rows, fin) in enumerate(steps):
        if i == first_timed:
            torch.cuda.synchronize()
            start.record(stream)
        now = time.perf_counter()
        for r in admits:
            seqs[r.rid] = stage.allocate_sequence(r.capacity)
            admit_t[r.rid] = now
        items = []
        for rid, first, count, sample, decode in rows:
            s = seqs[rid]
            if decode:
                ids = [last_tok[rid]]
                s.prefill_only = False
            else:
                ids = prompt_ids(rid, trace[rid].prompt_len, V)[first:first + count].tolist()
                s.prefill_only = not sample
            items.append(DecodeBatchItem(TokenInput(ids), first, s))
        outs = stage.execute_mixed_batch(items)
        t_done = time.perf_counter()
        for (rid, first, count, sample, decode), out in zip(rows, outs):
            if sample:
                last_tok[rid] = out.id
                if not decode and i >= first_timed:
                    ttft.append((t_done - admit_t[rid]) * 1e3)
        if i >= first_timed:
            tokens += sum(r[2] for r in rows)
            generated += sum(1 for r in rows if r[3])
            a, b = C.c_uint64(), C.c_uint64()
            _lib.check(L.hllm_b200_stage_last_transfer(stage.handle, C.byref(a), C.byref(b)))
            h2d += a.value
            d2h += b.value
        for rid in fin:
            stage.release(seqs.pop(rid))
    end.record(stream)
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    for s in seqs.values():
        stage.release(s)
    return ms, tokens, generated, h2d / max(1, K), d2h / max(1, K), ttft


def cpu_reference_sample(use_ref=True, layer_steps=3):
    """The reference CPU math on a bounded Qwen3-4B sample: decode tokens through
    one layer (the whole model is 36 such layers) plus one LM-head row.
    Returns (tokens/s extrapolated, per-token-layer s, head s, kind, detail)."""
    import oracle
    from hllm_b200.workload import QWEN3_4B as Q
    spec = oracle.ModelSpec(Q["hidden_size"], Q["intermediate_size"], Q["attention_heads"],
                            Q["key_value_heads"], Q["head_dimension"], Q["layers"],
                            Q["vocabulary_size"], Q["maximum_sequence_length"],
                            Q["rms_norm_epsilon"], Q["rope_theta"], Q["query_key_norm"], Q["tied"])
    kind = "reference" if (use_ref and oracle.ref() is not None) else "port"
    weights = oracle.synth_weights(spec, SEED, layers=[0])
    model = oracle.OracleModel(spec, weights, 0, 1, use_ref=(kind == "reference"))
    seq = model.new_sequence(64)
    rng = np.random.default_rng(1)
    x = (rng.standard_normal((4, spec.hidden_size)) * 0.02).astype(np.float32)
    model.forward(x, 0, seq)  # context of 4 positions
    times = []
    for i in range(layer_steps):
        t0 = time.perf_counter()
        model.forward(x[:1], 4 + i, seq)
        times.append(time.perf_counter() - t0)
    t_layer = statistics.median(times)
    model.logits(x[:1])  # builds the reference's head matrix once (untimed)
    t0 = time.perf_counter()
    model.logits(x[:1])
    t_head = time.perf_counter() - t0
    per_token = spec.layers * t_layer + GEN_FRACTION * t_head
    return 1.0 / per_token, t_layer, t_head, kind, model, seq


def host_cores():
    try:
        return os.cpu_count()
    except Exception:
        return None


def ours(args, world, rank, local):
    import torch
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    W, K, F = args.warmup, args.steps, args.fast_forward
    total_steps = F + W + K
    trace, steps = plan_schedule(total_steps)
    stage, cfg = make_stage(local)
    first_timed = F + W
    # value: device-resident inputs, steps enqueued back to back
    clocks = ClockSampler(local)
    dev_ms, dev_tokens, launches, _, clock_info = run_device_phase(
        stage, cfg, trace, steps, first_timed, K, clocks=clocks,
        profiler_range=args.profiler_range)
    if args.device_phase_only:
        print(json.dumps({"device_phase_ms_per_step": round(dev_ms / K, 4),
                          "tokens_per_s": round(dev_tokens / (dev_ms / 1e3), 1),
                          "launches_per_step": launches / K}), flush=True)
        stage.close()
        return
    # e2e: the public call with host buffers and token feedback
    import copy
    trace2, steps2 = plan_schedule(total_steps)
    e2e_ms, e2e_tokens, generated, h2d, d2h, ttft = run_host_phase(stage, cfg, trace2, steps2,
                                                                    first_timed, K)
    # profile pass (events around every launch) for the roofline
    trace3, steps3 = plan_schedule(total_steps)
    _, _, _, prof, _ = run_device_phase(stage, cfg, trace3, steps3, first_timed, K, profile=True)
    del copy
    times = torch.tensor([dev_ms, e2e_ms], dtype=torch.float64, device="cuda")
    toks = torch.tensor([dev_tokens, e2e_tokens], dtype=torch.float64, device="cuda")
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
        dist.all_reduce(toks, op=dist.ReduceOp.SUM)
    dev_ms, e2e_ms = times.tolist()
    all_dev_tokens, all_e2e_tokens = toks.tolist()
    if rank != 0:
        stage.close()
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()
        return
    hbm, tf_burst, tf_sust, peak_src = peaks()
    # dominant kernel class by device time
    dom = max(prof, key=lambda k: prof[k]["ms"] if (prof[k]["bytes"] or prof[k]["flops"]) else -1)
    p = prof[dom]
    per_launch_s = p["ms"] / 1e3 / max(1, p["launches"])
    intensity = p["flops"] / max(1.0, p["bytes"])
    tensor_bound = intensity > (tf_sust * 1e12) / (hbm * 1e9)
    if tensor_bound:
        achieved = p["flops"] / max(1, p["launches"]) / per_launch_s / 1e12
        roof = {"bound": "tensor", "achieved": round(achieved, 2), "peak": tf_sust,
                "unit": "TFLOP/s", "frac": round(achieved / tf_sust, 4)}
    else:
        achieved = p["bytes"] / max(1, p["launches"]) / per_launch_s / 1e9
        roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                "frac": round(achieved / hbm, 4)}
    roof.update({"kernel": dom, "peak_source": f"{peak_src} (MEASURED_PEAKS.json)"
                 if peak_src == "measured" else "fallback", "traffic": None,
                 "launches": p["launches"], "avg_launch_us": round(per_launch_s * 1e6, 2)})
    kernels = {k: {"ms": round(v["ms"], 3), "share": round(v["ms"] / max(1e-9, sum(
        x["ms"] for x in prof.values())), 4), "launches": v["launches"],
        "gbs": round(v["bytes"] / max(1e-12, v["ms"] / 1e3) / 1e9, 1) if v["bytes"] else None,
        "tflops": round(v["flops"] / max(1e-12, v["ms"] / 1e3) / 1e12, 1) if v["flops"] else None}
        for k, v in prof.items()}
    value = all_dev_tokens / (dev_ms / 1e3)
    e2e_value = all_e2e_tokens / (e2e_ms / 1e3)
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        tps, t_layer, t_head, kind, _, _ = cpu_reference_sample()
        cpu = {"value": round(tps, 5), "unit": "tokens/s", "cores": 1, "kind": kind,
               "sample": (f"3 decode tokens through one Qwen3-4B layer (median {t_layer:.3f} s) "
                          f"+ one LM-head row ({t_head:.3f} s), -O2 -ffp-contract=off, one "
                          f"thread (the reference CPU stage is single-threaded); extrapolated "
                          f"as 36 layers + {GEN_FRACTION:.3f} LM-head rows per token"),
               "host_cores": host_cores()}
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
        "steps": K, "warmup": W, "ms_per_step": round(dev_ms / K, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": "configuration 3: Qwen3-4B, 64 concurrent requests, prompts "
                               "lognormal(512, 1.0) in [32, 4096], outputs U[64, 512], 512-token "
                               "chunks mixed into decode batches, greedy",
                   "model": "Qwen3-4B-architecture random init (seeded), F16 weights, F32 accumulate",
                   "global_batch": MAX_ACTIVE * world, "seq_len": 4608,
                   "parallelism": "single stage" if world == 1 else f"replicas x{world}",
                   "fast_forward_steps": F,
                   "l2": "inputs larger than L2: 8.0 GB of weights and the KV cache stream every step"},
        "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s",
                "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                "ms_per_step": round(e2e_ms / K, 4)},
        "ttft_p50_ms": round(statistics.median(ttft), 3) if ttft else None,
        "output_tokens_per_s_e2e": round(generated * world / (e2e_ms / 1e3), 1),
        "roofline": roof, "kernels": kernels, "cpu_baseline": cpu, "clocks": clock_info,
        "gpu_launches": launches,
    }
    print(json.dumps(line), flush=True)
    stage.close()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


def reference(args, world, rank):
    """The reference's CPU math as the baseline arm (rank 0 only)."""
    if rank != 0:
        return
    import oracle
    if oracle.ref() is None:
        kind_note = "oracle/_ref absent: the C restatement of the reference CPU math"
    else:
        kind_note = "oracle/_ref: the reference's own CPU sources (-O2)"
    tps0, t_layer, t_head, kind, model, seq = cpu_reference_sample(layer_steps=1)
    rng = np.random.default_rng(2)
    x = (rng.standard_normal((1, model.spec.hidden_size)) * 0.02).astype(np.float32)
    pos = 5
    for _ in range(args.warmup):
        model.forward(x, pos, seq)
        pos += 1
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        model.forward(x, pos, seq)
        times.append(time.perf_counter() - t0)
        pos += 1
    t_layer = statistics.median(times)
    per_token = model.spec.layers * t_layer + GEN_FRACTION * t_head
    value = 1.0 / per_token
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 5), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(t_layer * 1e3, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "configuration 3 (Qwen3-4B), bounded CPU sample",
                       "model": "Qwen3-4B-architecture random init (seeded)",
                       "parallelism": "one CPU thread (the reference CPU stage has no threading)"},
            "cpu_baseline": {"value": round(value, 5), "unit": "tokens/s", "cores": 1,
                             "kind": kind,
                             "sample": f"each step one decode token through one Qwen3-4B layer "
                                       f"({kind_note}); tokens/s = 1 / (36 x median step + "
                                       f"{GEN_FRACTION:.3f} x LM-head row {t_head:.3f} s)"},
            "e2e": {"value": round(value, 5), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--fast-forward", type=int, default=150)
    ap.add_argument("--profiler-range", action="store_true",
                    help="bracket the timed device-phase steps with cudaProfilerStart/Stop")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--device-phase-only", action="store_true",
                    help="run only the device-resident phase (for profiler launch lists)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        reference(args, world, rank)
    else:
        ours(args, world, rank, local)


if __name__ == "__main__":
    main()
