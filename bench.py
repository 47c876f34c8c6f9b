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
Multi-GPU (torchrun, N > 1): an N-stage pipeline, one rank per GPU.  Rank r
owns a contiguous layer range (split by streamed bytes, hllm_b200.pipeline);
F16 boundaries go rank to rank with NCCL send/recv; N micro-batches of 64
concurrent requests each (independent traces) keep every stage busy, so the
global batch is 64 N (weak scaling).  A timed tick is one micro-batch step on
every rank; value = tokens completed by the last stage / max time over ranks.
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
PIPELINE_LIMIT_S = float(os.environ.get("HLLM_B200_PIPELINE_LIMIT_S", "300"))
# wall-clock limit of a multi-GPU (pipeline) run
PIPELINE_PROGRESS = {"phase": "init", "tick": -1, "where": "start"}  # reported on a stall


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d["bf16_tflops_sustained"]), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


# ---------------------------------------------------------------------------- clocks
class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled during the timed
    region: NVML polled every 10 ms from a thread (read only), or nvidia-smi
    -lms 50 where NVML is unavailable."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clock-event reason bits (nvml.h nvmlClocksEventReason*)
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines = []
        self.samples = []  # (sm MHz, max MHz, reason bits)
        self.stop_flag = threading.Event()
        self.thread = None

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        try:
            import torch
            props = torch.cuda.get_device_properties(self.device)
            bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.device)

    def start(self):
        try:
            nv, handle = self._nvml_handle()
            event_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
            mx = nv.nvmlDeviceGetMaxClockInfo(handle, nv.NVML_CLOCK_SM)

            def poll():
                while not self.stop_flag.is_set():
                    try:
                        sm = nv.nvmlDeviceGetClockInfo(handle, nv.NVML_CLOCK_SM)
                        bits = event_reasons(handle)
                    except Exception:
                        break
                    self.samples.append((float(sm), float(mx), int(bits)))
                    self.stop_flag.wait(0.01)

            self.thread = threading.Thread(target=poll, daemon=True)
            self.thread.start()
            return
        except Exception:
            self.thread = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.device), "-lms", "50"], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except FileNotFoundError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.thread:
            self.stop_flag.set()
            self.thread.join(timeout=5)
            sm = [x[0] for x in self.samples]
            reasons = {name for bits in (x[2] for x in self.samples)
                       for bit, name in self.REASONS.items() if bits & bit}
            return {"sm_mhz": statistics.median(sm) if sm else None,
                    "sm_max_mhz": self.samples[0][1] if self.samples else None,
                    "reasons": sorted(reasons), "samples": len(sm), "source": "nvml"}
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
                "reasons": sorted(reasons), "samples": len(sm), "source": "nvidia-smi"}


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


# ---------------------------------------------------------------------------- configuration 4
C4_ACTIVE = 128


def ours_c4(args, world, rank, local):
    """Configuration 4 on one GPU: the Falcon3-3B geometry (d 256, 12 query / 4 KV
    heads, untied head) with seeded random-init weights; a burst of 256
    requests at t = 0, 128 running at once, prompts U[128, 2048], 256 output
    tokens, temperature 0.7 / top-p 0.9 with a seed per request, and a random
    25% cancelled mid-decode (their KV blocks and slots go to waiting requests).
    The timed region is the whole burst, arrival to the last token, after
    `--warmup` steps of a different burst on the same stage."""
    import torch
    from hllm_b200 import B200Stage, ModelConfig, _lib
    from hllm_b200.workload import FALCON3_3B as Fm, MixedPlanner, make_burst_trace
    if world > 1:
        if rank == 0:
            print(json.dumps({"workload": "c4", "unavailable": "configuration 4 runs on one GPU "
                              "in bench.py; its pipeline at 2/4 GPUs is not wired"}), flush=True)
        return
    torch.cuda.set_device(local)
    cfg = ModelConfig(Fm["hidden_size"], Fm["intermediate_size"], Fm["attention_heads"],
                      Fm["key_value_heads"], Fm["head_dimension"], Fm["maximum_sequence_length"],
                      Fm["rms_norm_epsilon"], Fm["rope_theta"], Fm["query_key_norm"],
                      Fm["vocabulary_size"], Fm["layers"], Fm["tied"])
    stage = B200Stage(cfg, 0, Fm["layers"], first=True, final=True, device=local,
                      kv_pool_tokens=C4_ACTIVE * Fm["maximum_sequence_length"] + 4096,
                      max_step_tokens=C4_ACTIVE + CHUNK + 64, max_step_rows=C4_ACTIVE + 16,
                      max_sequences=C4_ACTIVE + 16)
    stage.init_synthetic(SEED)

    def plan(seed):
        trace = make_burst_trace(seed)
        planner = MixedPlanner(trace, max_active=C4_ACTIVE, prefill_budget=CHUNK)
        steps = []
        while planner.active or planner.next_req < len(trace):
            admits = []
            planner.admit(on_admit=admits.append)
            rows = planner.plan()
            info = [(r.req.rid, r.first_position, r.tokens, r.sample, r.decode) for r in rows]
            fin = planner.commit(rows)
            steps.append((admits, info, [r.rid for r in fin]))
        return trace, steps

    def sampling_for(rid):
        return _lib.Sampling(0.7, 0.9, 0, 1000 + rid, 0, 0)

    # warm-up: the first steps of another burst (its sequences are released after them)
    wtrace, wsteps = plan(SEED + 1)
    wsteps = wsteps[:args.warmup]
    run_device_phase(stage, cfg, wtrace, wsteps, 0, len(wsteps), sampling_for=sampling_for)
    trace, steps = plan(SEED)
    clocks = ClockSampler(local)
    ms, tokens, launches, _, clock_info = run_device_phase(stage, cfg, trace, steps, 0, len(steps),
                                                            clocks=clocks,
                                                            sampling_for=sampling_for)
    step_rows, step_ms = run_device_phase.last_steps
    stage.close()
    decode_tokens = sum(sum(c for _, c, _ in rows) for rows, dec in step_rows if dec)
    dec_ms = sum(t for (rows, dec), t in zip(step_rows, step_ms) if dec)
    cancelled = sum(1 for r in trace if r.cancelled)
    line = {
        "metric": "Falcon3-3B F16 burst tokens/s (configuration 4)", "value": round(tokens / (ms / 1e3), 1),
        "unit": "tokens/s", "n_gpus": 1, "steps": len(steps), "warmup": len(wsteps),
        "ms_per_step": round(ms / len(steps), 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16 weights, f32 accumulate", "data": "synthetic",
        "config": {"workload": "configuration 4: Falcon3-3B architecture (22 layers, hidden 3072, "
                   "12 query / 4 KV heads, head_dim 256, untied head) with seeded random-init "
                   "F16 weights; 256 requests arriving at t=0, 128 at once, prompts U[128, 2048], "
                   "256 output tokens, temperature 0.7 / top-p 0.9 with per-request seeds, "
                   f"{cancelled} of 256 cancelled mid-decode", "global_batch": C4_ACTIVE,
                   "seq_len": Fm["maximum_sequence_length"], "parallelism": "single stage",
                   "l2": "inputs larger than L2: 6.5 GB of weights and the KV cache stream every step"},
        "burst_ms": round(ms, 1), "tokens": tokens,
        "decode_only_steps": {"steps": sum(1 for _, d in step_rows if d),
                              "tokens_per_s": round(decode_tokens / max(1e-9, dec_ms / 1e3), 1)},
        "clocks": clock_info, "gpu_launches": launches,
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------- our arm
def make_stage(device: int, layer_start=0, layer_end=None, first=True, final=True,
               microbatches=1):
    """The Qwen3-4B stage for layers [layer_start, layer_end) with KV room for
    `microbatches` x 64 concurrent requests."""
    from hllm_b200 import B200Stage, ModelConfig
    from hllm_b200.workload import QWEN3_4B as Q
    cfg = ModelConfig(Q["hidden_size"], Q["intermediate_size"], Q["attention_heads"],
                      Q["key_value_heads"], Q["head_dimension"], Q["maximum_sequence_length"],
                      Q["rms_norm_epsilon"], Q["rope_theta"], Q["query_key_norm"],
                      Q["vocabulary_size"], Q["layers"], Q["tied"])
    end = Q["layers"] if layer_end is None else layer_end
    stage = B200Stage(cfg, layer_start, end, first=first, final=final, device=device,
                      kv_pool_tokens=microbatches * (MAX_ACTIVE * Q["maximum_sequence_length"]
                                                     + 4096),
                      max_step_tokens=MAX_ACTIVE + CHUNK + 64, max_step_rows=MAX_ACTIVE + 16,
                      max_sequences=microbatches * (MAX_ACTIVE + 16))
    stage.init_synthetic(SEED)
    return stage, cfg


KERNEL_CLASSES = ("gemm_decode", "gemm_prefill", "attn_decode", "attn_prefill", "misc", "norm",
                  "qkv_rope", "swiglu", "sampler")

# DRAM bytes per launch relative to the algorithmic bytes, from ncu captures of
# a smaller case of the same kernel (committed summaries under profiles/);
# traffic = algorithmic bytes per launch x ratio (traffic grows with the units).
TRAFFIC_RATIO = {
    "attn_decode": (279.5 / 271.7, "profiles/attention_decode_64rows.md"),
    "gemm_decode": (21.54 / 22.8, "profiles/gemm_o_proj_decode64.md"),
    "gemm_prefill": (106.24 / 113.7, "profiles/gemm_gate_up_prefill575.md"),
}


def read_profile(stage):
    """Per-class totals of the stage's launch profile (ms, launches, bytes, flops)."""
    from hllm_b200 import _lib
    L = _lib.lib()
    prof = {}
    for kind, name in enumerate(KERNEL_CLASSES):
        v = [C.c_double(), C.c_uint64(), C.c_double(), C.c_double()]
        _lib.check(L.hllm_b200_stage_profile_read(stage.handle, kind, C.byref(v[0]),
                                                  C.byref(v[1]), C.byref(v[2]), C.byref(v[3])))
        prof[name] = dict(ms=v[0].value, launches=v[1].value, bytes=v[2].value, flops=v[3].value)
    return prof


def run_device_phase(stage, cfg, trace, steps, first_timed, K, profile=False, clocks=None,
                     profiler_range=False, sampling_for=None):
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
    step_events, step_rows = [], []
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
            arr[j].sampling = sampling_for(rid) if sampling_for else greedy
        _lib.check(L.hllm_b200_step_async(stage.handle, arr, len(rows), base + 4 * offsets[i]))
        if i >= first_timed:
            tokens += sum(r[2] for r in rows)
            launches += int(L.hllm_b200_stage_last_launches(stage.handle))
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(stream)
            step_events.append(ev)
            step_rows.append(([(r[1], r[2], r[3]) for r in rows], all(r[4] for r in rows)))
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
        prof = read_profile(stage)
        _lib.check(L.hllm_b200_stage_profile(stage.handle, 0))
    for s in seqs.values():
        stage.release(s)
    marks = [start] + step_events
    run_device_phase.last_steps = (step_rows, [a.elapsed_time(b) for a, b in zip(marks, marks[1:])])
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


def run_arrival_phase(stage, cfg, seconds: float = 4.0):
    """Open-loop TTFT: requests arrive at their trace's Poisson times (8 req/s)
    in wall-clock time, are admitted once arrived (at most 64 running), and
    run through the public call; TTFT = first token - arrival, for requests
    that arrive within `seconds`.  Returns (ttft ms list, steps run)."""
    from hllm_b200 import DecodeBatchItem, TokenInput
    from hllm_b200.workload import MixedPlanner, make_trace
    V = cfg.vocabulary_size
    trace = make_trace(SEED + 7)
    planner = MixedPlanner(trace, max_active=MAX_ACTIVE, prefill_budget=CHUNK)
    seqs, last_tok, ttft = {}, {}, []
    t0 = time.perf_counter()
    steps = 0
    while True:
        now = time.perf_counter() - t0
        planner.admit(on_admit=lambda r: seqs.__setitem__(r.rid, stage.allocate_sequence(r.capacity)),
                      until=now)
        rows = planner.plan()
        if not rows:
            nxt = planner.trace[planner.next_req].arrival if planner.next_req < len(trace) else None
            if nxt is None or nxt > seconds:
                break
            time.sleep(max(0.0, nxt - now))
            continue
        items = []
        for row in rows:
            r, s = row.req, seqs[row.req.rid]
            if row.decode:
                ids = [last_tok[r.rid]]
                s.prefill_only = False
            else:
                ids = prompt_ids(r.rid, r.prompt_len, V)[row.first_position:
                                                         row.first_position + row.tokens].tolist()
                s.prefill_only = not row.sample
            items.append(DecodeBatchItem(TokenInput(ids), row.first_position, s))
        outs = stage.execute_mixed_batch(items)
        done_t = time.perf_counter() - t0
        steps += 1
        for row, out in zip(rows, outs):
            if row.sample:
                last_tok[row.req.rid] = out.id
                if not row.decode and row.req.arrival <= seconds:
                    ttft.append((done_t - row.req.arrival) * 1e3)
        for r in planner.commit(rows):
            stage.release(seqs.pop(r.rid))
        if done_t > seconds and not any(r.arrival <= seconds and r.generated == 0
                                        for r in planner.active):
            break
    for s in seqs.values():
        stage.release(s)
    return ttft, steps


def reference_threads() -> int:
    """Host threads this process may run on."""
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except AttributeError:
        return max(1, os.cpu_count() or 1)


def _parallel(threads: int, fn) -> float:
    """fn(i) on `threads` Python threads at once; wall seconds.  The reference's
    C++ runs inside ctypes calls, which release the GIL, so the threads run
    side by side."""
    errors = []

    def run(i):
        try:
            fn(i)
        except BaseException as e:  # re-raised below
            errors.append(e)

    ts = [threading.Thread(target=run, args=(i,)) for i in range(threads)]
    t0 = time.perf_counter()
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    wall = time.perf_counter() - t0
    if errors:
        raise errors[0]
    return wall


def workload_mix(steps, first_timed):
    """The timed steps' token mix: decode rows' context lengths, prefill rows'
    (first position, tokens), and the number of sampled rows."""
    dec_ctx, pre_rows, samples = [], [], 0
    for _, rows, _ in steps[first_timed:]:
        for rid, first, count, sample, decode in rows:
            if decode:
                dec_ctx.append(first + 1)
            else:
                pre_rows.append((first, count))
            samples += int(sample)
    return dec_ctx, pre_rows, samples


def _midpoints(values, n):
    """n values at the quantile midpoints of `values` (sorted)."""
    v = sorted(values)
    return [v[min(len(v) - 1, (2 * i + 1) * len(v) // (2 * n))] for i in range(n)]


class ReferenceSample:
    """The reference CPU math on a bounded sample of the configuration-3
    workload: one Qwen3-4B layer (the model is 36 such layers) and the LM head,
    one independent stream per host thread.  The reference CPU stage is
    single-threaded (cpp/src/cpu has no threading), so all host cores are used
    by running streams side by side over the shared weights.

    Stream i decodes at a context length taken from the timed GPU steps'
    decode rows (their quantile midpoints) and prefills a short chunk at a
    position taken from the timed steps' prefill tokens; each stream's KV cache
    is first filled to that length with synthetic keys and values (the cost of
    a step depends on the context length, not on the cached values).  Per-token
    layer costs then give tokens/s for the timed steps' own mix of decode
    tokens, prefill tokens and sampled rows."""

    PREFILL_TOKENS = 8

    def __init__(self, threads: int, mix, use_ref=True, decode_steps: int = 2):
        import oracle
        from hllm_b200.workload import QWEN3_4B as Q
        spec = oracle.ModelSpec(Q["hidden_size"], Q["intermediate_size"], Q["attention_heads"],
                                Q["key_value_heads"], Q["head_dimension"], Q["layers"],
                                Q["vocabulary_size"], Q["maximum_sequence_length"],
                                Q["rms_norm_epsilon"], Q["rope_theta"], Q["query_key_norm"],
                                Q["tied"])
        self.spec, self.threads = spec, threads
        self.kind = "reference" if (use_ref and oracle.ref() is not None) else "port"
        weights = oracle.synth_weights(spec, SEED, layers=[0])
        self.model = oracle.OracleModel(spec, weights, 0, 1, use_ref=(self.kind == "reference"))
        dec_ctx, pre_rows, self.samples = mix
        self.decode_tokens = len(dec_ctx)
        self.prefill_tokens = sum(c for _, c in pre_rows)
        pre_pos = [f + j for f, c in pre_rows for j in range(c)]
        self.dec_ctx = _midpoints(dec_ctx, threads)
        self.pre_pos = _midpoints(pre_pos, threads) if pre_pos else [0] * threads
        rng = np.random.default_rng(1)
        self.x = (rng.standard_normal((self.PREFILL_TOKENS, spec.hidden_size)) * 0.02).astype(
            np.float32)
        cap = max(self.dec_ctx) + decode_steps + 8
        self.dec_seqs, self.pos = [], []
        for i, c in enumerate(self.dec_ctx):
            seq = self.model.new_sequence(cap)
            self.model.fill_context(seq, c - 1, seed=i)
            self.dec_seqs.append(seq)
            self.pos.append(c - 1)
        self.model.logits(self.x[:1])  # builds the reference's head matrix once (untimed)

    def decode(self, steps: int) -> float:
        """`steps` decode tokens through the layer on every stream; wall seconds."""
        def run(i):
            for _ in range(steps):
                self.model.forward(self.x[:1], self.pos[i], self.dec_seqs[i])
                self.pos[i] += 1
        return _parallel(self.threads, run)

    def prefill(self) -> float:
        """A PREFILL_TOKENS-token chunk through the layer on every stream, each at
        its sampled position; wall seconds (cache fills are not timed)."""
        seqs = []
        for i, p in enumerate(self.pre_pos):
            seq = self.model.new_sequence(p + self.PREFILL_TOKENS + 1)
            if p:
                self.model.fill_context(seq, p, seed=1000 + i)
            seqs.append(seq)
        wall = _parallel(self.threads,
                         lambda i: self.model.forward(self.x, self.pre_pos[i], seqs[i]))
        for seq in seqs:
            self.model.free_sequence(seq)
        return wall

    def head(self) -> float:
        """One LM-head row on every stream; wall seconds."""
        return _parallel(self.threads, lambda i: self.model.logits(self.x[:1]))

    def rates(self, dec_wall: float, steps: int, pre_wall: float, head_wall: float):
        """(tokens/s over the timed mix, decode tokens/s, prefill tokens/s,
        per-token-layer decode s, prefill s, per-row head s), all streams
        together."""
        t_dec = dec_wall / (steps * self.threads)
        t_pre = pre_wall / (self.PREFILL_TOKENS * self.threads)
        t_head = head_wall / self.threads
        L = self.spec.layers
        total = L * (self.decode_tokens * t_dec + self.prefill_tokens * t_pre) + \
            self.samples * t_head
        mixed = (self.decode_tokens + self.prefill_tokens) / total
        return (mixed, 1.0 / (L * t_dec + t_head), 1.0 / (L * t_pre), t_dec, t_pre, t_head)

    def describe(self, t_dec, t_pre, t_head) -> str:
        return (f"{self.threads} streams side by side (the reference CPU stage is "
                f"single-threaded), one Qwen3-4B layer + the LM head, -O2 -ffp-contract=off: "
                f"decode at the timed steps' context quantiles ({min(self.dec_ctx)}-"
                f"{max(self.dec_ctx)} tokens, mean {np.mean(self.dec_ctx):.0f}) "
                f"{t_dec * self.threads:.3f} s per token-layer per stream; a "
                f"{self.PREFILL_TOKENS}-token prefill chunk at the timed prefill tokens' "
                f"position quantiles (mean {np.mean(self.pre_pos):.0f}) "
                f"{t_pre * self.threads:.3f} s per token-layer per stream; LM-head row "
                f"{t_head * self.threads:.3f} s per stream; tokens/s = (decode + prefill tokens "
                f"of the timed steps: {self.decode_tokens} + {self.prefill_tokens}) / (36 x token-"
                f"layer costs + {self.samples} head rows), all streams together")


def cpu_reference_sample(mix, use_ref=True, decode_steps=2):
    """cpu_baseline of the timed mix on all host threads (a dict for the JSON line)."""
    threads = reference_threads()
    ref = ReferenceSample(threads, mix, use_ref, decode_steps)
    dec = ref.decode(decode_steps)
    pre = ref.prefill()
    head = ref.head()
    mixed, dec_rate, pre_rate, t_dec, t_pre, t_head = ref.rates(dec, decode_steps, pre, head)
    return {"value": round(mixed, 5), "unit": "tokens/s", "cores": threads, "kind": ref.kind,
            "decode_tokens_per_s": round(dec_rate, 5),
            "prefill_tokens_per_s": round(pre_rate, 5),
            "sample": ref.describe(t_dec, t_pre, t_head), "host_cores": host_cores()}


def host_cores():
    try:
        return os.cpu_count()
    except Exception:
        return None


def ours(args, world, rank, local):
    if world > 1:
        ours_pipeline(args, world, rank, local)
        return
    import torch
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
    dev_steps = run_device_phase.last_steps
    if args.device_phase_only:
        print(json.dumps({"device_phase_ms_per_step": round(dev_ms / K, 4),
                          "tokens_per_s": round(dev_tokens / (dev_ms / 1e3), 1),
                          "launches_per_step": launches / K}), flush=True)
        stage.close()
        return
    # e2e: the public call with host buffers and token feedback
    trace2, steps2 = plan_schedule(total_steps)
    e2e_ms, e2e_tokens, generated, h2d, d2h, ttft = run_host_phase(stage, cfg, trace2, steps2,
                                                                    first_timed, K)
    # profile pass (events around every launch) for the roofline
    trace3, steps3 = plan_schedule(total_steps)
    _, _, _, prof, _ = run_device_phase(stage, cfg, trace3, steps3, first_timed, K, profile=True)
    # open-loop arrivals for TTFT from each request's arrival
    ttft_open, open_steps = run_arrival_phase(stage, cfg)
    stage.close()
    cpu = None
    if not args.no_cpu_baseline:
        cpu = cpu_reference_sample(workload_mix(steps, first_timed))
    hbm, _, tf_sust, _ = peaks()
    phases = phase_summary(*dev_steps, hbm, tf_sust)
    emit_line(args, 1, dev_ms, dev_tokens, e2e_ms, e2e_tokens, launches, h2d, d2h, ttft,
              generated, prof, clock_info, cpu, parallelism="single stage", phases=phases,
              ttft_open=(ttft_open, open_steps))


WORKLOAD = ("configuration 3: Qwen3-4B architecture with seeded random-init F16 weights "
            "(F32 accumulate), 64 concurrent requests, prompts lognormal(512, 1.0) in "
            "[32, 4096], outputs U[64, 512], 512-token chunks mixed into decode batches, greedy")


def workload_config(world, parallelism, fast_forward):
    """The `config` object both arms report."""
    return {"workload": WORKLOAD, "global_batch": MAX_ACTIVE * world, "seq_len": 4608,
            "parallelism": parallelism, "fast_forward_steps": fast_forward,
            "l2": "inputs larger than L2: 8.0 GB of weights and the KV cache stream every step"}


def emit_line(args, world, dev_ms, dev_tokens, e2e_ms, e2e_tokens, launches, h2d_step, d2h_step,
              ttft, generated, prof, clock_info, cpu, parallelism, phases=None, ttft_open=None):
    """Prints the benchmark's JSON line (rank 0)."""
    K = args.steps
    steps_timed = K * world  # micro-batch steps completed in the timed region
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
    traffic, traffic_src = None, None
    if dom in TRAFFIC_RATIO and p["bytes"]:
        ratio, traffic_src = TRAFFIC_RATIO[dom]
        traffic = round(p["bytes"] / max(1, p["launches"]) * ratio / 1e6, 2)
    roof.update({"kernel": dom, "peak_source": f"{peak_src} (MEASURED_PEAKS.json)"
                 if peak_src == "measured" else "fallback (MEASURED_PEAKS.json absent)",
                 "traffic": traffic, "traffic_unit": "MB per launch",
                 "traffic_source": traffic_src,
                 "launches": p["launches"], "avg_launch_us": round(per_launch_s * 1e6, 2)})
    total_ms = sum(x["ms"] for x in prof.values())
    kernels = {k: {"ms": round(v["ms"], 3), "share": round(v["ms"] / max(1e-9, total_ms), 4),
                   "launches": v["launches"],
                   "gbs": round(v["bytes"] / max(1e-12, v["ms"] / 1e3) / 1e9, 1) if v["bytes"] else None,
                   "tflops": round(v["flops"] / max(1e-12, v["ms"] / 1e3) / 1e12, 1) if v["flops"] else None}
               for k, v in prof.items()}
    value = dev_tokens / (dev_ms / 1e3)
    e2e_value = e2e_tokens / (e2e_ms / 1e3)
    config = workload_config(world, parallelism, args.fast_forward)
    if world > 1:
        config["microbatches"] = world
        config["timed_microbatch_steps"] = steps_timed
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
        "steps": K, "warmup": args.warmup, "ms_per_step": round(dev_ms / steps_timed, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic", "config": config,
        "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s",
                "h2d_bytes_per_step": int(h2d_step), "d2h_bytes_per_step": int(d2h_step),
                "ms_per_step": round(e2e_ms / steps_timed, 4)},
        # open-loop TTFT (from arrival) where measured, else from admission
        "ttft_p50_ms": (round(statistics.median(ttft_open[0]), 3)
                        if ttft_open and ttft_open[0]
                        else round(statistics.median(ttft), 3) if ttft else None),
        "ttft": {"p50_ms": round(statistics.median(ttft_open[0]), 3),
                 "p90_ms": round(float(np.percentile(ttft_open[0], 90)), 3),
                 "requests": len(ttft_open[0]), "steps": ttft_open[1],
                 "how": "open loop: requests arrive at their Poisson times (8 req/s) in wall-clock "
                        "time for 4 s and run through the public call; first token - arrival"}
                if ttft_open and ttft_open[0] else None,
        "ttft_saturated_p50_ms": round(statistics.median(ttft), 3) if ttft else None,
        "output_tokens_per_s_e2e": round(generated / (e2e_ms / 1e3), 1),
        "roofline": roof, "kernels": kernels, "phases": phases, "cpu_baseline": cpu,
        "clocks": clock_info,
        "gpu_launches": int(launches),
    }
    if world > 1:  # the planner's per-GPU split (hllm_b200.planner)
        plan = pipeline_plan(world)
        line["pipeline"] = {"ranges": [list(r) for r in pipeline_ranges(world)],
                            "memory_pressure": [round(g["memory"]["pressure"], 4)
                                                for g in plan["gpus"]]}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------- pipeline (N > 1)
def qwen_stage_bytes():
    """F16 bytes one Qwen3-4B layer and the LM head stream per step."""
    from hllm_b200.workload import QWEN3_4B as Q
    h, i, d = Q["hidden_size"], Q["intermediate_size"], Q["head_dimension"]
    q, kv = Q["attention_heads"] * d, Q["key_value_heads"] * d
    layer = 2.0 * (h * (q + 2 * kv) + q * h + 2 * i * h + i * h)
    return layer, 2.0 * Q["vocabulary_size"] * h


def step_work(rows, layers=None):
    """Algorithmic work of one Qwen3-4B step from its rows (first position,
    token count, samples): (bytes, FLOPs).

    bytes follow the decode-step formula: every owned layer's weights, the LM
    head, each row's K/V context read, the new K/V written, and the hidden
    rows in and out.  FLOPs follow the prefill formula: 2 x layer parameters
    per token, causal attention 4 x Hq x d per (token, key) pair per layer,
    and 2 x V x h per sampled row."""
    from hllm_b200.workload import QWEN3_4B as Q
    L = Q["layers"] if layers is None else layers
    h, d = Q["hidden_size"], Q["head_dimension"]
    hq, hkv, V = Q["attention_heads"], Q["key_value_heads"], Q["vocabulary_size"]
    layer_bytes, head_bytes = qwen_stage_bytes()
    kv_token = 2 * hkv * d * 2  # K and V, F16, one layer
    nbytes = L * layer_bytes + head_bytes
    flops = 0.0
    for first, count, sample in rows:
        keys = sum(first + j + 1 for j in range(count))  # causal (query, key) pairs
        nbytes += L * kv_token * (first + count) + L * kv_token * count + count * h * 2 * 2
        flops += (layer_bytes / 2.0) * 2.0 * L * count + 4.0 * hq * d * L * keys
        if sample:
            flops += 2.0 * V * h
    return nbytes, flops


def phase_summary(steps, step_ms, hbm_gbs, tflops):
    """Decode-only steps against the HBM roof, steps carrying a prefill chunk
    against the tensor roof: {phase: steps, ms per step, tokens/s, achieved,
    frac}.  steps: per step (rows, decode_only) with rows as for step_work."""
    out = {}
    for name, decode in (("decode", True), ("prefill", False)):
        picked = [(rows, ms) for (rows, only), ms in zip(steps, step_ms) if only == decode]
        if not picked:
            continue
        ms = sum(m for _, m in picked)
        tokens = sum(c for rows, _ in picked for _, c, _ in rows)
        nbytes = sum(step_work(rows)[0] for rows, _ in picked)
        flops = sum(step_work(rows)[1] for rows, _ in picked)
        entry = {"steps": len(picked), "ms_per_step": round(ms / len(picked), 4),
                 "tokens_per_s": round(tokens / (ms / 1e3), 1)}
        if decode:
            achieved = nbytes / (ms / 1e3) / 1e9
            entry.update(bound="hbm", achieved=round(achieved, 1), unit="GB/s",
                         frac=round(achieved / hbm_gbs, 4))
        else:
            achieved = flops / (ms / 1e3) / 1e12
            entry.update(bound="tensor", achieved=round(achieved, 1), unit="TFLOP/s",
                         frac=round(achieved / tflops, 4))
        out[name] = entry
    return out


def pipeline_plan(world: int) -> dict:
    """The per-GPU plan of the whole Qwen3-4B stage over `world` B200s
    (hllm_b200.planner): layers split by the weight bytes each rank streams per
    step (the LM head on the last rank), and each GPU's memory by the reference
    planner's model for this workload (64 concurrent requests of up to 4,608
    tokens, 512-token chunks)."""
    from hllm_b200 import planner as P
    from hllm_b200.workload import QWEN3_4B as Q
    workload = dict(workload_id="configuration-3", prompt_tokens=CHUNK, output_tokens=512,
                    concurrency=MAX_ACTIVE, total_cached_tokens=MAX_ACTIVE * 4608)
    return P.plan_worker(P.shape_from_geometry(**Q), P.B200_WORKER, workload, world,
                         kv_tokens=0)


def pipeline_ranges(world: int):
    from hllm_b200.planner import ranges_of
    return ranges_of(pipeline_plan(world))


def run_pipeline_phase(stage, cfg, rank, world, links, plans, traces, F, W, K, host_mode,
                       profile=False, clocks=None):
    """All ticks of the micro-batch schedule on this rank; times ticks [T0, T1).

    host_mode False (value): rank 0 reads pre-uploaded token ids (synthetic ids
    for decode rows), boundaries go rank to rank over NCCL, nothing returns to
    the host.  host_mode True (e2e): rank 0 copies each step's ids from pinned
    host memory (decode rows: the tokens the last rank sampled one tick
    earlier, sent back over gloo), and the last rank reads its sampled tokens
    back to the host every step.  Returns this rank's (ms, tokens completed on
    the last rank, launches, h2d, d2h, prof, clocks, ttft samples, generated)."""
    import torch
    import torch.distributed as dist
    from hllm_b200 import _lib
    from hllm_b200.pipeline import Schedule, device_view, run_ticks
    L = _lib.lib()
    V, H = cfg.vocabulary_size, cfg.hidden_size
    S = F + W + K + 1
    sched = Schedule(world, S)
    T0 = world * (F + W) + world - 1
    T1 = T0 + world * K
    first, final = rank == 0, rank == world - 1
    stream = torch.cuda.ExternalStream(L.hllm_b200_stage_stream(stage.handle))
    max_tokens = MAX_ACTIVE + CHUNK + 64
    base = None
    offsets = {}
    if first and not host_mode:
        chunks, off = [], 0
        for m in range(world):
            for j in range(S):
                offsets[(m, j)] = off
                for rid, fpos, count, sample, decode in plans[m][j][1]:
                    if decode:
                        ids = np.asarray([(rid * 7919 + fpos) % V], np.int32)
                    else:
                        ids = prompt_ids(rid, traces[m][rid].prompt_len, V)[fpos:fpos + count]
                    chunks.append(np.asarray(ids, np.int32))
                    off += count
        all_ids = torch.from_numpy(np.concatenate(chunks)).cuda()
        base = all_ids.data_ptr()
    if first and host_mode:
        ids_dev = torch.empty(max_tokens, dtype=torch.int32, device="cuda")
    boundary = None if final else device_view(L.hllm_b200_stage_boundary(stage.handle),
                                              (max_tokens, H))
    seqs = [dict() for _ in range(world)]
    last_tok = {}
    admit_wall, first_wall = {}, {}
    acc = dict(tokens=0, launches=0, h2d=0, d2h=0, generated=0)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    greedy = _lib.Sampling(0.0, 1.0, 0, 0, 0, 0)

    def tick(t, m, j):
        admits, rows, fin = plans[m][j]
        n_tok = sum(r[2] for r in rows)
        PIPELINE_PROGRESS.update(tick=t, where="recv")
        ptr = None
        if not first:
            ptr = links.recv_activation(n_tok)  # posted before any synchronisation
        if t == T0:
            PIPELINE_PROGRESS["where"] = "timing barrier"
            torch.cuda.synchronize()
            dist.barrier()
            if profile:
                _lib.check(L.hllm_b200_stage_profile(stage.handle, 1))
            if clocks:
                clocks.start()
            start.record(stream)
        now = time.time()
        for r in admits:
            seqs[m][r.rid] = stage.allocate_sequence(r.capacity)
            admit_wall[(m, r.rid)] = now
        arr = (_lib.Row * len(rows))()
        for k, (rid, fpos, count, sample, decode) in enumerate(rows):
            arr[k].sequence = seqs[m][rid].handle
            arr[k].first_position = fpos
            arr[k].tokens = count
            arr[k].sample = int(sample)
            arr[k].sampling = greedy
        h2d = 0
        if first:
            if not host_mode:
                ptr = base + 4 * offsets[(m, j)]
            else:
                if j > 0:
                    prev = [r[0] for r in plans[m][j - 1][1] if r[3]]
                    if prev:
                        PIPELINE_PROGRESS["where"] = "recv tokens"
                        for rid, tok in zip(prev, links.recv_tokens(len(prev))):
                            last_tok[(m, rid)] = int(tok)
                ids = []
                for rid, fpos, count, sample, decode in rows:
                    if decode:
                        ids.append(np.asarray([last_tok[(m, rid)]], np.int32))
                    else:
                        ids.append(prompt_ids(rid, traces[m][rid].prompt_len, V)[fpos:fpos + count]
                                   .astype(np.int32))
                # a pinned copy per step: the caching host allocator keeps it
                # until the asynchronous upload has run
                ids_host = torch.from_numpy(np.concatenate(ids)).pin_memory()
                with torch.cuda.stream(stream):
                    ids_dev[:n_tok].copy_(ids_host, non_blocking=True)
                ptr = ids_dev.data_ptr()
                h2d += 4 * n_tok
        PIPELINE_PROGRESS["where"] = "step"
        _lib.check(L.hllm_b200_step_async(stage.handle, arr, len(rows), ptr))
        a, b = C.c_uint64(), C.c_uint64()
        _lib.check(L.hllm_b200_stage_last_transfer(stage.handle, C.byref(a), C.byref(b)))
        h2d += a.value
        d2h = b.value
        PIPELINE_PROGRESS["where"] = "send"
        if not final:
            links.send_activation(boundary, n_tok)
        elif host_mode:
            PIPELINE_PROGRESS["where"] = "sync for tokens"
            _lib.check(L.hllm_b200_stage_sync(stage.handle))
            samp = [r for r in rows if r[3]]
            if samp:
                out = (_lib.Sampled * len(samp))()
                _lib.check(L.hllm_b200_stage_results(stage.handle, out, len(samp)))
                d2h += 104 * len(samp)
                toks = np.asarray([out[k].token_id for k in range(len(samp))], np.int64)
                now = time.time()
                for (rid, fpos, count, sample, decode), tok in zip(samp, toks):
                    if not decode and (m, rid) not in first_wall:
                        first_wall[(m, rid)] = (now, T0 <= t < T1)
                if j + 1 < S:
                    links.send_tokens(toks)
                if T0 <= t < T1:
                    acc["generated"] += len(samp)
        if T0 <= t < T1:
            if final:
                acc["tokens"] += n_tok
            acc["launches"] += int(L.hllm_b200_stage_last_launches(stage.handle))
            acc["h2d"] += h2d
            acc["d2h"] += d2h
        if t == T1 - 1:
            end.record(stream)
        PIPELINE_PROGRESS["where"] = "release"
        for rid in fin:
            stage.release(seqs[m].pop(rid))

    run_ticks(sched, rank, tick)
    PIPELINE_PROGRESS.update(where="drain")
    links.drain()
    _lib.check(L.hllm_b200_stage_sync(stage.handle))
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    clock_info = clocks.stop() if clocks else None
    prof = None
    if profile:
        prof = read_profile(stage)
        _lib.check(L.hllm_b200_stage_profile(stage.handle, 0))
    for d in seqs:
        for s in d.values():
            stage.release(s)
    ttft = []
    if host_mode:
        # admission wall times live on rank 0, first tokens on the last rank;
        # every rank of the token group takes part in the broadcast
        obj = [admit_wall if first else None]
        dist.broadcast_object_list(obj, src=0, group=links.token_group)
        if final:
            for key, (tw, timed) in first_wall.items():
                if timed and key in obj[0]:
                    ttft.append((tw - obj[0][key]) * 1e3)
    return (ms, acc["tokens"], acc["launches"], acc["h2d"], acc["d2h"], prof, clock_info, ttft,
            acc["generated"])


def ours_pipeline(args, world, rank, local):
    """N > 1: the stage executor as an N-stage pipeline, one rank per GPU."""
    import datetime
    import torch
    import torch.distributed as dist
    from hllm_b200 import _lib
    from hllm_b200.pipeline import DeviceLinks, make_groups
    torch.cuda.set_device(local)
    # A stalled pipeline must end the run, not hold N GPUs: every rank exits
    # with an error after PIPELINE_LIMIT_S seconds (a normal run takes a few
    # minutes at 8 GPUs).
    def stalled():
        import faulthandler
        print(json.dumps({"error": f"pipeline run on rank {rank} exceeded {PIPELINE_LIMIT_S} s",
                          "progress": PIPELINE_PROGRESS}), file=sys.stderr, flush=True)
        faulthandler.dump_traceback(file=sys.stderr, all_threads=True)
        os._exit(3)
    watchdog = threading.Timer(PIPELINE_LIMIT_S, stalled)
    watchdog.daemon = True
    watchdog.start()
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    pair_groups, token_group = make_groups(world)
    W, K, F = args.warmup, args.steps, args.fast_forward
    S = F + W + K + 1
    ranges = pipeline_ranges(world)
    lo, hi = ranges[rank]
    stage, cfg = make_stage(local, lo, hi, rank == 0, rank == world - 1, microbatches=world)
    L = _lib.lib()
    stream = torch.cuda.ExternalStream(L.hllm_b200_stage_stream(stage.handle))
    links = DeviceLinks(rank, world, stream, MAX_ACTIVE + CHUNK + 64, cfg.hidden_size,
                        token_group=token_group, pair_groups=pair_groups)
    PIPELINE_PROGRESS["where"] = "connect"
    links.connect()

    def fresh_plans():
        traces, plans = [], []
        for m in range(world):
            tr, st = plan_schedule(S, seed=SEED + m)
            traces.append(tr)
            plans.append(st)
        return traces, plans

    traces, plans = fresh_plans()
    clocks = ClockSampler(local) if rank == 0 else None
    PIPELINE_PROGRESS["phase"] = "device"
    dev = run_pipeline_phase(stage, cfg, rank, world, links, plans, traces, F, W, K, False,
                             clocks=clocks)
    traces, plans = fresh_plans()
    PIPELINE_PROGRESS["phase"] = "e2e"
    e2e = run_pipeline_phase(stage, cfg, rank, world, links, plans, traces, F, W, K, True)
    traces, plans = fresh_plans()
    PIPELINE_PROGRESS["phase"] = "profile"
    prof = run_pipeline_phase(stage, cfg, rank, world, links, plans, traces, F, W, K, False,
                              profile=True)[5]
    # times: max over ranks; tokens: completed on the last rank; launches: sum
    PIPELINE_PROGRESS.update(phase="results", where="all_reduce")
    t = torch.tensor([dev[0], e2e[0]], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    n = torch.tensor([dev[1], e2e[1], dev[2], e2e[3], e2e[4], e2e[8]], dtype=torch.float64,
                     device="cuda")
    dist.all_reduce(n, op=dist.ReduceOp.SUM)
    profs = [None] * world
    dist.all_gather_object(profs, prof)
    ttfts = [None] * world
    dist.all_gather_object(ttfts, e2e[7])
    dev_ms, e2e_ms = t.tolist()
    dev_tokens, e2e_tokens, launches, h2d, d2h, generated = n.tolist()
    stage.close()
    if rank == 0:
        merged = {}
        for p in profs:
            for k, v in p.items():
                m = merged.setdefault(k, dict(ms=0.0, launches=0, bytes=0.0, flops=0.0))
                for f in m:
                    m[f] += v[f]
        ttft = [x for lst in ttfts for x in lst]
        emit_line(args, world, dev_ms, dev_tokens, e2e_ms, e2e_tokens, int(launches),
                  h2d / (world * K), d2h / (world * K), ttft, generated, merged, dev[6], None,
                  parallelism=f"pipeline x{world}, layers {ranges}")
    dist.barrier()
    dist.destroy_process_group()
    watchdog.cancel()


def reference(args, world, rank):
    """The reference's CPU math as the baseline arm (rank 0 only), on all host
    threads, over the same timed steps' token mix as our arm: each step one
    decode token through one Qwen3-4B layer on every stream (streams at the
    timed steps' decode contexts), plus one prefill chunk and one LM-head row
    per stream, weighted by the mix (ReferenceSample)."""
    if rank != 0:
        return
    import oracle
    W, K, F = args.warmup, args.steps, args.fast_forward
    _, steps = plan_schedule(F + W + K)
    threads = reference_threads()
    ref = ReferenceSample(threads, workload_mix(steps, F + W), decode_steps=W + K)
    ref.decode(W)
    wall = ref.decode(K)
    pre = ref.prefill()
    head = ref.head()
    value, dec_rate, pre_rate, t_dec, t_pre, t_head = ref.rates(wall, K, pre, head)
    kind_note = ("oracle/_ref: the reference's own CPU sources" if oracle.ref() is not None
                 else "oracle/_ref absent: the C restatement of the reference CPU math")
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 5), "unit": "tokens/s",
            "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": round(wall / K * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload_config(
                world, f"reference CPU math on {threads} host threads, one stream each "
                       f"(the reference CPU stage is single-threaded); a bounded sample of the "
                       f"workload, see cpu_baseline.sample", F),
            "cpu_baseline": {"value": round(value, 5), "unit": "tokens/s", "cores": threads,
                             "kind": ref.kind, "decode_tokens_per_s": round(dec_rate, 5),
                             "prefill_tokens_per_s": round(pre_rate, 5),
                             "sample": f"{kind_note}; each timed step one decode token per "
                                       f"stream; " + ref.describe(t_dec, t_pre, t_head)},
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
    ap.add_argument("--workload", default="c3", choices=["c3", "c4"],
                    help="c3: the headline (configuration 3); c4: configuration 4's burst")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.workload == "c4":
        ours_c4(args, world, rank, local)
    elif args.impl == "reference":
        reference(args, world, rank)
    else:
        ours(args, world, rank, local)


if __name__ == "__main__":
    main()
