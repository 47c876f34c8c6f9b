"""Per-GPU split of a worker's stage: the planner side of the multi-GPU pipeline.

The reference planner (python/hllm_control/planner/planner.py:246-330) places a
model on two workers as one or two contiguous stages; its DeploymentPlan holds
at most two (python/hllm_control/models.py:371-385).  A B200 worker with
several GPUs runs its stage as a pipeline of contiguous layer ranges, one per
GPU (``hllm_b200.pipeline``).  This module chooses that split from the
manifest's tensor records and checks every GPU with the reference's memory
model:

* ``stage_weight_bytes`` and ``stage_memory`` restate ``_stage_weight_bytes``
  and ``_stage_memory`` (planner.py:43-129) term for term, in the same
  arithmetic order, so one GPU's figures are the ones the reference planner
  prints for a stage of the same layers on that device;
* ``split_stage`` partitions a layer range over G GPUs so that the largest
  per-GPU cost is minimal.  The cost is either the bytes a GPU streams per
  decode step (``"stream"``: its layers' weights and their KV reads, the LM
  head on the last GPU, the embedding rows on the first), which sets the
  pipeline's period, or the reference's memory pressure (``"pressure"``, the
  quantity feasibility mode ranks first, planner.py:176-185).  A split in which
  some GPU's memory does not fit is never chosen while a fitting one exists;
  among equal optima the earlier GPUs take the extra layers;
* ``plan_worker`` applies it to one reference StageAssignment (or the whole
  model) and returns per-GPU assignments with the reference's ownership flags,
  memory records and rejection reasons in the reference's format
  (``<DOMAIN>_MEMORY_EXCEEDED:<worker>``, planner.py:283-285), the worker id
  of GPU g being ``<worker>/gpu<g>``.

Inputs use the reference's field names: a ModelManifest as a pydantic object
or its JSON form, and WorkerProfile / WorkloadProfile / StageAssignment as
objects or dicts; defaults are the reference models' defaults
(python/hllm_control/models.py:210-290).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Any, Callable, List, Mapping, Optional, Tuple

__all__ = ["DTYPE_BYTES", "PlanningError", "NoFeasibleSplit", "Tensor", "ModelShape", "usable_bytes",
           "stage_weight_bytes", "stage_memory", "stream_bytes", "split_costs",
           "split_stage", "plan_worker", "ranges_of", "shape_from_geometry", "B200_WORKER"]

# python/hllm_control/models.py:43-57
DTYPE_BYTES = {"BOOL": 1, "U8": 1, "I8": 1, "I16": 2, "U16": 2, "I32": 4, "U32": 4,
               "I64": 8, "U64": 8, "F16": 2, "BF16": 2, "F32": 4, "F64": 8}

_LAYER = "TRANSFORMER_LAYER"
_EMBED = "TOKEN_EMBEDDING"
_NORM = "FINAL_NORM"
_HEAD = "LM_HEAD"
_STATE = "ARCHITECTURE_STATE"


class PlanningError(ValueError):
    """Inconsistent planner inputs (the reference's PlanningError, planner.py:37)."""


class NoFeasibleSplit(PlanningError):
    """Every split of the stage leaves some GPU over its memory budget."""


def _get(obj: Any, name: str, default: Any = None) -> Any:
    if isinstance(obj, Mapping):
        return obj.get(name, default)
    return getattr(obj, name, default)


def _value(v: Any) -> Any:
    """Enum members (the reference's StrEnums) as their string values."""
    return getattr(v, "value", v)


@dataclass(frozen=True)
class Tensor:
    role: str
    layer_index: Optional[int]
    num_elements: int


@dataclass(frozen=True)
class ModelShape:
    """What the planner reads of a ModelManifest (models.py:196-207)."""
    num_layers: int
    hidden_size: int
    num_kv_heads: int
    head_dim: int
    vocabulary_size: int
    tied_embeddings: bool
    tensors: Tuple[Tensor, ...]

    @classmethod
    def from_manifest(cls, manifest: Any) -> "ModelShape":
        """From a ModelManifest object, its JSON form, or the compact form
        {"config": {...}, "tensors": [[role, layer_index, elements], ...]}."""
        config = _get(manifest, "config")
        tensors = []
        for t in _get(manifest, "tensors"):
            if isinstance(t, (list, tuple)):
                role, layer, n = t
            else:
                role, layer = _value(_get(t, "role")), _get(t, "layer_index")
                n = _get(t, "num_elements")
                if n is None:
                    n = 1
                    for dim in _get(t, "shape"):
                        n *= int(dim)
            tensors.append(Tensor(str(role), None if layer is None else int(layer), int(n)))
        return cls(num_layers=int(_get(config, "num_layers")),
                   hidden_size=int(_get(config, "hidden_size")),
                   num_kv_heads=int(_get(config, "num_kv_heads")),
                   head_dim=int(_get(config, "head_dim")),
                   vocabulary_size=int(_get(config, "vocabulary_size")),
                   tied_embeddings=bool(_get(config, "tied_embeddings")),
                   tensors=tuple(tensors))


class _Sums:
    """Element counts by role and a prefix sum over layers, so that a stage's
    weight bytes cost O(1) for any [start, end)."""

    def __init__(self, shape: ModelShape):
        L = shape.num_layers
        per_layer = [0] * L
        self.embed = self.norm = self.head = self.state = 0
        for t in shape.tensors:
            if t.role == _LAYER:
                if t.layer_index is not None and 0 <= t.layer_index < L:
                    per_layer[t.layer_index] += t.num_elements
            elif t.role == _EMBED:
                self.embed += t.num_elements
            elif t.role == _NORM:
                self.norm += t.num_elements
            elif t.role == _HEAD:
                self.head += t.num_elements
            elif t.role == _STATE:
                self.state += t.num_elements
        self.prefix = [0]
        for n in per_layer:
            self.prefix.append(self.prefix[-1] + n)
        self.tied = shape.tied_embeddings

    def elements(self, start: int, end: int, is_first: bool, is_final: bool) -> int:
        """planner.py:52-69: the stage's layers, the embedding on the first stage
        (and on the final one when tied), the final norm and untied head on the
        final stage, architecture state everywhere."""
        n = self.prefix[end] - self.prefix[start] + self.state
        if is_first or (is_final and self.tied):
            n += self.embed
        if is_final:
            n += self.norm
            if not self.tied:
                n += self.head
        return n


def shape_from_geometry(*, hidden_size: int, intermediate_size: int, attention_heads: int,
                        key_value_heads: int, head_dimension: int, layers: int,
                        vocabulary_size: int, query_key_norm: bool, tied: bool,
                        **_ignored) -> ModelShape:
    """The tensor records a Llama/Qwen3 checkpoint of this geometry carries, as
    the reference's prepare_model classifies them (embedding, final norm,
    untied LM head, and per layer the two norms, q/k/v/o, gate/up/down and the
    q/k norms when present): what the planner needs without a manifest."""
    h, I, d = hidden_size, intermediate_size, head_dimension
    q, kv = attention_heads * d, key_value_heads * d
    per_layer = [h, h, q * h, kv * h, kv * h, h * q, I * h, I * h, h * I]
    if query_key_norm:
        per_layer += [d, d]
    tensors = [Tensor(_EMBED, None, vocabulary_size * h), Tensor(_NORM, None, h)]
    if not tied:
        tensors.append(Tensor(_HEAD, None, vocabulary_size * h))
    for li in range(layers):
        tensors += [Tensor(_LAYER, li, n) for n in per_layer]
    return ModelShape(num_layers=layers, hidden_size=h, num_kv_heads=key_value_heads,
                      head_dim=d, vocabulary_size=vocabulary_size, tied_embeddings=tied,
                      tensors=tuple(tensors))


# One B200 as a planner worker profile (field names of the reference's
# WorkerProfile): 183,359 MiB of HBM3e, 2 GiB kept for the driver and context.
B200_WORKER = dict(worker_id="b200", endpoint="", backend="cuda",
                   primary_memory_domain="DEVICE",
                   supported_architectures=["llama.v1", "qwen3.v1"],
                   supported_execution_dtypes=["F16", "F32"],
                   memory_budgets=[dict(domain="DEVICE", capacity_bytes=183359 * 1024 * 1024,
                                        runtime_reserve_bytes=2 * 1024 ** 3,
                                        safety_fraction=0.05)],
                   fixed_workspace_bytes=4 * 1024 ** 3, activation_buffer_count=2,
                   allocator_allowance_fraction=0.05)


def usable_bytes(budget: Any) -> int:
    """MemoryBudget.usable_bytes (models.py:216-219)."""
    capacity = int(_get(budget, "capacity_bytes"))
    safety = int(capacity * float(_get(budget, "safety_fraction", 0.1)))
    return max(0, capacity - int(_get(budget, "runtime_reserve_bytes", 0)) - safety)


def _budget(worker: Any, domain: str) -> Any:
    for b in _get(worker, "memory_budgets", ()):
        if _value(_get(b, "domain")) == domain:
            return b
    return None


def stage_weight_bytes(shape: ModelShape, *, start: int, end: int, is_first: bool,
                       is_final: bool, dtype: str = "F16") -> int:
    """Resident weight bytes of layers [start, end) (planner.py:43-70)."""
    return _Sums(shape).elements(start, end, is_first, is_final) * DTYPE_BYTES[dtype]


class _Memory:
    """stage_memory's constants for one (shape, worker, workload, dtype)."""

    def __init__(self, shape: ModelShape, worker: Any, workload: Any, execution_dtype: str,
                 weight_dtype: Optional[str]):
        self.sums = _Sums(shape)
        self.domain = _value(_get(worker, "primary_memory_domain"))
        budget = _budget(worker, self.domain)
        if budget is None:
            raise PlanningError(f"worker {_get(worker, 'worker_id')} has no primary memory budget")
        self.usable = usable_bytes(budget)
        self.wbytes = DTYPE_BYTES[weight_dtype or execution_dtype]
        self.kv_per_layer_token = (2 * shape.num_kv_heads * shape.head_dim *
                                   DTYPE_BYTES[_value(_get(workload, "kv_dtype", "F16"))])
        self.cached = int(_get(workload, "total_cached_tokens"))
        self.overhead = float(_get(workload, "kv_overhead_factor", 1.1))
        payload = (int(_get(workload, "concurrency", 1)) * int(_get(workload, "prompt_tokens")) *
                   shape.hidden_size *
                   DTYPE_BYTES[_value(_get(workload, "activation_dtype", "F16"))])
        self.activation = payload * int(_get(worker, "activation_buffer_count", 2))
        workspace = int(_get(worker, "fixed_workspace_bytes", 0))
        if self.domain in ("HOST", "UNIFIED"):
            workspace += int(_get(worker, "host_transport_buffer_bytes", 0))
        self.workspace = workspace
        self.allowance = float(_get(worker, "allocator_allowance_fraction", 0.05))

    def record(self, worker_id: str, start: int, end: int, is_first: bool,
               is_final: bool) -> dict:
        # The same expressions, in the same order, as planner.py:87-129.
        weight = self.sums.elements(start, end, is_first, is_final) * self.wbytes
        kv = math.ceil((end - start) * self.cached * self.kv_per_layer_token * self.overhead)
        subtotal = weight + kv + self.workspace + self.activation
        allowance = math.ceil(subtotal * self.allowance)
        required = subtotal + allowance
        pressure = required / self.usable if self.usable else math.inf
        return {"worker_id": worker_id, "domain": self.domain, "layer_start": start,
                "layer_end": end, "weight_bytes": weight, "kv_cache_bytes": kv,
                "workspace_bytes": self.workspace, "activation_buffer_bytes": self.activation,
                "allocator_allowance_bytes": allowance, "required_bytes": required,
                "usable_bytes": self.usable, "pressure": pressure}


def stage_memory(shape: ModelShape, worker: Any, workload: Any, *, start: int, end: int,
                 is_first: bool, is_final: bool, execution_dtype: str = "F16",
                 weight_dtype: Optional[str] = None, worker_id: Optional[str] = None) -> dict:
    """The reference's StageMemory (planner.py:73-129) as a dict with its field
    names, for layers [start, end) on one device of `worker`."""
    m = _Memory(shape, worker, workload, execution_dtype, weight_dtype)
    return m.record(worker_id or _get(worker, "worker_id"), start, end, is_first, is_final)


def stream_bytes(shape: ModelShape, workload: Any, *, start: int, end: int, is_first: bool,
                 is_final: bool, dtype: str = "F16", kv_tokens: Optional[int] = None) -> int:
    """Bytes a GPU holding layers [start, end) reads per decode step: its layers'
    weights, `kv_tokens` (default: the workload's total_cached_tokens) of K/V
    per layer, the LM head (the embedding when tied) and final norm on the
    final stage, and one embedding row per concurrent request on the first."""
    return _Stream(shape, workload, dtype, kv_tokens)(start, end, is_first, is_final)


class _Stream:
    """stream_bytes with its per-model sums computed once."""

    def __init__(self, shape: ModelShape, workload: Any, dtype: str, kv_tokens: Optional[int]):
        self.sums = _Sums(shape)
        self.b = DTYPE_BYTES[dtype]
        self.kv_tokens = (int(_get(workload, "total_cached_tokens")) if kv_tokens is None
                          else int(kv_tokens))
        self.kv = 2 * shape.num_kv_heads * shape.head_dim * DTYPE_BYTES[
            _value(_get(workload, "kv_dtype", "F16"))]
        self.rows = int(_get(workload, "concurrency", 1)) * shape.hidden_size

    def __call__(self, start: int, end: int, is_first: bool, is_final: bool) -> int:
        sums = self.sums
        n = (sums.prefix[end] - sums.prefix[start]) * self.b + (end - start) * self.kv_tokens * self.kv
        if is_final:
            n += (sums.norm + (sums.embed if sums.tied else sums.head)) * self.b
        if is_first:
            n += self.rows * self.b
        return n


def split_costs(lo: int, hi: int, parts: int,
                cost: Callable[[int, int, int], float]) -> List[Tuple[int, int]]:
    """Contiguous ranges of [lo, hi) over `parts` parts, each non-empty, that
    minimise max_g cost(g, start_g, end_g); an infinite cost marks a range
    that is not allowed.  Among the splits with that least maximum it takes the
    one with the least sum of squared costs (the most even one), and among
    equal ones the one whose earlier parts are longer.  Raises PlanningError
    when every split has an infinite cost."""
    n = hi - lo
    if parts < 1 or n < parts:
        raise PlanningError(f"cannot split {n} layers over {parts} GPUs")
    inf = math.inf
    memo: dict = {}

    def c(g: int, s: int, e: int) -> float:
        key = (g, s, e)
        if key not in memo:
            memo[key] = float(cost(g, s, e))
        return memo[key]

    def ends(g: int, s: int) -> range:  # ends that leave a layer for every later part
        return range(s + 1, hi - (parts - 2 - g)) if g < parts - 1 else range(hi, hi + 1)

    def starts(g: int) -> range:
        return range(lo + g, hi - (parts - 1 - g))

    # Pass 1, suf[g][s]: the least max cost of parts g.. covering [s, hi).
    suf = [[inf] * (hi + 1) for _ in range(parts)]
    for g in range(parts - 1, -1, -1):
        for s in starts(g):
            suf[g][s] = min((max(c(g, s, e), suf[g + 1][e] if g < parts - 1 else -inf)
                             for e in ends(g, s)), default=inf)
    opt = suf[0][lo]
    if opt == inf:
        raise NoFeasibleSplit("no split of the stage fits every GPU")
    cap = opt + abs(opt) * 1e-12
    # Pass 2, sq[g][s]: the least sum of squares of parts g.. with every cost <= cap.
    sq = [[inf] * (hi + 1) for _ in range(parts + 1)]
    sq[parts][hi] = 0.0
    for g in range(parts - 1, -1, -1):
        for s in starts(g):
            best = inf
            for e in ends(g, s):
                v = c(g, s, e)
                if v <= cap and sq[g + 1][e] < inf:
                    best = min(best, v * v + sq[g + 1][e])
            sq[g][s] = best
    ranges, s = [], lo
    for g in range(parts):
        target = sq[g][s]
        for e in reversed(ends(g, s)):  # the longest part that keeps the optimum
            v = c(g, s, e)
            if v <= cap and sq[g + 1][e] < inf and \
                    v * v + sq[g + 1][e] <= target + abs(target) * 1e-12:
                ranges.append((s, e))
                s = e
                break
    return ranges


def _assignment(shape: ModelShape, assignment: Any) -> dict:
    if assignment is None:
        return {"stage_index": 0, "layer_start": 0, "layer_end": shape.num_layers,
                "owns_token_embedding": True, "owns_final_norm": True, "owns_lm_head": True,
                "owns_sampling": True}
    return {k: _get(assignment, k) for k in ("stage_index", "worker_id", "layer_start",
                                              "layer_end", "owns_token_embedding",
                                              "owns_final_norm", "owns_lm_head",
                                              "owns_sampling")}


def split_stage(shape: ModelShape, worker: Any, workload: Any, gpus: int, *,
                assignment: Any = None, objective: str = "stream",
                execution_dtype: str = "F16", weight_dtype: Optional[str] = None,
                kv_tokens: Optional[int] = None) -> List[Tuple[int, int]]:
    """Layer ranges of the assignment's stage (default: the whole model) over
    `gpus` GPUs of `worker`, each GPU with the worker's own budget."""
    a = _assignment(shape, assignment)
    lo, hi = int(a["layer_start"]), int(a["layer_end"])
    if objective not in ("stream", "pressure"):
        raise PlanningError(f"unknown objective {objective!r}")
    mem = _Memory(shape, worker, workload, execution_dtype, weight_dtype)
    first_owner, final_owner = bool(a["owns_token_embedding"]), bool(a["owns_lm_head"] or
                                                                       a["owns_final_norm"])
    dtype = weight_dtype or execution_dtype

    def flags(g: int) -> Tuple[bool, bool]:
        return first_owner and g == 0, final_owner and g == gpus - 1

    def fits(g: int, s: int, e: int) -> Optional[dict]:
        first, final = flags(g)
        rec = mem.record("", s, e, first, final)
        return rec if rec["required_bytes"] <= rec["usable_bytes"] else None

    stream = _Stream(shape, workload, dtype, kv_tokens)

    def cost(g: int, s: int, e: int) -> float:
        rec = fits(g, s, e)
        if rec is None:
            return math.inf
        if objective == "pressure":
            return rec["pressure"]
        return float(stream(s, e, *flags(g)))

    return split_costs(lo, hi, gpus, cost)


def plan_worker(shape: ModelShape, worker: Any, workload: Any, gpus: int, *,
                assignment: Any = None, objective: str = "stream",
                execution_dtype: str = "F16", weight_dtype: Optional[str] = None,
                kv_tokens: Optional[int] = None) -> dict:
    """The per-GPU plan of one worker's stage.  When no split fits, the plan is
    the pressure-balanced split with feasible=False and the reasons of every
    GPU that does not fit."""
    if gpus < 1:
        raise PlanningError("a worker needs at least one GPU")
    a = _assignment(shape, assignment)
    worker_id = str(_get(worker, "worker_id"))
    lo, hi = int(a["layer_start"]), int(a["layer_end"])
    if not 0 <= lo < hi <= shape.num_layers:
        raise PlanningError(f"stage layers [{lo}, {hi}) outside the model's {shape.num_layers}")
    if hi - lo < gpus:
        raise PlanningError(f"cannot split {hi - lo} layers over {gpus} GPUs")
    if objective not in ("stream", "pressure"):
        raise PlanningError(f"unknown objective {objective!r}")
    mem = _Memory(shape, worker, workload, execution_dtype, weight_dtype)
    try:
        ranges = split_stage(shape, worker, workload, gpus, assignment=assignment,
                             objective=objective, execution_dtype=execution_dtype,
                             weight_dtype=weight_dtype, kv_tokens=kv_tokens)
    except NoFeasibleSplit:
        # Nothing fits: show the split that comes closest.
        first_owner = bool(a["owns_token_embedding"])
        final_owner = bool(a["owns_lm_head"] or a["owns_final_norm"])
        ranges = split_costs(lo, hi, gpus, lambda g, s, e: mem.record(
            "", s, e, first_owner and g == 0, final_owner and g == gpus - 1)["pressure"])
    dtype = weight_dtype or execution_dtype
    entries, reasons = [], []
    for g, (s, e) in enumerate(ranges):
        first = bool(a["owns_token_embedding"]) and g == 0
        last = g == gpus - 1
        gid = f"{worker_id}/gpu{g}"
        rec = mem.record(gid, s, e, first, last and bool(a["owns_lm_head"] or
                                                         a["owns_final_norm"]))
        if rec["required_bytes"] > rec["usable_bytes"]:
            reasons.append(f"{rec['domain']}_MEMORY_EXCEEDED:{gid}")
        entries.append({
            "gpu": g, "worker_id": gid, "layer_start": s, "layer_end": e,
            "owns_token_embedding": first,
            "owns_final_norm": last and bool(a["owns_final_norm"]),
            "owns_lm_head": last and bool(a["owns_lm_head"]),
            "owns_sampling": last and bool(a["owns_sampling"]),
            "stream_bytes": stream_bytes(shape, workload, start=s, end=e, is_first=first,
                                         is_final=last and bool(a["owns_lm_head"] or
                                                                a["owns_final_norm"]),
                                         dtype=dtype, kv_tokens=kv_tokens),
            "memory": rec,
        })
    return {"worker_id": worker_id, "stage_index": a["stage_index"], "layer_start": lo,
            "layer_end": hi, "objective": objective, "gpus": entries,
            "feasible": not reasons, "rejection_reasons": reasons,
            "period_bytes": max(x["stream_bytes"] for x in entries),
            "max_pressure": max(x["memory"]["pressure"] for x in entries)}


def ranges_of(plan: Mapping) -> List[Tuple[int, int]]:
    """The per-GPU layer ranges of a plan_worker result, for pipeline ranks."""
    return [(g["layer_start"], g["layer_end"]) for g in plan["gpus"]]
