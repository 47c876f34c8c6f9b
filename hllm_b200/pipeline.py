"""Pipeline stages across GPUs: one process per GPU, one contiguous layer range per rank.

hLLM splits a model into contiguous layer ranges ("stages"); the first stage
embeds token ids, every stage passes its F16 boundary activation to the next,
and the final stage applies the final norm and LM head and samples
(cpp/src/cpu/stage.cpp:129-191; the F16 boundary encode/decode at :143-158 and
:179-190; two-stage plans from python/hllm_control/planner/planner.py:246-330).
Here every rank of a torch.distributed job owns one stage on its own B200:

* layers are split by the bytes each stage streams per step
  (``partition_layers``), the LM head counting as V*h / P_layer layers on the
  last stage;
* boundaries go GPU to GPU with NCCL send/recv on the stage's CUDA stream (no
  host round trip), through two send slots so that a stage can start its next
  step while its last boundary is still in flight;
* N independent micro-batches keep the N stages busy: at tick t rank r runs
  micro-batch (t - r) mod N (``Schedule``), so rank r + 1 receives at tick
  t + 1 what rank r sent at tick t, and the tokens the last rank samples at
  tick t are exactly what rank 0 needs at tick t + 1;
* sampled token ids travel back from the last rank to rank 0 over a gloo
  group on the host (they feed rank 0's host-side inputs).

``HostLinks`` carries the same messages between CPU processes over gloo, so
the schedule and the message order can be tested without GPUs.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, List, Optional, Sequence, Tuple

import numpy as np

__all__ = ["partition_layers", "Schedule", "run_ticks", "HostLinks", "DeviceLinks",
           "device_view", "stage_bytes", "make_groups"]


def partition_layers(n_layers: int, n_stages: int, layer_bytes: float,
                     head_bytes: float = 0.0) -> List[Tuple[int, int]]:
    """Contiguous ranges [(start, end)] of `n_layers` layers over `n_stages`
    stages that minimise the most bytes any stage streams per step: a stage
    costs (its layers) x `layer_bytes`, plus `head_bytes` on the last stage.
    Every stage gets at least one layer; among equal optima the most even
    split wins, then the one whose earlier stages are longer
    (``hllm_b200.planner.split_costs``, which also plans from a manifest's
    per-layer bytes)."""
    from .planner import split_costs

    return split_costs(0, n_layers, n_stages,
                       lambda g, s, e: (e - s) * layer_bytes +
                       (head_bytes if g == n_stages - 1 else 0.0))


def stage_bytes(ranges: Sequence[Tuple[int, int]], layer_bytes: float,
                head_bytes: float) -> List[float]:
    """Per-stage streamed bytes of a partition (the head on the last stage)."""
    out = [(e - s) * layer_bytes for s, e in ranges]
    out[-1] += head_bytes
    return out


@dataclass(frozen=True)
class Schedule:
    """Micro-batch schedule of an N-stage pipeline.

    Every micro-batch runs `steps` steps; step j of micro-batch m is run by
    rank r at tick j * N + m + r.  Rank r is busy for ticks
    [r, r + N * steps); the whole run takes N * steps + N - 1 ticks."""
    world: int
    steps: int

    @property
    def ticks(self) -> int:
        return self.world * self.steps + self.world - 1

    def work(self, rank: int, tick: int) -> Optional[Tuple[int, int]]:
        """(micro-batch, step) that `rank` runs at `tick`, or None."""
        k = tick - rank
        if k < 0 or k >= self.world * self.steps:
            return None
        j, m = divmod(k, self.world)
        return m, j

    def tick_of(self, rank: int, microbatch: int, step: int) -> int:
        return step * self.world + microbatch + rank


def run_ticks(schedule: Schedule, rank: int, on_tick: Callable[[int, int, int], None],
              ticks: Optional[range] = None) -> None:
    """Calls on_tick(tick, microbatch, step) for every tick at which `rank` works."""
    for t in (ticks if ticks is not None else range(schedule.ticks)):
        w = schedule.work(rank, t)
        if w is not None:
            on_tick(t, w[0], w[1])


# ---------------------------------------------------------------------------- links
class HostLinks:
    """Boundary activations (F16 bits as int16) and sampled tokens between CPU
    processes over gloo: the same messages, in the same order, as DeviceLinks.
    Sends do not block (a blocking send of rank r's boundary and of the last
    rank's tokens would wait for each other within one tick); drain() waits
    for them."""

    def __init__(self, rank: int, world: int, hidden: int, group=None):
        self.rank, self.world, self.hidden, self.group = rank, world, hidden, group
        self.pending = []

    def recv_activation(self, tokens: int) -> np.ndarray:
        import torch
        import torch.distributed as dist
        buf = torch.empty((tokens, self.hidden), dtype=torch.int16)
        dist.recv(buf, src=self.rank - 1, group=self.group)
        return buf.numpy().view(np.uint16)

    def send_activation(self, bits: np.ndarray) -> None:
        import torch
        import torch.distributed as dist
        t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16).copy())
        self.pending.append((dist.isend(t, dst=self.rank + 1, group=self.group), t))

    def send_tokens(self, ids: np.ndarray) -> None:
        import torch
        import torch.distributed as dist
        t = torch.from_numpy(np.array(ids, np.int64))
        self.pending.append((dist.isend(t, dst=0, group=self.group), t))

    def drain(self) -> None:
        for work, _ in self.pending:
            work.wait()
        self.pending = []

    def recv_tokens(self, count: int) -> np.ndarray:
        import torch
        import torch.distributed as dist
        buf = torch.empty(count, dtype=torch.int64)
        dist.recv(buf, src=self.world - 1, group=self.group)
        return buf.numpy()


def make_groups(world: int, pairs: bool = True, timeout_s: float = 120.0):
    """The pipeline's process groups, created collectively by every rank, in
    one order: (NCCL group of each neighbour pair (r, r + 1), or None when
    `pairs` is false so that boundaries use the default group; a gloo group of
    all ranks for the sampled tokens, which only ranks 0 and N - 1 exchange,
    with a `timeout_s` limit on each exchange).

    Every group has every rank as a member or, for the NCCL pairs, is NCCL
    itself.  With a process group bound to its device (eager NCCL
    initialisation), ``new_group`` makes each rank outside a new group join a
    no-colour split of the default NCCL communicator, which the group's
    members also run only when the new group is NCCL.  A gloo group {0, N - 1}
    therefore left ranks 1 .. N - 2 blocked in that split at N >= 3 (observed
    at four GPUs: ranks 0 and 3 then waited in their first send and receive).
    Separate pair groups give each link its own NCCL communicator and stream,
    so a middle rank's receive from the left and send to the right do not
    serialise on one communicator."""
    import datetime
    import torch.distributed as dist
    pair_groups = [dist.new_group([r, r + 1]) for r in range(world - 1)] if pairs else None
    tokens = dist.new_group(list(range(world)), backend="gloo",
                            timeout=datetime.timedelta(seconds=timeout_s))
    return pair_groups, tokens


class _CudaArray:
    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3,
                                         "strides": None}


def device_view(ptr: int, shape, dtype="float16"):
    """A torch CUDA tensor over device memory the library owns (no copy)."""
    import torch
    typestr = {"float16": "<f2", "int32": "<i4", "float32": "<f4"}[dtype]
    return torch.as_tensor(_CudaArray(ptr, shape, typestr), device="cuda")


class DeviceLinks:
    """A rank's links: NCCL point-to-point for F16 boundaries on the stage's
    stream, and a host-side gloo group (all ranks; only 0 and N-1 exchange)
    for sampled tokens.

    recv_activation posts the receive on the stage stream (the stage's next
    work waits for it; the host does not).  send_activation copies the
    boundary into one of two send slots on the stage stream and posts the
    send; a slot is reused only after its previous send completed (the stage
    stream waits for it), so the boundary buffer itself is free as soon as the
    copy ran."""

    def __init__(self, rank: int, world: int, stream, max_tokens: int, hidden: int,
                 token_group=None, pair_groups=None):
        import torch
        self.rank, self.world, self.stream = rank, world, stream
        self.hidden = hidden
        self.token_group = token_group
        # optional NCCL communicator per neighbour pair (else the default group)
        self.recv_group = pair_groups[rank - 1] if pair_groups and rank > 0 else None
        self.send_group = pair_groups[rank] if pair_groups and rank < world - 1 else None
        dev = torch.device("cuda", torch.cuda.current_device())
        self.recv_buf = torch.empty((max_tokens, hidden), dtype=torch.float16, device=dev)
        self.send_bufs = [torch.empty((max_tokens, hidden), dtype=torch.float16, device=dev)
                          for _ in range(2)]
        self.send_work = [None, None]
        self.sends = 0
        self.token_sends = []

    def connect(self) -> None:
        """Opens every neighbour link before the first step, in one order on all
        ranks.  NCCL point-to-point communicators are created on first use, and
        creating one blocks the host until both ends take part; a link first
        used inside the schedule could then hold one rank's host in creation
        while its peer waits in a collective.  Here the links open as a chain
        (0 -> 1, then 1 -> 2, ...): each rank first receives from its left
        neighbour, then sends to its right one, so every creation meets its
        peer.  Called collectively by all ranks after construction."""
        import torch
        import torch.distributed as dist
        probe = torch.zeros(1, self.hidden, dtype=torch.float16, device=self.recv_buf.device)
        with torch.cuda.stream(self.stream):
            if self.rank > 0:
                dist.recv(self.recv_buf[:1], src=self.rank - 1, group=self.recv_group)
            if self.rank < self.world - 1:
                dist.send(probe, dst=self.rank + 1, group=self.send_group)
        self.stream.synchronize()

    def recv_activation(self, tokens: int) -> int:
        import torch
        import torch.distributed as dist
        with torch.cuda.stream(self.stream):
            dist.recv(self.recv_buf[:tokens], src=self.rank - 1, group=self.recv_group)
        return self.recv_buf.data_ptr()

    def send_activation(self, boundary, tokens: int) -> None:
        import torch
        import torch.distributed as dist
        k = self.sends % 2
        self.sends += 1
        with torch.cuda.stream(self.stream):
            if self.send_work[k] is not None:
                self.send_work[k].wait()
            self.send_bufs[k][:tokens].copy_(boundary[:tokens])
            self.send_work[k] = dist.isend(self.send_bufs[k][:tokens], dst=self.rank + 1,
                                           group=self.send_group)

    def drain(self) -> None:
        """Waits for the sends still in flight (boundaries: on the stage stream)."""
        import torch
        with torch.cuda.stream(self.stream):
            for k in range(2):
                if self.send_work[k] is not None:
                    self.send_work[k].wait()
                    self.send_work[k] = None
        for work, _ in self.token_sends:
            work.wait()
        self.token_sends = []

    def send_tokens(self, ids: np.ndarray) -> None:
        """Posts the last rank's sampled ids to rank 0 (host, non-blocking)."""
        import torch
        import torch.distributed as dist
        t = torch.from_numpy(np.array(ids, np.int64))
        self.token_sends = [w for w in self.token_sends if not w[0].is_completed()]
        self.token_sends.append((dist.isend(t, dst=0, group=self.token_group), t))

    def recv_tokens(self, count: int) -> np.ndarray:
        import torch
        import torch.distributed as dist
        buf = torch.empty(count, dtype=torch.int64)
        dist.recv(buf, src=self.world - 1, group=self.token_group)
        return buf.numpy()
