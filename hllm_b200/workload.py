"""Continuous-batching workload of hLLM's Qwen3-4B configuration and a
mixed prefill/decode step planner.

The reference scheduler (cpp/src/worker/scheduler.cpp:27-67) runs a prefill
chunk alone or a decode batch of at most 8; it never mixes them.  This planner
is the optional mixed-batch extension: every step carries one decode row for
each running sequence plus prefill chunks from the oldest still-prefilling
requests, up to a per-step prefill token budget (512 = the chunk size of the
configuration).  Rows of intermediate chunks produce no token
(PrefillProgress); the row holding a prompt's last chunk samples the first
token.

Workload (configuration 3): 64 concurrent requests; Poisson arrivals at
8 req/s (kept as the admission order; throughput runs admit a request as soon
as a slot frees); prompt lengths log-normal (median 512, sigma 1.0) clipped to
[32, 4096]; output lengths uniform in [64, 512]; uniform random token ids;
greedy decoding.  All draws come from one recorded seed.

Workload (configuration 4, ``make_burst_trace``): Falcon3-3B geometry; every
request arrives at t = 0; prompt lengths uniform in [128, 2048]; 256 output
tokens each; temperature 0.7 / top-p 0.9 with a seed per request; a random
25% are cancelled mid-decode (after a uniform 1..255 of their tokens), which
frees their KV blocks and slots for requests still waiting.  128 run at once.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

QWEN3_4B = dict(hidden_size=2560, intermediate_size=9728, attention_heads=32, key_value_heads=8,
                head_dimension=128, layers=36, vocabulary_size=151936,
                maximum_sequence_length=4608, rms_norm_epsilon=1e-6, rope_theta=1e6,
                query_key_norm=True, tied=True)


FALCON3_3B = dict(hidden_size=3072, intermediate_size=9216, attention_heads=12,
                  key_value_heads=4, head_dimension=256, layers=22, vocabulary_size=131072,
                  maximum_sequence_length=2304, rms_norm_epsilon=1e-6, rope_theta=1e6,
                  query_key_norm=False, tied=False)


@dataclass
class Request:
    rid: int
    arrival: float
    prompt_len: int
    output_len: int
    prefilled: int = 0
    generated: int = 0
    admitted_step: int = -1
    first_token_step: int = -1
    cancel_at: int = 0  # cancelled once this many tokens are generated (0: never)

    @property
    def cancelled(self) -> bool:
        return 0 < self.cancel_at <= self.generated < self.output_len

    @property
    def done(self) -> bool:
        return self.generated >= self.output_len or self.cancelled

    @property
    def capacity(self) -> int:
        return self.prompt_len + self.output_len


def make_trace(seed: int, n_requests: int = 2048, rate: float = 8.0, median: float = 512.0,
               sigma: float = 1.0, lo: int = 32, hi: int = 4096, out_lo: int = 64,
               out_hi: int = 512):
    rng = np.random.default_rng(seed)
    arrivals = np.cumsum(rng.exponential(1.0 / rate, n_requests))
    prompts = np.clip(np.round(rng.lognormal(np.log(median), sigma, n_requests)), lo, hi)
    outs = rng.integers(out_lo, out_hi + 1, n_requests)
    return [Request(i, float(arrivals[i]), int(prompts[i]), int(outs[i]))
            for i in range(n_requests)]


def make_burst_trace(seed: int, n_requests: int = 256, prompt_lo: int = 128,
                     prompt_hi: int = 2048, output_len: int = 256,
                     cancel_fraction: float = 0.25):
    """Configuration 4's bursty trace: every request arrives at t = 0, and a
    random `cancel_fraction` of them are cancelled mid-decode."""
    rng = np.random.default_rng(seed)
    prompts = rng.integers(prompt_lo, prompt_hi + 1, n_requests)
    cancel = rng.random(n_requests) < cancel_fraction
    at = rng.integers(1, output_len, n_requests)
    return [Request(i, 0.0, int(prompts[i]), output_len,
                    cancel_at=int(at[i]) if cancel[i] else 0) for i in range(n_requests)]


@dataclass
class RowPlan:
    req: Request
    first_position: int
    tokens: int
    sample: bool
    decode: bool


@dataclass
class MixedPlanner:
    """Plans steps over a request trace; token values play no part in the plan."""
    trace: list
    max_active: int = 64
    prefill_budget: int = 512
    active: list = field(default_factory=list)
    next_req: int = 0
    step_index: int = 0

    def admit(self, on_admit=None, until=None):
        """Admits requests in trace order while slots are free; with `until`,
        only requests that have arrived by then (open-loop arrivals)."""
        while len(self.active) < self.max_active and self.next_req < len(self.trace):
            r = self.trace[self.next_req]
            if until is not None and r.arrival > until:
                break
            self.next_req += 1
            r.admitted_step = self.step_index
            self.active.append(r)
            if on_admit:
                on_admit(r)

    def plan(self):
        rows = []
        for r in self.active:
            if r.prefilled == r.prompt_len and 0 < r.generated < r.output_len:
                rows.append(RowPlan(r, r.prompt_len + r.generated - 1, 1, True, True))
        budget = self.prefill_budget
        for r in self.active:
            if budget <= 0:
                break
            if r.prefilled < r.prompt_len:
                c = min(budget, r.prompt_len - r.prefilled)
                rows.append(RowPlan(r, r.prefilled, c, r.prefilled + c == r.prompt_len, False))
                budget -= c
        return rows

    def commit(self, rows, on_finish=None):
        for row in rows:
            r = row.req
            if row.decode:
                r.generated += 1
            else:
                r.prefilled += row.tokens
                if row.sample:
                    r.generated = 1
                    r.first_token_step = self.step_index
        finished = [r for r in self.active if r.done]
        self.active = [r for r in self.active if not r.done]
        if on_finish:
            for r in finished:
                on_finish(r)
        self.step_index += 1
        return finished


def step_tokens(rows) -> int:
    return sum(r.tokens for r in rows)
