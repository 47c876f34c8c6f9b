"""Configuration 4's burst trace and the planner's cancellation (host only).

Every request arrives at t = 0; a random quarter is cancelled mid-decode; the
planner frees a cancelled request's slot the step its cancel point is reached,
and a waiting request takes it.
"""
from hllm_b200.workload import MixedPlanner, make_burst_trace


def run(trace, active=128):
    p = MixedPlanner(trace, max_active=active, prefill_budget=512)
    admitted_late, finished, steps, most = 0, [], 0, 0
    while p.active or p.next_req < len(trace):
        before = p.next_req
        p.admit()
        if steps > 0:
            admitted_late += p.next_req - before
        most = max(most, len(p.active))
        rows = p.plan()
        finished += p.commit(rows)
        steps += 1
        assert steps < 10000
    return finished, admitted_late, most


def test_burst_trace_shape():
    t = make_burst_trace(3)
    assert len(t) == 256
    assert all(r.arrival == 0.0 and 128 <= r.prompt_len <= 2048 and r.output_len == 256 for r in t)
    cancelled = [r for r in t if r.cancel_at]
    assert 0.15 * len(t) < len(cancelled) < 0.35 * len(t)
    assert all(1 <= r.cancel_at < 256 for r in cancelled)
    assert make_burst_trace(3)[17].prompt_len == t[17].prompt_len  # seeded


def test_cancelled_requests_stop_mid_decode_and_free_their_slots():
    t = make_burst_trace(5)
    finished, admitted_late, most = run(t)
    assert len(finished) == len(t) and most == 128
    assert admitted_late == len(t) - 128  # the second half runs in freed slots
    for r in t:
        if r.cancel_at:
            assert r.cancelled and r.generated == r.cancel_at
        else:
            assert r.generated == r.output_len and not r.cancelled
