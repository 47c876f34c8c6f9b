"""Pipeline host logic on CPU: layer partition, micro-batch schedule, and the
message order of a 2-rank pipeline over gloo.

The 2-rank test runs configuration 1 (tiny Llama) as stages 0-1 | 2-3 in two
processes, each rank computing its layers with the oracle, with the F16
boundary and the sampled tokens exchanged by hllm_b200.pipeline.HostLinks on
the ticks hllm_b200.pipeline.Schedule assigns (two micro-batches of two
requests).  The generated tokens must equal the reference's own two-stage run
(tests/golden/tiny_llama_pipeline.npz, made by oracle/_ref) exactly.
"""
import os
import socket

import numpy as np
import pytest

from hllm_b200.pipeline import Schedule, partition_layers, run_ticks, stage_bytes

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_partition_balances_streamed_bytes():
    layer, head = 201.85e6, 777.9e6  # Qwen3-4B layer and LM-head F16 bytes
    assert partition_layers(36, 1, layer, head) == [(0, 36)]
    assert partition_layers(36, 2, layer, head) == [(0, 20), (20, 36)]
    assert partition_layers(36, 4, layer, head) == [(0, 10), (10, 20), (20, 30), (30, 36)]
    eight = partition_layers(36, 8, layer, head)
    assert eight[-1] == (35, 36) and all(e - s == 5 for s, e in eight[:-1])
    for n in range(1, 9):
        r = partition_layers(36, n, layer, head)
        assert r[0][0] == 0 and r[-1][1] == 36
        assert all(a[1] == b[0] and a[1] > a[0] for a, b in zip(r, r[1:]))
        best = max(stage_bytes(r, layer, head))
        # no single-layer move between neighbours lowers the maximum
        for i in range(n - 1):
            for d in (-1, 1):
                moved = [list(x) for x in r]
                moved[i][1] += d
                moved[i + 1][0] += d
                if all(e > s for s, e in moved):
                    assert max(stage_bytes(moved, layer, head)) >= best - 1e-6
    with pytest.raises(ValueError):
        partition_layers(3, 4, 1.0)


def test_schedule_hands_each_step_to_the_next_rank_one_tick_later():
    for world in (1, 2, 3, 8):
        s = Schedule(world, 5)
        seen = {r: [] for r in range(world)}
        for t in range(s.ticks):
            for r in range(world):
                w = s.work(r, t)
                if w is None:
                    continue
                seen[r].append(w)
                m, j = w
                assert s.tick_of(r, m, j) == t
                if r + 1 < world:
                    assert s.work(r + 1, t + 1) == w          # boundary: one tick later
                if r == world - 1 and j + 1 < s.steps:
                    assert s.work(0, t + 1) == (m, j + 1)     # sampled tokens: next tick
        for r in range(world):
            assert sorted(seen[r]) == sorted((m, j) for m in range(world) for j in range(5))
        calls = []
        run_ticks(s, world - 1, lambda t, m, j: calls.append((t, m, j)))
        assert len(calls) == world * 5


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _rank_main(rank, world, port, out_q, fail_at=None, pg_timeout_s=None):
    """One pipeline rank over gloo.  `fail_at` = (rank, tick) makes that rank
    raise at the start of that tick (a host-side failure); every rank reports
    an exception as ("error", rank, text) on `out_q`."""
    import datetime
    import torch.distributed as dist
    import oracle
    from hllm_b200.pipeline import HostLinks, Schedule, partition_layers, run_ticks
    from tests.golden.make_golden import C1, C1_SEED, c1_workload

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    kw = {"timeout": datetime.timedelta(seconds=pg_timeout_s)} if pg_timeout_s else {}
    dist.init_process_group("gloo", rank=rank, world_size=world, **kw)
    try:
        steps = 32
        lo, hi = partition_layers(C1.layers, world, 1.0)[rank]
        weights = oracle.synth_weights(C1, C1_SEED)
        model = oracle.OracleModel(C1, weights, lo, hi)
        prompts = c1_workload()
        # micro-batch m holds requests m, m + world, ...
        mbs = [list(range(m, len(prompts), world)) for m in range(world)]
        seqs = {r: model.new_sequence(len(prompts[r]) + steps) for r in range(len(prompts))}
        pos = {r: 0 for r in range(len(prompts))}
        last = {}
        tokens = np.zeros((len(prompts), steps), np.int64)
        links = HostLinks(rank, world, C1.hidden_size)
        sched = Schedule(world, steps)

        def tick(t, m, j):
            if fail_at == (rank, t):
                raise RuntimeError(f"injected failure on rank {rank} at tick {t}")
            reqs = mbs[m]
            if rank == 0 and j > 0:
                fed = links.recv_tokens(len(reqs)) if world > 1 else np.asarray(
                    [last[r] for r in reqs])
                for r, tok in zip(reqs, fed):
                    last[r] = int(tok)
            # every rank knows the rows' lengths; only rank 0 needs the ids
            lens = [len(prompts[r]) if j == 0 else 1 for r in reqs]
            if rank == 0:
                hs = [model.embed(list(prompts[r]) if j == 0 else [last[r]]) for r in reqs]
            else:
                bits = links.recv_activation(sum(lens))
                hs, o = [], 0
                for n in lens:
                    hs.append(oracle.f16_decode(bits[o:o + n]))
                    o += n
            outs = []
            for r, h in zip(reqs, hs):
                outs.append(model.forward(h, pos[r], seqs[r]))
                pos[r] += h.shape[0]
            if rank < world - 1:
                links.send_activation(np.concatenate([oracle.f16_encode(h) for h in outs]))
                return
            ids = np.asarray([oracle.greedy(model.logits(h[-1:])) for h in outs], np.int64)
            for r, tok in zip(reqs, ids):
                tokens[r, j] = tok
                last[r] = int(tok)
            if world > 1 and j + 1 < steps:
                links.send_tokens(ids)

        try:
            run_ticks(sched, rank, tick)
            links.drain()
        except Exception as e:  # noqa: BLE001 -- reported to the parent, then re-raised
            out_q.put(("error", rank, repr(e)))
            raise
        if rank == world - 1:
            out_q.put(tokens)
    finally:
        dist.destroy_process_group()


def _in_process_tokens(world, steps=32):
    """The same pipeline run stage after stage in one process (F16 boundary
    between consecutive stages), request by request."""
    import oracle
    from tests.golden.make_golden import C1, C1_SEED, c1_workload
    weights = oracle.synth_weights(C1, C1_SEED)
    models = [oracle.OracleModel(C1, weights, lo, hi)
              for lo, hi in partition_layers(C1.layers, world, 1.0)]
    prompts = c1_workload()
    tokens = np.zeros((len(prompts), steps), np.int64)
    for r, prompt in enumerate(prompts):
        seqs = [m.new_sequence(len(prompt) + steps) for m in models]
        inp, pos = list(prompt), 0
        for j in range(steps):
            h = models[0].embed(inp)
            for k, (m, sq) in enumerate(zip(models, seqs)):
                if k:
                    h = oracle.f16_round(h)
                h = m.forward(h, pos, sq)
            tokens[r, j] = oracle.greedy(models[-1].logits(h[-1:]))
            pos += len(inp)
            inp = [int(tokens[r, j])]
    return tokens


def _run_ranks(world):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        tokens = q.get(timeout=240)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    return tokens


@pytest.mark.timeout(300)
def test_three_rank_pipeline_over_gloo_matches_the_in_process_run():
    """A middle rank receives from rank 0 and sends to rank 2 on every tick;
    three micro-batches (requests {0, 3}, {1}, {2}) follow the schedule."""
    np.testing.assert_array_equal(_run_ranks(3), _in_process_tokens(3))


@pytest.mark.timeout(300)
def test_four_rank_pipeline_over_gloo_matches_the_in_process_run():
    """One layer per rank; four micro-batches ({0}, {1}, {2}, {3}) keep every
    rank busy, two middle ranks relay every tick."""
    np.testing.assert_array_equal(_run_ranks(4), _in_process_tokens(4))


@pytest.mark.timeout(300)
def test_two_rank_pipeline_over_gloo_matches_the_reference_two_stage_run():
    g = np.load(os.path.join(GOLD, "tiny_llama_pipeline.npz"))
    np.testing.assert_array_equal(_run_ranks(2), g["tokens"])


@pytest.mark.timeout(300)
def test_a_failing_rank_ends_the_others_with_an_error_not_a_hang():
    """Rank 1 of three raises at tick 4 (a host-side failure between its
    exchanges).  Its neighbours learn of it at their next exchange with it:
    the receive fails (the peer closed its connection, or the process group's
    10 s timeout ran out) and each surviving rank exits with its own error
    well inside the limit, instead of waiting forever."""
    import multiprocessing as mp
    import time
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    world = 3
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q, (1, 4), 10))
             for r in range(world)]
    t0 = time.monotonic()
    for p in procs:
        p.start()
    errors = {}
    try:
        while len(errors) < world and time.monotonic() - t0 < 120:
            try:
                msg = q.get(timeout=5)
            except Exception:  # noqa: BLE001 -- queue.Empty: keep waiting
                continue
            if isinstance(msg, tuple) and msg[0] == "error":
                errors[msg[1]] = msg[2]
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert "injected failure on rank 1 at tick 4" in errors.get(1, "")
    assert set(errors) == {0, 1, 2}, errors
    assert all(p.exitcode not in (0, None) for p in procs)
    assert time.monotonic() - t0 < 200
