"""One rank of the 2-GPU pipeline parity check (run by tests/test_gpu_pipeline.py
under torch.distributed.run, one process per GPU).

Configuration 1 (tiny Llama) as stages 0-1 | 2-3 on two B200s: rank 0 embeds and
runs layers 0-1, sends its F16 boundary to rank 1 over NCCL
(hllm_b200.pipeline.DeviceLinks); rank 1 runs layers 2-3, the final norm and
LM head, samples greedily and sends the tokens back to rank 0.  Two
micro-batches of two requests follow hllm_b200.pipeline.Schedule.  Rank 1
then checks, per request and step, the GPU logits against the oracle on the
GPU's own token path and the tokens against the reference's two-stage golden
run up to the first near-tie, and writes the verdict to argv[1].
"""
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

LOGIT_TOL = 2e-2
GAP = 1e-2
STEPS = 32


def main(out_path):
    import datetime
    import torch
    import torch.distributed as dist
    import oracle
    from hllm_b200 import B200Stage, ModelConfig, _lib
    from hllm_b200.pipeline import DeviceLinks, Schedule, device_view, make_groups, run_ticks
    from tests.golden.make_golden import C1, C1_SEED

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    assert world == 2
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", local))
    pair_groups, token_group = make_groups(world)
    L = _lib.lib()
    g = np.load(os.path.join(ROOT, "tests", "golden", "tiny_llama_pipeline.npz"))
    lens = g["prompt_lengths"]
    offs = np.concatenate([[0], np.cumsum(lens)])
    prompts = [[int(x) for x in g["prompt_ids"][offs[r]:offs[r + 1]]] for r in range(4)]
    spec = C1
    cfg = ModelConfig(spec.hidden_size, spec.intermediate_size, spec.attention_heads,
                      spec.key_value_heads, spec.head_dimension, spec.maximum_sequence_length,
                      spec.rms_norm_epsilon, spec.rope_theta, spec.query_key_norm,
                      spec.vocabulary_size, spec.layers, spec.tied)
    lo, hi = (0, 2) if rank == 0 else (2, 4)
    stage = B200Stage(cfg, lo, hi, first=rank == 0, final=rank == 1, device=local,
                      kv_pool_tokens=4096, max_step_tokens=128, max_step_rows=8, max_sequences=8)
    stage.init_synthetic(C1_SEED)
    stream = torch.cuda.ExternalStream(L.hllm_b200_stage_stream(stage.handle))
    links = DeviceLinks(rank, world, stream, 128, cfg.hidden_size, token_group=token_group,
                        pair_groups=pair_groups)
    links.connect()
    boundary = None if rank == 1 else device_view(L.hllm_b200_stage_boundary(stage.handle),
                                                  (128, cfg.hidden_size))
    mbs = [[0, 2], [1, 3]]
    seqs = {r: stage.allocate_sequence(len(prompts[r]) + STEPS) for r in range(4)}
    pos = {r: 0 for r in range(4)}
    last = {}
    tokens = np.zeros((4, STEPS), np.int64)
    logits = {r: [] for r in range(4)}
    ids_dev = torch.empty(128, dtype=torch.int32, device="cuda")
    greedy = _lib.Sampling(0.0, 1.0, 0, 0, 0, 0)

    def tick(t, m, j):
        reqs = mbs[m]
        if rank == 0 and j > 0:
            for r, tok in zip(reqs, links.recv_tokens(len(reqs))):
                last[r] = int(tok)
        rows_ids = [prompts[r] if j == 0 else [last[r]] for r in reqs]
        n_tok = sum(len(x) for x in rows_ids)
        arr = (_lib.Row * len(reqs))()
        for k, (r, ids) in enumerate(zip(reqs, rows_ids)):
            arr[k].sequence = seqs[r].handle
            arr[k].first_position = pos[r]
            arr[k].tokens = len(ids)
            arr[k].sample = 1
            arr[k].sampling = greedy
        if rank == 0:
            flat = torch.tensor([x for ids in rows_ids for x in ids], dtype=torch.int32).pin_memory()
            with torch.cuda.stream(stream):
                ids_dev[:n_tok].copy_(flat, non_blocking=True)
            ptr = ids_dev.data_ptr()
        else:
            ptr = links.recv_activation(n_tok)
        _lib.check(L.hllm_b200_step_async(stage.handle, arr, len(reqs), ptr))
        for r, ids in zip(reqs, rows_ids):
            pos[r] += len(ids)
        if rank == 0:
            links.send_activation(boundary, n_tok)
            return
        _lib.check(L.hllm_b200_stage_sync(stage.handle))
        out = (_lib.Sampled * len(reqs))()
        _lib.check(L.hllm_b200_stage_results(stage.handle, out, len(reqs)))
        lg = stage.read_logits(len(reqs))
        ids = np.asarray([out[k].token_id for k in range(len(reqs))], np.int64)
        for k, r in enumerate(reqs):
            tokens[r, j] = ids[k]
            last[r] = int(ids[k])
            logits[r].append(lg[k].copy())
        if j + 1 < STEPS:
            links.send_tokens(ids)

    run_ticks(Schedule(world, STEPS), rank, tick)
    links.drain()
    _lib.check(L.hllm_b200_stage_sync(stage.handle))
    torch.cuda.synchronize()
    verdict = {"ok": True, "detail": []}
    if rank == 1:
        weights = oracle.synth_weights(spec, C1_SEED)
        o0 = oracle.OracleModel(spec, weights, 0, 2)
        o1 = oracle.OracleModel(spec, weights, 2, 4)
        for r in range(4):
            oa, ob = o0.new_sequence(len(prompts[r]) + STEPS), o1.new_sequence(len(prompts[r]) + STEPS)
            inp, p, agree = prompts[r], 0, True
            for j in range(STEPS):
                h = oracle.f16_round(o0.forward(o0.embed(inp), p, oa))
                ol = o1.logits(o1.forward(h, p, ob)[-1:])[0]
                err = float(np.max(np.abs(logits[r][j] - ol)))
                if err >= LOGIT_TOL:
                    verdict["ok"] = False
                    verdict["detail"].append(f"request {r} step {j}: logit error {err}")
                if agree:
                    part = np.partition(ol, -2)
                    if part[-1] - part[-2] < GAP:
                        agree = False
                    elif not (tokens[r, j] == int(np.argmax(ol)) == int(g["tokens"][r, j])):
                        verdict["ok"] = False
                        verdict["detail"].append(f"request {r} step {j}: token {tokens[r, j]}")
                p += len(inp)
                inp = [int(tokens[r, j])]
        verdict["tokens"] = tokens.tolist()
        with open(out_path, "w") as f:
            json.dump(verdict, f)
    for s in seqs.values():
        stage.release(s)
    stage.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1])
