"""Regenerates the golden fixtures in this folder.

Run in a container that has the reference tree (read-only) and its CPU math
built into oracle/_ref (``make -C oracle``):

    python tests/golden/make_golden.py /path/to/reference

Outputs (small, committed):

* ``qwen3_tiny_reference.npz`` -- the reference's Transformers oracle fixture
  (tests/fixtures/qwen3/tiny-reference.json in the reference tree: a 2-layer
  Qwen3 with h=6, I=10, Hq=4, Hkv=2, d=4, V=11, tied, eps 1e-6, theta 1e6, tokens
  [1,4,2,8,3]), converted to arrays: every weight, the embeddings, per-layer
  outputs, K/V caches ([kv_head, seq, dim]) and logits.
* ``tiny_llama_pipeline.npz`` -- configuration 1 (tiny Llama, F32, 4 layers,
  h256, 4q/2kv, d64, I688, V4096, untied, theta 1e4, eps 1e-5) run by the
  reference's own CPU math (oracle/_ref) as a 2-stage pipeline 0-1 | 2-3 with
  the F16 boundary between stages, on the seeded synthetic weights: 4 requests,
  prompt lengths U[7,33], ids U[0,4096), 32 greedy tokens each, plus the final
  logits of every step of request 0.
* ``sampling_kat.npz`` -- sample_token outputs of the reference sampler for
  seeded logits and option sets (greedy, temperature, top-k, top-p, logprobs).
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle  # noqa: E402

C1 = oracle.ModelSpec(hidden_size=256, intermediate_size=688, attention_heads=4,
                      key_value_heads=2, head_dimension=64, layers=4, vocabulary_size=4096,
                      maximum_sequence_length=128, rms_norm_epsilon=1e-5, rope_theta=1e4,
                      query_key_norm=False, tied=False)
C1_SEED = 20261201


def tiny_qwen(ref_root: str) -> None:
    path = os.path.join(ref_root, "tests", "fixtures", "qwen3", "tiny-reference.json")
    with open(path) as f:
        d = json.load(f)
    arrays = {}
    for name, t in d["weights"].items():
        arrays["w/" + name] = np.asarray(t["values"], np.float64).reshape(t["shape"])
    for key in ("embeddings", "logits"):
        arrays[key] = np.asarray(d[key]["values"], np.float64).reshape(d[key]["shape"])
    for key in ("layer_outputs", "keys", "values"):
        for i, t in enumerate(d[key]):
            arrays[f"{key}/{i}"] = np.asarray(t["values"], np.float64).reshape(t["shape"])
    c = d["config"]
    arrays["config"] = np.asarray([c["hidden_size"], c["intermediate_size"],
                                   c["num_attention_heads"], c["num_key_value_heads"],
                                   c["head_dim"], c["max_position_embeddings"],
                                   c["num_hidden_layers"], c["vocab_size"]], np.int64)
    arrays["config_f"] = np.asarray([c["rms_norm_eps"], c["rope_theta"]], np.float64)
    arrays["tokens"] = np.asarray([1, 4, 2, 8, 3], np.int64)
    np.savez_compressed(os.path.join(HERE, "qwen3_tiny_reference.npz"), **arrays)


def c1_workload(seed=C1_SEED):
    rng = np.random.default_rng(seed)
    lengths = rng.integers(7, 34, size=4)
    prompts = [rng.integers(0, 4096, size=int(n)) for n in lengths]
    return prompts


def tiny_llama() -> None:
    assert oracle.ref() is not None, "build oracle/_ref first (make -C oracle)"
    weights = oracle.synth_weights(C1, C1_SEED)
    stage0 = oracle.OracleModel(C1, weights, 0, 2, use_ref=True)
    stage1 = oracle.OracleModel(C1, weights, 2, 4, use_ref=True)
    prompts = c1_workload()
    steps = 32
    tokens = np.zeros((4, steps), np.int64)
    logits0 = []
    for r, prompt in enumerate(prompts):
        s0 = stage0.new_sequence(len(prompt) + steps)
        s1 = stage1.new_sequence(len(prompt) + steps)
        inp = list(prompt)
        pos = 0
        for step in range(steps):
            h = stage0.forward(stage0.embed(inp), pos, s0)
            h = oracle.f16_round(h)  # cpp/src/cpu/stage.cpp:179-190 then :143-158
            h = stage1.forward(h, pos, s1)
            lg = stage1.logits(h[-1:])
            tok = oracle.greedy(lg)
            tokens[r, step] = tok
            if r == 0:
                logits0.append(lg[0])
            pos += len(inp)
            inp = [tok]
        stage0.free_sequence(s0)
        stage1.free_sequence(s1)
    lens = np.asarray([len(p) for p in prompts], np.int64)
    flat = np.concatenate(prompts).astype(np.int64)
    np.savez_compressed(os.path.join(HERE, "tiny_llama_pipeline.npz"), prompt_lengths=lens,
                        prompt_ids=flat, tokens=tokens, logits_request0=np.asarray(logits0),
                        seed=np.asarray([C1_SEED]))


def sampling_kat() -> None:
    r = oracle.ref()
    rng = np.random.default_rng(7)
    cases = []
    option_sets = [
        (0.0, 1.0, 0, 3, 0, 0), (0.0, 1.0, 0, 3, 1, 5), (0.7, 0.9, 0, 11, 0, 0),
        (1.0, 1.0, 0, 42, 1, 2), (0.8, 0.95, 8, 43, 1, 3), (1.3, 0.5, 0, 99, 0, 0),
        (0.7, 1.0, 50, 5, 0, 0), (2.0, 0.2, 3, 77, 1, 1),
    ]
    logits_all, opts, idx, out_tok, out_lp, out_top_ids, out_top_lp, out_ntop = \
        [], [], [], [], [], [], [], []
    for n in (3, 11, 4096):
        for k in range(6):
            lg = (rng.standard_normal(n) * (1.0 + k)).astype(np.float32)
            if k == 5:
                lg[:] = np.round(lg)  # many exact ties
            for o in option_sets:
                gi = int(rng.integers(0, 1000))
                s = oracle.sampling(*o)
                res = oracle.Sampled()
                import ctypes as C
                st = r.ref_sample_token(oracle.fp(lg), n, C.byref(s), gi, C.byref(res))
                assert st == 0
                cases.append(n)
                logits_all.append(np.pad(lg, (0, 4096 - n)))
                opts.append(o)
                idx.append(gi)
                out_tok.append(res.token_id)
                out_lp.append(res.logprob if res.has_logprob else np.nan)
                out_top_ids.append(list(res.top_ids))
                out_top_lp.append(list(res.top_logprobs))
                out_ntop.append(res.n_top)
    np.savez_compressed(os.path.join(HERE, "sampling_kat.npz"), n=np.asarray(cases),
                        logits=np.asarray(logits_all, np.float32), options=np.asarray(opts,
                                                                                      np.float64),
                        generated_index=np.asarray(idx, np.uint64),
                        token=np.asarray(out_tok, np.uint64), logprob=np.asarray(out_lp),
                        top_ids=np.asarray(out_top_ids, np.uint64),
                        top_logprobs=np.asarray(out_top_lp), n_top=np.asarray(out_ntop))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <reference tree>")
    root = sys.argv[1]
    tiny_qwen(root)
    tiny_llama()
    sampling_kat()
    print("golden fixtures written to", HERE)
