"""Pins the CPU oracle before anything is checked against it.

* Against the reference's Transformers fixture (tests/fixtures/qwen3/
  tiny-reference.json in the reference tree, converted into
  tests/golden/qwen3_tiny_reference.npz) at the reference's own 2e-5 tolerance
  (tests/cpp/qwen3_test.cpp:78-116).
* Against the reference's own CPU math: the golden tiny-Llama pipeline tokens
  and logits made by oracle/_ref must be reproduced bit for bit, and, where
  oracle/_ref is present, every function is compared element by element.
* The reference's hand-computed checks (tests/cpp/llama_test.cpp:70-150) and
  sampling known answers (tests/cpp/sampling_test.cpp).
"""
import ctypes as C
import math
import os

import numpy as np
import pytest

import oracle

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def tiny_qwen():
    d = np.load(os.path.join(GOLD, "qwen3_tiny_reference.npz"))
    h, I, Hq, Hkv, dim, maxpos, L, V = [int(x) for x in d["config"]]
    eps, theta = [float(x) for x in d["config_f"]]
    spec = oracle.ModelSpec(h, I, Hq, Hkv, dim, L, V, maxpos, eps, theta, True, True)
    weights = {k[2:]: d[k].astype(np.float32) for k in d.files if k.startswith("w/")}
    return spec, weights, d


@pytest.mark.parametrize("use_ref", [False, True])
def test_full_prefill_matches_transformers_layers_caches_logits(use_ref):
    if use_ref and oracle.ref() is None:
        pytest.skip("oracle/_ref not built")
    spec, weights, d = tiny_qwen()
    model = oracle.OracleModel(spec, weights, use_ref=use_ref)
    seq = model.new_sequence(spec.maximum_sequence_length)
    hidden = d["embeddings"][0].astype(np.float32)
    trace = []
    hidden = model.forward(hidden, 0, seq, trace)
    for layer in range(2):
        np.testing.assert_allclose(trace[layer], d[f"layer_outputs/{layer}"][0], atol=2e-5, rtol=0)
        k, v = model.kv(seq, layer)
        # Transformers stores [batch, kv_head, sequence, head_dim].
        np.testing.assert_allclose(k.transpose(1, 0, 2), d[f"keys/{layer}"][0], atol=2e-5, rtol=0)
        np.testing.assert_allclose(v.transpose(1, 0, 2), d[f"values/{layer}"][0], atol=2e-5,
                                   rtol=0)
    np.testing.assert_allclose(model.logits(hidden), d["logits"][0], atol=2e-5, rtol=0)
    model.free_sequence(seq)


def test_prefill_and_two_decode_steps_match_transformers():
    spec, weights, d = tiny_qwen()
    model = oracle.OracleModel(spec, weights)
    seq = model.new_sequence(spec.maximum_sequence_length)
    for position, count in ((0, 3), (3, 1), (4, 1)):
        hidden = d["embeddings"][0][position:position + count].astype(np.float32)
        trace = []
        hidden = model.forward(hidden, position, seq, trace)
        for layer in range(2):
            np.testing.assert_allclose(trace[layer],
                                       d[f"layer_outputs/{layer}"][0][position:position + count],
                                       atol=2e-5, rtol=0)
        np.testing.assert_allclose(model.logits(hidden),
                                   d["logits"][0][position:position + count], atol=2e-5, rtol=0)


def test_restatement_equals_reference_bit_for_bit_on_tiny_llama_pipeline():
    """Golden tokens/logits were made by oracle/_ref; the C restatement must
    reproduce them exactly (same order of F32 operations)."""
    from tests.golden.make_golden import C1, C1_SEED
    g = np.load(os.path.join(GOLD, "tiny_llama_pipeline.npz"))
    weights = oracle.synth_weights(C1, C1_SEED)
    s0 = oracle.OracleModel(C1, weights, 0, 2)
    s1 = oracle.OracleModel(C1, weights, 2, 4)
    lens = g["prompt_lengths"]
    offs = np.concatenate([[0], np.cumsum(lens)])
    for r in range(2):  # two requests keep the CPU suite fast; all four run on the GPU box
        prompt = g["prompt_ids"][offs[r]:offs[r + 1]]
        a, b = s0.new_sequence(len(prompt) + 32), s1.new_sequence(len(prompt) + 32)
        inp, pos = list(prompt), 0
        for step in range(32):
            h = oracle.f16_round(s0.forward(s0.embed(inp), pos, a))
            h = s1.forward(h, pos, b)
            lg = s1.logits(h[-1:])
            if r == 0:
                assert np.array_equal(lg[0], g["logits_request0"][step])
            tok = oracle.greedy(lg)
            assert tok == g["tokens"][r, step]
            pos += len(inp)
            inp = [tok]


# The attention geometry of the benchmark configurations, on small hidden and
# vocabulary sizes: C2 (16q/8kv, d 128, q/k-norm, tied), C3 (32q/8kv, d 128,
# q/k-norm, tied), C4 (12q/4kv: G = 3, d 256, no q/k-norm, untied).
GEOMETRIES = {
    "c2": dict(attention_heads=16, key_value_heads=8, head_dimension=128, query_key_norm=True,
               tied=True),
    "c3": dict(attention_heads=32, key_value_heads=8, head_dimension=128, query_key_norm=True,
               tied=True),
    "c4": dict(attention_heads=12, key_value_heads=4, head_dimension=256, query_key_norm=False,
               tied=False),
}


@pytest.mark.parametrize("name", sorted(GEOMETRIES))
def test_restatement_equals_reference_layers_at_config_geometries(name):
    """Two layers of the C restatement against the reference's own
    transformer_layer and final_logits (oracle/_ref, built from
    cpp/src/cpu/llama.cpp): a 37-token prefill, then three decode tokens;
    every layer output, every logit and both layers' K/V caches equal bit
    for bit."""
    if oracle.ref() is None:
        pytest.skip("oracle/_ref not built")
    spec = oracle.ModelSpec(hidden_size=256, intermediate_size=512, layers=2,
                            vocabulary_size=640, maximum_sequence_length=4096,
                            rms_norm_epsilon=1e-6, rope_theta=1e6, **GEOMETRIES[name])
    weights = oracle.synth_weights(spec, 77)
    ours = oracle.OracleModel(spec, weights)
    theirs = oracle.OracleModel(spec, weights, use_ref=True)
    a, b = ours.new_sequence(64), theirs.new_sequence(64)
    rng = np.random.default_rng(len(name))
    inp, pos = [int(x) for x in rng.integers(0, spec.vocabulary_size, 37)], 0
    for _ in range(4):
        ta, tb = [], []
        ha = ours.forward(ours.embed(inp), pos, a, trace=ta)
        hb = theirs.forward(theirs.embed(inp), pos, b, trace=tb)
        for x, y in zip(ta, tb):
            assert np.array_equal(x, y)
        la, lb = ours.logits(ha[-1:]), theirs.logits(hb[-1:])
        assert np.array_equal(la, lb)
        pos += len(inp)
        inp = [oracle.greedy(la)]
    for layer in range(spec.layers):  # the caches hold the same K and V
        for x, y in zip(ours.kv(a, layer), theirs.kv(b, layer)):
            assert x.shape == (pos, spec.key_value_heads, spec.head_dimension)
            assert np.array_equal(x, y)
    theirs.free_sequence(b)


def test_restatement_equals_reference_functions():
    r = oracle.ref()
    if r is None:
        pytest.skip("oracle/_ref not built")
    rng = np.random.default_rng(3)
    x = rng.standard_normal((5, 96)).astype(np.float32)
    w = rng.standard_normal(96).astype(np.float32)
    a = oracle.rms_norm(x, w, 1e-6)
    b = np.empty_like(x)
    assert r.ref_rms_norm(oracle.fp(x), oracle.fp(w), 5, 96, 1e-6, oracle.fp(b)) == 0
    assert np.array_equal(a, b)
    W = rng.standard_normal((33, 96)).astype(np.float32)
    a = oracle.linear(x, W)
    b = np.empty((5, 33), np.float32)
    assert r.ref_linear(oracle.fp(x), 5, 96, oracle.fp(W), 33, oracle.fp(b)) == 0
    assert np.array_equal(a, b)
    q = rng.standard_normal((7, 3 * 128)).astype(np.float32)
    a = oracle.apply_rope(q, 3, 128, 4000, 1e6)
    b = q.copy()
    assert r.ref_apply_rope(oracle.fp(b), 7, 3, 128, 4000, 1e6) == 0
    assert np.array_equal(a, b)
    vals = np.concatenate([rng.standard_normal(20000).astype(np.float32) * 10,
                           np.float32([0, -0.0, 65504, 65520, 1e-8, 6e-8, 3e-5, -7e4, np.inf,
                                       -np.inf, np.nan])])
    for v in vals:
        assert oracle.lib().oracle_f32_to_f16(float(v)) == r.ref_float_to_float16(float(v))
    for bits in range(0, 65536, 7):
        fa = oracle.lib().oracle_f16_to_f32(bits)
        fb = r.ref_float16_to_float(bits)
        assert (fa == fb) or (math.isnan(fa) and math.isnan(fb))


def test_sampler_restatement_equals_reference_at_full_vocabulary():
    """oracle.sample_token against the reference's own sample_token
    (cpp/src/sampling.cpp:19-90, in oracle/_ref) on full-vocabulary rows of the
    benchmark models: configuration 4's seeded T 0.7 / top-p 0.9 draws over many
    draw counters, greedy, top-k with logprobs and top-5 logprobs, and rows with
    tied maxima.  Tokens, logprobs and top lists are equal exactly."""
    r = oracle.ref()
    if r is None:
        pytest.skip("oracle/_ref not built")
    rng = np.random.default_rng(11)
    opts = [oracle.sampling(0.7, 0.9, 0, 1000 + i) for i in range(4)] + [
        oracle.sampling(),
        oracle.sampling(0.0, 1.0, 0, 0, True, 5),
        oracle.sampling(1.0, 1.0, 40, 7, True, 5),
        oracle.sampling(1.3, 0.5, 0, 9, True, 2),
        oracle.sampling(0.7, 0.9, 100, 123, True, 0)]
    for V in (131072, 151936):
        rows = [rng.standard_normal(V).astype(np.float32) * 3]
        tied = rng.standard_normal(V).astype(np.float32)
        tied[[5, 77, V - 1]] = tied.max() + 1.0  # three equal maxima
        rows.append(tied)
        rows.append(np.round(rng.standard_normal(V) * 2).astype(np.float32))  # many ties
        for lg in rows:
            for o in opts:
                for gi in (0, 1, 17):
                    st_a, a = oracle.sample_token(lg, o, gi)
                    b = oracle.Sampled()
                    st_b = r.ref_sample_token(oracle.fp(lg), V, C.byref(o), gi, C.byref(b))
                    assert st_a == st_b == 0
                    assert a.token_id == b.token_id
                    assert (a.has_logprob, a.n_top) == (b.has_logprob, b.n_top)
                    assert a.logprob == b.logprob
                    assert list(a.top_ids[:a.n_top]) == list(b.top_ids[:b.n_top])
                    assert list(a.top_logprobs[:a.n_top]) == list(b.top_logprobs[:b.n_top])


def test_rms_norm_hand_calculation():
    out = oracle.rms_norm(np.float32([[3.0, 4.0]]), np.float32([1.0, 2.0]), 1e-6)
    inv = 1.0 / math.sqrt(12.5 + 1e-6)
    assert abs(out[0, 0] - 3 * inv) < 1e-6 and abs(out[0, 1] - 8 * inv) < 1e-6


def test_rope_half_rotation_layout():
    v = oracle.apply_rope(np.float32([[1, 2, 3, 4]]), 1, 4, 1, 1e4)
    assert abs(v[0, 0] - (math.cos(1) - 3 * math.sin(1))) < 1e-6
    assert abs(v[0, 2] - (3 * math.cos(1) + math.sin(1))) < 1e-6
    assert abs(v[0, 1] - (2 * math.cos(0.01) - 4 * math.sin(0.01))) < 1e-6


def test_greedy_first_maximum_and_nonfinite_refusal():
    assert oracle.greedy(np.float32([[9, 1, 2, 3], [-1, 4, 4, 0]])) == 1
    for row in ([np.nan, 1, 2], [1, np.nan, 2], [1, 2, np.inf], [-np.inf, 0, 1]):
        assert oracle.greedy(np.float32([[0, 0, 0], row])) == -1
    assert oracle.greedy(np.float32([[np.nan] * 3, [0, 5, 1]])) == 1


def test_sampling_known_answers_from_reference():
    g = np.load(os.path.join(GOLD, "sampling_kat.npz"))
    for i in range(len(g["n"])):
        n = int(g["n"][i])
        o = g["options"][i]
        opts = oracle.sampling(o[0], o[1], int(o[2]), int(o[3]), bool(o[4]), int(o[5]))
        st, res = oracle.sample_token(g["logits"][i][:n], opts, int(g["generated_index"][i]))
        assert st == 0
        assert res.token_id == g["token"][i], i
        if o[4]:
            assert res.logprob == g["logprob"][i]
            assert res.n_top == g["n_top"][i]
            for k in range(res.n_top):
                assert res.top_ids[k] == g["top_ids"][i][k]
                assert res.top_logprobs[k] == g["top_logprobs"][i][k]


def test_sampling_greedy_filtering_and_invalid_inputs():
    lg = np.float32([0, 2, 2])
    assert oracle.sample_token(lg, oracle.sampling(), 0)[1].token_id == 1
    for seed in range(100):
        assert oracle.sample_token(lg, oracle.sampling(1.0, 1.0, 1, seed), 0)[1].token_id == 1
        assert oracle.sample_token(lg, oracle.sampling(1.0, 0.1, 0, seed), 0)[1].token_id == 1
    assert oracle.sample_token(lg, oracle.sampling(-1.0), 0)[0] != 0
    assert oracle.sample_token(lg, oracle.sampling(1.0, 0.0), 0)[0] != 0
    assert oracle.sample_token(np.float32([np.nan]), oracle.sampling(), 0)[0] != 0


def test_sampling_request_randomness_and_distribution():
    lg = np.float32([0, 0, 0])
    counts = [0, 0, 0]
    for step in range(6000):
        t = oracle.sample_token(lg, oracle.sampling(1.0, 1.0, 0, 42), step)[1].token_id
        counts[t] += 1
        assert t == oracle.sample_token(lg, oracle.sampling(1.0, 1.0, 0, 42), step)[1].token_id
    assert all(1800 < c < 2200 for c in counts)


def test_logprobs_known_answer():
    st, res = oracle.sample_token(np.float32([0, 0, 0]), oracle.sampling(0.0, 1.0, 0, 42, True, 2), 0)
    assert st == 0 and res.token_id == 0
    assert abs(res.logprob + math.log(3)) < 1e-12
    assert res.n_top == 2 and res.top_ids[0] == 0 and res.top_ids[1] == 1
    assert oracle.sample_token(np.float32([0, 0, 0]),
                               oracle.sampling(0.0, 1.0, 0, 42, True, 6), 0)[0] != 0


def test_combine_decode_inputs_reference_rules():
    """cpp/src/decode_batch.cpp:8-38 through oracle/_ref: ready, distinct
    single-token sequences combine; anything else is an invalid request."""
    r = oracle.ref()
    if r is None:
        pytest.skip("oracle/_ref not built")

    def run(ids, counts, positions, prefilling, prefill_only, same):
        n = len(counts)
        ids = np.asarray(ids, np.uint64)
        out = np.zeros(max(1, ids.size), np.uint64)
        u8 = lambda a: np.asarray(a, np.uint8).ctypes.data_as(C.POINTER(C.c_uint8))
        keep = [np.asarray(prefilling, np.uint8), np.asarray(prefill_only, np.uint8)]
        st = r.ref_combine_decode_tokens(
            ids.ctypes.data_as(C.POINTER(C.c_uint64)),
            np.asarray(counts, np.uint64).ctypes.data_as(C.POINTER(C.c_uint64)),
            np.asarray(positions, np.uint64).ctypes.data_as(C.POINTER(C.c_uint64)),
            keep[0].ctypes.data_as(C.POINTER(C.c_uint8)), keep[1].ctypes.data_as(C.POINTER(C.c_uint8)),
            np.asarray(same, np.int32).ctypes.data_as(C.POINTER(C.c_int32)), n,
            out.ctypes.data_as(C.POINTER(C.c_uint64)))
        del u8
        return st, out

    st, out = run([4, 5, 6], [1, 1, 1], [7, 2, 4], [0, 0, 0], [0, 0, 0], [-1, -1, -1])
    assert st == 0 and list(out) == [4, 5, 6]
    assert run([4, 5], [1, 1], [7, 0], [0, 0], [0, 0], [-1, -1])[0] == 1      # position 0
    assert run([4, 5], [1, 1], [7, 3], [0, 1], [0, 0], [-1, -1])[0] == 1      # prefilling
    assert run([4, 5], [1, 1], [7, 3], [0, 0], [0, 1], [-1, -1])[0] == 1      # prefill_only
    assert run([4, 5], [1, 1], [7, 3], [0, 0], [0, 0], [-1, 0])[0] == 1       # same sequence
    assert run([4, 5, 6], [2, 1], [7, 3], [0, 0], [0, 0], [-1, -1])[0] == 1   # two tokens


def test_packer_restatement_properties():
    rng = np.random.default_rng(11)
    slots, mb, B = 12, 40, 16
    perm = rng.permutation(slots * mb).astype(np.int32)
    blocks = perm.reshape(slots, mb)
    row_slot = np.int32([3, 0, 7, 11])
    row_first = np.int32([0, 35, 600, 17])
    row_count = np.int32([29, 1, 33, 1])
    p = oracle.pack(row_slot, row_first, row_count, blocks, B)
    assert list(p["cu_seqlens"]) == [0, 29, 30, 63, 64]
    assert list(p["seq_lens"]) == [29, 36, 633, 18]
    for t in range(64):
        r = p["token_row"][t]
        pos = p["positions"][t]
        assert row_first[r] <= pos < row_first[r] + row_count[r]
        assert p["slot_mapping"][t] == blocks[row_slot[r], pos // B] * B + pos % B
    need = (p["seq_lens"] + B - 1) // B
    for r in range(4):
        assert np.array_equal(p["block_tables"][r, :need[r]], blocks[row_slot[r], :need[r]])
        assert (p["block_tables"][r, need[r]:] == -1).all()
    holes = blocks.copy()
    holes[7, 39] = -1
    assert oracle.pack(row_slot, row_first, row_count, holes, B) is None
    assert oracle.pack(row_slot, np.int32([0, 35, 630, 17]), row_count, blocks, B) is None


def test_synthetic_generator_statistics_and_determinism():
    a = oracle.synth_matrix(5, 17, (512, 512))
    b = oracle.synth_matrix(5, 17, (512, 512))
    assert np.array_equal(a, b)
    x = oracle.f16_decode(a)
    assert abs(float(x.mean())) < 5e-4
    assert abs(float(x.std()) - 0.02) < 5e-4
    assert not np.array_equal(a, oracle.synth_matrix(5, 18, (512, 512)))
    n = oracle.f16_decode(oracle.synth_norm(5, 3, 4096))
    assert n.min() >= 0.899 and n.max() <= 1.1
