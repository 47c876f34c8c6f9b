"""Per-kernel parity of the sm_100a kernels against the CPU oracle, called
through the C ABI (include/hllm_b200.h, kernel entry points).

Tolerances: integer/index work (packer, KV placement) is bit-exact; GEMMs are
checked against float64 products of the same F16 inputs (F32 accumulate:
atol/rtol 1e-4 for F32 outputs, 2e-3 for F16 outputs); attention against the
oracle's F32 attention on the same F16 q/k/v (2e-3, the outputs are F16);
sampled tokens are exact, logprobs within 1e-9.
"""
import ctypes as C
import math
import os

import numpy as np
import pytest

import oracle
from hllm_b200 import _lib
from tests.gpu_util import check, dev, f16_bits, f16_vals, host, ptr, stream, sync, torch_cuda

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def lib():
    torch_cuda()
    return _lib.lib()


# ----------------------------------------------------------------------------- GEMM
def run_gemm(W, X, n, epi, Y, m, k_pad, pair=1, second_row=0, bn=0, grid=0, ldy=None):
    check(lib().hllm_b200_gemm(ptr(W), m, k_pad, pair, second_row, ptr(X), n, epi, ptr(Y),
                               ldy if ldy is not None else Y.shape[1], bn, grid, stream()))
    sync()


def padded(a, k_pad):
    out = np.zeros((a.shape[0], k_pad), a.dtype)
    out[:, :a.shape[1]] = a
    return out


@pytest.mark.parametrize("m,k,n,bn,grid", [
    (256, 256, 16, 0, 0), (300, 688, 5, 0, 7), (1024, 2560, 64, 0, 0), (128, 64, 1, 0, 0),
    (6144, 2560, 575, 0, 0), (2560, 4096, 64, 0, 0), (1000, 1024, 100, 16, 0),
    (1000, 1024, 100, 32, 3), (1000, 1024, 100, 64, 148), (1000, 1024, 100, 128, 1),
    (1000, 1024, 300, 256, 5), (4096, 256, 48, 0, 0), (129, 128, 17, 0, 2)])
def test_gemm_store_f32_matches_float64_reference(m, k, n, bn, grid):
    rng = np.random.default_rng(m * 7 + k + n)
    k_pad = (k + 63) // 64 * 64
    Wb = f16_bits(rng.standard_normal((m, k)).astype(np.float32) * 0.05)
    Xb = f16_bits(rng.standard_normal((n, k)).astype(np.float32))
    ref = f16_vals(Xb).astype(np.float64) @ f16_vals(Wb).astype(np.float64).T
    W = dev(padded(Wb, k_pad))
    X = dev(padded(Xb, k_pad))
    torch = torch_cuda()
    Y = torch.full((n, m), float("nan"), dtype=torch.float32, device="cuda")
    run_gemm(W, X, n, 0, Y, m, k_pad, bn=bn, grid=grid)
    np.testing.assert_allclose(host(Y), ref, rtol=1e-4, atol=1e-4)


def test_gemm_f16_store_residual_and_repeat_determinism():
    torch = torch_cuda()
    rng = np.random.default_rng(5)
    m, k, n = 2560, 9728, 40
    Wb = f16_bits(rng.standard_normal((m, k)).astype(np.float32) * 0.02)
    Xb = f16_bits(rng.standard_normal((n, k)).astype(np.float32))
    ref = f16_vals(Xb).astype(np.float64) @ f16_vals(Wb).astype(np.float64).T
    W, X = dev(Wb), dev(Xb)
    Y16 = torch.zeros((n, m), dtype=torch.int16, device="cuda")
    run_gemm(W, X, n, 1, Y16, m, k)
    np.testing.assert_allclose(f16_vals(host(Y16, np.uint16)), ref, rtol=2e-3, atol=2e-3)
    base = rng.standard_normal((n, m)).astype(np.float32)
    Y = dev(base)
    run_gemm(W, X, n, 2, Y, m, k)
    first = host(Y)
    np.testing.assert_allclose(first, base + ref, rtol=1e-4, atol=1e-4)
    # Split tiles are reduced in a fixed order: repeated runs are bit-identical.
    for grid in (0, 0, 37):
        Y2 = dev(base)
        run_gemm(W, X, n, 2, Y2, m, k, grid=grid)
        if grid == 0:
            assert np.array_equal(host(Y2), first)


@pytest.mark.parametrize("I,k,n,grid", [(1000, 256, 33, 0), (9728, 2560, 64, 0),
                                        (256, 128, 7, 5), (9728, 2560, 200, 0)])
def test_gemm_swiglu_pair(I, k, n, grid):
    torch = torch_cuda()
    rng = np.random.default_rng(I + n)
    Wb = f16_bits(rng.standard_normal((2 * I, k)).astype(np.float32) * 0.05)
    Xb = f16_bits(rng.standard_normal((n, k)).astype(np.float32))
    full = f16_vals(Xb).astype(np.float64) @ f16_vals(Wb).astype(np.float64).T
    g, u = full[:, :I], full[:, I:]
    ref = g / (1.0 + np.exp(-g)) * u
    Y = torch.zeros((n, I), dtype=torch.int16, device="cuda")
    run_gemm(dev(Wb), dev(Xb), n, 3, Y, I, k, pair=2, second_row=I, grid=grid)
    np.testing.assert_allclose(f16_vals(host(Y, np.uint16)), ref, rtol=3e-3, atol=3e-3)


def test_gemm_refuses_a_grid_beyond_its_scratch():
    """The library's stream-K scratch holds one CTA per SM: a grid override of
    two CTAs per SM with wide tiles would write past it and is refused before
    any launch."""
    torch = torch_cuda()
    m, k, n = 2560, 4096, 256
    W = torch.zeros((m, k), dtype=torch.float16, device="cuda")
    X = torch.zeros((n, k), dtype=torch.float16, device="cuda")
    Y = torch.zeros((n, m), dtype=torch.float32, device="cuda")
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    st = lib().hllm_b200_gemm(ptr(W), m, k, 1, 0, ptr(X), n, 0, ptr(Y), m, 256, 2 * sms, stream())
    assert st == _lib.RESOURCE_EXHAUSTED
    assert "scratch holds" in _lib.last_error()


# ----------------------------------------------------------------------------- RMSNorm
def test_rmsnorm_matches_oracle():
    torch = torch_cuda()
    rng = np.random.default_rng(1)
    for rows, width in ((5, 6), (64, 2560), (3, 1024), (17, 3072)):
        x = rng.standard_normal((rows, width)).astype(np.float32)
        w = (1 + 0.1 * rng.standard_normal(width)).astype(np.float32)
        ref = oracle.rms_norm(x, w, 1e-6)
        out = torch.zeros((rows, width + 64), dtype=torch.int16, device="cuda")
        xd, wd = dev(x), dev(w)  # keep device inputs alive until the kernel has run
        check(lib().hllm_b200_rmsnorm(ptr(xd), rows, width, ptr(wd), 1e-6, ptr(out),
                                      width + 64, stream()))
        sync()
        got = f16_vals(host(out, np.uint16))
        np.testing.assert_allclose(got[:, :width], ref, rtol=2e-3, atol=1e-3)
        assert (host(out)[:, width:] == 0).all()


# ----------------------------------------------------------------------------- packer
def pack_case(rng, slots=24, max_blocks=64, rows=17):
    perm = rng.permutation(slots * max_blocks).astype(np.int32)
    blocks = perm.reshape(slots, max_blocks)
    row_slot = rng.choice(slots, size=rows, replace=False).astype(np.int32)
    row_count = np.where(rng.random(rows) < 0.6, 1, rng.integers(2, 80, rows)).astype(np.int32)
    row_first = rng.integers(0, max_blocks * 16 - 80, rows).astype(np.int32)
    return blocks, row_slot, row_first, row_count


@pytest.mark.parametrize("seed", range(6))
def test_pack_bit_exact_against_oracle(seed):
    torch = torch_cuda()
    rng = np.random.default_rng(seed)
    blocks, row_slot, row_first, row_count = pack_case(rng)
    # ragged edge cases: a single row, maximum positions, one-token rows only
    if seed == 4:
        row_slot, row_first, row_count = row_slot[:1], row_first[:1], row_count[:1]
    if seed == 5:
        row_count[:] = 1
        row_first[:] = 64 * 16 - 1
    R, T, MB = row_slot.size, int(row_count.sum()), blocks.shape[1]
    ref = oracle.pack(row_slot, row_first, row_count, blocks, 16)
    split, qt = 48, 16
    o = {k: torch.full(v.shape if v.ndim else (1,), -7, dtype=torch.int32, device="cuda")
         for k, v in ref.items()}
    cu_splits = torch.zeros(R + 1, dtype=torch.int32, device="cuda")
    cu_qtiles = torch.zeros(R + 1, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    ins = [dev(x) for x in (row_slot, row_first, row_count, blocks)]
    check(lib().hllm_b200_pack(ptr(ins[0]), ptr(ins[1]), ptr(ins[2]), R, T,
                               ptr(ins[3]), MB, split, qt, ptr(o["cu_seqlens"]),
                               ptr(o["positions"]), ptr(o["slot_mapping"]), ptr(o["token_row"]),
                               ptr(o["seq_lens"]), ptr(o["block_tables"]), ptr(cu_splits),
                               ptr(cu_qtiles), ptr(status), stream()))
    sync()
    for k, v in ref.items():
        assert np.array_equal(host(o[k]), v), k
    assert int(host(status)[0]) == 0
    ctx = row_first + row_count
    exp_s = np.concatenate([[0], np.cumsum(np.where(row_count == 1, (ctx + split - 1) // split, 0))])
    exp_q = np.concatenate([[0], np.cumsum(np.where(row_count == 1, 0, (row_count + qt - 1) // qt))])
    assert np.array_equal(host(cu_splits), exp_s)
    assert np.array_equal(host(cu_qtiles), exp_q)


def test_pack_flags_missing_blocks():
    torch = torch_cuda()
    rng = np.random.default_rng(9)
    blocks, row_slot, row_first, row_count = pack_case(rng, rows=4)
    blocks[row_slot[2], (row_first[2] + row_count[2] - 1) // 16] = -1
    R, T, MB = 4, int(row_count.sum()), blocks.shape[1]
    outs = [torch.zeros(n, dtype=torch.int32, device="cuda") for n in (R + 1, T, T, T, R, R * MB,
                                                                       R + 1, R + 1)]
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    ins = [dev(x) for x in (row_slot, row_first, row_count, blocks)]
    check(lib().hllm_b200_pack(ptr(ins[0]), ptr(ins[1]), ptr(ins[2]), R, T,
                               ptr(ins[3]), MB, 64, 16, *[ptr(t) for t in outs], ptr(status),
                               stream()))
    sync()
    assert int(host(status)[0]) != 0


# ----------------------------------------------------------------------------- q/k/v epilogue
@pytest.mark.parametrize("hq,hkv,d,qk_norm", [(32, 8, 128, True), (4, 2, 64, False),
                                              (4, 2, 4, True), (12, 4, 256, False)])
def test_qkv_post_norm_rope_and_paged_write(hq, hkv, d, qk_norm):
    torch = torch_cuda()
    rng = np.random.default_rng(hq + d)
    T, nblocks = 37, 64
    theta = 1e6
    qkv = rng.standard_normal((T, (hq + 2 * hkv) * d)).astype(np.float32)
    positions = np.sort(rng.choice(4000, T, replace=False)).astype(np.int32)
    slots = rng.choice(nblocks * 16, T, replace=False).astype(np.int32)
    qn = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    kn = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    pw = np.array([np.float32(theta) ** (np.float32(2 * i) / np.float32(d)) for i in range(d // 2)],
                  np.float32)
    q_out = torch.zeros((T, hq * d), dtype=torch.int16, device="cuda")
    kc = torch.zeros((nblocks, hkv, 16, d), dtype=torch.int16, device="cuda")
    vc = torch.zeros_like(kc)
    ins = [dev(x) for x in (qkv, positions, slots, qn, kn, pw)]
    check(lib().hllm_b200_qkv_post(ptr(ins[0]), T, hq, hkv, d, ptr(ins[1]), ptr(ins[2]),
                                   ptr(ins[3]) if qk_norm else None,
                                   ptr(ins[4]) if qk_norm else None, 1e-6, ptr(ins[5]),
                                   ptr(q_out), ptr(kc), ptr(vc), stream()))
    sync()
    q = qkv[:, :hq * d]
    k = qkv[:, hq * d:(hq + hkv) * d]
    v = qkv[:, (hq + hkv) * d:]
    if qk_norm:
        q = oracle.normalize_heads(q, qn, 1e-6)
        k = oracle.normalize_heads(k, kn, 1e-6)
    qr = np.stack([oracle.apply_rope(q[t:t + 1], hq, d, int(positions[t]), theta)[0] for t in range(T)])
    kr = np.stack([oracle.apply_rope(k[t:t + 1], hkv, d, int(positions[t]), theta)[0] for t in range(T)])
    np.testing.assert_allclose(f16_vals(host(q_out, np.uint16)), qr, rtol=2e-3, atol=2e-3)
    K = f16_vals(host(kc, np.uint16))
    Vv = host(vc, np.uint16)
    for t in range(T):
        b, o = divmod(int(slots[t]), 16)
        np.testing.assert_allclose(K[b, :, o, :].reshape(-1), kr[t], rtol=2e-3, atol=2e-3)
        assert np.array_equal(Vv[b, :, o, :].reshape(-1), f16_bits(v[t]))
    # untouched slots stay zero
    used = set((int(s) // 16, int(s) % 16) for s in slots)
    for b in range(nblocks):
        for o in range(16):
            if (b, o) not in used:
                assert not host(kc[b, :, o, :]).any()


# ----------------------------------------------------------------------------- attention
def attention_case(rng, hq, hkv, d, rows_spec, nblocks=None):
    """rows_spec: list of (first, count).  Builds a randomly permuted paged cache
    holding every row's keys [0, first+count)."""
    ctx = [f + c for f, c in rows_spec]
    need = [(c + 15) // 16 for c in ctx]
    total = sum(need)
    nblocks = nblocks or int(total * 1.2) + 1
    perm = rng.permutation(nblocks)[:total].astype(np.int32)
    mb = max(need)
    tables = np.full((len(rows_spec), mb), -1, np.int32)
    o = 0
    for r, n in enumerate(need):
        tables[r, :n] = perm[o:o + n]
        o += n
    kc = f16_bits((rng.standard_normal((nblocks, hkv, 16, d)) / math.sqrt(d)).astype(np.float32))
    vc = f16_bits(rng.standard_normal((nblocks, hkv, 16, d)).astype(np.float32))
    T = sum(c for _, c in rows_spec)
    q = f16_bits((rng.standard_normal((T, hq * d)) / math.sqrt(d) * 4).astype(np.float32))
    return kc, vc, q, tables


def run_attention(kc, vc, q, tables, rows_spec, hq, hkv, d, split):
    torch = torch_cuda()
    R = len(rows_spec)
    row_first = np.int32([f for f, _ in rows_spec])
    row_count = np.int32([c for _, c in rows_spec])
    T = int(row_count.sum())
    ctx = row_first + row_count
    cu = np.concatenate([[0], np.cumsum(row_count)]).astype(np.int32)
    qt = int(lib().hllm_b200_attention_qtile_tokens(hq // hkv))
    sp = np.where(row_count == 1, (ctx + split - 1) // split, 0)
    qq = np.where(row_count == 1, 0, (row_count + qt - 1) // qt)
    cu_s = np.concatenate([[0], np.cumsum(sp)]).astype(np.int32)
    cu_q = np.concatenate([[0], np.cumsum(qq)]).astype(np.int32)
    out = torch.zeros((T, hq * d), dtype=torch.int16, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    keep = [dev(x) for x in (q, kc, vc, row_first, row_count, cu, ctx.astype(np.int32), tables,
                             cu_s, cu_q)]
    check(lib().hllm_b200_attention(*[ptr(t) for t in keep], R, int(cu_s[-1]), int(cu_q[-1]), hq,
                                    hkv, d, tables.shape[1], split, ptr(out), hq * d, T,
                                    kc.shape[0], ptr(status), stream()))
    sync()
    assert int(host(status)[0]) == 0
    return f16_vals(host(out, np.uint16))


def oracle_attention(kc, vc, q, tables, rows_spec, hq, hkv, d):
    K, V, Q = f16_vals(kc), f16_vals(vc), f16_vals(q)
    cfg = oracle.Config(hq * d, 1, hq, hkv, d, 1 << 20, 1e-6, 1e4, 0)
    outs = []
    t = 0
    for r, (first, count) in enumerate(rows_spec):
        ctx = first + count
        kk = np.zeros((ctx, hkv, d), np.float32)
        vv = np.zeros_like(kk)
        for p in range(ctx):
            b = tables[r, p // 16]
            kk[p] = K[b, :, p % 16, :]
            vv[p] = V[b, :, p % 16, :]
        kv = oracle.KV(ctx, hkv, d, ctx, oracle.fp(kk), oracle.fp(vv))
        qr = np.ascontiguousarray(Q[t:t + count])
        out = np.zeros((count, hq * d), np.float32)
        oracle.lib().oracle_attention(oracle.fp(qr), count, C.byref(cfg), first, C.byref(kv),
                                      oracle.fp(out))
        outs.append(out)
        t += count
    return np.concatenate(outs)


@pytest.mark.parametrize("hq,hkv,d", [(32, 8, 128), (16, 8, 128), (4, 2, 64), (12, 4, 256),
                                      (4, 2, 4)])
def test_attention_mixed_decode_and_prefill_rows(hq, hkv, d):
    rng = np.random.default_rng(hq * 3 + d)
    rows_spec = [(700, 1), (0, 37), (15, 1), (0, 1), (130, 70), (2047, 1), (64, 16), (5, 3)]
    kc, vc, q, tables = attention_case(rng, hq, hkv, d, rows_spec)
    got = run_attention(kc, vc, q, tables, rows_spec, hq, hkv, d, split=256)
    ref = oracle_attention(kc, vc, q, tables, rows_spec, hq, hkv, d)
    np.testing.assert_allclose(got, ref, rtol=5e-3, atol=3e-3)


@pytest.mark.parametrize("split", [64, 512, 4096])
def test_decode_attention_split_invariance_long_context(split):
    hq, hkv, d = 32, 8, 128
    rng = np.random.default_rng(split)
    rows_spec = [(int(c) - 1, 1) for c in np.exp(rng.uniform(np.log(128), np.log(8192), 6)).astype(int)]
    kc, vc, q, tables = attention_case(rng, hq, hkv, d, rows_spec)
    got = run_attention(kc, vc, q, tables, rows_spec, hq, hkv, d, split=split)
    ref = oracle_attention(kc, vc, q, tables, rows_spec, hq, hkv, d)
    np.testing.assert_allclose(got, ref, rtol=5e-3, atol=3e-3)


@pytest.mark.parametrize("hq,hkv", [(32, 8), (16, 8)])
def test_prefill_attention_long_chunks(hq, hkv):
    """512-token chunks at configuration 3's positions (first chunk, last chunk
    of a 4,096-token prompt) and a short chunk, one batch: many key tiles per
    query tile and key splits merged across CTAs."""
    d = 128
    rng = np.random.default_rng(hq + 7)
    rows_spec = [(0, 512), (3584, 512), (1000, 100), (777, 1)]
    kc, vc, q, tables = attention_case(rng, hq, hkv, d, rows_spec)
    got = run_attention(kc, vc, q, tables, rows_spec, hq, hkv, d, split=256)
    ref = oracle_attention(kc, vc, q, tables, rows_spec, hq, hkv, d)
    np.testing.assert_allclose(got, ref, rtol=5e-3, atol=3e-3)


def oracle_row(kpages, vpages, q_row, ctx, hq, hkv, d):
    """The oracle's attention for one decode row whose pages are given in
    order ([pages][Hkv][16][d] F16 bits)."""
    K = f16_vals(kpages).transpose(0, 2, 1, 3).reshape(-1, hkv, d)[:ctx]
    V = f16_vals(vpages).transpose(0, 2, 1, 3).reshape(-1, hkv, d)[:ctx]
    kk, vv = np.ascontiguousarray(K), np.ascontiguousarray(V)
    cfg = oracle.Config(hq * d, 1, hq, hkv, d, 1 << 20, 1e-6, 1e4, 0)
    kv = oracle.KV(ctx, hkv, d, ctx, oracle.fp(kk), oracle.fp(vv))
    qr = np.ascontiguousarray(f16_vals(q_row)[None, :])
    out = np.zeros((1, hq * d), np.float32)
    oracle.lib().oracle_attention(oracle.fp(qr), 1, C.byref(cfg), ctx - 1, C.byref(kv),
                                  oracle.fp(out))
    return out[0]


@pytest.mark.parametrize("B", [128, 256])
def test_decode_attention_configuration5_batches(B):
    """Configuration 5 at full size: B decode rows (Qwen3-4B heads), contexts
    log-uniform over [128, 32768] (one row at each end), pages randomly placed
    in a pool 1.2x the KV, Q/K/V ~ N(0,1)/sqrt(128) generated on the device.
    Every row runs; twelve rows, the longest and shortest among them, are
    checked against the oracle."""
    torch = torch_cuda()
    hq, hkv, d = 32, 8, 128
    rng = np.random.default_rng(B)
    ctx = np.exp(rng.uniform(np.log(128), np.log(32768), B)).astype(np.int64)
    ctx[0], ctx[1] = 32768, 128
    need = (ctx + 15) // 16
    nblocks = int(need.sum() * 1.2) + 1
    perm = rng.permutation(nblocks)[:need.sum()].astype(np.int32)
    mb = int(need.max())
    tables = np.full((B, mb), -1, np.int32)
    off = np.concatenate([[0], np.cumsum(need)])
    for r in range(B):
        tables[r, :need[r]] = perm[off[r]:off[r + 1]]
    gen = torch.Generator(device="cuda").manual_seed(B)
    scale = 1.0 / math.sqrt(d)
    kc = (torch.randn((nblocks, hkv, 16, d), generator=gen, device="cuda") * scale).half()
    vc = (torch.randn((nblocks, hkv, 16, d), generator=gen, device="cuda") * scale).half()
    q = (torch.randn((B, hq * d), generator=gen, device="cuda") * scale).half()
    row_first = (ctx - 1).astype(np.int32)
    row_count = np.ones(B, np.int32)
    cu = np.arange(B + 1, dtype=np.int32)
    split = 512
    sp = (ctx + split - 1) // split
    cu_s = np.concatenate([[0], np.cumsum(sp)]).astype(np.int32)
    cu_q = np.zeros(B + 1, np.int32)
    out = torch.zeros((B, hq * d), dtype=torch.int16, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    keep = [dev(x) for x in (row_first, row_count, cu, ctx.astype(np.int32), tables, cu_s, cu_q)]
    check(lib().hllm_b200_attention(ptr(q), ptr(kc), ptr(vc), *[ptr(t) for t in keep], B,
                                    int(cu_s[-1]), 0, hq, hkv, d, mb, split, ptr(out), hq * d, B,
                                    nblocks, ptr(status), stream()))
    sync()
    assert int(host(status)[0]) == 0
    got = f16_vals(host(out, np.uint16))
    assert np.isfinite(got).all()
    kcv, vcv, qv = kc.view(torch.int16), vc.view(torch.int16), q.view(torch.int16)
    for r in [0, 1] + list(rng.choice(np.arange(2, B), 10, replace=False)):
        pages = torch.from_numpy(tables[r, :need[r]].astype(np.int64)).cuda()
        ref = oracle_row(host(kcv[pages], np.uint16), host(vcv[pages], np.uint16),
                         host(qv[r], np.uint16), int(ctx[r]), hq, hkv, d)
        np.testing.assert_allclose(got[r], ref, rtol=5e-3, atol=3e-3, err_msg=f"row {r}")


# ----------------------------------------------------------------------------- sampler
def run_sample(logits_rows, opts, gidx):
    torch = torch_cuda()
    L = np.ascontiguousarray(np.atleast_2d(logits_rows), np.float32)
    rows, V = L.shape
    o = (_lib.Sampling * rows)(*[_lib.Sampling(*x) for x in opts])
    g = (C.c_uint64 * rows)(*gidx)
    out = (_lib.Sampled * rows)()
    d = dev(L)
    st = lib().hllm_b200_sample(ptr(d), rows, V, V, o, g, out, stream())
    return st, out


def test_sampler_matches_reference_known_answers():
    g = np.load(os.path.join(GOLD, "sampling_kat.npz"))
    for i in range(len(g["n"])):
        n = int(g["n"][i])
        o = g["options"][i]
        opts = [(o[0], o[1], int(o[2]), int(o[3]), int(o[4]), int(o[5]))]
        st, out = run_sample(g["logits"][i][:n], opts, [int(g["generated_index"][i])])
        check(st)
        assert out[0].token_id == g["token"][i], (i, n, tuple(o))
        if o[4]:
            assert abs(out[0].logprob - g["logprob"][i]) < 1e-9
            assert out[0].n_top == g["n_top"][i]
            for k in range(out[0].n_top):
                assert out[0].top_ids[k] == g["top_ids"][i][k]
                assert abs(out[0].top_logprobs[k] - g["top_logprobs"][i][k]) < 1e-9


def test_sampler_full_vocab_against_oracle_and_greedy_ties():
    rng = np.random.default_rng(21)
    V = 151936
    rows = rng.standard_normal((6, V)).astype(np.float32)
    rows[1, [5, 77, 1000]] = 50.0  # tie for the maximum: the lowest id wins
    opts = [(0.0, 1.0, 0, 1, 0, 0), (0.0, 1.0, 0, 1, 1, 5), (0.7, 0.9, 0, 123, 0, 0),
            (0.7, 0.9, 0, 124, 1, 3), (1.0, 1.0, 40, 9, 0, 0), (0.3, 0.5, 0, 77, 0, 0)]
    gidx = [0, 1, 2, 3, 4, 5]
    st, out = run_sample(rows, opts, gidx)
    check(st)
    assert out[1].token_id == 5
    for i in range(6):
        s, ref = oracle.sample_token(rows[i], oracle.sampling(*opts[i][:4], bool(opts[i][4]),
                                                              opts[i][5]), gidx[i])
        assert s == 0
        assert out[i].token_id == ref.token_id, i
        if opts[i][4]:
            assert abs(out[i].logprob - ref.logprob) < 1e-6
            for k in range(ref.n_top):
                assert out[i].top_ids[k] == ref.top_ids[k]


def test_sampler_refuses_nonfinite_logits():
    lg = np.zeros((1, 100), np.float32)
    lg[0, 40] = np.nan
    st, _ = run_sample(lg, [(0.0, 1.0, 0, 0, 0, 0)], [0])
    assert st == _lib.INTERNAL
    lg[0, 40] = np.inf
    st, _ = run_sample(lg, [(0.8, 1.0, 0, 0, 0, 0)], [0])
    assert st == _lib.INTERNAL
