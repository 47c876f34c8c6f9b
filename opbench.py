"""Per-operator timing of the executor's kernels through the C ABI.

    python opbench.py [gemm|attn|prefill|envelope|c5|all] [--ncu-gemm M,K,N,PAIR,EPI]
                      [--ncu-attn ROWS] [--ncu-prefill FIRST,COUNT]

Times the projection GEMM at the Qwen3-4B shapes (decode width 16/64 tokens,
prefill width 575 tokens) and the paged decode attention at configuration-5
batch sizes (contexts log-uniform in [128, 32768], 16-token pages randomly
placed in a pool), with CUDA events on the current stream after warm-up.
Inputs are far larger than L2 for the weight-streaming shapes.  `--ncu-gemm`
runs three launches of one GEMM shape and `--ncu-attn` three of the decode
attention over ROWS configuration-3-like contexts (for profiler captures).
`c5` runs configuration 5 (decode attention and GEMVs at batch 1-256, each
launch after an L2 flush) as a markdown table of HBM GB/s against the roof.
`envelope` times the boundary wire codec (host encode/decode, and the
envelope built from device memory when a GPU is present).
Device memory comes from torch; all compute is libhllm_b200.so.
"""
from __future__ import annotations

import math
import sys

import numpy as np


def _torch():
    import torch
    if not torch.cuda.is_available():
        raise SystemExit("opbench needs a CUDA device")
    return torch


_FLUSH = None


def ev_time(fn, iters=20, warm=3, cold=False):
    """Microseconds per call, with CUDA events on the current stream after
    `warm` untimed calls.  cold=True writes a 512 MB buffer (4x L2) before
    every call, outside the timed region, and times each call alone, so that
    inputs smaller than L2 are read from HBM."""
    global _FLUSH
    torch = _torch()
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    if cold:
        if _FLUSH is None:
            _FLUSH = torch.empty(512 << 20, dtype=torch.uint8, device="cuda")
        total = 0.0
        for _ in range(iters):
            _FLUSH.fill_(1)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            total += a.elapsed_time(b)
        return total / iters * 1e3
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters * 1e3  # microseconds per call


def hbm_peak():
    """(GB/s, source) of the HBM roof: MEASURED_PEAKS.json when present."""
    import json
    import os
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            v = json.load(f).get("hbm_gbs")
        if v:
            return float(v), "measured"
    except (OSError, ValueError):
        pass
    return 6650.0, "fallback"


def gemm_case(m, k, n, pair=1, epi=0, bn=0, grid=0, iters=20, cold=False):
    torch = _torch()
    from hllm_b200 import _lib
    L = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    rows = m * pair
    W = (torch.randn(rows, k, device="cuda") * 0.02).half()
    X = torch.randn(max(n, 1), k, device="cuda").half()
    outdt = torch.float32 if epi in (0, 2) else torch.float16
    Y = torch.zeros(n, m, device="cuda", dtype=outdt)

    def fn():
        _lib.check(L.hllm_b200_gemm(W.data_ptr(), m, k, pair, m if pair == 2 else 0, X.data_ptr(),
                                    n, epi, Y.data_ptr(), m, bn, grid, stream))
    us = ev_time(fn, iters, cold=cold)
    nbytes = rows * k * 2 + n * k * 2 + n * m * (4 if outdt == torch.float32 else 2)
    flops = 2 * rows * n * k
    print(f"gemm m={m} pair={pair} k={k} n={n} epi={epi}: {us:8.1f} us  "
          f"{nbytes / us / 1e3:8.1f} GB/s  {flops / us / 1e6:8.1f} TFLOP/s", flush=True)
    gemm_case.last = (us, nbytes, flops)
    return us


def attn_case(rows_ctx, hq=32, hkv=8, d=128, split=256, iters=10, cold=False):
    """Decode attention over rows with the given contexts (one new token each)."""
    torch = _torch()
    from hllm_b200 import _lib
    L = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    R = len(rows_ctx)
    need = [(c + 15) // 16 for c in rows_ctx]
    nblocks = int(sum(need) * 1.2) + 8
    perm = np.random.default_rng(0).permutation(nblocks).astype(np.int32)
    mb = max(need)
    tables = np.full((R, mb), -1, np.int32)
    o = 0
    for r, nb in enumerate(need):
        tables[r, :nb] = perm[o:o + nb]
        o += nb
    kc = (torch.randn(nblocks, hkv, 16, d, device="cuda") / math.sqrt(d)).half()
    vc = (torch.randn(nblocks, hkv, 16, d, device="cuda") / math.sqrt(d)).half()
    q = (torch.randn(R, hq * d, device="cuda") / math.sqrt(d)).half()
    ctx = np.asarray(rows_ctx, np.int32)
    first = ctx - 1
    count = np.ones(R, np.int32)
    cu = np.arange(R + 1, dtype=np.int32)
    sp = (ctx + split - 1) // split
    cu_s = np.concatenate([[0], np.cumsum(sp)]).astype(np.int32)
    cu_q = np.zeros(R + 1, np.int32)
    dv = [torch.from_numpy(x).cuda() for x in (first, count, cu, ctx, tables, cu_s, cu_q)]
    out = torch.zeros(R, hq * d, device="cuda").half()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")

    def fn():
        _lib.check(L.hllm_b200_attention(q.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                         *[t.data_ptr() for t in dv], R, int(cu_s[-1]), 0, hq,
                                         hkv, d, mb, split, out.data_ptr(), hq * d, R, nblocks,
                                         status.data_ptr(), stream))
    us = ev_time(fn, iters, cold=cold)
    nbytes = sum(rows_ctx) * hkv * d * 2 * 2 + R * hq * d * 4
    print(f"decode attention B={R} sum_ctx={sum(rows_ctx)} split={split}: {us:8.1f} us  "
          f"{nbytes / us / 1e3:8.1f} GB/s", flush=True)
    attn_case.last = (us, nbytes)
    return us


def prefill_case(first, count, rows=1, hq=32, hkv=8, d=128, iters=10):
    """Prefill attention of `rows` chunks of `count` tokens at positions
    [first, first + count) (causal over first + count keys each)."""
    torch = _torch()
    from hllm_b200 import _lib
    L = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    ctx = first + count
    need = (ctx + 15) // 16
    nblocks = int(need * rows * 1.2) + 8
    perm = np.random.default_rng(1).permutation(nblocks).astype(np.int32)
    tables = perm[:need * rows].reshape(rows, need).copy()
    kc = (torch.randn(nblocks, hkv, 16, d, device="cuda") / math.sqrt(d)).half()
    vc = torch.randn(nblocks, hkv, 16, d, device="cuda").half()
    T = rows * count
    q = torch.randn(T, hq * d, device="cuda").half()
    qt = int(L.hllm_b200_attention_qtile_tokens(hq // hkv))
    tiles = (count + qt - 1) // qt
    first_a = np.full(rows, first, np.int32)
    count_a = np.full(rows, count, np.int32)
    cu = (np.arange(rows + 1) * count).astype(np.int32)
    lens = np.full(rows, ctx, np.int32)
    cu_s = np.zeros(rows + 1, np.int32)
    cu_q = (np.arange(rows + 1) * tiles).astype(np.int32)
    dv = [torch.from_numpy(x).cuda() for x in (first_a, count_a, cu, lens, tables, cu_s, cu_q)]
    out = torch.zeros(T, hq * d, device="cuda").half()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")

    def fn():
        _lib.check(L.hllm_b200_attention(q.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                         *[t.data_ptr() for t in dv], rows, 0, rows * tiles, hq,
                                         hkv, d, need, 16, out.data_ptr(), hq * d, T, nblocks,
                                         status.data_ptr(), stream))
    us = ev_time(fn, iters)
    pairs = rows * (count * first + count * (count + 1) / 2)
    flops = 4.0 * hq * d * pairs
    print(f"prefill attention rows={rows} first={first} count={count}: {us:8.1f} us  "
          f"{flops / us / 1e6:8.1f} TFLOP/s", flush=True)
    return us


def stage_split(rows_ctx, hkv=8, sm=148):
    """The decode split size the stage picks (stage.cu plan_step): about 16
    (row, kv head, split) items per SM, at least 64 keys, a multiple of 16."""
    keys = sum(c for c in rows_ctx)
    target = max(1, (16 * sm) // hkv)
    return max(64, -(-(-(-keys // target)) // 16) * 16)


def c5_sweep():
    """Configuration 5: the isolated decode-attention and GEMV sweep at Qwen3-4B
    layer shapes, each launch timed alone after an L2 flush, as achieved HBM
    GB/s against the roof.  Contexts log-uniform in [128, 32768] (seeded), 16-token
    pages randomly placed in a pool 1.2x the KV."""
    peak, src = hbm_peak()
    print(f"| kernel | shape | B | µs | GB/s | of {src} {peak:.0f} GB/s |")
    print("| --- | --- | --- | --- | --- | --- |")
    rng = np.random.default_rng(5)
    for B in (1, 8, 32, 128, 256):
        ctx = np.exp(rng.uniform(np.log(128), np.log(32768), B)).astype(int).tolist()
        attn_case(ctx, split=stage_split(ctx), cold=True)
        us, nbytes = attn_case.last
        gbs = nbytes / us / 1e3
        print(f"| decode attention | Σctx {sum(ctx)} | {B} | {us:.1f} | {gbs:.0f} | "
              f"{gbs / peak:.1%} |", flush=True)
    shapes = [("QKV", 6144, 2560, 1, 0), ("O", 2560, 4096, 1, 2), ("gate/up", 9728, 2560, 2, 3),
              ("down", 2560, 9728, 1, 2), ("LM head", 151936, 2560, 1, 0)]
    for B in (1, 8, 32, 128, 256):
        for name, m, k, pair, epi in shapes:
            gemm_case(m, k, B, pair, epi, cold=True)
            us, nbytes, _ = gemm_case.last
            gbs = nbytes / us / 1e3
            print(f"| GEMV {name} | {m * pair}x{k} | {B} | {us:.1f} | {gbs:.0f} | "
                  f"{gbs / peak:.1%} |", flush=True)


def gemm_suite():
    # (m, k, n, pair, epilogue): Qwen3-4B QKV, gate/up, down, o, LM head
    for args in [(6144, 2560, 64, 1, 0), (9728, 2560, 64, 2, 3), (2560, 9728, 64, 1, 2),
                 (2560, 4096, 64, 1, 2), (151936, 2560, 64, 1, 0), (6144, 2560, 16, 1, 0),
                 (6144, 2560, 575, 1, 0), (9728, 2560, 575, 2, 3), (2560, 9728, 575, 1, 2),
                 (2560, 4096, 575, 1, 2)]:
        gemm_case(*args)


def prefill_suite():
    for first, count in ((0, 512), (512, 512), (2048, 512), (3584, 512), (1000, 100)):
        prefill_case(first, count)


def attn_suite():
    rng = np.random.default_rng(5)
    for B in (1, 8, 32, 128, 256):
        ctx = np.exp(rng.uniform(np.log(128), np.log(32768), B)).astype(int).tolist()
        for split in (128, 512, 2048):
            attn_case(ctx, split=split)


def steady_decode_contexts(rows=64, seed=3):
    """Decode contexts like configuration 3's steady state: prompt
    log-normal(median 512, sigma 1) in [32, 4096] plus U[1, 512] generated."""
    rng = np.random.default_rng(seed)
    prompt = np.clip(np.exp(rng.normal(math.log(512), 1.0, rows)), 32, 4096)
    return (prompt + rng.integers(1, 513, rows)).astype(int).tolist()


def envelope_suite(tokens=512, width=2560, iters=200):
    """The boundary wire codec at a 512-token Qwen3-4B chunk (2.6 MB of F16):
    host encode and decode through the C ABI (no GPU needed), then, on a GPU,
    the envelope built from a non-final stage's device boundary
    (hllm_b200_stage_envelope + _wait) into pinned memory."""
    import ctypes as C
    import time
    from hllm_b200 import _lib
    L = _lib.lib()
    ident = _lib.BoundaryIdentity(b"qwen3-4b-plan", 3, b"request-000001", 4608, width)
    x = (np.random.default_rng(0).standard_normal(tokens * width)).astype("<f2")
    n = C.c_uint64()
    args = (C.byref(ident), 0, 0, 1, x.ctypes.data, x.nbytes, tokens, width)
    _lib.check(L.hllm_b200_envelope_encode(*args, None, 0, C.byref(n)))
    out = np.empty(n.value, np.uint8)
    t0 = time.perf_counter()
    for _ in range(iters):
        _lib.check(L.hllm_b200_envelope_encode(*args, out.ctypes.data, n.value, C.byref(n)))
    enc = (time.perf_counter() - t0) / iters
    off, tok = C.c_uint64(), C.c_uint64()
    t0 = time.perf_counter()
    for _ in range(iters):
        _lib.check(L.hllm_b200_envelope_decode(out.ctypes.data, n.value, C.byref(ident), 0, 0, 1,
                                               C.byref(off), C.byref(tok)))
    dec = (time.perf_counter() - t0) / iters
    print(f"envelope host  {tokens}x{width}: encode {enc * 1e6:8.1f} us "
          f"({x.nbytes / enc / 1e9:6.1f} GB/s), decode {dec * 1e6:8.1f} us "
          f"({x.nbytes / dec / 1e9:6.1f} GB/s), message {n.value} bytes", flush=True)
    try:
        import torch
        if not torch.cuda.is_available():
            return
    except ImportError:
        return
    from hllm_b200.backend import B200Stage, DecodeBatchItem, ModelConfig, TokenInput
    cfg = ModelConfig(width, 9728, 32, 8, 128, 4608, 1e-6, 1e6, True, 151936, 36, True)
    stage = B200Stage(cfg, 0, 1, first=True, final=False, kv_pool_tokens=8192,
                      max_step_tokens=tokens + 64, max_step_rows=80, max_sequences=80)
    stage.init_synthetic(1)
    ids = [int(v) for v in np.random.default_rng(2).integers(0, 151936, tokens)]
    seq = stage.allocate_sequence(tokens + 8)
    stage.execute_mixed_batch([DecodeBatchItem(TokenInput(ids), 0, seq)])
    pinned = torch.empty(n.value, dtype=torch.uint8, pin_memory=True)
    dev_args = (stage.handle, 0, tokens, C.byref(ident), 0, 0, 1)
    for _ in range(3):
        _lib.check(L.hllm_b200_stage_envelope(*dev_args, pinned.data_ptr(), n.value, C.byref(n)))
        _lib.check(L.hllm_b200_stage_envelope_wait(stage.handle))
    t0 = time.perf_counter()
    for _ in range(iters):
        _lib.check(L.hllm_b200_stage_envelope(*dev_args, pinned.data_ptr(), n.value, C.byref(n)))
        _lib.check(L.hllm_b200_stage_envelope_wait(stage.handle))
    devt = (time.perf_counter() - t0) / iters
    assert bytes(pinned[:16].numpy()) == bytes(out[:16])  # same frame as the host encoding
    print(f"envelope device {tokens}x{width}: stage_envelope+wait {devt * 1e6:8.1f} us "
          f"({x.nbytes / devt / 1e9:6.1f} GB/s device->host into the message)", flush=True)
    stage.release(seq)
    stage.close()


def main(argv):
    if "--ncu-prefill" in argv:
        first, count = (int(x) for x in argv[argv.index("--ncu-prefill") + 1].split(","))
        prefill_case(first, count, iters=3)
        return
    if "--ncu-attn" in argv:
        rows = int(argv[argv.index("--ncu-attn") + 1])
        attn_case(steady_decode_contexts(rows), iters=3)
        return
    if "--ncu-gemm" in argv:
        m, k, n, pair, epi = (int(x) for x in argv[argv.index("--ncu-gemm") + 1].split(","))
        gemm_case(m, k, n, pair, epi, iters=3)
        return
    what = argv[1] if len(argv) > 1 else "all"
    if what in ("gemm", "all"):
        gemm_suite()
    if what in ("attn", "all"):
        attn_suite()
    if what in ("prefill", "all"):
        prefill_suite()
    if what in ("envelope", "all"):
        envelope_suite()
    if what == "c5":
        c5_sweep()


if __name__ == "__main__":
    main(sys.argv)
