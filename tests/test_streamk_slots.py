"""Host restatement of the stream-K slot arithmetic (hllm_b200/csrc/gemm.cuh:
gemm_unit_begin, gemm_tile_ctas, gemm_first_slot; the GEMM kernel's slot_id).

CTA c of G owns units [U c / G, U (c + 1) / G) of U = tiles * kb units and
writes the partial sums of the j-th tile it touches to slot 3 c + j.  A
consumer finds a tile's CTAs as c0 = ((u0 + 1) G - 1) / U .. c1 = ((u0 + kb) G
- 1) / U with u0 = tile * kb, reads c0's slot through its first tile, and
slot 3 c for every later CTA (which starts inside the tile).  The checks
compare that with a direct walk of every CTA's units, for plans the planner
can make (tiles < 2 G, G <= 14 tiles, U (G + 1) < 2^31).
"""
import numpy as np

SLOTS_PER_CTA = 3


def walk(tiles, kb, G):
    """tile -> [(cta, slot)] by walking each CTA's unit range, as the GEMM does."""
    U = tiles * kb
    owners = {t: [] for t in range(tiles)}
    for c in range(G):
        ub, ue = U * c // G, U * (c + 1) // G
        if ub >= ue:
            continue
        first_tile = ub // kb
        u = ub
        while u < ue:
            t = u // kb
            end = min((t + 1) * kb, ue)
            slot = c * SLOTS_PER_CTA + (t - first_tile)
            assert t - first_tile < SLOTS_PER_CTA, (tiles, kb, G, c)
            owners[t].append((c, slot))
            u = end
    return owners


def formulas(tiles, kb, G, tile):
    U = tiles * kb
    u0 = tile * kb
    c0 = ((u0 + 1) * G - 1) // U
    c1 = ((u0 + kb) * G - 1) // U
    begin = U * c0 // G
    first = c0 * SLOTS_PER_CTA + (tile - begin // kb)
    return [(c0, first)] + [(c, c * SLOTS_PER_CTA) for c in range(c0 + 1, c1 + 1)]


def test_consumer_slots_match_the_gemm_walk():
    rng = np.random.default_rng(5)
    cases = 0
    while cases < 400:
        tiles = int(rng.integers(1, 513))
        kb = int(rng.integers(1, 200))
        G = int(rng.integers(1, 300))
        U = tiles * kb
        G = max(1, min(G, U))
        if not (tiles < 2 * G and G <= tiles * 14 and U * (G + 1) < 2 ** 31):
            continue
        cases += 1
        owners = walk(tiles, kb, G)
        for t in range(tiles):
            assert formulas(tiles, kb, G, t) == owners[t], (tiles, kb, G, t)
            assert len(owners[t]) <= 16  # the consumers' per-tile bound


def test_decode_shapes():
    # Qwen3-4B projections at 64 tokens (BN 64: one token tile) on 148 CTAs
    for m, k in ((6144, 2560), (2560, 4096), (9728, 2560), (2560, 9728)):
        tiles, kb = (m + 127) // 128, k // 64
        G = min(148, max(1, tiles * kb // 4))
        owners = walk(tiles, kb, G)
        for t in range(tiles):
            assert formulas(tiles, kb, G, t) == owners[t]
