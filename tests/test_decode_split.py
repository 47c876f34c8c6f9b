"""Host restatement of the balanced decode split's index arithmetic
(hllm_b200/csrc/attention.cu, decode_attn_mma_kernel and decode_merge_kernel).

The decode rows' pages form one sequence ordered (row, kv head, page); warp w
of W takes pages [P w / W, P (w + 1) / W).  A (row, kv head) stream of n pages
starting at f0 is covered by warps w0 = ((f0 + 1) W - 1) / P through
w1 = ((f0 + n) W - 1) / P; the warp holding its first page writes the record
w0 | w1 << 16, and each covering warp stores its piece at index stream + w.
These checks run the formulas over random batches: the covering warps are
exactly the ones whose ranges meet the stream, the record writer is w0, piece
indices never collide and stay inside the buffer the stage sizes for them
(R * Hkv + 4 * CTAs pieces).
"""
import numpy as np


def split(ctx, count, hkv, ctas):
    pages = [((c + 15) // 16 if n == 1 else 0) for c, n in zip(ctx, count)]
    total = sum(pages) * hkv
    W = min(ctas * 4, total)
    return pages, total, W


def warp_of(p, total, W):
    # the w with total*w//W <= p < total*(w+1)//W
    w = (p * W) // total
    while total * (w + 1) // W <= p:
        w += 1
    while total * w // W > p:
        w -= 1
    return w


def check_batch(ctx, count, hkv, ctas):
    pages, total, W = split(ctx, count, hkv, ctas)
    if total == 0:
        return
    assert W <= total and W >= 1
    seen_pieces = set()
    cum = 0
    for r, n in enumerate(pages):
        for kvh in range(hkv):
            if n == 0:
                continue
            f0 = cum * hkv + kvh * n
            w0 = ((f0 + 1) * W - 1) // total
            w1 = ((f0 + n) * W - 1) // total
            covering = sorted({warp_of(p, total, W) for p in range(f0, f0 + n)})
            assert covering == list(range(w0, w1 + 1)), (r, kvh)
            assert warp_of(f0, total, W) == w0          # the record writer
            assert w0 < (1 << 16) and w1 < (1 << 16)    # the record's packing
            stream = r * hkv + kvh
            for w in range(w0, w1 + 1):
                piece = stream + w
                assert piece not in seen_pieces
                seen_pieces.add(piece)
                assert piece < len(ctx) * hkv + 4 * ctas
        cum += n


def test_balanced_split_covers_and_indexes_every_stream():
    rng = np.random.default_rng(11)
    for trial in range(300):
        R = int(rng.integers(1, 96))
        ctx = rng.integers(1, 4500, R).tolist()
        count = [1 if rng.random() < 0.85 else int(rng.integers(2, 600)) for _ in range(R)]
        hkv = int(rng.choice([1, 2, 4, 8]))
        ctas = int(rng.integers(1, 297))
        check_batch(ctx, count, hkv, ctas)


def test_edge_batches():
    check_batch([1], [1], 8, 296)            # one page, many warps
    check_batch([16, 17, 4096], [1, 1, 1], 8, 1)  # one CTA
    check_batch([32768] * 4, [1] * 4, 8, 296)     # long rows
    check_batch([5, 100], [7, 1], 4, 2)      # a prefill row contributes no pages
