"""bench.py's per-phase roofline arithmetic (decode-only steps against HBM,
steps carrying a prefill chunk against the tensor roof), on the CPU, against
the Qwen3-4B figures: 201.85 MB of F16 weights per layer, a 777.9 MB head,
147,456 bytes of K/V per token over 36 layers, 7.267 GFLOP per token."""
import pytest

import bench


def test_step_work_matches_the_configuration_3_formulas():
    layer, head = bench.qwen_stage_bytes()
    assert layer == pytest.approx(201.85e6, rel=1e-3) and head == pytest.approx(777.9e6, rel=1e-3)
    dec = [(999, 1, True)] * 64  # 64 decode rows with 1,000 keys each
    nbytes, flops = bench.step_work(dec)
    ctx = 64 * 1000
    expect = 36 * layer + head + 147456 * ctx + 64 * 147456 + 64 * 2560 * 4
    assert nbytes == pytest.approx(expect, rel=1e-9)
    expect_flops = 64 * 7.267e9 + 4 * 32 * 128 * 36 * ctx + 64 * 2 * 151936 * 2560
    assert flops == pytest.approx(expect_flops, rel=2e-3)
    # a 512-token chunk at position 0: 512 * 513 / 2 causal pairs
    _, f = bench.step_work([(0, 512, True)])
    assert f == pytest.approx(512 * 7.267e9 + 4 * 32 * 128 * 36 * (512 * 513 // 2)
                              + 2 * 151936 * 2560, rel=2e-3)


def test_phase_summary_splits_decode_and_prefill_steps():
    dec = [(999, 1, True)] * 64
    pre = [(999, 1, True)] * 63 + [(0, 512, True)]
    out = bench.phase_summary([(dec, True), (pre, False), (dec, True)], [5.0, 10.0, 6.0],
                              6650.0, 1400.0)
    assert out["decode"]["steps"] == 2 and out["prefill"]["steps"] == 1
    assert out["decode"]["ms_per_step"] == 5.5 and out["decode"]["bound"] == "hbm"
    b = bench.step_work(dec)[0]
    assert out["decode"]["achieved"] == pytest.approx(2 * b / 11e-3 / 1e9, rel=1e-3)
    assert out["prefill"]["bound"] == "tensor"
    assert out["prefill"]["tokens_per_s"] == pytest.approx(575 / 10e-3, rel=1e-3)
    assert bench.phase_summary([(dec, True)], [5.0], 6650.0, 1400.0).keys() == {"decode"}
