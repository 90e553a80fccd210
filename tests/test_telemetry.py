"""Per-step telemetry: the snapshot arithmetic against the reference's
known answers (tests/test_telemetry.cpp:38-65, nearest-rank percentiles of
compute_stats, src/core/telemetry.hpp:88-113), and on a GPU the step
latencies recorded by the layer itself."""
import numpy as np
import pytest


def test_nearest_rank_known_answer():
    from aethermoe_b200 import _lib
    s = _lib.metric_stats_of(np.arange(1, 101, dtype=np.uint64) * 1000)
    assert s["count"] == 100
    assert (s["p50_ns"], s["p95_ns"], s["p99_ns"]) == (50000.0, 95000.0, 99000.0)
    assert s["max_ns"] == 100000.0 and s["mean_ns"] == 50500.0


def test_empty_and_single_sample():
    from aethermoe_b200 import _lib
    e = _lib.metric_stats_of(np.zeros(0, np.uint64))
    assert e["count"] == 0 and e["p50_ns"] == 0.0 and e["max_ns"] == 0.0
    one = _lib.metric_stats_of([7])
    assert one["p50_ns"] == one["p99_ns"] == one["max_ns"] == one["mean_ns"] == 7.0


def test_unsorted_input_matches_restatement():
    from aethermoe_b200 import _lib
    rng = np.random.default_rng(3)
    for n in (2, 3, 19, 20, 21, 1000):
        v = rng.integers(1, 10 ** 9, size=n, dtype=np.uint64)
        s = _lib.metric_stats_of(v)
        srt = np.sort(v)
        pct = lambda p: float(srt[min(max(int(np.ceil(p * n)), 1), n) - 1])
        assert s["p50_ns"] == pct(0.50) and s["p95_ns"] == pct(0.95)
        assert s["p99_ns"] == pct(0.99) and s["max_ns"] == float(srt[-1])
        assert abs(s["mean_ns"] - float(v.astype(np.float64).mean())) <= 1e-9 * s["mean_ns"]


def test_disabled_records_nothing():
    from aethermoe_b200 import _lib
    _lib.telemetry_enable(False)
    _lib.telemetry_reset()
    assert _lib.telemetry_snapshot(_lib.METRIC_MOE_STEP)[0]["count"] == 0
    assert not _lib.lib().aem_telemetry_enabled()


@pytest.mark.gpu
def test_layer_steps_are_recorded(cuda):
    import torch
    import aem_oracle as O
    from aethermoe_b200 import _lib
    from aethermoe_b200.moe import MoELayer
    rng = np.random.default_rng(5)
    d, f, e, k, t = 256, 384, 8, 2, 512
    qu = rng.integers(-127, 128, size=(e, d, f), dtype=np.int8)
    qd = rng.integers(-127, 128, size=(e, f, d), dtype=np.int8)
    su = np.full((e, 1, f), 2e-4, np.float32)
    sd = np.full((e, 1, d), 2e-4, np.float32)
    gw = (rng.normal(size=(d, e)) / np.sqrt(d)).astype(np.float32)
    layer = MoELayer(gw, O.zipf_bias(e), qu, su, qd, sd, k)
    x = torch.randn(t, d, device="cuda").to(torch.bfloat16)
    _lib.telemetry_reset()
    _lib.telemetry_enable(True)
    try:
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        ev[0].record()
        for _ in range(10):
            layer.forward(x)
        ev[1].record()
        torch.cuda.synchronize()
        stats, dropped = _lib.telemetry_snapshot(_lib.METRIC_MOE_STEP)
    finally:
        _lib.telemetry_enable(False)
    assert stats["count"] == 10 and dropped == 0
    total_ns = ev[0].elapsed_time(ev[1]) * 1e6
    assert 0 < stats["p50_ns"] <= stats["p99_ns"] <= stats["max_ns"]
    assert stats["mean_ns"] * 10 <= total_ns * 1.05  # steps fit inside the bracket
    assert _lib.telemetry_snapshot(_lib.METRIC_EP_STEP)[0]["count"] == 0
    layer.close()
