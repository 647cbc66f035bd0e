"""Host arithmetic of the decode timeline (shardlm_b200.microbench.timeline_summary) on synthetic
stamps laid out as shd_model_timeline returns them: per launch 8 u64, fields 0/2/4 first entry /
first wait return / first exit as %globaltimer nanoseconds, fields 1/3/5 last entry / last end of
prologue / last exit stored complemented. No GPU needed."""
import numpy as np
import pytest


def _launch(e0, e1, w0, r1, x0, x1):
    c = lambda v: np.uint64(~np.uint64(v) & np.uint64(0xFFFFFFFFFFFFFFFF))
    return [np.uint64(e0), c(e1), np.uint64(w0), c(r1), np.uint64(x0), c(x1), np.uint64(0), np.uint64(0)]


def test_costs_sum_to_the_step_and_fields_decode():
    from shardlm_b200.microbench import timeline_summary

    # qkv, attention, gate/up, exchange, lm_head; times in ns from an arbitrary origin
    kinds = np.array([0, 5, 2, 6, 4], np.int32)
    st = np.array([
        _launch(1_000, 1_200, 3_000, 5_000, 9_000, 10_000),
        _launch(10_100, 10_300, 11_000, 11_000, 15_000, 18_000),    # starts after qkv ended
        _launch(12_000, 20_000, 19_000, 24_000, 60_000, 62_000),    # resident 6 us before attention ended
        _launch(55_000, 55_100, 62_800, 63_500, 64_000, 64_500),
        _launch(63_000, 63_500, 65_000, 68_000, 200_000, 210_000),
    ], dtype=np.uint64)
    s = timeline_summary(kinds, st)
    assert s["attention"] == {"n": 1, "cost": 8.0, "lead": -0.1, "dep": 1.0, "prologue": 0.0, "body": 7.0,
                              "exit_spread": 3.0, "entry_spread": 0.2}
    assert s["gateup"]["cost"] == 44.0 and s["gateup"]["lead"] == 6.0 and s["gateup"]["dep"] == 1.0
    assert s["gateup"]["prologue"] == 5.0 and s["gateup"]["body"] == 38.0
    assert s["exchange"]["cost"] == 2.5 and s["exchange"]["dep"] == 0.8
    assert s["lm_head"]["cost"] == 145.5
    assert "qkv" not in s  # the first launch has no predecessor to measure against
    total = sum(s[k]["cost"] for k in ("attention", "gateup", "exchange", "lm_head"))
    assert total == pytest.approx((210_000 - 10_000) / 1e3)
    assert s["traced_span_us"] == 209.0


def test_unstamped_launch_is_rejected():
    from shardlm_b200.microbench import timeline_summary

    kinds = np.array([0, 1], np.int32)
    st = np.array([_launch(0, 1, 2, 3, 4, 5), [np.uint64(0xFFFFFFFFFFFFFFFF)] * 8], dtype=np.uint64)
    with pytest.raises(AssertionError, match="not stamped"):
        timeline_summary(kinds, st)
