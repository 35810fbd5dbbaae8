"""Device-trace summaries (CPU): utils.trace_bench.summarise on a synthetic Chrome trace."""
from originccl_b200.utils.trace_bench import summarise


def _ev(name, rnd, cta, ts, kernel=7):
    return {"name": f"{name} r{rnd}", "ph": "i", "s": "t", "ts": ts, "pid": 0, "tid": cta * 4,
            "args": {"kernel": kernel, "group": 0, "round": rnd}}


def test_summary_per_iteration_median_and_max():
    evs = []
    for cta, skew in ((0, 0.0), (1, 2.0), (2, 4.0)):
        evs.append(_ev("begin", 0, cta, 100.0 + skew))
        evs.append(_ev("staged", 0, cta, 110.0 + skew))
        evs.append(_ev("barrier", 0, cta, 118.0 + skew))
        evs.append(_ev("staged", 1, cta, 130.0 + skew))
        evs.append(_ev("barrier", 1, cta, 140.0 + skew))
        evs.append(_ev("end", 2, cta, 141.0 + skew))
    evs.append(_ev("begin", 0, 0, 500.0, kernel=8))  # a launch without an end is skipped
    (rec,) = summarise({"traceEvents": evs})
    assert rec["kernel"] == 7 and rec["ctas"] == 3
    assert rec["span_us"] == 45.0 and rec["begin_spread_us"] == 4.0
    it0, it1 = rec["iters"]
    assert it0 == {"iter": 0, "staged_med": 12.0, "staged_max": 14.0, "barrier_med": 20.0, "barrier_max": 22.0}
    assert it1["barrier_max"] == 44.0
