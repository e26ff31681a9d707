"""The autotuner's benchmark procedure and selection policy against the
reference's recorded fixture (runtime/autotuning-policy.json), with a fake
clock device exactly like inference/tests/autotuning.rs:16-80 -- no GPU."""
import json
import math
import os

import pytest

from imagine_b200 import autotune as A

POLICY = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "autotuning_policy.json")))


class ClockDevice:
    def __init__(self):
        self.trace = []
        self.next_event = 0

    def synchronize(self):
        self.trace.append(["sync"])

    def cache(self):
        self.trace.append(["cache", 256 * 1024 * 1024])
        return None

    def clear(self, _cache):
        self.trace.append(["clear"])

    def event(self):
        i = self.next_event
        self.next_event += 1
        self.trace.append(["event", i])
        return i

    def record(self, e):
        self.trace.append(["record", e])

    def elapsed(self, s, e):
        self.trace.append(["elapsed", s, e])
        return 50.0 if s == 0 else [1., 3., 2., 5., 4., 9., 6., 7., 8., 10.][s - 2]


def test_do_bench_trace_and_quantiles_match_reference():
    clock = ClockDevice()
    q = A.do_bench(clock, lambda: clock.trace.append(["launch"]))
    assert q == pytest.approx(POLICY["benchmark"]["quantiles"], abs=0)
    assert clock.trace == POLICY["benchmark"]["trace"]


def test_selection_ties_failures_and_cache_match_reference():
    timings = POLICY["selection"]["timings"]
    # as many candidates as the recorded trace has (the policy does not look
    # inside a candidate)
    tuner = A.GemmAutotuner(configs=tuple((i,) for i in range(len(timings))))
    trace, winners = [], []
    for dtype in ["torch.float32", "torch.float32", "torch.float16"]:
        key = (16, 128, 128, "torch.int8", "torch.int8", dtype, "torch.float32", "torch.float32", dtype)

        def bench(i, _cfg):
            trace.append(["launch", i])
            if timings[i] is None:
                raise A.ConfigRejected("out of resources")
            trace.append(["benchmark", i])
            return timings[i]

        w = tuner.select(key, bench)
        trace.append(["launch", w])
        winners.append(w)
    assert winners == POLICY["selection"]["winners"]
    assert trace == POLICY["selection"]["trace"]
    assert len(tuner.cache) == POLICY["selection"]["cache_entries"]
    assert tuner.best_config == 3


def test_unexpected_errors_propagate():
    tuner = A.GemmAutotuner()

    def bench(i, _cfg):
        raise RuntimeError("boom")

    with pytest.raises(RuntimeError):
        tuner.select(("k",), bench)
    assert tuner.cache == {}


def test_quantiles_interpolate():
    assert A.quantiles([4.0]) == [4.0, 4.0, 4.0]
    assert A.quantiles([1.0, 2.0, 3.0, 4.0])[0] == pytest.approx(2.5)
    with pytest.raises(ValueError):
        A.quantiles([])
    assert math.isfinite(A.quantiles([1.0, 1e9])[2])
