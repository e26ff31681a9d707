"""Per-shape tile-configuration selection for the tcgen05 GEMM.

Mirrors the reference's INT8 autotuner (inference/src/autotuning.rs:86-268):

* one tuner instance per kernel, a cache keyed by (m, n, k, operand dtypes);
* on a cache miss every candidate is timed with ``do_bench`` -- one launch, a
  5-launch estimate with the 256 MiB L2 flush before each, warm-up and repeat
  counts from 25 ms / 100 ms, per-repeat CUDA events, quantiles (0.5, 0.2, 0.8);
* a candidate that the library rejects (an invalid configuration) scores
  +inf, any other error propagates;
* the winner is the lexicographic minimum of the quantile triples, first
  candidate on ties (Python ``min`` semantics, autotuning.rs:118-126).

The candidates are this library's configurations (block_n, group_m, max_ctas,
cta_group) instead of Triton block shapes.  Timing goes through the ``BenchmarkDevice``
protocol so the policy is testable with a fake clock on the CPU.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Protocol, Sequence, Tuple

# (block_n, group_m, max_ctas, cta_group); max_ctas 0 = one persistent CTA
# (pair) per SM; cta_group 2 = CTA pairs with 2-SM MMAs on 256-row tiles
GEMM_CONFIGS: Tuple[Tuple[int, ...], ...] = (
    (256, 8, 0, 1),
    (256, 4, 0, 1),
    (256, 16, 0, 1),
    (128, 8, 0, 1),
    (128, 16, 0, 1),
    (256, 8, 132, 1),
    (256, 8, 0, 2),
)


class BenchmarkDevice(Protocol):
    def synchronize(self) -> None: ...
    def cache(self): ...
    def clear(self, cache) -> None: ...
    def event(self): ...
    def record(self, event) -> None: ...
    def elapsed(self, start, end) -> float: ...


class CudaBenchmark:
    """BenchmarkDevice on the current CUDA stream (autotuning.rs:159-188)."""

    def __init__(self, device=None):
        import torch

        self.torch = torch
        self.device = device if device is not None else torch.device("cuda", torch.cuda.current_device())

    def synchronize(self):
        self.torch.cuda.synchronize(self.device)

    def cache(self):
        return self.torch.empty(256 * 1024 * 1024 // 4, dtype=self.torch.int32, device=self.device)

    def clear(self, cache):
        cache.zero_()

    def event(self):
        return self.torch.cuda.Event(enable_timing=True)

    def record(self, event):
        event.record(self.torch.cuda.current_stream(self.device))

    def elapsed(self, start, end):
        return start.elapsed_time(end)


def quantiles(times: Sequence[float], qs=(0.5, 0.2, 0.8)) -> List[float]:
    """Linear-interpolation quantiles (autotuning.rs:255-268)."""
    if not times:
        raise ValueError("empty benchmark sample")
    s = sorted(times)
    out = []
    for q in qs:
        point = q * (len(s) - 1)
        lo, hi = math.floor(point), math.ceil(point)
        t = point - lo
        out.append((1.0 - t) * s[lo] + t * s[hi])
    return out


def do_bench(device: BenchmarkDevice, launch: Callable[[], None], warmup_ms: float = 25.0,
             rep_ms: float = 100.0) -> List[float]:
    """triton.testing.do_bench as the reference restates it (autotuning.rs:197-254)."""
    launch()
    device.synchronize()
    cache = device.cache()
    start, end = device.event(), device.event()
    device.record(start)
    for _ in range(5):
        device.clear(cache)
        launch()
    device.record(end)
    device.synchronize()
    estimate = device.elapsed(start, end) / 5.0

    def count(t: float) -> int:
        v = math.trunc(t / estimate) if estimate > 0 else math.inf
        if not math.isfinite(v):
            raise ValueError("cannot convert float infinity or NaN to integer")
        return max(1, int(v))

    warmup, repeat = count(warmup_ms), count(rep_ms)
    starts = [device.event() for _ in range(repeat)]
    ends = [device.event() for _ in range(repeat)]
    for _ in range(warmup):
        launch()
    for i in range(repeat):
        device.clear(cache)
        device.record(starts[i])
        launch()
        device.record(ends[i])
    device.synchronize()
    return quantiles([device.elapsed(s, e) for s, e in zip(starts, ends)])


class ConfigRejected(Exception):
    """A candidate the library refuses (the reference's OutOfResources /
    CompileTimeAssertion / PTXAS failures, autotuning.rs:109-117)."""


@dataclass
class GemmAutotuner:
    configs: Tuple[Tuple[int, ...], ...] = GEMM_CONFIGS
    cache: Dict[tuple, int] = field(default_factory=dict)
    best_config: Optional[int] = None
    last_timings: Optional[List[List[float]]] = None

    def select(self, key: tuple, bench: Callable[[int, Tuple[int, ...]], List[float]]) -> int:
        if key in self.cache:
            index = self.cache[key]
        else:
            timings = []
            for i, cfg in enumerate(self.configs):
                try:
                    timings.append(list(bench(i, cfg)))
                except ConfigRejected:
                    timings.append([math.inf] * 3)
            best = 0
            for i in range(1, len(timings)):
                if timings[i] < timings[best]:  # lexicographic, first wins ties
                    best = i
            self.cache[key] = best
            self.last_timings = timings
            index = best
        self.best_config = index
        return index

    def clear(self):
        self.cache.clear()


_TUNERS: Dict[str, GemmAutotuner] = {}


def tuner(kernel: str) -> GemmAutotuner:
    """One tuner per kernel (the reference keeps the tensorwise and per-row
    kernels' caches apart, autotuning.rs:86-93)."""
    return _TUNERS.setdefault(kernel, GemmAutotuner())


def tune_gemm(kernel: str, key: tuple, run: Callable[[Tuple[int, ...]], None],
              device: Optional[BenchmarkDevice] = None) -> Tuple[int, ...]:
    """Pick (and cache) the configuration for `key`; `run(cfg)` launches the
    GEMM once with that configuration (raising ValueError if it is rejected)."""
    dev = device or CudaBenchmark()
    t = tuner(kernel)

    def bench(_i, cfg):
        try:
            return do_bench(dev, lambda: run(cfg))
        except ValueError as e:
            raise ConfigRejected(str(e)) from e

    return t.configs[t.select(key, bench)]
