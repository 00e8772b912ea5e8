"""Timing harness for generate() calls: synced timestamps, per-configuration warm-up, seeded
interleaving of configurations, and a record of the environment.

Same API and semantics as the reference's bench/harness.py:
- `synchronizer` (bench/harness.py:28-33): the device's synchronize, or a no-op on the CPU.
- `Stopwatch` (bench/harness.py:36-65): every timestamp is read after a sync, so it marks
  finished device work; `mark` keeps the first occurrence of an event only.
- `measure` (bench/harness.py:96-144): warm-up calls and measured rounds both run the
  configurations in an order drawn from `random.Random(seed)` (one `sample` of all names per
  round), so each configuration warms up itself and slow drift spreads over all of them;
  `after_each(config, round)` runs outside the timed window, with round -1 during warm-up.
- `environment` (bench/harness.py:147-168): git commit and dirtiness, versions, platform, CPU,
  device and seed; the GPU line also names the SM version, SM count and memory.

On the engine's fused path a sync at a mark costs no extra pipeline drain: generate() has
already read the first token and each round's results to the host when it emits its events, so
the device is idle there anyway.
"""
from __future__ import annotations

import importlib.metadata
import platform
import random
import subprocess
import sys
import time
from collections.abc import Callable
from dataclasses import dataclass, field

import torch

Clock = Callable[[], float]
Sync = Callable[[], None]


def _no_sync() -> None:
    return None


def synchronizer(device: torch.device) -> Sync:
    """The call that waits for all queued work on `device`'s kind of device."""
    kind = torch.device(device).type
    if kind == "cuda":
        return torch.cuda.synchronize
    if kind == "mps":
        return torch.mps.synchronize
    return _no_sync


class Stopwatch:
    """One timed request. start/stop belong to the harness; the workload calls `mark` (or
    `first_token`) when an event happens. Times are seconds from `start`."""

    def __init__(self, sync: Sync, clock: Clock = time.perf_counter) -> None:
        self.sync = sync
        self.clock = clock
        self.start_at: float | None = None
        self.stop_at: float | None = None
        self.marks: dict[str, float] = {}
        self.tokens = 0

    def _now(self) -> float:
        self.sync()
        return self.clock()

    def start(self) -> None:
        self.start_at = self._now()

    def mark(self, event: str) -> None:
        if event in self.marks:
            return
        self.marks[event] = self._now() - self.start_at

    def first_token(self) -> None:
        self.mark("first_token")

    def stop(self) -> None:
        self.stop_at = self._now()


@dataclass(frozen=True)
class Sample:
    config: str
    round: int
    slot: int        # index of the configuration in its round's order
    total: float     # seconds from the request's start to its end
    tokens: int
    marks: dict[str, float]

    @property
    def ttft(self) -> float:
        return self.marks["first_token"]


# A workload runs one request: it marks its events on the stopwatch ("first_token" at least)
# and returns the number of output tokens.
Workload = Callable[[Stopwatch], int]


@dataclass
class Run:
    samples: list[Sample]
    warmup: int
    repeats: int
    orders: list[list[str]] = field(default_factory=list)


def _timed(name: str, workload: Workload, sync: Sync, clock: Clock) -> Stopwatch:
    watch = Stopwatch(sync, clock)
    watch.start()
    tokens = workload(watch)
    watch.stop()
    if "first_token" not in watch.marks:
        raise RuntimeError(f"{name}: workload never reported its first token")
    watch.tokens = tokens
    return watch


def measure(workloads: dict[str, Workload], warmup: int, repeats: int, sync: Sync, seed: int,
            clock: Clock = time.perf_counter, after_each: Callable[[str, int], None] | None = None) -> Run:
    """Runs every workload `warmup` times unmeasured, then `repeats` measured rounds, each
    round in a fresh seeded order."""
    order_rng = random.Random(seed)
    names = list(workloads)
    for _ in range(warmup):
        for name in order_rng.sample(names, len(names)):
            _timed(name, workloads[name], sync, clock)
            if after_each is not None:
                after_each(name, -1)
    run = Run(samples=[], warmup=warmup, repeats=repeats)
    for rnd in range(repeats):
        order = order_rng.sample(names, len(names))
        run.orders.append(order)
        for slot, name in enumerate(order):
            w = _timed(name, workloads[name], sync, clock)
            run.samples.append(Sample(config=name, round=rnd, slot=slot, total=w.stop_at - w.start_at,
                                      tokens=w.tokens, marks=dict(w.marks)))
            if after_each is not None:
                after_each(name, rnd)
    return run


def _git(*args: str) -> str | None:
    """git's output, or None outside a checkout (the reference raises there; an exported tree
    on a GPU host has no .git)."""
    try:
        return subprocess.run(["git", *args], capture_output=True, text=True, check=True).stdout.strip()
    except (OSError, subprocess.CalledProcessError):
        return None


def cpu_name() -> str:
    if sys.platform == "darwin":
        r = subprocess.run(["sysctl", "-n", "machdep.cpu.brand_string"], capture_output=True, text=True)
        if r.returncode == 0 and r.stdout.strip():
            return r.stdout.strip()
    return platform.processor() or platform.machine()


def gpu_name(device: torch.device) -> str | None:
    device = torch.device(device)
    if device.type == "cuda":
        props = torch.cuda.get_device_properties(device)
        return (f"{props.name} (sm_{props.major}{props.minor}, {props.multi_processor_count} SMs, "
                f"{props.total_memory / 2**30:.0f} GiB; torch CUDA {torch.version.cuda})")
    if device.type == "mps":
        return f"{cpu_name()} integrated GPU (MPS)"
    return None


def environment(device: torch.device, seed: int, models: dict | None = None) -> dict:
    """What a result was measured on. `git_dirty` looks at tracked files only, so results
    written earlier in the same run do not count; both git fields are None outside a checkout."""
    versions = {}
    for pkg in ("torch", "transformers", "numpy", "scipy"):
        try:
            versions[pkg] = importlib.metadata.version(pkg)
        except importlib.metadata.PackageNotFoundError:
            versions[pkg] = None
    commit = _git("rev-parse", "HEAD")
    status = _git("status", "--porcelain", "--untracked-files=no") if commit is not None else None
    record = {
        "git_commit": commit,
        "git_dirty": bool(status) if status is not None else None,
        "python": sys.version.split()[0],
        "packages": versions,
        "platform": platform.platform(),
        "cpu": cpu_name(),
        "device": str(device),
        "gpu": gpu_name(device),
        "seed": seed,
    }
    if models is not None:
        record["models"] = models
    return record
