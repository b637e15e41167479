"""CPU baseline of the optimizer step on the host cores — TEST / BENCHMARK INFRASTRUCTURE ONLY.

Runs the oracle (``muzo_oracle``, the numpy restatement of the reference's arithmetic) through
one optimizer step on one Llama-3-8B k_proj-shaped bf16 block (1024 x 4096): three
perturbation passes, the H-step normal-noise momentum rebuild, five Newton-Schulz iterations and
the update. ``throughput_sample`` runs one such block per host core in a spawn process pool
(BLAS limited to one thread per worker, so the cores are not oversubscribed; at most 32
workers) and reports the
wall time of the whole batch with each worker's phase split; the caller extrapolates to the full
model. Only ``bench.py`` uses it, for its reported CPU baseline and its reference arm.
"""

from __future__ import annotations

import multiprocessing as mp
import os
import time
from concurrent.futures import ProcessPoolExecutor

import numpy as np

ROWS, COLS = 1024, 4096


def block_step(seed: int, horizon: int = 8) -> tuple[float, float, float, float]:
    """Seconds spent in (perturbation passes, rebuild, Newton-Schulz, update) for one block."""
    import muzo_oracle as orc

    rng = np.random.default_rng(seed)
    w = orc.bf16_round(rng.standard_normal((ROWS, COLS), dtype=np.float32) * 0.02)
    keys = [int(k) for k in rng.integers(0, 2**63 - 1, size=horizon + 1, dtype=np.int64)]
    ps = np.clip(rng.standard_normal(horizon), -3, 3)
    t0 = time.perf_counter()
    for alpha in (1e-3, -2e-3, 1e-3):
        w = orc.perturb(w, keys[0], alpha, "normal", "bf16")
    t1 = time.perf_counter()
    coeffs = [0.9 ** a for a in range(horizon)]
    m = orc.rebuild((ROWS, COLS), keys[1:], [c * p for c, p in zip(coeffs, ps)], "normal", "bf16",
                    float(np.float32(1.0) / np.float32(sum(coeffs))))
    t2 = time.perf_counter()
    x = orc.ns5_bf16(m, 5)
    t3 = time.perf_counter()
    orc.apply_update(w, x, 1e-5, 0.2, 0.01, 0.01, "bf16")
    t4 = time.perf_counter()
    return t1 - t0, t2 - t1, t3 - t2, t4 - t3


def _worker_init(oracle_dir: str) -> None:
    import sys

    if oracle_dir not in sys.path:
        sys.path.insert(0, oracle_dir)
    try:
        from threadpoolctl import threadpool_limits

        threadpool_limits(1)
    except Exception:
        os.environ["OMP_NUM_THREADS"] = "1"
    import muzo_oracle  # noqa: F401  (imported before the timed batch)


def _ready(_: int) -> int:
    time.sleep(1.0)  # concurrent sleepers make the executor start every worker
    return os.getpid()


class HostPool:
    """One spawn worker per host core (started and initialised on entry), reusable for several
    timed batches."""

    MAX_WORKERS = 32  # every spawn worker re-imports the caller's main module

    def __init__(self, workers: int | None = None):
        try:
            usable = len(os.sched_getaffinity(0))
        except (AttributeError, OSError):
            usable = os.cpu_count() or 1
        self.workers = workers or max(1, min(usable, self.MAX_WORKERS))
        self._ex = None

    def __enter__(self) -> "HostPool":
        ctx = mp.get_context("spawn")
        self._ex = ProcessPoolExecutor(max_workers=self.workers, mp_context=ctx, initializer=_worker_init,
                                       initargs=(os.path.dirname(os.path.abspath(__file__)),))
        list(self._ex.map(_ready, range(self.workers)))  # every worker started and initialised
        return self

    def __exit__(self, *exc) -> None:
        self._ex.shutdown()

    def batch(self, seed: int = 0) -> tuple[float, list[tuple]]:
        """One block per worker, all at once: the batch's wall seconds and every block's phases."""
        t0 = time.perf_counter()
        phases = list(self._ex.map(block_step, range(seed, seed + self.workers)))
        return time.perf_counter() - t0, phases


def throughput_sample(seed: int = 0, workers: int | None = None) -> tuple[float, list[tuple], int]:
    """One timed batch on a fresh pool: (wall seconds, per-block phase times, worker count)."""
    with HostPool(workers) as pool:
        wall, phases = pool.batch(seed)
        return wall, phases, pool.workers
