"""Thread-parallel evaluation of the oracle's large elementwise passes
(test infrastructure only).

numpy's ufunc loops release the GIL, so row chunks of one large array can be
processed on every host core by plain threads.  Every chunk runs exactly the
same element-wise operations as the whole array would, so results are
bit-identical to the serial evaluation.  BLAS calls are left alone (the BLAS
library threads them itself).
"""

from __future__ import annotations

import os
import threading
from concurrent.futures import ThreadPoolExecutor

import numpy as np

def usable_cpus() -> int:
    """Cores this process may run on: the CPU affinity set, capped by a cgroup
    v2 CPU quota (``cpu.max``) when one is set.  os.cpu_count() reports the
    host's cores, which in a container can be many more than it may use
    (thread pools sized to it then oversubscribe the quota)."""
    n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    try:
        with open("/sys/fs/cgroup/cpu.max") as f:
            quota, period = f.read().split()[:2]
        if quota != "max":
            n = min(n, max(1, int(int(quota) / int(period))))
    except (OSError, ValueError):
        pass
    return max(1, n)


THREADS = usable_cpus()
MIN_ELEMS = 1 << 22  # below this, one thread is faster than the hand-off

_pool: ThreadPoolExecutor | None = None


def _get_pool() -> ThreadPoolExecutor:
    global _pool
    if _pool is None:
        _pool = ThreadPoolExecutor(max_workers=THREADS, thread_name_prefix="oracle")
    return _pool


_in_worker = threading.local()


def chunked(fn, x: np.ndarray, *vecs, out_dtype=None) -> np.ndarray:
    """``fn(x_rows, *vecs)`` over row chunks of ``x`` (2-D view over the last
    axis), written into one output of x's shape.  ``vecs`` broadcast over rows
    (per-channel vectors); ``fn`` must be element-wise along rows.  A call
    made from inside a chunk (``fn`` itself calling ``chunked``) runs
    serially: its tasks would otherwise wait behind the very workers that
    wait for them."""
    x = np.asarray(x)
    if x.size < MIN_ELEMS or THREADS == 1 or x.ndim == 0 or getattr(_in_worker, "active", False):
        return fn(x, *vecs)
    shape = x.shape
    x2 = x.reshape(-1, shape[-1]) if x.ndim > 1 else x.reshape(-1, 1)
    n = x2.shape[0]
    parts = min(THREADS * 2, n)
    bounds = np.linspace(0, n, parts + 1).astype(np.int64)
    def run(lo, hi):
        _in_worker.active = True
        try:
            return fn(x2[lo:hi], *vecs)
        finally:
            _in_worker.active = False

    first = run(bounds[0], bounds[1])
    out = np.empty((n,) + first.shape[1:], dtype=out_dtype or first.dtype)
    out[bounds[0]:bounds[1]] = first

    def work(i):
        out[bounds[i]:bounds[i + 1]] = run(bounds[i], bounds[i + 1])

    list(_get_pool().map(work, range(1, parts)))
    return out.reshape(shape[:-1] + out.shape[1:]) if x.ndim > 1 else out.reshape(shape)
