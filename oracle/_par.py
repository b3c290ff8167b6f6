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
from concurrent.futures import ThreadPoolExecutor

import numpy as np

THREADS = max(1, os.cpu_count() or 1)
MIN_ELEMS = 1 << 22  # below this, one thread is faster than the hand-off

_pool: ThreadPoolExecutor | None = None


def _get_pool() -> ThreadPoolExecutor:
    global _pool
    if _pool is None:
        _pool = ThreadPoolExecutor(max_workers=THREADS, thread_name_prefix="oracle")
    return _pool


def chunked(fn, x: np.ndarray, *vecs, out_dtype=None) -> np.ndarray:
    """``fn(x_rows, *vecs)`` over row chunks of ``x`` (2-D view over the last
    axis), written into one output of x's shape.  ``vecs`` broadcast over rows
    (per-channel vectors); ``fn`` must be element-wise along rows."""
    x = np.asarray(x)
    if x.size < MIN_ELEMS or THREADS == 1 or x.ndim == 0:
        return fn(x, *vecs)
    shape = x.shape
    x2 = x.reshape(-1, shape[-1]) if x.ndim > 1 else x.reshape(-1, 1)
    n = x2.shape[0]
    parts = min(THREADS * 2, n)
    bounds = np.linspace(0, n, parts + 1).astype(np.int64)
    first = fn(x2[bounds[0]:bounds[1]], *vecs)
    out = np.empty((n,) + first.shape[1:], dtype=out_dtype or first.dtype)
    out[bounds[0]:bounds[1]] = first

    def work(i):
        out[bounds[i]:bounds[i + 1]] = fn(x2[bounds[i]:bounds[i + 1]], *vecs)

    list(_get_pool().map(work, range(1, parts)))
    return out.reshape(shape[:-1] + out.shape[1:]) if x.ndim > 1 else out.reshape(shape)
