"""Failure detection on the GPU without a GPU fault.

Every mbarrier wait of the library's kernels is bounded: when a phase does
not complete in time, the waiting thread raises the device error word, the
CTA unwinds and the kernel returns.  ltxq_selftest_wait_timeout runs that
same wait on a barrier that nothing completes, with a limit of a few
milliseconds.  The test checks that the expiry is reported (status, message,
error word), that reading the word clears it, and that the context keeps
working: a quantized GEMM launched afterwards in the same process still
matches the oracle.  Nothing here traps, faults or hangs.
"""

import time

import pytest

from helpers import from_dev_bf16, normal_bf16, rng, to_dev_bf16
from oracle import quant as oq
from oracle import ref_ops as ro

pytestmark = pytest.mark.gpu

WAIT_TIMEOUT_CODE = 1  # kErrWaitTimeout


def test_expired_wait_is_reported_and_the_context_survives(cuda):
    import torch

    import ltxq
    from ltxq import _lib

    lib = _lib.load()
    assert _lib.device_error() == 0  # start with a clear error word
    for limit_ns in (2_000_000, 500_000):
        t0 = time.perf_counter()
        st = lib.ltxq_selftest_wait_timeout(limit_ns, None)
        elapsed = time.perf_counter() - t0
        assert st == _lib.ERR_DEVICE, lib.ltxq_last_error()
        assert b"expired" in lib.ltxq_last_error()
        assert elapsed < 2.0, elapsed  # gave up near its limit, far below the production 2 s
        assert _lib.device_error() == WAIT_TIMEOUT_CODE  # read ...
        assert _lib.device_error() == 0  # ... and cleared

    # the context still answers: a GEMM with a K-split schedule against the oracle
    g = rng(71)
    M, K, N = 201, 2048, 2048
    x = normal_bf16(g, (M, K))
    W = normal_bf16(g, (N, K), 0.02)
    b = normal_bf16(g, (N,), 0.01)
    ql = ltxq.QuantizedLinear.from_linear(to_dev_bf16(W), to_dev_bf16(b), mode="mxfp8")
    out = from_dev_bf16(ql(to_dev_bf16(x)))
    torch.cuda.synchronize()
    ref = ro.linear(x, oq.dequantize(oq.quantize(W, "mxfp8"), K), b)
    assert ro.max_abs_rel(out, ref) <= 2e-2 and ro.cosine(out, ref) >= 0.9995
    assert _lib.device_error() == 0


def test_selftest_rejects_limits_out_of_range(cuda):
    from ltxq import _lib

    lib = _lib.load()
    assert lib.ltxq_selftest_wait_timeout(10, None) == _lib.ERR_INVALID
    assert lib.ltxq_selftest_wait_timeout(5_000_000_000, None) == _lib.ERR_INVALID
    assert _lib.device_error() == 0
