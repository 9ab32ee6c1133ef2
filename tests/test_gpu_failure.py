"""Failure detection on the GPU without a fault: a bounded device-side wait that runs out.

ulb_wait_flag waits on the device for a flag that nothing ever sets; the wait must give up
within its limit, the next ulb_stream_sync must report ULB_ETIMEOUT (the device error flag
the kernel raised), and the context must stay usable: a GEMM enqueued afterwards runs and
matches the oracle, and the following sync is clean.  The peer-death paths of tensor
parallelism are covered on the host (tests/test_failure_cpu.py)."""
import ctypes as C
import time

import numpy as np
import pytest

import gguf
from oracle import ulb_oracle as orc

pytestmark = pytest.mark.gpu


def test_flag_wait_times_out_and_context_stays_usable(ctx):
    import ulb_capi as U
    L = U.lib()
    flag = ctx.buffer(np.zeros(1, np.int32))  # nothing ever writes it
    t0 = time.perf_counter()
    U.check(L.ulb_wait_flag(ctx.h, flag.ptr, 1, 20_000_000))  # 20 ms
    rc = L.ulb_stream_sync(ctx.h)
    dt = time.perf_counter() - t0
    assert rc == U.ETIMEOUT, rc
    assert b"bounded wait" in L.ulb_last_error()
    assert 0.015 < dt < 5.0, dt
    # the flag set: the same wait returns at once and the stream is clean
    flag.upload(np.ones(1, np.int32))
    U.check(L.ulb_wait_flag(ctx.h, flag.ptr, 1, 1_000_000_000))
    assert L.ulb_stream_sync(ctx.h) == U.OK
    # the context still computes
    rng = np.random.default_rng(0)
    N, K = 256, 1024
    raw = gguf.quants.quantize((rng.standard_normal((N, K)) * 0.02).astype(np.float32),
                               gguf.GGMLQuantizationType.Q4_0)
    h = ctx.upload_tensor(orc.T_Q4_0, (K, N), raw)
    x = rng.standard_normal((3, K)).astype(np.float16)
    try:
        y = ctx.qgemm(h, x, N)
    finally:
        ctx.free_tensor(h)
    ref = orc.qgemv(orc.T_Q4_0, raw, N, K, x)
    assert np.abs(y - ref).max() / np.abs(ref).max() < 1e-4
    assert L.ulb_stream_sync(ctx.h) == U.OK
    flag.free()


def test_flag_wait_rejects_unbounded_timeouts(ctx):
    import ulb_capi as U
    null = C.c_void_p(16)
    assert U.lib().ulb_wait_flag(ctx.h, null, 1, 0) == U.EINVAL
    assert U.lib().ulb_wait_flag(ctx.h, null, 1, 60 * 10**9) == U.EINVAL
