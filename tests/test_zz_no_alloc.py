"""ulb_attention_noalloc: the allocation-free attention entry point, for callers that must not
call cudaMalloc / cudaFree (between the kernels of a latency-bound decode step, under another
allocator's reserved memory, or without memory headroom).

Checked through the C ABI against the allocating entry point ulb_attention on the same
inputs, on two calls in a row (the static scratch keeps the previous call's contents, so the
second call also checks that leftover partials and counters do not leak into a result).
This file is collected last so a failure here leaves every other test already run; it also
passes alone in a fresh process."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ATTN_ATOL = 2e-3  # the attention tolerance of tests/test_gpu_kernels.py


def _inputs(rng, H, Hkv, hd, S, rps, positions, cap):
    M = S * rps
    q = rng.standard_normal((M, H * hd)).astype(np.float32)
    k = rng.standard_normal((S, Hkv, cap, hd)).astype(np.float16)
    v = rng.standard_normal((S, Hkv, cap, hd)).astype(np.float16)
    row_seq = np.repeat(np.arange(S, dtype=np.int32), rps)
    row_pos = np.concatenate([np.asarray(p, np.int32) for p in positions])
    return q, k, v, row_seq, row_pos


def _run(ctx, fn_name, desc, arrays, M, rps, out_elems):
    import ulb_capi as U
    bufs = [ctx.buffer(a) for a in arrays]
    out = ctx.buffer(nbytes=out_elems * 2)
    U.check(getattr(U.lib(), fn_name)(ctx.h, C.byref(desc), bufs[0].ptr, bufs[1].ptr, bufs[2].ptr, bufs[3].ptr,
                                      bufs[4].ptr, M, rps, out.ptr))
    ctx.sync()  # the allocation-free call does not synchronise; device errors surface here
    got = out.download(np.float16, (out_elems,))
    for b in bufs + [out]:
        b.free()
    return got.astype(np.float32)


@pytest.mark.parametrize("H,Hkv,hd,S,rps,positions", [
    # caches past 2048 positions: more than 8 key splits, which merge through the scratch
    # (shorter caches merge inside a thread-block cluster and use none)
    (32, 32, 128, 1, 6, [[2434, 2435, 2436, 2437, 2438, 2439]]),      # 7B verify rows, 10 key splits
    (32, 4, 64, 2, 2, [[2600, 2601], [130, 131]]),                    # TinyLlama-like GQA, ragged
])
def test_noalloc_attention_matches_allocating_entry_point(ctx, H, Hkv, hd, S, rps, positions):
    import ulb_capi as U
    rng = np.random.default_rng(hd + S)
    cap = max(max(p) for p in positions) + 5
    desc = U.AttnDesc(H, Hkv, hd, cap, S, 1.0 / np.sqrt(hd))
    M = S * rps
    for call in range(2):
        arrays = _inputs(rng, H, Hkv, hd, S, rps, positions, cap)
        want = _run(ctx, "ulb_attention", desc, arrays, M, rps, M * H * hd)
        got = _run(ctx, "ulb_attention_noalloc", desc, arrays, M, rps, M * H * hd)
        assert np.isfinite(got).all()
        assert np.abs(got - want).max() <= ATTN_ATOL, (call, float(np.abs(got - want).max()))


def test_noalloc_attention_rejects_oversized_shapes(ctx):
    import ulb_capi as U
    # 64 sequences x 32 kv heads x 64 splits of partials exceed the static scratch
    desc = U.AttnDesc(32, 32, 128, 4096, 64, 1.0 / np.sqrt(128))
    null = C.c_void_p(16)
    rc = U.lib().ulb_attention_noalloc(ctx.h, C.byref(desc), null, null, null, null, null, 64 * 9, 9, null)
    assert rc == U.EINVAL
    assert b"static scratch" in U.lib().ulb_last_error()
