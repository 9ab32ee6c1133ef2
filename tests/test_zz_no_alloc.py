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


def _ragged(rng, S, rps, lo, hi):
    """S sequences of rps consecutive rows each, the first row at a position in [lo, hi)"""
    starts = rng.integers(lo, hi, S)
    return [list(range(int(s0), int(s0) + rps)) for s0 in starts]


_R = np.random.default_rng(77)


@pytest.mark.parametrize("H,Hkv,hd,S,rps,positions,cap", [
    # caches past 2048 positions: more than 8 key splits, which merge through the scratch
    (32, 32, 128, 1, 6, [[2434, 2435, 2436, 2437, 2438, 2439]], None),  # 7B verify rows, 10 key splits
    (32, 4, 64, 2, 2, [[2600, 2601], [130, 131]], None),                # TinyLlama-like GQA, ragged
    # one key split (capacity <= 256): neither the scratch nor the counters are used
    (32, 8, 128, 5, 3, _ragged(_R, 5, 3, 0, 250), 256),
    # 2..8 splits merged in a thread-block cluster: 64 sequences of a config-4-like batch, whose
    # global-merge scratch (4.3 Mi floats) would not fit the static array, are accepted
    (32, 8, 128, 64, 1, _ragged(_R, 64, 1, 0, 1020), 1024),
    (32, 4, 64, 9, 2, _ragged(_R, 9, 2, 200, 2040), 2048),
    # a global merge whose partials (11 x 8 heads x 11 splits x 16 x 130 floats = 2.01 Mi) just fit
    (32, 8, 128, 11, 1, _ragged(_R, 11, 1, 2400, 2595), 2600),
])
@pytest.mark.parametrize("form", [0, 1])  # the form the library picks; the per-split form (which uses the scratch)
def test_noalloc_attention_matches_allocating_entry_point(ctx, H, Hkv, hd, S, rps, positions, cap, form):
    import ulb_capi as U
    rng = np.random.default_rng(hd + S)
    cap = cap or max(max(p) for p in positions) + 5
    desc = U.AttnDesc(H, Hkv, hd, cap, S, 1.0 / np.sqrt(hd))
    M = S * rps
    U.check(U.lib().ulb_attention_set_form(ctx.h, form))
    try:
        for call in range(2):
            arrays = _inputs(rng, H, Hkv, hd, S, rps, positions, cap)
            want = _run(ctx, "ulb_attention", desc, arrays, M, rps, M * H * hd)
            got = _run(ctx, "ulb_attention_noalloc", desc, arrays, M, rps, M * H * hd)
            assert np.isfinite(got).all()
            assert np.abs(got - want).max() <= ATTN_ATOL, (call, float(np.abs(got - want).max()))
    finally:
        U.check(U.lib().ulb_attention_set_form(ctx.h, 0))


def test_noalloc_attention_rejects_oversized_shapes(ctx):
    import ulb_capi as U
    # in the per-split form, 64 sequences x 32 kv heads x 16 splits of partials exceed the static
    # scratch; the call is rejected before anything is launched (the pointers are never read)
    desc = U.AttnDesc(32, 32, 128, 4096, 64, 1.0 / np.sqrt(128))
    null = C.c_void_p(16)
    U.check(U.lib().ulb_attention_set_form(ctx.h, 1))
    try:
        rc = U.lib().ulb_attention_noalloc(ctx.h, C.byref(desc), null, null, null, null, null, 64 * 9, 9, null)
    finally:
        U.check(U.lib().ulb_attention_set_form(ctx.h, 0))
    assert rc == U.EINVAL
    assert b"static scratch" in U.lib().ulb_last_error()


@pytest.mark.parametrize("fn", ["ulb_attention", "ulb_attention_noalloc"])
def test_attention_rejects_bad_descriptors_with_einval(ctx, fn):
    """No head count of zero, rows_per_seq of zero or ragged M reaches the host arithmetic."""
    import ulb_capi as U
    null = C.c_void_p(16)
    for desc, M, rps in ((U.AttnDesc(32, 0, 128, 512, 1, 0.1), 6, 6),
                         (U.AttnDesc(32, 8, 128, 512, 1, 0.1), 6, 0),
                         (U.AttnDesc(32, 8, 128, 512, 1, 0.1), 7, 6),
                         (U.AttnDesc(32, 5, 128, 512, 1, 0.1), 6, 6)):
        rc = getattr(U.lib(), fn)(ctx.h, C.byref(desc), null, null, null, null, null, M, rps, null)
        assert rc == U.EINVAL, (fn, rc)
