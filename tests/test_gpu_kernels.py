"""GPU parity of the sm_100a kernels against the CPU oracle, through the C ABI.

Bars: dequantised weights bit-exact; GEMM relative error <= 1e-2 of the fp32-accumulate
oracle (observed ~1e-6 in the GEMV regime, where both apply each block's scale to an exact
integer dot product; ~2e-4 in the tensor-core regimes, which round each weight once to fp16);
attention within 2e-3 absolute on fp16 outputs; identical accept/reject decisions and
sampled tokens when both sides get the same logits and Philox uniforms."""
import ctypes as C

import numpy as np
import pytest

import gguf
from oracle import ulb_oracle as orc

pytestmark = pytest.mark.gpu

GEMM_RTOL = 1e-2  # GEMM outputs within 1e-2 relative error (fp32 accumulate)
# the tensor-core regimes (M > 32 rows) round each dequantised weight once to fp16 (<= 2^-12
# relative per weight; ~2e-4 of the largest output on these shapes); the GEMV keeps them exact
TC_RTOL = 1e-3


def _q40(rng, N, K):
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    return gguf.quants.quantize(w, gguf.GGMLQuantizationType.Q4_0)


def _q4k(rng, N, K):
    b = rng.integers(0, 256, (N * K // 256, 144), dtype=np.uint8)
    d = (np.abs(rng.standard_normal(N * K // 256)) * 0.002 + 1e-4).astype(np.float16)
    dm = (np.abs(rng.standard_normal(N * K // 256)) * 0.002).astype(np.float16)
    b[:, 0:2] = d.view(np.uint8).reshape(-1, 2)
    b[:, 2:4] = dm.view(np.uint8).reshape(-1, 2)
    return b.reshape(N, -1)


# ulb_qgemm's regimes by row count: the mma.sync GEMV up to 32 rows, the tcgen05 GEMM with
# 64-token tiles and K split a fixed number of ways per matrix for 33 ... 255 rows, the
# tcgen05 GEMM without a K split from 256 rows; a row's arithmetic is fixed within a regime
REGIME_FIRST_ROW = (1, 33, 256)


def _regime_first(M):
    return max(r for r in REGIME_FIRST_ROW if r <= M)


def _rel(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.mark.parametrize("qt,N,K", [("q4_0", 48, 256), ("q4_0", 4096, 4096), ("q4_k", 32, 512),
                                    ("q4_k", 11008, 4096), ("q4_0", 1000, 1408)])
def test_dequant_bit_exact(ctx, qt, N, K):
    rng = np.random.default_rng(N + K)
    raw = _q40(rng, N, K) if qt == "q4_0" else _q4k(rng, N, K)
    t = orc.T_Q4_0 if qt == "q4_0" else orc.T_Q4_K
    h = ctx.upload_tensor(t, (K, N), raw)
    try:
        got = ctx.dequant(h, N, K)
    finally:
        ctx.free_tensor(h)
    want = orc.dequant(t, raw, N * K).reshape(N, K)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    ref = gguf.quants.dequantize(raw.reshape(-1, 18 if qt == "q4_0" else 144),
                                 gguf.GGMLQuantizationType.Q4_0 if qt == "q4_0" else
                                 gguf.GGMLQuantizationType.Q4_K).reshape(N, K)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("qt", ["q4_0", "q4_k"])
@pytest.mark.parametrize("M", [1, 2, 5, 8, 13, 16, 32, 33, 64, 70, 100, 200, 255, 256, 576])
def test_qgemm_matches_oracle_small(ctx, qt, M):
    rng = np.random.default_rng(100 + M)
    N, K = 208, 1024
    raw = _q40(rng, N, K) if qt == "q4_0" else _q4k(rng, N, K)
    t = orc.T_Q4_0 if qt == "q4_0" else orc.T_Q4_K
    x = rng.standard_normal((M, K)).astype(np.float16)
    h = ctx.upload_tensor(t, (K, N), raw)
    try:
        y = ctx.qgemm(h, x, N)
    finally:
        ctx.free_tensor(h)
    ref = orc.qgemv(t, raw, N, K, x)
    assert _rel(y, ref) < (1e-5 if M <= 32 else TC_RTOL), _rel(y, ref)


@pytest.mark.parametrize("qt", ["q4_0", "q4_k"])
@pytest.mark.parametrize("NK", [(4096, 4096), (11008, 4096), (4096, 11008)])
@pytest.mark.parametrize("M", [1, 5, 8, 16, 64, 256, 576])
def test_qgemm_op_sweep(ctx, qt, NK, M):
    """Config-3 op sweep shapes: every (N, K) x M, Q4_0 and Q4_K, x ~ fp16 N(0,1)."""
    N, K = NK
    rng = np.random.default_rng(N * 7 + K + M)
    raw = _q40(rng, N, K) if qt == "q4_0" else _q4k(rng, N, K)
    t = orc.T_Q4_0 if qt == "q4_0" else orc.T_Q4_K
    x = rng.standard_normal((M, K)).astype(np.float16)
    h = ctx.upload_tensor(t, (K, N), raw)
    try:
        y = ctx.qgemm(h, x, N)
        # the same last row computed in the smallest batch of the same regime
        lo = _regime_first(M)
        y_last = ctx.qgemm(h, x[M - lo:M], N)[-1]
        y_gemv = ctx.qgemm(h, x[M - 1:M], N)[0]
    finally:
        ctx.free_tensor(h)
    # rows the oracle checks: the first 8, and the first and last row of every 64-token tile
    # of the tensor-core regimes plus the batch's last row (0, 63, 64, 127, ..., M - 1)
    rows = sorted({r for r in range(min(M, 8))} | {r for t0 in range(0, M, 64) for r in (t0, t0 + 63) if r < M} |
                  {M - 1})
    ref = orc.qgemv(t, raw, N, K, x[rows])
    assert _rel(y[rows], ref) < GEMM_RTOL
    assert _rel(y[rows], ref) < (1e-4 if M <= 32 else TC_RTOL)
    # within a regime every row is computed with the same arithmetic whatever M is
    assert np.array_equal(y_last, y[M - 1])
    # across regimes (tensor-core GEMM vs GEMV) rows agree to the GEMM's fp16 weights and fp32
    # accumulation order: the GEMM chains K/16 fp32 tensor-core accumulations over the whole row
    # of fp16-rounded weights; the GEMV sums scaled 32-weight blocks of exact weights
    assert _rel(y[M - 1], y_gemv) < (1e-4 if M <= 32 else TC_RTOL)


@pytest.mark.parametrize("qt", ["q4_0", "q4_k"])
def test_qgemm_split_regime_in_several_launches(ctx, qt):
    """250 rows of an 11008 x 4096 matrix: the K-split partial sums of all 64-token tiles do
    not fit the context workspace at once, so the token tiles go in several launches; every
    row still matches the oracle and the same row computed in a 33-row batch, bit for bit."""
    N, K, M = 11008, 4096, 250
    rng = np.random.default_rng(7)
    raw = _q40(rng, N, K) if qt == "q4_0" else _q4k(rng, N, K)
    t = orc.T_Q4_0 if qt == "q4_0" else orc.T_Q4_K
    x = rng.standard_normal((M, K)).astype(np.float16)
    h = ctx.upload_tensor(t, (K, N), raw)
    try:
        y = ctx.qgemm(h, x, N)
        y33 = ctx.qgemm(h, x[M - 33:M], N)
        y_again = ctx.qgemm(h, x, N)
    finally:
        ctx.free_tensor(h)
    pick = [0, 63, 64, 191, 192, 249]  # rows on both sides of the launch boundaries
    ref = orc.qgemv(t, raw, N, K, x[pick])
    assert _rel(y[pick], ref) < TC_RTOL
    assert np.array_equal(y[M - 33:], y33)
    assert np.array_equal(y, y_again)


def test_qgemm_rows_independent_of_batch(ctx):
    rng = np.random.default_rng(1)
    N, K = 512, 2048
    raw = _q40(rng, N, K)
    x = rng.standard_normal((6, K)).astype(np.float16)
    h = ctx.upload_tensor(orc.T_Q4_0, (K, N), raw)
    try:
        y6 = ctx.qgemm(h, x, N)
        for m in range(6):
            assert np.array_equal(ctx.qgemm(h, x[m:m + 1], N)[0], y6[m])
    finally:
        ctx.free_tensor(h)


def test_graph_capture_replays_per_op_calls(ctx):
    """ulb_capture_begin / end record ulb_qgemm calls; a replay gives the direct result."""
    import ulb_capi as U
    rng = np.random.default_rng(2)
    N, K, M = 256, 1024, 5
    h = ctx.upload_tensor(orc.T_Q4_0, (K, N), _q40(rng, N, K))
    x = rng.standard_normal((M, K)).astype(np.float16)
    xb = ctx.buffer(x)
    yb = ctx.buffer(nbytes=M * N * 4)
    try:
        want = ctx.qgemm(h, x, N)
        yb.upload(np.zeros((M, N), np.float32))
        g = ctx.capture(lambda: U.check(U.lib().ulb_qgemm(ctx.h, h, xb.ptr, M, yb.ptr, N)))
        assert not yb.download(np.float32, (M, N)).any()  # recorded, not run
        U.check(U.lib().ulb_graph_launch(ctx.h, g))
        ctx.sync()
        assert np.array_equal(yb.download(np.float32, (M, N)), want)
        U.lib().ulb_graph_free(g)
    finally:
        xb.free()
        yb.free()
        ctx.free_tensor(h)


def _attn_case(ctx, H, Hkv, hd, S, rps, positions, seed):
    import ulb_capi as U
    rng = np.random.default_rng(seed)
    cap = max(max(p) for p in positions) + 3
    M = S * rps
    q = rng.standard_normal((M, H * hd)).astype(np.float32)
    k = (rng.standard_normal((S, Hkv, cap, hd))).astype(np.float16)
    v = (rng.standard_normal((S, Hkv, cap, hd))).astype(np.float16)
    row_seq = np.repeat(np.arange(S, dtype=np.int32), rps)
    row_pos = np.concatenate([np.asarray(p, np.int32) for p in positions])
    want = orc.attention(H, Hkv, hd, cap, 1.0 / np.sqrt(hd), q, k.view(np.uint16), v.view(np.uint16),
                         row_seq, row_pos)
    bufs = [ctx.buffer(a) for a in (q, k, v, row_seq, row_pos)]
    out = ctx.buffer(nbytes=M * H * hd * 2)
    d = U.AttnDesc(H, Hkv, hd, cap, S, 1.0 / np.sqrt(hd))
    U.check(U.lib().ulb_attention(ctx.h, C.byref(d), bufs[0].ptr, bufs[1].ptr, bufs[2].ptr, bufs[3].ptr,
                                  bufs[4].ptr, M, rps, out.ptr))
    got = out.download(np.float16, (M, H * hd))
    for b in bufs + [out]:
        b.free()
    return got.astype(np.float32), want.astype(np.float32)


@pytest.mark.parametrize("H,Hkv,hd,S,rps,positions", [
    (32, 32, 128, 1, 6, [[639, 640, 641, 642, 643, 644]]),        # 7B verify rows (k=5)
    (32, 4, 64, 1, 2, [[700, 701]]),                               # TinyLlama draft step 0
    (32, 4, 64, 1, 1, [[63]]),                                     # single chunk
    (8, 8, 64, 3, 5, [[10, 11, 12, 13, 14], [127, 128, 129, 130, 131], [0, 1, 2, 3, 4]]),
    (32, 8, 128, 2, 9, [list(range(300, 309)), list(range(4000, 4009))]),  # Llama-3 GQA k=8
    (8, 8, 64, 1, 64, [list(range(0, 64))]),                       # prefill chunk
    # three sequences with 2, 4 and 1 live key splits of a 4-split cache: thread-block clusters
    # whose CTAs past a sequence's end only join the cluster barriers
    (8, 2, 64, 3, 4, [list(range(300, 304)), list(range(1000, 1004)), list(range(5, 9))]),
])
def test_attention_matches_oracle(ctx, H, Hkv, hd, S, rps, positions):
    got, want = _attn_case(ctx, H, Hkv, hd, S, rps, positions, seed=H + hd + S)
    assert np.abs(got - want).max() < 2e-3


def _attn_form(ctx, form, H, Hkv, hd, S, rps, positions, cap, arrays, paged=None):
    """attention output (fp16 bits) with the kernel form forced to `form`"""
    import ulb_capi as U
    M = S * rps
    bufs = [ctx.buffer(a) for a in arrays]
    out = ctx.buffer(nbytes=M * H * hd * 2)
    d = U.AttnDesc(H, Hkv, hd, cap, S, 1.0 / np.sqrt(hd))
    U.check(U.lib().ulb_attention_set_form(ctx.h, form))
    try:
        if paged is None:
            U.check(U.lib().ulb_attention(ctx.h, C.byref(d), bufs[0].ptr, bufs[1].ptr, bufs[2].ptr, bufs[3].ptr,
                                          bufs[4].ptr, M, rps, out.ptr))
        else:
            tb = ctx.buffer(paged[0])
            U.check(U.lib().ulb_attention_paged(ctx.h, C.byref(d), bufs[0].ptr, bufs[1].ptr, bufs[2].ptr, tb.ptr,
                                                paged[1], bufs[3].ptr, bufs[4].ptr, M, rps, out.ptr))
            tb.free()
    finally:
        U.check(U.lib().ulb_attention_set_form(ctx.h, 0))
    got = out.download(np.uint16, (M, H * hd))
    for b in bufs + [out]:
        b.free()
    return got


_RF = np.random.default_rng(5)


@pytest.mark.parametrize("H,Hkv,hd,S,rps,positions", [
    (32, 32, 128, 1, 6, [list(range(2434, 2440))]),                                    # 7B verify, 10 splits
    (32, 8, 128, 24, 9, [list(range(int(a), int(a) + 9)) for a in _RF.integers(100, 3000, 24)]),  # config-4 verify
    (32, 8, 64, 40, 1, [[int(a)] for a in _RF.integers(0, 2900, 40)]),                  # config-4 draft rows
    (64, 8, 128, 8, 7, [list(range(int(a), int(a) + 7)) for a in _RF.integers(1900, 2300, 8)]),  # config-5 verify
    (32, 4, 64, 3, 2, [[700, 701], [30, 31], [1500, 1501]]),                             # 1..6 splits, ragged
])
def test_attention_forms_give_the_same_bits(ctx, H, Hkv, hd, S, rps, positions):
    """The per-split and the streaming attention kernels compute every row with the same
    arithmetic: forcing either form gives bit-identical outputs (so the form chosen for a
    batch never changes a sequence's result), contiguous and paged caches alike; the streaming
    form also matches the oracle."""
    rng = np.random.default_rng(hd * S + rps)
    cap = max(max(p) for p in positions) + 3
    M = S * rps
    q = rng.standard_normal((M, H * hd)).astype(np.float32)
    k = rng.standard_normal((S, Hkv, cap, hd)).astype(np.float16)
    v = rng.standard_normal((S, Hkv, cap, hd)).astype(np.float16)
    row_seq = np.repeat(np.arange(S, dtype=np.int32), rps)
    row_pos = np.concatenate([np.asarray(p, np.int32) for p in positions])
    arrays = (q, k, v, row_seq, row_pos)
    a = _attn_form(ctx, 1, H, Hkv, hd, S, rps, positions, cap, arrays)
    b = _attn_form(ctx, 2, H, Hkv, hd, S, rps, positions, cap, arrays)
    assert np.array_equal(a, b), "forms differ at %d of %d outputs" % (int((a != b).sum()), a.size)
    # the same keys over a shuffled pool of 256-position pages
    PAGE = 256
    maxp = (cap + PAGE - 1) // PAGE
    n_pages = S * maxp
    perm = rng.permutation(n_pages)
    table = perm.reshape(S, maxp).astype(np.int32)
    kp = np.zeros((n_pages, Hkv, PAGE, hd), np.float16)
    vp = np.zeros((n_pages, Hkv, PAGE, hd), np.float16)
    for s_ in range(S):
        for j in range(maxp):
            n = min(PAGE, cap - j * PAGE)
            kp[table[s_, j], :, :n] = k[s_, :, j * PAGE:j * PAGE + n]
            vp[table[s_, j], :, :n] = v[s_, :, j * PAGE:j * PAGE + n]
    pa = _attn_form(ctx, 1, H, Hkv, hd, S, rps, positions, cap, (q, kp, vp, row_seq, row_pos), (table, maxp))
    pb = _attn_form(ctx, 2, H, Hkv, hd, S, rps, positions, cap, (q, kp, vp, row_seq, row_pos), (table, maxp))
    assert np.array_equal(pa, pb)
    assert np.array_equal(pa, a), "paged and contiguous caches differ"
    if M * cap <= 200000:
        want = orc.attention(H, Hkv, hd, cap, 1.0 / np.sqrt(hd), q, k.view(np.uint16), v.view(np.uint16),
                             row_seq, row_pos)
        assert np.abs(b.view(np.float16).astype(np.float32) - want.astype(np.float32)).max() < 2e-3


@pytest.mark.parametrize("H,Hkv,hd,S,rps,positions", [
    (32, 32, 128, 1, 6, [[639, 640, 641, 642, 643, 644]]),                      # 7B verify rows, 3 pages
    (32, 4, 64, 3, 2, [[700, 701], [30, 31], [1500, 1501]]),                     # draft rows, ragged
    (32, 8, 128, 2, 9, [list(range(2300, 2309)), list(range(4000, 4009))]),      # > 8 splits: global merge
])
def test_paged_attention_matches_oracle(ctx, H, Hkv, hd, S, rps, positions):
    """ulb_attention_paged: the same keys as a contiguous cache, scattered over a shuffled pool
    of 256-position pages through the block table (pages past a sequence's last position left
    unmapped), give the oracle's attention."""
    import ulb_capi as U
    rng = np.random.default_rng(hd + S + 100)
    PAGE = 256
    cap = max(max(p) for p in positions) + 3
    maxp = (cap + PAGE - 1) // PAGE
    M = S * rps
    q = rng.standard_normal((M, H * hd)).astype(np.float32)
    k = rng.standard_normal((S, Hkv, maxp * PAGE, hd)).astype(np.float16)
    v = rng.standard_normal((S, Hkv, maxp * PAGE, hd)).astype(np.float16)
    row_seq = np.repeat(np.arange(S, dtype=np.int32), rps)
    row_pos = np.concatenate([np.asarray(p, np.int32) for p in positions])
    want = orc.attention(H, Hkv, hd, maxp * PAGE, 1.0 / np.sqrt(hd), q, k.view(np.uint16), v.view(np.uint16),
                         row_seq, row_pos)
    n_pages = S * maxp + 3
    perm = rng.permutation(n_pages)
    table = np.full((S, maxp), -1, np.int32)
    kp = np.zeros((n_pages, Hkv, PAGE, hd), np.float16)
    vp = np.zeros((n_pages, Hkv, PAGE, hd), np.float16)
    for s in range(S):
        for j in range(max(positions[s]) // PAGE + 1):
            pg = perm[s * maxp + j]
            table[s, j] = pg
            kp[pg] = k[s, :, j * PAGE:(j + 1) * PAGE]
            vp[pg] = v[s, :, j * PAGE:(j + 1) * PAGE]
    bufs = [ctx.buffer(a) for a in (q, kp, vp, table, row_seq, row_pos)]
    out = ctx.buffer(nbytes=M * H * hd * 2)
    d = U.AttnDesc(H, Hkv, hd, cap, S, 1.0 / np.sqrt(hd))
    U.check(U.lib().ulb_attention_paged(ctx.h, C.byref(d), bufs[0].ptr, bufs[1].ptr, bufs[2].ptr, bufs[3].ptr, maxp,
                                        bufs[4].ptr, bufs[5].ptr, M, rps, out.ptr))
    got = out.download(np.float16, (M, H * hd)).astype(np.float32)
    for b in bufs + [out]:
        b.free()
    assert np.abs(got - want.astype(np.float32)).max() < 2e-3


def _sample_gpu(ctx, logits, warp, seed, rnd, slot, tag):
    import ulb_capi as U
    rows, V = logits.shape
    lb = ctx.buffer(np.ascontiguousarray(logits, np.float32))
    ob = ctx.buffer(nbytes=rows * 4)
    w = U.Warp(*warp)
    U.check(U.lib().ulb_sample(ctx.h, lb.ptr, rows, V, V, C.byref(w), seed, rnd, slot, tag, ob.ptr))
    out = ob.download(np.int32, (rows,))
    lb.free(); ob.free()
    return out


@pytest.mark.parametrize("warp", [(0.0, 0, 1.0), (0.8, 40, 1.0), (1.0, 0, 1.0), (0.8, 0, 0.9),
                                  (1.2, 100, 0.5)])
def test_sample_matches_oracle(ctx, warp):
    rng = np.random.default_rng(4)
    rows, V = 24, 32000
    logits = (rng.standard_normal((rows, V)) * 3).astype(np.float32)
    got = _sample_gpu(ctx, logits, warp, seed=77, rnd=3, slot=1, tag=1)
    want = [orc.sample(logits[r], orc.uniform(77, 3, r, 1, 1), *warp) for r in range(rows)]
    assert got.tolist() == want


def test_sample_top_p_large_vocab(ctx):
    rng = np.random.default_rng(8)
    rows, V = 6, 128256
    logits = (rng.standard_normal((rows, V)) * 2).astype(np.float32)
    warp = (0.8, 0, 0.9)
    got = _sample_gpu(ctx, logits, warp, seed=5, rnd=0, slot=0, tag=1)
    want = [orc.sample(logits[r], orc.uniform(5, 0, r, 0, 1), *warp) for r in range(rows)]
    assert got.tolist() == want


@pytest.mark.parametrize("kind", ["flat", "ties", "narrow_large_vocab", "one_hot"])
@pytest.mark.parametrize("warp", [(0.8, 40, 1.0), (0.8, 0, 0.9), (1.0, 1000, 0.5)])
def test_sample_cut_selection_paths(ctx, kind, warp):
    """The top-k / top-p cut on rows that stress its selection: all logits equal (one bin holds
    the whole row: the whole-row fallback), logits on a coarse grid (many exact ties), a narrow
    128256-wide row (the cut bin overflows the candidate buffer) and a single dominant logit."""
    rng = np.random.default_rng(21)
    rows = 4
    if kind == "flat":
        logits = np.zeros((rows, 32000), np.float32)
    elif kind == "ties":
        logits = (np.round(rng.standard_normal((rows, 32000)) * 4) / 4).astype(np.float32)
    elif kind == "narrow_large_vocab":
        logits = (rng.standard_normal((rows, 128256)) * 0.4).astype(np.float32)
    else:
        logits = (rng.standard_normal((rows, 32000)) * 0.1).astype(np.float32)
        logits[:, 17] = 30.0
    got = _sample_gpu(ctx, logits, warp, seed=31, rnd=2, slot=0, tag=1)
    want = [orc.sample(logits[r], orc.uniform(31, 2, r, 0, 1), *warp) for r in range(rows)]
    assert got.tolist() == want


def _accept_gpu(ctx, pl, ql, draft, warp, seed, rnd):
    import ulb_capi as U
    B, k = draft.shape
    V = pl.shape[-1]
    bufs = [ctx.buffer(np.ascontiguousarray(a)) for a in (pl, ql if k else np.zeros(4, np.float32),
                                                          draft if k else np.zeros(4, np.int32))]
    ot = ctx.buffer(nbytes=B * (k + 1) * 4)
    on = ctx.buffer(nbytes=B * 4)
    w = U.Warp(*warp)
    U.check(U.lib().ulb_spec_accept(ctx.h, bufs[0].ptr, bufs[1].ptr, bufs[2].ptr, B, k, V, C.byref(w),
                                    seed, rnd, ot.ptr, on.ptr))
    out = ot.download(np.int32, (B, k + 1))
    n = on.download(np.int32, (B,))
    for b in bufs + [ot, on]:
        b.free()
    return out, n


@pytest.mark.parametrize("warp", [(0.0, 0, 1.0), (1.0, 0, 1.0), (0.8, 40, 1.0), (0.8, 0, 0.9)])
def test_spec_accept_matches_oracle(ctx, warp):
    """Config-3 rejection shapes: p [64, 9, 32000], q [64, 8, 32000] ~ N(0, 3); draft ~ q."""
    rng = np.random.default_rng(12)
    B, k, V = 64, 8, 32000
    pl = (rng.standard_normal((B, k + 1, V)) * 3).astype(np.float32)
    ql = (rng.standard_normal((B, k, V)) * 3).astype(np.float32)
    # make some drafts agree with the target so accept paths are exercised
    ql[: B // 2] = pl[: B // 2, :k] + 0.3 * ql[: B // 2]
    draft = np.array([[orc.sample(ql[b, i], orc.uniform(9, 0, b, i, 1), *warp) for i in range(k)]
                      for b in range(B)], np.int32)
    got_t, got_n = _accept_gpu(ctx, pl, ql, draft, warp, seed=9, rnd=4)
    want_t, want_n = orc.spec_accept(pl, ql, draft, warp, seed=9, rnd=4)
    assert got_n.tolist() == want_n.tolist()
    for b in range(B):
        assert got_t[b, :want_n[b] + 1].tolist() == want_t[b, :want_n[b] + 1].tolist()
    assert want_n.max() > 0 and want_n.min() < k  # both branches covered


def test_spec_accept_is_lossless_chi2(ctx):
    """Committed first token of a round ~ p exactly (Leviathan et al. 2023): 6000 sequences
    with the same p / q logits and independent Philox uniforms, drafts sampled on the GPU."""
    import ulb_capi as U
    B, V = 6000, 6
    rng = np.random.default_rng(3)
    p1 = (rng.standard_normal(V) * 1.5).astype(np.float32)
    q1 = (rng.standard_normal(V) * 1.5).astype(np.float32)
    pl = np.broadcast_to(p1, (B, 2, V)).copy()
    ql = np.broadcast_to(q1, (B, 1, V)).copy()
    qb = ctx.buffer(ql)
    db = ctx.buffer(nbytes=B * 4)
    w = U.Warp(1.0, 0, 1.0)
    U.check(U.lib().ulb_sample(ctx.h, qb.ptr, B, V, V, C.byref(w), 11, 0, 0, U.RNG_DRAFT, db.ptr))
    draft = db.download(np.int32, (B, 1))
    qb.free(); db.free()
    out, n = _accept_gpu(ctx, pl, ql, draft, (1.0, 0, 1.0), seed=11, rnd=0)
    p = orc.warp_probs(p1, 1.0)
    q = orc.warp_probs(q1, 1.0)
    dcount = np.bincount(draft[:, 0], minlength=V)
    assert ((dcount - q * B) ** 2 / (q * B)).sum() < 25.0  # drafts ~ q
    counts = np.bincount(out[:, 0], minlength=V)
    chi2 = ((counts - p * B) ** 2 / (p * B)).sum()
    assert chi2 < 25.0, (chi2, counts, p * B)  # 5 dof: p-value ~ 1e-4
    assert 0 < (n == 1).mean() < 1


def test_spec_accept_k0_is_plain_sampling(ctx):
    rng = np.random.default_rng(2)
    pl = (rng.standard_normal((4, 1, 1000))).astype(np.float32)
    got_t, got_n = _accept_gpu(ctx, pl, None, np.zeros((4, 0), np.int32), (1.0, 0, 1.0), 3, 7)
    want_t, want_n = orc.spec_accept(pl, np.zeros((4, 0, 1000), np.float32), np.zeros((4, 0), np.int32),
                                     (1.0, 0, 1.0), 3, 7)
    assert (got_n == 0).all() and got_t[:, 0].tolist() == want_t[:, 0].tolist()
