"""CPU tests of bench.py's trace analysis: CTA records grouped into launches (two launches of
different kernels may overlap under programmatic dependent launch; consecutive launches of one
kernel follow each other), ordered by completion, named by their tags."""
import numpy as np

import bench


def _recs(rows):
    r = np.zeros(len(rows), np.dtype(bench.TRACE_REC))
    for i, (tag, cta, grid, arg, t0, t1, t2) in enumerate(rows):
        r[i]["tag"], r[i]["cta"], r[i]["grid"], r[i]["arg"] = tag, cta, grid, arg
        r[i]["t_entry"], r[i]["t_wait"], r[i]["t_exit"] = t0, t1, t2
    return r


def test_overlapping_launches_are_separated_and_ordered_by_completion():
    gemv = 1000 + 1 * 100 + 10  # residual epilogue, one n-tile
    attn = 2001                 # per-split attention with a cluster merge
    rows = [
        # GEMV launch 1 (3 CTAs), the attention (2 CTAs) starting before its last CTA, GEMV launch 2
        (gemv, 0, 3, 2048, 100, 110, 200), (gemv, 1, 3, 2048, 101, 111, 210),
        (attn, 0, 2, 64, 150, 215, 300),
        (gemv, 2, 3, 2048, 160, 170, 205),
        (attn, 1, 2, 64, 151, 216, 310),
        (gemv, 0, 3, 2048, 305, 312, 400), (gemv, 1, 3, 2048, 306, 313, 405), (gemv, 2, 3, 2048, 307, 314, 420),
    ]
    r = _recs(rows)
    L = bench.trace_launches([r[[0, 1, 3, 5, 6, 7]], r[[2, 4]]])
    assert [l["name"] for l in L] == ["qgemv_resid_N2048", "attn_split_hd64_cluster", "qgemv_resid_N2048"]
    assert [l["ctas"] for l in L] == [3, 2, 3]
    assert [l["exit"] for l in L] == [210, 310, 420]
    assert [l["wait"] for l in L] == [170, 216, 314]


def test_kernel_names():
    assert bench.trace_kernel_name(1000 + 3 * 100 + 10 + 1, 2560) == "qgemv_qkv_N2560_rmsnorm"
    assert bench.trace_kernel_name(3002, 128) == "attn_stream_hd128_tiles2"
    assert bench.trace_kernel_name(4002, 64) == "qgemm_tc_epi2_nt64"
    assert bench.trace_kernel_name(7200, 0) == "accept"
