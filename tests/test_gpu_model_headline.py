"""Whole-model GPU parity against the CPU oracle at the benchmark configurations' target shapes.

The op-level tests cover every kernel at these shapes; these run the models themselves, from
the same synthetic GGUF files bench.py decodes (written once per machine into the bench's
model cache):
  - config 2's Llama-2-7B-architecture Q4_0 target (32 layers, d 4096, 32 heads of 128, FFN
    11008, vocabulary 32000, RoPE theta 1e4);
  - config 4's Llama-3-8B-architecture Q4_K target (32 layers, GQA 32 / 8 heads, FFN 14336,
    vocabulary 128256, RoPE theta 5e5).
Each gets a 32-token prefill (last-row logits) and then one 6-row verify block (every row's
logits), on the GPU through the C ABI and on the oracle with identical inputs.

Two depths of each: the first 2 layers (a file with the same seed holds the same tensors, so
this is the full-width model cut after layer 2) within FWD_RTOL like every other forward test,
and all 32 layers within DEEP_RTOL.  The two sides sum each GEMV row in a different fp32 order
(~1e-7 relative), which now and then moves an fp16 activation by one ulp; a random-weight
network amplifies such perturbations with depth, so the 32-layer logits differ by a few 1e-3
of the largest logit (measured) although every op matches to 1e-4 at these shapes.  Every row's
argmax must still agree at both depths, and the depth series is printed in the run summary."""
import os

import numpy as np
import pytest

from oracle import ulb_oracle as orc

pytestmark = pytest.mark.gpu

FWD_RTOL = 2e-3  # as the other forward tests: fp16 activations / KV may round 1 ulp apart
DEEP_RTOL = 1e-2  # 32 layers of a random-weight model: the same roundings, amplified by depth


def _bench_model(spec, n_layer=None):
    import bench
    import vulkangguf as vg
    if n_layer is not None and n_layer != spec["n_layer"]:
        spec = dict(spec, n_layer=n_layer, name="%s-first%d" % (spec["name"], n_layer))
    path = bench.model_paths(spec, spec)[0]
    if not os.path.exists(path):
        tmp = path + ".part%d" % os.getpid()
        vg.write_synthetic_gguf(tmp, spec)
        os.replace(tmp, path)
    return path


def _forward_parity(ctx, path, vocab, label, rtol):
    from conftest import PARITY_LOG
    from test_gpu_model import GpuModel
    gm = GpuModel(ctx, path)
    try:
        kvg = gm.kv(1, 64)
        kvo = orc.KV(gm.om, 1, 64)
        toks = np.random.default_rng(9).integers(0, vocab, 32).astype(np.int32)
        g = gm.forward(kvg, toks, [0] * 32, range(32), 32, logits_mode=1)
        o = orc.forward(gm.om, kvo, toks, [0] * 32, list(range(32)), 32, logits_mode=1)
        r_pre = float(np.abs(g - o).max() / np.abs(o).max())
        top_pre = bool(g.argmax() == o.argmax())
        blk = np.random.default_rng(10).integers(0, vocab, 6).astype(np.int32)
        g = gm.forward(kvg, blk, [0] * 6, range(32, 38), 6)
        o = orc.forward(gm.om, kvo, blk, [0] * 6, list(range(32, 38)), 6)
        r_ver = float(np.abs(g - o).max() / np.abs(o).max())
        top_ver = bool((g.argmax(1) == o.argmax(1)).all())
        PARITY_LOG.append("%s: prefill logits rel. diff %.2e (argmax equal: %s), verify block %.2e (argmax equal "
                          "in all 6 rows: %s); bar %.0e" % (label, r_pre, top_pre, r_ver, top_ver, rtol))
        assert r_pre < rtol and r_ver < rtol, (r_pre, r_ver)
        assert top_pre and top_ver
        gm.U.lib().ulb_kv_free(kvg)
    finally:
        gm.close()


@pytest.mark.parametrize("n_layer", [2, 32])
def test_c2_7b_target_forward_matches_oracle(ctx, n_layer):
    import bench
    _forward_parity(ctx, _bench_model(bench.TARGET, n_layer), bench.TARGET["n_vocab"],
                    "config-2 7B-arch Q4_0 target, %d layers" % n_layer, FWD_RTOL if n_layer <= 8 else DEEP_RTOL)


@pytest.mark.parametrize("n_layer", [2, 32])
def test_c4_llama3_8b_target_forward_matches_oracle(ctx, n_layer):
    import bench
    _forward_parity(ctx, _bench_model(bench.C4_TARGET, n_layer), bench.C4_TARGET["n_vocab"],
                    "config-4 Llama-3-8B-arch Q4_K target, %d layers" % n_layer,
                    FWD_RTOL if n_layer <= 8 else DEEP_RTOL)
