"""Whole-model GPU parity against the CPU oracle at the benchmark configurations' target shapes.

The op-level tests cover every kernel at these shapes; these run the models themselves, from
the same synthetic GGUF files bench.py decodes (written once per machine into the bench's
model cache):
  - config 2's Llama-2-7B-architecture Q4_0 target (32 layers, d 4096, 32 heads of 128, FFN
    11008, vocabulary 32000, RoPE theta 1e4);
  - config 4's Llama-3-8B-architecture Q4_K target (32 layers, GQA 32 / 8 heads, FFN 14336,
    vocabulary 128256, RoPE theta 5e5).
Each gets a 32-token prefill (last-row logits) and then one 6-row verify block (every row's
logits), on the GPU through the C ABI and on the oracle with identical inputs: logits within
FWD_RTOL of the largest oracle logit, the same argmax in every row."""
import os

import numpy as np
import pytest

from oracle import ulb_oracle as orc

pytestmark = pytest.mark.gpu

FWD_RTOL = 2e-3  # as the other forward tests: fp16 activations / KV may round 1 ulp apart


def _bench_model(spec):
    import bench
    import vulkangguf as vg
    path = bench.model_paths(spec, spec)[0]
    if not os.path.exists(path):
        tmp = path + ".part%d" % os.getpid()
        vg.write_synthetic_gguf(tmp, spec)
        os.replace(tmp, path)
    return path


def _forward_parity(ctx, path, vocab, label):
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
        assert r_pre < FWD_RTOL, r_pre
        assert g.argmax() == o.argmax()
        blk = np.random.default_rng(10).integers(0, vocab, 6).astype(np.int32)
        g = gm.forward(kvg, blk, [0] * 6, range(32, 38), 6)
        o = orc.forward(gm.om, kvo, blk, [0] * 6, list(range(32, 38)), 6)
        r_ver = float(np.abs(g - o).max() / np.abs(o).max())
        PARITY_LOG.append("%s: prefill logits rel. diff %.2e, verify block %.2e, argmax equal in all 6 rows: %s"
                          % (label, r_pre, r_ver, bool((g.argmax(1) == o.argmax(1)).all())))
        assert r_ver < FWD_RTOL, r_ver
        assert (g.argmax(1) == o.argmax(1)).all()
        gm.U.lib().ulb_kv_free(kvg)
    finally:
        gm.close()


def test_c2_7b_target_forward_matches_oracle(ctx):
    import bench
    _forward_parity(ctx, _bench_model(bench.TARGET), bench.TARGET["n_vocab"], "config-2 7B-arch Q4_0 target")


def test_c4_llama3_8b_target_forward_matches_oracle(ctx):
    import bench
    _forward_parity(ctx, _bench_model(bench.C4_TARGET), bench.C4_TARGET["n_vocab"],
                    "config-4 Llama-3-8B-arch Q4_K target")
