"""Tensor parallelism (config 5) on two GPUs: one process per GPU, NCCL over NVLink.

Each rank keeps half of the target's heads and FFN features (the draft is replicated); the
attn_output and ffn_down partial outputs are summed with an fp32 all-reduce inside every
forward, including the captured speculative round.  Checked against the CPU oracle's
unsharded model: last-position logits within the forward tolerance, greedy streams token for
token up to an oracle-flagged near-tie, and both ranks bitwise identical.  Skipped with fewer
than two GPUs."""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

from oracle import ulb_oracle as orc

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
FWD_RTOL = 2e-3
NEAR_TIE = 2e-3

CHILD = r'''
import json, os, sys
sys.path.insert(0, os.path.join(os.environ["ULB_ROOT"], "universal-loader_b200"))
import vulkangguf as vg
rank, world, idfile, tgt, drf, out = int(sys.argv[1]), int(sys.argv[2]), sys.argv[3], sys.argv[4], sys.argv[5], sys.argv[6]
nccl_id = open(idfile, "rb").read()
api = vg.InferenceAPI()
assert api.init_tensor_parallel(rank, world, nccl_id)
assert api.load_model(tgt) and api.load_draft_model(drf)
prompt = [int(x) for x in os.environ["ULB_PROMPT"].split(",")]
logits = api.get_token_logits(prompt)
api.enable_speculative_decoding(True)
api.set_speculation_length(3)
cfg = vg.GenerationConfig()
cfg.max_tokens, cfg.temperature, cfg.do_sample = 32, 0.0, False
toks = api.generate_tokens(prompt, cfg)
st = api.get_last_stats()
json.dump({"logits": logits, "tokens": toks, "rounds": st["rounds"]}, open(out, "w"))
'''


def _n_gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


# a LLaMA model whose per-rank slices at TP=2 are whole 128-weight Q4_0 tiles (the config-1
# target's FFN of 1408 splits into 704, which is not); the draft shares its first two blocks
TP_TARGET = dict(n_layer=4, d_model=512, n_head=8, n_head_kv=4, d_ff=1536, n_vocab=4096, rms_eps=1e-5,
                 rope_base=1e4, wtype="q4_0", seed=3, ctx_len=512)
TP_DRAFT = dict(TP_TARGET, n_layer=2)


@pytest.fixture(scope="module")
def tp_models(tmp_path_factory):
    import vulkangguf as vg
    d = tmp_path_factory.mktemp("tp_models")
    tgt, drf = str(d / "tp_target.gguf"), str(d / "tp_draft.gguf")
    vg.write_synthetic_gguf(tgt, dict(TP_TARGET, name="tp-target"))
    vg.write_synthetic_gguf(drf, dict(TP_DRAFT, name="tp-draft"))
    return tgt, drf


@pytest.mark.skipif(_n_gpus() < 2, reason="tensor parallelism needs two GPUs")
def test_tensor_parallel_two_ranks_match_oracle(tmp_path, tp_models):
    import ctypes as C
    import ulb_capi as U
    tiny_target, tiny_draft = tp_models
    idbuf = C.create_string_buffer(128)
    U.check(U.lib().ulb_tp_unique_id(idbuf))
    idfile = tmp_path / "nccl.id"
    idfile.write_bytes(idbuf.raw)
    prompt = np.random.default_rng(11).integers(0, TP_TARGET["n_vocab"], 70).astype(np.int32)
    procs = []
    for r in range(2):
        env = dict(os.environ, CUDA_VISIBLE_DEVICES=str(r), ULB_ROOT=ROOT, ULB_PROMPT=",".join(map(str, prompt)),
                   NCCL_DEBUG="WARN")
        procs.append(subprocess.Popen([sys.executable, "-c", CHILD, str(r), "2", str(idfile), tiny_target, tiny_draft,
                                       str(tmp_path / ("out%d.json" % r))], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.PIPE, text=True))
    try:
        for p in procs:
            _, err = p.communicate(timeout=300)
            assert p.returncode == 0, err[-3000:]
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
    res = [json.load(open(tmp_path / ("out%d.json" % r))) for r in range(2)]
    # both ranks hold the same residual stream: identical logits and tokens
    assert res[0]["logits"] == res[1]["logits"] and res[0]["tokens"] == res[1]["tokens"]
    t, d = orc.Model(tiny_target), orc.Model(tiny_draft)
    want_logits = orc.forward(t, orc.KV(t, 1, 70), prompt, [0] * 70, list(range(70)), 70, logits_mode=1)[0]
    got_logits = np.array(res[0]["logits"], np.float32)
    assert np.abs(got_logits - want_logits).max() / np.abs(want_logits).max() < FWD_RTOL
    want, _, _, _, tm = orc.spec_generate(t, d, [prompt], 32, 3, (0.0, 0, 1.0), seed=0, with_margins=True)
    got = res[0]["tokens"]
    assert len(got) == 32
    for i, (a, b) in enumerate(zip(got, want[0].tolist())):
        if a != b:
            assert tm[0][i] < NEAR_TIE, "first mismatch at %d with oracle margin %.3g" % (i, tm[0][i])
            break
