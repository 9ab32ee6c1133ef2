"""Shared fixtures.  GPU tests are marked `gpu`; everything else runs on the CPU."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "universal-loader_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

# The tiny speculative pair of the CPU-runnable configuration: LLaMA d=512, 8 heads (hd 64),
# SwiGLU 1408, vocab 32000, eps 1e-5, theta 1e4; target 8 layers, draft 2 layers, both from
# seed 0 so the draft shares the target's first two blocks, embeddings and head.
TINY_TARGET = dict(n_layer=8, d_model=512, n_head=8, n_head_kv=8, d_ff=1408, n_vocab=32000,
                   rms_eps=1e-5, rope_base=1e4, wtype="q4_0", seed=0, name="tiny-target")
TINY_DRAFT = dict(TINY_TARGET, n_layer=2, name="tiny-draft")
# a draft sharing the target's first 7 of 8 blocks: one that agrees with the target often
# enough for whole tree paths to be accepted
TINY_NEAR_DRAFT = dict(TINY_TARGET, n_layer=7, name="tiny-near-draft")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


# One line per greedy-stream comparison (matched length, where and why a stream stopped
# matching), printed at the end of the run so a passing run still shows the evidence.
PARITY_LOG = []


def pytest_terminal_summary(terminalreporter):
    if PARITY_LOG:
        terminalreporter.write_sep("-", "greedy stream parity against the oracle")
        for line in PARITY_LOG:
            terminalreporter.write_line(line)


def _build():
    from oracle import build as obuild
    obuild.build()
    sys.path.insert(0, PKG)
    import build as pbuild  # universal-loader_b200/build.py
    pbuild.build()


@pytest.fixture(scope="session", autouse=True)
def built():
    _build()
    return True


@pytest.fixture(scope="session")
def model_dir(tmp_path_factory):
    return tmp_path_factory.mktemp("models")


def _synth(model_dir, spec, name):
    import vulkangguf as vg
    path = os.path.join(str(model_dir), name)
    if not os.path.exists(path):
        vg.write_synthetic_gguf(path, spec)
    return path


@pytest.fixture(scope="session")
def tiny_target(model_dir):
    return _synth(model_dir, TINY_TARGET, "tiny_target.gguf")


@pytest.fixture(scope="session")
def tiny_draft(model_dir):
    return _synth(model_dir, TINY_DRAFT, "tiny_draft.gguf")


@pytest.fixture(scope="session")
def q4km_mix(model_dir):
    """The tensor mix of llama.cpp's Q4_K_M files: Q4_K linears with Q6_K attn_v and ffn_down (and
    here a Q8_0 attn_output), a Q6_K output.weight; GQA."""
    spec = dict(n_layer=2, d_model=512, n_head=8, n_head_kv=2, d_ff=1536, n_vocab=4096, rms_eps=1e-5,
                rope_base=5e5, wtype="q4_k", embd_type="q4_k", out_type="q6_k", v_type="q6_k", o_type="q8_0",
                down_type="q6_k", seed=13, name="q4km-mix")
    return _synth(model_dir, spec, "q4km_mix.gguf")


@pytest.fixture(scope="session")
def near_draft(model_dir):
    return _synth(model_dir, TINY_NEAR_DRAFT, "tiny_near_draft.gguf")


@pytest.fixture(scope="session")
def tiny_gqa_q4k(model_dir):
    spec = dict(n_layer=3, d_model=512, n_head=8, n_head_kv=2, d_ff=1536, n_vocab=4096,
                rms_eps=1e-5, rope_base=5e5, wtype="q4_k", seed=3, name="tiny-gqa-q4k")
    return _synth(model_dir, spec, "tiny_gqa_q4k.gguf")


@pytest.fixture(scope="session")
def mid_q40(model_dir):
    """Large enough that every GEMV spans all SMs (d = 1024, FFN 2816, 2 layers)."""
    spec = dict(n_layer=2, d_model=1024, n_head=8, n_head_kv=8, d_ff=2816, n_vocab=4096,
                rms_eps=1e-5, rope_base=1e4, wtype="q4_0", seed=5, name="mid-q40")
    return _synth(model_dir, spec, "mid_q40.gguf")


@pytest.fixture(scope="session")
def llamacpp_q40(model_dir):
    """The tensor types of llama.cpp's Q4_0 files: Q4_0 token_embd and linears, Q6_K output."""
    spec = dict(n_layer=2, d_model=512, n_head=8, n_head_kv=8, d_ff=1408, n_vocab=4096, rms_eps=1e-5,
                rope_base=1e4, wtype="q4_0", embd_type="q4_0", out_type="q6_k", seed=11, name="llamacpp-q40")
    return _synth(model_dir, spec, "llamacpp_q40.gguf")


@pytest.fixture(scope="session")
def q6k_embd_q80_head(model_dir):
    """Q6_K token_embd and a Q8_0 output.weight over Q4_K linears (GQA)."""
    spec = dict(n_layer=2, d_model=512, n_head=8, n_head_kv=2, d_ff=1536, n_vocab=4096, rms_eps=1e-5,
                rope_base=5e5, wtype="q4_k", embd_type="q6_k", out_type="q8_0", seed=12, name="q6k-embd-q80-head")
    return _synth(model_dir, spec, "q6k_embd_q80_head.gguf")


def has_gpu():
    try:
        import ulb_capi
        ctx = ulb_capi.Context(0)
        ctx.close()
        return True
    except Exception:
        return False


@pytest.fixture(scope="session")
def ctx():
    import ulb_capi
    c = ulb_capi.Context(0)
    yield c
    c.close()
