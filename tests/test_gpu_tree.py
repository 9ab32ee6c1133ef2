"""Tree speculation on the GPU against the CPU oracle.

The acceptance kernel (ulb_spec_tree_accept) must take the oracle's decisions and tokens given
the same logits and Philox uniforms, and keep the target distribution (chi-square on the first
committed token).  The whole tree loop (draft levels with tree attention, one verify over every
node, multi-candidate acceptance, the KV cache compaction of the accepted path) at T = 0 must
commit the target's greedy stream: the oracle's greedy stream, token for token up to a near-tie
of the oracle's own logits (the rule of test_gpu_model.py)."""
import ctypes as C

import numpy as np
import pytest

from oracle import ulb_oracle as orc
from test_gpu_model import _api, _cfg, _match_greedy, _prompt
from test_oracle import _tree_inputs

pytestmark = pytest.mark.gpu


def _tree_accept_gpu(ctx, pl, ql, tok, w, D, warp, seed, rnd):
    import ulb_capi as U
    B, V = tok.shape[0], pl.shape[-1]
    bufs = [ctx.buffer(np.ascontiguousarray(a)) for a in (pl, ql, tok)]
    bp, bn, bt = ctx.buffer(nbytes=B * D * 4), ctx.buffer(nbytes=B * 4), ctx.buffer(nbytes=B * 4)
    wp = U.Warp(*warp)
    U.check(U.lib().ulb_spec_tree_accept(ctx.h, bufs[0].ptr, bufs[1].ptr, bufs[2].ptr, B, w, D, V, C.byref(wp), seed,
                                         rnd, bp.ptr, bn.ptr, bt.ptr))
    path, n, t = bp.download(np.int32, (B, D)), bn.download(np.int32, (B,)), bt.download(np.int32, (B,))
    for b in bufs + [bp, bn, bt]:
        b.free()
    return path, n, t


@pytest.mark.parametrize("w,D", [(2, 3), (3, 2), (4, 2)])
@pytest.mark.parametrize("warp", [(0.0, 0, 1.0), (1.0, 0, 1.0), (0.8, 40, 1.0), (0.8, 0, 0.9)])
def test_tree_accept_matches_oracle(ctx, w, D, warp):
    """Same logits and uniforms: the same accepted nodes, counts and correction / bonus tokens."""
    rng = np.random.default_rng(31 + w * 7 + D)
    B, V = 24, 32000
    pl, ql, tok = _tree_inputs(rng, B, w, D, V, warp, seed=4, rnd=2)
    got = _tree_accept_gpu(ctx, pl, ql, tok, w, D, warp, 4, 2)
    want = orc.tree_accept(pl, ql, tok, w, D, warp, 4, 2)
    assert got[1].tolist() == want[1].tolist()
    assert got[0].tolist() == want[0].tolist()
    assert got[2].tolist() == want[2].tolist()
    assert want[1].max() > 0 and want[1].min() < D  # accept and reject paths both taken


def test_tree_accept_is_lossless_chi2(ctx):
    """Three children drawn on the GPU from q at the root (ulb_sample, slot = child node): the
    first committed token of the round is distributed as p."""
    import ulb_capi as U
    B, V, w = 6000, 6, 3
    rng = np.random.default_rng(8)
    p1 = (rng.standard_normal(V) * 1.5).astype(np.float32)
    q1 = (rng.standard_normal(V) * 1.5).astype(np.float32)
    pl = np.broadcast_to(p1, (B, 1 + w, V)).copy()
    ql = np.broadcast_to(q1, (B, 1, V)).copy()
    qb = ctx.buffer(ql)
    tok = np.zeros((B, w), np.int32)
    wp = U.Warp(1.0, 0, 1.0)
    for c in range(w):
        db = ctx.buffer(nbytes=B * 4)
        U.check(U.lib().ulb_sample(ctx.h, qb.ptr, B, V, V, C.byref(wp), 13, 0, c, U.RNG_DRAFT, db.ptr))
        tok[:, c] = db.download(np.int32, (B,))
        db.free()
    qb.free()
    path, n, t = _tree_accept_gpu(ctx, pl, ql, tok, w, 1, (1.0, 0, 1.0), 13, 0)
    first = np.where(n > 0, tok[np.arange(B), np.maximum(path[:, 0], 0)], t)
    p = orc.warp_probs(p1, 1.0)
    counts = np.bincount(first, minlength=V)
    chi2 = ((counts - p * B) ** 2 / (p * B)).sum()
    assert chi2 < 25.0, (chi2, counts, p * B)  # 5 dof: p-value ~ 1e-4


def _tree_api(target, draft, w, D):
    api = _api(target, draft, k=D)
    api.enable_tree_speculation(w, D)
    return api


@pytest.mark.parametrize("w,D", [(2, 3), (3, 2)])
def test_tree_spec_greedy_stream_matches_oracle(tiny_target, near_draft, w, D):
    """The tree loop at T = 0 commits the target's greedy stream (config-1 shapes, a draft
    sharing 7 of the target's 8 blocks), accepting drafts at several levels of the tree."""
    prompt = _prompt(128, seed=1)
    api = _tree_api(tiny_target, near_draft, w, D)
    got = api.generate_tokens(prompt.tolist(), _cfg(96))
    st = api.get_last_stats()
    t, d = orc.Model(tiny_target), orc.Model(near_draft)
    want, _, _, _, tm = orc.spec_generate(t, d, [prompt], 96, 4, (0.0, 0, 1.0), seed=0, with_margins=True)
    assert len(got) == 96
    _match_greedy(got, want[0], tm[0], "tree speculation w=%d D=%d greedy stream (96 tokens)" % (w, D))
    assert st["accepted"] > 0 and st["rounds"] < 96
    rounds = api.get_speculation_results(0)
    assert len(rounds) == st["rounds"]
    assert sum(r.num_accepted for r in rounds) == st["committed"]


@pytest.mark.parametrize("temperature", [0.0, 0.8])
def test_tree_spec_self_draft_accepts_whole_paths(tiny_target, temperature):
    """Draft = target: p = q at every node, so every round accepts a whole root-to-leaf path
    through the first children plus the leaf's bonus token (depth + 1 tokens a round), and the
    cache compaction moves those nodes into place; at T = 0 the stream is the oracle's greedy
    stream."""
    prompt = _prompt(64, seed=2)
    w, D, n = 2, 3, 48
    api = _tree_api(tiny_target, tiny_target, w, D)
    got = api.generate_tokens(prompt.tolist(), _cfg(n, temperature, 0, 1.0, seed=3))
    st = api.get_last_stats()
    assert st["accepted"] == st["drafted"] and st["rounds"] == (n - 1 + D) // (D + 1)
    if temperature == 0.0:
        t = orc.Model(tiny_target)
        want, _, _, _, tm = orc.spec_generate(t, t, [prompt], n, 3, (0.0, 0, 1.0), seed=0, with_margins=True)
        _match_greedy(got, want[0], tm[0], "tree speculation, draft = target (48 tokens)")


def test_tree_spec_accepts_more_than_the_chain(tiny_target, near_draft):
    """Same depth, greedy: the tree's extra candidates accept drafts where the chain of first
    candidates does not, so the same greedy stream takes fewer rounds."""
    prompt = _prompt(128, seed=1)
    chain = _api(tiny_target, near_draft, k=3)
    a = chain.generate_tokens(prompt.tolist(), _cfg(64))
    sc = chain.get_last_stats()
    tree = _tree_api(tiny_target, near_draft, 2, 3)
    b = tree.generate_tokens(prompt.tolist(), _cfg(64))
    stt = tree.get_last_stats()
    n = min(len(a), len(b))
    first = next((i for i in range(n) if a[i] != b[i]), n)
    assert first >= 32  # both are the greedy stream (up to a near-tie of the two verify shapes)
    assert stt["accepted"] > sc["accepted"] and stt["rounds"] < sc["rounds"]


def test_tree_spec_sampled_seeded(tiny_target, near_draft):
    """T = 0.8, top_k = 40 through the tree loop: a pure function of the Philox seed, with real
    acceptance."""
    prompt = _prompt(128, seed=1)
    api = _tree_api(tiny_target, near_draft, 2, 3)
    a = api.generate_tokens(prompt.tolist(), _cfg(96, 0.8, 40, 1.0, seed=0))
    st = api.get_last_stats()
    b = api.generate_tokens(prompt.tolist(), _cfg(96, 0.8, 40, 1.0, seed=0))
    c = api.generate_tokens(prompt.tolist(), _cfg(96, 0.8, 40, 1.0, seed=1))
    assert a == b and a != c and len(a) == 96
    assert 0 < st["accepted"] < st["drafted"]
    assert 95 <= st["committed"] <= 95 + 3


def test_tree_spec_batch_and_continuous_batching(tiny_target, near_draft):
    """Three ragged prompts, two slots (continuous batching, paged caches): each stream is the
    greedy stream of its prompt."""
    prompts = [_prompt(n, seed=40 + n) for n in (23, 70, 41)]
    api = _tree_api(tiny_target, near_draft, 2, 2)
    api.set_max_batch_size(2)
    got = api.generate_tokens([p.tolist() for p in prompts], _cfg(40))
    st = api.get_last_stats()
    t, d = orc.Model(tiny_target), orc.Model(near_draft)
    want, _, _, _, tm = orc.spec_generate(t, d, prompts, 40, 3, (0.0, 0, 1.0), seed=5, with_margins=True)
    for i, (g, w_, m) in enumerate(zip(got, want, tm)):
        _match_greedy(g, w_, m, "tree speculation, continuous batching, prompt %d" % i)
    assert st["admitted"] >= 1 and st["accepted"] > 0
