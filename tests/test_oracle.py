"""CPU tests of the oracle: pinned against the GGUF format oracle (the `gguf` package),
published Philox4x32-10 known-answer vectors, hand-built blocks and mathematical known
answers.  The oracle is the checker of the CUDA path, so it is checked first."""
import numpy as np
import pytest

import gguf
from oracle import ulb_oracle as orc


# ---------------------------------------------------------------- Philox4x32-10
# Known-answer vectors of the Random123 distribution (kat_vectors, philox4x32_10).
PHILOX_KAT = [
    ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
    ((0xFFFFFFFF,) * 4, (0xFFFFFFFF,) * 2, (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
    ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
     (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
]


@pytest.mark.parametrize("ctr,key,want", PHILOX_KAT)
def test_philox_known_answers(ctr, key, want):
    assert tuple(int(x) for x in orc.philox(ctr, key)) == want


def _philox_py(ctr, key):
    """independent pure-Python restatement for cross-checking random counters"""
    c = list(ctr)
    k = list(key)
    for _ in range(10):
        p0 = 0xD2511F53 * c[0]
        p1 = 0xCD9E8D57 * c[2]
        c = [((p1 >> 32) ^ c[1] ^ k[0]) & 0xFFFFFFFF, p1 & 0xFFFFFFFF,
             ((p0 >> 32) ^ c[3] ^ k[1]) & 0xFFFFFFFF, p0 & 0xFFFFFFFF]
        k = [(k[0] + 0x9E3779B9) & 0xFFFFFFFF, (k[1] + 0xBB67AE85) & 0xFFFFFFFF]
    return tuple(c)


def test_philox_random_counters():
    rng = np.random.default_rng(7)
    for _ in range(200):
        ctr = tuple(int(x) for x in rng.integers(0, 2**32, 4))
        key = tuple(int(x) for x in rng.integers(0, 2**32, 2))
        assert tuple(int(x) for x in orc.philox(ctr, key)) == _philox_py(ctr, key)


def test_uniform_is_top24_bits():
    seed = 0x1234_5678_9ABC_DEF0
    o = _philox_py((3, 1, 2, 2), (seed & 0xFFFFFFFF, seed >> 32))
    assert orc.uniform(seed, 3, 1, 2, 2) == (o[0] >> 8) / 16777216.0


# ---------------------------------------------------------------- block formats
def _q4_0_block(d_bits, nibbles):
    """hand-built GGUF Q4_0 block: fp16 d then 16 bytes (low nibble = w[j], high = w[j+16])"""
    b = np.zeros(18, np.uint8)
    b[0:2] = np.frombuffer(np.uint16(d_bits).tobytes(), np.uint8)
    for j in range(16):
        b[2 + j] = nibbles[j] | (nibbles[j + 16] << 4)
    return b


def test_q4_0_hand_built_block():
    nib = np.arange(32) % 16
    blk = _q4_0_block(0x3C00, nib)  # d = 1.0
    out = orc.dequant(orc.T_Q4_0, blk, 32)
    np.testing.assert_array_equal(out, (nib - 8).astype(np.float32))
    ref = gguf.quants.dequantize(blk.reshape(1, 18), gguf.GGMLQuantizationType.Q4_0).ravel()
    np.testing.assert_array_equal(out, ref)


def test_q4_0_subnormal_and_negative_scale():
    nib = (np.arange(32) * 7) % 16
    for d_bits in (0x0001, 0x03FF, 0x8001, 0xBC00, 0x7BFF):  # subnormals, -1, max
        blk = _q4_0_block(d_bits, nib)
        out = orc.dequant(orc.T_Q4_0, blk, 32)
        ref = gguf.quants.dequantize(blk.reshape(1, 18), gguf.GGMLQuantizationType.Q4_0).ravel()
        assert np.array_equal(out.view(np.uint32), ref.view(np.uint32)), hex(d_bits)


def _random_q4k_blocks(n, seed):
    rng = np.random.default_rng(seed)
    b = rng.integers(0, 256, (n, 144), dtype=np.uint8)
    # finite, mixed-sign fp16 d / dmin including subnormals
    d = rng.choice(np.array([0x3C00, 0x2E66, 0x0001, 0x03FF, 0x1800, 0xB400], np.uint16), n)
    dm = rng.choice(np.array([0x3800, 0x2A00, 0x0002, 0x0000, 0x1C00], np.uint16), n)
    b[:, 0:2] = d.view(np.uint8).reshape(n, 2)
    b[:, 2:4] = dm.view(np.uint8).reshape(n, 2)
    return b


def test_q4_k_decode_matches_gguf_bit_exact():
    blocks = _random_q4k_blocks(64, 11)
    out = orc.dequant(orc.T_Q4_K, blocks, 64 * 256)
    ref = gguf.quants.dequantize(blocks, gguf.GGMLQuantizationType.Q4_K).ravel()
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))


def test_q4_k_scale_min_corner_cases():
    # all 6-bit scale / min bits set, d = dmin = 1: sc = m = 63 for every sub-block
    b = np.zeros((1, 144), np.uint8)
    b[0, 0:2] = np.frombuffer(np.float16(1.0).tobytes(), np.uint8)
    b[0, 2:4] = np.frombuffer(np.float16(1.0).tobytes(), np.uint8)
    b[0, 4:16] = 0xFF
    b[0, 16:] = 0x5F  # low nibble 15, high nibble 5
    out = orc.dequant(orc.T_Q4_K, b, 256)
    ref = gguf.quants.dequantize(b, gguf.GGMLQuantizationType.Q4_K).ravel()
    np.testing.assert_array_equal(out, ref)
    assert set(np.unique(out)) == {63 * 15 - 63.0, 63 * 5 - 63.0}


def test_q4_0_random_tensor_bit_exact():
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((64, 256)) * 0.02).astype(np.float32)
    q = gguf.quants.quantize(x, gguf.GGMLQuantizationType.Q4_0)
    out = orc.dequant(orc.T_Q4_0, q, x.size)
    ref = gguf.quants.dequantize(q, gguf.GGMLQuantizationType.Q4_0).ravel()
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))


def test_oracle_quantizer_matches_gguf():
    rng = np.random.default_rng(9)
    x = (rng.standard_normal((16, 512)) * 0.02).astype(np.float32)
    x[0, :32] = 0.0  # all-zero block
    q = gguf.quants.quantize(x, gguf.GGMLQuantizationType.Q4_0).ravel()
    assert np.array_equal(orc.quantize_q4_0(x), q)


# ---------------------------------------------------------------- Q8_0 / Q6_K (llama.cpp's token_embd / output.weight types)
def _random_q6k_blocks(n, seed):
    rng = np.random.default_rng(seed)
    b = rng.integers(0, 256, (n, 210), dtype=np.uint8)  # any ql / qh / int8 scales
    d = rng.choice(np.array([0x1C00, 0x2E66, 0x0001, 0x9800, 0x03FF], np.uint16), n)
    b[:, 208:210] = d.view(np.uint8).reshape(n, 2)
    return b


def test_q8_0_decode_matches_gguf_bit_exact():
    rng = np.random.default_rng(21)
    x = (rng.standard_normal((32, 256)) * 0.02).astype(np.float32)
    q = gguf.quants.quantize(x, gguf.GGMLQuantizationType.Q8_0)
    out = orc.dequant(orc.T_Q8_0, q, x.size)
    ref = gguf.quants.dequantize(q, gguf.GGMLQuantizationType.Q8_0).ravel()
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))


def test_q6_k_decode_matches_gguf_bit_exact():
    blocks = _random_q6k_blocks(48, 22)
    out = orc.dequant(orc.T_Q6_K, blocks, 48 * 256)
    ref = gguf.quants.dequantize(blocks, gguf.GGMLQuantizationType.Q6_K).ravel()
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))


QERR = {"q4_0": 0.13, "q8_0": 0.006, "q6_k": 0.04}  # max |dequant - value| / max |value| (Q4_0: up to d = amax / 8)


@pytest.mark.parametrize("embd,out", [("q4_0", "q6_k"), ("q6_k", "q8_0"), ("q8_0", "q6_k")])
def test_synthetic_embd_and_head_types(tmp_path, embd, out):
    """The synthetic writer's Q4_0 / Q8_0 / Q6_K token_embd and output.weight (the engine's
    quantisers) decode identically through the oracle and the gguf package, and stay within
    the format's quantisation error of the same seeded values written as F32 / F16."""
    import vulkangguf as vg
    base = dict(n_layer=1, d_model=256, n_head=4, n_head_kv=4, d_ff=512, n_vocab=512, wtype="q4_0", seed=7)
    pq, pf = str(tmp_path / "q.gguf"), str(tmp_path / "f.gguf")
    vg.write_synthetic_gguf(pq, dict(base, embd_type=embd, out_type=out))
    vg.write_synthetic_gguf(pf, dict(base, embd_type="f32"))
    mq, mf = orc.Model(pq), orc.Model(pf)
    gt = {"q4_0": gguf.GGMLQuantizationType.Q4_0, "q8_0": gguf.GGMLQuantizationType.Q8_0,
          "q6_k": gguf.GGMLQuantizationType.Q6_K}
    for name, ty in (("token_embd.weight", embd), ("output.weight", out)):
        t, ne, raw = mq.tensor(name)
        n = ne[0] * ne[1]
        mine = orc.dequant(t, raw, n)
        ref = gguf.quants.dequantize(raw.reshape(ne[1], -1), gt[ty]).ravel()
        assert np.array_equal(mine.view(np.uint32), ref.view(np.uint32)), name
        if name == "token_embd.weight":
            tf, nef, rawf = mf.tensor(name)
            vals = orc.dequant(tf, rawf, n)
            assert np.abs(mine - vals).max() / np.abs(vals).max() < QERR[ty], name
    mq.close()
    mf.close()


def test_synthetic_linear_type_mix(tmp_path):
    """v_type / o_type / down_type write attn_v / attn_output / ffn_down of every layer in their
    own types (llama.cpp's Q4_K_M mix), decoding through the oracle as through the gguf package."""
    import vulkangguf as vg
    p = str(tmp_path / "mix.gguf")
    vg.write_synthetic_gguf(p, dict(n_layer=2, d_model=512, n_head=8, n_head_kv=2, d_ff=1536, n_vocab=512,
                                    wtype="q4_k", v_type="q6_k", o_type="q8_0", down_type="q6_k", seed=9))
    m = orc.Model(p)
    gt = {orc.T_Q4_K: gguf.GGMLQuantizationType.Q4_K, 8: gguf.GGMLQuantizationType.Q8_0,
          14: gguf.GGMLQuantizationType.Q6_K}
    want = {"attn_q": orc.T_Q4_K, "attn_v": 14, "attn_output": 8, "ffn_gate": orc.T_Q4_K, "ffn_down": 14}
    for l in range(2):
        for nm, ty in want.items():
            t, ne, raw = m.tensor("blk.%d.%s.weight" % (l, nm))
            assert t == ty, (nm, t)
            mine = orc.dequant(t, raw, ne[0] * ne[1])
            ref = gguf.quants.dequantize(raw.reshape(ne[1], -1), gt[t]).ravel()
            assert np.array_equal(mine.view(np.uint32), ref.view(np.uint32)), nm
    m.close()


# ---------------------------------------------------------------- GEMV structure
@pytest.mark.parametrize("qt", ["q4_0", "q4_k", "q8_0", "q6_k"])
@pytest.mark.parametrize("M", [1, 5, 8])
def test_qgemv_matches_float64_dot(qt, M):
    rng = np.random.default_rng(M)
    N, K = 48, 512
    if qt in ("q4_0", "q8_0"):
        gq = gguf.GGMLQuantizationType.Q4_0 if qt == "q4_0" else gguf.GGMLQuantizationType.Q8_0
        t = orc.T_Q4_0 if qt == "q4_0" else orc.T_Q8_0
        w = gguf.quants.quantize((rng.standard_normal((N, K)) * 0.02).astype(np.float32), gq)
        wf = gguf.quants.dequantize(w, gq).reshape(N, K)
    elif qt == "q6_k":
        t = orc.T_Q6_K
        w = _random_q6k_blocks(N * K // 256, M)
        wf = gguf.quants.dequantize(w, gguf.GGMLQuantizationType.Q6_K).reshape(N, K)
    else:
        t = orc.T_Q4_K
        w = _random_q4k_blocks(N * K // 256, M)
        wf = gguf.quants.dequantize(w, gguf.GGMLQuantizationType.Q4_K).reshape(N, K)
    x = rng.standard_normal((M, K)).astype(np.float16)
    y = orc.qgemv(t, w, N, K, x)
    ref = x.astype(np.float64) @ wf.astype(np.float64).T
    rel = np.abs(y - ref).max() / np.abs(ref).max()
    assert rel < 1e-5, rel


# ---------------------------------------------------------------- warp-weight exponential
def test_warp_exp_accuracy_and_range():
    """orc_warp_exp (Cody-Waite reduction + degree-7 Taylor) is within a few ulp of exp."""
    rng = np.random.default_rng(3)
    xs = np.concatenate([-rng.random(40000) * 87.0, -rng.random(2000) * 1e-3,
                         np.array([0.0, -1e-30, -0.34657359, -0.34657360, -86.99999])]).astype(np.float32)
    got = np.array([orc.warp_exp(x) for x in xs], np.float64)
    want = np.exp(xs.astype(np.float64))
    assert np.max(np.abs(got - want) / want) < 4e-7
    assert orc.warp_exp(0.0) == 1.0
    assert orc.warp_exp(-87.5) == 0.0 and orc.warp_exp(float("-inf")) == 0.0


def test_warp_exp_header_matches_oracle(tmp_path):
    """The device header's ulb_warp_exp, compiled for the host, is bit-identical to the
    oracle's restatement (the device build compiles the same source with __fmaf_rn /
    __fmul_rn / rintf, which are the same IEEE operations)."""
    import ctypes as C
    import os
    import subprocess
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    src = tmp_path / "hx.c"
    src.write_text('#include "ulb_common.h"\nfloat hx(float x) { return ulb_warp_exp(x); }\n')
    so = tmp_path / "hx.so"
    subprocess.run(["gcc", "-O2", "-ffp-contract=off", "-fPIC", "-shared", "-I",
                    os.path.join(root, "universal-loader_b200", "csrc"), "-o", str(so), str(src), "-lm"], check=True)
    lib = C.CDLL(str(so))
    lib.hx.restype = C.c_float
    lib.hx.argtypes = [C.c_float]
    rng = np.random.default_rng(5)
    xs = (-rng.random(30000) * 90.0).astype(np.float32)
    for x in xs:
        a, b = np.float32(lib.hx(x)), np.float32(orc.warp_exp(x))
        assert a.view(np.uint32) == b.view(np.uint32), (float(x), float(a), float(b))


# ---------------------------------------------------------------- sampling known answers
def test_warp_probs_greedy_and_topk():
    logits = np.array([0.5, 3.0, -1.0, 3.0, 2.0], np.float32)
    p = orc.warp_probs(logits, temperature=0.0)
    np.testing.assert_array_equal(p, [0, 1, 0, 0, 0])  # lowest index on ties
    p = orc.warp_probs(logits, temperature=1.0, top_k=2)
    assert p[1] == p[3] and p[0] == p[2] == p[4] == 0 and abs(p.sum() - 1) < 1e-15
    p = orc.warp_probs(logits, temperature=1.0, top_k=3)
    assert (p > 0).sum() == 3 and p[4] > 0


def test_warp_probs_top_p():
    logits = np.log(np.array([0.5, 0.3, 0.15, 0.05], np.float64)).astype(np.float32)
    p = orc.warp_probs(logits, temperature=1.0, top_p=0.7)  # keeps 0.5 and 0.3
    assert (p > 0).tolist() == [True, True, False, False]
    p = orc.warp_probs(logits, temperature=1.0, top_p=0.5)  # first token alone reaches 0.5
    assert (p > 0).tolist() == [True, False, False, False]


def test_accept_p_equals_q_accepts_all():
    rng = np.random.default_rng(0)
    B, k, V = 3, 4, 64
    pl = rng.standard_normal((B, k + 1, V)).astype(np.float32)
    ql = pl[:, :k].copy()
    draft = rng.integers(0, V, (B, k)).astype(np.int32)
    out, n = orc.spec_accept(pl, ql, draft, (1.0, 0, 1.0), seed=1, rnd=0)
    assert (n == k).all()
    assert (out[:, :k] == draft).all()


def test_accept_one_hot_rejects_at_first():
    B, k, V = 2, 3, 16
    pl = np.full((B, k + 1, V), -30.0, np.float32)
    pl[:, :, 7] = 30.0  # target puts all mass on token 7
    ql = np.zeros((B, k, V), np.float32)
    draft = np.full((B, k), 3, np.int32)
    out, n = orc.spec_accept(pl, ql, draft, (1.0, 0, 1.0), seed=5, rnd=2)
    assert (n == 0).all() and (out[:, 0] == 7).all()


def test_accept_greedy_rules():
    B, k, V = 1, 4, 10
    pl = np.zeros((B, k + 1, V), np.float32)
    am = [2, 5, 5, 1, 9]
    for i, a in enumerate(am):
        pl[0, i, a] = 1.0
    draft = np.array([[2, 5, 4, 1]], np.int32)
    out, n = orc.spec_accept(pl, np.zeros((B, k, V), np.float32), draft, (0.0, 0, 1.0), 0, 0)
    assert n[0] == 2 and out[0, :3].tolist() == [2, 5, 5]
    draft = np.array([[2, 5, 5, 1]], np.int32)
    out, n = orc.spec_accept(pl, np.zeros((B, k, V), np.float32), draft, (0.0, 0, 1.0), 0, 0)
    assert n[0] == 4 and out[0].tolist() == [2, 5, 5, 1, 9]


def test_spec_sampling_is_lossless_chi2():
    """The committed first token of a round is distributed as p (Leviathan et al. 2023)."""
    V = 6
    rng = np.random.default_rng(3)
    p_log = rng.standard_normal(V).astype(np.float32) * 1.5
    q_log = rng.standard_normal(V).astype(np.float32) * 1.5
    p = orc.warp_probs(p_log, 1.0)
    q = orc.warp_probs(q_log, 1.0)
    n_trials = 6000
    counts = np.zeros(V)
    pl = np.broadcast_to(p_log, (1, 2, V)).copy()
    ql = q_log.reshape(1, 1, V)
    for r in range(n_trials):
        x = orc.sample(q_log, orc.uniform(11, r, 0, 0, 1), 1.0)
        out, n = orc.spec_accept(pl, ql, np.array([[x]], np.int32), (1.0, 0, 1.0), 11, r)
        counts[out[0, 0]] += 1
    exp = p * n_trials
    chi2 = ((counts - exp) ** 2 / exp).sum()
    assert chi2 < 25.0, (chi2, counts, exp)  # 5 dof, p ~ 1e-4
    assert not np.allclose(p, q)


# ---------------------------------------------------------------- speculation trees (oracle)
def _tree_inputs(rng, B, w, D, V, warp, seed=4, rnd=2, agree=0.5):
    """p / q logits of every tree row and children drawn as the GPU loop draws them: the w
    most likely tokens (T = 0) or w independent draws from the warped q (slot = child node)."""
    N, NI = orc.tree_nodes(w, D), orc.tree_nodes(w, D - 1)
    pl = (rng.standard_normal((B, 1 + N, V)) * 2).astype(np.float32)
    ql = (rng.standard_normal((B, 1 + NI, V)) * 2).astype(np.float32)
    nb = int(B * agree)
    ql[:nb] = pl[:nb, :1 + NI] + 0.3 * ql[:nb]  # drafts that often agree with the target
    tok = np.zeros((B, N), np.int32)
    for b in range(B):
        for u in [-1] + list(range(NI)):
            ch = orc.tree_children(w, D, u)
            lq = ql[b, u + 1]
            if warp[0] <= 0:
                order = np.argsort(-lq, kind="stable")  # most likely first, lowest index on ties
                for c, t in zip(ch, order[:w]):
                    tok[b, c] = t
            else:
                for c in ch:
                    tok[b, c] = orc.sample(lq, orc.uniform(seed, rnd, b, c, 1), *warp)
    return pl, ql, tok


def test_tree_geometry():
    assert orc.tree_nodes(2, 3) == 14 and orc.tree_nodes(3, 2) == 12 and orc.tree_nodes(1, 5) == 5
    assert orc.tree_children(2, 3, -1) == [0, 1]
    assert orc.tree_children(2, 3, 1) == [4, 5]
    assert orc.tree_children(2, 3, 5) == [12, 13]
    assert orc.tree_children(2, 3, 6) == []  # depth-3 leaves


@pytest.mark.parametrize("warp", [(0.0, 0, 1.0), (1.0, 0, 1.0), (0.8, 40, 1.0)])
def test_tree_of_width_one_is_the_chain(warp):
    """A tree of width 1 is a chain of k drafts: the same decisions and tokens as orc_spec_accept
    given the same logits and uniforms."""
    rng = np.random.default_rng(21)
    B, D, V = 24, 4, 500
    pl, ql, tok = _tree_inputs(rng, B, 1, D, V, warp)
    path, n, t = orc.tree_accept(pl, ql, tok, 1, D, warp, 4, 2)
    out, n2 = orc.spec_accept(pl, ql, tok, warp, 4, 2)
    assert n.tolist() == n2.tolist()
    for b in range(B):
        assert path[b, :n[b]].tolist() == list(range(n[b]))
        assert t[b] == out[b, n[b]]
    assert n.max() > 0 and n.min() < D


def test_tree_greedy_walk_known_answers():
    """T = 0: the walk follows the child equal to the target's argmax; p == q accepts every level
    through the first children and ends with the bonus argmax of the leaf."""
    rng = np.random.default_rng(5)
    B, w, D, V = 6, 3, 3, 80
    pl, ql, tok = _tree_inputs(rng, B, w, D, V, (0.0, 0, 1.0), agree=0.0)
    NI = orc.tree_nodes(w, D - 1)
    ql = pl[:, :1 + NI].copy()
    # children: top-3 of q == p; every level's argmax is its first child
    for b in range(B):
        for u in [-1] + list(range(NI)):
            order = np.argsort(-ql[b, u + 1], kind="stable")
            for c, x in zip(orc.tree_children(w, D, u), order[:w]):
                tok[b, c] = x
    path, n, t = orc.tree_accept(pl, ql, tok, w, D, (0.0, 0, 1.0), 1, 0)
    assert n.tolist() == [D] * B
    for b in range(B):
        assert path[b].tolist() == [0, w, w + w * w]  # the first child at every level
        assert t[b] == int(np.argmax(pl[b, 1 + path[b, -1]]))
    # the second child holds the argmax at the root: the walk goes there and stops below it
    tok[:, 1] = tok[:, 0]
    tok[:, 0] = (tok[:, 1] + 1) % V
    for b in range(B):
        tok[b, w + w:w + 2 * w] = (np.argmax(pl[b, 2]) + 1 + np.arange(w)) % V  # no child of node 1 matches
    path, n, t = orc.tree_accept(pl, ql, tok, w, D, (0.0, 0, 1.0), 1, 0)
    assert n.tolist() == [1] * B and path[:, 0].tolist() == [1] * B
    for b in range(B):
        assert t[b] == int(np.argmax(pl[b, 2]))


def test_tree_sampling_is_lossless_chi2():
    """Multi-candidate speculative sampling keeps the target distribution: with w = 3 children
    drawn independently from q at the root, the first committed token is distributed as p."""
    V, w = 6, 3
    rng = np.random.default_rng(8)
    p_log = (rng.standard_normal(V) * 1.5).astype(np.float32)
    q_log = (rng.standard_normal(V) * 1.5).astype(np.float32)
    p = orc.warp_probs(p_log, 1.0)
    B = 6000
    pl = np.broadcast_to(p_log, (B, 1 + w, V)).copy()
    ql = np.broadcast_to(q_log, (B, 1, V)).copy()
    tok = np.array([[orc.sample(q_log, orc.uniform(13, 0, b, c, 1), 1.0) for c in range(w)] for b in range(B)],
                   np.int32)
    path, n, t = orc.tree_accept(pl, ql, tok, w, 1, (1.0, 0, 1.0), 13, 0)
    first = np.where(n > 0, tok[np.arange(B), np.maximum(path[:, 0], 0)], t)
    counts = np.bincount(first, minlength=V)
    chi2 = ((counts - p * B) ** 2 / (p * B)).sum()
    assert chi2 < 25.0, (chi2, counts, p * B)  # 5 dof, p ~ 1e-4
    # and more candidates are accepted than with one child
    path1, n1, _ = orc.tree_accept(pl[:, :2], ql, tok[:, :1], 1, 1, (1.0, 0, 1.0), 13, 0)
    assert n.sum() > n1.sum()
