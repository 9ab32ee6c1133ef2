"""ctypes wrapper over the CPU oracle (oracle/oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline leg as the checker; the product path never imports it.
"""
import ctypes as C
import os

import numpy as np

from . import build as _build  # noqa: F401  (package-relative when imported as oracle.*)

_lib = None

T_F32, T_F16, T_Q4_0, T_Q4_K = 0, 1, 2, 12
T_Q8_0, T_Q6_K = 8, 14


class Desc(C.Structure):
    _fields_ = [("n_layer", C.c_int), ("d_model", C.c_int), ("n_head", C.c_int),
                ("n_head_kv", C.c_int), ("head_dim", C.c_int), ("d_ff", C.c_int),
                ("n_vocab", C.c_int), ("rms_eps", C.c_float), ("rope_base", C.c_float),
                ("wtype", C.c_int)]


class Warp(C.Structure):
    _fields_ = [("temperature", C.c_float), ("top_k", C.c_int), ("top_p", C.c_float)]


def lib():
    global _lib
    if _lib is None:
        path = _build.build()
        L = C.CDLL(path)
        P = C.c_void_p
        L.orc_type_nbytes.restype = C.c_size_t
        L.orc_type_nbytes.argtypes = [C.c_int, C.c_uint64]
        L.orc_dequant.argtypes = [C.c_int, P, C.c_uint64, P]
        L.orc_qgemv.argtypes = [C.c_int, P, C.c_int, C.c_int, P, C.c_int, P, C.c_int]
        L.orc_quantize_q4_0.argtypes = [P, C.c_uint64, P]
        L.orc_rope_table.argtypes = [C.c_float, C.c_int, C.c_int, P, P]
        L.orc_attention.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, P, P, P, P, P,
                                    C.c_int, P]
        L.orc_model_load.restype = P
        L.orc_model_load.argtypes = [C.c_char_p, C.c_char_p, C.c_int]
        L.orc_model_free.argtypes = [P]
        L.orc_model_get_desc.argtypes = [P, C.POINTER(Desc)]
        L.orc_model_tensor.restype = P
        L.orc_model_tensor.argtypes = [P, C.c_char_p, C.POINTER(C.c_int),
                                       C.POINTER(C.c_uint64), C.POINTER(C.c_size_t)]
        L.orc_kv_alloc.restype = P
        L.orc_kv_alloc.argtypes = [P, C.c_int, C.c_int]
        L.orc_kv_free.argtypes = [P]
        L.orc_forward.argtypes = [P, P, C.c_int, C.c_int, P, P, P, C.c_int, P, C.c_int]
        L.orc_uniform.restype = C.c_float
        L.orc_uniform.argtypes = [C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32]
        L.orc_philox.argtypes = [C.c_uint32] * 6 + [P]
        L.orc_warp_probs.argtypes = [P, C.c_int, C.POINTER(Warp), P]
        L.orc_warp_exp.restype = C.c_float
        L.orc_warp_exp.argtypes = [C.c_float]
        L.orc_warp_weights.argtypes = [P, C.c_int, C.POINTER(Warp), P, C.POINTER(C.c_double)]
        L.orc_sample.argtypes = [P, C.c_int, C.POINTER(Warp), C.c_float]
        L.orc_spec_accept.argtypes = [P, P, P, C.c_int, C.c_int, C.c_int, C.POINTER(Warp),
                                      C.c_uint64, C.c_uint32, P, P]
        L.orc_tree_accept.argtypes = [P, P, P, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(Warp),
                                      C.c_uint64, C.c_uint32, P, P, P]
        L.orc_spec_generate.argtypes = [P, P, C.c_int, P, P, C.c_int, C.c_int, C.c_int,
                                        C.POINTER(Warp), C.c_uint64, P, P, P,
                                        C.POINTER(C.c_double), P]
        L.orc_set_threads.argtypes = [C.c_int]
        L.orc_bench_rounds.argtypes = [P, P, C.c_int, C.c_int, C.c_int, C.POINTER(Warp), C.c_uint64, P]
        _lib = L
    return _lib


def _p(a):
    return a.ctypes.data_as(C.c_void_p)


def type_nbytes(t, n):
    return int(lib().orc_type_nbytes(t, n))


def dequant(t, blocks: np.ndarray, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    rc = lib().orc_dequant(t, _p(np.ascontiguousarray(blocks)), n, _p(out))
    assert rc == 0, rc
    return out


def qgemv(t, w_bytes: np.ndarray, N: int, K: int, x16: np.ndarray) -> np.ndarray:
    x16 = np.ascontiguousarray(x16, dtype=np.float16)
    M = x16.shape[0]
    y = np.empty((M, N), np.float32)
    rc = lib().orc_qgemv(t, _p(np.ascontiguousarray(w_bytes)), N, K, _p(x16.view(np.uint16)), M,
                         _p(y), N)
    assert rc == 0, rc
    return y


def quantize_q4_0(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    out = np.empty(x.size // 32 * 18, np.uint8)
    assert lib().orc_quantize_q4_0(_p(x), x.size, _p(out)) == 0
    return out


def rope_table(base, head_dim, n_pos):
    c = np.empty((n_pos, head_dim // 2), np.float32)
    s = np.empty_like(c)
    lib().orc_rope_table(base, head_dim, n_pos, _p(c), _p(s))
    return c, s


def attention(n_head, n_head_kv, head_dim, cap, scale, q, k, v, row_seq, row_pos):
    q = np.ascontiguousarray(q, np.float32)
    M = q.shape[0]
    out = np.empty((M, n_head * head_dim), np.uint16)
    lib().orc_attention(n_head, n_head_kv, head_dim, cap, scale, _p(q),
                        _p(np.ascontiguousarray(k, np.uint16)), _p(np.ascontiguousarray(v, np.uint16)),
                        _p(np.ascontiguousarray(row_seq, np.int32)),
                        _p(np.ascontiguousarray(row_pos, np.int32)), M, _p(out))
    return out.view(np.float16)


def philox(c, k):
    out = np.empty(4, np.uint32)
    lib().orc_philox(*(int(x) for x in c), *(int(x) for x in k), _p(out))
    return out


def uniform(seed, rnd, seq, slot, tag):
    return float(lib().orc_uniform(seed, rnd, seq, slot, tag))


def warp_probs(logits, temperature=1.0, top_k=0, top_p=1.0):
    logits = np.ascontiguousarray(logits, np.float32)
    p = np.empty(logits.size, np.float64)
    w = Warp(temperature, top_k, top_p)
    lib().orc_warp_probs(_p(logits), logits.size, C.byref(w), _p(p))
    return p


def warp_exp(x):
    return float(lib().orc_warp_exp(float(x)))


def warp_weights(logits, temperature=1.0, top_k=0, top_p=1.0):
    logits = np.ascontiguousarray(logits, np.float32)
    e = np.empty(logits.size, np.float64)
    Z = C.c_double()
    w = Warp(temperature, top_k, top_p)
    lib().orc_warp_weights(_p(logits), logits.size, C.byref(w), _p(e), C.byref(Z))
    return e, Z.value


def sample(logits, u, temperature=1.0, top_k=0, top_p=1.0):
    logits = np.ascontiguousarray(logits, np.float32)
    w = Warp(temperature, top_k, top_p)
    return int(lib().orc_sample(_p(logits), logits.size, C.byref(w), u))


def spec_accept(p_logits, q_logits, draft, warp, seed, rnd):
    p_logits = np.ascontiguousarray(p_logits, np.float32)
    q_logits = np.ascontiguousarray(q_logits, np.float32)
    draft = np.ascontiguousarray(draft, np.int32)
    B, k = draft.shape
    V = p_logits.shape[-1]
    out = np.full((B, k + 1), -1, np.int32)
    n = np.empty(B, np.int32)
    w = Warp(*warp)
    lib().orc_spec_accept(_p(p_logits), _p(q_logits), _p(draft), B, k, V, C.byref(w), seed, rnd,
                          _p(out), _p(n))
    return out, n


def tree_nodes(width, depth):
    """nodes of a full tree of this width and depth (breadth first, the root not counted)"""
    return sum(width ** d for d in range(1, depth + 1))


def tree_children(width, depth, node):
    """breadth-first indices of the children of `node` (-1: the root)"""
    if node < 0:
        return list(range(width))
    d, first = 1, 0
    while node >= first + width ** d:
        first += width ** d
        d += 1
    if d >= depth:
        return []
    nxt = first + width ** d
    return [nxt + (node - first) * width + c for c in range(width)]


def tree_accept(p_logits, q_logits, tokens, width, depth, warp, seed, rnd):
    """orc_tree_accept: p [B][1 + N][V], q [B][1 + internal][V], tokens [B][N] -> path [B][depth]
    (accepted nodes, -1 after), n [B], tok [B]"""
    p_logits = np.ascontiguousarray(p_logits, np.float32)
    q_logits = np.ascontiguousarray(q_logits, np.float32)
    tokens = np.ascontiguousarray(tokens, np.int32)
    B = tokens.shape[0]
    V = p_logits.shape[-1]
    path = np.full((B, depth), -1, np.int32)
    n = np.empty(B, np.int32)
    tok = np.empty(B, np.int32)
    w = Warp(*warp)
    lib().orc_tree_accept(_p(p_logits), _p(q_logits), _p(tokens), B, width, depth, V, C.byref(w), seed, rnd,
                          _p(path), _p(n), _p(tok))
    return path, n, tok


class Model:
    def __init__(self, path):
        err = C.create_string_buffer(256)
        self.h = lib().orc_model_load(path.encode(), err, 256)
        if not self.h:
            raise RuntimeError("oracle load failed: " + err.value.decode())
        self.desc = Desc()
        lib().orc_model_get_desc(self.h, C.byref(self.desc))

    def tensor(self, name):
        t = C.c_int()
        ne = (C.c_uint64 * 4)()
        nb = C.c_size_t()
        ptr = lib().orc_model_tensor(self.h, name.encode(), C.byref(t), ne, C.byref(nb))
        if not ptr:
            raise KeyError(name)
        buf = (C.c_uint8 * nb.value).from_address(ptr)
        return t.value, tuple(int(x) for x in ne), np.frombuffer(buf, np.uint8)

    def close(self):
        if self.h:
            lib().orc_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class KV:
    def __init__(self, model: Model, n_seq, cap):
        self.h = lib().orc_kv_alloc(model.h, n_seq, cap)
        self.cap = cap

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_kv_free(self.h)
            self.h = None


def forward(model: Model, kv: KV, tokens, row_seq, row_pos, rows_per_seq, logits_mode=0):
    tokens = np.ascontiguousarray(tokens, np.int32)
    M = tokens.size
    V = model.desc.n_vocab
    n_out = M // rows_per_seq if logits_mode == 1 else M
    logits = np.empty((n_out, V), np.float32)
    rc = lib().orc_forward(model.h, kv.h, M, rows_per_seq, _p(tokens),
                           _p(np.ascontiguousarray(row_seq, np.int32)),
                           _p(np.ascontiguousarray(row_pos, np.int32)), logits_mode, _p(logits), V)
    assert rc == 0, rc
    return logits


def bench_rounds(target: Model, draft, ctx_len, k, rounds, warp, seed=0, threads=0):
    """Returns (tokens committed, stats[4]) of `rounds` rounds at context ctx_len."""
    if threads:
        lib().orc_set_threads(threads)
    stats = np.zeros(4, np.uint64)
    w = Warp(*warp)
    n = lib().orc_bench_rounds(target.h, draft.h if draft is not None else None, ctx_len, k, rounds,
                               C.byref(w), seed, _p(stats))
    assert n >= 0, n
    return n, stats


def spec_generate(target: Model, draft, prompts, max_new, k, warp, seed, threads=0, with_margins=False):
    """Returns (tokens [S][max_new], counts [S], stats[4], min top-2 margin (greedy)), plus,
    with_margins, the top-2 logit margin that decided each committed token [S][max_new]."""
    prompts = [np.asarray(p, np.int32) for p in prompts]
    S = len(prompts)
    P = max(p.size for p in prompts)
    pr = np.zeros((S, P), np.int32)
    for i, p in enumerate(prompts):
        pr[i, :p.size] = p
    plen = np.array([p.size for p in prompts], np.int32)
    out = np.empty((S, max_new), np.int32)
    cnt = np.empty(S, np.int32)
    stats = np.zeros(4, np.uint64)
    margin = C.c_double(0.0)
    if threads:
        lib().orc_set_threads(threads)
    w = Warp(*warp)
    tm = np.full((S, max_new), np.inf)
    rc = lib().orc_spec_generate(target.h, draft.h if draft is not None else None, S, _p(pr),
                                 _p(plen), P, max_new, k, C.byref(w), seed, _p(out), _p(cnt),
                                 _p(stats), C.byref(margin), _p(tm))
    assert rc == 0, rc
    if with_margins:
        return out, cnt, stats, margin.value, tm
    return out, cnt, stats, margin.value
