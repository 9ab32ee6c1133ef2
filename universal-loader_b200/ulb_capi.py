"""ctypes binding of libulb_cuda.so (include/ulb.h).

This is the binding a Python caller of the C ABI uses (the reference's own FFI for this
path is pybind11; see vulkangguf for that surface).  Device memory is handled through the
library itself (ulb_malloc / ulb_memcpy_*), so no other GPU framework is involved.
"""
import ctypes as C
import os
import re

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libulb_cuda.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "ulb.h")

OK, EINVAL, ENOMEM, ECUDA, ENCCL, ETIMEOUT, EFORMAT, EUNSUPPORTED = 0, -1, -2, -3, -4, -5, -6, -7
T_F32, T_F16, T_Q4_0, T_Q4_K = 0, 1, 2, 12
RNG_DRAFT, RNG_ACCEPT, RNG_RESID, RNG_FIRST = 1, 2, 3, 4

P = C.c_void_p


class AttnDesc(C.Structure):
    _fields_ = [("n_head", C.c_int), ("n_head_kv", C.c_int), ("head_dim", C.c_int),
                ("capacity", C.c_int), ("n_seq", C.c_int), ("scale", C.c_float)]


class Warp(C.Structure):
    _fields_ = [("temperature", C.c_float), ("top_k", C.c_int), ("top_p", C.c_float)]


class ModelDesc(C.Structure):
    _fields_ = [("n_layer", C.c_int), ("d_model", C.c_int), ("n_head", C.c_int),
                ("n_head_kv", C.c_int), ("head_dim", C.c_int), ("d_ff", C.c_int),
                ("n_vocab", C.c_int), ("rms_eps", C.c_float), ("rope_base", C.c_float),
                ("max_rows", C.c_int)]


class SpecDesc(C.Structure):
    _fields_ = [("n_seq", C.c_int), ("k", C.c_int), ("max_prompt", C.c_int),
                ("max_new", C.c_int), ("warp", Warp), ("seed", C.c_uint64),
                ("use_graphs", C.c_int), ("kv_pages", C.c_int), ("tree_width", C.c_int)]


_SIGS = {
    "ulb_last_error": (C.c_char_p, []),
    "ulb_version": (C.c_char_p, []),
    "ulb_init": (C.c_int, [C.c_int, C.POINTER(P)]),
    "ulb_destroy": (C.c_int, [P]),
    "ulb_stream": (P, [P]),
    "ulb_stream_sync": (C.c_int, [P]),
    "ulb_mem_used": (C.c_int, [P, C.POINTER(C.c_size_t)]),
    "ulb_malloc": (C.c_int, [P, C.c_size_t, C.POINTER(P)]),
    "ulb_free": (C.c_int, [P, P]),
    "ulb_memcpy_h2d": (C.c_int, [P, P, P, C.c_size_t]),
    "ulb_memcpy_d2h": (C.c_int, [P, P, P, C.c_size_t]),
    "ulb_event_create": (C.c_int, [P, C.POINTER(P)]),
    "ulb_event_record": (C.c_int, [P, P]),
    "ulb_event_elapsed_ms": (C.c_int, [P, P, C.POINTER(C.c_float)]),
    "ulb_event_destroy": (C.c_int, [P]),
    "ulb_tp_unique_id": (C.c_int, [P]),
    "ulb_tp_init": (C.c_int, [P, C.c_int, C.c_int, P]),
    "ulb_tp_set_timeout": (C.c_int, [P, C.c_int]),
    "ulb_wait_flag": (C.c_int, [P, P, C.c_int32, C.c_uint64]),
    "ulb_model_set_tp": (C.c_int, [P, C.c_int, C.c_int]),
    "ulb_capture_begin": (C.c_int, [P]),
    "ulb_capture_end": (C.c_int, [P, C.POINTER(P)]),
    "ulb_graph_launch": (C.c_int, [P, P]),
    "ulb_graph_free": (C.c_int, [P]),
    "ulb_tensor_upload": (C.c_int, [P, C.c_int, C.POINTER(C.c_uint64), P, C.c_size_t, C.POINTER(P)]),
    "ulb_tensor_free": (C.c_int, [P]),
    "ulb_tensor_info": (C.c_int, [P, C.POINTER(C.c_int), C.POINTER(C.c_uint64), C.POINTER(C.c_size_t)]),
    "ulb_dequant": (C.c_int, [P, P, P]),
    "ulb_qgemm": (C.c_int, [P, P, P, C.c_int, P, C.c_int]),
    "ulb_attention": (C.c_int, [P, C.POINTER(AttnDesc), P, P, P, P, P, C.c_int, C.c_int, P]),
    "ulb_attention_noalloc": (C.c_int, [P, C.POINTER(AttnDesc), P, P, P, P, P, C.c_int, C.c_int, P]),
    "ulb_attention_set_form": (C.c_int, [P, C.c_int]),
    "ulb_attention_paged": (C.c_int, [P, C.POINTER(AttnDesc), P, P, P, P, C.c_int, P, P, C.c_int, C.c_int, P]),
    "ulb_sample": (C.c_int, [P, P, C.c_int, C.c_int, C.c_int, C.POINTER(Warp), C.c_uint64,
                             C.c_uint32, C.c_uint32, C.c_uint32, P]),
    "ulb_spec_accept": (C.c_int, [P, P, P, P, C.c_int, C.c_int, C.c_int, C.POINTER(Warp),
                                  C.c_uint64, C.c_uint32, P, P]),
    "ulb_spec_tree_accept": (C.c_int, [P, P, P, P, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(Warp),
                                       C.c_uint64, C.c_uint32, P, P, P]),
    "ulb_model_create": (C.c_int, [P, C.POINTER(ModelDesc), C.POINTER(P)]),
    "ulb_model_set_weight": (C.c_int, [P, C.c_char_p, C.c_int, C.POINTER(C.c_uint64), P, C.c_size_t]),
    "ulb_model_finalize": (C.c_int, [P]),
    "ulb_model_free": (C.c_int, [P]),
    "ulb_model_weight_bytes": (C.c_int, [P, C.POINTER(C.c_size_t)]),
    "ulb_kv_alloc": (C.c_int, [P, P, C.c_int, C.c_int, C.POINTER(P)]),
    "ulb_kv_alloc_paged": (C.c_int, [P, P, C.c_int, C.c_int, C.c_int, C.POINTER(P)]),
    "ulb_kv_map": (C.c_int, [P, C.c_int, C.c_int, C.c_int, P]),
    "ulb_kv_free": (C.c_int, [P]),
    "ulb_model_forward": (C.c_int, [P, P, P, C.c_int, C.c_int, P, P, P, C.c_int, P, C.c_int]),
    "ulb_spec_create": (C.c_int, [P, P, P, C.POINTER(SpecDesc), C.POINTER(P)]),
    "ulb_spec_prefill": (C.c_int, [P, P, P]),
    "ulb_spec_run": (C.c_int, [P, C.c_int, C.POINTER(C.c_int)]),
    "ulb_spec_read": (C.c_int, [P, P, P, P]),
    "ulb_spec_free": (C.c_int, [P]),
    "ulb_spec_profile_round": (C.c_int, [P, C.POINTER(C.c_float)]),
    "ulb_spec_profile_round_ex": (C.c_int, [P, C.POINTER(C.c_float)]),
    "ulb_spec_read_rounds": (C.c_int, [P, C.c_int, C.c_int, P, C.POINTER(C.c_int)]),
    "ulb_spec_admit": (C.c_int, [P, C.c_int, P, C.c_int]),
    "ulb_spec_launch_count": (C.c_int, [P, C.POINTER(C.c_uint64)]),
}

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError("libulb_cuda.so is not built (run __graft_entry__.build())")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def header_functions():
    """Names of every function include/ulb.h declares."""
    with open(HEADER) as f:
        text = f.read()
    return sorted(set(re.findall(r"^ULB_API\s+[\w\s\*]+?\b(ulb_\w+)\s*\(", text, flags=re.M)))


class UlbError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__("ULB error %d: %s" % (code, msg))
        self.code = code


def check(rc):
    if rc != OK:
        raise UlbError(rc, lib().ulb_last_error().decode())
    return rc


def _ptr(a):
    return a.ctypes.data_as(P)


class DeviceBuffer:
    def __init__(self, ctx, nbytes):
        self.ctx = ctx
        self.nbytes = int(nbytes)
        p = P()
        check(lib().ulb_malloc(ctx.h, self.nbytes, C.byref(p)))
        self.ptr = p

    @property
    def value(self):
        return self.ptr.value

    def upload(self, arr):
        arr = np.ascontiguousarray(arr)
        assert arr.nbytes <= self.nbytes
        check(lib().ulb_memcpy_h2d(self.ctx.h, self.ptr, _ptr(arr), arr.nbytes))
        return self

    def download(self, dtype, shape):
        out = np.empty(shape, dtype)
        assert out.nbytes <= self.nbytes
        check(lib().ulb_memcpy_d2h(self.ctx.h, _ptr(out), self.ptr, out.nbytes))
        return out

    def free(self):
        if self.ptr is not None and self.ptr.value:
            lib().ulb_free(self.ctx.h, self.ptr)
        self.ptr = None


class Context:
    def __init__(self, device=0):
        h = P()
        check(lib().ulb_init(device, C.byref(h)))
        self.h = h

    def close(self):
        if self.h:
            lib().ulb_destroy(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def sync(self):
        check(lib().ulb_stream_sync(self.h))

    def buffer(self, arr=None, nbytes=None):
        if arr is not None:
            arr = np.ascontiguousarray(arr)
            return DeviceBuffer(self, max(arr.nbytes, 16)).upload(arr)
        return DeviceBuffer(self, max(int(nbytes), 16))

    def upload_tensor(self, ggml_type, ne, raw):
        raw = np.ascontiguousarray(raw, np.uint8)
        ne4 = (C.c_uint64 * 4)(*(list(ne) + [1] * (4 - len(ne))))
        t = P()
        check(lib().ulb_tensor_upload(self.h, ggml_type, ne4, _ptr(raw), raw.nbytes, C.byref(t)))
        return t

    def free_tensor(self, t):
        lib().ulb_tensor_free(t)

    def dequant(self, t, n_rows, n_cols):
        out = self.buffer(nbytes=n_rows * n_cols * 4)
        check(lib().ulb_dequant(self.h, t, out.ptr))
        r = out.download(np.float32, (n_rows, n_cols))
        out.free()
        return r

    def qgemm(self, t, x16, N):
        x16 = np.ascontiguousarray(x16, np.float16)
        M = x16.shape[0]
        xb = self.buffer(x16)
        yb = self.buffer(nbytes=max(M, 1) * N * 4)
        check(lib().ulb_qgemm(self.h, t, xb.ptr, M, yb.ptr, N))
        y = yb.download(np.float32, (M, N))
        xb.free()
        yb.free()
        return y

    def event(self):
        e = P()
        check(lib().ulb_event_create(self.h, C.byref(e)))
        return e

    def record(self, e):
        check(lib().ulb_event_record(self.h, e))

    def capture(self, fn):
        """Record the device work of fn() into a CUDA graph (returns the graph handle)."""
        check(lib().ulb_capture_begin(self.h))
        try:
            fn()
        finally:
            g = P()
            rc = lib().ulb_capture_end(self.h, C.byref(g))
        check(rc)
        return g

    def time_graph(self, g, reps=10):
        """Device milliseconds of one replay of g (CUDA events, after one warm replay)."""
        check(lib().ulb_graph_launch(self.h, g))
        a, b = self.event(), self.event()
        self.record(a)
        for _ in range(reps):
            check(lib().ulb_graph_launch(self.h, g))
        self.record(b)
        self.sync()
        ms = self.elapsed_ms(a, b) / reps
        lib().ulb_event_destroy(a)
        lib().ulb_event_destroy(b)
        return ms

    def elapsed_ms(self, a, b):
        ms = C.c_float()
        check(lib().ulb_event_elapsed_ms(a, b, C.byref(ms)))
        return ms.value
