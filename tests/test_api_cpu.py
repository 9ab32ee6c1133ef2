"""CPU tests: the C ABI library loads and exports every function include/ulb.h declares,
the reference-compatible Python surface exists with the reference's behaviours, the GGUF
reader/writer round-trips, and errors come back as status codes (no CPU fallback)."""
import os

import numpy as np
import pytest

import gguf
from conftest import has_gpu


def test_library_exports_every_header_function():
    import ulb_capi
    names = ulb_capi.header_functions()
    assert len(names) >= 30
    lib = ulb_capi.lib()
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert set(names) == set(ulb_capi._SIGS), set(names) ^ set(ulb_capi._SIGS)


def test_version_and_no_cpu_fallback():
    import ulb_capi
    assert b"sm_100a" in ulb_capi.lib().ulb_version()
    if has_gpu():
        pytest.skip("a CUDA device is present")
    with pytest.raises(ulb_capi.UlbError) as e:
        ulb_capi.Context(0)
    assert e.value.code == ulb_capi.ECUDA


def test_null_arguments_are_rejected_with_status():
    import ctypes as C
    import ulb_capi as U
    L = U.lib()
    assert L.ulb_stream_sync(None) == U.EINVAL
    assert L.ulb_dequant(None, None, None) == U.EINVAL
    assert L.ulb_qgemm(None, None, None, 1, None, 1) == U.EINVAL
    assert L.ulb_spec_run(None, 1, None) == U.EINVAL
    assert b"NULL" in L.ulb_last_error()
    assert L.ulb_tensor_free(None) == U.OK


@pytest.mark.parametrize("fn", ["ulb_attention", "ulb_attention_noalloc"])
def test_attention_descriptor_checked_before_any_host_arithmetic(fn):
    """A zero kv-head count or rows_per_seq must come back as ULB_EINVAL, not as a host
    division by zero.  The descriptor is checked before the context is used at all, so a
    stand-in (never dereferenced) context handle is enough to reach the check on the CPU."""
    import ctypes as C
    import ulb_capi as U
    L = U.lib()
    fake = C.c_void_p(16)
    for desc, M, rps in ((U.AttnDesc(32, 0, 128, 512, 1, 0.1), 6, 6),
                         (U.AttnDesc(32, 8, 128, 512, 1, 0.1), 6, 0),
                         (U.AttnDesc(32, 8, 0, 512, 1, 0.1), 6, 6),
                         (U.AttnDesc(32, 8, 128, 0, 1, 0.1), 6, 6)):
        rc = getattr(L, fn)(fake, C.byref(desc), fake, fake, fake, fake, fake, M, rps, fake)
        assert rc in (U.EINVAL, U.EUNSUPPORTED), rc
        assert b"attention" in L.ulb_last_error()


def test_surface_matches_reference():
    import vulkangguf as vg
    for cls in ("InferenceAPI", "GenerationConfig", "GenerationResult", "GenerationProgress", "ModelMetrics",
                "QuantizationType", "SpeculationResult", "SpeculativeToken"):
        assert hasattr(vg, cls)
    ref_methods = ["load_model", "unload_model", "generate", "generate_default", "generate_streaming",
                   "generate_with_progress", "generate_batch", "enable_gpu", "is_gpu_enabled", "get_model_info",
                   "get_model_architecture", "set_max_batch_size", "enable_speculative_decoding",
                   "enable_multi_gpu", "get_acceptance_rate", "get_throughput", "set_temperature", "set_top_p",
                   "set_top_k", "set_cache_size_mb", "set_num_threads", "save_pipeline_cache",
                   "load_pipeline_cache", "enable_profiling", "get_performance_report", "get_token_logits",
                   "set_adapter_alpha", "enable_adapter", "disable_adapter", "get_loaded_adapters",
                   "register_custom_tokenizer", "register_custom_kernel"]
    api = vg.InferenceAPI()
    for m in ref_methods:
        assert callable(getattr(api, m)), m
    assert vg.get_quantization_type_name(vg.QuantizationType.NF4) == "NF4"


def test_generation_config_value_initialised_to_zero():
    import vulkangguf as vg
    c = vg.GenerationConfig()
    assert (c.max_tokens, c.temperature, c.top_p, c.top_k, c.frequency_penalty, c.presence_penalty,
            c.do_sample) == (0, 0.0, 0.0, 0, 0.0, 0.0, False)


def test_generate_without_model():
    import vulkangguf as vg
    api = vg.InferenceAPI()
    assert api.generate("hello", vg.GenerationConfig()) == "Error: No model loaded"
    assert api.get_acceptance_rate() == 0.0
    assert api.save_pipeline_cache("/tmp/x") and api.load_pipeline_cache("/tmp/x")
    assert api.get_model_architecture() == "llama"


def test_synthetic_gguf_readable_by_gguf_package(tiny_draft):
    r = gguf.GGUFReader(tiny_draft)
    names = [t.name for t in r.tensors]
    assert names[0] == "token_embd.weight" and names[-1] == "output.weight"
    assert "blk.1.ffn_down.weight" in names and len(names) == 3 + 2 * 9
    fields = {f.name: f for f in r.fields.values()}
    assert int(fields["llama.block_count"].parts[-1][0]) == 2
    q = next(t for t in r.tensors if t.name == "blk.0.attn_q.weight")
    assert q.tensor_type == gguf.GGMLQuantizationType.Q4_0 and list(q.shape) == [512, 512]


def test_synthetic_weights_are_seeded_normals(tiny_draft):
    import vulkangguf as vg
    r = gguf.GGUFReader(tiny_draft)
    q = next(t for t in r.tensors if t.name == "blk.1.attn_v.weight")
    w = gguf.quants.dequantize(q.data, q.tensor_type).ravel()
    assert abs(w.std() - 0.02) < 0.002 and abs(w.mean()) < 0.001
    x = np.array([vg.synth_normal(0, "blk.1.attn_v.weight", i) for i in range(64)], np.float32) * 0.02
    qq = gguf.quants.quantize(x.reshape(2, 32), gguf.GGMLQuantizationType.Q4_0).ravel()
    assert np.array_equal(np.asarray(q.data).ravel()[:36], qq)


def test_shared_seed_shares_blocks(tiny_target, tiny_draft):
    a = {t.name: t for t in gguf.GGUFReader(tiny_target).tensors}
    b = {t.name: t for t in gguf.GGUFReader(tiny_draft).tensors}
    for n in ("token_embd.weight", "blk.0.attn_q.weight", "blk.1.ffn_down.weight", "output.weight"):
        assert np.array_equal(np.asarray(a[n].data), np.asarray(b[n].data)), n


def test_q4k_synthetic_decodes(tiny_gqa_q4k):
    r = gguf.GGUFReader(tiny_gqa_q4k)
    t = next(t for t in r.tensors if t.name == "blk.0.ffn_gate.weight")
    assert t.tensor_type == gguf.GGMLQuantizationType.Q4_K
    w = gguf.quants.dequantize(t.data, t.tensor_type)
    x = np.array([__import__("vulkangguf").synth_normal(3, "blk.0.ffn_gate.weight", i) for i in range(256)]) * 0.02
    assert np.abs(w.ravel()[:256] - x).max() < 0.02  # within a quantisation step
    assert abs(w.std() - 0.02) < 0.003


def test_truncated_gguf_rejected(tmp_path, tiny_draft):
    from oracle import ulb_oracle as orc
    data = open(tiny_draft, "rb").read()
    bad = tmp_path / "trunc.gguf"
    bad.write_bytes(data[: len(data) // 2])
    with pytest.raises(RuntimeError):
        orc.Model(str(bad))
    import vulkangguf as vg
    api = vg.InferenceAPI()
    assert api.load_model(str(bad)) is False


@pytest.mark.parametrize("field,value", [
    ("ne1", 1 << 62),             # element count ne0 * ne1 wraps past 64 bits
    ("ne1", 1 << 40),             # no wrap, but 316 TB of data past the end of the file
    ("offset", (1 << 64) - 64),    # data start + offset wraps around
])
def test_gguf_with_overflowing_tensor_info_rejected(tmp_path, tiny_draft, field, value):
    """A crafted tensor info whose sizes or offset overflow 64-bit arithmetic is refused, not
    read past the end of the mapping."""
    import struct
    data = bytearray(open(tiny_draft, "rb").read())
    name = b"blk.0.attn_q.weight"
    at = data.index(struct.pack("<Q", len(name)) + name) + 8 + len(name)
    n_dims = struct.unpack_from("<I", data, at)[0]
    assert n_dims == 2
    off = {"ne1": at + 4 + 8, "offset": at + 4 + 8 * n_dims + 4}[field]
    struct.pack_into("<Q", data, off, value)
    bad = tmp_path / ("overflow_%s.gguf" % field)
    bad.write_bytes(bytes(data))
    import vulkangguf as vg
    api = vg.InferenceAPI()
    assert api.load_model(str(bad)) is False


def test_trace_build_exports_its_dump_functions_and_the_product_build_none():
    """The CTA timeline trace is compiled into libulb_cuda_trace.so only (bench.py --mode trace
    reads one ring per translation unit); both builds carry the soname the Python module binds."""
    import subprocess
    import bench
    import build as pbuild
    pbuild.build_cuda(trace=True)

    def dyn_symbols(path):
        out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True, check=True).stdout
        return {line.split()[-1] for line in out.splitlines() if line.strip()}

    tr = dyn_symbols(pbuild.CUDA_LIB_TRACE)
    assert {"ulb_trace_dump_" + u for u in bench.TRACE_UNITS} <= tr
    assert not {n for n in dyn_symbols(pbuild.CUDA_LIB) if n.startswith("ulb_trace_")}
    for path in (pbuild.CUDA_LIB, pbuild.CUDA_LIB_TRACE):
        dyn = subprocess.run(["readelf", "-d", path], capture_output=True, text=True, check=True).stdout
        assert "Library soname: [libulb_cuda.so]" in dyn
