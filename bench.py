#!/usr/bin/env python
"""Benchmark: accepted tok/s of the speculative draft -> verify -> accept loop.

Headline workload: Llama-2-7B-architecture Q4_0 target (seed 0) +
TinyLlama-1.1B-architecture Q4_0 draft (seed 2), weights N(0, 0.02) -> Q4_0, one 512-token
uniform random prompt, k = 5, 256 committed tokens, T = 0 (and a T = 0.8 figure beside it).
Synthetic GGUF files are written once per machine.

A step is one generation of 256 tokens from a fresh prefill.  `value` is committed tokens of
all ranks / the slowest rank's device time of the generation phase (CUDA events on the
engine's stream; prefill reported separately); `e2e` is the same count over host wall time of
the public API call (prompt copied in, tokens copied out, prefill included).  With N GPUs each
rank decodes its own C2 sequence (replicas, no collective: one sequence does not shard).

The configurations that do shard are measured in the same run, each in a child process group
of its own (so one cannot take the headline down with it) and reported as objects of the
headline line:
  "c4"  config 4 at every N: 64 Llama-3-8B / 3.2-1B Q4_K sequences sharded round-robin over
        the GPUs (data parallel, no collective on the data path);
  "c5"  config 5 at N >= 2: the Llama-2-70B-architecture Q4_0 target tensor-parallel over the
        GPUs (NCCL all-reduce after attn-out and FFN-down), the 7B draft replicated.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload c2|c4|c5] [--extras auto|none|c4|c5|c4,c5]
  python bench.py --mode ops [--only CASE]     the config-3 kernel sweep
  python bench.py --mode trace [--workload c4] the CTA timeline of one C2 (C4) round
"""
import argparse
import json
import os
import shutil
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "universal-loader_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

# CUDA_VISIBLE_DEVICES as the launcher set it (each rank narrows it to its own GPU later; the
# child process groups of the c4 / c5 workloads choose their GPU from the original list)
ORIG_CUDA_VISIBLE = os.environ.get("CUDA_VISIBLE_DEVICES")
T_START = time.time()
METRIC = "accepted tok/s (Llama-2-7B-arch Q4_0, k=5) at 1-8 B200; verify HBM GB/s vs peak"
TARGET = dict(n_layer=32, d_model=4096, n_head=32, n_head_kv=32, d_ff=11008, n_vocab=32000, rms_eps=1e-5,
              rope_base=1e4, wtype="q4_0", seed=0, ctx_len=4096, name="llama2-7b-arch-q4_0-s0")
DRAFT = dict(n_layer=22, d_model=2048, n_head=32, n_head_kv=4, d_ff=5632, n_vocab=32000, rms_eps=1e-5,
             rope_base=1e4, wtype="q4_0", seed=2, ctx_len=2048, name="tinyllama-1.1b-arch-q4_0-s2")
PROMPT_LEN, K_SPEC, NEW_TOKENS = 512, 5, 256
# ncu (dram__bytes_read.sum + dram__bytes_write.sum) / algorithmic bytes of one fused Q4_0 GEMV
# launch (N=11008, K=4096, M=5: 25.48 MB measured vs 25.62 MB algorithmic)
QGEMV_TRAFFIC_RATIO = 0.994
WORKLOAD = ("C2: Llama-2-7B-arch Q4_0 target + TinyLlama-1.1B-arch Q4_0 draft, B=1 per GPU, "
            "prompt 512, k=5, 256 new tokens, T=0")


def q4_0_bytes(n):
    return n // 32 * 18


def linear_weights(s):
    hd = s["d_model"] // s["n_head"]
    d, f = s["d_model"], s["d_ff"]
    per_layer = d * s["n_head"] * hd * 2 + d * s["n_head_kv"] * hd * 2 + 3 * d * f
    return s["n_layer"] * per_layer + d * s["n_vocab"]


def kv_bytes_per_token(s):
    hd = s["d_model"] // s["n_head"]
    return s["n_layer"] * s["n_head_kv"] * hd * 2 * 2


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            pk = json.load(f)
        return float(pk["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# Llama-3-8B-arch target + Llama-3.2-1B-arch draft, both Q4_K, N(0, 0.02) from
# seed 0; 64 sequences, context lengths U[256, 4096], k = 8, T = 0.8, top_p = 0.9
C4_TARGET = dict(n_layer=32, d_model=4096, n_head=32, n_head_kv=8, d_ff=14336, n_vocab=128256, rms_eps=1e-5,
                 rope_base=5e5, wtype="q4_k", seed=0, ctx_len=8192, name="llama3-8b-arch-q4_k-s0")
C4_DRAFT = dict(n_layer=16, d_model=2048, n_head=32, n_head_kv=8, d_ff=8192, n_vocab=128256, rms_eps=1e-5,
                rope_base=5e5, wtype="q4_k", seed=0, ctx_len=8192, name="llama3.2-1b-arch-q4_k-s0")
C4_SEQS, C4_K, C4_NEW, C4_CTX = 64, 8, 256, (256, 4096)
C4_WORKLOAD = ("C4: Llama-3-8B-arch Q4_K target + Llama-3.2-1B-arch Q4_K draft, 64 sequences sharded round-robin "
               "over the GPUs (64/N per GPU), prompt lengths U[256,4096] (seed 1), k=8, 256 new tokens per "
               "sequence, T=0.8, top_p=0.9")


# all synthetic model files of the bench (C2 + C4 + C5) take ~50 GB
CACHE_NEED_BYTES = 64 << 30


def cache_dir():
    """Where the synthetic GGUF files live: ULB_BENCH_CACHE, else a machine-wide directory
    that already holds them, else whichever of /tmp and /dev/shm has room for all of them."""
    d = os.environ.get("ULB_BENCH_CACHE")
    if d:
        return d
    cands = ["/tmp/ulb_bench_models", "/dev/shm/ulb_bench_models"]
    for c in cands:
        if os.path.isdir(c):
            return c
    for c in cands:
        try:
            if shutil.disk_usage(os.path.dirname(c)).free >= CACHE_NEED_BYTES:
                return c
        except OSError:
            continue
    return cands[0]


def model_paths(target=None, draft=None):
    target, draft = target or TARGET, draft or DRAFT
    d = cache_dir()
    os.makedirs(d, exist_ok=True)
    return os.path.join(d, target["name"] + ".gguf"), os.path.join(d, draft["name"] + ".gguf")


def write_model(path, spec):
    """Write one synthetic GGUF file (atomically: another process never sees a partial file)."""
    import vulkangguf as vg
    tmp = "%s.part%d" % (path, os.getpid())
    t0 = time.time()
    vg.write_synthetic_gguf(tmp, spec)
    os.replace(tmp, path)
    print("[bench] wrote %s in %.1fs" % (path, time.time() - t0), file=sys.stderr)


def ensure_models(rank, barrier, target=None, draft=None):
    target, draft = target or TARGET, draft or DRAFT
    tp, dp = model_paths(target, draft)
    if rank == 0:
        for path, spec in ((tp, target), (dp, draft)):
            if not os.path.exists(path):
                write_model(path, spec)
    barrier()
    return tp, dp


def ensure_models_in_child(target=None, draft=None):
    """ensure_models for the reference arm: the files are written by a separate process, so
    the arm's own process loads no library of this package (only the oracle it times)."""
    target, draft = target or TARGET, draft or DRAFT
    tp, dp = model_paths(target, draft)
    if not (os.path.exists(tp) and os.path.exists(dp)):
        code = ("import sys; sys.path[:0] = [%r, %r]; import bench; bench.ensure_models(0, lambda: None)"
                % (ROOT, PKG))
        subprocess.run([sys.executable, "-c", code], check=True)
    return tp, dp


def prompt_for(rank):
    import numpy as np
    return np.random.default_rng(1 + 1000 * rank).integers(0, 32000, PROMPT_LEN).astype(np.int32).tolist()


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "--query-gpu=" + self.Q, "--format=csv,noheader,nounits",
                                          "-i", str(self.idx), "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons, power = [], None, set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
                power.append(float(f[3]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(power) if power else None}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        # a child process group (the c4 / c5 workloads) gives up sooner: its parent's time limit
        # must end it with an error, not with the whole bench's
        secs = 400 if "--child" in sys.argv else 900
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=secs))

        def barrier():
            dist.barrier()

        def allmax(x):
            import torch
            t = torch.tensor([float(x)], dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return float(t.item())

        def allsum(x):
            import torch
            t = torch.tensor([float(x)], dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.SUM)
            return float(t.item())

        def done():
            dist.destroy_process_group()
    else:
        def barrier():
            pass

        def allmax(x):
            return float(x)

        def allsum(x):
            return float(x)

        def done():
            pass
    return world, rank, local, barrier, allmax, allsum, done


def gpu_smi_index(local_rank):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v.strip() for v in vis.split(",") if v.strip()]
        if local_rank < len(ids) and ids[local_rank].isdigit():
            return int(ids[local_rank])
    return local_rank


# ---------------------------------------------------------------- roofline of the GEMV kernel
def qgemv_roofline(device, reps=10):
    """Time ulb_qgemm (the fused Q4_0 dequant-GEMV) on the 7B verify shapes (M = k+1 = 6 rows):
    per shape, 4 layers' distinct copies are recorded in a CUDA graph and replayed, timed with
    CUDA events on the library's stream; 456 MB of weights in all, so every launch streams its
    weights from HBM (working set > L2)."""
    import numpy as np
    import ulb_capi as U
    ctx = U.Context(device)
    d, f, V = TARGET["d_model"], TARGET["d_ff"], TARGET["n_vocab"]
    shapes = [(3 * d, d), (d, d), (2 * f, d), (d, f)]
    rng = np.random.default_rng(0)
    mats = []
    try:
        for _layer in range(4):
            for (N, K) in shapes:
                raw = rng.integers(0, 256, (N, K // 32, 18), dtype=np.uint8)
                raw[:, :, 0:2] = np.frombuffer(np.float16(0.01).tobytes(), np.uint8)
                mats.append((ctx.upload_tensor(U.T_Q4_0, (K, N), raw.reshape(N, -1)), N, K))
        M = K_SPEC + 1
        xb = ctx.buffer(rng.standard_normal((M, f)).astype(np.float16))
        yb = ctx.buffer(nbytes=M * 2 * f * 4)
        for h, N, K in mats:
            U.check(U.lib().ulb_qgemm(ctx.h, h, xb.ptr, M, yb.ptr, N))
        per = {}
        tot_b = tot_t = 0.0
        for (N, K) in shapes:
            # the 4 layers' copies of this matrix, recorded in a CUDA graph: back-to-back launches
            mine = [(h, n, k) for (h, n, k) in mats if (n, k) == (N, K)]
            g = ctx.capture(lambda: [U.check(U.lib().ulb_qgemm(ctx.h, h, xb.ptr, M, yb.ptr, n)) for h, n, k in mine])
            ms = ctx.time_graph(g, reps) / len(mine)
            U.lib().ulb_graph_free(g)
            alg = q4_0_bytes(N * K) + M * K * 2 + M * N * 4
            per["%dx%d" % (N, K)] = {"ms": ms, "gbs": alg / ms / 1e6}
            tot_b += alg
            tot_t += ms
        for h, _, _ in mats:
            ctx.free_tensor(h)
        xb.free()
        yb.free()
        return {"achieved_gbs": tot_b / tot_t / 1e6, "bytes_per_layer": tot_b, "ms_per_layer": tot_t, "shapes": per}
    finally:
        ctx.close()


# ---------------------------------------------------------------- CPU baseline (oracle port)
def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_port_rounds(tp, dp, rounds, warp=(0.0, 0, 1.0)):
    """`rounds` speculative rounds of the C2 models on the host cores (the oracle port, OpenMP
    over every core this process may use: a launcher's OMP_NUM_THREADS does not shrink it)."""
    from oracle import ulb_oracle as orc
    t, d = orc.Model(tp), orc.Model(dp)
    t0 = time.perf_counter()
    n, stats = orc.bench_rounds(t, d, PROMPT_LEN, K_SPEC, rounds, warp, seed=0, threads=host_cores())
    dt = time.perf_counter() - t0
    t.close()
    d.close()
    return n, dt, stats


def reference_kernels(min_s=0.3):
    """The reference's own CPU kernels (src/cpu_backend/gemm_avx2.cpp:6-25 gemm_avx2_f32 and
    dequantize_cpu.cpp:6-49 dequantize_q4_0_f32, built from its sources with its flags by
    oracle/ref_build.py), timed single-threaded as the reference runs them, at the config-3
    shapes with M = 1.  Their results are not valid (a lane-wise product that reads every
    eighth row of B; 20-byte Q4_0 blocks): the figures are speeds only."""
    import ctypes as C
    import numpy as np
    path = os.path.join(ROOT, "oracle", "_ref", "libref_cpu.so")
    if not os.path.exists(path):
        return {"unavailable": "oracle/_ref/libref_cpu.so not built (oracle/ref_build.py needs the reference tree)"}
    lib = C.CDLL(path)
    lib.ref_gemm_avx2_f32.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint32]
    lib.ref_dequantize_q4_0_f32.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t]
    rng = np.random.default_rng(0)

    def timed(fn):
        fn()
        reps, t0 = 0, time.perf_counter()
        while True:
            fn()
            reps += 1
            dt = time.perf_counter() - t0
            if dt >= min_s:
                return dt / reps

    out = {}
    for (N, K) in ((4096, 4096), (11008, 4096), (4096, 11008)):
        n = N * K
        blocks = np.zeros((n // 32 + 1, 20), np.uint8)  # one block past the range: the decoder reads it
        blocks[:, 4:] = rng.integers(0, 256, (n // 32 + 1, 16), dtype=np.uint8)
        blocks[:, :4] = np.frombuffer(np.float32(0.01).tobytes(), np.uint8)
        dst = np.empty(n, np.float32)
        t_dq = timed(lambda: lib.ref_dequantize_q4_0_f32(blocks.ctypes.data, dst.ctypes.data, n))
        a = rng.standard_normal(K).astype(np.float32)
        b = rng.standard_normal((K, N)).astype(np.float32)
        c = np.empty(N, np.float32)
        t_mm = timed(lambda: lib.ref_gemm_avx2_f32(a.ctypes.data, b.ctypes.data, c.ctypes.data, 1, N, K))
        q4 = n // 32 * 18
        out["%dx%d" % (N, K)] = {
            "dequantize_q4_0_f32_us": t_dq * 1e6, "gemm_avx2_f32_m1_us": t_mm * 1e6,
            "dequant_plus_gemm_us": (t_dq + t_mm) * 1e6,
            "q4_gbs_equivalent": q4 / (t_dq + t_mm) / 1e9}
        del blocks, dst, b
    return {"kind": "reference", "cores": 1,
            "sample": "cpu::dequantize_q4_0_f32 then cpu::gemm_avx2_f32 at M=1 (the reference's CPU linear), "
                      "single-threaded as the reference calls them, g++ -mavx2 -mfma -mf16c -O3 -ffast-math",
            "validity": "numerically invalid: the GEMM multiplies lane-wise and reads every eighth row of B; the "
                        "decoder reads 20-byte blocks (fp32 scale); speeds only",
            "shapes": out}


def cpu_baseline(tp, dp, budget_s=20.0):
    n, dt, _ = cpu_port_rounds(tp, dp, 1)
    rounds = 1
    if dt < budget_s / 3:
        extra = max(1, int(budget_s / dt) - 1)
        n2, dt2, _ = cpu_port_rounds(tp, dp, extra)
        n, dt, rounds = n + n2, dt + dt2, 1 + extra
    return {"value": n / dt, "unit": "tok/s", "cores": host_cores(), "kind": "port",
            "sample": "%d speculative round(s) of the C2 models at context %d (KV caches pre-filled), k=%d, T=0, "
                      "oracle/oracle.c with OpenMP over %d cores; %.1f s" % (rounds, PROMPT_LEN, K_SPEC, host_cores(), dt),
            "reference_kernels": reference_kernels()}


def run_reference(args):
    world, rank, local, barrier, allmax, allsum, done = dist_setup()
    if rank != 0:
        done()
        return 0
    tp, dp = ensure_models_in_child()
    for _ in range(args.warmup):
        cpu_port_rounds(tp, dp, 1)
    toks, tsum = 0, 0.0
    for _ in range(args.steps):
        n, dt, _ = cpu_port_rounds(tp, dp, 1)
        toks += n
        tsum += dt
    value = toks / tsum
    cores = host_cores()
    line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": tsum / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "q4_0xf16->f32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": WORKLOAD, "step": "one speculative round at context 512 on the host cores"},
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": cores, "kind": "port",
                             "sample": "one round per step of the C2 workload at context %d (KV pre-filled), OpenMP "
                                       "over all %d host cores of the box (rank 0 alone; the host is shared by every "
                                       "N); the reference's own CPU path cannot run this loop (its engine computes "
                                       "only Q/K/V and its AVX2 GEMM/dequant are not valid), so the oracle port "
                                       "stands in; the reference's own kernels are timed under reference_kernels"
                                       % (PROMPT_LEN, cores),
                             "reference_kernels": reference_kernels()},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    done()
    return 0


def _timed_generations(api, prompt, cfg, steps, before=None):
    """`steps` generations through the public API; returns summed stats"""
    agg = dict(toks=0, dec_ms=0.0, pre_ms=0.0, launches=0, accepted=0, drafted=0, rounds=0, h2d=0.0, d2h=0.0)
    outs = []
    t0 = time.perf_counter()
    for i in range(steps):
        if before is not None and i > 0:
            before()
        out = api.generate_tokens(prompt, cfg)
        st = api.get_last_stats()
        outs.append(out)
        agg["toks"] += len(out) if out and isinstance(out[0], int) else sum(len(o) for o in out)
        agg["dec_ms"] += st["decode_ms"]
        agg["pre_ms"] += st["prefill_ms"]
        agg["launches"] += st["launches"]
        agg["accepted"] += st["accepted"]
        agg["drafted"] += st["drafted"]
        agg["rounds"] += st["rounds"]
        agg["h2d"], agg["d2h"] = st["h2d_bytes"], st["d2h_bytes"]
    agg["wall"] = time.perf_counter() - t0
    agg["outs"] = outs
    return agg


def run_ours(args):
    world, rank, local, barrier, allmax, allsum, done = dist_setup()
    smi_index = gpu_smi_index(local)
    if world > 1:  # one GPU per rank, chosen before CUDA initialises in this process
        os.environ["CUDA_VISIBLE_DEVICES"] = str(smi_index)
    import vulkangguf as vg
    tp, dp = ensure_models(rank, barrier)
    api = vg.InferenceAPI()
    if not api.load_model(tp) or not api.load_draft_model(dp):
        print("[bench] model load failed", file=sys.stderr)
        return 1
    api.enable_speculative_decoding(True)
    api.set_speculation_length(K_SPEC)

    def cfg_t(temp):
        cfg = vg.GenerationConfig()
        cfg.max_tokens = NEW_TOKENS
        cfg.temperature = temp
        cfg.do_sample = temp > 0
        cfg.seed = 0
        return cfg

    prompt = prompt_for(rank)
    for _ in range(args.warmup):
        api.generate_tokens(prompt, cfg_t(0.0))
    barrier()
    clocks = ClockSampler(smi_index)
    clocks.start()
    g = _timed_generations(api, prompt, cfg_t(0.0), args.steps)
    barrier()
    clk = clocks.stop()
    assert all(o == g["outs"][0] for o in g["outs"]), "greedy generation is not deterministic"
    prof = api.profile_round()
    # config 2 at T = 0.8 (sampled drafts and rejection sampling), a few steps after one warm-up
    api.generate_tokens(prompt, cfg_t(0.8))
    t08_steps = max(1, min(args.steps, 5))
    barrier()
    g8 = _timed_generations(api, prompt, cfg_t(0.8), t08_steps)
    prof8 = api.profile_round()
    tot_toks = allsum(g["toks"])
    max_dec = allmax(g["dec_ms"])
    max_wall = allmax(g["wall"])
    max_step = allmax((g["dec_ms"] + g["pre_ms"]) / args.steps)
    tot_launch = allsum(g["launches"])
    value = tot_toks / (max_dec / 1e3)
    e2e = tot_toks / max_wall
    value8 = allsum(g8["toks"]) / (allmax(g8["dec_ms"]) / 1e3)
    e2e8 = allsum(g8["toks"]) / allmax(g8["wall"])
    line = None
    if rank == 0:
        peak, peak_src = load_peaks()
        ctx_len = PROMPT_LEN + NEW_TOKENS
        verify_bytes = (q4_0_bytes(linear_weights(TARGET)) + kv_bytes_per_token(TARGET) * ctx_len
                        + (K_SPEC + 1) * kv_bytes_per_token(TARGET) + (K_SPEC + 1) * TARGET["n_vocab"] * 4)
        verify_gbs = verify_bytes / (prof["verify_ms"] / 1e3) / 1e9
        draft_bytes = K_SPEC * (q4_0_bytes(linear_weights(DRAFT)) + kv_bytes_per_token(DRAFT) * ctx_len)
        draft_gbs = draft_bytes / (prof["draft_ms"] / 1e3) / 1e9
        rl = qgemv_roofline(0)
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": max_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "q4_0xf16->f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "parallelism": "replicas (one sequence per GPU, no collective)",
                       "l2": "inputs larger than L2 (3.7 GB of target weights per verify)",
                       "timed": "generation phase, CUDA events on the engine stream; prefill reported separately"},
            "acceptance_rate": g["accepted"] / g["drafted"] if g["drafted"] else 0.0,
            "rounds_per_step": g["rounds"] / args.steps,
            "prefill_ms": g["pre_ms"] / args.steps,
            "decode_ms": g["dec_ms"] / args.steps,
            "round_profile_ms": prof,
            "verify": {"bytes": verify_bytes, "ms": prof["verify_ms"], "gbs": verify_gbs,
                       "frac": verify_gbs / peak, "peak": peak, "peak_source": peak_src,
                       "frac_of_8tbs": verify_gbs / 8000.0},
            "draft": {"bytes": draft_bytes, "ms": prof["draft_ms"], "steps": K_SPEC, "gbs": draft_gbs,
                      "frac": draft_gbs / peak, "note": "k draft steps of one round: TinyLlama weights + KV read"},
            "t08": {"value": value8, "unit": "tok/s", "e2e": e2e8, "steps": t08_steps,
                    "acceptance_rate": g8["accepted"] / g8["drafted"] if g8["drafted"] else 0.0,
                    "rounds_per_step": g8["rounds"] / t08_steps, "round_profile_ms": prof8,
                    "config": "config 2 at T=0.8 (no top-k / top-p), Philox seed 0"},
            "value_t08": value8,
            "roofline": {"bound": "hbm", "achieved": rl["achieved_gbs"], "peak": peak, "unit": "GB/s",
                         "frac": rl["achieved_gbs"] / peak,
                         "traffic": rl["bytes_per_layer"] / 4 * QGEMV_TRAFFIC_RATIO,
                         "traffic_note": "bytes per average launch: algorithmic bytes x %.3f, the DRAM read+write / "
                                         "algorithmic ratio of an ncu capture of the Q4_0 11008x4096 M=5 launch "
                                         "(no re-reads)" % QGEMV_TRAFFIC_RATIO,
                         "kernel": "qgemv_kernel<Q4_0, NT=1> (warp-streamed fused Q4_0 dequant-GEMV, 7B verify shapes, M=6)",
                         "peak_source": peak_src + " (MEASURED_PEAKS.json hbm_gbs)" if peak_src == "measured" else peak_src,
                         "shapes": rl["shapes"]},
            "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": g["h2d"], "d2h_bytes_per_step": g["d2h"],
                    "note": "public API generate_tokens (host prompt in, host tokens out), prefill included"},
            "gpu_launches": int(tot_launch),
            "clocks": clk,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(tp, dp)
    # the GPU memory of the C2 models goes back before the sharded workloads run
    del api
    import gc
    gc.collect()
    barrier()
    for wl in extras_for(args, world):
        obj = run_child(wl, args, world, rank, barrier)
        if line is not None:
            line[wl] = obj
    if line is not None:
        print(json.dumps(line), flush=True)
    done()
    return 0


def run_pgtest(args):
    """Process-group plumbing of the child workloads without a GPU (for tests on the CPU):
    parent ranks spawn one child each, the children form their own gloo group, all-reduce
    their ranks and rank 0's child prints a JSON line the parent folds into its own."""
    world, rank, local, barrier, allmax, allsum, done = dist_setup()
    if args.child:
        total = allsum(rank)
        if rank == 0:
            print(json.dumps({"world": world, "rank_sum": total}), flush=True)
        done()
        return 0
    obj = run_child("pgtest", args, world, rank, barrier)
    if rank == 0:
        print(json.dumps({"pgtest": obj}), flush=True)
    done()
    return 0


def extras_for(args, world):
    if args.child or args.extras == "none":
        return []
    if args.extras == "auto":
        return ["c4"] + (["c5"] if world >= 2 else [])
    return [w for w in args.extras.split(",") if w in ("c4", "c5")]


# wall-clock budget of one bench run (the sharded workloads get what the headline leaves)
BENCH_BUDGET_S = float(os.environ.get("ULB_BENCH_BUDGET_S", "840"))
CHILD_CAP_S = {"c4": 300.0, "c5": 480.0, "pgtest": 120.0}


def run_child(wl, args, world, rank, barrier):
    """Run workload `wl` as its own process group (one child per rank, the same rank / world,
    a port of its own) and return rank 0's JSON line as an object; an error or a timeout in the
    child is reported, not raised."""
    left = BENCH_BUDGET_S - (time.time() - T_START) - 20.0
    timeout = min(CHILD_CAP_S[wl], left)
    obj = None
    if timeout < 60:
        obj = {"skipped": "%.0f s of the bench's %.0f s budget left" % (max(left, 0), BENCH_BUDGET_S)}
    else:
        # the children form a process group of their own: without torchrun's agent store (with
        # TORCHELASTIC_USE_AGENT_STORE set, rank 0 would connect to a store nobody serves)
        env = {k: v for k, v in os.environ.items() if not k.startswith("TORCHELASTIC")}
        if ORIG_CUDA_VISIBLE is None:
            env.pop("CUDA_VISIBLE_DEVICES", None)
        else:
            env["CUDA_VISIBLE_DEVICES"] = ORIG_CUDA_VISIBLE
        if world > 1:
            env["MASTER_PORT"] = str(int(os.environ.get("MASTER_PORT", "29500")) + {"c4": 11, "c5": 13}.get(wl, 17))
        if wl == "c5":
            env.setdefault("NCCL_DEBUG", "INFO")
            env.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
        cmd = [sys.executable, os.path.abspath(__file__), "--workload", wl, "--steps", "1", "--warmup", "1",
               "--gpus", str(world), "--child"]
        t0 = time.time()
        try:
            r = subprocess.run(cmd, env=env, stdout=subprocess.PIPE, text=True, timeout=timeout)
            out, rc = r.stdout, r.returncode
        except subprocess.TimeoutExpired as e:
            out = e.stdout.decode() if isinstance(e.stdout, bytes) else (e.stdout or "")
            rc = "killed after %.0f s (time limit)" % timeout
        parsed = None
        for ln in out.splitlines():
            if ln.startswith("{"):
                try:
                    parsed = json.loads(ln)
                    continue
                except ValueError:
                    pass
            print(ln, file=sys.stderr)
        if rank == 0:
            obj = parsed if (parsed is not None and rc == 0) else {"error": "child exit %s" % rc, "partial": parsed}
            obj["child_wall_s"] = time.time() - t0
    barrier()
    return obj


# Llama-2-70B-arch Q4_0 target (N(0, 0.02), seed 0), tensor-parallel over the GPUs with an
# all-reduce after attn-out and FFN-down; Llama-2-7B-arch Q4_0 draft replicated per GPU; batch 8, 2048-token
# prompts, k = 6, T = 0
C5_TARGET = dict(n_layer=80, d_model=8192, n_head=64, n_head_kv=8, d_ff=28672, n_vocab=32000, rms_eps=1e-5,
                 rope_base=1e4, wtype="q4_0", seed=0, ctx_len=4096, name="llama2-70b-arch-q4_0-s0")
C5_SEQS, C5_PROMPT, C5_K, C5_NEW = 8, 2048, 6, 256
C5_WORKLOAD = ("C5: Llama-2-70B-arch Q4_0 target tensor-parallel over the GPUs (all-reduce after attn-out and "
               "FFN-down) + Llama-2-7B-arch Q4_0 draft replicated per GPU, batch 8, 2048-token prompts, k=6, "
               "256 new tokens, T=0")


def run_c5(args):
    """Config 5: every rank holds 1/N of the 70B target's heads and FFN features and all of the
    7B draft; all ranks decode the same 8 sequences in lock step (NCCL all-reduces inside each
    target forward), so tokens are counted once."""
    world, rank, local, barrier, allmax, allsum, done = dist_setup()
    smi_index = gpu_smi_index(local)
    if world > 1:
        os.environ["CUDA_VISIBLE_DEVICES"] = str(smi_index)
    import numpy as np
    import vulkangguf as vg
    tp, dp = ensure_models(rank, barrier, C5_TARGET, TARGET)
    api = vg.InferenceAPI()
    mon = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        from ulb_tp import PeerMonitor
        box = [vg.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        if not api.init_tensor_parallel(rank, world, box[0]):
            print("[bench] tensor-parallel init failed", file=sys.stderr)
            return 1
        # a lost rank is found on the host between generations (PeerMonitor), and a wait for a
        # collective whose peer is gone mid-generation gives up (set_collective_timeout)
        store = dist.TCPStore(os.environ.get("MASTER_ADDR", "127.0.0.1"), int(os.environ["MASTER_PORT"]) + 1, world,
                              rank == 0, timeout=datetime.timedelta(seconds=120))
        mon = PeerMonitor(store, rank, world, timeout_s=120.0)
        api.set_collective_timeout(300.0)
    step = [0]

    def peers_ready():
        if mon is not None:
            mon.wait_step(step[0])
        step[0] += 1
    t_load = time.time()
    if not api.load_model(tp) or not api.load_draft_model(dp):
        print("[bench] model load failed", file=sys.stderr)
        return 1
    t_load = time.time() - t_load
    api.enable_speculative_decoding(True)
    api.set_speculation_length(C5_K)
    rng = np.random.default_rng(1)
    prompts = [rng.integers(0, C5_TARGET["n_vocab"], C5_PROMPT).astype(np.int32).tolist() for _ in range(C5_SEQS)]

    def cfg(n):
        c = vg.GenerationConfig()
        c.max_tokens, c.temperature, c.do_sample, c.seed = n, 0.0, False, 0
        return c

    for _ in range(args.warmup):  # warm-up generations: every kernel shape and the round graph
        peers_ready()
        api.generate_tokens(prompts, cfg(8))
    peers_ready()
    barrier()
    clocks = ClockSampler(smi_index)
    clocks.start()
    g = _timed_generations(api, prompts, cfg(C5_NEW), args.steps, before=peers_ready)
    barrier()
    clk = clocks.stop()
    prof = api.profile_round()
    max_dec = allmax(g["dec_ms"])
    max_wall = allmax(g["wall"])
    max_step = allmax((g["dec_ms"] + g["pre_ms"]) / args.steps)
    tot_launch = allsum(g["launches"])
    verify_ms = allmax(prof["verify_ms"])
    ar_ms = allmax(prof.get("allreduce_ms", 0.0))
    if rank != 0:
        done()
        return 0
    peak, peak_src = load_peaks()
    ctx_len = C5_PROMPT + C5_NEW // 2
    w_bytes = q4_0_bytes(linear_weights(C5_TARGET))
    hd = C5_TARGET["d_model"] // C5_TARGET["n_head"]
    kv_tok = C5_TARGET["n_layer"] * C5_TARGET["n_head_kv"] * hd * 2 * 2
    # per GPU and verify: the rank's weight slice (the LM head is replicated) + its KV heads
    lm_head = q4_0_bytes(C5_TARGET["d_model"] * C5_TARGET["n_vocab"])
    verify_bytes = (w_bytes - lm_head) / world + lm_head + C5_SEQS * ctx_len * kv_tok / world
    gbs = verify_bytes / (verify_ms / 1e3) / 1e9
    rows = C5_SEQS * (C5_K + 1)
    ar_bytes = rows * C5_TARGET["d_model"] * 4  # one fp32 all-reduce payload (attn_output or ffn_down partials)
    line = {
        "metric": "accepted tok/s (Llama-2-70B-arch Q4_0 tensor-parallel, batch 8, k=6)",
        "value": g["toks"] / (max_dec / 1e3), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": max_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "q4_0xf16->f32", "data": "synthetic",
        "config": {"workload": C5_WORKLOAD, "parallelism": "tp%d (NCCL all-reduce, fp32 partial sums)" % world,
                   "l2": "inputs larger than L2 (38.6 GB of target weights)", "warmup_tokens": 8,
                   "timed": "generation phase, CUDA events, max over ranks; prefill separate"},
        "acceptance_rate": g["accepted"] / g["drafted"] if g["drafted"] else 0.0,
        "rounds_per_step": g["rounds"] / args.steps,
        "prefill_ms": g["pre_ms"] / args.steps, "decode_ms": g["dec_ms"] / args.steps,
        "load_s": t_load,
        "round_profile_ms": prof,
        "allreduce": {"ms_per_verify": ar_ms, "count_per_verify": prof.get("allreduces", 0),
                      "bytes_each": ar_bytes, "share_of_verify": ar_ms / verify_ms if verify_ms else None,
                      "note": "CUDA events on the engine stream around each ncclAllReduce of one profiled round "
                              "(includes waiting for the slowest rank), max over ranks"},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                     "traffic": None, "kernel": "target verify forward of one round per GPU (weights slice + KV)",
                     "peak_source": peak_src},
        "e2e": {"value": g["toks"] / max_wall, "unit": "tok/s", "h2d_bytes_per_step": g["h2d"],
                "d2h_bytes_per_step": g["d2h"], "note": "public API generate_tokens, prefill included"},
        "gpu_launches": int(tot_launch),
        "clocks": clk,
    }
    print(json.dumps(line), flush=True)
    done()
    return 0


def c4_prompts():
    """The 64 config-4 prompts (lengths U[256, 4096], ids U[0, vocab), seed 1)."""
    import numpy as np
    rng = np.random.default_rng(1)
    lens = rng.integers(C4_CTX[0], C4_CTX[1] + 1, C4_SEQS)
    return [rng.integers(0, C4_TARGET["n_vocab"], int(n)).astype(np.int32).tolist() for n in lens]


def shard(items, rank, world):
    """Round-robin data-parallel shard of the sequences: rank r decodes items r, r + N, ..."""
    return items[rank::world]


def run_c4(args):
    """Config 4, data-parallel: each rank decodes its 64/N sequences on its own GPU with its own
    replica of both models; no collective on the data path (the host reduces counts and times)."""
    world, rank, local, barrier, allmax, allsum, done = dist_setup()
    smi_index = gpu_smi_index(local)
    if world > 1:
        os.environ["CUDA_VISIBLE_DEVICES"] = str(smi_index)
    import vulkangguf as vg
    tp, dp = ensure_models(rank, barrier, C4_TARGET, C4_DRAFT)
    api = vg.InferenceAPI()
    if not api.load_model(tp) or not api.load_draft_model(dp):
        print("[bench] model load failed", file=sys.stderr)
        return 1
    api.enable_speculative_decoding(True)
    api.set_speculation_length(C4_K)
    prompts = shard(c4_prompts(), rank, world)

    def cfg(n):
        c = vg.GenerationConfig()
        c.max_tokens, c.temperature, c.top_p, c.top_k, c.do_sample, c.seed = n, 0.8, 0.9, 0, True, 0
        return c

    for _ in range(args.warmup):  # warm-up generations: every kernel shape and the round graph
        api.generate_tokens(prompts, cfg(8))
    barrier()
    clocks = ClockSampler(smi_index)
    clocks.start()
    g = _timed_generations(api, prompts, cfg(C4_NEW), args.steps)
    barrier()
    clk = clocks.stop()
    prof = api.profile_round()
    tot_toks = allsum(g["toks"])
    max_dec = allmax(g["dec_ms"])
    max_wall = allmax(g["wall"])
    max_step = allmax((g["dec_ms"] + g["pre_ms"]) / args.steps)
    tot_launch = allsum(g["launches"])
    verify_ms = allmax(prof["verify_ms"])
    draft_ms = allmax(prof["draft_ms"])
    rows = len(prompts) * (C4_K + 1)
    # KV bytes one verify of this rank reads: its sequences' caches at mid-generation
    ctx_sum = sum(len(p) for p in prompts) + len(prompts) * C4_NEW // 2
    kv_read = allmax(ctx_sum * kv_bytes_per_token(C4_TARGET))
    if rank != 0:
        done()
        return 0
    hd = C4_TARGET["d_model"] // C4_TARGET["n_head"]
    w_per_layer = C4_TARGET["d_model"] * hd * (C4_TARGET["n_head"] * 2 + C4_TARGET["n_head_kv"] * 2) + \
        3 * C4_TARGET["d_model"] * C4_TARGET["d_ff"]
    n_w = C4_TARGET["n_layer"] * w_per_layer + C4_TARGET["d_model"] * C4_TARGET["n_vocab"]
    flop = 2.0 * n_w * rows  # verify GEMM work of one round on one GPU (64/N sequences x (k+1) rows)
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except Exception:
        pass
    tf_peak = float(peaks.get("bf16_tflops_sustained", 1385.6))
    hbm_peak = float(peaks.get("hbm_gbs", 6650.0))
    achieved = flop / (verify_ms / 1e3) / 1e12
    verify_bytes = n_w * 144 / 256 + kv_read + rows * C4_TARGET["n_vocab"] * 4
    line = {
        "metric": "accepted tok/s (Llama-3-8B-arch Q4_K, 64 sequences, k=8, T=0.8, top_p=0.9), data-parallel",
        "value": tot_toks / (max_dec / 1e3), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": max_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "q4_kxf16->f32", "data": "synthetic",
        "config": {"workload": C4_WORKLOAD, "parallelism": "dp%d (sequences sharded, no collective)" % world,
                   "sequences_per_gpu": len(prompts), "l2": "inputs larger than L2 (4.2 GB of weights, ~18 GB KV)",
                   "warmup_tokens": 8, "timed": "generation phase, CUDA events, max over ranks; prefill separate"},
        "sequences_per_gpu": len(prompts),
        "acceptance_rate": g["accepted"] / g["drafted"] if g["drafted"] else 0.0,
        "rounds_per_step": g["rounds"] / args.steps,
        "prefill_ms": g["pre_ms"] / args.steps, "decode_ms": g["dec_ms"] / args.steps,
        "round_profile_ms": prof,
        "verify": {"rows": rows, "ms": verify_ms, "tflops": achieved, "tflops_frac": achieved / tf_peak,
                   "bytes": verify_bytes, "gbs": verify_bytes / (verify_ms / 1e3) / 1e9,
                   "hbm_frac": verify_bytes / (verify_ms / 1e3) / 1e9 / hbm_peak, "draft_ms": draft_ms},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": tf_peak, "unit": "TFLOP/s",
                     "frac": achieved / tf_peak, "traffic": None,
                     "kernel": "verify forward of one round (tcgen05 dequant-GEMM at %d rows + attention)" % rows,
                     "peak_source": "MEASURED_PEAKS.json bf16_tflops_sustained" if peaks else "fallback"},
        "e2e": {"value": tot_toks / max_wall, "unit": "tok/s", "h2d_bytes_per_step": g["h2d"],
                "d2h_bytes_per_step": g["d2h"],
                "note": "public API generate_tokens on each rank's sequences, prefill included"},
        "gpu_launches": int(tot_launch),
        "clocks": clk,
    }
    print(json.dumps(line), flush=True)
    done()
    return 0


def _rand_q4(rng, qt, N, K):
    import numpy as np
    if qt == "q4_0":
        raw = rng.integers(0, 256, (N, K // 32, 18), dtype=np.uint8)
        raw[:, :, 0:2] = np.frombuffer(np.float16(0.01).tobytes(), np.uint8)
    else:
        raw = rng.integers(0, 256, (N, K // 256, 144), dtype=np.uint8)
        raw[:, :, 0:2] = np.frombuffer(np.float16(0.002).tobytes(), np.uint8)
        raw[:, :, 2:4] = np.frombuffer(np.float16(0.001).tobytes(), np.uint8)
    return raw.reshape(N, -1)


TRACE_UNITS = ("qgemv", "attention", "model", "sampling", "spec", "qgemm_tc", "runtime")
# one CTA record of the trace build (ulb::TraceRec)
TRACE_REC = [("tag", "<u4"), ("cta", "<u4"), ("grid", "<u4"), ("arg", "<u4"), ("t_entry", "<u8"),
             ("t_wait", "<u8"), ("t_exit", "<u8"), ("pad", "<u8"), ("mark", "<u8", (8,))]
TRACE_NAMES = {6000: "embed", 6100: "rmsnorm", 6200: "add", 7000: "sample", 7100: "stats", 7200: "accept",
               7300: "tree_children", 7400: "tree_decide", 8000: "stage_draft", 8100: "stage_verify",
               8200: "stage_prefill", 8300: "stage_tree_draft", 8301: "stage_tree_verify", 8350: "kv_tree_compact",
               9000: "wait_flag"}


def trace_kernel_name(tag, arg):
    if 1000 <= tag < 2000:
        epi = {0: "store", 1: "resid", 2: "swiglu", 3: "qkv"}.get((tag - 1000) // 100, "?")
        return "qgemv_%s_N%d%s" % (epi, arg, "_rmsnorm" if tag % 10 else "")
    if 2000 <= tag < 3000:
        return "attn_split_hd%d%s%s" % (arg, "_cluster" if tag & 1 else "", "_tree" if tag & 2 else "")
    if 3000 <= tag < 4000:
        return "attn_stream_hd%d_tiles%d" % (arg, tag - 3000)
    if 4000 <= tag < 5000:
        return "qgemm_tc_epi%d_nt%d" % (tag - 4000, arg)
    if 5000 <= tag < 6000:
        return "rowgemv_N%d" % arg
    return TRACE_NAMES.get(tag, str(tag))


def trace_launches(rings):
    """CTA records of every unit, within the window all busy rings still cover, grouped into
    launches (consecutive entries of one kernel with distinct CTA indices)."""
    import numpy as np
    live = [r[r["t_entry"] > 0] for r in rings]
    busy = [r for r in live if len(r) > 1000]
    t_min = max(int(r["t_entry"].min()) for r in busy) if busy else 0
    rec = np.concatenate(live)
    rec = rec[rec["t_entry"] >= t_min]
    rec = rec[np.argsort(rec["t_entry"], kind="stable")]
    # a record joins the open launch of its kernel (tag, argument, grid) unless that launch
    # already holds its CTA index or is full; under programmatic dependent launch at most two
    # consecutive launches overlap, and consecutive launches of one kernel do not
    launches, open_l = [], {}
    for x in rec:
        key = (int(x["tag"]), int(x["arg"]), int(x["grid"]))
        cur = open_l.get(key)
        if cur is None or int(x["cta"]) in cur["seen"] or len(cur["seen"]) >= key[2]:
            cur = {"key": key, "recs": [], "seen": set()}
            open_l[key] = cur
            launches.append(cur)
        cur["recs"].append(x)
        cur["seen"].add(int(x["cta"]))
    out = []
    for l in launches:
        r = np.array(l["recs"], dtype=rec.dtype)
        waits = r["t_wait"][r["t_wait"] > 0]
        last = r[int(np.argmax(r["t_exit"]))]
        out.append({"name": trace_kernel_name(*l["key"][:2]), "ctas": len(r), "entry": int(r["t_entry"].min()),
                    "wait": int(waits.max()) if len(waits) else 0, "exit": int(r["t_exit"].max()),
                    "last_marks": [int(m) - int(last["t_wait"]) if m and last["t_wait"] else None for m in last["mark"]]})
    out.sort(key=lambda l: l["exit"])  # a kernel completes after the one before it in the stream
    return out


def run_trace(args):
    """Timeline of one C2 round from the trace build (libulb_cuda_trace.so: every kernel's CTAs
    record the global-timer times of their entry, of the return of their wait for the previous
    kernel and of their exit, plus marks inside the GEMV and the per-split attention).  The
    traced generation is the bench's C2 workload shortened to 64 tokens; its last complete
    round is reported kernel by kernel: `exposed` = this launch's last CTA exit - the previous
    launch's, `after_wait` = its last exit - its last wait, and the marks of the CTA that
    exits last, relative to its own wait."""
    import ctypes as C
    import numpy as np
    import build as pbuild
    lib_path = pbuild.build_cuda(trace=True)
    lib = C.CDLL(lib_path, mode=C.RTLD_GLOBAL)  # the Python module binds to it (same soname)
    import vulkangguf as vg
    maps = open("/proc/self/maps").read()
    assert "/libulb_cuda.so" not in maps and "libulb_cuda_trace.so" in maps, "the trace build is not the one loaded"
    rec_t = np.dtype(TRACE_REC)
    cap = 1 << 18

    def dump():
        rings = []
        for u in TRACE_UNITS:
            buf = np.zeros(cap, rec_t)
            n = C.c_uint(0)
            rc = getattr(lib, "ulb_trace_dump_" + u)(buf.ctypes.data_as(C.c_void_p), C.byref(n))
            assert rc == 0, (u, rc)
            rings.append(buf)
        return rings

    c4 = args.workload == "c4"
    tp, dp = ensure_models(0, lambda: None, *((C4_TARGET, C4_DRAFT) if c4 else ()))
    api = vg.InferenceAPI()
    if not api.load_model(tp) or not api.load_draft_model(dp):
        return 1
    api.enable_speculative_decoding(True)
    api.set_speculation_length(C4_K if c4 else K_SPEC)
    cfg = vg.GenerationConfig()
    if c4:  # config 4 on one GPU: 64 sequences, T = 0.8, top_p = 0.9, a few rounds
        cfg.max_tokens, cfg.temperature, cfg.top_p, cfg.top_k, cfg.do_sample, cfg.seed = 24, 0.8, 0.9, 0, True, 0
        prompt = c4_prompts()
    else:
        cfg.max_tokens, cfg.temperature, cfg.do_sample = 64, 0.0, False
        prompt = prompt_for(0)
    for _ in range(max(1, args.warmup)):
        api.generate_tokens(prompt, cfg)
    dump()
    api.generate_tokens(prompt, cfg)
    rings = dump()
    if args.trace_dump:  # the raw records, for analyses of one's own
        np.savez_compressed(args.trace_dump, **{u: r for u, r in zip(TRACE_UNITS, rings)})
    L = trace_launches(rings)
    acc = [i for i, l in enumerate(L) if l["name"] == "accept"]
    if len(acc) < 2:
        print(json.dumps({"mode": "trace", "error": "fewer than two rounds in the trace"}))
        return 1
    a, b = acc[-2] + 1, acc[-1] + 1
    rnd = L[a:b]
    phase, prev, agg = "draft", L[a - 1]["exit"], {}
    for l in rnd:
        if l["name"] == "stage_verify":
            phase = "verify"
        if l["name"] == "accept":
            phase = "accept"
        exposed = (l["exit"] - prev) / 1e3
        after = (l["exit"] - l["wait"]) / 1e3 if l["wait"] else 0.0
        prev = l["exit"]
        g = agg.setdefault((phase, l["name"]), {"phase": phase, "kernel": l["name"], "launches": 0, "ctas": l["ctas"],
                                                "exposed_us": 0.0, "after_wait_us": 0.0, "marks": []})
        g["launches"] += 1
        g["exposed_us"] += exposed
        g["after_wait_us"] += after
        g["marks"].append(l["last_marks"])
    kernels, phases = [], {}
    for g in agg.values():
        n = g["launches"]
        mk = np.array([[np.nan if m is None else m / 1e3 for m in ms] for ms in g.pop("marks")])
        means = [round(float(np.nanmean(mk[:, j])), 2) for j in range(8) if not np.all(np.isnan(mk[:, j]))]
        g.update(exposed_us=round(g["exposed_us"], 1), mean_exposed_us=round(g["exposed_us"] / n, 2),
                 mean_after_wait_us=round(g["after_wait_us"] / n, 2), last_cta_marks_after_wait_us=means)
        phases[g["phase"]] = round(phases.get(g["phase"], 0.0) + g["exposed_us"], 1)
        kernels.append(g)
    wl = ("c4 round (64 sequences, k=8, T=0.8, top_p=0.9), 24-token generation" if c4 else
          "c2 round (k=5, T=0), 64-token generation after a 512-token prompt")
    print(json.dumps({"mode": "trace", "workload": wl,
                      "round_us": round((rnd[-1]["exit"] - L[a - 1]["exit"]) / 1e3, 1), "launches": len(rnd),
                      "phases_us": phases, "kernels": kernels}), flush=True)
    return 0


def run_ops(args):
    """Config-3 op sweep on one GPU: fused Q4_0 / Q4_K dequant-GEMM for (N, K) in
    {(4096,4096), (11008,4096), (4096,11008)} x M in {1,5,8,16,64,256}, and the rejection
    kernel at p [64, 9, 32000] / q [64, 8, 32000], and the attention kernel at the verify / draft
    shapes.  Each case's launches are recorded in a CUDA graph and replayed, timed with CUDA
    events on the library stream (so host call overhead is not in the figure); enough distinct
    weight copies are cycled that every GEMM launch streams its weights from HBM."""
    import ctypes as C
    import numpy as np
    import ulb_capi as U
    peak, peak_src = load_peaks()
    ctx = U.Context(0)
    rng = np.random.default_rng(0)
    cases = []
    for qt in ("q4_0", "q4_k"):
        for (N, K) in ((4096, 4096), (11008, 4096), (4096, 11008)):
            for M in (1, 5, 8, 16, 64, 256):
                name = "%s:%dx%d:m%d" % (qt, N, K, M)
                if args.only and args.only != name and not name.startswith(args.only):
                    continue
                cases.append((qt, N, K, M, name))
    results = {}
    cache = {}
    for qt, N, K, M, name in cases:
        key = (qt, N, K)
        if key not in cache:
            copies = max(2, int(300e6 // (N * K * 0.5625)) + 1)  # > 2x L2 of weights
            cache.clear()
            cache[key] = [ctx.upload_tensor(U.T_Q4_0 if qt == "q4_0" else U.T_Q4_K, (K, N), _rand_q4(rng, qt, N, K))
                          for _ in range(copies)]
        mats = cache[key]
        xb = ctx.buffer(rng.standard_normal((M, K)).astype(np.float16))
        yb = ctx.buffer(nbytes=M * N * 4)
        for h in mats[: max(1, args.warmup)]:
            U.check(U.lib().ulb_qgemm(ctx.h, h, xb.ptr, M, yb.ptr, N))
        # one launch per weight copy, recorded in a CUDA graph so the device runs them back to back
        g = ctx.capture(lambda: [U.check(U.lib().ulb_qgemm(ctx.h, h, xb.ptr, M, yb.ptr, N)) for h in mats])
        ms = ctx.time_graph(g, max(args.steps, 3)) / len(mats)
        U.lib().ulb_graph_free(g)
        alg = N * K * 0.5625 + 2 * M * K + 4 * M * N
        results[name] = {"us": ms * 1e3, "gbs": alg / ms / 1e6, "hbm_frac": alg / ms / 1e6 / peak,
                         "tflops": 2.0 * M * N * K / ms / 1e9}
        xb.free()
        yb.free()
    for mats in cache.values():
        for h in mats:
            ctx.free_tensor(h)
    # block-causal attention of the verify / draft rows against a KV cache (ulb_attention_noalloc:
    # no allocation or synchronisation inside the timed loop); bytes = the K/V rows read
    # (label, heads, kv heads, head dim, rows per sequence, sequences, context): one sequence at the
    # config-2 verify / draft shapes, and config 4's 64 sequences (contexts U[256, 4096] + 128, seed 1)
    # for the verify (9 rows, hd 128) and the draft (1 row, hd 64)
    c4_ctx = np.random.default_rng(1).integers(256, 4097, 64) + 128
    for (label, H, Hkv, hd, rps, S, Ls) in (("attn:7b_verify", 32, 32, 128, 6, 1, [768]),
                                            ("attn:tinyllama_draft", 32, 4, 64, 2, 1, [768]),
                                            ("attn:7b_verify_4k", 32, 32, 128, 6, 1, [4096]),
                                            ("attn:c4_verify", 32, 8, 128, 9, 64, c4_ctx),
                                            ("attn:c4_draft", 32, 8, 64, 1, 64, c4_ctx)):
        if args.only and not label.startswith(args.only):
            continue
        cap = int(max(Ls)) + 8
        desc = U.AttnDesc(H, Hkv, hd, cap, S, 1.0 / float(np.sqrt(hd)))
        M = S * rps
        q = rng.standard_normal((M, H * hd)).astype(np.float32)
        kc = (rng.standard_normal((S, Hkv, cap, hd), dtype=np.float32)).astype(np.float16)
        vc = (rng.standard_normal((S, Hkv, cap, hd), dtype=np.float32)).astype(np.float16)
        rs = np.repeat(np.arange(S, dtype=np.int32), rps)
        rp = np.concatenate([np.arange(int(L) - rps, int(L), dtype=np.int32) for L in Ls])
        bufs = [ctx.buffer(a) for a in (q, kc, vc, rs, rp)]
        out = ctx.buffer(nbytes=M * H * hd * 2)
        call = lambda: U.check(U.lib().ulb_attention_noalloc(ctx.h, C.byref(desc), bufs[0].ptr, bufs[1].ptr, bufs[2].ptr,
                                                             bufs[3].ptr, bufs[4].ptr, M, rps, out.ptr))
        for _ in range(max(1, args.warmup)):
            call()
        ctx.sync()
        reps = 20 if S == 1 else 4
        g = ctx.capture(lambda: [call() for _ in range(reps)])  # each call: counter reset + kernel
        ms = ctx.time_graph(g, max(args.steps, 3)) / reps
        U.lib().ulb_graph_free(g)
        kv = 2 * int(sum(int(L) for L in Ls)) * Hkv * hd * 2
        alg = kv + q.nbytes + M * H * hd * 2
        results[label] = {"us": ms * 1e3, "gbs": alg / ms / 1e6, "hbm_frac": alg / ms / 1e6 / peak,
                          "note": ("K/V of one sequence (%.1f MB) fit in L2: a latency figure" % (kv / 1e6)) if S == 1
                          else "K/V of %d sequences: %.0f MB" % (S, kv / 1e6)}
        for b in bufs + [out]:
            b.free()
    # rejection sampling: config 3's [64, 9 | 8, 32000] at T = 1 and T = 0, and config 4's vocabulary
    # (128256) at T = 0.8, top_p = 0.9; draft sampling of 64 rows at config 4's warp
    for (label, V, warps) in (("accept", 32000, ((1.0, 0, 1.0), (0.0, 0, 1.0))),
                              ("accept_c4", 128256, ((0.8, 0, 0.9),))):
        if args.only and not label.startswith(args.only) and args.only.split(":")[0] != label:
            continue
        B, k = 64, 8
        pl = (rng.standard_normal((B, k + 1, V)) * 3).astype(np.float32)
        ql = (rng.standard_normal((B, k, V)) * 3).astype(np.float32)
        bp, bq = ctx.buffer(pl), ctx.buffer(ql)
        ot, on = ctx.buffer(nbytes=B * (k + 1) * 4), ctx.buffer(nbytes=B * 4)
        st = ctx.buffer(nbytes=B * 4)
        for warp in warps:
            w = U.Warp(*warp)
            # the drafts as the loop makes them: token i of each sequence drawn from q_i under the warp
            draft = np.zeros((B, k), np.int32)
            tb = ctx.buffer(nbytes=B * 4)
            for i in range(k):
                U.check(U.lib().ulb_sample(ctx.h, C.c_void_p(bq.ptr.value + i * V * 4), B, V, k * V, C.byref(w), 7, 0,
                                           i, U.RNG_DRAFT, tb.ptr))
                draft[:, i] = tb.download(np.int32, (B,))
            tb.free()
            bd = ctx.buffer(draft)
            for _ in range(max(1, args.warmup)):
                U.check(U.lib().ulb_spec_accept(ctx.h, bp.ptr, bq.ptr, bd.ptr, B, k, V, C.byref(w), 1, 0, ot.ptr, on.ptr))
            ctx.sync()
            g = ctx.capture(lambda: [U.check(U.lib().ulb_spec_accept(ctx.h, bp.ptr, bq.ptr, bd.ptr, B, k, V, C.byref(w),
                                                                      1, r, ot.ptr, on.ptr)) for r in range(4)])
            ms = ctx.time_graph(g, max(args.steps, 3)) / 4
            U.lib().ulb_graph_free(g)
            # the walk reads p_i (and q_i when sampling) for each position it tests, and p_k after a
            # full accept: the algorithmic bytes of the rows it needs
            n_acc = on.download(np.int32, (B,))
            rows = sum(min(int(n) + 1, k) * (1 if warp[0] <= 0 else 2) + (1 if n == k else 0) for n in n_acc)
            alg = rows * V * 4
            name = "%s:T%g%s" % (label, warp[0], ":top_p%g" % warp[2] if warp[2] < 1 else "")
            results[name] = {"us": ms * 1e3, "gbs": alg / ms / 1e6, "hbm_frac": alg / ms / 1e6 / peak,
                             "rows_read": rows, "rows_total": B * (2 * k + 1),
                             "accepted_mean": float(n_acc.mean()), "drafts": "sampled from q"}
            if warp[0] > 0:  # draft-token sampling of one step: B rows
                call = lambda: U.check(U.lib().ulb_sample(ctx.h, bq.ptr, B, V, k * V, C.byref(w), 1, 0, 0, 1, st.ptr))
                call()
                ctx.sync()
                g = ctx.capture(lambda: [call() for _ in range(4)])
                ms = ctx.time_graph(g, max(args.steps, 3)) / 4
                U.lib().ulb_graph_free(g)
                results[name.replace("accept", "sample")] = {"us": ms * 1e3, "rows": B,
                                                             "gbs": B * V * 4 / ms / 1e6}
            bd.free()
        for b in (bp, bq, ot, on, st):
            b.free()
    ctx.close()
    print(json.dumps({"mode": "ops", "peak_gbs": peak, "peak_source": peak_src, "results": results}), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--mode", default="spec", choices=["spec", "ops", "trace"],
                    help="spec: the C2 speculative workload (default); ops: the config-3 kernel sweep; "
                         "trace: the CTA timeline of one C2 round (trace build)")
    ap.add_argument("--trace-dump", default="", help="trace mode: also save the raw CTA records (.npz)")
    ap.add_argument("--only", default="", help="ops mode: run one case, e.g. q4_0:11008x4096:m5 or accept")
    ap.add_argument("--workload", default="c2", choices=["c2", "c4", "c5", "pgtest"],
                    help="c2: 7B + TinyLlama, B=1 (default, the headline); c4: Llama-3-8B + 3.2-1B, 64 sequences "
                         "sharded data-parallel over the GPUs; c5: 70B target tensor-parallel over the GPUs + "
                         "replicated 7B draft, batch 8")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--extras", default="auto",
                    help="sharded workloads reported inside the c2 line: auto (c4 at every N, c5 at N >= 2), none, "
                         "or a list such as c4,c5")
    ap.add_argument("--child", action="store_true", help=argparse.SUPPRESS)
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.mode == "ops":
        return run_ops(args)
    if args.mode == "trace":
        return run_trace(args)
    if args.workload == "pgtest":
        return run_pgtest(args)
    if args.workload == "c4":
        return run_c4(args)
    if args.workload == "c5":
        return run_c5(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
