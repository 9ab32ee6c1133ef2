"""Data-parallel host logic of bench.py on CPU: two gloo ranks on 127.0.0.1.

Config 4 shards 64 independent sequences round-robin over the ranks and reduces only counts
and times on the host (no collective on the data path).  This checks, with real
torch.distributed ranks, that the shards partition the sequences exactly, that every rank
sees the same prompts for its indices, and that the sum / max reductions bench.py uses
combine the ranks' numbers."""
import json
import os
import socket
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r'''
import json, os, sys
sys.path.insert(0, os.environ["ULB_ROOT"])
import bench
world, rank, local, barrier, allmax, allsum, done = bench.dist_setup()
prompts = bench.c4_prompts()
mine = bench.shard(list(range(len(prompts))), rank, world)
toks = sum(len(prompts[i]) for i in mine)
out = {"rank": rank, "world": world, "idx": mine, "first": [prompts[i][:4] for i in mine[:2]],
       "sum_tokens": allsum(toks), "max_rank": allmax(rank), "n_seq": allsum(len(mine))}
barrier()
done()
print("RESULT " + json.dumps(out), flush=True)
'''


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_c4_sequences_shard_over_two_gloo_ranks():
    port = _free_port()
    procs = []
    for r in range(2):
        env = dict(os.environ, RANK=str(r), LOCAL_RANK=str(r), WORLD_SIZE="2", MASTER_ADDR="127.0.0.1",
                   MASTER_PORT=str(port), ULB_ROOT=ROOT)
        procs.append(subprocess.Popen([sys.executable, "-c", CHILD], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.PIPE, text=True))
    outs = []
    for p in procs:
        o, e = p.communicate(timeout=240)
        assert p.returncode == 0, e[-2000:]
        outs.append(json.loads([ln for ln in o.splitlines() if ln.startswith("RESULT ")][-1][7:]))
    outs.sort(key=lambda d: d["rank"])
    sys.path.insert(0, ROOT)
    import bench
    prompts = bench.c4_prompts()
    assert len(prompts) == 64 and all(256 <= len(p) <= 4096 for p in prompts)
    idx = outs[0]["idx"] + outs[1]["idx"]
    assert sorted(idx) == list(range(64)) and len(set(idx)) == 64      # an exact partition
    assert outs[0]["idx"] == list(range(0, 64, 2)) and outs[1]["idx"] == list(range(1, 64, 2))
    for o in outs:
        assert o["first"] == [prompts[i][:4] for i in o["idx"][:2]]     # same prompts on every rank
        assert o["sum_tokens"] == sum(len(p) for p in prompts)           # host sum over ranks
        assert o["max_rank"] == 1 and o["n_seq"] == 64                   # host max / sum


def test_child_workload_groups_under_torchrun():
    """bench.py runs the sharded workloads (c4, c5) as child process groups of its own ranks.
    Under torchrun the children must form their own gloo group (not torchrun's agent store) on
    a port of their own, and rank 0's child line must come back to the parent: checked with the
    GPU-free pgtest workload on two ranks."""
    port = _free_port()
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                        "--master-addr", "127.0.0.1", "--master-port", str(port), os.path.join(ROOT, "bench.py"),
                        "--workload", "pgtest", "--gpus", "2"], capture_output=True, text=True, timeout=240)
    assert r.returncode == 0, r.stderr[-3000:]
    line = json.loads([ln for ln in r.stdout.splitlines() if ln.startswith("{")][-1])
    assert line["pgtest"]["world"] == 2 and line["pgtest"]["rank_sum"] == 1.0
