"""Failure detection on the host, without a GPU (nothing here faults or hangs a device).

- watchdog.h's bounded wait (the library's guard around waits for tensor-parallel
  collectives): driven by fakes of the stream query, the communicator's error state and the
  abort, compiled from the product header into a small host program.
- ulb_tp.PeerMonitor on two gloo ranks: a rank that exits between steps, or raises and
  announces that it leaves, is detected by the survivor before its next step, within the
  timeout."""
import json
import os
import socket
import subprocess
import sys
import time

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "universal-loader_b200")

DRIVER = r'''
#include <cstdio>
#include <chrono>
#include "watchdog.h"
using namespace ulb;
int main() {
  using clk = std::chrono::steady_clock;
  int aborts = 0;
  auto none = [] { return false; };
  auto ab = [&] { ++aborts; };
  /* done after a few polls */
  int polls = 0;
  int rc1 = bounded_wait([&] { return ++polls < 5 ? Poll::kPending : Poll::kDone; }, none, ab, 1.0);
  int a1 = aborts;
  /* a peer that never answers: the deadline, one abort */
  auto t0 = clk::now();
  int rc2 = bounded_wait([] { return Poll::kPending; }, none, ab, 0.2);
  double dt2 = std::chrono::duration<double>(clk::now() - t0).count();
  int a2 = aborts;
  /* an asynchronous communicator error: abort at once */
  t0 = clk::now();
  int rc3 = bounded_wait([] { return Poll::kPending; }, [] { return true; }, ab, 5.0);
  double dt3 = std::chrono::duration<double>(clk::now() - t0).count();
  int a3 = aborts;
  /* a stream error: reported, no abort */
  int rc4 = bounded_wait([] { return Poll::kError; }, none, ab, 5.0);
  int a4 = aborts;
  std::printf("{\"rc1\": %d, \"a1\": %d, \"rc2\": %d, \"dt2\": %.4f, \"a2\": %d, \"rc3\": %d, \"dt3\": %.4f, "
              "\"a3\": %d, \"rc4\": %d, \"a4\": %d}\n", rc1, a1, rc2, dt2, a2, rc3, dt3, a3, rc4, a4);
  return 0;
}
'''


def test_bounded_wait_aborts_once_and_reports(tmp_path):
    src = tmp_path / "wd.cpp"
    src.write_text(DRIVER)
    exe = tmp_path / "wd"
    subprocess.run(["g++", "-std=c++17", "-O1", "-I" + os.path.join(PKG, "csrc"), "-o", str(exe), str(src),
                    "-pthread"], check=True)
    r = json.loads(subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout)
    ULB_OK, ULB_ECUDA, ULB_ENCCL, ULB_ETIMEOUT = 0, -3, -4, -5
    assert (r["rc1"], r["a1"]) == (ULB_OK, 0)
    assert (r["rc2"], r["a2"]) == (ULB_ETIMEOUT, 1) and 0.2 <= r["dt2"] < 1.0
    assert (r["rc3"], r["a3"]) == (ULB_ENCCL, 2) and r["dt3"] < 0.5
    assert (r["rc4"], r["a4"]) == (ULB_ECUDA, 2)


CHILD = r'''
import json, os, sys, time
sys.path.insert(0, os.environ["ULB_PKG"])
import datetime
import torch.distributed as dist
from ulb_tp import PeerMonitor, PeerLost
rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
store = dist.TCPStore("127.0.0.1", int(os.environ["MASTER_PORT"]), world, rank == 0,
                      timeout=datetime.timedelta(seconds=60))
mon = PeerMonitor(store, rank, world, timeout_s=float(os.environ["ULB_TIMEOUT"]))
mode = os.environ["ULB_MODE"]
out = {"rank": rank, "steps": []}
try:
    for step in range(4):
        if rank == 1 and step == 2:
            if mode == "exit":      # the process ends between steps, silently
                os._exit(0)
            raise RuntimeError("rank 1 failed")  # an exception: the handler below announces it
        t0 = time.monotonic()
        mon.wait_step(step)
        out["steps"].append(step)
except PeerLost as e:
    out["lost"] = {"ranks": e.ranks, "step": e.step, "after_s": time.monotonic() - t0, "msg": str(e)}
except RuntimeError:
    mon.leave()
    out["raised"] = True
if rank == 0:
    time.sleep(0.5)   # the store lives in rank 0's process: keep it up until the others are done
print("RESULT " + json.dumps(out), flush=True)
'''


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("mode,timeout", [("exit", 2.0), ("raise", 30.0)])
def test_peer_lost_between_steps_is_detected(mode, timeout):
    port = _free_port()
    procs = []
    for r in range(2):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE="2", MASTER_PORT=str(port), ULB_PKG=PKG,
                   ULB_TIMEOUT=str(timeout), ULB_MODE=mode)
        procs.append(subprocess.Popen([sys.executable, "-c", CHILD], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.PIPE, text=True))
        if r == 0:
            time.sleep(0.5)  # rank 0 hosts the store
    outs = {}
    for p in procs:
        o, e = p.communicate(timeout=120)
        lines = [ln for ln in o.splitlines() if ln.startswith("RESULT ")]
        if lines:
            d = json.loads(lines[-1][7:])
            outs[d["rank"]] = d
        else:
            assert mode == "exit", e[-2000:]  # the rank that exited silently prints nothing
    r0 = outs[0]
    assert r0["steps"] == [0, 1]
    assert r0["lost"]["ranks"] == [1] and r0["lost"]["step"] == 2
    if mode == "exit":
        # a silent exit is noticed when the timeout runs out, and not much later
        assert timeout <= r0["lost"]["after_s"] < timeout + 2.0
    else:
        # an announced departure is noticed at once, long before the timeout
        assert r0["lost"]["after_s"] < 5.0 and "left" in r0["lost"]["msg"]
        assert outs[1]["raised"]
