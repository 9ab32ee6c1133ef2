"""KV cache page allocator of the speculative loop (paging.h), on the CPU: slots grow page by
page as their sequences do, a finished slot's pages return to the pool and serve the next
sequence, the pool never hands out a page twice, capacity and exhaustion are respected, and
the mapping is deterministic (lowest free page first)."""
import json
import os
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

DRIVER = r'''
#include <cstdio>
#include <set>
#include "paging.h"
using namespace ulb;
int main() {
  PagePool pool(10, 3, 4, 256);   /* 10 pages, 3 slots of at most 4 pages of 256 positions */
  int first; std::vector<int> added;
  bool ok1 = pool.ensure(0, 300, &first, &added);              /* 2 pages */
  int f1 = first; std::vector<int> a1 = added;
  bool ok2 = pool.ensure(0, 512, &first, &added);              /* still 2 */
  int n2 = (int)added.size();
  bool ok3 = pool.ensure(1, 1000, &first, &added);             /* 4 pages */
  std::vector<int> a3 = added;
  bool ok4 = pool.ensure(0, 5000, &first, &added);             /* capped at 4: 2 more */
  int f4 = first; int n4 = (int)added.size();
  bool ok5 = pool.ensure(2, 1024, &first, &added);             /* 4 wanted, 2 free: refused, nothing taken */
  int free5 = pool.free_pages(); int m5 = pool.mapped(2);
  int rel = pool.release(1);                                   /* 4 back */
  bool ok6 = pool.ensure(2, 1024, &first, &added);             /* now fits: lowest ids first */
  std::vector<int> a6 = added;
  std::set<int> all;
  int total = 0;
  for (int s = 0; s < 3; ++s) for (int p : pool.pages(s)) { all.insert(p); ++total; }
  std::printf("{\"ok\": [%d,%d,%d,%d,%d,%d], \"f1\": %d, \"a1\": [%d,%d], \"n2\": %d, \"a3\": [%d,%d,%d,%d], "
              "\"f4\": %d, \"n4\": %d, \"free5\": %d, \"m5\": %d, \"rel\": %d, \"a6\": [%d,%d,%d,%d], "
              "\"unique\": %d, \"total\": %d, \"free\": %d}\n",
              ok1, ok2, ok3, ok4, ok5, ok6, f1, a1[0], a1[1], n2, a3[0], a3[1], a3[2], a3[3], f4, n4, free5, m5, rel,
              a6[0], a6[1], a6[2], a6[3], (int)all.size(), total, pool.free_pages());
  return 0;
}
'''


def test_page_pool(tmp_path):
    src = tmp_path / "pp.cpp"
    src.write_text(DRIVER)
    exe = tmp_path / "pp"
    subprocess.run(["g++", "-std=c++17", "-O1", "-I" + os.path.join(ROOT, "universal-loader_b200", "csrc"),
                    "-o", str(exe), str(src)], check=True)
    r = json.loads(subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout)
    assert r["ok"] == [1, 1, 1, 1, 0, 1]
    assert r["f1"] == 0 and r["a1"] == [0, 1] and r["n2"] == 0
    assert r["a3"] == [2, 3, 4, 5]
    assert r["f4"] == 2 and r["n4"] == 2            # slot 0 grows to its cap of 4 pages (6, 7)
    assert r["free5"] == 2 and r["m5"] == 0         # a refused request takes nothing
    assert r["rel"] == 4
    assert r["a6"] == [2, 3, 4, 5]                  # slot 1's pages serve slot 2, lowest first
    assert r["unique"] == r["total"] == 8 and r["free"] == 2
