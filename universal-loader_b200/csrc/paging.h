/*
 * paging.h — host allocator of KV cache pages for the speculative loop's sequence slots.
 *
 * The loop's caches (target and draft) are page pools with one block table row per slot
 * (ulb_kv_alloc_paged); both use the same page ids, so one allocator serves both.  A slot
 * holds pages for positions [0, mapped * kPage); ensure() extends that ahead of the positions
 * the next rounds will write, release() returns every page of a finished slot to the pool,
 * so memory follows the live sequences' lengths instead of n_slots * capacity.  Pages are
 * handed out lowest id first (a sorted free set), so a run's mapping is deterministic.
 * Replaces the reference's stub batcher, which pads requests into fixed batches and never
 * touches a cache (src/inference/continuous_batcher.cpp:20-122, model.h:49-77).
 *
 * Host-only (no CUDA types): unit tested on the CPU (tests/test_paging_cpu.py).
 */
#pragma once

#include <set>
#include <vector>

namespace ulb {

class PagePool {
 public:
  PagePool(int n_pages, int n_slots, int max_pages_per_slot, int page_positions)
      : max_pages_(max_pages_per_slot), page_(page_positions), slots_(n_slots) {
    for (int p = 0; p < n_pages; ++p) free_.insert(p);
  }

  /* map pages so slot s covers positions [0, positions) (capped at max_pages); on success the
     new pages are appended to *added (in table order, starting at table index *first) */
  bool ensure(int s, int positions, int* first, std::vector<int>* added) {
    std::vector<int>& have = slots_[s];
    int want = (positions + page_ - 1) / page_;
    if (want > max_pages_) want = max_pages_;
    *first = (int)have.size();
    added->clear();
    if (want <= (int)have.size()) return true;
    if ((int)free_.size() < want - (int)have.size()) return false;
    while ((int)have.size() < want) {
      const int p = *free_.begin();
      free_.erase(free_.begin());
      have.push_back(p);
      added->push_back(p);
    }
    return true;
  }

  /* return every page of slot s; the number of table entries to unmap */
  int release(int s) {
    const int n = (int)slots_[s].size();
    for (int p : slots_[s]) free_.insert(p);
    slots_[s].clear();
    return n;
  }

  int free_pages() const { return (int)free_.size(); }
  int mapped(int s) const { return (int)slots_[s].size(); }
  const std::vector<int>& pages(int s) const { return slots_[s]; }

 private:
  int max_pages_, page_;
  std::vector<std::vector<int>> slots_;
  std::set<int> free_;
};

}  // namespace ulb
