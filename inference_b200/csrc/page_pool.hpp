// page_pool.hpp -- the KV page pool of batched decode (batch.cu), host only.
//
// Pages are the 64-position units of the per-layer K/V pools; the same page
// index is used in every layer.  A sequence owns a page table of physical page
// indices.  Pages carry reference counts: q3_batch_fork gives a new sequence
// the full pages of its source by reference (neither writes them again: a
// sequence writes only at its own position, which is past them) and fresh
// pages for the rest, the partial page's contents copied.  A page returns to
// the free list when its last reference is dropped.
#pragma once

#include <cstdint>
#include <vector>

namespace q3 {

class PagePool {
  public:
    explicit PagePool(int pages) : refs_(pages, 0) {
        for (int p = pages - 1; p >= 0; --p) free_.push_back(p);
    }
    int size() const { return static_cast<int>(refs_.size()); }
    int free_count() const { return static_cast<int>(free_.size()); }
    int refs(int32_t p) const { return refs_[p]; }

    // A free page with one reference; false if none is left.
    bool take(int32_t* out) {
        if (free_.empty()) return false;
        *out = free_.back();
        free_.pop_back();
        refs_[*out] = 1;
        return true;
    }
    void ref(int32_t p) { ++refs_[p]; }
    void drop(int32_t p) {
        if (refs_[p] > 0 && --refs_[p] == 0) free_.push_back(p);
    }
    void drop_all(const std::vector<int32_t>& pages) {
        for (int32_t p : pages) drop(p);
    }

    // `n` fresh pages, or none (and false) if the pool cannot give them all.
    bool take_n(int n, std::vector<int32_t>& out) {
        std::vector<int32_t> got;
        for (int i = 0; i < n; ++i) {
            int32_t p = 0;
            if (!take(&p)) {
                drop_all(got);
                return false;
            }
            got.push_back(p);
        }
        out.insert(out.end(), got.begin(), got.end());
        return true;
    }

    // The page table of a fork of a sequence with page table `src` whose next
    // position is kv_len: its pages before the position are shared, the rest
    // fresh.  *copy_index = the logical page whose written part (positions
    // up to kv_len) must be copied into the fork's own page, or -1 when kv_len
    // is on a page boundary.  False (nothing taken) if the pool runs out.
    bool fork(const std::vector<int32_t>& src, int kv_len, int page_size, std::vector<int32_t>& out,
              int* copy_index) {
        const int full = kv_len / page_size;
        std::vector<int32_t> fresh;
        if (!take_n(static_cast<int>(src.size()) - full, fresh)) return false;
        out.clear();
        for (int i = 0; i < full; ++i) {
            ref(src[i]);
            out.push_back(src[i]);
        }
        out.insert(out.end(), fresh.begin(), fresh.end());
        *copy_index = (kv_len % page_size) ? full : -1;
        return true;
    }

  private:
    std::vector<int> refs_;
    std::vector<int32_t> free_;
};

}  // namespace q3
