// CPU check of the batched-decode KV page pool (inference_b200/csrc/page_pool.hpp):
// reference counts, all-or-nothing allocation, fork sharing, release, and a
// seeded random sequence of adds / forks / releases against the invariants.
// Built and run by tests/test_page_pool.py; prints FAIL lines, exits non-zero on any.
#include <cstdio>
#include <map>
#include <random>
#include <vector>

#include "page_pool.hpp"

static int failures = 0;
#define CHECK(c)                                                    \
    do {                                                            \
        if (!(c)) {                                                 \
            std::printf("FAIL line %d: %s\n", __LINE__, #c);        \
            ++failures;                                             \
        }                                                           \
    } while (0)

using q3::PagePool;

// Every page's count equals its uses by the live tables; free pages are unused.
static void check_invariants(const PagePool& pool, const std::map<int, std::vector<int32_t>>& seqs) {
    std::vector<int> uses(pool.size(), 0);
    for (const auto& s : seqs)
        for (int32_t p : s.second) ++uses[p];
    int used = 0;
    for (int p = 0; p < pool.size(); ++p) {
        CHECK(pool.refs(p) == uses[p]);
        used += uses[p] > 0;
    }
    CHECK(pool.free_count() + used == pool.size());
}

int main() {
    {  // all-or-nothing allocation
        PagePool pool(10);
        std::vector<int32_t> a, b;
        CHECK(pool.take_n(4, a) && a.size() == 4 && pool.free_count() == 6);
        CHECK(!pool.take_n(7, b) && b.empty() && pool.free_count() == 6);
        pool.drop_all(a);
        CHECK(pool.free_count() == 10);
        pool.drop(a[0]);  // a second drop of a free page changes nothing
        CHECK(pool.free_count() == 10 && pool.refs(a[0]) == 0);
    }
    {  // fork in the middle of a page: two pages shared, the partial one copied
        PagePool pool(10);
        std::vector<int32_t> src, f;
        CHECK(pool.take_n(4, src));
        int copy = -2;
        CHECK(pool.fork(src, 129, 64, f, &copy));
        CHECK(f.size() == 4 && f[0] == src[0] && f[1] == src[1] && f[2] != src[2] && f[3] != src[3]);
        CHECK(copy == 2 && pool.refs(src[0]) == 2 && pool.refs(src[2]) == 1 && pool.free_count() == 4);
        pool.drop_all(src);  // the source goes: its shared pages stay with the fork
        CHECK(pool.refs(f[0]) == 1 && pool.free_count() == 6);
        pool.drop_all(f);
        CHECK(pool.free_count() == 10);
    }
    {  // fork on a page boundary and at position 0: nothing to copy
        PagePool pool(8);
        std::vector<int32_t> src, f, g;
        CHECK(pool.take_n(3, src));
        int copy = 0;
        CHECK(pool.fork(src, 128, 64, f, &copy) && copy == -1 && f[1] == src[1] && f[2] != src[2]);
        CHECK(pool.fork(src, 0, 64, g, &copy) && copy == -1 && g[0] != src[0]);
        CHECK(pool.free_count() == 8 - 3 - 1 - 3);
    }
    {  // a fork the pool cannot serve takes nothing
        PagePool pool(5);
        std::vector<int32_t> src, f;
        CHECK(pool.take_n(4, src));
        int copy = 0;
        CHECK(!pool.fork(src, 10, 64, f, &copy));  // needs 4 fresh pages, 1 is left
        CHECK(pool.free_count() == 1 && pool.refs(src[0]) == 1);
    }
    {  // seeded random adds, forks (of forks) and releases
        PagePool pool(64);
        std::map<int, std::vector<int32_t>> seqs;
        std::map<int, int> pos;
        std::mt19937 rng(7);
        int next_id = 0;
        for (int step = 0; step < 5000; ++step) {
            const int op = static_cast<int>(rng() % 3);
            if (op == 0 || seqs.empty()) {
                std::vector<int32_t> t;
                const int n = 1 + static_cast<int>(rng() % 6);
                if (pool.take_n(n, t)) {
                    seqs[next_id] = t;
                    pos[next_id] = static_cast<int>(rng() % (n * 64));
                    ++next_id;
                }
            } else {
                auto it = seqs.begin();
                std::advance(it, rng() % seqs.size());
                if (op == 1) {
                    std::vector<int32_t> f;
                    int copy = 0;
                    const int kv = pos[it->first];
                    if (pool.fork(it->second, kv, 64, f, &copy)) {
                        CHECK(copy == ((kv % 64) ? kv / 64 : -1));
                        for (int i = 0; i < kv / 64; ++i) CHECK(f[i] == it->second[i]);
                        seqs[next_id] = f;
                        pos[next_id] = kv + static_cast<int>(rng() % 2);  // it may have stepped since
                        ++next_id;
                    }
                } else {
                    pool.drop_all(it->second);
                    pos.erase(it->first);
                    seqs.erase(it);
                }
            }
            check_invariants(pool, seqs);
        }
        for (auto& s : seqs) pool.drop_all(s.second);
        CHECK(pool.free_count() == 64);
    }
    std::printf("%s (%d failures)\n", failures ? "FAILED" : "ok", failures);
    return failures ? 1 : 0;
}
