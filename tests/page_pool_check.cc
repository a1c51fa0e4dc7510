// Randomised check of the pooled KV cache's page bookkeeping
// (mojostream_b200/csrc/ms_pages.h), host only: tests/test_page_pool.py
// compiles it with g++ and runs it.  Each operation is followed by the
// invariants: a page's count equals the table entries that hold it, the
// free list holds exactly the pages nobody holds, each once; a call that
// fails leaves table, counts and free list exactly as they were; and the
// device's copy of the table, updated as ms_api.cu updates it (changed rows
// after a call that succeeded, released / shared / reset rows), always
// equals the host's, so no kernel meets an entry the host thinks is there.
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <random>
#include <vector>

#include "ms_pages.h"

using ms::PagePool;

static int g_fail = 0;
#define CHECK(c, ...)                                           \
  do {                                                          \
    if (!(c)) {                                                 \
      std::fprintf(stderr, "line %d: %s: ", __LINE__, #c);      \
      std::fprintf(stderr, __VA_ARGS__);                        \
      std::fprintf(stderr, "\n");                               \
      if (++g_fail > 20) std::exit(1);                          \
    }                                                           \
  } while (0)

struct Snapshot {
  std::vector<int> table, refs;
  int free_count;
};

static Snapshot snap(const PagePool& p) {
  Snapshot s{p.table(), {}, p.free_count()};
  for (int i = 0; i < p.pages(); ++i) s.refs.push_back(p.refs(i));
  return s;
}

static void invariants(const PagePool& p, int step) {
  std::vector<int> held(p.pages(), 0);
  for (int e : p.table())
    if (e >= 0) {
      CHECK(e < p.pages(), "step %d: page %d out of range", step, e);
      ++held[e];
    }
  int unheld = 0;
  for (int i = 0; i < p.pages(); ++i) {
    CHECK(p.refs(i) == held[i], "step %d: page %d refs %d held %d", step, i, p.refs(i), held[i]);
    unheld += held[i] == 0;
  }
  CHECK(p.free_count() == unheld, "step %d: free %d, unheld %d", step, p.free_count(), unheld);
}

static void upload(std::vector<int>& dev, const PagePool& p, int seq) {
  for (int j = 0; j < p.per_seq(); ++j) dev[(size_t)seq * p.per_seq() + j] = p.row(seq)[j];
}

// kv_assign_all's bookkeeping over several sequences: all or nothing.
static bool call(PagePool& p, std::vector<int>& dev, const std::vector<int>& lo,
                 const std::vector<int>& hi, int page, int step) {
  const Snapshot before = snap(p);
  p.begin();
  std::vector<int> dirty_seqs;
  for (size_t q = 0; q < hi.size(); ++q) {
    if (hi[q] < 0) continue;
    bool dirty = false;
    const int short_at = p.assign((int)q, lo[q], hi[q], &dirty);
    if (dirty) dirty_seqs.push_back((int)q);
    if (short_at >= 0) {
      CHECK(short_at <= hi[q], "step %d: short at %d past %d", step, short_at, hi[q]);
      CHECK(p.free_count() == 0, "step %d: short with %d pages free", step, p.free_count());
      p.rollback();
      const Snapshot after = snap(p);
      CHECK(after.table == before.table && after.refs == before.refs &&
                after.free_count == before.free_count,
            "step %d: rollback left changes", step);
      return false;
    }
  }
  for (const PagePool::Copy& c : p.copies()) {
    CHECK(c.from != c.to, "step %d: copy onto itself", step);
    CHECK(p.refs(c.from) >= 1, "step %d: copy from a page nobody holds", step);
    CHECK(p.refs(c.to) == 1, "step %d: copy target shared", step);
  }
  for (int q : dirty_seqs) upload(dev, p, q);
  for (size_t q = 0; q < hi.size(); ++q) {
    if (hi[q] < 0) continue;
    const int* r = p.row((int)q);
    for (int j = 0; j <= hi[q] / page; ++j) CHECK(r[j] >= 0, "step %d: seq %zu entry %d empty", step, q, j);
    for (int j = lo[q] / page; j <= hi[q] / page; ++j)
      CHECK(p.refs(r[j]) == 1, "step %d: seq %zu writes shared page %d", step, q, r[j]);
  }
  p.begin();
  return true;
}

int main() {
  const int n_seq = 5, per_seq = 9, page = 4;
  for (int pages : {6, 12, 40}) {
    for (unsigned seed = 1; seed <= 40; ++seed) {
      std::mt19937 rng(seed * 7919u + pages);
      PagePool p;
      p.init(n_seq, per_seq, pages, page);
      std::vector<int> dev = p.table();
      invariants(p, -1);
      const int max_pos = per_seq * page;
      int fails = 0, shares = 0;
      for (int step = 0; step < 400; ++step) {
        const int op = (int)(rng() % 10);
        if (op < 5) {  // a call writing rows of one to three sequences
          std::vector<int> lo(n_seq, 1 << 30), hi(n_seq, -1);
          const int k = 1 + (int)(rng() % 3);
          for (int i = 0; i < k; ++i) {
            const int q = (int)(rng() % n_seq);
            const int a = (int)(rng() % max_pos), len = 1 + (int)(rng() % 9);
            lo[q] = std::min(lo[q], a);
            hi[q] = std::max(hi[q], std::min(max_pos - 1, a + len - 1));
          }
          if (!call(p, dev, lo, hi, page, step)) ++fails;
        } else if (op < 7) {
          const int q = (int)(rng() % n_seq);
          p.release(q);
          upload(dev, p, q);
          for (int j = 0; j < per_seq; ++j) CHECK(p.row(q)[j] == -1, "step %d: release", step);
        } else if (op < 9) {
          const int src = (int)(rng() % n_seq), dst = (int)(rng() % n_seq);
          if (src == dst) continue;
          if (rng() % 2) {
            p.release(dst);
            upload(dev, p, dst);
          }
          const int n_pos = 1 + (int)(rng() % max_pos);
          const Snapshot before = snap(p);
          PagePool::Copy cp{};
          bool has_copy = false;
          const int rc = p.share_prefix(src, dst, n_pos, &cp, &has_copy);
          if (rc != 0) {
            const Snapshot after = snap(p);
            CHECK(after.table == before.table && after.refs == before.refs,
                  "step %d: refused share changed state (%d)", step, rc);
          } else {
            ++shares;
            upload(dev, p, dst);
            const int full = n_pos / page;
            for (int j = 0; j < full; ++j)
              CHECK(p.row(dst)[j] == p.row(src)[j], "step %d: page %d not shared", step, j);
            CHECK(has_copy == (n_pos % page != 0), "step %d: copy flag", step);
            if (has_copy) {
              CHECK(cp.from == p.row(src)[full] && cp.to == p.row(dst)[full] &&
                        p.refs(cp.to) == 1,
                    "step %d: partial page", step);
            }
          }
        } else {
          p.reset();
          dev = p.table();
          CHECK(p.free_count() == pages, "step %d: reset", step);
        }
        invariants(p, step);
        CHECK(dev == p.table(), "step %d: the device table differs from the host's", step);
      }
      if (seed == 1)
        std::printf("pages %d: %d refused calls, %d shares in 400 steps\n", pages, fails, shares);
    }
  }
  if (g_fail) {
    std::printf("FAILED %d checks\n", g_fail);
    return 1;
  }
  std::printf("ok\n");
  return 0;
}
