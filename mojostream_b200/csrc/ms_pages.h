// Host bookkeeping of a pooled KV cache's full-attention pages
// (ms_kv_create_pooled): the block table [n_seq][per_seq] (page id, -1 =
// none), a reference count per page and the free list.  The device holds a
// copy of the table (bt_full); this file only decides which pages change,
// and ms_api.cu moves the data and uploads the rows.
//
// The reference has no page pool: its KVCache (src/main.mojo:257-301) owns
// max_pos rows per sequence, and paged allocation with continuous batching
// is its roadmap item (README.md:487-489).  Page ids index every
// full-attention layer's pool at once, so one table serves all of them.
//
// Every change of one call is journalled, so a call that cannot get all its
// pages (MS_ERR_CAPACITY) is undone as a whole before anything reaches the
// device: the table, the counts and the free list are then exactly as
// before the call, and the device table stays equal to the host one.
// Plain C++ (no CUDA) so the host tests compile it with g++ alone.
#pragma once
#include <vector>

namespace ms {

class PagePool {
 public:
  struct Copy {  // copy-on-write: page `from`'s rows to page `to`
    int from, to;
  };

  // n_seq sequences of per_seq table entries, `pages` pages of `page`
  // positions; every entry unassigned, every page free.
  void init(int n_seq, int per_seq, int pages, int page) {
    n_seq_ = n_seq;
    per_seq_ = per_seq;
    pages_ = pages;
    page_ = page;
    reset();
  }

  // Every entry unassigned, every page free (pages are handed out in
  // ascending id order from a fresh pool).
  void reset() {
    table_.assign((size_t)n_seq_ * per_seq_, -1);
    refs_.assign((size_t)pages_, 0);
    free_.clear();
    for (int p = pages_ - 1; p >= 0; --p) free_.push_back(p);
    journal_.clear();
  }

  int pages() const { return pages_; }
  int per_seq() const { return per_seq_; }
  int free_count() const { return (int)free_.size(); }
  int refs(int p) const { return refs_[p]; }
  const int* row(int seq) const { return table_.data() + (size_t)seq * per_seq_; }
  const std::vector<int>& table() const { return table_; }

  // Start a call: the journal of the previous one is dropped.
  void begin() { journal_.clear(); }

  // Give sequence seq a page for every table entry up to position pos_hi's
  // (entries below it too, so no position a kernel may read maps to no
  // page), and a private page in place of each shared one that positions
  // lo_write .. pos_hi fall in.  Returns -1 on success, else the first
  // position whose page the pool could not supply (the changes made so far
  // stay in the journal: rollback() undoes them).  *dirty: seq's row changed.
  int assign(int seq, int lo_write, int pos_hi, bool* dirty) {
    int* r = table_.data() + (size_t)seq * per_seq_;
    const int j_lo = lo_write / page_;
    for (int j = 0; j <= pos_hi / page_; ++j) {
      const int old = r[j];
      if (old >= 0 && !(j >= j_lo && refs_[old] > 1)) continue;
      if (free_.empty()) return j * page_;
      const int fresh = free_.back();
      free_.pop_back();
      if (old >= 0) --refs_[old];
      refs_[fresh] = 1;
      r[j] = fresh;
      journal_.push_back({seq, j, old, fresh});
      *dirty = true;
    }
    return -1;
  }

  // Undo every change since begin(), newest first; the sequences whose rows
  // it touched (each once) go to *seqs when given.
  void rollback(std::vector<int>* seqs = nullptr) {
    for (size_t i = journal_.size(); i-- > 0;) {
      const Change& ch = journal_[i];
      table_[(size_t)ch.seq * per_seq_ + ch.j] = ch.old;
      if (ch.old >= 0) ++refs_[ch.old];
      refs_[ch.fresh] = 0;
      free_.push_back(ch.fresh);
      if (seqs && (seqs->empty() || !contains(*seqs, ch.seq))) seqs->push_back(ch.seq);
    }
    journal_.clear();
  }

  // The page copies the changes since begin() need: a private page that
  // replaced a shared one starts as a copy of it.
  std::vector<Copy> copies() const {
    std::vector<Copy> out;
    for (const Change& ch : journal_)
      if (ch.old >= 0) out.push_back({ch.old, ch.fresh});
    return out;
  }

  // Sequence seq gives up all its pages (a page returns to the free list
  // when no other sequence refers to it).
  void release(int seq) {
    int* r = table_.data() + (size_t)seq * per_seq_;
    for (int j = 0; j < per_seq_; ++j) {
      if (r[j] < 0) continue;
      if (--refs_[r[j]] == 0) free_.push_back(r[j]);
      r[j] = -1;
    }
  }

  // Sequence dst (holding no pages) starts with src's first n_pos positions:
  // whole pages are shared by reference, the page the prefix ends inside (if
  // any) becomes a private copy in *copy.  Returns 0, or 1 when dst holds
  // pages, 2 when src lacks a page of the prefix, 3 when the pool has no
  // page for the copy; nothing changes unless it returns 0.
  int share_prefix(int src, int dst, int n_pos, Copy* copy, bool* has_copy) {
    int* rs = table_.data() + (size_t)src * per_seq_;
    int* rd = table_.data() + (size_t)dst * per_seq_;
    for (int j = 0; j < per_seq_; ++j)
      if (rd[j] >= 0) return 1;
    const int full = n_pos / page_, part = n_pos % page_;
    for (int j = 0; j < full + (part ? 1 : 0); ++j)
      if (rs[j] < 0) return 2;
    if (part && free_.empty()) return 3;
    for (int j = 0; j < full; ++j) {
      rd[j] = rs[j];
      ++refs_[rs[j]];
    }
    *has_copy = part != 0;
    if (part) {
      const int fresh = free_.back();
      free_.pop_back();
      refs_[fresh] = 1;
      rd[full] = fresh;
      *copy = {rs[full], fresh};
    }
    return 0;
  }

 private:
  struct Change {
    int seq, j, old, fresh;
  };
  static bool contains(const std::vector<int>& v, int x) {
    for (int y : v)
      if (y == x) return true;
    return false;
  }
  int n_seq_ = 0, per_seq_ = 0, pages_ = 0, page_ = 16;
  std::vector<int> table_, refs_, free_;
  std::vector<Change> journal_;
};

}  // namespace ms
