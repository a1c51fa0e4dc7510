// The launch plan of one Q4 projection (which kernel, m-group, k-segment,
// k-split) from its shape and the context's limits: host arithmetic only,
// kept apart from ms_api.cu so tests/test_plan.py can check its invariants
// over many shapes without a GPU.
#pragma once
#include <algorithm>
#include <cstddef>

#include "ms_kernels.h"

namespace ms {

// What the plan depends on besides the shape: SMs, the context's split-K
// partial-sum floats and arrival tickets, and the largest batch of the
// decode-batch tensor-core kernel.
struct PlanLimits {
  int sm_count;
  size_t part_floats, n_counters;
  int sk_rows_max;
};

// Launch plan of one projection: decode kernel (M <= 8) or the tiled kernel,
// m-group size, chunks per round, k-segment and the number of k-segments.
struct GemvPlan {
  bool dec, tc, sk;  // sk: the decode-batch tensor-core kernel (tc is set too)
  int mg, ch, kseg, ksplit;
};

// Rows above which projections run on the tensor cores (tcgen05 GEMM).
constexpr int kTcMinRows = 9;

constexpr int kMaxDecodeCluster = 8;  // k-segments that merge inside one cluster

// The streaming decode kernel holds a k-segment's activations in registers:
// at most 2560 / mg values per row, i.e. 40 (mg 1) or 20 (mg 2) chunks
// (launch_gemv_stream refuses longer segments).
constexpr int decode_seg_max(int mg) { return mg == 1 ? 40 : 20; }

inline GemvPlan plan_gemv(const PlanLimits* c, int M, int K, int n_tiles, bool allow_tc = true,
                         bool allow_sk = true) {
  GemvPlan pl{};
  const int chunks = K / kChunkK;
  if (allow_tc && allow_sk && M >= kTcMinRows && M <= c->sk_rows_max) {
    // decode batches: weights on the MMA's 128-row side, about one CTA per SM
    // (tile groups x k-slices), the slices of a group one cluster (<= 8)
    pl.tc = pl.sk = true;
    const int groups = padded_tiles(n_tiles) / kGroupTiles;
    int ks = std::max(1, (c->sm_count + groups / 2) / groups);
    ks = std::min(std::min(ks, 8), chunks);
    const int seg = (chunks + ks - 1) / ks;
    pl.kseg = seg * kChunkK;
    pl.ksplit = (chunks + seg - 1) / seg;
    return pl;
  }
  if (allow_tc && M >= kTcMinRows) {
    // one CTA per (tile group, 128-row tile), all of K -- or k slices when
    // that grid cannot fill the GPU (small batches of narrow projections);
    // the slices' fp32 tiles are summed in k order by the last one
    pl.tc = true;
    const long tiles = (long)(padded_tiles(n_tiles) / kGroupTiles) * ((M + 127) / 128);
    int ks = 1;
    if (tiles < c->sm_count) ks = (int)std::min<long>((c->sm_count + tiles - 1) / tiles, 16);
    ks = std::max(1, std::min(ks, chunks / 4));
    while (ks > 1 && ((size_t)tiles * ks * 128 * 128 > c->part_floats || (size_t)tiles > c->n_counters))
      --ks;
    const int seg = (chunks + ks - 1) / ks;
    pl.kseg = seg * kChunkK;
    pl.ksplit = (chunks + seg - 1) / seg;
    return pl;
  }
  if (M <= 8) {
    // streaming kernel: one CTA per (tile group, k-segment); about one CTA per
    // SM, a k-segment of at most 40 chunks (mg 1) / 20 (mg 2) so stages +
    // fragments stay near 100 KB and the next kernel's CTAs co-reside
    pl.dec = true;
    pl.mg = M <= 4 ? 1 : 2;
    const int mb = 4 * pl.mg;
    const int groups = padded_tiles(n_tiles) / kGroupTiles;
    const int seg_max = decode_seg_max(pl.mg);
    // at least one CTA per SM (rounded up; at most a cluster of 8 k-segments)
    int ksplit = std::max(1, std::min(kMaxDecodeCluster, (c->sm_count + groups - 1) / groups));
    ksplit = std::max(ksplit, (chunks + seg_max - 1) / seg_max);
    ksplit = std::min(ksplit, chunks);
    // a group whose whole K is at most 32 chunks (128 KB of weights, twice
    // what the stage ring holds before the dependency release) runs as one
    // CTA: the cluster merge of a split costs more than the longer stream
    // (measured on the E4B O projection, K 2048: 2.906 -> 2.82 ms per step;
    // the QKV projection, 40 chunks, is faster split)
    if (chunks <= std::min(32, seg_max)) ksplit = 1;
    auto fits = [&](int ks) {
      return ks == 1 || ((size_t)padded_tiles(n_tiles) * ks * kTileN * mb <= c->part_floats &&
                         (size_t)groups <= c->n_counters);
    };
    while (ksplit > 1 && !fits(ksplit)) --ksplit;
    const int seg = (chunks + ksplit - 1) / ksplit;
    pl.kseg = seg * kChunkK;
    pl.ksplit = (chunks + seg - 1) / seg;
    pl.ch = 0;
    return pl;
  }
  int mg = 1;
  while (mg < 16 && 4 * mg < M) mg *= 2;
  pl.mg = mg;
  const int mb = 4 * mg;
  const int mblocks = (M + mb - 1) / mb;
  const int nct = (n_tiles + 3) / 4;
  const long base = (long)mblocks * nct;
  const long target = 3L * c->sm_count;  // CTAs wanted in flight
  pl.ch = mg <= 2 ? 8 : (mg == 4 ? 4 : (mg == 8 ? 4 : 2));
  if (mg <= 2 && base * ((chunks + 7) / 8) < target) pl.ch = 4;  // small matrix: finer split
  const int rounds = (chunks + pl.ch - 1) / pl.ch;  // rounds if one CTA covered all of K
  int ksplit = (int)std::min<long>(rounds, std::max<long>(1, (target + base - 1) / base));
  auto need = [&](int ks) { return ks > 1 ? (size_t)base * ks * 4 * kTileN * mb : (size_t)0; };
  while (ksplit > 1 && (need(ksplit) > c->part_floats || (size_t)base > c->n_counters)) --ksplit;
  const int rounds_per = (rounds + ksplit - 1) / ksplit;
  pl.kseg = rounds_per * pl.ch * kChunkK;
  pl.ksplit = (K + pl.kseg - 1) / pl.kseg;
  return pl;
}

// Partial-sum floats and tickets a projection plan uses (0 without a k-split).
inline void plan_scratch(const GemvPlan& pl, int M, int n_tiles, size_t* floats,
                         size_t* tickets) {
  *floats = 0;
  *tickets = 0;
  if (pl.ksplit <= 1) return;
  const int mb = 4 * pl.mg;
  if (pl.dec) {
    *floats = (size_t)padded_tiles(n_tiles) * pl.ksplit * kTileN * mb;
    *tickets = (size_t)padded_tiles(n_tiles) / kGroupTiles;
  } else {
    const size_t base = (size_t)((M + mb - 1) / mb) * ((n_tiles + 3) / 4);
    *floats = base * pl.ksplit * 4 * kTileN * mb;
    *tickets = base;
  }
}

// Flash-decode attention of one layer: position splits per (row, KV head)
// and whether they merge inside a thread-block cluster.  Limits: SMs, the
// context's partial-sum floats, the kernel's largest split count and
// cluster (0: clusters unavailable), and whether the global-memory merge is
// forced (MS_SPLITK_GLOBAL=1).
struct AttnLimits {
  int sm_count;
  size_t part_floats;
  int max_splits, max_cluster;
  bool global_forced;
};
struct AttnPlan {
  int splits;
  bool cluster;
};
constexpr int kAttnMinPerSplit = 8;  // positions per split at least

// span: the longest run of positions a row of this layer can attend (the
// window, or the cache's max_pos); the kernel sizes each row's ranges itself
// (short rows leave splits idle), so one launch shape -- and one captured
// graph -- serves every position.
inline AttnPlan plan_attention(const AttnLimits* c, int M, int n_kv, int G, int hd, int span) {
  // about one CTA per SM
  const long ctas_per_split = (long)M * n_kv;
  const int min_per = kAttnMinPerSplit;
  int splits = (int)std::max<long>(1, (c->sm_count + ctas_per_split - 1) / ctas_per_split);
  // long spans: at most ~256 positions per split, so a large batch at long
  // context still has enough CTAs to keep every SM streaming
  splits = std::max(splits, (span + 255) / 256);
  splits = std::min(splits, std::max(1, (span + min_per - 1) / min_per));
  splits = std::min(splits, c->max_splits);
  // merge inside a thread-block cluster when the splits fit one (up to 16;
  // a fill-rule count a little above that is trimmed to it), unless the
  // global-memory merge is forced
  const int max_cl = c->max_cluster;
  const bool try_cl = max_cl > 0 && !c->global_forced;
  if (try_cl && splits > max_cl && splits <= max_cl + max_cl / 2 &&
      (span + 255) / 256 <= max_cl)
    splits = max_cl;
  while (splits > 1 && (size_t)M * n_kv * splits * G * (hd + 4) > c->part_floats)
    splits = (splits + 1) / 2;
  return AttnPlan{splits, try_cl && splits > 1 && splits <= max_cl};
}

}  // namespace ms
