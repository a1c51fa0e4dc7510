// Host-only check of the Q4 projection planner (mojostream_b200/csrc/ms_plan.h):
// tests/test_plan.py compiles it with nvcc (the planner's header pulls in the
// kernels' shared definitions) and runs it; nothing here touches a GPU.  For
// every shape of a broad grid, under the library's default context limits
// and a small-scratch variant, each plan must
//   * cover all of K with non-empty k-segments of whole 64-value chunks;
//   * pick the kernel the row count calls for (streaming decode up to 8 rows,
//     the decode-batch tensor-core kernel for 9..64, the tensor-core GEMM
//     above, the tiled CUDA-core kernel when tensor cores are not allowed);
//   * keep its split-K partial sums and tickets inside the context's scratch;
//   * keep a decode k-segment within what the streaming kernel holds in
//     registers, unless even the split that would allow that exceeds the
//     scratch (ms_q4_gemm then refuses the shape with MS_ERR_CAPACITY);
//   * merge decode-batch k-slices inside one cluster (at most 8).
// And every decode attention plan (position splits per row and KV head) must
// stay within the kernel's split count, give no split less than 8
// positions of the span, keep its partial sums inside the scratch, and merge
// inside a cluster only where clusters exist, are not overridden and hold
// all the splits.
#include <cstdio>
#include <cstdlib>

#include "ms_plan.h"

namespace ms {
int sk_rows_max() { return 64; }  // the kernel's constant, for the declaration
}  // namespace ms

using namespace ms;

static long g_fail = 0;
#define CHECK(c, ...)                                          \
  do {                                                         \
    if (!(c)) {                                                \
      std::fprintf(stderr, "%s: ", #c);                        \
      std::fprintf(stderr, __VA_ARGS__);                       \
      std::fprintf(stderr, "\n");                              \
      if (++g_fail > 20) std::exit(1);                         \
    }                                                          \
  } while (0)

static void check(const PlanLimits& L, int M, int K, int nt, bool at, bool as) {
  const GemvPlan p = plan_gemv(&L, M, K, nt, at, as);
  const int chunks = K / kChunkK;
  CHECK(p.kseg > 0 && p.kseg % kChunkK == 0 && p.ksplit >= 1, "M%d K%d nt%d: kseg %d ksplit %d",
        M, K, nt, p.kseg, p.ksplit);
  CHECK((long)(p.ksplit - 1) * p.kseg < K && (long)p.ksplit * p.kseg >= K,
        "M%d K%d nt%d: %d segments of %d do not cover K exactly", M, K, nt, p.ksplit, p.kseg);
  const bool want_sk = at && as && M >= kTcMinRows && M <= L.sk_rows_max;
  const bool want_tc = at && M >= kTcMinRows;
  CHECK(p.sk == want_sk && p.tc == want_tc && p.dec == (!want_tc && M <= 8),
        "M%d K%d nt%d at%d as%d: kernel dec%d tc%d sk%d", M, K, nt, at, as, p.dec, p.tc, p.sk);
  if (p.sk) {
    CHECK(p.ksplit <= 8, "M%d K%d nt%d: %d k-slices in one cluster", M, K, nt, p.ksplit);
    return;
  }
  if (p.tc) {
    const long tiles = (long)(padded_tiles(nt) / kGroupTiles) * ((M + 127) / 128);
    CHECK(p.ksplit == 1 || ((size_t)tiles * p.ksplit * 128 * 128 <= L.part_floats &&
                            (size_t)tiles <= L.n_counters),
          "M%d K%d nt%d: tensor-core split %d over the scratch", M, K, nt, p.ksplit);
    return;
  }
  size_t floats = 0, tickets = 0;
  plan_scratch(p, M, nt, &floats, &tickets);
  CHECK(floats <= L.part_floats && tickets <= L.n_counters,
        "M%d K%d nt%d: split %d needs %zu floats, %zu tickets", M, K, nt, p.ksplit, floats, tickets);
  if (p.dec) {
    CHECK(p.mg == (M <= 4 ? 1 : 2), "M%d: mg %d", M, p.mg);
    const int seg_max = decode_seg_max(p.mg);
    if (p.kseg > seg_max * kChunkK) {  // only when the needed split cannot fit
      GemvPlan q = p;
      q.ksplit = (chunks + seg_max - 1) / seg_max;
      size_t f = 0, t = 0;
      plan_scratch(q, M, nt, &f, &t);
      CHECK(f > L.part_floats || t > L.n_counters,
            "M%d K%d nt%d: segment of %d chunks though a split of %d fits", M, K, nt,
            p.kseg / kChunkK, q.ksplit);
    }
  } else {
    CHECK(p.mg >= 1 && p.mg <= 16 && (p.mg & (p.mg - 1)) == 0 && (4 * p.mg >= M || p.mg == 16),
          "M%d: tiled mg %d", M, p.mg);
    CHECK(p.ch == 2 || p.ch == 4 || p.ch == 8, "M%d: tiled ch %d", M, p.ch);
  }
}

static void check_attn(const AttnLimits& L, int M, int n_kv, int G, int hd, int span) {
  const AttnPlan a = plan_attention(&L, M, n_kv, G, hd, span);
  CHECK(a.splits >= 1 && a.splits <= L.max_splits, "attn M%d span%d: %d splits", M, span, a.splits);
  CHECK(a.splits <= std::max(1, (span + kAttnMinPerSplit - 1) / kAttnMinPerSplit),
        "attn M%d span%d: %d splits of fewer than %d positions", M, span, a.splits,
        kAttnMinPerSplit);
  CHECK(a.splits == 1 || (size_t)M * n_kv * a.splits * G * (hd + 4) <= L.part_floats,
        "attn M%d kv%d G%d hd%d: %d splits over the scratch", M, n_kv, G, hd, a.splits);
  CHECK(!a.cluster || (L.max_cluster > 0 && !L.global_forced && a.splits > 1 &&
                       a.splits <= L.max_cluster),
        "attn M%d span%d: cluster merge of %d splits", M, span, a.splits);
}

int main() {
  // the library's context (ms_init) on a 148-SM B200, and one with 1/128 of
  // its partial-sum scratch so that the fallbacks are reached
  const PlanLimits limits[] = {{148, (size_t)8 << 20, (size_t)1 << 20, 64},
                               {148, (size_t)1 << 16, (size_t)1 << 20, 64}};
  const int tiles[] = {1, 7, 8, 16, 32, 64, 160, 161, 320, 1280, 2048, 16384};
  long n = 0;
  for (const PlanLimits& L : limits)
    for (int M = 1; M <= 2100; M += (M < 80 ? 1 : 37))
      for (int K = 64; K <= 65536; K = K < 1024 ? K + 64 : K + K / 4 - (K / 4) % 64)
        for (int nt : tiles)
          for (int at = 0; at < 2; ++at)
            for (int as = 0; as < 2; ++as, ++n) check(L, M, K, nt, at, as);
  long na = 0;
  for (size_t pf : {(size_t)8 << 20, (size_t)1 << 14})
    for (int mcl : {16, 0})
      for (int forced = 0; forced < 2; ++forced) {
        const AttnLimits L{148, pf, 64, mcl, forced != 0};
        for (int M = 1; M <= 2048; M = M < 16 ? M + 1 : M * 2)
          for (int n_kv : {1, 2, 8})
            for (int G : {1, 4, 8})
              for (int hd : {64, 256, 512})
                for (int span = 1; span <= 131072; span = span < 64 ? span + 1 : span * 2 - 1, ++na)
                  check_attn(L, M, n_kv, G, hd, span);
      }
  if (g_fail) {
    std::printf("FAILED %ld checks of %ld plans\n", g_fail, n);
    return 1;
  }
  std::printf("ok: %ld projection plans, %ld attention plans\n", n, na);
  return 0;
}
