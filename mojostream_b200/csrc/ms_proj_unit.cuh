// ms_proj_unit.cuh -- one unit of the decode Q4 projection (M <= 8 rows): a
// tile group (8 x 16 output columns) over one k-segment, run by the
// one-launch-per-projection kernel of ms_gemv_stream.cu.
//
// Reference: matmul_q4_bpack_raw (src/linalg/kernels.mojo:201-267) with the
// steps fused around its call sites (src/main.mojo:538-613,
// src/inference/gemma4_e4b.mojo:459-540) in the epilogue.
//
// Integer tensor-core math (mma.m16n8k32, u8 x s8 -> s32):
//   * weights: a packed word of the fragment-tile layout masked with
//     0x0F0F0F0F gives the four nibbles u (0..15) of tile row g for k
//     {2t, 2t+8, 2t+1, 2t+9} of a 16-k subtile, as u8 bytes; masked with
//     0xF0F0F0F0 it gives the same k of row g + 8 as 16 u.  Two words (two
//     subtiles) are one k32 A fragment: 2 logic ops per word, no conversion.
//   * activations: the unit reads its k-segment of the fp32 input rows,
//     takes the per-row absolute maximum a, and writes q = rint(x 2^30 / a)
//     as four signed 8-bit limbs (q = d0 + 2^8 d1 + 2^16 d2 + 2^24 d3) into
//     shared memory in the B-fragment layout, with the k order the weight
//     words use.  The 8 MMA columns are 2 rows x 4 limbs.
//   * the s32 sums are exact; per row: sum_k (u - 8) q = sum_k u q - 8 sum_k q
//     (the reference's dequant (nibble - 8) * scale), combined in int64 and
//     scaled by a 2^-30 * weight scale once.  The quantisation error is
//     |x| 2^-31 relative to the row maximum: below fp32 rounding of the sums.
// A producer thread streams the unit's weights with cp.async.bulk (16 KB
// stages = 4 k-chunks x 8 tiles) through an mbarrier ring; 16 consumer warps,
// two per tile, each take two chunks of every stage.  Split-K partials of a
// group are summed in k order, either inside a thread-block cluster of the
// group's k-segments (distributed shared memory, no global round trip) or by
// the last unit through global memory and an arrival ticket (splits above 8):
// results do not depend on timing.  Activations are read through L2
// (ld.global.cg), never through the non-coherent L1 / texture path.
#pragma once

#include "ms_common.cuh"
#include "ms_epilogue.cuh"
#include "ms_kernels.h"

namespace ms {

constexpr int kSHalves = 2;
constexpr int kSWarps = kGroupTiles * kSHalves;       // consumer warps
constexpr int kSConsumers = kSWarps * kWarp;          // 512
constexpr int kSThreads = kSConsumers + kWarp;        // + producer warp
constexpr int kStageChunks = 4;
constexpr int kStageU4 = kStageChunks * kGroupTiles * kWarp;  // 1024 uint4 = 16 KB
constexpr int kStageBytes = kStageU4 * 16;
constexpr float kQuantOne = 1073741824.0f;  // 2^30: |q| <= 2^30 at the row maximum
// Input values a consumer thread holds in the prologue: a k-segment of at
// most 2560 (MG 1) / 1280 (MG 2) per row, 4 values per item.
constexpr int kMaxItems = 5;
constexpr int kConsumerBar = 1;  // named barrier of the 512 consumer threads
// Most k-segments of one tile group that run as a cluster (portable size).
constexpr int kMaxClusterK = 8;

// B fragments of one k-segment: per k32 block, 2*MG MMA column blocks x 32
// lanes x 8 bytes = 512*MG bytes (1 KB per 64-k chunk at MG 1).
__host__ __device__ inline size_t proj_frag_bytes(int mg, int kseg) {
  return (size_t)(kseg / kChunkK) * 2 * (2 * mg) * kWarp * 8;
}
// The same buffer later holds the two-halves merge: 8 tiles x 2*MG column
// blocks x 2 rows x 32 lanes floats.  Size it for the larger of the two.
__host__ __device__ inline size_t proj_scratch_bytes(int mg, int kseg) {
  const size_t merge = (size_t)kGroupTiles * (2 * mg) * 2 * kWarp * sizeof(float);
  const size_t frag = proj_frag_bytes(mg, kseg);
  return frag > merge ? frag : merge;
}

// Weight-stage ring of one CTA.  `seq` counts the stages issued (producer) or
// consumed (consumers) since the ring was set up: slot seq % n, phase
// (seq / n) & 1.  full[] completes on the bytes of a stage, empty[] on the
// arrival of the 16 consumer warps.
struct StageRing {
  uint4* stages;
  uint64_t* full;
  uint64_t* empty;
  int n;
};

struct ProjShared {
  float fin[8], fres[8], deq[8];
  float pmax[kSWarps];
  long long wq[kSWarps];  // sum_k q per warp
  int last, bad;
};

__device__ __forceinline__ int proj_stages(const GemvParams& p, int kidx) {
  const int nchunks = p.K / kChunkK, seg = p.kseg / kChunkK;
  const int c_begin = kidx * seg, c_end = min(nchunks, c_begin + seg);
  return (c_end - c_begin + kStageChunks - 1) / kStageChunks;
}

// An mbarrier wait that also gives up when *abort is set (checked every 64
// tries); both cases return false.
__device__ __forceinline__ bool mbar_wait_abort(uint64_t* bar, uint32_t parity,
                                                const volatile int* abort) {
  for (uint32_t i = 0; i < kWaitTries; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (abort && (i & 63) == 63 && *abort) return false;
  }
  return false;
}

// Producer (one thread): issue the unit's stages into the ring.  False when
// a wait for a free slot gave up (timeout or abort).
__device__ __forceinline__ bool proj_produce(const GemvParams& p, int group, int kidx,
                                             const StageRing& r, uint32_t& seq,
                                             const volatile int* abort) {
  const int nchunks = p.K / kChunkK, seg = p.kseg / kChunkK;
  const int c_begin = kidx * seg, c_end = min(nchunks, c_begin + seg);
  const uint4* wg = p.w + (size_t)group * nchunks * kGroupTiles * kWarp;
  for (int c0 = c_begin; c0 < c_end; c0 += kStageChunks, ++seq) {
    const int slot = (int)(seq % (uint32_t)r.n);
    if (seq >= (uint32_t)r.n &&
        !mbar_wait_abort(&r.empty[slot], ((seq / (uint32_t)r.n) - 1) & 1, abort))
      return false;
    const int nc = min(kStageChunks, c_end - c0);
    const uint32_t bytes = (uint32_t)nc * kGroupTiles * kWarp * 16;
    mbar_expect_tx(&r.full[slot], bytes);
    bulk_g2s(r.stages + (size_t)slot * kStageU4, wg + (size_t)c0 * kGroupTiles * kWarp, bytes,
             &r.full[slot]);
  }
  return true;
}

// Producer, before the CTA exits: wait (bounded) until the last stages it
// issued have landed, so no bulk copy writes shared memory after exit.
__device__ __forceinline__ void ring_drain(const StageRing& r, uint32_t issued) {
  const uint32_t n = (uint32_t)r.n;
  for (uint32_t s = issued > n ? issued - n : 0; s < issued; ++s)
    if (!mbar_wait(&r.full[s % n], (s / n) & 1)) break;
}

__device__ __forceinline__ void imma_u8s8(int (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint2 lds_u2(const uint2* p) {
  uint2 r;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "r"(smem_u32(p)));
  return r;
}

// sum over i = lane, lane + 32, ... < n of a[i * M + m], in that order, with
// the loads of 8 terms in flight at once (one L2 round trip per 256 terms).
__device__ __forceinline__ float strided_sum(const float* a, int n, int M, int m, int lane) {
  float s = 0.f;
  for (int i0 = lane; i0 < n; i0 += 8 * kWarp) {
    float v[8];
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      const int i = i0 + b * kWarp;
      v[b] = i < n ? __ldcg(a + (size_t)i * M + m) : 0.f;
    }
#pragma unroll
    for (int b = 0; b < 8; ++b) s += v[b];
  }
  return s;
}

// Outcome of a consumed unit.
enum ProjResult : int {
  kProjPartial = 0,  // a k-segment whose partial another unit sums
  kProjFinished = 1, // this unit wrote the group's outputs (epilogue done)
  kProjFailed = -1,  // a wait gave up: error word set, outputs skipped
};

// Consumers (the CTA's threads 0..511, warps 0..15): one unit.  The caller
// has made the inputs visible (griddepcontrol.wait / a completed dependency).
// Every consumer thread reaches every barrier; the result is CTA-uniform.
// sB: the B-fragment / merge buffer (proj_scratch_bytes(MG, p.kseg) bytes).
template <int MG>
__device__ int proj_consume(const GemvParams& p, int group, int kidx, const StageRing& r,
                            uint32_t& seq, uint2* sB, ProjShared& sh,
                            const volatile int* abort) {
  constexpr int MB = 4 * MG;  // rows of the m-block
  constexpr int NJ = 2 * MG;  // MMA column blocks: 2 rows x 4 limbs each
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int nchunks = p.K / kChunkK;
  const int seg = p.kseg / kChunkK;
  const int c_begin = kidx * seg;
  const int c_end = min(nchunks, c_begin + seg);
  const int n_cta = c_end - c_begin;
  const int n_st = (n_cta + kStageChunks - 1) / kStageChunks;
  const int tl = warp & (kGroupTiles - 1), half = warp / kGroupTiles;
  const int tile = group * kGroupTiles + tl;
  const int g = lane >> 2, t = lane & 3;
  const int k0 = c_begin * kChunkK, klen = n_cta * kChunkK;

  // the previous unit's readers of sh / sB are done before anything is reused
  bar_sync_n(kConsumerBar, kSConsumers);
  if (tid == 0) sh.bad = 0;

  // ---- B fragments, one pass: thread tid owns row tid / kRowThreads and
  //      items (kb, h, t) = 4 values k {2t, 2t+1, 2t+8, 2t+9} of subtile
  //      2kb + h; all its loads are issued before anything waits on them ----
  constexpr int kRowThreads = kSConsumers / MB;  // 128 (MG 1) / 64 (MG 2): whole warps
  constexpr int kRowWarps = kRowThreads / kWarp;
  const int xr_row = tid / kRowThreads, sub = tid % kRowThreads;
  const int n_items = klen / 4;  // <= kMaxItems * kRowThreads (launcher check)
  float2 va[kMaxItems], vb[kMaxItems];
  {
    const float* xr = p.x + (size_t)xr_row * p.ldx + k0;
#pragma unroll
    for (int jt = 0; jt < kMaxItems; ++jt) {
      const int i = sub + jt * kRowThreads;
      va[jt] = vb[jt] = make_float2(0.f, 0.f);
      if (xr_row < p.M && i < n_items) {
        const int kk = (i >> 3) * 32 + ((i >> 2) & 1) * 16 + 2 * (i & 3);
        va[jt] = __ldcg(reinterpret_cast<const float2*>(xr + kk));
        vb[jt] = __ldcg(reinterpret_cast<const float2*>(xr + kk + 8));
      }
    }
  }
  const bool act = half == 0;      // half 0 finishes the tile
  const bool own = (t & 1) == 0;   // lanes that carry the values on
  // per-row factors of the epilogue (warps < MB), while the loads fly
  if (warp < MB) {
    const int m = warp;
    float fin = p.in_ple, fres = 1.f;
    if (m < p.M) {
      if (p.in_stats) {
        const float s = warp_sum(strided_sum(p.in_stats, p.in_nstat, p.M, m, lane));
        fin = p.in_ple / sqrtf(p.in_ple * p.in_ple * s / (float)p.in_D + 1e-6f);
      }
      if (p.epi == kEpiResid && p.resid_stats) {
        const float s = warp_sum(strided_sum(p.resid_stats, p.resid_nstat, p.M, m, lane));
        fres = 1.0f / sqrtf(p.resid_ple * p.resid_ple * s / (float)p.in_D + 1e-6f);
      }
    }
    if (lane == 0) {
      sh.fin[m] = fin;
      sh.fres[m] = fres;
    }
  }
  {
    float amax = 0.f;
#pragma unroll
    for (int jt = 0; jt < kMaxItems; ++jt)
      amax = fmaxf(amax, fmaxf(fmaxf(fabsf(va[jt].x), fabsf(va[jt].y)),
                               fmaxf(fabsf(vb[jt].x), fabsf(vb[jt].y))));
    amax = warp_max(amax);
    if (lane == 0) sh.pmax[warp] = amax;
  }
  bar_sync_n(kConsumerBar, kSConsumers);
  {
    const int rr = xr_row;
    float a = 0.f;
#pragma unroll
    for (int q = 0; q < kRowWarps; ++q) a = fmaxf(a, sh.pmax[rr * kRowWarps + q]);
    const float inv = a > 0.f ? kQuantOne / a : 0.f;
    if (sub == 0) sh.deq[rr] = a / kQuantOne;
    uint32_t* sB32 = reinterpret_cast<uint32_t*>(sB);
    long long qs = 0;
#pragma unroll
    for (int jt = 0; jt < kMaxItems; ++jt) {
      const int i = sub + jt * kRowThreads;
      if (i < n_items) {
        // byte order of a weight word: k 2t, 2t+8, 2t+1, 2t+9
        const int q[4] = {__float2int_rn(va[jt].x * inv), __float2int_rn(vb[jt].x * inv),
                          __float2int_rn(va[jt].y * inv), __float2int_rn(vb[jt].y * inv)};
        // balanced base-256 limbs q = d0 + 2^8 d1 + 2^16 d2 + 2^24 d3, d0..d2
        // in [-128, 127], |d3| <= 64: adding 128 to each of the low three
        // digits makes them the bytes of u = q + 0x808080 (no carries), so
        // byte l of u ^ 0x808080 is d_l as a signed byte; a byte transpose
        // then gathers limb l of the four values into word l
        uint32_t L[4];
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          qs += q[v];
          L[v] = (uint32_t)(q[v] + 0x808080) ^ 0x808080u;
        }
        const uint32_t t0 = __byte_perm(L[0], L[1], 0x5140), t1 = __byte_perm(L[2], L[3], 0x5140);
        const uint32_t t2 = __byte_perm(L[0], L[1], 0x7362), t3 = __byte_perm(L[2], L[3], 0x7362);
        const uint32_t wl[4] = {__byte_perm(t0, t1, 0x5410), __byte_perm(t0, t1, 0x7632),
                                __byte_perm(t2, t3, 0x5410), __byte_perm(t2, t3, 0x7632)};
        const int kb = i >> 3, h = (i >> 2) & 1, tt = i & 3;
        // lane (g = 4 (r % 2) + l, tt) of column block r / 2, register h
        const int base = ((kb * NJ + (rr >> 1)) * kWarp + 16 * (rr & 1) + tt) * 2 + h;
#pragma unroll
        for (int l = 0; l < 4; ++l) sB32[base + 8 * l] = wl[l];
      }  // rows >= M hold zeros: their fragments come out zero
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) qs += __shfl_xor_sync(0xffffffffu, qs, o);
    if (lane == 0) sh.wq[warp] = qs;
  }
  bar_sync_n(kConsumerBar, kSConsumers);

  // ---- main loop: 2 k32 blocks per chunk, 2 accumulator chains --------------
  int acc[2][NJ][4];
#pragma unroll
  for (int q = 0; q < 2; ++q)
#pragma unroll
    for (int j = 0; j < NJ; ++j)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[q][j][i] = 0;
  bool ok = true;
  int j = 0;
  for (; j < n_st; ++j, ++seq) {
    const int slot = (int)(seq % (uint32_t)r.n);
    if (!mbar_wait_abort(&r.full[slot], (seq / (uint32_t)r.n) & 1, abort)) {
      ok = false;
      break;
    }
    const int nc = min(kStageChunks, n_cta - j * kStageChunks);
    const uint4* st = r.stages + (size_t)slot * kStageU4 + tl * kWarp + lane;
#pragma unroll
    for (int c2 = 0; c2 < kStageChunks / kSHalves; ++c2) {
      const int cc = half * (kStageChunks / kSHalves) + c2;
      if (cc < nc) {
        const uint4 wv = lds_u4(st + cc * kGroupTiles * kWarp);
        const int kb0 = (j * kStageChunks + cc) * 2;
        const uint2* bp = sB + (size_t)kb0 * NJ * kWarp + lane;
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const uint32_t w0 = q ? wv.z : wv.x, w1 = q ? wv.w : wv.y;
          const uint32_t a[4] = {w0 & 0x0F0F0F0Fu, w0 & 0xF0F0F0F0u, w1 & 0x0F0F0F0Fu,
                                 w1 & 0xF0F0F0F0u};
#pragma unroll
          for (int jn = 0; jn < NJ; ++jn) {
            const uint2 b = lds_u2(bp + (q * NJ + jn) * kWarp);
            imma_u8s8(acc[q][jn], a, b.x, b.y);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&r.empty[slot]);
  }
  if (!ok) {
    // a copy never arrived: report it and skip this unit's outputs; the
    // stages not consumed stay issued (the producer drains them at exit)
    if (lane == 0) {
      atomicOr(p.err, kErrWaitTimeout);
      sh.bad = 1;
    }
    seq += (uint32_t)(n_st - j);
  }

  // ---- exact integer combine: lanes t and t^1 hold limbs {0,1} / {2,3} of
  //      row 2jn + t/2; tile rows g (u) and g+8 (16 u) ------------------------
  float rv[NJ][2];  // [column block][tile row g / g+8], valid on even t
#pragma unroll
  for (int jn = 0; jn < NJ; ++jn) {
    const int c0 = acc[0][jn][0] + acc[1][jn][0], c1 = acc[0][jn][1] + acc[1][jn][1];
    const int c2 = acc[0][jn][2] + acc[1][jn][2], c3 = acc[0][jn][3] + acc[1][jn][3];
    const int sh_ = (t & 1) ? 16 : 0;
    long long vg = ((long long)c0 << sh_) + ((long long)c1 << (sh_ + 8));
    long long vh = ((long long)c2 << sh_) + ((long long)c3 << (sh_ + 8));
    vg += __shfl_xor_sync(0xffffffffu, vg, 1);
    vh += __shfl_xor_sync(0xffffffffu, vh, 1);
    vh >>= 4;  // row g + 8 was multiplied by 16 (exact)
    const int m = 2 * jn + (t >> 1);
    // the -8 sum_k q of the whole segment, once per tile (half 0)
    long long qsum = 0;
#pragma unroll
    for (int q = 0; q < kRowWarps; ++q) qsum += sh.wq[m * kRowWarps + q];
    const long long corr = half == 0 ? 8 * qsum : 0;
    const float dq = sh.deq[m];
    rv[jn][0] = (float)(vg - corr) * dq;
    rv[jn][1] = (float)(vh - corr) * dq;
  }

  // ---- merge the two halves of each tile (half 0 + half 1, fixed order) ------
  float* red = reinterpret_cast<float*>(sB);  // the fragments are consumed
  bar_sync_n(kConsumerBar, kSConsumers);      // every warp is past its MMAs
  if (half == 1 && own) {
#pragma unroll
    for (int jn = 0; jn < NJ; ++jn) {
      red[((tl * NJ + jn) * 2 + 0) * kWarp + lane] = rv[jn][0];
      red[((tl * NJ + jn) * 2 + 1) * kWarp + lane] = rv[jn][1];
    }
  }
  bar_sync_n(kConsumerBar, kSConsumers);
  // the k-segments of a group run as one cluster (grid-uniform); such a CTA
  // goes through both cluster barriers below on every path, failed or not
  const bool cl = p.cluster && p.ksplit > 1;
  const bool bad = sh.bad != 0;  // CTA-uniform after the barrier
  if (bad && !cl) return kProjFailed;
  if (act && own) {
#pragma unroll
    for (int jn = 0; jn < NJ; ++jn) {
      rv[jn][0] += red[((tl * NJ + jn) * 2 + 0) * kWarp + lane];
      rv[jn][1] += red[((tl * NJ + jn) * 2 + 1) * kWarp + lane];
    }
  }

  bool finish = true;  // this CTA runs the epilogue of its tiles
  if (cl) {
    // ---- k-segments as one cluster: every CTA leaves its segment's sums in
    //      its own shared memory; CTA r (= k-segment r) finishes the tiles tl
    //      with tl % ksplit == r, summing the ksplit partials in k order (the
    //      order of the global path below, so the same bits) ----------------
    if (act && own) {
#pragma unroll
      for (int jn = 0; jn < NJ; ++jn) {
        red[((tl * NJ + jn) * 2 + 0) * kWarp + lane] = rv[jn][0];
        red[((tl * NJ + jn) * 2 + 1) * kWarp + lane] = rv[jn][1];
      }
    }
    cluster_arrive();
    cluster_wait();  // every CTA's partials and bad flag are in its shared memory
    finish = !bad && (tl % p.ksplit) == kidx;  // warp-uniform
    // a CTA whose weight stream gave up left unfinished partials: no CTA of
    // the cluster writes tiles from them.  The flags are loaded together with
    // the partials below (one distributed-shared-memory round trip) and
    // checked after (every lane reads the same flags: warp-uniform).
    int peer_bad[kMaxClusterK];
#pragma unroll
    for (int r0 = 0; r0 < kMaxClusterK; ++r0) peer_bad[r0] = 0;
    if (finish) {
      const uint32_t bad0 = smem_u32(&sh.bad);
#pragma unroll
      for (int r0 = 0; r0 < kMaxClusterK; ++r0)
        if (r0 < p.ksplit) peer_bad[r0] = ld_dsmem_s32(dsmem_addr(bad0, (uint32_t)r0));
    }
    if (act && own && finish) {
      // the loads of kB CTAs' partials are in flight at once
      constexpr int kB = kMaxClusterK / MG;
      const uint32_t red0 = smem_u32(red);
#pragma unroll
      for (int jn = 0; jn < NJ; ++jn) rv[jn][0] = rv[jn][1] = 0.f;
#pragma unroll
      for (int r0 = 0; r0 < kMaxClusterK; r0 += kB) {
        float v[kB][NJ][2];
#pragma unroll
        for (int b = 0; b < kB; ++b) {
          if (r0 + b < p.ksplit) {
            const uint32_t rb = dsmem_addr(red0, (uint32_t)(r0 + b));
#pragma unroll
            for (int jn = 0; jn < NJ; ++jn) {
              v[b][jn][0] = ld_dsmem(rb + 4u * (((tl * NJ + jn) * 2 + 0) * kWarp + lane));
              v[b][jn][1] = ld_dsmem(rb + 4u * (((tl * NJ + jn) * 2 + 1) * kWarp + lane));
            }
          }
        }
#pragma unroll
        for (int b = 0; b < kB; ++b) {
          if (r0 + b < p.ksplit) {
#pragma unroll
            for (int jn = 0; jn < NJ; ++jn) {
              rv[jn][0] += v[b][jn][0];
              rv[jn][1] += v[b][jn][1];
            }
          }
        }
      }
    }
    int any_bad = 0;
#pragma unroll
    for (int r0 = 0; r0 < kMaxClusterK; ++r0) any_bad |= peer_bad[r0];
    finish = finish && any_bad == 0;
    cluster_arrive();  // done reading the other CTAs' shared memory
  } else if (p.ksplit > 1) {
    // ---- k-segments of the group: the last unit sums the partials in k order
    if (act && own) {
      float* my = p.part + ((size_t)tile * p.ksplit + kidx) * (kTileN * MB);
#pragma unroll
      for (int jn = 0; jn < NJ; ++jn) {
        const int m = 2 * jn + (t >> 1);
        __stcg(my + g * MB + m, rv[jn][0]);
        __stcg(my + (g + 8) * MB + m, rv[jn][1]);
      }
    }
    bar_sync_n(kConsumerBar, kSConsumers);  // partials written
    if (tid == 0) sh.last = (ticket_acq_rel(p.counters + group) == p.ksplit - 1);
    bar_sync_n(kConsumerBar, kSConsumers);
    if (!sh.last) return kProjPartial;  // CTA-uniform
    if (act && own) {
      // sum in k order; the loads of kB segments are in flight at once
      constexpr int kB = 2;
#pragma unroll
      for (int jn = 0; jn < NJ; ++jn) rv[jn][0] = rv[jn][1] = 0.f;
      for (int k0 = 0; k0 < p.ksplit; k0 += kB) {
        float v[kB][NJ][2];
#pragma unroll
        for (int b = 0; b < kB; ++b) {
          const float* pp = p.part + ((size_t)tile * p.ksplit + k0 + b) * (kTileN * MB);
#pragma unroll
          for (int jn = 0; jn < NJ; ++jn) {
            const int m = 2 * jn + (t >> 1);
            const bool in = k0 + b < p.ksplit;
            v[b][jn][0] = in ? __ldcg(pp + g * MB + m) : 0.f;
            v[b][jn][1] = in ? __ldcg(pp + (g + 8) * MB + m) : 0.f;
          }
        }
#pragma unroll
        for (int b = 0; b < kB; ++b)
#pragma unroll
          for (int jn = 0; jn < NJ; ++jn) {
            rv[jn][0] += v[b][jn][0];
            rv[jn][1] += v[b][jn][1];
          }
      }
    }
    if (tid == 0) p.counters[group] = 0;
  }

  // ---- epilogue: half-0 warps finish their tiles ----------------------------
  if (finish && act && tile < p.n_tiles) {
#pragma unroll
    for (int jn = 0; jn < NJ; ++jn) {
      const int m = 2 * jn + (t >> 1);
      float sq = 0.f;
      if (own && m < p.M) {
        const float f = sh.fin[m];
        epilogue_row(p, tile, g, m, rv[jn][0] * f, rv[jn][1] * f, sh.fres[m], sq);
      }
      if (p.epi == kEpiResid && p.out_stats) {
        // sum over the 8 lane groups g (rows g and g+8 of the tile)
        sq += __shfl_xor_sync(0xffffffffu, sq, 4);
        sq += __shfl_xor_sync(0xffffffffu, sq, 8);
        sq += __shfl_xor_sync(0xffffffffu, sq, 16);
        if (g == 0 && own && m < p.M) p.out_stats[(size_t)tile * p.M + m] = sq;
      }
    }
  }
  if (cl) {
    cluster_wait();  // the other CTAs are done reading this CTA's partials
    return bad ? kProjFailed : kProjFinished;
  }
  return kProjFinished;
}

}  // namespace ms
