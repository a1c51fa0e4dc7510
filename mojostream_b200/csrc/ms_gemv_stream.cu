// ms_gemv_stream.cu -- Q4 projection for decode batches (M <= 8 rows), the
// hot op of the token loop at batch 4 (reference: matmul_q4_bpack_raw,
// src/linalg/kernels.mojo:201-267, with the steps fused around its call
// sites in src/main.mojo:538-613 and src/inference/gemma4_e4b.mojo:459-540).
//
// A decode step reads every weight once with only a few activation rows, so
// the kernel is a weight stream; its inner product must cost few
// instructions per weight byte or the SMs, not HBM, set the pace.  Hence
// integer tensor-core math (mma.m16n8k32, u8 x s8 -> s32):
//   * weights: a packed word of the fragment-tile layout masked with
//     0x0F0F0F0F gives the four nibbles u (0..15) of tile row g for k
//     {2t, 2t+8, 2t+1, 2t+9} of a 16-k subtile, as u8 bytes; masked with
//     0xF0F0F0F0 it gives the same k of row g + 8 as 16 u.  Two words (two
//     subtiles) are one k32 A fragment: 2 logic ops per word, no conversion.
//   * activations: each CTA reads its k-segment of the fp32 input rows,
//     takes the per-row absolute maximum a, and writes q = rint(x 2^30 / a)
//     as four signed 8-bit limbs (q = d0 + 2^8 d1 + 2^16 d2 + 2^24 d3) into
//     shared memory in the B-fragment layout, with the k order the weight
//     words use.  The 8 MMA columns are 2 rows x 4 limbs.
//   * the s32 sums are exact; per row: sum_k (u - 8) q = sum_k u q - 8 sum_k q
//     (the reference's dequant (nibble - 8) * scale), combined in int64 and
//     scaled by a 2^-30 * weight scale once.  The quantisation error is
//     |x| 2^-31 relative to the row maximum: below fp32 rounding of the sums.
// Per CTA: one producer thread streams the tile group's k-segment with
// cp.async.bulk (16 KB stages = 4 k-chunks x 8 tiles) through a 4-stage
// mbarrier ring, issuing the first stages before griddepcontrol.wait (weights
// do not depend on the previous kernel); 16 consumer warps, two per tile,
// each take two chunks of every stage.  Split-K partials of a group are
// summed by the last CTA in k order: results do not depend on timing.
#include "ms_common.cuh"
#include "ms_epilogue.cuh"
#include "ms_kernels.h"

namespace ms {

constexpr int kSHalves = 2;
constexpr int kSWarps = kGroupTiles * kSHalves;       // consumer warps
constexpr int kSConsumers = kSWarps * kWarp;          // 512
constexpr int kSThreads = kSConsumers + kWarp;        // + producer warp
constexpr int kSTileThreads = kGroupTiles * kWarp;    // one warp per tile (after the halves merge)
constexpr int kStageChunks = 4;
constexpr int kStages = 4;
constexpr int kStageU4 = kStageChunks * kGroupTiles * kWarp;  // 1024 uint4 = 16 KB
constexpr int kStageBytes = kStageU4 * 16;
constexpr float kQuantOne = 1073741824.0f;  // 2^30: |q| <= 2^30 at the row maximum
// Input values a consumer thread holds in the prologue: a k-segment of at
// most 2560 (MG 1) / 1280 (MG 2) per row, 4 values per item.
constexpr int kMaxItems = 5;

// B fragments of one k-segment: per k32 block, 2*MG MMA column blocks x 32
// lanes x 8 bytes = 512*MG bytes (1 KB per 64-k chunk at MG 1).
size_t gemv_stream_smem(int mg, int kseg) {
  const int chunks = kseg / kChunkK;
  return (size_t)kStages * kStageBytes + (size_t)chunks * 2 * (2 * mg) * kWarp * sizeof(uint2);
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
template <int MG>
__global__ void __launch_bounds__(kSThreads, 2) gemv_stream_kernel(const GemvParams p) {
  constexpr int MB = 4 * MG;  // rows of the m-block
  constexpr int NJ = 2 * MG;  // MMA column blocks: 2 rows x 4 limbs each
  extern __shared__ __align__(128) uint8_t dsm[];
  uint4* stages = reinterpret_cast<uint4*>(dsm);
  uint2* sB = reinterpret_cast<uint2*>(dsm + kStages * kStageBytes);  // [kb][NJ][32]
  __shared__ __align__(8) uint64_t full[kStages], empty[kStages];
  __shared__ float s_fin[MB], s_fres[MB], s_deq[MB];
  __shared__ float s_pmax[kSWarps];
  __shared__ long long s_wq[kSWarps];  // sum_k q per warp (kRowWarps warps per row)
  __shared__ int s_last, s_bad;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int group = blockIdx.x, kidx = blockIdx.y;
  const int nchunks = p.K / kChunkK;
  const int seg = p.kseg / kChunkK;
  const int c_begin = kidx * seg;
  const int c_end = min(nchunks, c_begin + seg);
  const int n_cta = c_end - c_begin;
  const int n_st = (n_cta + kStageChunks - 1) / kStageChunks;
  const uint4* wg = p.w + (size_t)group * nchunks * kGroupTiles * kWarp;

  if (threadIdx.x == 0) {
    s_bad = 0;
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kSWarps);
    }
    mbar_fence_init();
  }
  __syncthreads();
  pdl_trigger();

  // ------------------------------------------------------------ producer --
  // Reads weights only, which no earlier kernel writes: no griddepcontrol.wait.
  if (warp == kSWarps) {
    if (lane == 0) {
      auto issue = [&](int j) {
        const int slot = j % kStages;
        const int c0 = c_begin + j * kStageChunks;
        const int nc = min(kStageChunks, c_end - c0);
        const uint32_t bytes = (uint32_t)nc * kGroupTiles * kWarp * 16;
        mbar_expect_tx(&full[slot], bytes);
        bulk_g2s(stages + (size_t)slot * kStageU4, wg + (size_t)c0 * kGroupTiles * kWarp, bytes,
                 &full[slot]);
      };
      const int first = min(n_st, kStages);
      for (int j = 0; j < first; ++j) issue(j);
      for (int j = first; j < n_st; ++j) {
        if (!mbar_wait(&empty[j % kStages], ((j / kStages) - 1) & 1)) {
          atomicOr(p.err, kErrWaitTimeout);
          break;  // consumers time out on the stages never issued
        }
        issue(j);
      }
    }
    return;
  }

  // ----------------------------------------------------------- consumers --
  pdl_wait();
  const int tl = warp & (kGroupTiles - 1), half = warp / kGroupTiles;
  const int tile = group * kGroupTiles + tl;
  const int g = lane >> 2, t = lane & 3;
  const int k0 = c_begin * kChunkK, klen = n_cta * kChunkK;

  // ---- B fragments, one pass: thread tid owns row tid / kRowThreads and
  //      items (kb, h, t) = 4 values k {2t, 2t+1, 2t+8, 2t+9} of subtile
  //      2kb + h; all its loads are issued before anything waits on them ----
  constexpr int kRowThreads = kSConsumers / MB;  // 128 (MG 1) / 64 (MG 2): whole warps
  constexpr int kRowWarps = kRowThreads / kWarp;
  const int xr_row = threadIdx.x / kRowThreads, sub = threadIdx.x % kRowThreads;
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
        va[jt] = __ldg(reinterpret_cast<const float2*>(xr + kk));
        vb[jt] = __ldg(reinterpret_cast<const float2*>(xr + kk + 8));
      }
    }
  }
  // per-row factors of the epilogue (warps < MB), while the loads fly
  if (warp < MB) {
    const int m = warp;
    float fin = p.in_ple, fres = 1.f;
    if (m < p.M) {
      if (p.in_stats) {
        float s = 0.f;
#pragma unroll 4
        for (int i = lane; i < p.in_nstat; i += kWarp) s += p.in_stats[(size_t)i * p.M + m];
        s = warp_sum(s);
        fin = p.in_ple / sqrtf(p.in_ple * p.in_ple * s / (float)p.in_D + 1e-6f);
      }
      if (p.epi == kEpiResid && p.resid_stats) {
        float s = 0.f;
#pragma unroll 4
        for (int i = lane; i < p.resid_nstat; i += kWarp) s += p.resid_stats[(size_t)i * p.M + m];
        s = warp_sum(s);
        fres = 1.0f / sqrtf(p.resid_ple * p.resid_ple * s / (float)p.in_D + 1e-6f);
      }
    }
    if (lane == 0) {
      s_fin[m] = fin;
      s_fres[m] = fres;
    }
  }
  {
    float amax = 0.f;
#pragma unroll
    for (int jt = 0; jt < kMaxItems; ++jt)
      amax = fmaxf(amax, fmaxf(fmaxf(fabsf(va[jt].x), fabsf(va[jt].y)),
                               fmaxf(fabsf(vb[jt].x), fabsf(vb[jt].y))));
    amax = warp_max(amax);
    if (lane == 0) s_pmax[warp] = amax;
  }
  bar_sync_n(1, kSConsumers);
  {
    const int r = xr_row;
    float a = 0.f;
#pragma unroll
    for (int q = 0; q < kRowWarps; ++q) a = fmaxf(a, s_pmax[r * kRowWarps + q]);
    const float inv = a > 0.f ? kQuantOne / a : 0.f;
    if (sub == 0) s_deq[r] = a / kQuantOne;
    uint32_t* sB32 = reinterpret_cast<uint32_t*>(sB);
    long long qs = 0;
#pragma unroll
    for (int jt = 0; jt < kMaxItems; ++jt) {
      const int i = sub + jt * kRowThreads;
      if (i < n_items) {
        // byte order of a weight word: k 2t, 2t+8, 2t+1, 2t+9
        const int q[4] = {__float2int_rn(va[jt].x * inv), __float2int_rn(vb[jt].x * inv),
                          __float2int_rn(va[jt].y * inv), __float2int_rn(vb[jt].y * inv)};
        uint32_t wl[4] = {0u, 0u, 0u, 0u};
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          qs += q[v];
          int rest = q[v];
#pragma unroll
          for (int l = 0; l < 3; ++l) {  // balanced base-256 limbs
            const int d = (int)(int8_t)(rest & 0xFF);
            wl[l] |= ((uint32_t)d & 0xFFu) << (8 * v);
            rest = (rest - d) >> 8;  // exact: rest - d is a multiple of 256
          }
          wl[3] |= ((uint32_t)rest & 0xFFu) << (8 * v);  // |rest| <= 64
        }
        const int kb = i >> 3, h = (i >> 2) & 1, tt = i & 3;
        // lane (g = 4 (r % 2) + l, tt) of column block r / 2, register h
        const int base = ((kb * NJ + (r >> 1)) * kWarp + 16 * (r & 1) + tt) * 2 + h;
#pragma unroll
        for (int l = 0; l < 4; ++l) sB32[base + 8 * l] = wl[l];
      }  // rows >= M hold zeros: their fragments come out zero
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) qs += __shfl_xor_sync(0xffffffffu, qs, o);
    if (lane == 0) s_wq[warp] = qs;
  }
  bar_sync_n(1, kSConsumers);

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
  for (; j < n_st; ++j) {
    const int slot = j % kStages;
    if (!mbar_wait(&full[slot], (j / kStages) & 1)) {
      ok = false;
      break;
    }
    const int nc = min(kStageChunks, n_cta - j * kStageChunks);
    const uint4* st = stages + (size_t)slot * kStageU4 + tl * kWarp + lane;
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
    if (lane == 0) mbar_arrive(&empty[slot]);
  }
  if (!ok) {
    // a copy never arrived: report, let issued copies land (bounded), and
    // make the whole CTA skip its output after the barriers below
    if (lane == 0) {
      atomicOr(p.err, kErrWaitTimeout);
      s_bad = 1;
    }
    for (int jj = j; jj < n_st && jj < j + kStages; ++jj)
      if (!mbar_wait(&full[jj % kStages], (jj / kStages) & 1)) break;
  }

  // ---- exact integer combine: lanes t and t^1 hold limbs {0,1} / {2,3} of
  //      row 2jn + t/2; tile rows g (u) and g+8 (16 u) ------------------------
  float r[NJ][2];  // [column block][tile row g / g+8], valid on even t
#pragma unroll
  for (int jn = 0; jn < NJ; ++jn) {
    const int c0 = acc[0][jn][0] + acc[1][jn][0], c1 = acc[0][jn][1] + acc[1][jn][1];
    const int c2 = acc[0][jn][2] + acc[1][jn][2], c3 = acc[0][jn][3] + acc[1][jn][3];
    const int sh = (t & 1) ? 16 : 0;
    long long vg = ((long long)c0 << sh) + ((long long)c1 << (sh + 8));
    long long vh = ((long long)c2 << sh) + ((long long)c3 << (sh + 8));
    vg += __shfl_xor_sync(0xffffffffu, vg, 1);
    vh += __shfl_xor_sync(0xffffffffu, vh, 1);
    vh >>= 4;  // row g + 8 was multiplied by 16 (exact)
    const int m = 2 * jn + (t >> 1);
    // the -8 sum_k q of the whole segment, once per tile (half 0)
    long long qsum = 0;
#pragma unroll
    for (int q = 0; q < kRowWarps; ++q) qsum += s_wq[m * kRowWarps + q];
    const long long corr = half == 0 ? 8 * qsum : 0;
    const float dq = s_deq[m];
    r[jn][0] = (float)(vg - corr) * dq;
    r[jn][1] = (float)(vh - corr) * dq;
  }
  const bool tile_ok = tile < p.n_tiles;
  const bool own = (t & 1) == 0;  // lanes that carry the values on

  // ---- merge the two halves of each tile (half 0 + half 1, fixed order) ------
  {
    float* red = reinterpret_cast<float*>(stages);  // the stage ring is drained
    bar_sync_n(1, kSConsumers);                     // every warp is past its last stage
    if (half == 1 && own) {
#pragma unroll
      for (int jn = 0; jn < NJ; ++jn) {
        red[((tl * NJ + jn) * 2 + 0) * kWarp + lane] = r[jn][0];
        red[((tl * NJ + jn) * 2 + 1) * kWarp + lane] = r[jn][1];
      }
    }
    bar_sync_n(1, kSConsumers);
    if (half == 1 || s_bad) return;  // CTA-uniform after the barrier (s_bad)
    if (own) {
#pragma unroll
      for (int jn = 0; jn < NJ; ++jn) {
        r[jn][0] += red[((tl * NJ + jn) * 2 + 0) * kWarp + lane];
        r[jn][1] += red[((tl * NJ + jn) * 2 + 1) * kWarp + lane];
      }
    }
  }

  // ---- k-segments of the group: the last CTA sums the partials in k order --
  if (p.ksplit > 1) {
    float* my = p.part + ((size_t)tile * p.ksplit + kidx) * (kTileN * MB);
    if (own) {
#pragma unroll
      for (int jn = 0; jn < NJ; ++jn) {
        const int m = 2 * jn + (t >> 1);
        __stcg(my + g * MB + m, r[jn][0]);
        __stcg(my + (g + 8) * MB + m, r[jn][1]);
      }
    }
    __threadfence();
    bar_sync_n(1, kSTileThreads);
    if (threadIdx.x == 0) s_last = (atomicAdd(p.counters + group, 1) == p.ksplit - 1);
    bar_sync_n(1, kSTileThreads);
    if (!s_last) return;
    __threadfence();
    if (own) {
#pragma unroll
      for (int jn = 0; jn < NJ; ++jn) r[jn][0] = r[jn][1] = 0.f;
      for (int kk = 0; kk < p.ksplit; ++kk) {
        const float* pp = p.part + ((size_t)tile * p.ksplit + kk) * (kTileN * MB);
#pragma unroll
        for (int jn = 0; jn < NJ; ++jn) {
          const int m = 2 * jn + (t >> 1);
          r[jn][0] += __ldcg(pp + g * MB + m);
          r[jn][1] += __ldcg(pp + (g + 8) * MB + m);
        }
      }
    }
    if (threadIdx.x == 0) p.counters[group] = 0;
  }

  // ---- epilogue: each warp finishes its tile --------------------------------
  if (!tile_ok) return;
#pragma unroll
  for (int jn = 0; jn < NJ; ++jn) {
    const int m = 2 * jn + (t >> 1);
    float sq = 0.f;
    if (own && m < p.M) {
      const float f = s_fin[m];
      epilogue_row(p, tile, g, m, r[jn][0] * f, r[jn][1] * f, s_fres[m], sq);
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

template <int MG>
static cudaError_t launch_stream_t(const GemvParams& p, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(padded_tiles(p.n_tiles) / kGroupTiles, p.ksplit, 1);
  cfg.blockDim = dim3(kSThreads);
  cfg.dynamicSmemBytes = gemv_stream_smem(MG, p.kseg);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gemv_stream_kernel<MG>, p);
}

// M <= 4 (MG 1) or M <= 8 (MG 2).  A k-segment holds at most 2560 / MG
// values per row (the prologue's registers; the int32 sums of tile rows g + 8,
// 16 u x |limb| <= 30720 per product, are exact far beyond that).
// x: 16-byte aligned rows, ldx % 4 == 0.
cudaError_t launch_gemv_stream(const GemvParams& p, int mg, cudaStream_t s, bool pdl) {
  if (p.M > 4 * mg || !p.x || (p.ldx & 3) || ((uintptr_t)p.x & 15) ||
      gemv_stream_smem(mg, p.kseg) > 200 * 1024 || p.kseg % kChunkK ||
      p.kseg > kMaxItems * 4 * (kSConsumers / (4 * mg)))
    return cudaErrorInvalidConfiguration;
  if (mg == 1) return launch_stream_t<1>(p, s, pdl);
  if (mg == 2) return launch_stream_t<2>(p, s, pdl);
  return cudaErrorInvalidConfiguration;
}

cudaError_t prepare_gemv_stream() {
  cudaError_t e = cudaFuncSetAttribute(gemv_stream_kernel<1>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gemv_stream_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             200 * 1024);
  return e;
}

}  // namespace ms
