// ms_gemv_stream.cu -- Q4 projection for decode batches (M <= 8 rows), the
// hot op of the token loop at batch 4 (reference: matmul_q4_bpack_raw,
// src/linalg/kernels.mojo:201-267, with the steps fused around its call
// sites in src/main.mojo:538-613 and src/inference/gemma4_e4b.mojo:459-540).
//
// A decode step reads every weight once with only 4 activation rows, so the
// kernel is an HBM stream.  Per CTA:
//   * 8 consumer warps own the 8 tiles (128 output columns) of one tile group;
//     one producer thread streams the group's k-segment with cp.async.bulk
//     (16 KB stages = 4 k-chunks x 8 tiles, contiguous in the weight layout)
//     through a 4-stage mbarrier ring.  The first stages are issued before
//     griddepcontrol.wait: weights do not depend on the previous kernel, so
//     under programmatic dependent launch their fetch overlaps its tail;
//   * the activations arrive already in MMA-fragment layout (bf16 hi | lo,
//     written by the kernel that produced them) with one more bulk copy
//     right after the wait: no conversion pass on the critical path;
//   * each warp dequantises its tile in registers (int4 -> bf16, exact) and
//     runs mma.m16n8k16 with the 4 rows x {hi, lo} as the 8 B columns, over
//     4 independent accumulator chains (one per 16-k subtile of a chunk);
//   * RMSNorm and PLE are per-row scalars applied to the finished sums;
//   * k-segments of one group (long K, or to fill the GPU) are summed by the
//     last CTA of the group in k order: deterministic results.
#include "ms_common.cuh"
#include "ms_epilogue.cuh"
#include "ms_kernels.h"

namespace ms {

// Two consumer warps per tile (16 per CTA): warp w computes tile w % 8 over
// chunks {2h, 2h+1} of every stage, h = w / 8.  Two warps per tile double the
// instruction streams a scheduler can interleave (the dequant -> MMA chain
// is latency-bound with one warp per tile).
constexpr int kSHalves = 2;
constexpr int kSWarps = kGroupTiles * kSHalves;       // consumer warps
constexpr int kSConsumers = kSWarps * kWarp;          // 512
constexpr int kSThreads = kSConsumers + kWarp;        // + producer warp
constexpr int kSTileThreads = kGroupTiles * kWarp;    // one warp per tile (after the halves merge)
constexpr int kStageChunks = 4;
constexpr int kStages = 4;
constexpr int kStageU4 = kStageChunks * kGroupTiles * kWarp;  // 1024 uint4 = 16 KB
constexpr int kStageBytes = kStageU4 * 16;

size_t gemv_stream_smem(int mg, int kseg) {
  const int chunks = kseg / kChunkK;
  return (size_t)kStages * kStageBytes + (size_t)chunks * 4 * mg * kWarp * sizeof(uint2);
}

template <int MG>
__global__ void __launch_bounds__(kSThreads, 2) gemv_stream_kernel(const GemvParams p) {
  constexpr int MB = 4 * MG;
  extern __shared__ __align__(128) uint8_t dsm[];
  uint4* stages = reinterpret_cast<uint4*>(dsm);
  uint2* sB = reinterpret_cast<uint2*>(dsm + kStages * kStageBytes);  // [G][ks][32]
  __shared__ __align__(8) uint64_t full[kStages], empty[kStages], bready;
  __shared__ float s_fin[MB], s_fres[MB];
  __shared__ int s_last, s_bad;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int group = blockIdx.x, kidx = blockIdx.y;
  if (threadIdx.x == 0) s_bad = 0;
  const int nchunks = p.K / kChunkK;
  const int seg = p.kseg / kChunkK;
  const int c_begin = kidx * seg;
  const int c_end = min(nchunks, c_begin + seg);
  const int n_cta = c_end - c_begin;
  const int n_st = (n_cta + kStageChunks - 1) / kStageChunks;
  const int ks_cta = n_cta * 4;  // 16-k subtiles of the segment
  const uint4* wg = p.w + (size_t)group * nchunks * kGroupTiles * kWarp;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kSWarps);
    }
    mbar_init(&bready, 1);
    mbar_fence_init();
  }
  __syncthreads();
  pdl_trigger();

  // ------------------------------------------------------------ producer --
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
      for (int j = 0; j < first; ++j) issue(j);  // weights: before the wait
      pdl_wait();
      // the k-segment's activation fragments, one copy per 4-row block
      const int KS = p.K / 16;
      const uint32_t gbytes = (uint32_t)ks_cta * kWarp * sizeof(uint2);
      mbar_expect_tx(&bready, gbytes * MG);
      for (int G = 0; G < MG; ++G)
        bulk_g2s(sB + (size_t)G * ks_cta * kWarp, p.xfrag + ((size_t)G * KS + c_begin * 4) * kWarp,
                 gbytes, &bready);
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
  // per-row factors, used by the epilogue only
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

  // 4 accumulator chains x MG row blocks
  float acc[4][MG][4];
#pragma unroll
  for (int s = 0; s < 4; ++s)
#pragma unroll
    for (int G = 0; G < MG; ++G)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[s][G][i] = 0.f;
  bool ok = mbar_wait(&bready, 0);
  int j = 0;
  for (; ok && j < n_st; ++j) {
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
        const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
        const int ks0 = (j * kStageChunks + cc) * 4;
#pragma unroll
        for (int s = 0; s < 4; ++s) {
          uint32_t a[4];
          dequant_word(words[s], a);
#pragma unroll
          for (int G = 0; G < MG; ++G) {
            const uint2 b = sB[((size_t)G * ks_cta + ks0 + s) * kWarp + lane];
            mma_bf16_16816(acc[s][G], a, b.x, b.y);
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
    mbar_wait(&bready, 0);
    for (int jj = j; jj < n_st && jj < j + kStages; ++jj)
      if (!mbar_wait(&full[jj % kStages], (jj / kStages) & 1)) break;
  }
  float r[MG][4];
#pragma unroll
  for (int G = 0; G < MG; ++G)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float v = (acc[0][G][i] + acc[1][G][i]) + (acc[2][G][i] + acc[3][G][i]);
      r[G][i] = v + __shfl_xor_sync(0xffffffffu, v, 2);  // fold lo (cols 4-7) onto hi
    }
  const int g = lane >> 2, tq = lane & 3;
  const bool tile_ok = tile < p.n_tiles;

  // ---- merge the two halves of each tile (half 0 + half 1, fixed order) ------
  {
    float* red = reinterpret_cast<float*>(stages);  // the stage ring is drained
    bar_sync_n(1, kSConsumers);                     // every warp is past its last stage
    if (half == 1 && tq < 2) {
#pragma unroll
      for (int G = 0; G < MG; ++G)
#pragma unroll
        for (int i = 0; i < 4; ++i) red[((tl * MG + G) * 4 + i) * 64 + lane] = r[G][i];
    }
    bar_sync_n(1, kSConsumers);
    if (half == 1 || s_bad) return;  // CTA-uniform after the barrier (s_bad)
    if (tq < 2) {
#pragma unroll
      for (int G = 0; G < MG; ++G)
#pragma unroll
        for (int i = 0; i < 4; ++i) r[G][i] += red[((tl * MG + G) * 4 + i) * 64 + lane];
    }
  }

  // ---- k-segments of the group: the last CTA sums the partials in k order --
  if (p.ksplit > 1) {
    float* my = p.part + ((size_t)tile * p.ksplit + kidx) * (kTileN * MB);
    if (tq < 2) {
#pragma unroll
      for (int G = 0; G < MG; ++G) {
        const int mc = 4 * G + 2 * tq;
        __stcg(reinterpret_cast<float2*>(my + g * MB + mc), make_float2(r[G][0], r[G][1]));
        __stcg(reinterpret_cast<float2*>(my + (g + 8) * MB + mc), make_float2(r[G][2], r[G][3]));
      }
    }
    __threadfence();
    bar_sync_n(1, kSTileThreads);
    if (threadIdx.x == 0) s_last = (atomicAdd(p.counters + group, 1) == p.ksplit - 1);
    bar_sync_n(1, kSTileThreads);
    if (!s_last) return;
    __threadfence();
    if (tq < 2) {
#pragma unroll
      for (int G = 0; G < MG; ++G)
#pragma unroll
        for (int i = 0; i < 4; ++i) r[G][i] = 0.f;
      for (int kk = 0; kk < p.ksplit; ++kk) {
        const float* pp = p.part + ((size_t)tile * p.ksplit + kk) * (kTileN * MB);
#pragma unroll
        for (int G = 0; G < MG; ++G) {
          const int mc = 4 * G + 2 * tq;
          const float2 a = __ldcg(reinterpret_cast<const float2*>(pp + g * MB + mc));
          const float2 b = __ldcg(reinterpret_cast<const float2*>(pp + (g + 8) * MB + mc));
          r[G][0] += a.x;
          r[G][1] += a.y;
          r[G][2] += b.x;
          r[G][3] += b.y;
        }
      }
    }
    if (threadIdx.x == 0) p.counters[group] = 0;
  }

  // ---- epilogue: each warp finishes its tile --------------------------------
  if (!tile_ok) return;
#pragma unroll
  for (int G = 0; G < MG; ++G) {
#pragma unroll
    for (int b = 0; b < 2; ++b) {
      const int m = 4 * G + 2 * (tq & 1) + b;
      float sq = 0.f;
      if (tq < 2 && m < p.M) {
        const float f = s_fin[m];
        epilogue_row(p, tile, g, m, r[G][b] * f, r[G][2 + b] * f, s_fres[m], sq);
      }
      if (p.epi == kEpiResid && p.out_stats) {
        sq += __shfl_xor_sync(0xffffffffu, sq, 4);
        sq += __shfl_xor_sync(0xffffffffu, sq, 8);
        sq += __shfl_xor_sync(0xffffffffu, sq, 16);
        if (g == 0 && tq < 2 && m < p.M) p.out_stats[(size_t)tile * p.M + m] = sq;
      }
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

// M <= 4 (MG 1) or M <= 8 (MG 2); p.xfrag holds the input rows as fragments;
// the k-segment's fragments must fit in shared memory next to the stage ring.
cudaError_t launch_gemv_stream(const GemvParams& p, int mg, cudaStream_t s, bool pdl) {
  if (p.M > 4 * mg || !p.xfrag || gemv_stream_smem(mg, p.kseg) > 200 * 1024 || p.kseg % kChunkK)
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
