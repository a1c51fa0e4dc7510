// ms_gemv_stream.cu -- Q4 projection for decode batches (M <= 8 rows), the
// hot op of the token loop at batch 4 (reference: matmul_q4_bpack_raw,
// src/linalg/kernels.mojo:201-267, with the steps fused around its call
// sites in src/main.mojo:538-613 and src/inference/gemma4_e4b.mojo:459-540).
//
// A decode step reads every weight once with only 4 activation rows, so the
// kernel is an HBM stream, balanced "stream-K" style over the whole matrix:
//   * the weights are one contiguous sequence of stage units (tile group g,
//     k-chunks 4s..4s+3: 16 KB); CTA i of C (one per SM) takes units
//     [i T / C, (i+1) T / C), so every SM streams the same number of bytes;
//   * one producer thread moves each unit with cp.async.bulk through a
//     4-deep mbarrier ring, together with the unit's slice of the activation
//     rows, which arrive pre-split into bf16 hi | lo MMA fragments (written by
//     the kernel that produced them).  The first units' weights are requested
//     before griddepcontrol.wait (they do not depend on the previous kernel);
//   * 16 consumer warps, two per tile of the group, dequantise int4 -> bf16
//     in registers (exact) and run mma.m16n8k16 with 4 rows x {hi, lo} as the
//     8 B columns, over 4 independent accumulator chains;
//   * when a CTA leaves a group it flushes the group: the epilogue directly if
//     the CTA covered the group's whole K, else a partial to scratch; the last
//     CTA to flush a shared group (atomic ticket) sums the partials in CTA
//     order and runs the epilogue -- deterministic results;
//   * RMSNorm and PLE are per-row scalars applied to the finished sums.
#include <algorithm>

#include "ms_common.cuh"
#include "ms_epilogue.cuh"
#include "ms_kernels.h"

namespace ms {

// Two consumer warps per tile (16 per CTA): warp w computes tile w % 8 over
// chunks {2h, 2h+1} of every unit, h = w / 8.
constexpr int kSHalves = 2;
constexpr int kSWarps = kGroupTiles * kSHalves;       // consumer warps
constexpr int kSConsumers = kSWarps * kWarp;          // 512
constexpr int kSThreads = kSConsumers + kWarp;        // + producer warp
constexpr int kSTileThreads = kGroupTiles * kWarp;    // one warp per tile after the merge
constexpr int kStageChunks = 4;
constexpr int kStages = 4;
constexpr int kStageU4 = kStageChunks * kGroupTiles * kWarp;  // 1024 uint4 = 16 KB of weights
constexpr int kStageBytes = kStageU4 * 16;
constexpr int kUnitKs = kStageChunks * 4;                     // 16-k subtiles per unit

// Per stage: 16 KB of weights + the unit's fragments (4 KB per 4-row block);
// plus the merge buffer of the two halves.
size_t gemv_stream_smem(int mg) {
  return (size_t)kStages * (kStageBytes + (size_t)kUnitKs * kWarp * sizeof(uint2) * mg) +
         (size_t)kGroupTiles * mg * 4 * kWarp * sizeof(float);
}

// CTA owning stage unit u when T units are split over C CTAs.
__device__ __forceinline__ int unit_owner(long u, long T, int C) {
  int i = (int)((u * C) / T);
  while (i + 1 < C && ((long)(i + 1) * T) / C <= u) ++i;
  while (i > 0 && ((long)i * T) / C > u) --i;
  return i;
}

template <int MG>
// minBlocks 2: register budget for two CTAs per SM, so that under
// programmatic dependent launch the next projection's CTA fits beside this one
__global__ void __launch_bounds__(kSThreads, 2) gemv_stream_kernel(const GemvParams p) {
  constexpr int MB = 4 * MG;
  constexpr int kBU2 = kUnitKs * kWarp * MG;  // fragment uint2 per stage
  extern __shared__ __align__(128) uint8_t dsm[];
  uint4* stages = reinterpret_cast<uint4*>(dsm);
  uint2* sB = reinterpret_cast<uint2*>(dsm + kStages * kStageBytes);  // [stage][G][ks][32]
  float* red = reinterpret_cast<float*>(dsm + kStages * kStageBytes + kStages * kBU2 * 8);
  __shared__ __align__(8) uint64_t full[kStages], empty[kStages];
  __shared__ float s_fin[MB], s_fres[MB];
  __shared__ int s_last, s_bad, s_issued;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int C = gridDim.x, cta = blockIdx.x;
  const int nchunks = p.K / kChunkK;
  const int S = (nchunks + kStageChunks - 1) / kStageChunks;  // units per group
  const int n_groups = padded_tiles(p.n_tiles) / kGroupTiles;
  const long T = (long)n_groups * S;
  const long u_begin = ((long)cta * T) / C, u_end = ((long)(cta + 1) * T) / C;
  const int n_units = (int)(u_end - u_begin);
  const int KS = p.K / 16;

  if (threadIdx.x == 0) {
    s_bad = 0;
    s_issued = 0;
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kSWarps);
    }
    mbar_fence_init();
  }
  __syncthreads();
  pdl_trigger();

  // ------------------------------------------------------------ producer --
  if (warp == kSWarps) {
    if (lane == 0) {
      auto unit_chunks = [&](long u, int& g, int& c0) {
        g = (int)(u / S);
        c0 = (int)(u % S) * kStageChunks;
        return min(kStageChunks, nchunks - c0);
      };
      auto issue_w = [&](int j) {
        int g, c0;
        const int nc = unit_chunks(u_begin + j, g, c0);
        const int slot = j % kStages;
        const uint32_t wbytes = (uint32_t)nc * kGroupTiles * kWarp * 16;
        const uint32_t bbytes = (uint32_t)nc * 4 * kWarp * sizeof(uint2) * MG;
        mbar_expect_tx(&full[slot], wbytes + bbytes);
        bulk_g2s(stages + (size_t)slot * kStageU4,
                 p.w + ((size_t)g * nchunks + c0) * kGroupTiles * kWarp, wbytes, &full[slot]);
      };
      auto issue_b = [&](int j) {
        int g, c0;
        const int nc = unit_chunks(u_begin + j, g, c0);
        const int slot = j % kStages;
        const uint32_t gb = (uint32_t)nc * 4 * kWarp * sizeof(uint2);
        for (int G = 0; G < MG; ++G)
          bulk_g2s(sB + (size_t)slot * kBU2 + (size_t)G * kUnitKs * kWarp,
                   p.xfrag + ((size_t)G * KS + c0 * 4) * kWarp, gb, &full[slot]);
      };
      const int first = min(n_units, kStages);
      for (int j = 0; j < first; ++j) issue_w(j);  // weights: before the wait
      *reinterpret_cast<volatile int*>(&s_issued) = first;
      pdl_wait();
      for (int j = 0; j < first; ++j) issue_b(j);
      for (int j = first; j < n_units; ++j) {
        if (!mbar_wait(&empty[j % kStages], ((j / kStages) - 1) & 1)) {
          atomicOr(p.err, kErrWaitTimeout);
          s_bad = 1;
          break;  // consumers stop at the first unit never issued
        }
        issue_w(j);
        issue_b(j);
        *reinterpret_cast<volatile int*>(&s_issued) = j + 1;
      }
    }
    return;
  }

  // ----------------------------------------------------------- consumers --
  pdl_wait();
  const int tl = warp & (kGroupTiles - 1), half = warp / kGroupTiles;
  const int g8 = lane >> 2, tq = lane & 3;
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
  bar_sync_n(1, kSConsumers);  // factors visible

  float acc[4][MG][4];
#pragma unroll
  for (int s = 0; s < 4; ++s)
#pragma unroll
    for (int G = 0; G < MG; ++G)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[s][G][i] = 0.f;
  bool ok = true;
  // group / stage index of the current unit, stepped without divisions (a
  // 64-bit division per unit cost more than the unit's math)
  int g = (int)(u_begin / S), s_idx = (int)(u_begin % S);
  int g_first_s = s_idx;  // stage index at which this CTA entered group g
  auto mma_chunk = [&](const uint4* st, const uint2* bs, int cc) {
    const uint4 wv = lds_u4(st + cc * kGroupTiles * kWarp);
    const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      uint32_t a[4];
      dequant_word(words[s], a);
#pragma unroll
      for (int G = 0; G < MG; ++G) {
        const uint2 b = bs[(G * kUnitKs + cc * 4 + s) * kWarp];
        mma_bf16_16816(acc[s][G], a, b.x, b.y);
      }
    }
  };
  for (int j = 0; j < n_units; ++j) {
    const int slot = j & (kStages - 1);
    if (ok && *reinterpret_cast<volatile int*>(&s_bad)) ok = false;  // another warp gave up
    if (ok && !mbar_wait(&full[slot], (j / kStages) & 1)) {
      ok = false;
      if (lane == 0) {
        atomicOr(p.err, kErrWaitTimeout);
        s_bad = 1;
      }
    }
    if (ok) {
      const uint4* st = stages + slot * kStageU4 + tl * kWarp + lane;
      const uint2* bs = sB + slot * kBU2 + lane;
      constexpr int kHalf = kStageChunks / kSHalves;
      const int nc = nchunks - s_idx * kStageChunks;  // chunks left in the group
      if (nc >= kStageChunks) {                        // full stage: no branches
#pragma unroll
        for (int c2 = 0; c2 < kHalf; ++c2) mma_chunk(st, bs, half * kHalf + c2);
      } else {
        for (int c2 = 0; c2 < kHalf; ++c2)
          if (half * kHalf + c2 < nc) mma_chunk(st, bs, half * kHalf + c2);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }

    // ---- leaving group g: flush it ------------------------------------------
    const bool last_of_group = (s_idx + 1 == S);
    const bool group_end = (j + 1 == n_units) || last_of_group;
    const bool whole = (g_first_s == 0) && last_of_group;
    const int g_cur = g;
    if (last_of_group) {
      ++g;
      s_idx = 0;
      g_first_s = 0;
    } else {
      ++s_idx;
    }
    if (!group_end) continue;
    float r[MG][4];
#pragma unroll
    for (int G = 0; G < MG; ++G)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float v = (acc[0][G][i] + acc[1][G][i]) + (acc[2][G][i] + acc[3][G][i]);
        r[G][i] = v + __shfl_xor_sync(0xffffffffu, v, 2);  // fold lo (cols 4-7) onto hi
        acc[0][G][i] = acc[1][G][i] = acc[2][G][i] = acc[3][G][i] = 0.f;
      }
    // merge the two halves of each tile (half 0 + half 1, fixed order)
    bar_sync_n(1, kSConsumers);  // previous flush's readers are done with `red`
    if (half == 1 && tq < 2) {
#pragma unroll
      for (int G = 0; G < MG; ++G)
#pragma unroll
        for (int i = 0; i < 4; ++i) red[((tl * MG + G) * 4 + i) * kWarp + lane] = r[G][i];
    }
    bar_sync_n(1, kSConsumers);
    const int tile = g_cur * kGroupTiles + tl;
    // (after a timeout the sums are garbage but every warp still takes the
    // same barriers; the host sees the error word)
    if (half == 0) {
      if (tq < 2) {
#pragma unroll
        for (int G = 0; G < MG; ++G)
#pragma unroll
          for (int i = 0; i < 4; ++i) r[G][i] += red[((tl * MG + G) * 4 + i) * kWarp + lane];
      }
      bool finish = whole;
      if (!whole) {
        // group shared with neighbouring CTAs: partial, ticket, last one sums
        const int c_first = unit_owner((long)g_cur * S, T, C);
        const int c_last = unit_owner((long)(g_cur + 1) * S - 1, T, C);
        float* my = p.part +
                    (((size_t)g_cur * p.ksplit + (cta - c_first)) * kGroupTiles + tl) * (kTileN * MB);
        if (tq < 2) {
#pragma unroll
          for (int G = 0; G < MG; ++G) {
            const int mc = 4 * G + 2 * tq;
            __stcg(reinterpret_cast<float2*>(my + g8 * MB + mc), make_float2(r[G][0], r[G][1]));
            __stcg(reinterpret_cast<float2*>(my + (g8 + 8) * MB + mc),
                   make_float2(r[G][2], r[G][3]));
          }
        }
        // the barrier orders the warps' stores before thread 0's release fence
        // and ticket; the last CTA's acquire fence orders its reads after
        bar_sync_n(2, kSTileThreads);
        if (threadIdx.x == 0) {
          asm volatile("fence.acq_rel.gpu;" ::: "memory");
          s_last = (atomicAdd(p.counters + g_cur, 1) == c_last - c_first);
          if (s_last) asm volatile("fence.acq_rel.gpu;" ::: "memory");
        }
        bar_sync_n(2, kSTileThreads);
        finish = s_last;
        if (finish) {
          if (tq < 2) {
#pragma unroll
            for (int G = 0; G < MG; ++G)
#pragma unroll
              for (int i = 0; i < 4; ++i) r[G][i] = 0.f;
            for (int c = 0; c <= c_last - c_first; ++c) {
              const float* pp =
                  p.part + (((size_t)g_cur * p.ksplit + c) * kGroupTiles + tl) * (kTileN * MB);
#pragma unroll
              for (int G = 0; G < MG; ++G) {
                const int mc = 4 * G + 2 * tq;
                const float2 a = __ldcg(reinterpret_cast<const float2*>(pp + g8 * MB + mc));
                const float2 b = __ldcg(reinterpret_cast<const float2*>(pp + (g8 + 8) * MB + mc));
                r[G][0] += a.x;
                r[G][1] += a.y;
                r[G][2] += b.x;
                r[G][3] += b.y;
              }
            }
          }
          if (threadIdx.x == 0) p.counters[g_cur] = 0;
        }
      }
      if (finish && tile < p.n_tiles) {
#pragma unroll
        for (int G = 0; G < MG; ++G) {
#pragma unroll
          for (int b = 0; b < 2; ++b) {
            const int m = 4 * G + 2 * (tq & 1) + b;
            float sq = 0.f;
            if (tq < 2 && m < p.M) {
              const float f = s_fin[m];
              epilogue_row(p, tile, g8, m, r[G][b] * f, r[G][2 + b] * f, s_fres[m], sq);
            }
            if (p.epi == kEpiResid && p.out_stats) {
              sq += __shfl_xor_sync(0xffffffffu, sq, 4);
              sq += __shfl_xor_sync(0xffffffffu, sq, 8);
              sq += __shfl_xor_sync(0xffffffffu, sq, 16);
              if (g8 == 0 && tq < 2 && m < p.M) p.out_stats[(size_t)tile * p.M + m] = sq;
            }
          }
        }
      }
    }
  }
  // fault path: let every copy the producer issued land before the CTA (and
  // its shared memory) goes away; bounded waits
  if (*reinterpret_cast<volatile int*>(&s_bad) && threadIdx.x == 0) {
    const int issued = *reinterpret_cast<volatile int*>(&s_issued);
    for (int jj = max(0, issued - kStages); jj < issued; ++jj)
      mbar_wait(&full[jj % kStages], (jj / kStages) & 1);
  }
}

template <int MG>
static cudaError_t launch_stream_t(const GemvParams& p, int ctas, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas, 1, 1);
  cfg.blockDim = dim3(kSThreads);
  cfg.dynamicSmemBytes = gemv_stream_smem(MG);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gemv_stream_kernel<MG>, p);
}

// Host mirror of the partition: the most CTAs any group is shared by (the
// partial-slot count the scratch needs), for `ctas` CTAs.
int gemv_stream_max_share(int n_tiles, int K, int ctas) {
  const int nchunks = K / kChunkK;
  const long S = (nchunks + kStageChunks - 1) / kStageChunks;
  const long T = (long)(padded_tiles(n_tiles) / kGroupTiles) * S;
  auto owner = [&](long u) {
    int i = (int)((u * ctas) / T);
    while (i + 1 < ctas && ((long)(i + 1) * T) / ctas <= u) ++i;
    while (i > 0 && ((long)i * T) / ctas > u) --i;
    return i;
  };
  int best = 1;
  for (long g = 0; g * S < T; ++g) best = std::max(best, owner((g + 1) * S - 1) - owner(g * S) + 1);
  return best;
}

// M <= 4 (MG 1) or M <= 8 (MG 2); p.xfrag holds the input rows as fragments;
// p.ksplit carries the partial-slot count per group (gemv_stream_max_share).
cudaError_t launch_gemv_stream(const GemvParams& p, int mg, int ctas, cudaStream_t s, bool pdl) {
  if (p.M > 4 * mg || !p.xfrag || p.K % kChunkK || ctas < 1) return cudaErrorInvalidConfiguration;
  if (mg == 1) return launch_stream_t<1>(p, ctas, s, pdl);
  if (mg == 2) return launch_stream_t<2>(p, ctas, s, pdl);
  return cudaErrorInvalidConfiguration;
}

cudaError_t prepare_gemv_stream() {
  cudaError_t e = cudaFuncSetAttribute(gemv_stream_kernel<1>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)gemv_stream_smem(1));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gemv_stream_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)gemv_stream_smem(2));
  return e;
}

}  // namespace ms
