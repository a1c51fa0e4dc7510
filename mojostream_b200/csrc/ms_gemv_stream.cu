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
//   * after the wait the consumers split the activations of the k-segment
//     into bf16 hi | lo MMA fragments once (shared by the 8 tiles);
//   * each warp dequantises its tile in registers (int4 -> bf16, exact) and
//     runs mma.m16n8k16 with the 4 rows x {hi, lo} as the 8 B columns;
//   * RMSNorm and PLE are per-row scalars applied to the finished sums;
//   * k-segments of one group (long K, or to fill the GPU) are summed by the
//     last CTA of the group in k order: deterministic results.
#include "ms_common.cuh"
#include "ms_epilogue.cuh"
#include "ms_kernels.h"

namespace ms {

constexpr int kSWarps = kGroupTiles;                   // consumer warps = tiles per group
constexpr int kSConsumers = kSWarps * kWarp;          // 256
constexpr int kSThreads = kSConsumers + kWarp;        // + producer warp
constexpr int kStageChunks = 4;
constexpr int kStages = 4;
constexpr int kStageU4 = kStageChunks * kGroupTiles * kWarp;  // 1024 uint4 = 16 KB
constexpr int kStageBytes = kStageU4 * 16;

size_t gemv_stream_smem(int mg, int kseg) {
  const int chunks = kseg / kChunkK;
  return (size_t)kStages * kStageBytes + (size_t)chunks * 4 * mg * kWarp * sizeof(uint2);
}

template <int MG>
__global__ void __launch_bounds__(kSThreads) gemv_stream_kernel(const GemvParams p) {
  constexpr int MB = 4 * MG;
  extern __shared__ __align__(128) uint8_t dsm[];
  uint4* stages = reinterpret_cast<uint4*>(dsm);
  uint2* sB = reinterpret_cast<uint2*>(dsm + kStages * kStageBytes);
  __shared__ __align__(8) uint64_t full[kStages], empty[kStages];
  __shared__ float s_fin[MB], s_fres[MB];
  __shared__ int s_last;

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
      for (int j = 0; j < n_st; ++j) {
        const int slot = j % kStages;
        if (j >= kStages && !mbar_wait(&empty[slot], ((j / kStages) - 1) & 1)) {
          atomicOr(p.err, kErrWaitTimeout);
          break;  // consumers time out on the stages never issued
        }
        const int c0 = c_begin + j * kStageChunks;
        const int nc = min(kStageChunks, c_end - c0);
        const uint32_t bytes = (uint32_t)nc * kGroupTiles * kWarp * 16;
        mbar_expect_tx(&full[slot], bytes);
        bulk_g2s(stages + (size_t)slot * kStageU4, wg + (size_t)c0 * kGroupTiles * kWarp, bytes,
                 &full[slot]);
      }
    }
    return;
  }

  // ----------------------------------------------------------- consumers --
  pdl_wait();
  const int tile = group * kGroupTiles + warp;
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
  // activations of the k-segment -> bf16 hi | lo fragments [subtile][G][lane]
  {
    uint32_t* sBw = reinterpret_cast<uint32_t*>(sB);
    const int k_base = c_begin * kChunkK;
    const int items = n_cta * 4 * MB * 4;  // (subtile, row, quad of 4 k)
#pragma unroll 4
    for (int it = threadIdx.x; it < items; it += kSConsumers) {
      const int q = it & 3;
      const int ml = (it >> 2) % MB;
      const int ks = (it >> 2) / MB;
      uint32_t hi0 = 0, lo0 = 0, hi1 = 0, lo1 = 0;
      if (ml < p.M) {
        const float4 xv = *reinterpret_cast<const float4*>(p.x + (size_t)ml * p.ldx + k_base +
                                                          ks * 16 + 4 * q);
        uint32_t h0, l0, h1, l1, h2, l2, h3, l3;
        split_bf16(xv.x, h0, l0);
        split_bf16(xv.y, h1, l1);
        split_bf16(xv.z, h2, l2);
        split_bf16(xv.w, h3, l3);
        hi0 = h0 | (h1 << 16);
        lo0 = l0 | (l1 << 16);
        hi1 = h2 | (h3 << 16);
        lo1 = l2 | (l3 << 16);
      }
      // k pairs 2q (k 4q, 4q+1) and 2q+1 (k 4q+2, 4q+3) of the subtile
      const int G = ml >> 2, mm = ml & 3;
      const int row = (ks * MG + G) * kWarp;
      const int kp0 = 2 * q, kp1 = 2 * q + 1;
      sBw[(row + mm * 4 + (kp0 & 3)) * 2 + (kp0 >> 2)] = hi0;
      sBw[(row + (mm + 4) * 4 + (kp0 & 3)) * 2 + (kp0 >> 2)] = lo0;
      sBw[(row + mm * 4 + (kp1 & 3)) * 2 + (kp1 >> 2)] = hi1;
      sBw[(row + (mm + 4) * 4 + (kp1 & 3)) * 2 + (kp1 >> 2)] = lo1;
    }
  }
  bar_sync_n(1, kSConsumers);

  float acc[MG][4];
#pragma unroll
  for (int G = 0; G < MG; ++G)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[G][i] = 0.f;
  bool ok = true;
  int j = 0;
  for (; j < n_st; ++j) {
    const int slot = j % kStages;
    if (!mbar_wait(&full[slot], (j / kStages) & 1)) {
      ok = false;
      break;
    }
    const int nc = min(kStageChunks, n_cta - j * kStageChunks);
    const uint4* st = stages + (size_t)slot * kStageU4 + warp * kWarp + lane;
#pragma unroll
    for (int cc = 0; cc < kStageChunks; ++cc) {
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
            const uint2 b = sB[((ks0 + s) * MG + G) * kWarp + lane];
            mma_bf16_16816(acc[G], a, b.x, b.y);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }
  if (!ok) {
    // a stage never arrived: report, let issued copies land, skip the output
    if (lane == 0) atomicOr(p.err, kErrWaitTimeout);
    for (int jj = j + 1; jj < n_st && jj < j + kStages; ++jj)
      if (!mbar_wait(&full[jj % kStages], (jj / kStages) & 1)) break;
    return;
  }
#pragma unroll
  for (int G = 0; G < MG; ++G)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[G][i] += __shfl_xor_sync(0xffffffffu, acc[G][i], 2);
  const int g = lane >> 2, tq = lane & 3;
  const bool tile_ok = tile < p.n_tiles;

  // ---- k-segments of the group: the last CTA sums the partials in k order --
  if (p.ksplit > 1) {
    float* my = p.part + ((size_t)tile * p.ksplit + kidx) * (kTileN * MB);
    if (tq < 2) {
#pragma unroll
      for (int G = 0; G < MG; ++G) {
        const int mc = 4 * G + 2 * tq;
        __stcg(reinterpret_cast<float2*>(my + g * MB + mc), make_float2(acc[G][0], acc[G][1]));
        __stcg(reinterpret_cast<float2*>(my + (g + 8) * MB + mc), make_float2(acc[G][2], acc[G][3]));
      }
    }
    __threadfence();
    bar_sync_n(1, kSConsumers);
    if (threadIdx.x == 0) s_last = (atomicAdd(p.counters + group, 1) == p.ksplit - 1);
    bar_sync_n(1, kSConsumers);
    if (!s_last) return;
    __threadfence();
    if (tq < 2) {
#pragma unroll
      for (int G = 0; G < MG; ++G)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[G][i] = 0.f;
      for (int kk = 0; kk < p.ksplit; ++kk) {
        const float* pp = p.part + ((size_t)tile * p.ksplit + kk) * (kTileN * MB);
#pragma unroll
        for (int G = 0; G < MG; ++G) {
          const int mc = 4 * G + 2 * tq;
          const float2 a = __ldcg(reinterpret_cast<const float2*>(pp + g * MB + mc));
          const float2 b = __ldcg(reinterpret_cast<const float2*>(pp + (g + 8) * MB + mc));
          acc[G][0] += a.x;
          acc[G][1] += a.y;
          acc[G][2] += b.x;
          acc[G][3] += b.y;
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
        epilogue_row(p, tile, g, m, acc[G][b] * f, acc[G][2 + b] * f, s_fres[m], sq);
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

// M <= 4 (MG 1) or M <= 8 (MG 2); the k-segment's fragments must fit in
// shared memory next to the stage ring (kseg <= 64 chunks for MG 1).
cudaError_t launch_gemv_stream(const GemvParams& p, int mg, cudaStream_t s, bool pdl) {
  if (p.M > 4 * mg || gemv_stream_smem(mg, p.kseg) > 200 * 1024 || p.kseg % kChunkK)
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
