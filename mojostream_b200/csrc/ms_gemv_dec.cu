// ms_gemv_dec.cu -- latency-optimised Q4 projection for decode batches
// (M <= 8 rows): the hot op of the token loop at batch 4
// (reference: matmul_q4_bpack_raw, src/linalg/kernels.mojo:201-267, and the
// steps fused around its call sites, src/main.mojo:538-613,
// src/inference/gemma4_e4b.mojo:459-540).
//
// At decode a layer's matrices are 2.6-26 MB, i.e. 0.4-4 us of HBM time, so
// the kernel is shaped around latency rather than reuse:
//   * one CTA = one 16-column tile x a k-segment; its 8 warps split the
//     segment and are reduced through shared memory in a fixed order;
//   * every weight word of the CTA is requested (128-bit, L1 no-allocate)
//     before griddepcontrol.wait, so under programmatic dependent launch the
//     weight stream of kernel i+1 overlaps the tail of kernel i;
//   * after the wait there is one dependent step: the activations (L2) are
//     split into bf16 hi | lo fragments in shared memory;
//   * RMSNorm and PLE are per-row scalars, so they are applied to the finished
//     sums in the epilogue instead of to the inputs (no dependency on the row
//     statistics before the MMAs);
//   * long-K matrices (the down projection) split K over a few CTAs; the last
//     CTA of a tile sums the partials in k order (deterministic).
// Tensor cores: mma.m16n8k16 bf16 with the weight tile as A (int4 -> bf16 in
// registers) and [hi | lo] of 4 rows as the 8 B columns.
#include "ms_common.cuh"
#include "ms_epilogue.cuh"
#include "ms_kernels.h"

namespace ms {

constexpr int kDecWarps = 8;
constexpr int kDecThreads = kDecWarps * kWarp;

template <int MG, int CH>
__global__ void __launch_bounds__(kDecThreads) gemv_dec_kernel(const GemvParams p) {
  constexpr int MB = 4 * MG;
  extern __shared__ uint2 sB[];                  // [chunks of the CTA * 4][MG][32]
  __shared__ float s_red[kDecWarps][kTileN * MB];  // per-warp partial sums
  __shared__ float s_fin[MB], s_fres[MB];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, kidx = blockIdx.y;
  const int nchunks = p.K / kChunkK;
  const int seg = p.kseg / kChunkK;
  const int c_begin = kidx * seg;
  const int c_end = min(nchunks, c_begin + seg);
  const int n_cta = c_end - c_begin;
  const int per_warp = (n_cta + kDecWarps - 1) / kDecWarps;  // <= CH (host guarantees)
  const int w_begin = c_begin + warp * per_warp;
  const int w_end = min(c_end, w_begin + per_warp);

  // ---- 1. the CTA's weights, requested before the dependency wait ---------
  uint4 wr[CH];
  {
    const uint4* wt = p.w + (size_t)tile * nchunks * kWarp + lane;
#pragma unroll
    for (int c = 0; c < CH; ++c)
      if (w_begin + c < w_end) wr[c] = ld_stream_u4(wt + (size_t)(w_begin + c) * kWarp);
  }
  pdl_trigger();
  pdl_wait();

  // ---- 2. per-row factors (consumed only by the epilogue) -----------------
  if (warp < MB) {
    const int m = warp;
    float fin = p.in_ple, fres = 1.f;
    if (m < p.M) {
      if (p.in_stats) {
        float s = 0.f;
        for (int i = lane; i < p.in_nstat; i += kWarp) s += p.in_stats[(size_t)i * p.M + m];
        s = warp_sum(s);
        fin = p.in_ple / sqrtf(p.in_ple * p.in_ple * s / (float)p.in_D + 1e-6f);
      }
      if (p.epi == kEpiResid && p.resid_stats) {
        float s = 0.f;
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

  // ---- 3. activations of the CTA's k-segment -> bf16 hi | lo fragments ----
  {
    uint32_t* sBw = reinterpret_cast<uint32_t*>(sB);
    const int k_base = c_begin * kChunkK;
    const int items = n_cta * 4 * MB * 4;  // (subtile, row, quad of 4 k)
#pragma unroll 4
    for (int it = threadIdx.x; it < items; it += kDecThreads) {
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
      // pairs kp = 2q (k 4q, 4q+1) and 2q + 1 (k 4q+2, 4q+3)
      const int G = ml >> 2, mm = ml & 3;
      const int row = (ks * MG + G) * kWarp;
      const int kp0 = 2 * q, kp1 = 2 * q + 1;
      sBw[(row + mm * 4 + (kp0 & 3)) * 2 + (kp0 >> 2)] = hi0;
      sBw[(row + (mm + 4) * 4 + (kp0 & 3)) * 2 + (kp0 >> 2)] = lo0;
      sBw[(row + mm * 4 + (kp1 & 3)) * 2 + (kp1 >> 2)] = hi1;
      sBw[(row + (mm + 4) * 4 + (kp1 & 3)) * 2 + (kp1 >> 2)] = lo1;
    }
  }
  __syncthreads();

  // ---- 4. tensor cores ------------------------------------------------------
  float acc[MG][4];
#pragma unroll
  for (int G = 0; G < MG; ++G)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[G][i] = 0.f;
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    if (w_begin + c < w_end) {
      const uint32_t words[4] = {wr[c].x, wr[c].y, wr[c].z, wr[c].w};
      const int ks0 = (w_begin - c_begin + c) * 4;
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
#pragma unroll
  for (int G = 0; G < MG; ++G)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[G][i] += __shfl_xor_sync(0xffffffffu, acc[G][i], 2);

  const int g = lane >> 2, tq = lane & 3;
  // ---- 5. reduce the 8 warps (fixed order) ------------------------------------
  if (tq < 2) {
#pragma unroll
    for (int G = 0; G < MG; ++G) {
      const int mc = 4 * G + 2 * tq;
      *reinterpret_cast<float2*>(&s_red[warp][g * MB + mc]) = make_float2(acc[G][0], acc[G][1]);
      *reinterpret_cast<float2*>(&s_red[warp][(g + 8) * MB + mc]) = make_float2(acc[G][2], acc[G][3]);
    }
  }
  __syncthreads();
  if (warp != 0) return;
  if (tq < 2) {
#pragma unroll
    for (int G = 0; G < MG; ++G) {
      const int mc = 4 * G + 2 * tq;
      float2 a = make_float2(0.f, 0.f), b = make_float2(0.f, 0.f);
#pragma unroll
      for (int w = 0; w < kDecWarps; ++w) {
        const float2 ra = *reinterpret_cast<const float2*>(&s_red[w][g * MB + mc]);
        const float2 rb = *reinterpret_cast<const float2*>(&s_red[w][(g + 8) * MB + mc]);
        a.x += ra.x;
        a.y += ra.y;
        b.x += rb.x;
        b.y += rb.y;
      }
      acc[G][0] = a.x;
      acc[G][1] = a.y;
      acc[G][2] = b.x;
      acc[G][3] = b.y;
    }
  }

  // ---- 6. split-K over CTAs: the last CTA of the tile sums in k order -------
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
    __syncwarp();
    int last = 0;
    if (lane == 0) last = (atomicAdd(p.counters + tile, 1) == p.ksplit - 1);
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) return;
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
    if (lane == 0) p.counters[tile] = 0;
  }

  // ---- 7. epilogue (warp 0) --------------------------------------------------
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

template <int MG, int CH>
static cudaError_t launch_dec_t(const GemvParams& p, cudaStream_t s, bool pdl) {
  const size_t smem = (size_t)(p.kseg / kChunkK) * 4 * MG * kWarp * sizeof(uint2);
  auto kern = gemv_dec_kernel<MG, CH>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.n_tiles, p.ksplit, 1);
  cfg.blockDim = dim3(kDecThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

// M <= 4 (MG 1) or M <= 8 (MG 2); kseg <= 8 warps x 8 chunks x 64 = 4096.
cudaError_t launch_gemv_dec(const GemvParams& p, int mg, cudaStream_t s, bool pdl) {
  if (p.kseg > kDecWarps * 8 * kChunkK || p.M > 4 * mg) return cudaErrorInvalidConfiguration;
  if (mg == 1) return launch_dec_t<1, 8>(p, s, pdl);
  if (mg == 2) return launch_dec_t<2, 8>(p, s, pdl);
  return cudaErrorInvalidConfiguration;
}

cudaError_t prepare_gemv_dec() {
  // dynamic shared memory above 48 KB (k-segments up to 4096), set once
  cudaError_t e = cudaFuncSetAttribute(gemv_dec_kernel<1, 8>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gemv_dec_kernel<2, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             128 * 1024);
  return e;
}

}  // namespace ms
