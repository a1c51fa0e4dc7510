// ms_gemv.cu -- Q4 projection kernel for decode and small batches (M <= 64
// rows per m-block), the hot op of MojoStream's token loop
// (reference: matmul_q4_bpack_raw, src/linalg/kernels.mojo:201-267, and the
// RMSNorm / RoPE / KV-write / SwiGLU / residual steps around each of its call
// sites in src/main.mojo:538-613 and src/inference/gemma4_e4b.mojo:459-540).
//
// Design (B200):
//   * Swap-AB tensor-core GEMV: the weight tile (16 output columns x 16 k) is
//     the MMA's A operand, the activations are B, with batch rows hi / lo in
//     the 8 MMA columns (4 rows x {hi, lo}).  int4 -> bf16 dequant happens in
//     registers (one word = one A fragment), no shared-memory round trip.
//   * Each warp streams one 16-column tile over the CTA's k-segment with
//     128-bit non-allocating loads issued before griddepcontrol.wait, so the
//     weight fetch of kernel i+1 overlaps the tail of kernel i (PDL).
//   * The activation prologue (PLE + RMSNorm from per-tile partial sums of
//     squares produced by the previous kernel) builds the B fragments once per
//     CTA in shared memory.
//   * Split-K partials go to scratch; the last CTA of a column group (atomic
//     ticket) sums them in k order, so results do not depend on timing.
#include "ms_common.cuh"
#include "ms_epilogue.cuh"
#include "ms_kernels.h"

namespace ms {

constexpr int kGemvWarps = 4;
constexpr int kGemvThreads = kGemvWarps * kWarp;

template <int MG, int CH>
__device__ __forceinline__ void load_round(uint4 (&wr)[CH], const uint4* __restrict__ wt, int c0,
                                           int c_end, int lane) {
#pragma unroll
  for (int c = 0; c < CH; ++c)
    if (c0 + c < c_end) wr[c] = ld_stream_u4(wt + (size_t)(c0 + c) * kGroupTiles * kWarp + lane);
}

// grid: (m-blocks, column groups of 4 tiles, k-segments); 4 warps, one tile each.
// A CTA walks its k-segment in rounds of CH chunks (64 k each); the weights of
// round r + 1 are in flight while round r computes.
template <int MG, int CH>
__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(const GemvParams p) {
  constexpr int MB = 4 * MG;  // rows per m-block
  extern __shared__ uint2 sB[];  // [CH*4][MG][32]
  __shared__ float s_inv_in[MB];
  __shared__ float s_inv_res[MB];
  __shared__ int s_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mblk = blockIdx.x, ncta = blockIdx.y, kidx = blockIdx.z;
  const int n_ctas = gridDim.y;
  const int tile = ncta * kGemvWarps + warp;
  const bool tile_ok = tile < p.n_tiles;
  const int nchunks = p.K / kChunkK;
  const int seg_chunks = p.kseg / kChunkK;
  const int c_begin = kidx * seg_chunks;
  const int c_end = min(nchunks, c_begin + seg_chunks);
  const uint4* wt = p.w + tile_chunk_u4(tile, 0, nchunks);

  // ---- 1. weight prefetch: independent of every earlier kernel ----------
  uint4 wr[CH];
  if (tile_ok) load_round<MG, CH>(wr, wt, c_begin, c_end, lane);
  pdl_trigger();
  pdl_wait();

  const int m_base = mblk * MB;
  // ---- 2. per-row norm factors (a warp per row, lanes over the partials) ---
  for (int ml = warp; ml < MB; ml += kGemvWarps) {
    const int m = m_base + ml;
    float inv = 1.f, invr = 1.f;
    if (m < p.M) {
      if (p.in_stats) {
        float s = 0.f;
        for (int i = lane; i < p.in_nstat; i += kWarp) s += p.in_stats[(size_t)i * p.M + m];
        s = warp_sum(s);
        inv = 1.0f / sqrtf(p.in_ple * p.in_ple * s / (float)p.in_D + 1e-6f);
      }
      if (p.epi == kEpiResid && p.resid_stats) {
        float s = 0.f;
        for (int i = lane; i < p.resid_nstat; i += kWarp) s += p.resid_stats[(size_t)i * p.M + m];
        s = warp_sum(s);
        invr = 1.0f / sqrtf(p.resid_ple * p.resid_ple * s / (float)p.in_D + 1e-6f);
      }
    }
    if (lane == 0) {
      s_inv_in[ml] = inv;
      s_inv_res[ml] = invr;
    }
  }

  float acc[MG][4];
#pragma unroll
  for (int G = 0; G < MG; ++G)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[G][i] = 0.f;

  uint32_t* sBw = reinterpret_cast<uint32_t*>(sB);
  for (int c0 = c_begin; c0 < c_end; c0 += CH) {
    const int nch = min(CH, c_end - c0);
    __syncthreads();  // norm factors ready / previous round's fragments consumed
    // ---- 3. B fragments of this pass: x -> (ple x) inv -> bf16 hi | lo ----
    {
      const int k_base = c0 * kChunkK;
      const int items = nch * 4 * MB * 8;
      for (int it = threadIdx.x; it < items; it += kGemvThreads) {
        const int kp = it & 7;
        const int ml = (it >> 3) % MB;
        const int ks = (it >> 3) / MB;
        const int m = m_base + ml;
        uint32_t hi = 0, lo = 0;
        if (m < p.M) {
          const int k = k_base + ks * 16 + 2 * kp;
          const float2 xv = *reinterpret_cast<const float2*>(p.x + (size_t)m * p.ldx + k);
          const float inv = s_inv_in[ml];
          uint32_t h0, l0, h1, l1;
          split_bf16((xv.x * p.in_ple) * inv, h0, l0);
          split_bf16((xv.y * p.in_ple) * inv, h1, l1);
          hi = h0 | (h1 << 16);
          lo = l0 | (l1 << 16);
        }
        const int G = ml >> 2, mm = ml & 3, tq = kp & 3, reg = kp >> 2;
        const int row = (ks * MG + G) * kWarp;
        sBw[(row + mm * 4 + tq) * 2 + reg] = hi;
        sBw[(row + (mm + 4) * 4 + tq) * 2 + reg] = lo;
      }
    }
    __syncthreads();
    if (tile_ok) {
      uint4 cur[CH];
#pragma unroll
      for (int c = 0; c < CH; ++c) cur[c] = wr[c];
      if (c0 + CH < c_end) load_round<MG, CH>(wr, wt, c0 + CH, c_end, lane);
      // ---- 4. tensor-core main loop ----------------------------------------
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        if (c < nch) {
          const uint32_t words[4] = {cur[c].x, cur[c].y, cur[c].z, cur[c].w};
#pragma unroll
          for (int s = 0; s < 4; ++s) {
            uint32_t a[4];
            dequant_word(words[s], a);
#pragma unroll
            for (int G = 0; G < MG; ++G) {
              const uint2 b = sB[((c * 4 + s) * MG + G) * kWarp + lane];
              mma_bf16_16816(acc[G], a, b.x, b.y);
            }
          }
        }
      }
    }
  }
  // columns 0-3 hold the hi part of 4 rows, 4-7 the lo part: fold lo onto hi
#pragma unroll
  for (int G = 0; G < MG; ++G)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[G][i] += __shfl_xor_sync(0xffffffffu, acc[G][i], 2);

  const int g = lane >> 2, tq = lane & 3;

  // ---- 5. split-K: partials to scratch, last CTA reduces in k order -------
  if (p.ksplit > 1) {
    const size_t grp = (size_t)mblk * n_ctas + ncta;
    float* my = p.part + ((grp * p.ksplit + kidx) * kGemvWarps + warp) * (kTileN * MB);
    if (tile_ok && tq < 2) {
#pragma unroll
      for (int G = 0; G < MG; ++G) {
        const int mc = 4 * G + 2 * tq;
        *reinterpret_cast<float2*>(my + g * MB + mc) = make_float2(acc[G][0], acc[G][1]);
        *reinterpret_cast<float2*>(my + (g + 8) * MB + mc) = make_float2(acc[G][2], acc[G][3]);
      }
    }
    __syncthreads();  // partials written
    if (threadIdx.x == 0) s_last = (ticket_acq_rel(p.counters + grp) == p.ksplit - 1);
    __syncthreads();
    if (!s_last) return;
    if (tile_ok && tq < 2) {
#pragma unroll
      for (int G = 0; G < MG; ++G)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[G][i] = 0.f;
      for (int kk = 0; kk < p.ksplit; ++kk) {
        const float* pp = p.part + ((grp * p.ksplit + kk) * kGemvWarps + warp) * (kTileN * MB);
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
    if (threadIdx.x == 0) p.counters[grp] = 0;
  }

  // ---- 6. epilogue -----------------------------------------------------------
  if (!tile_ok) return;
#pragma unroll
  for (int G = 0; G < MG; ++G) {
#pragma unroll
    for (int b = 0; b < 2; ++b) {
      const int ml = 4 * G + 2 * (tq & 1) + b;
      const int m = m_base + ml;
      float sq = 0.f;
      if (tq < 2 && m < p.M)
        epilogue_row(p, tile, g, m, acc[G][b], acc[G][2 + b], s_inv_res[ml], sq);
      if (p.epi == kEpiResid && p.out_stats) {
        // sum the 16 columns of this tile: lanes with equal tq share a row m
        sq += __shfl_xor_sync(0xffffffffu, sq, 4);
        sq += __shfl_xor_sync(0xffffffffu, sq, 8);
        sq += __shfl_xor_sync(0xffffffffu, sq, 16);
        if (g == 0 && tq < 2 && m < p.M) p.out_stats[(size_t)tile * p.M + m] = sq;
      }
    }
  }
}

template <int MG, int CH>
static cudaError_t launch_t(const GemvParams& p, cudaStream_t s, bool pdl) {
  constexpr int MB = 4 * MG;
  const size_t smem = (size_t)CH * 4 * MG * kWarp * sizeof(uint2);
  auto kern = gemv_kernel<MG, CH>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((p.M + MB - 1) / MB, (p.n_tiles + kGemvWarps - 1) / kGemvWarps, p.ksplit);
  cfg.blockDim = dim3(kGemvThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

// Supported (MG, CH) pairs; kseg (the CTA's k-segment) is a multiple of CH * 64.
cudaError_t launch_gemv(const GemvParams& p, int mg, int ch, cudaStream_t s, bool pdl) {
#define MS_GEMV_CASE(MGV, CHV) \
  if (mg == MGV && ch == CHV) return launch_t<MGV, CHV>(p, s, pdl);
  MS_GEMV_CASE(1, 4) MS_GEMV_CASE(1, 8)
  MS_GEMV_CASE(2, 4) MS_GEMV_CASE(2, 8)
  MS_GEMV_CASE(4, 2) MS_GEMV_CASE(4, 4)
  MS_GEMV_CASE(8, 2) MS_GEMV_CASE(8, 4)
  MS_GEMV_CASE(16, 2)
#undef MS_GEMV_CASE
  return cudaErrorInvalidConfiguration;
}

}  // namespace ms
