// ms_gemm_tc.cu -- Q4 projection for prefill and large batches on the
// 5th-generation tensor cores (tcgen05, accumulators in tensor memory).
// Reference: matmul_q4_bpack_raw (src/linalg/kernels.mojo:201-267) with the
// steps fused around its call sites (src/main.mojo:538-613,
// src/inference/gemma4_e4b.mojo:459-540) in the epilogue.
//
// Arithmetic (exact integer products, like the decode kernel's):
//   * each input row x (K values) is quantised once per projection by
//     quant_rows_kernel: a = max |x|, q = rint(x 2^22 / a), |q| <= 2^22, split
//     into three signed 8-bit limbs q = d0 + 2^8 d1 + 2^16 d2 (balanced
//     digits, |d2| <= 64).  The error is 2^-23 a per value, far below the
//     fp32 rounding of the sums.
//   * weights are the reference's nibbles u (0..15); the kernel unpacks them
//     in shared memory to s8 values u - 8 (the reference's dequant without
//     the per-tensor scale, which is applied once in fp32 at the end).
//   * per limb one s8 x s8 -> s32 MMA chain over all of K; |sum| <= K * 8 *
//     128 < 2^31 for K <= 2^21.  The epilogue combines the limbs in int64 and
//     scales by (a / 2^22) * (RMSNorm factor) * (weight scale).
//
// CTA tile: 128 rows x 128 columns (one tile group of 8 x 16 columns), the
// whole K.  Warp roles: warp 0 streams stages with cp.async.bulk (24 KB of
// limbs + 4 KB of packed nibbles per 64-k chunk, 5-stage mbarrier ring);
// warp 1 allocates 512 tensor-memory columns and one thread issues the
// MMAs (3 limbs x 2 k32 steps per chunk; M 128, N 128, K 32); warps 2-9
// unpack the nibbles into the B operand; warps 2-5 run the epilogue (tensor
// memory lane = row).  Every wait is bounded (error word + drain on timeout).
#include "ms_common.cuh"
#include "ms_epilogue.cuh"
#include "ms_kernels.h"
#include "ms_tc.cuh"

namespace ms {

constexpr int kTcBM = 128;
constexpr int kTcBN = kGroupTiles * kTileN;              // 128
constexpr int kTcLimbs = 3;
constexpr int kTcStages = 5;
constexpr int kTcPlane = kTcBM * kChunkK;                // 8 KB: one limb of 128 rows x 64 k
constexpr int kTcAStage = kTcLimbs * kTcPlane;           // 24 KB
constexpr int kTcBPacked = kGroupTiles * kWarp * 16;     // 4 KB
constexpr int kTcBConv = kTcBN * kChunkK;                // 8 KB
constexpr int kTcStageBytes = kTcAStage + kTcBPacked + kTcBConv;
constexpr int kTcConvWarps = 8;
constexpr int kTcThreads = (2 + kTcConvWarps) * kWarp;   // 320
constexpr uint32_t kTcCols = 512;                        // 3 x 128 used
constexpr float kTcQuantOne = 4194304.0f;                // 2^22
constexpr int kTcRowS = kTcBN + 4;  // staged output row (floats): 16-byte aligned, 4-way banks
constexpr size_t kTcSmem = (size_t)kTcStages * kTcStageBytes;
// Core matrices: K-adjacent 128 bytes apart, row groups 512 bytes apart.
constexpr uint32_t kTcLbo = 128, kTcSbo = 512;

static_assert(kTcStageBytes % 1024 == 0, "stage alignment");
static_assert((size_t)kTcBM * kTcRowS * 4 <= (size_t)kTcStages * kTcStageBytes, "staged tile");

int tc_rows_pad(int M) { return (M + kTcBM - 1) / kTcBM * kTcBM; }
size_t tc_limb_bytes(int M, int K) { return (size_t)tc_rows_pad(M) * K * kTcLimbs; }

// ------------------------------------------------------------- quantiser --
// Rows of x -> limb planes in the MMA's A layout:
//   lq[(m_tile * nchunks + chunk) * 3 + limb][row group][k16][row % 8][16 B]
// Byte j of a 16-byte core row holds k = 2t + 8 (e & 1) + (e >> 1) of its
// 16-k subtile (t = j / 4, e = j % 4): the order of the weight words.
// rowf[m] = {(a / 2^22) * fin, fres}: the factors the epilogue applies.
// CTA (row group, k slice): 8 rows, 256 threads; thread (row tid % 8,
// subtile tid / 8 + 32 j).  The k slices of a row group (up to 8, so small
// batches still spread over many CTAs) run as one thread-block cluster: each
// CTA takes the maximum over its own slice, the row maxima are exchanged
// through distributed shared memory, and every CTA quantises its slice with
// the whole row's maximum; slice 0 writes the row factors.  Rows >= M are
// written as zeros.
constexpr int kQThreads = 256;
__global__ void __launch_bounds__(kQThreads) quant_rows_kernel(const GemvParams p) {
  __shared__ float s_max[kQThreads / kWarp][8];
  const int r8 = threadIdx.x & 7, sub0 = threadIdx.x >> 3;
  const int m = blockIdx.x * 8 + r8;
  const int mt = m / kTcBM, r = m % kTcBM;
  const int nchunks = p.K / kChunkK, nsub = p.K / 16;
  const int s_begin = (int)((long long)nsub * blockIdx.y / gridDim.y);
  const int s_end = (int)((long long)nsub * (blockIdx.y + 1) / gridDim.y);
  const bool live = m < p.M;
  pdl_wait();
  pdl_trigger();
  const float* x = p.x + (size_t)(live ? m : 0) * p.ldx;
  // a thread's subtiles are i = s_begin + sub0 + 32 u; they are loaded kQB at
  // a time (all loads of a batch issued before any use)
  constexpr int kQB = 4, kQStep = kQThreads / 8;
  float a = 0.f;
  if (live)
    for (int i0 = s_begin + sub0; i0 < s_end; i0 += kQB * kQStep) {
      float4 b[kQB][4];
#pragma unroll
      for (int u = 0; u < kQB; ++u) {
        const int i = i0 + u * kQStep;
        const float4* v4 = reinterpret_cast<const float4*>(x + 16 * i);
#pragma unroll
        for (int q = 0; q < 4; ++q) b[u][q] = i < s_end ? __ldg(v4 + q) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < kQB; ++u)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 v = b[u][q];
          a = fmaxf(a, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
    }
  // lanes with equal lane % 8 share a row
  a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 8));
  a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 16));
  if ((threadIdx.x & 31) < 8) s_max[threadIdx.x >> 5][r8] = a;
  __syncthreads();
#pragma unroll
  for (int w = 0; w < kQThreads / kWarp; ++w) a = fmaxf(a, s_max[w][r8]);
  if (gridDim.y > 1) {
    // the other slices' maxima of these rows (the slices are one cluster)
    __shared__ float s_slice_max[8];
    if (threadIdx.x < 8) s_slice_max[threadIdx.x] = a;  // thread r8 = threadIdx.x
    cluster_arrive();
    cluster_wait();
    const uint32_t m0 = smem_u32(&s_slice_max[r8]);
    for (uint32_t r = 0; r < gridDim.y; ++r) a = fmaxf(a, ld_dsmem(dsmem_addr(m0, r)));
    cluster_arrive();  // done reading the other CTAs' maxima
    cluster_wait();
  }
  const float inv = a > 0.f ? kTcQuantOne / a : 0.f;

  // RMSNorm factors from the per-tile sums of squares: the 32 threads of a
  // row each sum a strided share, then one fixed-order tree (deterministic)
  if (blockIdx.y == 0) {
    __shared__ float s_part[2][kQThreads / 8][8];
    float si = 0.f, sr = 0.f;
    if (live && p.in_stats)
      for (int i = sub0; i < p.in_nstat; i += kQThreads / 8) si += p.in_stats[(size_t)i * p.M + m];
    if (live && p.epi == kEpiResid && p.resid_stats)
      for (int i = sub0; i < p.resid_nstat; i += kQThreads / 8)
        sr += p.resid_stats[(size_t)i * p.M + m];
    s_part[0][sub0][r8] = si;
    s_part[1][sub0][r8] = sr;
    __syncthreads();
    if (sub0 == 0) {
      si = 0.f;
      sr = 0.f;
      for (int i = 0; i < kQThreads / 8; ++i) {
        si += s_part[0][i][r8];
        sr += s_part[1][i][r8];
      }
      float fin = p.in_ple, fres = 1.f;
      if (live && p.in_stats) fin = p.in_ple / sqrtf(p.in_ple * p.in_ple * si / (float)p.in_D + 1e-6f);
      if (live && p.epi == kEpiResid && p.resid_stats)
        fres = 1.0f / sqrtf(p.resid_ple * p.resid_ple * sr / (float)p.in_D + 1e-6f);
      p.rowf[m] = live ? make_float2(a / kTcQuantOne * fin, fres) : make_float2(0.f, 0.f);
    }
  }

  for (int i0 = s_begin + sub0; i0 < s_end; i0 += kQB * kQStep) {
    float4 b[kQB][4];
#pragma unroll
    for (int u = 0; u < kQB; ++u) {
      const int i = i0 + u * kQStep;
      const float4* v4 = reinterpret_cast<const float4*>(x + 16 * i);
#pragma unroll
      for (int q = 0; q < 4; ++q)
        b[u][q] = (live && i < s_end) ? __ldg(v4 + q) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < kQB; ++u) {
      const int i = i0 + u * kQStep;
      if (i >= s_end) break;
      const float v[16] = {b[u][0].x, b[u][0].y, b[u][0].z, b[u][0].w,
                           b[u][1].x, b[u][1].y, b[u][1].z, b[u][1].w,
                           b[u][2].x, b[u][2].y, b[u][2].z, b[u][2].w,
                           b[u][3].x, b[u][3].y, b[u][3].z, b[u][3].w};
      uint32_t wl[kTcLimbs][4];
#pragma unroll
      for (int l = 0; l < kTcLimbs; ++l)
#pragma unroll
        for (int t = 0; t < 4; ++t) wl[l][t] = 0u;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int t = j >> 2, e = j & 3;
        const int k = 2 * t + (e & 1) * 8 + (e >> 1);
        int q = __float2int_rn(v[k] * inv);
        const int d0 = (int)(int8_t)(q & 0xFF);
        q = (q - d0) >> 8;  // exact: a multiple of 256
        const int d1 = (int)(int8_t)(q & 0xFF);
        q = (q - d1) >> 8;  // |q| <= 64
        wl[0][t] |= ((uint32_t)d0 & 0xFFu) << (8 * e);
        wl[1][t] |= ((uint32_t)d1 & 0xFFu) << (8 * e);
        wl[2][t] |= ((uint32_t)q & 0xFFu) << (8 * e);
      }
      const int c = i >> 2, s = i & 3;
      uint8_t* dst = p.lq + (size_t)(mt * nchunks + c) * kTcAStage + ((r >> 3) * 4 + s) * 128 +
                     (r & 7) * 16;
#pragma unroll
      for (int l = 0; l < kTcLimbs; ++l)
        *reinterpret_cast<uint4*>(dst + l * kTcPlane) =
            make_uint4(wl[l][0], wl[l][1], wl[l][2], wl[l][3]);
    }
  }
}

// --------------------------------------------------------------- GEMM --
__global__ void __launch_bounds__(kTcThreads, 1) gemm_tc_kernel(const GemvParams p) {
  extern __shared__ __align__(1024) uint8_t dsm[];
  __shared__ __align__(8) uint64_t full[kTcStages], conv[kTcStages], empty[kTcStages], done;
  __shared__ uint32_t s_tmem;
  __shared__ volatile int s_bad;
  __shared__ int s_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int group = blockIdx.x, mt = blockIdx.y;
  const int nchunks = p.K / kChunkK;
  // k slice of this CTA (split-K when the tile grid alone cannot fill the GPU)
  const int kidx = blockIdx.z, seg = p.kseg / kChunkK;
  const int c_begin = kidx * seg;
  const int n_loc = min(nchunks, c_begin + seg) - c_begin;

  if (threadIdx.x == 0) {
    s_bad = 0;
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], kTcConvWarps);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&done, 1);
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(&s_tmem, kTcCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  pdl_trigger();

  if (warp == 0) {
    // ------------------------------------------------------- producer --
    if (lane == 0) {
      pdl_wait();  // the limbs are the previous kernel's output
      const uint8_t* a_src = p.lq + ((size_t)mt * nchunks + c_begin) * kTcAStage;
      const uint4* b_src = p.w + ((size_t)group * nchunks + c_begin) * kGroupTiles * kWarp;
      int c = 0;
      for (; c < n_loc; ++c) {
        const int s = c % kTcStages;
        if (c >= kTcStages && !mbar_wait(&empty[s], ((c / kTcStages) - 1) & 1)) {
          atomicOr(p.err, kErrWaitTimeout);
          s_bad = 1;
          break;
        }
        uint8_t* st = dsm + (size_t)s * kTcStageBytes;
        mbar_expect_tx(&full[s], kTcAStage + kTcBPacked);
        bulk_g2s(st, a_src + (size_t)c * kTcAStage, kTcAStage, &full[s]);
        bulk_g2s(st + kTcAStage, b_src + (size_t)c * kGroupTiles * kWarp, kTcBPacked, &full[s]);
      }
      if (s_bad) {
        // let the copies already issued land before the CTA can exit
        for (int j = c - 1; j >= 0 && j >= c - kTcStages; --j)
          if (!mbar_wait(&full[j % kTcStages], (j / kTcStages) & 1)) break;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------ MMA issuer --
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_i8(kTcBM, kTcBN);
      for (int c = 0; c < n_loc; ++c) {
        const int s = c % kTcStages;
        const uint32_t ph = (c / kTcStages) & 1;
        if (!mbar_wait(&full[s], ph) || !mbar_wait(&conv[s], ph)) {
          atomicOr(p.err, kErrWaitTimeout);
          s_bad = 1;
          break;
        }
        tc_fence_after();
        const uint32_t a0 = smem_u32(dsm + (size_t)s * kTcStageBytes);
        const uint32_t b0 = a0 + kTcAStage + kTcBPacked;
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
          const uint64_t db = umma_desc(b0 + kk * 256, kTcLbo, kTcSbo);
#pragma unroll
          for (int l = 0; l < kTcLimbs; ++l)
            umma_i8(tmem + l * kTcBN, umma_desc(a0 + l * kTcPlane + kk * 256, kTcLbo, kTcSbo), db,
                    idesc, (c | kk) != 0);
        }
        umma_commit(&empty[s]);
      }
      umma_commit(&done);  // arrives when every MMA issued above has finished
    }
  } else {
    // ---------------------------------------------- nibble unpacking --
    // thread ci: tile ci / 32 of the group, fragment lane (g, t) = ci % 32;
    // word w of its uint4 is k-subtile w of the chunk: low nibbles are tile
    // row g, high nibbles row g + 8, k order {2t, 2t+8, 2t+1, 2t+9}.
    const int ci = threadIdx.x - 2 * kWarp;
    const int tl = ci >> 5, g = (ci & 31) >> 2, t = ci & 3;
    for (int c = 0; c < n_loc; ++c) {
      const int s = c % kTcStages;
      if (!mbar_wait(&full[s], (c / kTcStages) & 1)) {
        atomicOr(p.err, kErrWaitTimeout);
        s_bad = 1;
        break;
      }
      uint8_t* st = dsm + (size_t)s * kTcStageBytes;
      const uint4 wv = lds_u4(reinterpret_cast<const uint4*>(st + kTcAStage) + ci);
      uint8_t* bc = st + kTcAStage + kTcBPacked + g * 16 + 4 * t;
      const uint32_t wd[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        // (u + 0x78) ^ 0x80 per byte = two's complement of u - 8 (no carries)
        const uint32_t lo = ((wd[w] & 0x0F0F0F0Fu) + 0x78787878u) ^ 0x80808080u;
        const uint32_t hi = (((wd[w] >> 4) & 0x0F0F0F0Fu) + 0x78787878u) ^ 0x80808080u;
        sts_u32(bc + ((2 * tl) * 4 + w) * 128, lo);
        sts_u32(bc + ((2 * tl + 1) * 4 + w) * 128, hi);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&conv[s]);
    }

    // ------------------------------------------------------- epilogue --
    // Phase 1 (warps 2-5, tensor-memory lane = row): combine the limbs of
    // the 128 x 128 tile and stage it in shared memory (the stage ring is
    // idle: every copy landed and every MMA completed before `done`).
    // Phase 2 (warps 2-9): write the tile row by row, lanes along the
    // columns, so every store instruction covers contiguous bytes.
    pdl_wait();
    const bool ok = mbar_wait(&done, 0);
    tc_fence_after();
    if (!ok && threadIdx.x == 2 * kWarp) atomicOr(p.err, kErrWaitTimeout);
    float* S = reinterpret_cast<float*>(dsm);  // [kTcBM][kTcRowS]
    if (warp < 2 + 4) {
      const int quad = warp & 3;  // tensor-memory lanes 32 quad .. +31
      const int row = quad * kWarp + lane;
      const int m = mt * kTcBM + row;
      const float dq = (ok && m < p.M) ? p.rowf[m].x : 0.f;
      const uint32_t tl_addr = tmem + ((uint32_t)(quad * kWarp) << 16);
      for (int j = 0; j < kGroupTiles && ok; ++j) {
        uint32_t a0[16], a1[16], a2[16];
        tmem_ld16(tl_addr + 0 * kTcBN + 16 * j, a0);
        tmem_ld16(tl_addr + 1 * kTcBN + 16 * j, a1);
        tmem_ld16(tl_addr + 2 * kTcBN + 16 * j, a2);
        tmem_wait_ld();
        float v[16];
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          const long long iv = (long long)(int)a0[q] + 256LL * (long long)(int)a1[q] +
                               65536LL * (long long)(int)a2[q];
          v[q] = (float)iv * dq;
        }
        float4* dst = reinterpret_cast<float4*>(S + row * kTcRowS + 16 * j);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          dst[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
      }
    }
    bar_sync_n(2, kTcConvWarps * kWarp);
    bool finish = ok && !s_bad;
    if (finish && p.ksplit > 1) {
      // every k slice stores its rows < M; the last one (ticket) sums the
      // slices in k order into S and finishes the tile
      const int t8 = threadIdx.x - 2 * kWarp;  // 0 .. 255
      const int rows = min(kTcBM, p.M - mt * kTcBM);
      const size_t tile_id = (size_t)mt * gridDim.x + group;
      float* part = p.part + tile_id * p.ksplit * (kTcBM * kTcBN);
      for (int i = t8; i < rows * (kTcBN / 4); i += kTcConvWarps * kWarp) {
        const int r = i / (kTcBN / 4), c4 = i % (kTcBN / 4);
        __stcg(reinterpret_cast<float4*>(part + (size_t)kidx * kTcBM * kTcBN + r * kTcBN) + c4,
               *reinterpret_cast<const float4*>(S + r * kTcRowS + 4 * c4));
      }
      bar_sync_n(2, kTcConvWarps * kWarp);
      if (t8 == 0) s_last = ticket_acq_rel(p.counters + tile_id) == p.ksplit - 1;
      bar_sync_n(2, kTcConvWarps * kWarp);
      finish = s_last != 0;
      if (finish) {
        for (int i = t8; i < rows * (kTcBN / 4); i += kTcConvWarps * kWarp) {
          const int r = i / (kTcBN / 4), c4 = i % (kTcBN / 4);
          float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int kk = 0; kk < p.ksplit; ++kk) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(
                part + (size_t)kk * kTcBM * kTcBN + r * kTcBN) + c4);
            a.x += v.x; a.y += v.y; a.z += v.z; a.w += v.w;
          }
          *reinterpret_cast<float4*>(S + r * kTcRowS + 4 * c4) = a;
        }
        if (t8 == 0) p.counters[tile_id] = 0;
        bar_sync_n(2, kTcConvWarps * kWarp);
      }
    }
    if (finish && p.peer_tiles) {
      // tensor parallel: this rank's share of the tile -> its peer-visible
      // buffer, one release per tile (use counter), wait until every rank's
      // counter for the tile reached the same use, then sum the ranks' tiles
      // in rank order (the same bits on every rank) into S
      const int t8 = threadIdx.x - 2 * kWarp;
      const int rows = min(kTcBM, p.M - mt * kTcBM);
      const size_t tile_id = (size_t)mt * gridDim.x + group;
      float* mine = p.peer_tiles[p.tp_rank] + tile_id * (kTcBM * kTcBN);
      for (int i = t8; i < rows * (kTcBN / 4); i += kTcConvWarps * kWarp) {
        const int r = i / (kTcBN / 4), c4 = i % (kTcBN / 4);
        __stcg(reinterpret_cast<float4*>(mine + r * kTcBN) + c4,
               *reinterpret_cast<const float4*>(S + r * kTcRowS + 4 * c4));
      }
      bar_sync_n(2, kTcConvWarps * kWarp);
      if (t8 == 0) {
        fence_acq_rel_sys();
        const int use = atomicAdd_system(p.peer_flags[p.tp_rank] + tile_id, 1) + 1;
        int ok_all = 1;
        for (int r = 0; r < p.tp_world && ok_all; ++r)
          if (r != p.tp_rank) ok_all = wait_counter_sys(p.peer_flags[r] + tile_id, use);
        if (!ok_all) {
          atomicOr(p.err, kErrWaitTimeout);
          s_bad = 1;
        }
        fence_acq_rel_sys();
      }
      bar_sync_n(2, kTcConvWarps * kWarp);
      finish = !s_bad;
      if (finish) {
        for (int i = t8; i < rows * (kTcBN / 4); i += kTcConvWarps * kWarp) {
          const int r = i / (kTcBN / 4), c4 = i % (kTcBN / 4);
          float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int rk = 0; rk < p.tp_world; ++rk) {
            const float4 v = ld_sys_f4(reinterpret_cast<const float4*>(
                p.peer_tiles[rk] + tile_id * (kTcBM * kTcBN) + r * kTcBN) + c4);
            a.x += v.x; a.y += v.y; a.z += v.z; a.w += v.w;
          }
          *reinterpret_cast<float4*>(S + r * kTcRowS + 4 * c4) = a;
        }
        bar_sync_n(2, kTcConvWarps * kWarp);
      }
    }
    if (finish) {
      const int w8 = warp - 2;
      const int jt = lane >> 2;                  // tile of the group this lane covers
      const int tile = group * kGroupTiles + jt;
      const bool tile_ok = tile < p.n_tiles;
      for (int r = w8; r < kTcBM; r += kTcConvWarps) {
        const int m = mt * kTcBM + r;
        if (m >= p.M) break;  // warp-uniform
        const float* Sr = S + r * kTcRowS;
        if (p.epi == kEpiStore || p.epi == kEpiAccum || p.epi == kEpiResid) {
          const int c = group * kTcBN + 4 * lane;
          float4 v = *reinterpret_cast<const float4*>(Sr + 4 * lane);
          float4 o;
          float sq = 0.f;
          if (p.epi == kEpiResid) {
            const float fres = p.rowf[m].y;
            const float4 rr = __ldcg(reinterpret_cast<const float4*>(p.resid + (size_t)m * p.ldr + c));
            o.x = (rr.x * p.resid_ple) * fres + p.scale * v.x;
            o.y = (rr.y * p.resid_ple) * fres + p.scale * v.y;
            o.z = (rr.z * p.resid_ple) * fres + p.scale * v.z;
            o.w = (rr.w * p.resid_ple) * fres + p.scale * v.w;
            sq = o.x * o.x + o.y * o.y + o.z * o.z + o.w * o.w;
          } else {
            o = make_float4(p.scale * v.x, p.scale * v.y, p.scale * v.z, p.scale * v.w);
            if (p.epi == kEpiAccum && tile_ok) {
              const float4 cur = __ldcg(reinterpret_cast<const float4*>(p.out + (size_t)m * p.ldo + c));
              o.x = cur.x + o.x; o.y = cur.y + o.y; o.z = cur.z + o.z; o.w = cur.w + o.w;
            }
          }
          if (tile_ok) *reinterpret_cast<float4*>(p.out + (size_t)m * p.ldo + c) = o;
          if (p.epi == kEpiResid && p.out_stats) {
            sq += __shfl_xor_sync(0xffffffffu, sq, 1);
            sq += __shfl_xor_sync(0xffffffffu, sq, 2);
            if (tile_ok && (lane & 3) == 0) p.out_stats[(size_t)tile * p.M + m] = sq;
          }
        } else if (p.epi == kEpiSwiGLU) {
          // tile rows 0-7 gate, 8-15 up of the same output column
          const int g0 = 2 * (lane & 3);
          const float2 gv = *reinterpret_cast<const float2*>(Sr + 16 * jt + g0);
          const float2 uv = *reinterpret_cast<const float2*>(Sr + 16 * jt + 8 + g0);
          float h[2];
          const float gs[2] = {gv.x, gv.y}, us[2] = {uv.x, uv.y};
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const float gt = p.scale * gs[e], up = p.scale2 * us[e];
            const float sig = 1.0f / (1.0f + expf(-gt));
            h[e] = up * gt * sig;
          }
          if (tile_ok)
            *reinterpret_cast<float2*>(p.out + (size_t)m * p.ldo + group * (kTcBN / 2) + 2 * lane) =
                make_float2(h[0], h[1]);
        } else if (p.epi == kEpiQKV && tile_ok) {
          const int g0 = 2 * (lane & 3);
          const QkvTile td = p.tiles[tile];
          const float sc = td.dst == 0 ? p.sq : (td.dst == 1 ? p.sk : p.sv);
          const float2 lv = *reinterpret_cast<const float2*>(Sr + 16 * jt + g0);
          const float2 hv = *reinterpret_cast<const float2*>(Sr + 16 * jt + 8 + g0);
          float lo[2] = {sc * lv.x, sc * lv.y}, hi[2] = {sc * hv.x, sc * hv.y};
          const int pos = p.pos[m];
          if (td.rope_i0 >= 0) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const float th = (float)pos * p.inv_freq[td.rope_i0 + g0 + e];
              const float cs = cosf(th), sn = sinf(th);
              const float ra = lo[e] * cs - hi[e] * sn;
              const float rb = lo[e] * sn + hi[e] * cs;
              lo[e] = ra;
              hi[e] = rb;
            }
          }
          float* base;
          size_t off;
          int bf = 0;
          if (td.dst == 0) {
            base = p.q_out;
            off = (size_t)m * p.ldq;
          } else {
            base = kv_dst(p.kv, td.dst, m, p.seq[m], pos, off, bf);
          }
          kv_put2(base, bf, off + td.col_lo + g0, lo[0], lo[1]);
          kv_put2(base, bf, off + td.col_hi + g0, hi[0], hi[1]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    // no MMA may still write the columns being freed (bounded, as every wait)
    mbar_wait(&done, 0);
    tc_fence_after();
    tmem_dealloc(tmem, kTcCols);
  }
}

// The first `rows` rows (a multiple of 8; rows >= M written as zeros) of the
// limb planes and their row factors.
cudaError_t launch_quant_rows(const GemvParams& p, int rows, cudaStream_t s, bool pdl) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  // k slices so that a small batch still has about one CTA per SM (each
  // slice re-reads the rows for their maximum, so large batches keep one)
  const int groups = rows / 8, nsub = p.K / 16;
  int ks = (148 + groups - 1) / groups;
  ks = ks < 1 ? 1 : (ks > nsub / 32 ? (nsub / 32 > 0 ? nsub / 32 : 1) : ks);
  ks = ks > 8 ? 8 : ks;  // the slices of a row group form one (portable) cluster
  cudaLaunchAttribute attr2[2] = {attr[0], {}};
  int na = pdl ? 1 : 0;
  if (ks > 1) {
    attr2[na].id = cudaLaunchAttributeClusterDimension;
    attr2[na].val.clusterDim.x = 1;
    attr2[na].val.clusterDim.y = (unsigned)ks;
    attr2[na].val.clusterDim.z = 1;
    ++na;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(groups, ks);
  cfg.blockDim = dim3(kQThreads);
  cfg.stream = s;
  cfg.attrs = attr2;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, quant_rows_kernel, p);
}

cudaError_t launch_gemm_tc(const GemvParams& p, cudaStream_t s, bool pdl) {
  if (p.ksplit < 1 || p.kseg % kChunkK || p.kseg <= 0 || (p.ksplit > 1 && (!p.part || !p.counters)) ||
      (long long)p.kseg * (p.ksplit - 1) >= p.K)
    return cudaErrorInvalidConfiguration;
  if (p.K % kChunkK || !p.lq || !p.rowf || !p.x || (p.ldx & 3) || ((uintptr_t)p.x & 15) ||
      ((uintptr_t)p.lq & 15) || ((uintptr_t)p.rowf & 7) || p.M <= 0)
    return cudaErrorInvalidConfiguration;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  const int m_pad = tc_rows_pad(p.M);
  cudaError_t e = launch_quant_rows(p, m_pad, s, pdl);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(padded_tiles(p.n_tiles) / kGroupTiles, m_pad / kTcBM, p.ksplit);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = kTcSmem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;  // the quantiser just before it is always a PDL-aware kernel
  return cudaLaunchKernelEx(&cfg, gemm_tc_kernel, p);
}

cudaError_t prepare_gemm_tc() {
  return cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)kTcSmem);
}

}  // namespace ms
