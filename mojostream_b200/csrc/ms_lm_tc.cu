// ms_lm_tc.cu -- the lm_head for batches of 9 or more rows on the
// 5th-generation tensor cores.
// Reference: apply_final_norm (src/inference/lm_head.mojo:119-130 ->
// rmsnorm_weighted_inplace, src/linalg/kernels.mojo:598-613), project_lm_head
// (lm_head.mojo:146-168 -> matmul_fp32_raw, kernels.mojo:616-671) and the
// greedy branch of temperature_sampling (lm_head.mojo:224-230: the first
// maximum wins).
//
// Why: the CUDA-core kernel (ms_misc.cu) keeps 16 normalised rows per pass
// in shared memory and is bound by FMA issue from 8 rows up (4 passes over
// the 2.68 GB table at batch 64 take 2.5 ms; one read of the table at the
// measured copy bandwidth takes 0.42 ms).
//
// Arithmetic: logits[m][v] = sum_k xn[m][k] W[k][v] with xn the normalised
// row exactly as the CUDA-core kernel forms it (x * inv_rms * gamma, fp32).
// Both operands are split into bfloat16 pairs, a = a_hi + a_lo with
// a_hi = bf16(a), a_lo = bf16(a - a_hi) (|a - a_hi - a_lo| <= 2^-18 |a|), and
// three MMAs per k-step accumulate a_hi b_hi + a_hi b_lo + a_lo b_hi in fp32
// tensor memory (the dropped a_lo b_lo is below 2^-16 of the product): about
// 1e-5 relative per product, far inside the 1e-3 logits bar.
//
// Layout: the MMA's A operand (M = 128) is 128 vocabulary columns of W, B is
// the batch (N = rows rounded up to 16, <= 64 per launch).  lm_rows_kernel
// writes the rows' hi / lo planes once per launch, [k-chunk][hi | lo][N rows
// x 32 k] in the no-swizzle K-major core-matrix layout.  The main kernel is
// persistent: CTA b takes vocabulary groups b, b + grid, ...; per 32-k chunk
// warp 0 copies the group's 32 x 128 fp32 tile of W with one 2-D tensor copy
// (a tensor map over W; 32 row copies of 512 bytes each were bounded by the
// per-SM rate of copy requests) and the chunk's planes, warps 2-5 convert the fp32 tile in place to the hi | lo
// core matrices, warp 1 issues the MMAs into one of two tensor-memory
// accumulators (a group's MMAs overlap the previous group's epilogue), and
// warps 6-9 read the finished accumulator (lane = column, column = row),
// store the logits if asked and keep each row's running (max, first index).
// The CTAs' per-row results are merged by the last CTA (ticket) in index
// order.  Every wait is bounded (error word).
#include <cuda.h>

#include "ms_common.cuh"
#include "ms_kernels.h"
#include "ms_tc.cuh"

namespace ms {

// The 2-D box [y, y + 32) x [x, x + 128) of the tensor map into dst
// (row-major, no swizzle), completing on bar.  x * 4 bytes is a multiple of
// 16 (x is a multiple of 128); dst is 128-byte aligned.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

constexpr int kLtK = 32;                           // k per chunk: 64 bytes of bf16 per row
constexpr int kLtV = 128;                          // vocabulary columns per group (MMA M)
constexpr int kLtStages = 4;
constexpr int kLtMaxN = 64;                        // rows per launch
constexpr int kLtA = kLtV * kLtK * 4;              // 16 KB: fp32 [32 k][128 v], then hi | lo
constexpr int kLtHalf = kLtV * kLtK * 2;           // 8 KB: one bf16 part of A
constexpr int kLtBMax = 2 * kLtMaxN * kLtK * 2;    // 8 KB: hi | lo planes of 64 rows
constexpr int kLtStage = kLtA + kLtBMax;           // 24 KB
constexpr int kLtConvWarps = 4, kLtEpiWarps = 4;
constexpr int kLtThreads = (2 + kLtConvWarps + kLtEpiWarps) * kWarp;  // 320
constexpr uint32_t kLtCols = 2 * kLtMaxN;          // two accumulators of up to 64 columns
constexpr uint32_t kLtLbo = 128, kLtSbo = 512;
constexpr size_t kLtSmem = (size_t)kLtStages * kLtStage;

static_assert(kLtStage % 1024 == 0, "stage alignment");

// Byte offset of (row r, k-core kc) in a K-major no-swizzle operand whose
// rows hold 64 bytes (4 core matrices along k).
__device__ __forceinline__ uint32_t lm_core_off(int r, int kc) {
  return (uint32_t)((r >> 3) * kLtSbo + kc * kLtLbo + (r & 7) * 16);
}

// Eight fp32 values as bf16 hi and lo halves, packed in k order.
__device__ __forceinline__ void lm_split8(const float* v, uint4& hi, uint4& lo) {
  uint32_t h[8], l[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) split_bf16(v[j], h[j], l[j]);
  hi = make_uint4(h[0] | (h[1] << 16), h[2] | (h[3] << 16), h[4] | (h[5] << 16), h[6] | (h[7] << 16));
  lo = make_uint4(l[0] | (l[1] << 16), l[2] | (l[3] << 16), l[4] | (l[5] << 16), l[6] | (l[7] << 16));
}

// One CTA per plane row r (N of them; rows past the batch are zeros):
// xn = x * inv_rms * gamma as the CUDA-core kernel forms it, split to hi / lo.
__global__ void __launch_bounds__(256) lm_rows_kernel(const LmHeadParams p, int row0, int N) {
  __shared__ float s_inv;
  const int r = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool live = row0 + r < p.M;
  pdl_wait();
  pdl_trigger();
  if (warp == 0) {
    float inv = 1.f;
    if (live && p.stats) {
      float s = 0.f;
      for (int i = lane; i < p.nstat; i += kWarp) s += p.stats[(size_t)i * p.M + row0 + r];
      s = warp_sum(s);
      inv = 1.0f / sqrtf(s / (float)p.D + 1e-6f);
    }
    if (lane == 0) s_inv = inv;
  }
  __syncthreads();
  const float inv = s_inv;
  const size_t chunk = (size_t)2 * N * 64;  // hi | lo planes of one 32-k chunk
  for (int i = threadIdx.x; i < p.D / 8; i += blockDim.x) {
    const int k0 = 8 * i;
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float a = 0.f;
      if (live) {
        a = p.x[(size_t)(row0 + r) * p.D + k0 + j] * inv;
        if (p.gamma) a = a * p.gamma[k0 + j];
      }
      v[j] = a;
    }
    uint4 hi, lo;
    lm_split8(v, hi, lo);
    uint8_t* dst = p.planes + (size_t)(k0 / kLtK) * chunk + lm_core_off(r, (k0 % kLtK) / 8);
    *reinterpret_cast<uint4*>(dst) = hi;
    *reinterpret_cast<uint4*>(dst + (size_t)N * 64) = lo;
  }
}

__global__ void __launch_bounds__(kLtThreads, 2) lm_tc_kernel(const LmHeadParams p, int row0,
                                                              int N,
                                                              const __grid_constant__ CUtensorMap wmap) {
  extern __shared__ __align__(1024) uint8_t dsm[];
  __shared__ __align__(8) uint64_t full[kLtStages], conv[kLtStages], empty[kLtStages];
  __shared__ __align__(8) uint64_t acc_full[2], acc_empty[2], done;
  __shared__ uint32_t s_tmem;
  __shared__ volatile int s_bad, s_conv_bad;
  __shared__ float s_bv[kLtEpiWarps][kLtMaxN];
  __shared__ int s_bi[kLtEpiWarps][kLtMaxN];
  __shared__ int s_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_groups = p.V / kLtV, nk = p.D / kLtK;
  const int ng = n_groups > (int)blockIdx.x
                     ? (n_groups - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x
                     : 0;
  const int total = ng * nk;  // chunks this CTA streams
  const int rows = min(N, p.M - row0);
  const uint32_t b_bytes = (uint32_t)N * 64;  // one plane of a chunk

  if (threadIdx.x == 0) {
    s_bad = 0;
    s_conv_bad = 0;
    for (int s = 0; s < kLtStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], kLtConvWarps);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], kLtEpiWarps);
    }
    mbar_init(&done, 1);
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(&s_tmem, kLtCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  pdl_trigger();

  auto fail = [&]() {
    atomicOr(p.err, kErrWaitTimeout);
    s_bad = 1;
  };

  if (warp == 0) {
    // ------------------------------------------------------- producer --
    if (lane == 0) {
      auto w_rows = [&](int t, uint8_t* st) {  // the W tile of chunk t
        const int j = t / nk, c = t % nk;
        const int g = (int)blockIdx.x + j * (int)gridDim.x;
        tma_load_2d(st, &wmap, g * kLtV, c * kLtK, &full[t % kLtStages]);
      };
      auto planes = [&](int t, uint8_t* st) {
        const int c = t % nk;
        bulk_g2s(st + kLtA, p.planes + (size_t)c * 2 * b_bytes, 2 * b_bytes,
                 &full[t % kLtStages]);
      };
      const int first = min(total, kLtStages);
      for (int t = 0; t < first; ++t) {  // W does not depend on earlier kernels
        uint8_t* st = dsm + (size_t)t * kLtStage;
        mbar_expect_tx(&full[t], kLtA + 2 * b_bytes);
        w_rows(t, st);
      }
      pdl_wait();  // the planes are lm_rows_kernel's output
      for (int t = 0; t < first; ++t) planes(t, dsm + (size_t)t * kLtStage);
      int t = first;
      for (; t < total; ++t) {
        const int s = t % kLtStages;
        if (!mbar_wait(&empty[s], ((t / kLtStages) - 1) & 1)) {
          fail();
          break;
        }
        uint8_t* st = dsm + (size_t)s * kLtStage;
        mbar_expect_tx(&full[s], kLtA + 2 * b_bytes);
        w_rows(t, st);
        planes(t, st);
      }
      if (s_bad) {  // let the copies already issued land before the CTA can exit
        for (int j = t - 1; j >= 0 && j >= t - kLtStages; --j)
          if (!mbar_wait(&full[j % kLtStages], (j / kLtStages) & 1)) break;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------ MMA issuer --
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16(kLtV, N);
      for (int j = 0; j < ng && !s_bad; ++j) {
        const int a = j & 1;
        if (j >= 2 && !mbar_wait(&acc_empty[a], ((j >> 1) - 1) & 1)) {
          fail();
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(a * kLtMaxN);
        for (int c = 0; c < nk; ++c) {
          const int t = j * nk + c, s = t % kLtStages;
          const uint32_t ph = (t / kLtStages) & 1;
          if (!mbar_wait(&full[s], ph) || !mbar_wait(&conv[s], ph)) {
            fail();
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(dsm + (size_t)s * kLtStage);
          const uint32_t b0 = a0 + kLtA;
#pragma unroll
          for (int kk = 0; kk < 2; ++kk) {
            const uint64_t ah = umma_desc(a0 + kk * 256, kLtLbo, kLtSbo);
            const uint64_t al = umma_desc(a0 + kLtHalf + kk * 256, kLtLbo, kLtSbo);
            const uint64_t bh = umma_desc(b0 + kk * 256, kLtLbo, kLtSbo);
            const uint64_t bl = umma_desc(b0 + b_bytes + kk * 256, kLtLbo, kLtSbo);
            umma_bf16(d, ah, bh, idesc, (c | kk) != 0);
            umma_bf16(d, ah, bl, idesc, 1);
            umma_bf16(d, al, bh, idesc, 1);
          }
          umma_commit(&empty[s]);
        }
        if (s_bad) break;
        umma_commit(&acc_full[a]);
      }
      umma_commit(&done);  // arrives when every MMA issued above has finished
    }
  } else if (warp < 2 + kLtConvWarps) {
    // ------------------------------------------- fp32 -> bf16 hi | lo --
    // thread v: column v of the group; reads its 32 k values (consecutive
    // threads, consecutive words: no bank conflicts), then, after every
    // converter has read the tile, writes its row of the hi and lo operands
    // over it.
    // A timed-out wait is recorded in s_conv_bad before the barrier and
    // read after it, so every converter warp leaves at the same chunk (none
    // is left waiting at the barrier).
    const int v = threadIdx.x - 2 * kWarp;
    for (int t = 0; t < total; ++t) {
      const int s = t % kLtStages;
      uint8_t* st = dsm + (size_t)s * kLtStage;
      float w[kLtK];
      if (mbar_wait(&full[s], (t / kLtStages) & 1)) {
        const float* raw = reinterpret_cast<const float*>(st);
#pragma unroll
        for (int k = 0; k < kLtK; ++k) w[k] = raw[k * kLtV + v];
      } else {
        s_conv_bad = 1;
        fail();
      }
      bar_sync_n(1, kLtConvWarps * kWarp);  // the whole tile is read
      if (s_conv_bad) break;
#pragma unroll
      for (int kc = 0; kc < kLtK / 8; ++kc) {
        uint4 hi, lo;
        lm_split8(w + 8 * kc, hi, lo);
        *reinterpret_cast<uint4*>(st + lm_core_off(v, kc)) = hi;
        *reinterpret_cast<uint4*>(st + kLtHalf + lm_core_off(v, kc)) = lo;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&conv[s]);
    }
  } else {
    // ------------------------------------------------------- epilogue --
    // warp w reads tensor-memory lanes 32 (w % 4) .. +31: columns
    // g * 128 + 32 (w % 4) + lane; its running (max, index) per row stays in
    // registers of lane m % 32 (rows m and m + 32 -> two slots).
    const int quad = warp & 3, e = warp - 2 - kLtConvWarps;
    float bv0 = -INFINITY, bv1 = -INFINITY;
    int bi0 = 0x7fffffff, bi1 = 0x7fffffff;
    for (int j = 0; j < ng; ++j) {
      const int a = j & 1;
      if (!mbar_wait(&acc_full[a], (j >> 1) & 1)) {
        fail();
        break;
      }
      tc_fence_after();
      const int col = ((int)blockIdx.x + j * (int)gridDim.x) * kLtV + quad * kWarp + lane;
      for (int m0 = 0; m0 < N; m0 += 16) {
        uint32_t r[16];
        tmem_ld16(tmem + ((uint32_t)(quad * kWarp) << 16) + (uint32_t)(a * kLtMaxN + m0), r);
        tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          const int m = m0 + q;
          if (m >= rows) break;  // warp-uniform
          float v = __uint_as_float(r[q]);
          if (p.logits) p.logits[(size_t)(row0 + m) * p.V + col] = v;
          int i = col;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, v, o);
            const int oi = __shfl_xor_sync(0xffffffffu, i, o);
            argmax_merge(v, i, ov, oi);
          }
          if (lane == (m & 31)) {
            if (m < 32)
              argmax_merge(bv0, bi0, v, i);
            else
              argmax_merge(bv1, bi1, v, i);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[a]);
    }
    s_bv[e][lane] = bv0;
    s_bi[e][lane] = bi0;
    s_bv[e][32 + lane] = bv1;
    s_bi[e][32 + lane] = bi1;
  }

  // ---------------------------------------------------- CTA results --
  __syncthreads();
  if (threadIdx.x < rows) {
    const int m = threadIdx.x;
    float v = s_bv[0][m];
    int i = s_bi[0][m];
    for (int w = 1; w < kLtEpiWarps; ++w) argmax_merge(v, i, s_bv[w][m], s_bi[w][m]);
    p.part_val[(size_t)(row0 + m) * gridDim.x + blockIdx.x] = v;
    p.part_idx[(size_t)(row0 + m) * gridDim.x + blockIdx.x] = i;
  }
  if (warp == 1) {
    // no MMA may still write the columns being freed (bounded, as every wait)
    if (!mbar_wait(&done, 0)) atomicOr(p.err, kErrWaitTimeout);
    tc_fence_after();
  }
  tc_fence_before();
  __syncthreads();  // partials written; the MMAs are finished
  if (warp == 1) tmem_dealloc(tmem, kLtCols);
  if (!p.argmax) return;
  if (threadIdx.x == 0) s_last = (ticket_acq_rel(p.counter) == (int)gridDim.x - 1);
  __syncthreads();
  if (!s_last) return;
  const int nw = kLtThreads / kWarp;
  for (int m = warp; m < rows; m += nw) {
    float v = -INFINITY;
    int i = 0x7fffffff;
    for (int c = lane; c < (int)gridDim.x; c += kWarp)
      argmax_merge(v, i, __ldcg(p.part_val + (size_t)(row0 + m) * gridDim.x + c),
                         __ldcg(p.part_idx + (size_t)(row0 + m) * gridDim.x + c));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, i, o);
      argmax_merge(v, i, ov, oi);
    }
    if (lane == 0) {
      p.argmax[row0 + m] = i;
      if (p.maxval) p.maxval[row0 + m] = v;
    }
  }
  if (threadIdx.x == 0) *p.counter = 0;
}

// =========================================================================
// Up to 8 rows: fp32 FMAs on CUDA cores (the reference's arithmetic), with
// the table streamed through shared memory.  One persistent CTA per SM holds
// the normalised rows once and walks vocabulary groups b, b + grid, ...;
// warp 8 streams each group's 32 x 128 W tiles through an 8-stage ring of
// 2-D tensor copies (128 KB in flight per SM; the register-staged kernel in
// ms_misc.cu keeps about 57 KB in flight and its 40 KB of rows per CTA cap
// how many CTAs an SM holds).  Warps 0-7: thread (column c = t % 128,
// k-half h = t / 128) sums rows 16 h .. 16 h + 15 of every tile in k order;
// the halves are added per group (half 0 + half 1), then logits and each
// row's running (max, first index).
// =========================================================================
constexpr int kLrStages = 8;
constexpr int kLrWarps = 8;                        // compute warps
constexpr int kLrThreads = (kLrWarps + 1) * kWarp;  // + the copy warp
constexpr int kLrMaxM = 8;
constexpr size_t kLrRing = (size_t)kLrStages * kLtA;  // 128 KB

template <int MR>
__global__ void __launch_bounds__(kLrThreads, 1) lm_ring_kernel(const LmHeadParams p,
                                                                const __grid_constant__ CUtensorMap wmap) {
  extern __shared__ __align__(1024) uint8_t dsm[];
  float* ring = reinterpret_cast<float*>(dsm);                 // [stages][32][128]
  float* xs = reinterpret_cast<float*>(dsm + kLrRing);         // [MR][D]
  float* red = xs + (size_t)MR * p.D;                          // [MR][128] half-1 sums
  __shared__ __align__(8) uint64_t full[kLrStages], empty[kLrStages];
  __shared__ float s_inv[MR];
  __shared__ float s_bv[kLrWarps / 2][MR];
  __shared__ int s_bi[kLrWarps / 2][MR];
  __shared__ int s_last;
  __shared__ volatile int s_bad;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_groups = p.V / kLtV, nk = p.D / kLtK;
  const int ng = n_groups > (int)blockIdx.x
                     ? (n_groups - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x
                     : 0;
  const int total = ng * nk;
  const int rows = min(MR, p.M);

  if (tid == 0) {
    s_bad = 0;
    for (int s = 0; s < kLrStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kLrWarps);
    }
    mbar_fence_init();
  }
  __syncthreads();
  pdl_trigger();

  if (warp == kLrWarps) {
    // ------------------------------------------------ tile copies --
    if (lane == 0) {
      auto issue = [&](int t) {
        const int s = t % kLrStages, j = t / nk, c = t % nk;
        mbar_expect_tx(&full[s], kLtA);
        tma_load_2d(ring + (size_t)s * (kLtA / 4), &wmap,
                    ((int)blockIdx.x + j * (int)gridDim.x) * kLtV, c * kLtK, &full[s]);
      };
      const int first = min(total, kLrStages);
      for (int t = 0; t < first; ++t) issue(t);  // W does not depend on earlier kernels
      int t = first;
      for (; t < total; ++t) {
        if (!mbar_wait(&empty[t % kLrStages], ((t / kLrStages) - 1) & 1)) {
          atomicOr(p.err, kErrWaitTimeout);
          s_bad = 1;
          break;
        }
        issue(t);
      }
      if (s_bad)  // let the copies already issued land before the CTA can exit
        for (int j = t - 1; j >= 0 && j >= t - kLrStages; --j)
          if (!mbar_wait(&full[j % kLrStages], (j / kLrStages) & 1)) break;
    }
    pdl_wait();
  } else {
    // --------------------------------------------- rows, then FMAs --
    pdl_wait();
    for (int r = warp; r < MR; r += kLrWarps) {
      float inv = 1.f;
      if (r < rows && p.stats) {
        float s = 0.f;
        for (int i = lane; i < p.nstat; i += kWarp) s += p.stats[(size_t)i * p.M + r];
        s = warp_sum(s);
        inv = 1.0f / sqrtf(s / (float)p.D + 1e-6f);
      }
      if (lane == 0) s_inv[r] = inv;
    }
    bar_sync_n(1, kLrWarps * kWarp);
    for (int idx = tid; idx < MR * p.D; idx += kLrWarps * kWarp) {
      const int r = idx / p.D, k = idx % p.D;
      float v = 0.f;
      if (r < rows) {
        v = p.x[(size_t)r * p.D + k] * s_inv[r];
        if (p.gamma) v = v * p.gamma[k];
      }
      xs[idx] = v;
    }
    bar_sync_n(1, kLrWarps * kWarp);

    const int c = tid & (kLtV - 1), h = tid >> 7;  // column of the group, k-half
    float bv[MR];
    int bi[MR];
#pragma unroll
    for (int r = 0; r < MR; ++r) {
      bv[r] = -INFINITY;
      bi[r] = 0x7fffffff;
    }
    // Every compute thread walks every group and takes every barrier; after
    // a timed-out wait it stops waiting (the error word is set) and sums
    // whatever the ring holds, so no warp is left at a barrier.
    bool failed = false;
    for (int j = 0; j < ng; ++j) {
      float acc[MR];
#pragma unroll
      for (int r = 0; r < MR; ++r) acc[r] = 0.f;
      for (int ck = 0; ck < nk; ++ck) {
        const int t = j * nk + ck, s = t % kLrStages;
        if (!failed && !mbar_wait(&full[s], (t / kLrStages) & 1)) {
          atomicOr(p.err, kErrWaitTimeout);
          failed = true;
        }
        const float* w = ring + (size_t)s * (kLtA / 4) + (16 * h) * kLtV + c;
        const float* xk = xs + ck * kLtK + 16 * h;
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          const float wv = w[u * kLtV];
#pragma unroll
          for (int r = 0; r < MR; ++r) acc[r] = fmaf(xk[r * p.D + u], wv, acc[r]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }
      // the two halves of each column: half 1 parks its sums, half 0 adds them
      if (h == 1)
#pragma unroll
        for (int r = 0; r < MR; ++r) red[r * kLtV + c] = acc[r];
      bar_sync_n(1, kLrWarps * kWarp);
      if (h == 0) {
        const int col = ((int)blockIdx.x + j * (int)gridDim.x) * kLtV + c;
#pragma unroll
        for (int r = 0; r < MR; ++r) {
          float v = acc[r] + red[r * kLtV + c];
          if (r < rows && p.logits) p.logits[(size_t)r * p.V + col] = v;
          int i = col;
          if (r >= rows) v = -INFINITY;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, v, o);
            const int oi = __shfl_xor_sync(0xffffffffu, i, o);
            argmax_merge(v, i, ov, oi);
          }
          argmax_merge(bv[r], bi[r], v, i);
        }
      }
      bar_sync_n(1, kLrWarps * kWarp);  // red is free for the next group
    }
    if (h == 0 && lane == 0)
#pragma unroll
      for (int r = 0; r < MR; ++r) {
        s_bv[warp][r] = bv[r];
        s_bi[warp][r] = bi[r];
      }
  }
  __syncthreads();
  if (tid < rows) {
    float v = s_bv[0][tid];
    int i = s_bi[0][tid];
    for (int w = 1; w < kLrWarps / 2; ++w) argmax_merge(v, i, s_bv[w][tid], s_bi[w][tid]);
    p.part_val[(size_t)tid * gridDim.x + blockIdx.x] = v;
    p.part_idx[(size_t)tid * gridDim.x + blockIdx.x] = i;
  }
  if (!p.argmax) return;
  __syncthreads();  // partials written
  if (tid == 0) s_last = (ticket_acq_rel(p.counter) == (int)gridDim.x - 1);
  __syncthreads();
  if (!s_last) return;
  for (int r = warp; r < rows; r += kLrThreads / kWarp) {
    float v = -INFINITY;
    int i = 0x7fffffff;
    for (int cc = lane; cc < (int)gridDim.x; cc += kWarp)
      argmax_merge(v, i, __ldcg(p.part_val + (size_t)r * gridDim.x + cc),
                   __ldcg(p.part_idx + (size_t)r * gridDim.x + cc));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, i, o);
      argmax_merge(v, i, ov, oi);
    }
    if (lane == 0) {
      p.argmax[r] = i;
      if (p.maxval) p.maxval[r] = v;
    }
  }
  if (tid == 0) *p.counter = 0;
}

static size_t lm_ring_smem(int mr, int D) {
  return kLrRing + (size_t)mr * D * 4 + (size_t)mr * kLtV * 4;
}

bool lm_ring_ok(const LmHeadParams& p) {
  return p.err && p.M >= 1 && p.M <= kLrMaxM && p.V % kLtV == 0 && p.D % kLtK == 0 &&
         lm_ring_smem(p.M <= 4 ? 4 : 8, p.D) <= 220 * 1024;
}

cudaError_t launch_lm_ring(const LmHeadParams& p, const void* wmap, int ctas, cudaStream_t s,
                           bool pdl) {
  const CUtensorMap map = *reinterpret_cast<const CUtensorMap*>(wmap);
  const int mr = p.M <= 4 ? 4 : 8;
  const size_t smem = lm_ring_smem(mr, p.D);
  auto kern = mr == 4 ? lm_ring_kernel<4> : lm_ring_kernel<8>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int n_groups = p.V / kLtV;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas < n_groups ? ctas : n_groups);
  cfg.blockDim = dim3(kLrThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, p, map);
}

bool lm_tc_ok(const LmHeadParams& p) {
  return p.planes && p.err && p.M > 8 && p.V % kLtV == 0 && p.D % kLtK == 0 &&
         (size_t)2 * kLtMaxN * p.D * 2 <= p.planes_bytes;
}

// Tensor map over the fp32 table W [D][V] (V contiguous) with 32 x 128 boxes.
bool lm_tc_make_map(void* map_out, const float* W, int D, int V) {
  using Encode = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                              const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                              const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                              CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  static Encode encode = nullptr;
  if (!encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn) {
      cudaGetLastError();
      return false;
    }
    encode = reinterpret_cast<Encode>(fn);
  }
  if (((uintptr_t)W & 15) || V % kLtV || D % kLtK) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)V, (cuuint64_t)D};
  const cuuint64_t strides[1] = {(cuuint64_t)V * sizeof(float)};
  const cuuint32_t box[2] = {kLtV, kLtK};
  const cuuint32_t estr[2] = {1, 1};
  return encode(reinterpret_cast<CUtensorMap*>(map_out), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                const_cast<float*>(W), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t prepare_lm_tc() {
  return cudaFuncSetAttribute(lm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)kLtSmem);
}

// Rows in launches of up to 64: the planes kernel, then the persistent GEMM
// over at most `ctas` CTAs (each pass reads the table once).
cudaError_t launch_lm_tc(const LmHeadParams& p, const void* wmap, int ctas, cudaStream_t s,
                         bool pdl) {
  const CUtensorMap map = *reinterpret_cast<const CUtensorMap*>(wmap);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  const int n_groups = p.V / kLtV;
  const int grid = ctas < n_groups ? ctas : n_groups;
  for (int row0 = 0; row0 < p.M; row0 += kLtMaxN) {
    const int n = p.M - row0 < kLtMaxN ? p.M - row0 : kLtMaxN;
    const int N = (n + 15) / 16 * 16;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(N);
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = (pdl || row0 > 0) ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, lm_rows_kernel, p, row0, N);
    if (e != cudaSuccess) return e;
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kLtThreads);
    cfg.dynamicSmemBytes = kLtSmem;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, lm_tc_kernel, p, row0, N, map);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace ms
