// ms_gemm_sk.cu -- Q4 projection for decode batches of 9..64 rows on the
// 5th-generation tensor cores, weights on the MMA's 128-row side.
// Reference: matmul_q4_bpack_raw (src/linalg/kernels.mojo:201-267) with the
// steps fused around its call sites (src/main.mojo:538-613,
// src/inference/gemma4_e4b.mojo:459-540) in the epilogue.
//
// Why a second tensor-core kernel: with batch rows on the MMA's M side (the
// prefill GEMM, ms_gemm_tc.cu) a batch of 16 or 64 rows fills a 128-row tile
// to 1/8 or 1/2, and every 64-k chunk moves 24 KB of activation limbs for
// 4 KB of weights.  Here the tile is transposed: the MMA's A operand is 128
// output columns of the weights (M = 128), B is the batch's activation limbs
// (N = rows rounded up to 16), so a chunk moves 4 KB of weights and
// 3 x N x 64 bytes of limbs, and no MMA work is spent on padding rows beyond
// the next multiple of 16.
//
// Arithmetic: exactly that of the prefill GEMM -- rows quantised once per
// projection by quant_rows_kernel into three signed 8-bit limbs (q =
// d0 + 2^8 d1 + 2^16 d2, |q| <= 2^22 of the row maximum), weights unpacked to
// s8 (u - 8), one s8 x s8 -> s32 MMA chain per limb, limbs combined in int64
// and scaled by (a / 2^22) * (RMSNorm factor) in the epilogue, the weight
// scale applied there once.
//
// CTA: one tile group (128 output columns) over one k-slice.  Warp 0 streams
// stages with cp.async.bulk (4 KB packed nibbles + the N rows of the three
// limb planes per 64-k chunk; the weight copies of the first stages go out
// before griddepcontrol.wait, since no earlier kernel writes them); warp 1
// allocates 256 tensor-memory columns and one thread issues the MMAs;
// warps 2-9 unpack nibbles into the A operand and then run the epilogue
// (tensor-memory lane = output column, columns = batch rows).  The k-slices
// of a group run as one thread-block cluster (<= 8 CTAs): each leaves its
// partial tile in shared memory and CTA r finishes the rows m = r (mod
// slices), summing the slices in k order through distributed shared memory
// (the same order on every run).  Tensor parallel (O / down): the finished
// rows go to this rank's peer-visible buffer, CTA 0 of the cluster publishes
// the tile with a system-scope release, and each CTA sums every rank's rows
// in rank order after the peers' counters reached the same use (the protocol
// of the prefill GEMM's epilogue).  Every wait is bounded (error word).
#include "ms_common.cuh"
#include "ms_epilogue.cuh"
#include "ms_kernels.h"
#include "ms_tc.cuh"

namespace ms {

constexpr int kSkStages = 4;
constexpr int kSkLimbs = 3;
constexpr int kSkMaxN = 64;                                // batch rows per launch
constexpr int kSkAConv = 128 * kChunkK;                    // 8 KB: s8 weights, 128 x 64
constexpr int kSkAPacked = kGroupTiles * kWarp * 16;       // 4 KB: packed nibbles
constexpr int kSkPlane = 128 * kChunkK;                    // a quantiser limb plane (128 rows)
constexpr int kSkBMax = kSkLimbs * kSkMaxN * kChunkK;      // 12 KB: limbs of 64 rows
constexpr int kSkStageBytes = kSkAConv + kSkAPacked + kSkBMax;  // 24 KB
constexpr int kSkConvWarps = 8;
constexpr int kSkThreads = (2 + kSkConvWarps) * kWarp;     // 320
constexpr uint32_t kSkCols = 256;                          // >= 3 x 64 accumulator columns
constexpr int kSkRowS = 128 + 4;                           // staged partial row (floats)
constexpr size_t kSkSmem = (size_t)kSkStages * kSkStageBytes;
constexpr int kSkMaxCluster = 8;
constexpr uint32_t kSkLbo = 128, kSkSbo = 512;

static_assert(kSkStageBytes % 1024 == 0, "stage alignment");
static_assert((size_t)(kSkMaxN + kSkMaxN / 2) * kSkRowS * 4 <= kSkSmem,
              "staged partial + finished rows fit the ring");

int sk_rows_max() { return kSkMaxN; }

__global__ void __launch_bounds__(kSkThreads, 2) gemm_sk_kernel(const GemvParams p, int N) {
  extern __shared__ __align__(1024) uint8_t dsm[];
  __shared__ __align__(8) uint64_t full[kSkStages], conv[kSkStages], empty[kSkStages], done;
  __shared__ uint32_t s_tmem;
  __shared__ volatile int s_bad;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int group = blockIdx.x;
  const int nchunks = p.K / kChunkK;
  const int kidx = blockIdx.z, seg = p.kseg / kChunkK;
  const int c_begin = kidx * seg;
  const int n_loc = min(nchunks, c_begin + seg) - c_begin;
  const bool cl = p.ksplit > 1;
  const uint32_t b_bytes = (uint32_t)N * kChunkK;  // one limb's N rows of a chunk

  if (threadIdx.x == 0) {
    s_bad = 0;
    for (int s = 0; s < kSkStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], kSkConvWarps);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&done, 1);
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(&s_tmem, kSkCols);
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
      const uint4* a_src = p.w + ((size_t)group * nchunks + c_begin) * kGroupTiles * kWarp;
      const uint8_t* b_src = p.lq + (size_t)c_begin * kSkLimbs * kSkPlane;
      const int first = min(n_loc, kSkStages);
      // weights first: they do not depend on the previous kernel
      for (int c = 0; c < first; ++c) {
        uint8_t* st = dsm + (size_t)c * kSkStageBytes;
        mbar_expect_tx(&full[c], kSkAPacked + kSkLimbs * b_bytes);
        bulk_g2s(st + kSkAConv, a_src + (size_t)c * kGroupTiles * kWarp, kSkAPacked, &full[c]);
      }
      pdl_wait();  // the limbs are the quantiser's output
      for (int c = 0; c < first; ++c) {
        uint8_t* st = dsm + (size_t)c * kSkStageBytes + kSkAConv + kSkAPacked;
        for (int l = 0; l < kSkLimbs; ++l)
          bulk_g2s(st + l * b_bytes, b_src + ((size_t)c * kSkLimbs + l) * kSkPlane, b_bytes,
                   &full[c]);
      }
      int c = first;
      for (; c < n_loc; ++c) {
        const int s = c % kSkStages;
        if (!mbar_wait(&empty[s], ((c / kSkStages) - 1) & 1)) {
          atomicOr(p.err, kErrWaitTimeout);
          s_bad = 1;
          break;
        }
        uint8_t* st = dsm + (size_t)s * kSkStageBytes;
        mbar_expect_tx(&full[s], kSkAPacked + kSkLimbs * b_bytes);
        bulk_g2s(st + kSkAConv, a_src + (size_t)c * kGroupTiles * kWarp, kSkAPacked, &full[s]);
        for (int l = 0; l < kSkLimbs; ++l)
          bulk_g2s(st + kSkAConv + kSkAPacked + l * b_bytes,
                   b_src + ((size_t)c * kSkLimbs + l) * kSkPlane, b_bytes, &full[s]);
      }
      if (s_bad) {
        // let the copies already issued land before the CTA can exit
        for (int j = c - 1; j >= 0 && j >= c - kSkStages; --j)
          if (!mbar_wait(&full[j % kSkStages], (j / kSkStages) & 1)) break;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------ MMA issuer --
    if (lane == 0) {
      const uint32_t idesc = idesc_i8(128, N);
      for (int c = 0; c < n_loc; ++c) {
        const int s = c % kSkStages;
        const uint32_t ph = (c / kSkStages) & 1;
        if (!mbar_wait(&full[s], ph) || !mbar_wait(&conv[s], ph)) {
          atomicOr(p.err, kErrWaitTimeout);
          s_bad = 1;
          break;
        }
        tc_fence_after();
        const uint32_t a0 = smem_u32(dsm + (size_t)s * kSkStageBytes);
        const uint32_t b0 = a0 + kSkAConv + kSkAPacked;
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
          const uint64_t da = umma_desc(a0 + kk * 256, kSkLbo, kSkSbo);
#pragma unroll
          for (int l = 0; l < kSkLimbs; ++l)
            umma_i8(tmem + l * N, da, umma_desc(b0 + l * b_bytes + kk * 256, kSkLbo, kSkSbo),
                    idesc, (c | kk) != 0);
        }
        umma_commit(&empty[s]);
      }
      umma_commit(&done);  // arrives when every MMA issued above has finished
    }
  } else {
    // ---------------------------------------------- nibble unpacking --
    // thread ci: tile ci / 32 of the group, fragment lane (g, t) = ci % 32;
    // low nibbles are tile row g (A row 16 tile + g), high nibbles row g + 8.
    const int ci = threadIdx.x - 2 * kWarp;
    const int tl = ci >> 5, g = (ci & 31) >> 2, t = ci & 3;
    for (int c = 0; c < n_loc; ++c) {
      const int s = c % kSkStages;
      if (!mbar_wait(&full[s], (c / kSkStages) & 1)) {
        atomicOr(p.err, kErrWaitTimeout);
        s_bad = 1;
        break;
      }
      uint8_t* st = dsm + (size_t)s * kSkStageBytes;
      const uint4 wv = lds_u4(reinterpret_cast<const uint4*>(st + kSkAConv) + ci);
      uint8_t* ac = st + g * 16 + 4 * t;
      const uint32_t wd[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        // (u + 0x78) ^ 0x80 per byte = two's complement of u - 8 (no carries)
        const uint32_t lo = ((wd[w] & 0x0F0F0F0Fu) + 0x78787878u) ^ 0x80808080u;
        const uint32_t hi = (((wd[w] >> 4) & 0x0F0F0F0Fu) + 0x78787878u) ^ 0x80808080u;
        sts_u32(ac + ((2 * tl) * 4 + w) * 128, lo);
        sts_u32(ac + ((2 * tl + 1) * 4 + w) * 128, hi);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&conv[s]);
    }
  }

  // ------------------------------------------------------------ epilogue --
  // 1. warps 2-9 copy the accumulators to a staged partial tile S[m][c]
  //    (two warps per tensor-memory lane quarter: warp w reads lanes
  //    32 (w % 4) .. +31 = the group's tile rows c; the two warps of a
  //    quarter take alternate 16-row blocks); c = 16 tile + (g or g + 8) is
  //    the prefill GEMM's staged layout, so the row epilogue below is its;
  // 2. cluster: this CTA's rows m = kidx + ks i are summed over the slices
  //    in k order with 128-bit distributed-shared-memory loads into F[i][c];
  // 3. tensor parallel: the rows' rank sum (peer-visible buffers);
  // 4. rows finished with lanes along the columns (128-bit loads / stores).
  __shared__ float2 s_rowf[kSkMaxN];
  __shared__ int s_use, s_tp_ok;
  const bool epi_warp = warp >= 2;
  const int t8 = threadIdx.x - 2 * kWarp;              // 0 .. 255 on warps 2-9
  const int quad = warp & 3, half = (warp - 2) >> 2;
  const int arow = quad * kWarp + lane;                // tile row of the group (TMEM lane)
  float* S = reinterpret_cast<float*>(dsm);            // [kSkMaxN][kSkRowS]
  float* F = S + kSkMaxN * kSkRowS;                    // [kSkMaxN / 2][kSkRowS]
  bool ok = true;
  if (epi_warp) {
    pdl_wait();
    for (int m = t8; m < N; m += kSkConvWarps * kWarp)
      s_rowf[m] = m < p.M ? p.rowf[m] : make_float2(0.f, 0.f);
    ok = mbar_wait(&done, 0);
    tc_fence_after();
    if (!ok && lane == 0) {
      atomicOr(p.err, kErrWaitTimeout);
      s_bad = 1;
    }
    bar_sync_n(1, kSkConvWarps * kWarp);  // s_rowf complete
    if (ok) {
      for (int m0 = 16 * half; m0 < N; m0 += 32) {
        uint32_t a0[16], a1[16], a2[16];
        const uint32_t ta = tmem + ((uint32_t)(quad * kWarp) << 16) + m0;
        tmem_ld16(ta, a0);
        tmem_ld16(ta + N, a1);
        tmem_ld16(ta + 2 * N, a2);
        tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          const long long iv = (long long)(int)a0[q] + 256LL * (long long)(int)a1[q] +
                               65536LL * (long long)(int)a2[q];
          S[(m0 + q) * kSkRowS + arow] = (float)iv * s_rowf[m0 + q].x;
        }
      }
    }
  }
  __syncthreads();  // S and every warp's flag are in place
  // the rows this CTA finishes: m = m_first + m_step i, i < n_rows, values in Fr
  const int m_first = cl ? kidx : 0, m_step = cl ? p.ksplit : 1;
  const int n_rows = m_first < p.M ? (p.M - m_first + m_step - 1) / m_step : 0;
  const float* Fr = cl ? F : S;
  int any = s_bad;
  if (cl) {
    cluster_arrive();
    cluster_wait();  // every CTA's partial tile and flag are in its shared memory
    const uint32_t bad0 = smem_u32(const_cast<int*>(&s_bad));
    any = 0;
    for (int r = 0; r < p.ksplit; ++r) any |= ld_dsmem_s32(dsmem_addr(bad0, (uint32_t)r));
    if (epi_warp && !any) {
      const uint32_t s0 = smem_u32(S);
      for (int it = t8; it < n_rows * (128 / 4); it += kSkConvWarps * kWarp) {
        const int i = it >> 5, c4 = it & 31;
        const uint32_t off = 4u * ((m_first + m_step * i) * kSkRowS + 4 * c4);
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
        float4 v[kSkMaxCluster];
#pragma unroll
        for (int r = 0; r < kSkMaxCluster; ++r)
          if (r < p.ksplit) v[r] = ld_dsmem4(dsmem_addr(s0 + off, (uint32_t)r));
#pragma unroll
        for (int r = 0; r < kSkMaxCluster; ++r)
          if (r < p.ksplit) {
            a.x += v[r].x; a.y += v[r].y; a.z += v[r].z; a.w += v[r].w;
          }
        *reinterpret_cast<float4*>(F + i * kSkRowS + 4 * c4) = a;
      }
    }
    cluster_arrive();  // done reading the other CTAs' partials
    cluster_wait();
  }
  if (p.peer_tiles) {
    // ---- tensor parallel (cluster mode, checked at launch): this rank's
    //      rows to its peer-visible buffer (row m at m * 128); CTA 0
    //      publishes one use of the tile after every CTA's rows are written
    //      (system-scope release); each CTA waits for every peer's counter to
    //      reach it and sums the ranks' rows in rank order (the same bits on
    //      every rank) -- the protocol of the prefill GEMM's epilogue
    float* mine = p.peer_tiles[p.tp_rank] + (size_t)group * (128 * 128);
    if (epi_warp && !any)
      for (int it = t8; it < n_rows * 32; it += kSkConvWarps * kWarp) {
        const int i = it >> 5, c4 = it & 31;
        __stcg(reinterpret_cast<float4*>(mine + (size_t)(m_first + m_step * i) * 128) + c4,
               *reinterpret_cast<const float4*>(F + i * kSkRowS + 4 * c4));
      }
    __syncthreads();
    cluster_arrive();
    cluster_wait();  // every CTA's rows are written
    if (threadIdx.x == 2 * kWarp) {
      s_use = 0;
      if (kidx == 0 && !any) {
        fence_acq_rel_sys();
        s_use = atomicAdd_system(p.peer_flags[p.tp_rank] + group, 1) + 1;
      }
    }
    cluster_arrive();
    cluster_wait();  // CTA 0's use is in its shared memory
    if (threadIdx.x == 2 * kWarp) {
      const int use = ld_dsmem_s32(dsmem_addr(smem_u32(&s_use), 0u));
      int ok_all = use > 0;
      for (int r = 0; r < p.tp_world && ok_all; ++r)
        if (r != p.tp_rank) ok_all = wait_counter_sys(p.peer_flags[r] + group, use);
      if (use > 0 && !ok_all) atomicOr(p.err, kErrWaitTimeout);
      fence_acq_rel_sys();
      s_tp_ok = ok_all;
    }
    __syncthreads();
    if (!s_tp_ok) any = 1;
    if (epi_warp && !any) {
      for (int it = t8; it < n_rows * 32; it += kSkConvWarps * kWarp) {
        const int i = it >> 5, c4 = it & 31;
        const size_t off = (size_t)group * (128 * 128) + (size_t)(m_first + m_step * i) * 128;
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int rk = 0; rk < p.tp_world; ++rk) {
          const float4 v = ld_sys_f4(reinterpret_cast<const float4*>(p.peer_tiles[rk] + off) + c4);
          a.x += v.x; a.y += v.y; a.z += v.z; a.w += v.w;
        }
        *reinterpret_cast<float4*>(F + i * kSkRowS + 4 * c4) = a;
      }
    }
    cluster_arrive();  // CTA 0's shared memory may be released
    cluster_wait();
  }
  if (epi_warp && !any) {
    bar_sync_n(1, kSkConvWarps * kWarp);  // F complete
    const int w8 = warp - 2;
    const int jt = lane >> 2;             // tile of the group this lane covers
    const int tile = group * kGroupTiles + jt;
    const bool tile_ok = tile < p.n_tiles;
    for (int i = w8; i < n_rows; i += kSkConvWarps) {
      const int m = m_first + m_step * i;
      const float* Sr = Fr + (cl ? i : m) * kSkRowS;
      if (p.epi == kEpiStore || p.epi == kEpiAccum || p.epi == kEpiResid) {
        const int c = group * 128 + 4 * lane;
        const float4 v = *reinterpret_cast<const float4*>(Sr + 4 * lane);
        float4 o;
        float sq = 0.f;
        if (p.epi == kEpiResid) {
          const float fres = s_rowf[m].y;
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
          *reinterpret_cast<float2*>(p.out + (size_t)m * p.ldo + group * 64 + 2 * lane) =
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

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    // no MMA may still write the columns being freed (bounded, as every wait)
    mbar_wait(&done, 0);
    tc_fence_after();
    tmem_dealloc(tmem, kSkCols);
  }
}

// Rows quantised by quant_rows_kernel (only the first roundup(M, 16) rows of
// the limb planes are read), then the GEMM; both with PDL.
cudaError_t launch_gemm_sk(const GemvParams& p, cudaStream_t s, bool pdl) {
  const int N = (p.M + 15) / 16 * 16;
  // the rank sum runs in the cluster epilogue: tensor parallel needs k-slices
  if (p.peer_tiles && (p.ksplit < 2 || !p.peer_flags || p.tp_world < 2))
    return cudaErrorInvalidConfiguration;
  if (p.M < 1 || N > kSkMaxN || p.ksplit < 1 || p.ksplit > kSkMaxCluster || p.kseg % kChunkK ||
      p.kseg <= 0 || (long long)p.kseg * (p.ksplit - 1) >= p.K)
    return cudaErrorInvalidConfiguration;
  if (p.K % kChunkK || !p.lq || !p.rowf || !p.x || (p.ldx & 3) || ((uintptr_t)p.x & 15) ||
      ((uintptr_t)p.lq & 15) || ((uintptr_t)p.rowf & 7))
    return cudaErrorInvalidConfiguration;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaError_t e = launch_quant_rows(p, N, s, pdl);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(padded_tiles(p.n_tiles) / kGroupTiles, 1, p.ksplit);
  cfg.blockDim = dim3(kSkThreads);
  cfg.dynamicSmemBytes = kSkSmem;
  cfg.stream = s;
  int na = 1;  // the quantiser just before it is always a PDL-aware kernel
  if (p.ksplit > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = (unsigned)p.ksplit;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, gemm_sk_kernel, p, N);
}

cudaError_t prepare_gemm_sk() {
  return cudaFuncSetAttribute(gemm_sk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)kSkSmem);
}

}  // namespace ms
