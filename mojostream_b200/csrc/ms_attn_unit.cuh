// ms_attn_unit.cuh -- one unit of flash-decode GQA attention over the paged
// KV cache: (row m, KV head hk, position split).  Shared by the
// one-launch-per-layer kernel (ms_attn.cu) and the persistent decode-step
// kernel (ms_decode_mk.cu).
//
// Reference semantics: gqa_attention_decode (src/main.mojo:445-519),
// compute_sliding_attention / compute_full_attention
// (src/inference/gemma4_e4b.mojo:259-411): row m (sequence seq[m] at absolute
// position pos[m]) attends positions lo..pos, lo = max(0, pos + 1 - window)
// for sliding layers and 0 otherwise; score = (q . k) / sqrt(hd); softmax with
// the maximum subtracted; out = sum p * v.  Query head h reads KV head
// h / (n_heads / n_kv).
//
// A unit serves all G = n_heads / n_kv query heads of its KV head, so each
// K/V row is read once for G heads.  A row's positions are cut into at most
// n_splits contiguous ranges; a unit brings its range into shared memory in
// chunks with cp.async.bulk (one copy per K or V row of a KV head, two chunk
// buffers so chunk c + 1 streams while chunk c computes), then per chunk:
//   1. scores: warps take positions, lanes slices of the head dimension, one
//      warp reduction per (position, head);
//   2. softmax bookkeeping per head (running maximum, sum, rescale factor);
//   3. values: each thread owns float4 slices of the G x hd outputs and adds
//      p * V over the chunk's positions (conflict-free 128-bit shared loads).
// Splits are merged by the last unit of the (row, kv head) in split order
// (log-sum-exp weights; loads batched so they overlap): timing independent.
// Data written earlier in the same launch (q, K/V of the current position,
// partials) is read through L2 (ld.global.cg / bulk copies).
#pragma once

#include "ms_common.cuh"
#include "ms_kernels.h"

namespace ms {

constexpr int kAttnMaxSplits = 64;
constexpr int kAttnMergeBatch = 8;  // partial rows loaded per round of the merge
constexpr int kAttnMaxG = 8;
constexpr int kAttnScoreFloats = 1024;  // G x positions-per-chunk, all shapes
constexpr int kAttnMaxQ = 2048;         // G x head_dim, all shapes
constexpr int kAttnOffsets = 256;       // KV row offsets precomputed per unit

template <int HD, int BUF>
struct AttnShape {
  static constexpr int PL = HD / kWarp;                  // dims per lane (scores)
  static constexpr int VEC = PL >= 4 ? 4 : PL;           // floats per lane load
  static constexpr int NV = PL / VEC;                    // loads per lane per row
  static constexpr int PC = BUF / (2 * HD);              // positions per chunk
  static constexpr int ST = HD + 4;                      // partial row stride (16 B)
};

struct __align__(16) AttnShared {  // q is read and written as float4 / float2
  float q[kAttnMaxQ];         // [G][hd] query vectors of the unit
  float p[kAttnScoreFloats];  // [G][PC] scores, then weights
  float M[kAttnMaxG], L[kAttnMaxG], corr[kAttnMaxG];
  float w[kAttnMaxG][kAttnMaxSplits];
  unsigned int off[kAttnOffsets];  // KV row offsets (floats) of the unit's first positions
  int last, bad;
};

template <int VEC>
__device__ __forceinline__ void lds_vec_f(float* dst, const float* src) {
  if constexpr (VEC == 4) {
    const float4 v = *reinterpret_cast<const float4*>(src);
    dst[0] = v.x; dst[1] = v.y; dst[2] = v.z; dst[3] = v.w;
  } else {
    const float2 v = *reinterpret_cast<const float2*>(src);
    dst[0] = v.x; dst[1] = v.y;
  }
}
template <int VEC>
__device__ __forceinline__ void ldcg_vec(float* dst, const float* src) {
  if constexpr (VEC == 4) {
    const float4 v = __ldcg(reinterpret_cast<const float4*>(src));
    dst[0] = v.x; dst[1] = v.y; dst[2] = v.z; dst[3] = v.w;
  } else {
    const float2 v = __ldcg(reinterpret_cast<const float2*>(src));
    dst[0] = v.x; dst[1] = v.y;
  }
}

enum AttnResult : int {
  kAttnIdle = 0,      // no positions in this split
  kAttnPartial = 1,   // partial written, another unit merges
  kAttnFinished = 2,  // this unit wrote the (row, kv head) output
  kAttnFailed = -1,   // a wait gave up: error word set, outputs skipped
};

// NT consumer threads (threads 0 .. NT-1, named barrier `bar`); buf: two chunk
// buffers of BUF floats; full[2]: their mbarriers, used with the running
// chunk counter `ac` (buffer ac & 1, phase (ac >> 1) & 1).  CTA-uniform result.
template <int HD, int G, int NT, int BUF>
__device__ int attn_unit(const AttnParams& p, int split, int hk, int m, float* buf,
                         uint64_t* full, uint32_t& ac, AttnShared& sh, int bar) {
  using S = AttnShape<HD, BUF>;
  constexpr int PC = S::PC, ST = S::ST;
  constexpr int NW = NT / kWarp;
  constexpr int NOUT = G * HD / 4;                       // float4 outputs per unit
  constexpr int OPT = (NOUT + NT - 1) / NT;              // per thread
  static_assert(G * PC <= kAttnScoreFloats && G <= kAttnMaxG && G * HD <= kAttnMaxQ,
                "attention shape");
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  const int pos = p.pos[m], seq = p.seq[m];
  const int lo = p.window > 0 ? max(0, pos + 1 - p.window) : 0;
  const int n = pos + 1 - lo;
  // positions per split: every row fits n_splits, at least p.chunk each
  const int per = max((n + p.n_splits - 1) / p.n_splits, p.chunk);
  const int ns = (n + per - 1) / per;
  if (split >= ns) return kAttnIdle;
  const int t_begin = lo + split * per;
  const int t_end = min(pos + 1, t_begin + per);
  const int n_chunks = (t_end - t_begin + PC - 1) / PC;
  const size_t head_off = (size_t)hk * HD;

  bar_sync_n(bar, NT);  // the previous unit's readers of sh / buf are done
  if (tid < G) {
    sh.M[tid] = -INFINITY;
    sh.L[tid] = 0.f;
  }
  if (tid == 0) sh.bad = 0;
  // KV row offsets of the unit's positions, one block-table round trip for
  // all chunks (positions past kAttnOffsets are looked up when issued)
  const bool off_fit = p.kv.off32 != 0;
  for (int j = tid; off_fit && j < t_end - t_begin && j < kAttnOffsets; j += NT)
    sh.off[j] = (unsigned int)kv_row_offset(p.kv.block_table, p.kv.bt_stride, p.kv.page, p.kv.cap,
                                            p.kv.circular, seq, t_begin + j, p.kv.kv_dim);

  // warp 0 streams chunk c into buffer (ac + c) % 2: one bulk copy per K / V row
  auto issue = [&](int c) {
    const uint32_t k = ac + (uint32_t)c;
    const int c0 = t_begin + c * PC;
    const int np = min(PC, t_end - c0);
    float* b = buf + (size_t)(k & 1) * PC * 2 * HD;
    if (lane == 0) {
      // K / V of the current position may have been written by generic
      // stores of this launch, and the buffer by generic shared stores of a
      // previous unit: order both before the async-proxy copies
      asm volatile("fence.proxy.async;" ::: "memory");
      mbar_expect_tx(&full[k & 1], (uint32_t)(np * 2 * HD * sizeof(float)));
    }
    __syncwarp();
    for (int j = lane; j < np; j += kWarp) {
      const int jj = c0 + j - t_begin;
      const size_t off = (off_fit && jj < kAttnOffsets
                              ? (size_t)sh.off[jj]
                              : kv_row_offset(p.kv.block_table, p.kv.bt_stride, p.kv.page,
                                              p.kv.cap, p.kv.circular, seq, c0 + j,
                                              p.kv.kv_dim)) +
                         head_off;
      bulk_g2s(b + (size_t)j * 2 * HD, p.kv.k + off, HD * sizeof(float), &full[k & 1]);
      bulk_g2s(b + (size_t)j * 2 * HD + HD, p.kv.v + off, HD * sizeof(float), &full[k & 1]);
    }
  };
  bar_sync_n(bar, NT);  // buffers free (previous unit) and sh initialised
  if (warp == 0) {
    issue(0);
    if (n_chunks > 1) issue(1);
  }

  // the unit's G query vectors into shared memory (visible after the first
  // chunk's barrier); the outputs this thread owns
  for (int i = tid; i < G * HD / 4; i += NT) {
    const int h = i / (HD / 4), d4 = i % (HD / 4);
    reinterpret_cast<float4*>(sh.q)[i] = __ldcg(reinterpret_cast<const float4*>(
        p.q + (size_t)m * p.ldq + (size_t)(hk * G + h) * HD + 4 * d4));
  }
  float4 acc[OPT];
#pragma unroll
  for (int o = 0; o < OPT; ++o) acc[o] = make_float4(0.f, 0.f, 0.f, 0.f);

  int c = 0;
  for (; c < n_chunks; ++c) {
    const uint32_t k = ac + (uint32_t)c;
    const int np = min(PC, t_end - (t_begin + c * PC));
    const float* b = buf + (size_t)(k & 1) * PC * 2 * HD;
    if (!mbar_wait(&full[k & 1], (k >> 1) & 1)) {
      if (lane == 0) {
        atomicOr(p.err, kErrWaitTimeout);
        sh.bad = 1;
      }
    }
    bar_sync_n(bar, NT);
    if (sh.bad) break;  // uniform after the barrier
    // 1. scores
    for (int j = warp; j < np; j += NW) {
      float kk[S::PL];
#pragma unroll
      for (int v = 0; v < S::NV; ++v)
        lds_vec_f<S::VEC>(&kk[v * S::VEC], b + (size_t)j * 2 * HD + v * kWarp * S::VEC + lane * S::VEC);
#pragma unroll
      for (int h = 0; h < G; ++h) {
        float qq[S::PL];
#pragma unroll
        for (int v = 0; v < S::NV; ++v)
          lds_vec_f<S::VEC>(&qq[v * S::VEC], sh.q + h * HD + v * kWarp * S::VEC + lane * S::VEC);
        float d = 0.f;
#pragma unroll
        for (int e = 0; e < S::PL; ++e) d = fmaf(qq[e], kk[e], d);
        d = warp_sum(d);
        if (lane == 0) sh.p[h * PC + j] = d * p.scale;
      }
    }
    bar_sync_n(bar, NT);
    // 2. running maximum / sum per head; p becomes the weights
    for (int h = warp; h < G; h += NW) {
      float cm = -INFINITY;
      for (int j = lane; j < np; j += kWarp) cm = fmaxf(cm, sh.p[h * PC + j]);
      cm = warp_max(cm);
      const float m_old = sh.M[h];
      const float m_new = fmaxf(m_old, cm);
      float sum = 0.f;
      for (int j = lane; j < np; j += kWarp) {
        const float e = expf(sh.p[h * PC + j] - m_new);
        sh.p[h * PC + j] = e;
        sum += e;
      }
      sum = warp_sum(sum);
      if (lane == 0) {
        const float corr = expf(m_old - m_new);  // 0 on the first chunk
        sh.corr[h] = corr;
        sh.L[h] = sh.L[h] * corr + sum;
        sh.M[h] = m_new;
      }
    }
    bar_sync_n(bar, NT);
    // 3. values
#pragma unroll
    for (int o = 0; o < OPT; ++o) {
      const int idx = tid + o * NT;
      if (idx < NOUT) {
        const int h = idx / (HD / 4), d4 = idx % (HD / 4);
        const float cr = sh.corr[h];
        float4 a = acc[o];
        a.x *= cr; a.y *= cr; a.z *= cr; a.w *= cr;
        const float* vcol = b + HD + d4 * 4;
#pragma unroll 4
        for (int j = 0; j < np; ++j) {
          const float w = sh.p[h * PC + j];
          const float4 v = *reinterpret_cast<const float4*>(vcol + (size_t)j * 2 * HD);
          a.x = fmaf(w, v.x, a.x); a.y = fmaf(w, v.y, a.y);
          a.z = fmaf(w, v.z, a.z); a.w = fmaf(w, v.w, a.w);
        }
        acc[o] = a;
      }
    }
    bar_sync_n(bar, NT);  // buffer k % 2 and p are free again
    if (warp == 0 && c + 2 < n_chunks) issue(c + 2);
  }
  ac += (uint32_t)n_chunks;
  if (sh.bad) {
    // let this unit's issued copies land (bounded) before the buffers are reused
    if (tid == 0)
      for (int cc = c; cc < n_chunks && cc < c + 2; ++cc) {
        const uint32_t k = ac - (uint32_t)n_chunks + (uint32_t)cc;
        mbar_wait(&full[k & 1], (k >> 1) & 1);
      }
    return kAttnFailed;
  }

  if (ns == 1) {
#pragma unroll
    for (int o = 0; o < OPT; ++o) {
      const int idx = tid + o * NT;
      if (idx < NOUT) {
        const int h = idx / (HD / 4), d4 = idx % (HD / 4);
        const float inv = 1.0f / sh.L[h];
        float4 a = acc[o];
        a.x *= inv; a.y *= inv; a.z *= inv; a.w *= inv;
        *reinterpret_cast<float4*>(p.out + (size_t)m * p.ldo + (hk * G + h) * HD + d4 * 4) = a;
      }
    }
    return kAttnFinished;
  }

  // ---- partial of this split: unnormalised sums, running max and sum ------
  float* part_base = p.part + (((size_t)m * p.n_kv + hk) * p.n_splits + split) * G * ST;
#pragma unroll
  for (int o = 0; o < OPT; ++o) {
    const int idx = tid + o * NT;
    if (idx < NOUT) {
      const int h = idx / (HD / 4), d4 = idx % (HD / 4);
      __stcg(reinterpret_cast<float4*>(part_base + (size_t)h * ST + d4 * 4), acc[o]);
    }
  }
  if (tid < G) {
    __stcg(part_base + (size_t)tid * ST + HD, sh.M[tid]);
    __stcg(part_base + (size_t)tid * ST + HD + 1, sh.L[tid]);
  }

  // ---- merge the splits: the last unit of (row, kv head) does it in order ---
  bar_sync_n(bar, NT);  // partials written
  int* ctr = p.counters + (size_t)m * p.n_kv + hk;
  if (tid == 0) sh.last = (ticket_acq_rel(ctr) == ns - 1);
  bar_sync_n(bar, NT);
  if (!sh.last) return kAttnPartial;
  const float* pr0 = p.part + ((size_t)m * p.n_kv + hk) * p.n_splits * G * ST;
  for (int h = warp; h < G; h += NW) {
    // each lane's splits (ns <= 64): maxima and sums in one round of loads
    float Ms[kAttnMaxSplits / kWarp], Ls[kAttnMaxSplits / kWarp];
    float Mx = -INFINITY;
#pragma unroll
    for (int q = 0; q < kAttnMaxSplits / kWarp; ++q) {
      const int sp = lane + q * kWarp;
      const float* pp = pr0 + ((size_t)sp * G + h) * ST;
      Ms[q] = sp < ns ? __ldcg(pp + HD) : -INFINITY;
      Ls[q] = sp < ns ? __ldcg(pp + HD + 1) : 0.f;
    }
#pragma unroll
    for (int q = 0; q < kAttnMaxSplits / kWarp; ++q) Mx = fmaxf(Mx, Ms[q]);
    Mx = warp_max(Mx);
    float L = 0.f;
#pragma unroll
    for (int q = 0; q < kAttnMaxSplits / kWarp; ++q) {
      const int sp = lane + q * kWarp;
      if (sp < ns) {
        const float f = expf(Ms[q] - Mx);
        sh.w[h][sp] = f;
        L += Ls[q] * f;
      }
    }
    L = warp_sum(L);
    __syncwarp();
    const float invL = 1.0f / L;
    for (int sp = lane; sp < ns; sp += kWarp) sh.w[h][sp] *= invL;
  }
  bar_sync_n(bar, NT);
#pragma unroll
  for (int o = 0; o < OPT; ++o) {
    const int idx = tid + o * NT;
    if (idx < NOUT) {
      const int h = idx / (HD / 4), d4 = idx % (HD / 4);
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int sp0 = 0; sp0 < ns; sp0 += kAttnMergeBatch) {
        float4 v[kAttnMergeBatch];
#pragma unroll
        for (int bb = 0; bb < kAttnMergeBatch; ++bb)
          if (sp0 + bb < ns)
            v[bb] = __ldcg(reinterpret_cast<const float4*>(pr0 + ((size_t)(sp0 + bb) * G + h) * ST + d4 * 4));
#pragma unroll
        for (int bb = 0; bb < kAttnMergeBatch; ++bb)
          if (sp0 + bb < ns) {
            const float w = sh.w[h][sp0 + bb];
            a.x = fmaf(w, v[bb].x, a.x); a.y = fmaf(w, v[bb].y, a.y);
            a.z = fmaf(w, v[bb].z, a.z); a.w = fmaf(w, v[bb].w, a.w);
          }
      }
      *reinterpret_cast<float4*>(p.out + (size_t)m * p.ldo + (hk * G + h) * HD + d4 * 4) = a;
    }
  }
  if (tid == 0) *ctr = 0;
  return kAttnFinished;
}

}  // namespace ms
