// ms_attn.cu -- flash-decode GQA attention over the paged KV cache.
//
// Reference semantics: gqa_attention_decode (src/main.mojo:445-519),
// compute_sliding_attention / compute_full_attention
// (src/inference/gemma4_e4b.mojo:259-411): row m (sequence seq[m] at absolute
// position pos[m]) attends positions lo..pos, lo = max(0, pos + 1 - window)
// for sliding layers and 0 otherwise; score = (q . k) / sqrt(hd); softmax with
// the maximum subtracted; out = sum p * v.  Query head h reads KV head
// h / (n_heads / n_kv).
//
// B200 layout: grid (split, kv head, row), 8 warps, about one CTA per SM in
// decode.  One CTA serves all G = n_heads / n_kv query heads of its KV head,
// so each K/V row is read once for G heads.  A row's positions are cut into
// at most n_splits contiguous ranges; a CTA brings its range into shared
// memory in chunks with cp.async.bulk (one copy per K or V row of a KV head,
// two chunk buffers so chunk c + 1 streams while chunk c computes), then per
// chunk:
//   1. scores: warps take positions, lanes slices of the head dimension, one
//      warp reduction per (position, head);
//   2. softmax bookkeeping per head (running maximum, sum, rescale factor);
//   3. values: each thread owns float4 slices of the G x hd outputs and adds
//      p * V over the chunk's positions (conflict-free 128-bit shared loads).
// Splits are merged by the last CTA of the (row, kv head) in split order
// (log-sum-exp weights; loads batched so they overlap): timing independent.
#include "ms_common.cuh"
#include "ms_kernels.h"

namespace ms {

constexpr int kAttnWarps = 8;
constexpr int kAttnThreads = kAttnWarps * kWarp;
constexpr int kAttnBufFloats = 12288;  // one chunk buffer: 48 KB of K and V rows
constexpr int kAttnMaxSplits = 64;
constexpr int kAttnMergeBatch = 8;     // partial rows loaded per round of the merge

template <int HD>
struct AttnShape {
  static constexpr int PL = HD / kWarp;                  // dims per lane (scores)
  static constexpr int VEC = PL >= 4 ? 4 : PL;           // floats per lane load
  static constexpr int NV = PL / VEC;                    // loads per lane per row
  static constexpr int PC = kAttnBufFloats / (2 * HD);   // positions per chunk
  static constexpr int ST = HD + 4;                      // partial row stride (16 B)
};

template <int VEC>
__device__ __forceinline__ void lds_vec(float* dst, const float* src) {
  if constexpr (VEC == 4) {
    const float4 v = *reinterpret_cast<const float4*>(src);
    dst[0] = v.x; dst[1] = v.y; dst[2] = v.z; dst[3] = v.w;
  } else {
    const float2 v = *reinterpret_cast<const float2*>(src);
    dst[0] = v.x; dst[1] = v.y;
  }
}

template <int HD, int G>
__global__ void __launch_bounds__(kAttnThreads) attn_kernel(const AttnParams p) {
  using S = AttnShape<HD>;
  constexpr int PC = S::PC, ST = S::ST;
  constexpr int NOUT = G * HD / 4;                       // float4 outputs per CTA
  constexpr int OPT = (NOUT + kAttnThreads - 1) / kAttnThreads;  // per thread
  extern __shared__ __align__(128) float sm[];           // [2][PC][2][HD]
  __shared__ __align__(8) uint64_t full[2];
  __shared__ float s_p[G][PC];                           // scores, then weights
  __shared__ float s_M[G], s_L[G], s_corr[G];
  __shared__ float s_w[G][kAttnMaxSplits];
  __shared__ int s_last, s_bad;

  const int split = blockIdx.x, hk = blockIdx.y, m = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    mbar_fence_init();
    s_bad = 0;
  }
  if (threadIdx.x < G) {
    s_M[threadIdx.x] = -INFINITY;
    s_L[threadIdx.x] = 0.f;
  }
  __syncthreads();
  pdl_wait();
  pdl_trigger();

  const int pos = p.pos[m], seq = p.seq[m];
  const int lo = p.window > 0 ? max(0, pos + 1 - p.window) : 0;
  const int n = pos + 1 - lo;
  // positions per split: every row fits n_splits, at least p.chunk each
  const int per = max((n + p.n_splits - 1) / p.n_splits, p.chunk);
  const int ns = (n + per - 1) / per;
  if (split >= ns) return;
  const int t_begin = lo + split * per;
  const int t_end = min(pos + 1, t_begin + per);
  const int n_chunks = (t_end - t_begin + PC - 1) / PC;
  const size_t head_off = (size_t)hk * HD;

  // warp 0 streams chunk c into buffer c % 2: one bulk copy per K / V row
  auto issue = [&](int c) {
    const int c0 = t_begin + c * PC;
    const int np = min(PC, t_end - c0);
    float* buf = sm + (size_t)(c & 1) * PC * 2 * HD;
    if (lane == 0) mbar_expect_tx(&full[c & 1], (uint32_t)(np * 2 * HD * sizeof(float)));
    __syncwarp();
    for (int j = lane; j < np; j += kWarp) {
      const size_t off = kv_row_offset(p.kv.block_table, p.kv.bt_stride, p.kv.page, p.kv.cap,
                                       p.kv.circular, seq, c0 + j, p.kv.kv_dim) + head_off;
      bulk_g2s(buf + (size_t)j * 2 * HD, p.kv.k + off, HD * sizeof(float), &full[c & 1]);
      bulk_g2s(buf + (size_t)j * 2 * HD + HD, p.kv.v + off, HD * sizeof(float), &full[c & 1]);
    }
  };
  if (warp == 0) {
    issue(0);
    if (n_chunks > 1) issue(1);
  }

  // query slices of this lane (scores) and the outputs this thread owns
  float q[G][S::PL];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    const float* qh = p.q + (size_t)m * p.ldq + (size_t)(hk * G + h) * HD;
#pragma unroll
    for (int v = 0; v < S::NV; ++v) lds_vec<S::VEC>(&q[h][v * S::VEC], qh + v * kWarp * S::VEC + lane * S::VEC);
  }
  float4 acc[OPT];
#pragma unroll
  for (int o = 0; o < OPT; ++o) acc[o] = make_float4(0.f, 0.f, 0.f, 0.f);

  int c = 0;
  for (; c < n_chunks; ++c) {
    const int np = min(PC, t_end - (t_begin + c * PC));
    const float* buf = sm + (size_t)(c & 1) * PC * 2 * HD;
    if (!mbar_wait(&full[c & 1], (c >> 1) & 1)) {
      if (lane == 0) {
        atomicOr(p.err, kErrWaitTimeout);
        s_bad = 1;
      }
    }
    __syncthreads();
    if (s_bad) break;  // CTA-uniform after the barrier
    // 1. scores
    for (int j = warp; j < np; j += kAttnWarps) {
      float kk[S::PL];
#pragma unroll
      for (int v = 0; v < S::NV; ++v)
        lds_vec<S::VEC>(&kk[v * S::VEC], buf + (size_t)j * 2 * HD + v * kWarp * S::VEC + lane * S::VEC);
#pragma unroll
      for (int h = 0; h < G; ++h) {
        float d = 0.f;
#pragma unroll
        for (int e = 0; e < S::PL; ++e) d = fmaf(q[h][e], kk[e], d);
        d = warp_sum(d);
        if (lane == 0) s_p[h][j] = d * p.scale;
      }
    }
    __syncthreads();
    // 2. running maximum / sum per head; s_p becomes the weights
    for (int h = warp; h < G; h += kAttnWarps) {
      float cm = -INFINITY;
      for (int j = lane; j < np; j += kWarp) cm = fmaxf(cm, s_p[h][j]);
      cm = warp_max(cm);
      const float m_old = s_M[h];
      const float m_new = fmaxf(m_old, cm);
      float sum = 0.f;
      for (int j = lane; j < np; j += kWarp) {
        const float e = expf(s_p[h][j] - m_new);
        s_p[h][j] = e;
        sum += e;
      }
      sum = warp_sum(sum);
      if (lane == 0) {
        const float corr = expf(m_old - m_new);  // 0 on the first chunk
        s_corr[h] = corr;
        s_L[h] = s_L[h] * corr + sum;
        s_M[h] = m_new;
      }
    }
    __syncthreads();
    // 3. values
#pragma unroll
    for (int o = 0; o < OPT; ++o) {
      const int idx = threadIdx.x + o * kAttnThreads;
      if (idx < NOUT) {
        const int h = idx / (HD / 4), d4 = idx % (HD / 4);
        const float cr = s_corr[h];
        float4 a = acc[o];
        a.x *= cr; a.y *= cr; a.z *= cr; a.w *= cr;
        const float* vcol = buf + HD + d4 * 4;
#pragma unroll 4
        for (int j = 0; j < np; ++j) {
          const float w = s_p[h][j];
          const float4 v = *reinterpret_cast<const float4*>(vcol + (size_t)j * 2 * HD);
          a.x = fmaf(w, v.x, a.x); a.y = fmaf(w, v.y, a.y);
          a.z = fmaf(w, v.z, a.z); a.w = fmaf(w, v.w, a.w);
        }
        acc[o] = a;
      }
    }
    __syncthreads();  // buffer c % 2 and s_p are free again
    if (warp == 0 && c + 2 < n_chunks) issue(c + 2);
  }
  if (s_bad) {
    // let this CTA's issued copies land (bounded) before it exits
    if (threadIdx.x == 0)
      for (int cc = c; cc < n_chunks && cc < c + 2; ++cc) mbar_wait(&full[cc & 1], (cc >> 1) & 1);
    return;
  }

  if (ns == 1) {
#pragma unroll
    for (int o = 0; o < OPT; ++o) {
      const int idx = threadIdx.x + o * kAttnThreads;
      if (idx < NOUT) {
        const int h = idx / (HD / 4), d4 = idx % (HD / 4);
        const float inv = 1.0f / s_L[h];
        float4 a = acc[o];
        a.x *= inv; a.y *= inv; a.z *= inv; a.w *= inv;
        *reinterpret_cast<float4*>(p.out + (size_t)m * p.ldo + (hk * G + h) * HD + d4 * 4) = a;
      }
    }
    return;
  }

  // ---- partial of this split: unnormalised sums, running max and sum ------
  float* part_base = p.part + (((size_t)m * p.n_kv + hk) * p.n_splits + split) * G * ST;
#pragma unroll
  for (int o = 0; o < OPT; ++o) {
    const int idx = threadIdx.x + o * kAttnThreads;
    if (idx < NOUT) {
      const int h = idx / (HD / 4), d4 = idx % (HD / 4);
      __stcg(reinterpret_cast<float4*>(part_base + (size_t)h * ST + d4 * 4), acc[o]);
    }
  }
  if (threadIdx.x < G) {
    __stcg(part_base + (size_t)threadIdx.x * ST + HD, s_M[threadIdx.x]);
    __stcg(part_base + (size_t)threadIdx.x * ST + HD + 1, s_L[threadIdx.x]);
  }

  // ---- merge the splits: the last CTA of (row, kv head) does it in order ---
  __threadfence();
  __syncthreads();
  int* ctr = p.counters + (size_t)m * p.n_kv + hk;
  if (threadIdx.x == 0) s_last = (atomicAdd(ctr, 1) == ns - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const float* pr0 = p.part + ((size_t)m * p.n_kv + hk) * p.n_splits * G * ST;
  for (int h = warp; h < G; h += kAttnWarps) {
    float M = -INFINITY;
    for (int sp = lane; sp < ns; sp += kWarp) M = fmaxf(M, __ldcg(pr0 + ((size_t)sp * G + h) * ST + HD));
    M = warp_max(M);
    float L = 0.f;
    for (int sp = lane; sp < ns; sp += kWarp) {
      const float* pp = pr0 + ((size_t)sp * G + h) * ST;
      const float f = expf(__ldcg(pp + HD) - M);
      s_w[h][sp] = f;
      L += __ldcg(pp + HD + 1) * f;
    }
    L = warp_sum(L);
    __syncwarp();
    const float invL = 1.0f / L;
    for (int sp = lane; sp < ns; sp += kWarp) s_w[h][sp] *= invL;
  }
  __syncthreads();
#pragma unroll
  for (int o = 0; o < OPT; ++o) {
    const int idx = threadIdx.x + o * kAttnThreads;
    if (idx < NOUT) {
      const int h = idx / (HD / 4), d4 = idx % (HD / 4);
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int sp0 = 0; sp0 < ns; sp0 += kAttnMergeBatch) {
        float4 v[kAttnMergeBatch];
#pragma unroll
        for (int b = 0; b < kAttnMergeBatch; ++b)
          if (sp0 + b < ns)
            v[b] = __ldcg(reinterpret_cast<const float4*>(pr0 + ((size_t)(sp0 + b) * G + h) * ST + d4 * 4));
#pragma unroll
        for (int b = 0; b < kAttnMergeBatch; ++b)
          if (sp0 + b < ns) {
            const float w = s_w[h][sp0 + b];
            a.x = fmaf(w, v[b].x, a.x); a.y = fmaf(w, v[b].y, a.y);
            a.z = fmaf(w, v[b].z, a.z); a.w = fmaf(w, v[b].w, a.w);
          }
      }
      *reinterpret_cast<float4*>(p.out + (size_t)m * p.ldo + (hk * G + h) * HD + d4 * 4) = a;
    }
  }
  if (threadIdx.x == 0) *ctr = 0;
}

template <int HD, int G>
static size_t attn_smem() {
  return (size_t)2 * AttnShape<HD>::PC * 2 * HD * sizeof(float);
}

template <int HD, int G>
static cudaError_t launch_t(const AttnParams& p, cudaStream_t s, bool pdl) {
  const size_t smem = attn_smem<HD, G>();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.n_splits, p.n_kv, p.M);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, attn_kernel<HD, G>, p);
}

#define MS_ATTN_CASES(X)                                                        \
  X(64, 1) X(64, 2) X(64, 4) X(64, 5) X(64, 8) X(128, 1) X(128, 2) X(128, 4)  \
  X(128, 5) X(128, 8) X(256, 1) X(256, 2) X(256, 4) X(256, 5) X(256, 8)        \
  X(512, 1) X(512, 2) X(512, 4)

// q, out: 16-byte aligned rows (ldq, ldo multiples of 4); the KV pools 16-byte
// aligned; n_splits <= 64.
cudaError_t launch_attention(const AttnParams& p, cudaStream_t s, bool pdl) {
  if (p.n_splits < 1 || p.n_splits > kAttnMaxSplits || p.chunk < 1 || (p.ldq & 3) ||
      (p.ldo & 3) || (p.kv.kv_dim & 3))
    return cudaErrorInvalidConfiguration;
  const int G = p.n_heads / p.n_kv;
#define MS_ATTN_CASE(HDV, GV) \
  if (p.hd == HDV && G == GV) return launch_t<HDV, GV>(p, s, pdl);
  MS_ATTN_CASES(MS_ATTN_CASE)
#undef MS_ATTN_CASE
  return cudaErrorInvalidConfiguration;
}

// Positions of one chunk buffer for head_dim hd.
int attention_block_positions(int hd) { return kAttnBufFloats / (2 * hd); }
int attention_max_splits() { return kAttnMaxSplits; }

cudaError_t prepare_attention() {
  cudaError_t e = cudaSuccess;
#define MS_ATTN_PREP(HDV, GV)                                                                 \
  if (e == cudaSuccess && attn_smem<HDV, GV>() > 48 * 1024)                                  \
    e = cudaFuncSetAttribute(attn_kernel<HDV, GV>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                             (int)attn_smem<HDV, GV>());
  MS_ATTN_CASES(MS_ATTN_PREP)
#undef MS_ATTN_PREP
  return e;
}

}  // namespace ms
