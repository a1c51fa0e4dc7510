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
// B200 layout: grid (split, kv head, row), 8 warps.  One CTA serves all
// G = n_heads / n_kv query heads of its KV head, so each K/V row is read once
// for G heads.  A row's positions are cut into at most n_splits contiguous
// ranges (split-K over the sequence); a CTA walks its range in blocks of
// 8 * PW positions, each warp taking PW positions whose K and V rows it
// requests all at once (PW * hd / 32 floats per lane each), then an online
// softmax per head.  Warps are merged in shared memory, splits by the last
// CTA of the (row, kv head) in split order (log-sum-exp): timing independent.
#include "ms_common.cuh"
#include "ms_kernels.h"

namespace ms {

constexpr int kAttnWarps = 8;
constexpr int kAttnThreads = kAttnWarps * kWarp;

template <int HD, int G>
__global__ void __launch_bounds__(kAttnThreads) attn_kernel(const AttnParams p) {
  constexpr int VEC = HD >= 128 ? 4 : HD / 32;  // floats per lane per vector
  constexpr int NV = HD / (kWarp * VEC);         // vectors per lane per row
  constexpr int PL = NV * VEC;                   // dims per lane
  constexpr int PW = HD >= 512 ? 1 : 512 / HD;   // positions per warp per block
  constexpr int CP = kAttnWarps * PW;            // positions per CTA block
  constexpr int ST = HD + 2;
  extern __shared__ float sm[];                  // [kAttnWarps][G][HD + 2]
  __shared__ int s_last;

  const int split = blockIdx.x, hk = blockIdx.y, m = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  pdl_trigger();
  pdl_wait();

  const int pos = p.pos[m], seq = p.seq[m];
  const int lo = p.window > 0 ? max(0, pos + 1 - p.window) : 0;
  const int n = pos + 1 - lo;
  // positions per split: a multiple of the block, every row fits n_splits
  int per = (n + p.n_splits - 1) / p.n_splits;
  per = ((max(per, p.chunk) + CP - 1) / CP) * CP;
  const int ns = (n + per - 1) / per;
  if (split >= ns) return;
  const int t_begin = lo + split * per;
  const int t_end = min(pos + 1, t_begin + per);

  float q[G][PL];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    const float* qh = p.q + (size_t)m * p.ldq + (size_t)(hk * G + h) * HD;
#pragma unroll
    for (int v = 0; v < NV; ++v)
#pragma unroll
      for (int e = 0; e < VEC; ++e) q[h][v * VEC + e] = qh[v * kWarp * VEC + lane * VEC + e];
  }
  float mx[G], l[G], acc[G][PL];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    mx[h] = -INFINITY;
    l[h] = 0.f;
#pragma unroll
    for (int d = 0; d < PL; ++d) acc[h][d] = 0.f;
  }

  const size_t head_off = (size_t)hk * HD;
  for (int t0 = t_begin; t0 < t_end; t0 += CP) {
    // K and V rows of this warp's PW positions, all requested before use
    float kk[PW][PL], vv[PW][PL];
#pragma unroll
    for (int j = 0; j < PW; ++j) {
      const int t = t0 + warp * PW + j;
      if (t < t_end) {
        const size_t off = kv_row_offset(p.kv.block_table, p.kv.bt_stride, p.kv.page, p.kv.cap,
                                         p.kv.circular, seq, t, p.kv.kv_dim) + head_off;
        const float* kr = p.kv.k + off;
        const float* vr = p.kv.v + off;
#pragma unroll
        for (int v = 0; v < NV; ++v) {
          if constexpr (VEC == 4) {
            const float4 a = __ldcg(reinterpret_cast<const float4*>(kr + v * 128 + lane * 4));
            const float4 b = __ldcg(reinterpret_cast<const float4*>(vr + v * 128 + lane * 4));
            kk[j][v * 4 + 0] = a.x; kk[j][v * 4 + 1] = a.y; kk[j][v * 4 + 2] = a.z; kk[j][v * 4 + 3] = a.w;
            vv[j][v * 4 + 0] = b.x; vv[j][v * 4 + 1] = b.y; vv[j][v * 4 + 2] = b.z; vv[j][v * 4 + 3] = b.w;
          } else {
#pragma unroll
            for (int e = 0; e < VEC; ++e) {
              kk[j][v * VEC + e] = __ldcg(kr + v * kWarp * VEC + lane * VEC + e);
              vv[j][v * VEC + e] = __ldcg(vr + v * kWarp * VEC + lane * VEC + e);
            }
          }
        }
      }
    }
#pragma unroll
    for (int j = 0; j < PW; ++j) {
      const int t = t0 + warp * PW + j;
      if (t >= t_end) break;  // warp-uniform
#pragma unroll
      for (int h = 0; h < G; ++h) {
        float d = 0.f;
#pragma unroll
        for (int e = 0; e < PL; ++e) d = fmaf(q[h][e], kk[j][e], d);
        const float s = warp_sum(d) * p.scale;
        const float mn = fmaxf(mx[h], s);
        const float corr = expf(mx[h] - mn);
        const float pr = expf(s - mn);
        l[h] = l[h] * corr + pr;
#pragma unroll
        for (int e = 0; e < PL; ++e) acc[h][e] = acc[h][e] * corr + pr * vv[j][e];
        mx[h] = mn;
      }
    }
  }

  // ---- merge the warps of this CTA --------------------------------------
#pragma unroll
  for (int h = 0; h < G; ++h) {
    float* w = sm + ((size_t)warp * G + h) * ST;
#pragma unroll
    for (int v = 0; v < NV; ++v)
#pragma unroll
      for (int e = 0; e < VEC; ++e) w[v * kWarp * VEC + lane * VEC + e] = acc[h][v * VEC + e];
    if (lane == 0) {
      w[HD] = mx[h];
      w[HD + 1] = l[h];
    }
  }
  __syncthreads();

  float* part_base = p.part + ((((size_t)m * p.n_kv + hk) * p.n_splits + split) * G) * ST;
  for (int idx = threadIdx.x; idx < G * HD; idx += kAttnThreads) {
    const int h = idx / HD, d = idx % HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, sm[((size_t)w * G + h) * ST + HD]);
    float L = 0.f, A = 0.f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) {
      const float* ws = sm + ((size_t)w * G + h) * ST;
      const float f = ws[HD + 1] > 0.f ? expf(ws[HD] - M) : 0.f;
      L += ws[HD + 1] * f;
      A += ws[d] * f;
    }
    if (ns == 1) {
      const int c = (hk * G + h) * HD + d;
      p.out[(size_t)m * p.ldo + c] = A / L;
      if (p.out_frag) frag_store(p.out_frag, p.ldo / 16, m, c, A / L);
    } else {
      float* ps = part_base + (size_t)h * ST;
      __stcg(ps + d, A);
      if (d == 0) {
        __stcg(ps + HD, M);
        __stcg(ps + HD + 1, L);
      }
    }
  }
  if (ns == 1) return;

  // ---- merge the splits: the last CTA of (row, kv head) does it in order ---
  __threadfence();
  __syncthreads();
  int* ctr = p.counters + (size_t)m * p.n_kv + hk;
  if (threadIdx.x == 0) s_last = (atomicAdd(ctr, 1) == ns - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const float* pr0 = p.part + ((((size_t)m * p.n_kv + hk) * p.n_splits) * G) * ST;
  // per (head, split): running max and sum -> merge weights in shared memory
  // (sm is free again: reuse it as w[G][n_splits])
  float* wsm = sm;
  for (int idx = threadIdx.x; idx < ns * G; idx += kAttnThreads) {
    const int sp = idx / G, h = idx % G;
    wsm[h * p.n_splits + sp] = __ldcg(pr0 + ((size_t)sp * G + h) * ST + HD);
    wsm[(G + h) * p.n_splits + sp] = __ldcg(pr0 + ((size_t)sp * G + h) * ST + HD + 1);
  }
  __syncthreads();
  if (warp < G) {
    const int h = warp;
    float M = -INFINITY;
    for (int sp = lane; sp < ns; sp += kWarp) M = fmaxf(M, wsm[h * p.n_splits + sp]);
    M = warp_max(M);
    float L = 0.f;
    for (int sp = lane; sp < ns; sp += kWarp) {
      const float f = expf(wsm[h * p.n_splits + sp] - M);
      wsm[h * p.n_splits + sp] = f;
      L += wsm[(G + h) * p.n_splits + sp] * f;
    }
    L = warp_sum(L);
    __syncwarp();
    const float invL = 1.0f / L;
    for (int sp = lane; sp < ns; sp += kWarp) wsm[h * p.n_splits + sp] *= invL;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * HD; idx += kAttnThreads) {
    const int h = idx / HD, d = idx % HD;
    float A = 0.f;
#pragma unroll 8
    for (int sp = 0; sp < ns; ++sp)
      A += __ldcg(pr0 + ((size_t)sp * G + h) * ST + d) * wsm[h * p.n_splits + sp];
    const int c = (hk * G + h) * HD + d;
    p.out[(size_t)m * p.ldo + c] = A;
    if (p.out_frag) frag_store(p.out_frag, p.ldo / 16, m, c, A);
  }
  if (threadIdx.x == 0) *ctr = 0;
}

template <int HD, int G>
static size_t attn_smem() {
  return (size_t)kAttnWarps * G * (HD + 2) * sizeof(float);
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

cudaError_t launch_attention(const AttnParams& p, cudaStream_t s, bool pdl) {
  const int G = p.n_heads / p.n_kv;
#define MS_ATTN_CASE(HDV, GV) \
  if (p.hd == HDV && G == GV) return launch_t<HDV, GV>(p, s, pdl);
  MS_ATTN_CASES(MS_ATTN_CASE)
#undef MS_ATTN_CASE
  return cudaErrorInvalidConfiguration;
}

// Positions one CTA block covers (the split granularity) for head_dim hd.
int attention_block_positions(int hd) { return kAttnWarps * (hd >= 512 ? 1 : 512 / hd); }

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
