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
// B200 layout: grid (split, kv head, row).  One CTA serves all G = n_heads /
// n_kv query heads of its KV head, so each K/V row is read once for G heads.
// Positions are split into chunks (split-K over the sequence); each warp runs
// an online softmax over a strided subset of the chunk, warps are merged in
// shared memory, and splits are merged by the last CTA of the (row, kv head)
// in split order (log-sum-exp), so the result is timing independent.
#include "ms_common.cuh"
#include "ms_kernels.h"

namespace ms {

constexpr int kAttnWarps = 4;
constexpr int kAttnThreads = kAttnWarps * kWarp;

template <int HD, int G>
__global__ void __launch_bounds__(kAttnThreads) attn_kernel(const AttnParams p) {
  constexpr int VEC = HD >= 128 ? 4 : HD / 32;  // floats per lane per vector
  constexpr int NV = HD / (kWarp * VEC);         // vectors per lane
  constexpr int PL = NV * VEC;                   // dims per lane
  extern __shared__ float sm[];                  // [kAttnWarps][G][HD + 2]
  __shared__ int s_last;

  const int split = blockIdx.x, hk = blockIdx.y, m = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  pdl_trigger();
  pdl_wait();

  const int pos = p.pos[m], seq = p.seq[m];
  const int lo = p.window > 0 ? max(0, pos + 1 - p.window) : 0;
  const int n = pos + 1 - lo;
  // chunk per row: every row fits in n_splits splits whatever its length
  const int chunk = max(p.chunk, (n + p.n_splits - 1) / p.n_splits);
  const int ns = (n + chunk - 1) / chunk;
  if (split >= ns) return;
  const int t0 = lo + split * chunk;
  const int t1 = min(pos + 1, t0 + chunk);

  // query slices of the G heads this KV head serves
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
  for (int t = t0 + warp; t < t1; t += kAttnWarps) {
    const size_t off = kv_row_offset(p.kv.block_table, p.kv.bt_stride, p.kv.page, p.kv.cap,
                                     p.kv.circular, seq, t, p.kv.kv_dim) + head_off;
    const float* kr = p.kv.k + off;
    const float* vr = p.kv.v + off;
    float kk[PL], vv[PL];
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      if constexpr (VEC == 4) {
        const float4 a = __ldcg(reinterpret_cast<const float4*>(kr + v * 128 + lane * 4));
        const float4 b = __ldcg(reinterpret_cast<const float4*>(vr + v * 128 + lane * 4));
        kk[v * 4 + 0] = a.x; kk[v * 4 + 1] = a.y; kk[v * 4 + 2] = a.z; kk[v * 4 + 3] = a.w;
        vv[v * 4 + 0] = b.x; vv[v * 4 + 1] = b.y; vv[v * 4 + 2] = b.z; vv[v * 4 + 3] = b.w;
      } else {
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          kk[v * VEC + e] = __ldcg(kr + v * kWarp * VEC + lane * VEC + e);
          vv[v * VEC + e] = __ldcg(vr + v * kWarp * VEC + lane * VEC + e);
        }
      }
    }
#pragma unroll
    for (int h = 0; h < G; ++h) {
      float d = 0.f;
#pragma unroll
      for (int j = 0; j < PL; ++j) d = fmaf(q[h][j], kk[j], d);
      const float s = warp_sum(d) * p.scale;
      const float mn = fmaxf(mx[h], s);
      const float corr = expf(mx[h] - mn);
      const float pr = expf(s - mn);
      l[h] = l[h] * corr + pr;
#pragma unroll
      for (int j = 0; j < PL; ++j) acc[h][j] = acc[h][j] * corr + pr * vv[j];
      mx[h] = mn;
    }
  }

  // ---- merge the warps of this CTA --------------------------------------
  constexpr int ST = HD + 2;
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
      p.out[(size_t)m * p.ldo + (size_t)(hk * G + h) * HD + d] = A / L;
    } else {
      float* ps = part_base + (size_t)h * ST;
      ps[d] = A;
      if (d == 0) {
        ps[HD] = M;
        ps[HD + 1] = L;
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
  for (int idx = threadIdx.x; idx < G * HD; idx += kAttnThreads) {
    const int h = idx / HD, d = idx % HD;
    float M = -INFINITY;
    for (int sp = 0; sp < ns; ++sp) M = fmaxf(M, __ldcg(pr0 + ((size_t)sp * G + h) * ST + HD));
    float L = 0.f, A = 0.f;
    for (int sp = 0; sp < ns; ++sp) {
      const float* ps = pr0 + ((size_t)sp * G + h) * ST;
      const float f = expf(__ldcg(ps + HD) - M);
      L += __ldcg(ps + HD + 1) * f;
      A += __ldcg(ps + d) * f;
    }
    p.out[(size_t)m * p.ldo + (size_t)(hk * G + h) * HD + d] = A / L;
  }
  if (threadIdx.x == 0) *ctr = 0;
}

template <int HD, int G>
static cudaError_t launch_t(const AttnParams& p, cudaStream_t s, bool pdl) {
  const size_t smem = (size_t)kAttnWarps * G * (HD + 2) * sizeof(float);
  auto kern = attn_kernel<HD, G>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
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
  return cudaLaunchKernelEx(&cfg, kern, p);
}

cudaError_t launch_attention(const AttnParams& p, cudaStream_t s, bool pdl) {
  const int G = p.n_heads / p.n_kv;
#define MS_ATTN_CASE(HDV, GV) \
  if (p.hd == HDV && G == GV) return launch_t<HDV, GV>(p, s, pdl);
  MS_ATTN_CASE(64, 1) MS_ATTN_CASE(64, 2) MS_ATTN_CASE(64, 4) MS_ATTN_CASE(64, 5) MS_ATTN_CASE(64, 8)
  MS_ATTN_CASE(128, 1) MS_ATTN_CASE(128, 2) MS_ATTN_CASE(128, 4) MS_ATTN_CASE(128, 5) MS_ATTN_CASE(128, 8)
  MS_ATTN_CASE(256, 1) MS_ATTN_CASE(256, 2) MS_ATTN_CASE(256, 4) MS_ATTN_CASE(256, 5) MS_ATTN_CASE(256, 8)
  MS_ATTN_CASE(512, 1) MS_ATTN_CASE(512, 2) MS_ATTN_CASE(512, 4)
#undef MS_ATTN_CASE
  return cudaErrorInvalidConfiguration;
}

}  // namespace ms
