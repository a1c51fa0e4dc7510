// ms_attn_prefill.cu -- causal GQA attention for prefill chunks (many query
// rows of the same sequence per call).
//
// Reference semantics (as the decode kernel in ms_attn.cu):
// gqa_attention_decode (src/main.mojo:445-519), compute_sliding_attention /
// compute_full_attention (src/inference/gemma4_e4b.mojo:259-411): the query
// at absolute position P attends positions lo..P of its sequence,
// lo = max(0, P + 1 - window) on sliding layers and 0 otherwise;
// score = (q . k) / sqrt(hd); softmax with the maximum subtracted; out = sum p v.
//
// Decode reads every K/V row once per query row.  A prefill chunk has many
// query rows per sequence, so here one CTA serves a query block (up to R / G
// consecutive positions of one sequence, G = n_heads / n_kv query heads each:
// R query vectors) for one KV head, and every K/V chunk it stages in shared
// memory is used by all R query vectors:
//   1. scores S[R][32] = Q K^T: thread tile of R/32 rows x 4 keys, float4
//      steps over the head dimension (padded rows: conflict-free);
//   2. mask (causal + window), online softmax per row (one warp per row,
//      expf; running max / sum / rescale factor);
//   3. O[R][hd] += P V: thread tile of rows x float4 slices of hd.
// fp32 throughout (CUDA cores): the per-layer parity bound is 1e-4.  A bf16
// cache is widened to fp32 as the rows are staged.
#include "ms_common.cuh"
#include "ms_kernels.h"

namespace ms {

constexpr int kPfThreads = 256;

template <int HD>
struct PfShape {
  static constexpr int R = HD >= 512 ? 32 : 64;           // query vectors per CTA
  static constexpr int BK = 32;                            // keys per chunk
  static constexpr int QS = HD + 4;                        // padded Q / K / V row (floats)
  static constexpr int PS = BK + 1;                        // score row stride
  static constexpr int TD = (HD / 4) < 32 ? HD / 4 : 32;  // P.V threads along hd (float4)
  static constexpr int TR = kPfThreads / TD;               // P.V threads along rows
  static constexpr int RPT = R / TR;                       // P.V rows per thread
  static constexpr int DPT = HD / 4 / TD;                  // P.V float4 per thread
  static constexpr int SR = R / 32;                        // score rows per thread
  static constexpr size_t smem_floats = (size_t)R * QS + 2 * (size_t)BK * QS + (size_t)R * PS + 3 * R;
  static_assert(R % TR == 0 && (HD / 4) % TD == 0 && R % 32 == 0, "tile shape");
};

template <int HD, int G>
__global__ void __launch_bounds__(kPfThreads, 1) attn_prefill_kernel(const AttnParams p) {
  using S = PfShape<HD>;
  constexpr int R = S::R, BK = S::BK, QS = S::QS, PS = S::PS;
  constexpr int BQ = R / G;  // tokens per block
  extern __shared__ __align__(16) float sm[];
  float* sQ = sm;                       // [R][QS]
  float* sK = sQ + R * QS;              // [BK][QS]
  float* sV = sK + BK * QS;             // [BK][QS]
  float* sP = sV + BK * QS;             // [R][PS]
  float* sMax = sP + R * PS;            // [R] running maximum
  float* sSum = sMax + R;               // [R] running sum
  float* sCorr = sSum + R;              // [R] rescale factor of this chunk

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int4 blk = p.blocks[blockIdx.x];
  const int row0 = blk.x, nq = blk.y, seq = blk.z, pos0 = blk.w;
  const int hk = blockIdx.y;
  pdl_wait();
  pdl_trigger();

  // ---- query vectors r = token * G + head ----
  for (int i = tid; i < R * (HD / 4); i += kPfThreads) {
    const int r = i / (HD / 4), d4 = i % (HD / 4);
    const int tok = r / G, h = r % G;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (tok < nq && tok < BQ)
      v = *reinterpret_cast<const float4*>(p.q + (size_t)(row0 + tok) * p.ldq +
                                           (size_t)(hk * G + h) * HD + 4 * d4);
    *reinterpret_cast<float4*>(sQ + r * QS + 4 * d4) = v;
  }
  for (int r = tid; r < R; r += kPfThreads) {
    sMax[r] = -INFINITY;
    sSum[r] = 0.f;
  }

  const int t_begin = p.window > 0 ? max(0, pos0 + 1 - p.window) : 0;
  const int t_last = pos0 + nq - 1;
  const size_t head_off = (size_t)hk * HD;

  // P.V accumulators
  const int pr = tid / S::TD, pd = tid % S::TD;
  float4 acc[S::RPT][S::DPT];
#pragma unroll
  for (int i = 0; i < S::RPT; ++i)
#pragma unroll
    for (int q = 0; q < S::DPT; ++q) acc[i][q] = make_float4(0.f, 0.f, 0.f, 0.f);

  // score tile: rows sr + 32 i, keys 8 jj + sj
  const int sj = tid & 7, sr = tid >> 3;

  for (int t0 = t_begin; t0 <= t_last; t0 += BK) {
    __syncthreads();  // previous chunk's P and V are consumed
    // ---- stage K / V rows t0 .. t0 + BK - 1 ----
    for (int i = tid; i < BK * (HD / 4); i += kPfThreads) {
      const int j = i / (HD / 4), d4 = i % (HD / 4);
      const int t = t0 + j;
      float4 kv4 = make_float4(0.f, 0.f, 0.f, 0.f), vv4 = kv4;
      if (t <= t_last) {
        const size_t off = kv_row_offset(p.kv.block_table, p.kv.bt_stride, p.kv.page, p.kv.cap,
                                         p.kv.circular, seq, t, p.kv.kv_dim) + head_off + 4 * d4;
        kv4 = kv_get4(p.kv.k, p.kv.bf16, off);
        vv4 = kv_get4(p.kv.v, p.kv.bf16, off);
      }
      *reinterpret_cast<float4*>(sK + j * QS + 4 * d4) = kv4;
      *reinterpret_cast<float4*>(sV + j * QS + 4 * d4) = vv4;
    }
    __syncthreads();

    // ---- scores ----
    {
      float s[S::SR][4];
#pragma unroll
      for (int i = 0; i < S::SR; ++i)
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) s[i][jj] = 0.f;
#pragma unroll 4
      for (int d4 = 0; d4 < HD / 4; ++d4) {
        float4 qv[S::SR], kv[4];
#pragma unroll
        for (int i = 0; i < S::SR; ++i)
          qv[i] = *reinterpret_cast<const float4*>(sQ + (sr + 32 * i) * QS + 4 * d4);
#pragma unroll
        for (int jj = 0; jj < 4; ++jj)
          kv[jj] = *reinterpret_cast<const float4*>(sK + (8 * jj + sj) * QS + 4 * d4);
#pragma unroll
        for (int i = 0; i < S::SR; ++i)
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            s[i][jj] = fmaf(qv[i].x, kv[jj].x, s[i][jj]);
            s[i][jj] = fmaf(qv[i].y, kv[jj].y, s[i][jj]);
            s[i][jj] = fmaf(qv[i].z, kv[jj].z, s[i][jj]);
            s[i][jj] = fmaf(qv[i].w, kv[jj].w, s[i][jj]);
          }
      }
#pragma unroll
      for (int i = 0; i < S::SR; ++i) {
        const int r = sr + 32 * i;
        const int tok = r / G;
        const int P = pos0 + tok;
        const int lo = p.window > 0 ? max(0, P + 1 - p.window) : 0;
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const int t = t0 + 8 * jj + sj;
          const bool ok = tok < nq && tok < BQ && t <= P && t >= lo;
          sP[r * PS + 8 * jj + sj] = ok ? s[i][jj] * p.scale : -INFINITY;
        }
      }
    }
    __syncthreads();

    // ---- online softmax: one warp per row ----
    for (int r = warp; r < R; r += kPfThreads / kWarp) {
      const float sc = sP[r * PS + lane];
      const float mx = warp_max(sc);
      const float m_old = sMax[r];
      const float m_new = fmaxf(m_old, mx);
      const float pv = sc == -INFINITY ? 0.f : expf(sc - m_new);
      const float sum = warp_sum(pv);
      sP[r * PS + lane] = pv;
      if (lane == 0) {
        const float corr = m_old == -INFINITY ? (m_new == -INFINITY ? 1.f : 0.f) : expf(m_old - m_new);
        sCorr[r] = corr;
        sSum[r] = sSum[r] * corr + sum;
        sMax[r] = m_new;
      }
    }
    __syncthreads();

    // ---- O = O * corr + P V ----
#pragma unroll
    for (int i = 0; i < S::RPT; ++i) {
      const float c = sCorr[pr + S::TR * i];
#pragma unroll
      for (int q = 0; q < S::DPT; ++q) {
        acc[i][q].x *= c; acc[i][q].y *= c; acc[i][q].z *= c; acc[i][q].w *= c;
      }
    }
#pragma unroll 4
    for (int j = 0; j < BK; ++j) {
      float pj[S::RPT];
#pragma unroll
      for (int i = 0; i < S::RPT; ++i) pj[i] = sP[(pr + S::TR * i) * PS + j];
#pragma unroll
      for (int q = 0; q < S::DPT; ++q) {
        const float4 v = *reinterpret_cast<const float4*>(sV + j * QS + 4 * (pd + S::TD * q));
#pragma unroll
        for (int i = 0; i < S::RPT; ++i) {
          acc[i][q].x = fmaf(pj[i], v.x, acc[i][q].x);
          acc[i][q].y = fmaf(pj[i], v.y, acc[i][q].y);
          acc[i][q].z = fmaf(pj[i], v.z, acc[i][q].z);
          acc[i][q].w = fmaf(pj[i], v.w, acc[i][q].w);
        }
      }
    }
  }
  __syncthreads();

  // ---- out = O / sum ----
#pragma unroll
  for (int i = 0; i < S::RPT; ++i) {
    const int r = pr + S::TR * i;
    const int tok = r / G, h = r % G;
    if (tok >= nq || tok >= BQ) continue;
    const float inv = 1.0f / sSum[r];
    float* o = p.out + (size_t)(row0 + tok) * p.ldo + (size_t)(hk * G + h) * HD;
#pragma unroll
    for (int q = 0; q < S::DPT; ++q) {
      float4 v = acc[i][q];
      v.x *= inv; v.y *= inv; v.z *= inv; v.w *= inv;
      *reinterpret_cast<float4*>(o + 4 * (pd + S::TD * q)) = v;
    }
  }
}

template <int HD, int G>
static size_t pf_smem() {
  return PfShape<HD>::smem_floats * sizeof(float);
}

template <int HD, int G>
static cudaError_t launch_pf(const AttnParams& p, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.n_blocks, p.n_kv, 1);
  cfg.blockDim = dim3(kPfThreads);
  cfg.dynamicSmemBytes = pf_smem<HD, G>();
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, attn_prefill_kernel<HD, G>, p);
}

#define MS_PF_CASES(X)                                                                   \
  X(64, 1) X(64, 2) X(64, 4) X(64, 5) X(64, 8) X(128, 1) X(128, 2) X(128, 4) X(128, 5) \
  X(128, 8) X(256, 1) X(256, 2) X(256, 4) X(256, 5) X(256, 8) X(512, 1) X(512, 2)      \
  X(512, 4)

int attention_prefill_tokens(int hd, int group) {
  const int R = hd >= 512 ? 32 : 64;
  if (group <= 0 || group > R) return 0;
#define MS_PF_HAS(HDV, GV) \
  if (hd == HDV && group == GV) return R / GV;
  MS_PF_CASES(MS_PF_HAS)
#undef MS_PF_HAS
  return 0;  // no prefill kernel for this shape: the caller uses the decode kernel
}

// q, out: 16-byte aligned rows (ldq, ldo multiples of 4); the KV pools
// 16-byte aligned; every block has at most attention_prefill_tokens() rows.
cudaError_t launch_attention_prefill(const AttnParams& p, cudaStream_t s, bool pdl) {
  if (p.n_blocks < 1 || !p.blocks || (p.ldq & 3) || (p.ldo & 3) || (p.kv.kv_dim & 3) ||
      (p.kv.bf16 && (p.kv.kv_dim & 7)))
    return cudaErrorInvalidConfiguration;
  const int G = p.n_heads / p.n_kv;
#define MS_PF_CASE(HDV, GV) \
  if (p.hd == HDV && G == GV) return launch_pf<HDV, GV>(p, s, pdl);
  MS_PF_CASES(MS_PF_CASE)
#undef MS_PF_CASE
  return cudaErrorInvalidConfiguration;
}

cudaError_t prepare_attention_prefill() {
  cudaError_t e = cudaSuccess;
#define MS_PF_PREP(HDV, GV)                                                                     \
  if (e == cudaSuccess)                                                                        \
    e = cudaFuncSetAttribute(attn_prefill_kernel<HDV, GV>,                                     \
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pf_smem<HDV, GV>());
  MS_PF_CASES(MS_PF_PREP)
#undef MS_PF_PREP
  return e;
}

}  // namespace ms
