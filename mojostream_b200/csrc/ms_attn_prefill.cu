// ms_attn_prefill.cu -- causal GQA attention for prefill chunks (many query
// rows of the same sequence per call), on the tensor cores.
//
// Reference semantics (as the decode kernel in ms_attn.cu):
// gqa_attention_decode (src/main.mojo:445-519), compute_sliding_attention /
// compute_full_attention (src/inference/gemma4_e4b.mojo:259-411): the query
// at absolute position P attends positions lo..P of its sequence,
// lo = max(0, P + 1 - window) on sliding layers and 0 otherwise;
// score = (q . k) / sqrt(hd); softmax with the maximum subtracted; out = sum p v.
//
// One CTA serves a query block (up to R / G consecutive positions of one
// sequence, G = n_heads / n_kv query heads each: R query vectors, row
// r = token * G + head) for one KV head, flash-attention style:
//   * every warp owns 16 query rows (one mma m-tile); with hd 512 two warps
//     share the rows and split the output dims;
//   * K / V arrive in chunks of BK keys, double-buffered (cp.async; a bf16
//     cache is widened to fp32 while staging, an int8 cache multiplied out by
//     its (position, KV head) scale);
//   * S = Q K^T and O += P V run on mma.sync m16n8k8 TF32 with the 3xTF32
//     split (x = hi + lo, both TF32; hi.hi + hi.lo + lo.hi): products to
//     about 2^-21 relative, fp32 accumulation -- the per-layer parity bound
//     of 1e-4 holds as with fp32 CUDA-core math;
//   * the online softmax runs on the S fragments (row max / sum across the
//     lane quad), rescaling the O accumulators only when a row's maximum rises.
#include "ms_common.cuh"
#include "ms_kernels.h"

namespace ms {

constexpr int kPfWarps = 8;
constexpr int kPfThreads = kPfWarps * kWarp;

template <int HD>
struct PfTc {
  static constexpr int WS = HD >= 512 ? 2 : 1;   // warps sharing an m-tile (split of hd)
  static constexpr int MT = kPfWarps / WS;       // m-tiles per CTA
  static constexpr int R = 16 * MT;              // query vectors per CTA
  static constexpr int DH = HD / WS;             // output dims per warp
  static constexpr int BK = HD >= 512 ? 8 : 16;  // keys per chunk
  static constexpr int NT = BK / 8;              // S n-tiles per chunk
  static constexpr int OT = DH / 8;              // O n-tiles per warp
  static constexpr int KS = 4 / NT;              // S accumulator sets (independent MMA chains)
  static constexpr int QS = HD + 4;              // Q / K row stride (floats): conflict-free A / B loads
  static constexpr int VS = HD + 8;              // V row stride: conflict-free transposed B loads
  static constexpr size_t smem_floats = (size_t)R * QS + 2 * (size_t)BK * (QS + VS);
};

__device__ __forceinline__ uint32_t tf32_hi(float x) {
  uint32_t h;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(x));
  return h;
}
// x = hi + lo with hi, lo representable in TF32
__device__ __forceinline__ void tf32_split(float x, uint32_t& hi, uint32_t& lo) {
  hi = tf32_hi(x);
  lo = tf32_hi(x - __uint_as_float(hi));
}

__device__ __forceinline__ void mma_tf32(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// c += a b with both operands split: hi.hi + hi.lo + lo.hi
__device__ __forceinline__ void mma_3xtf32(float (&c)[4], const uint32_t (&ah)[4],
                                           const uint32_t (&al)[4], uint32_t bh0, uint32_t bh1,
                                           uint32_t bl0, uint32_t bl1) {
  mma_tf32(c, al, bh0, bh1);
  mma_tf32(c, ah, bl0, bl1);
  mma_tf32(c, ah, bh0, bh1);
}

template <int HD, int G, int DT>
__global__ void __launch_bounds__(kPfThreads, 1) attn_prefill_kernel(const AttnParams p) {
  using S = PfTc<HD>;
  constexpr int R = S::R, BK = S::BK, NT = S::NT, OT = S::OT, QS = S::QS, VS = S::VS, KS = S::KS;
  constexpr int BQ = R / G;  // tokens per block
  extern __shared__ __align__(16) float sm[];
  float* sQ = sm;                   // [R][QS]
  float* sK = sQ + R * QS;          // [2][BK][QS]
  float* sV = sK + 2 * BK * QS;     // [2][BK][VS]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int mt = warp / S::WS;                // this warp's m-tile
  const int d_base = (warp % S::WS) * S::DH;  // and its output dims
  const int4 blk = p.blocks[blockIdx.x];
  const int row0 = blk.x, nq = blk.y, seq = blk.z, pos0 = blk.w;
  const int hk = blockIdx.y;
  pdl_wait();
  pdl_trigger();

  const int t_begin = p.window > 0 ? max(0, pos0 + 1 - p.window) : 0;
  const int t_last = pos0 + nq - 1;
  const size_t head_off = (size_t)hk * HD;
  const int n_chunks = (t_last - t_begin) / BK + 1;

  // K / V rows t0 .. t0 + BK - 1 into buffer b (rows past t_last: zeros)
  auto stage = [&](int b, int t0) {
    float* k = sK + b * BK * QS;
    float* v = sV + b * BK * VS;
    for (int i = tid; i < BK * (HD / 4); i += kPfThreads) {
      const int j = i / (HD / 4), d4 = i % (HD / 4);
      const int tt = t0 + j;
      if (tt > t_last) {
        *reinterpret_cast<float4*>(k + j * QS + 4 * d4) = make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4*>(v + j * VS + 4 * d4) = make_float4(0.f, 0.f, 0.f, 0.f);
        continue;
      }
      if constexpr (DT == 2) {
        const size_t rb = kv_row_index(p.kv, seq, tt) * (size_t)p.kv.row_bytes;
        const unsigned char* kb = reinterpret_cast<const unsigned char*>(p.kv.k) + rb;
        const unsigned char* vb = reinterpret_cast<const unsigned char*>(p.kv.v) + rb;
        const float ks = reinterpret_cast<const float*>(kb + p.kv.kv_dim)[hk];
        const float vs = reinterpret_cast<const float*>(vb + p.kv.kv_dim)[hk];
        const uint32_t ku = *reinterpret_cast<const uint32_t*>(kb + head_off + 4 * d4);
        const uint32_t vu = *reinterpret_cast<const uint32_t*>(vb + head_off + 4 * d4);
        auto deq = [](uint32_t u, float s) {
          float f[4];
          i8x4_to_f32(u, f);
          return make_float4(__fmul_rn(f[0], s), __fmul_rn(f[1], s), __fmul_rn(f[2], s),
                             __fmul_rn(f[3], s));
        };
        *reinterpret_cast<float4*>(k + j * QS + 4 * d4) = deq(ku, ks);
        *reinterpret_cast<float4*>(v + j * VS + 4 * d4) = deq(vu, vs);
        continue;
      }
      const size_t off = kv_row_offset(p.kv.block_table, p.kv.bt_stride, p.kv.page, p.kv.cap,
                                       p.kv.circular, seq, tt, p.kv.kv_dim) + head_off + 4 * d4;
      if constexpr (DT == 1) {
        *reinterpret_cast<float4*>(k + j * QS + 4 * d4) = kv_get4(p.kv.k, 1, off);
        *reinterpret_cast<float4*>(v + j * VS + 4 * d4) = kv_get4(p.kv.v, 1, off);
      } else {
        cp_async16(k + j * QS + 4 * d4, p.kv.k + off);
        cp_async16(v + j * VS + 4 * d4, p.kv.v + off);
      }
    }
    cp_async_commit();
  };
  stage(0, t_begin);

  // ---- query vectors r = token * G + head (padding rows: zeros) ----
  for (int i = tid; i < R * (HD / 4); i += kPfThreads) {
    const int r = i / (HD / 4), d4 = i % (HD / 4);
    const int tok = r / G, h = r % G;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (tok < nq && tok < BQ)
      v = *reinterpret_cast<const float4*>(p.q + (size_t)(row0 + tok) * p.ldq +
                                           (size_t)(hk * G + h) * HD + 4 * d4);
    *reinterpret_cast<float4*>(sQ + r * QS + 4 * d4) = v;
  }

  // this lane's two rows of the m-tile: g and g + 8
  int pos_r[2], lo_r[2];
  bool ok_r[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = mt * 16 + g + 8 * h;
    const int tok = r / G;
    ok_r[h] = tok < nq && tok < BQ;
    pos_r[h] = pos0 + tok;
    lo_r[h] = p.window > 0 ? max(0, pos_r[h] + 1 - p.window) : 0;
  }
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  float o[OT][4];
#pragma unroll
  for (int n = 0; n < OT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  const float* qa = sQ + (mt * 16 + g) * QS + t;

  for (int c = 0; c < n_chunks; ++c) {
    const int t0 = t_begin + c * BK;
    if (c + 1 < n_chunks) {
      stage((c + 1) & 1, t0 + BK);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();  // chunk c (and, the first time, Q) is in shared memory
    const float* k = sK + (c & 1) * BK * QS;
    const float* v = sV + (c & 1) * BK * VS;

    // ---- S = Q K^T for this warp's 16 rows x BK keys ----
    // k-step j accumulates into set j % KS: KS x NT = 4 independent chains
    float sa[KS][NT][4];
#pragma unroll
    for (int q = 0; q < KS; ++q)
#pragma unroll
      for (int n = 0; n < NT; ++n) sa[q][n][0] = sa[q][n][1] = sa[q][n][2] = sa[q][n][3] = 0.f;
#pragma unroll 2
    for (int k0 = 0; k0 < HD; k0 += 8 * KS) {
#pragma unroll
      for (int q = 0; q < KS; ++q) {
        const int kk = k0 + 8 * q;
        uint32_t ah[4], al[4];
        tf32_split(qa[kk], ah[0], al[0]);
        tf32_split(qa[8 * QS + kk], ah[1], al[1]);
        tf32_split(qa[kk + 4], ah[2], al[2]);
        tf32_split(qa[8 * QS + kk + 4], ah[3], al[3]);
#pragma unroll
        for (int n = 0; n < NT; ++n) {
          const float* kr = k + (8 * n + g) * QS + kk + t;
          uint32_t bh0, bl0, bh1, bl1;
          tf32_split(kr[0], bh0, bl0);
          tf32_split(kr[4], bh1, bl1);
          mma_3xtf32(sa[q][n], ah, al, bh0, bh1, bl0, bl1);
        }
      }
    }
    float s[NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float v = sa[0][n][e];
#pragma unroll
        for (int q = 1; q < KS; ++q) v += sa[q][n][e];
        s[n][e] = v;
      }

    // ---- mask, online softmax on the fragments ----
    // s[n][0..1]: row g, keys 8n + 2t, +1; s[n][2..3]: row g + 8
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float mx = -INFINITY;
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int tt = t0 + 8 * n + 2 * t + e;
          const bool ok = ok_r[h] && tt <= pos_r[h] && tt >= lo_r[h];
          const float sv = ok ? s[n][2 * h + e] * p.scale : -INFINITY;
          s[n][2 * h + e] = sv;
          mx = fmaxf(mx, sv);
        }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      if (mx > m_run[h]) {  // the row's maximum rises: rescale (lanes of a quad agree)
        const float corr = expf(m_run[h] - mx);  // 0 the first time
        l_run[h] *= corr;
#pragma unroll
        for (int n = 0; n < OT; ++n) {
          o[n][2 * h] *= corr;
          o[n][2 * h + 1] *= corr;
        }
        m_run[h] = mx;
      }
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float sv = s[n][2 * h + e];
          const float pv = sv == -INFINITY ? 0.f : expf(sv - m_run[h]);
          s[n][2 * h + e] = pv;
          l_run[h] += pv;  // this lane's share; the quad is summed at the end
        }
    }

    // ---- O += P V ----
    // A fragment of P for keys 8n .. 8n + 7: (row g, key t), (g + 8, t),
    // (g, t + 4), (g + 8, t + 4); key j of row g sits in lane (g, j / 2),
    // element j % 2 of the S fragment
    const int src = (lane & ~3) | (t >> 1);
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const float x0 = __shfl_sync(0xffffffffu, s[n][0], src);
      const float x1 = __shfl_sync(0xffffffffu, s[n][1], src);
      const float x2 = __shfl_sync(0xffffffffu, s[n][2], src);
      const float x3 = __shfl_sync(0xffffffffu, s[n][3], src);
      const float y0 = __shfl_sync(0xffffffffu, s[n][0], src + 2);
      const float y1 = __shfl_sync(0xffffffffu, s[n][1], src + 2);
      const float y2 = __shfl_sync(0xffffffffu, s[n][2], src + 2);
      const float y3 = __shfl_sync(0xffffffffu, s[n][3], src + 2);
      const bool odd = t & 1;
      uint32_t ah[4], al[4];
      tf32_split(odd ? x1 : x0, ah[0], al[0]);  // (g, t)
      tf32_split(odd ? x3 : x2, ah[1], al[1]);  // (g + 8, t)
      tf32_split(odd ? y1 : y0, ah[2], al[2]);  // (g, t + 4)
      tf32_split(odd ? y3 : y2, ah[3], al[3]);  // (g + 8, t + 4)
      const float* vr = v + (8 * n + t) * VS + d_base + g;
#pragma unroll
      for (int d = 0; d < OT; ++d) {
        uint32_t bh0, bl0, bh1, bl1;
        tf32_split(vr[8 * d], bh0, bl0);           // (key t, dim 8d + g)
        tf32_split(vr[4 * VS + 8 * d], bh1, bl1);  // (key t + 4, dim 8d + g)
        mma_3xtf32(o[d], ah, al, bh0, bh1, bl0, bl1);
      }
    }
    __syncthreads();  // buffer c & 1 is free for chunk c + 2
  }

  // ---- out = O / sum (valid rows) ----
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float l = l_run[h];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    if (!ok_r[h]) continue;
    const int r = mt * 16 + g + 8 * h;
    const int tok = r / G, hq = r % G;
    const float inv = 1.0f / l;
    float* out = p.out + (size_t)(row0 + tok) * p.ldo + (size_t)(hk * G + hq) * HD + d_base + 2 * t;
#pragma unroll
    for (int d = 0; d < OT; ++d)
      *reinterpret_cast<float2*>(out + 8 * d) = make_float2(o[d][2 * h] * inv, o[d][2 * h + 1] * inv);
  }
}

template <int HD, int G, int DT>
static cudaError_t launch_pf(const AttnParams& p, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.n_blocks, p.n_kv, 1);
  cfg.blockDim = dim3(kPfThreads);
  cfg.dynamicSmemBytes = PfTc<HD>::smem_floats * sizeof(float);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, attn_prefill_kernel<HD, G, DT>, p);
}

#define MS_PF_CASES(X)                                                                   \
  X(64, 1) X(64, 2) X(64, 4) X(64, 5) X(64, 8) X(128, 1) X(128, 2) X(128, 4) X(128, 5) \
  X(128, 8) X(256, 1) X(256, 2) X(256, 4) X(256, 5) X(256, 8) X(512, 1) X(512, 2)      \
  X(512, 4)

int attention_prefill_tokens(int hd, int group) {
  const int R = hd >= 512 ? PfTc<512>::R : PfTc<256>::R;
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
      (p.kv.bf16 && (p.kv.kv_dim & 7)) ||
      (p.kv.i8 && ((p.kv.row_bytes & 15) || p.kv.hd != p.hd)))
    return cudaErrorInvalidConfiguration;
  const int G = p.n_heads / p.n_kv;
#define MS_PF_CASE(HDV, GV)                                                  \
  if (p.hd == HDV && G == GV)                                                \
    return p.kv.i8 ? launch_pf<HDV, GV, 2>(p, s, pdl)                        \
                   : (p.kv.bf16 ? launch_pf<HDV, GV, 1>(p, s, pdl) : launch_pf<HDV, GV, 0>(p, s, pdl));
  MS_PF_CASES(MS_PF_CASE)
#undef MS_PF_CASE
  return cudaErrorInvalidConfiguration;
}

cudaError_t prepare_attention_prefill() {
  cudaError_t e = cudaSuccess;
#define MS_PF_PREP1(HDV, GV, DTV)                                                            \
  if (e == cudaSuccess)                                                                      \
    e = cudaFuncSetAttribute(attn_prefill_kernel<HDV, GV, DTV>,                             \
                             cudaFuncAttributeMaxDynamicSharedMemorySize,                   \
                             (int)(PfTc<HDV>::smem_floats * sizeof(float)));
#define MS_PF_PREP(HDV, GV) MS_PF_PREP1(HDV, GV, 0) MS_PF_PREP1(HDV, GV, 1) MS_PF_PREP1(HDV, GV, 2)
  MS_PF_CASES(MS_PF_PREP)
#undef MS_PF_PREP
#undef MS_PF_PREP1
  return e;
}

}  // namespace ms
