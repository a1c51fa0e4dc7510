// ms_attn.cu -- flash-decode GQA attention over the paged KV cache, one
// launch per layer: grid (split, KV head, row).
//
// Reference semantics: gqa_attention_decode (src/main.mojo:445-519),
// compute_sliding_attention / compute_full_attention
// (src/inference/gemma4_e4b.mojo:259-411): row m (sequence seq[m] at absolute
// position pos[m]) attends positions lo..pos, lo = max(0, pos + 1 - window)
// on sliding layers and 0 otherwise; score = (q . k) / sqrt(hd); softmax with
// the maximum subtracted; out = sum p * v.  Query head h reads KV head
// h / (n_heads / n_kv); a CTA serves all G query heads of its KV head, so each
// K / V row is read once for G heads.
//
// Per-warp streams (no CTA barrier in the main loop): the CTA's positions go
// to its NW warps round-robin; every warp brings its next positions' K and V
// rows into a private ring of P slots, all 32 lanes issuing 16-byte cp.async
// copies (one commit group per position), so up to NW * P rows are in flight
// per CTA.  (One bulk copy per row, issued by one lane, was bounded by the
// per-SM rate of copy requests: the same time for half the bytes.)  A warp holds its lanes' slices
// of the G query vectors and of the G running outputs in registers; per
// position it forms the G scores (lane partial dot products, one warp
// all-reduce each), updates its running maximum / sum / output (online
// softmax, expf), and moves on.  At the end the warps are combined through
// shared memory (log-sum-exp weights), and the row's splits are merged by the
// last CTA of the (row, KV head) in split order: results do not depend on
// timing.
#include "ms_common.cuh"
#include "ms_kernels.h"

namespace ms {

constexpr int kAttnMaxSplits = 64;
constexpr int kAttnMergeBatch = 8;  // partial rows loaded per round of the merge

// Most splits of one (row, KV head) that run as a cluster (a non-portable
// size: B200 runs clusters of up to 16 CTAs), and whether every attention
// kernel can hold such a cluster (checked once by prepare_attention).
constexpr int kAttnMaxCluster = 16;
static bool g_attn_cluster_ok = false;

// DT: the cache's element type -- 0 fp32; 1 bfloat16 (rows half the bytes,
// widened to fp32 as they are read out of the ring); 2 int8 with one fp32
// scale per (position, KV head) (a quarter of the bytes; the two scales ride
// in the slot behind the K and V rows, the score takes the K scale after the
// dot product and the V weight the V scale).
template <int HD, int G, int DT>
struct WarpAttn {
  static constexpr int NW = (G * HD >= 2048) ? 4 : 8;  // warps (registers: q + out slices)
  static constexpr int NT = NW * kWarp;
  static constexpr int VEC = HD >= 128 ? 4 : 2;        // values per lane load
  static constexpr int NV = HD / (kWarp * VEC);        // loads per lane per row
  static constexpr int PL = NV * VEC;                  // dims per lane
  static constexpr int EB = DT == 0 ? 4 : (DT == 1 ? 2 : 1);  // bytes per cached value
  static constexpr int SLOTB = 2 * HD * EB + (DT == 2 ? 16 : 0);  // K row, V row (, scales)
  // slots per warp: about 64 KB of rows in flight per CTA, and at least enough
  // for the end-of-unit combine (NW x G x (HD + 2) floats) to reuse the rings
  static constexpr int P0 = 65536 / (NW * SLOTB);
  static constexpr int PMIN = (G * (HD + 2) * 4 + SLOTB - 1) / SLOTB;
  static constexpr int P1 = P0 > 8 ? 8 : (P0 < 2 ? 2 : P0);
  static constexpr int P = P1 < PMIN ? PMIN : P1;
  static constexpr size_t ring = (size_t)NW * P * SLOTB;
  static constexpr int ST = HD + 4;                    // partial row stride (16 B)
  // + this split's partial [G][ST] for the cluster merge
  static constexpr size_t smem = ring + (size_t)G * ST * 4;
  static_assert(NW * G * (HD + 2) * 4 <= ring, "combine buffer");
  static_assert(ring % 16 == 0, "partial alignment");
  static_assert(P <= 32, "row offsets are fetched 32 positions at a time");
};

// VEC cached values at src (shared memory) as floats.
template <int VEC, int DT>
__device__ __forceinline__ void ld_vec(float* dst, const unsigned char* src) {
  if constexpr (DT == 2) {  // int8: sign-extended bytes (exact in fp32)
    if constexpr (VEC == 4) {
      i8x4_to_f32(*reinterpret_cast<const uint32_t*>(src), dst);
    } else {
      float t[4];
      i8x4_to_f32(*reinterpret_cast<const unsigned short*>(src), t);
      dst[0] = t[0]; dst[1] = t[1];
    }
  } else if constexpr (DT == 1) {
    if constexpr (VEC == 4) {
      const uint2 u = *reinterpret_cast<const uint2*>(src);
      dst[0] = __uint_as_float(u.x << 16); dst[1] = __uint_as_float(u.x & 0xffff0000u);
      dst[2] = __uint_as_float(u.y << 16); dst[3] = __uint_as_float(u.y & 0xffff0000u);
    } else {
      const uint32_t u = *reinterpret_cast<const uint32_t*>(src);
      dst[0] = __uint_as_float(u << 16); dst[1] = __uint_as_float(u & 0xffff0000u);
    }
  } else if constexpr (VEC == 4) {
    const float4 v = *reinterpret_cast<const float4*>(src);
    dst[0] = v.x; dst[1] = v.y; dst[2] = v.z; dst[3] = v.w;
  } else {
    const float2 v = *reinterpret_cast<const float2*>(src);
    dst[0] = v.x; dst[1] = v.y;
  }
}


template <int HD, int G, int DT>
__global__ void __launch_bounds__(WarpAttn<HD, G, DT>::NT) attn_kernel(const AttnParams p) {
  using S = WarpAttn<HD, G, DT>;
  constexpr int NW = S::NW, NT = S::NT, P = S::P, PL = S::PL, VEC = S::VEC, ST = S::ST;
  constexpr int EB = S::EB;
  extern __shared__ __align__(128) unsigned char smb[];  // [NW][P][K row | V row], partial
  __shared__ float s_w[G][kAttnMaxSplits];
  __shared__ float s_f[NW][G], s_M[G], s_L[G];
  __shared__ int s_last;

  const int split = blockIdx.x, hk = blockIdx.y, m = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  pdl_wait();
  pdl_trigger();

  const int pos = p.pos[m], seq = p.seq[m];
  const int lo = p.window > 0 ? max(0, pos + 1 - p.window) : 0;
  const int n = pos + 1 - lo;
  const int per = max((n + p.n_splits - 1) / p.n_splits, p.chunk);
  const int ns = (n + per - 1) / per;
  // cluster mode: the n_splits CTAs of (row, KV head) are one cluster and
  // every one of them takes part in both cluster barriers; a split without
  // positions runs the (empty) loop and writes nothing
  const bool cl = p.cluster != 0;
  const bool active = split < ns;
  if (!active && !cl) {  // CTA-uniform
    return;
  }
  const int t_begin = lo + split * per;
  const int t_end = min(pos + 1, t_begin + per);
  const int n_pos = t_end - t_begin;
  const int cnt = n_pos > warp ? (n_pos - warp + NW - 1) / NW : 0;  // this warp's positions
  const size_t head_off = (size_t)hk * HD;
  unsigned char* ring = smb + (size_t)warp * P * S::SLOTB;
  float* cpart = reinterpret_cast<float*>(smb + S::ring);  // [G][ST] (cluster mode)
  const unsigned char* kpool = reinterpret_cast<const unsigned char*>(p.kv.k);
  const unsigned char* vpool = reinterpret_cast<const unsigned char*>(p.kv.v);

  // Byte offsets of this warp's positions' head rows, 32 at a time: lane j
  // holds that of position base + j (one batch of independent block-table
  // loads instead of a dependent load before every copy).
  auto row_offsets = [&](int base) -> unsigned long long {
    const int i = base + lane;
    if (i >= cnt) return 0ull;
    const size_t row = kv_row_index(p.kv, seq, t_begin + warp + NW * i);
    if constexpr (DT == 2) return row * (size_t)p.kv.row_bytes + head_off;
    return (row * (size_t)p.kv.kv_dim + head_off) * EB;
  };
  // the warp streams position i (t_begin + warp + NW i), whose head rows
  // start `off` bytes into the pools, into slot i % P, then closes the
  // position's commit group (always, so that group j is position j's)
  auto issue = [&](int i, unsigned long long off) {
    if (i < cnt) {
      unsigned char* dst = ring + (i % P) * S::SLOTB;
      const unsigned char* ks = kpool + off;
      const unsigned char* vs = vpool + off;
      constexpr int CH = HD * EB / 16;  // 16-byte chunks per row
#pragma unroll
      for (int c = lane; c < CH; c += kWarp) {
        cp_async16(dst + c * 16, ks + c * 16);
        cp_async16(dst + HD * EB + c * 16, vs + c * 16);
      }
      if constexpr (DT == 2) {
        if (lane == 0) {  // the row's scales: behind its kv_dim values
          const size_t so = (size_t)p.kv.kv_dim - head_off + 4 * (size_t)hk;
          cp_async4(dst + 2 * HD, ks + so);
          cp_async4(dst + 2 * HD + 4, vs + so);
        }
      }
    }
    cp_async_commit();
  };
  unsigned long long offs = row_offsets(0);  // positions 0..31 (P <= 32)
#pragma unroll
  for (int i = 0; i < P; ++i) issue(i, __shfl_sync(0xffffffffu, offs, i));

  // this lane's slices: dims (v * 32 + lane) * VEC + e
  float q[G][PL], acc[G][PL], mrun[G], lrun[G];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    const float* qh = p.q + (size_t)m * p.ldq + (size_t)(hk * G + h) * HD;
#pragma unroll
    for (int v = 0; v < S::NV; ++v) {
      if constexpr (VEC == 4) {
        const float4 t = __ldcg(reinterpret_cast<const float4*>(qh + (v * kWarp + lane) * VEC));
        q[h][v * 4] = t.x; q[h][v * 4 + 1] = t.y; q[h][v * 4 + 2] = t.z; q[h][v * 4 + 3] = t.w;
      } else {
        const float2 t = __ldcg(reinterpret_cast<const float2*>(qh + (v * kWarp + lane) * VEC));
        q[h][v * 2] = t.x; q[h][v * 2 + 1] = t.y;
      }
    }
#pragma unroll
    for (int e = 0; e < PL; ++e) acc[h][e] = 0.f;
    mrun[h] = -INFINITY;
    lrun[h] = 0.f;
  }

  for (int i = 0; i < cnt; ++i) {
    const int slot = i % P;
    cp_async_wait<P - 1>();  // this lane's copies of position i have landed
    __syncwarp();            // ... and every other lane's
    float kk[PL], vv[PL];
    const unsigned char* kr = ring + slot * S::SLOTB;
#pragma unroll
    for (int v = 0; v < S::NV; ++v) {
      ld_vec<VEC, DT>(&kk[v * VEC], kr + (v * kWarp + lane) * VEC * EB);
      ld_vec<VEC, DT>(&vv[v * VEC], kr + (HD + (v * kWarp + lane) * VEC) * EB);
    }
    float kscale = p.scale, vscale = 1.f;
    if constexpr (DT == 2) {
      kscale = reinterpret_cast<const float*>(kr + 2 * HD)[0] * p.scale;
      vscale = reinterpret_cast<const float*>(kr + 2 * HD)[1];
    }
    __syncwarp();  // every lane holds its slice: the slot can be refilled
    if (((i + P) & 31) == 0) offs = row_offsets(i + P);  // warp-uniform
    issue(i + P, __shfl_sync(0xffffffffu, offs, (i + P) & 31));
    // dot products on packed FMAs: dims 2j and 2j + 1 in two chains, added at the end
    float sc[G];
#pragma unroll
    for (int h = 0; h < G; ++h) {
      float2 d2 = make_float2(0.f, 0.f);
#pragma unroll
      for (int e = 0; e < PL; e += 2)
        fma2(d2, make_float2(q[h][e], q[h][e + 1]), make_float2(kk[e], kk[e + 1]));
      sc[h] = d2.x + d2.y;
    }
#pragma unroll
    for (int h = 0; h < G; ++h) sc[h] = warp_sum(sc[h]) * kscale;  // G independent chains
#pragma unroll
    for (int h = 0; h < G; ++h) {
      const float s = sc[h];
      // the running maximum only moves up: rescale when it does (s is the
      // same in every lane, so the branch is warp-uniform); otherwise the
      // factor is exactly 1 and the products are unchanged
      if (s > mrun[h]) {
        const float corr = expf(mrun[h] - s);  // 0 on the first position
        lrun[h] *= corr;
#pragma unroll
        for (int e = 0; e < PL; ++e) acc[h][e] *= corr;
        mrun[h] = s;
      }
      const float ew = expf(s - mrun[h]);
      lrun[h] += ew;
      const float wv = DT == 2 ? ew * vscale : ew;
#pragma unroll
      for (int e = 0; e < PL; e += 2) {
        float2 a2 = make_float2(acc[h][e], acc[h][e + 1]);
        fma2(a2, make_float2(wv, wv), make_float2(vv[e], vv[e + 1]));
        acc[h][e] = a2.x;
        acc[h][e + 1] = a2.y;
      }
    }
  }
  cp_async_wait<0>();  // (only empty groups remain)
  __syncthreads();     // every warp is past its ring: it becomes the combine buffer

  // ---- combine the warps: comb[w][h][0..HD) outputs, [HD] max, [HD+1] sum ----
  float* comb = reinterpret_cast<float*>(smb);
#pragma unroll
  for (int h = 0; h < G; ++h) {
    float* c = comb + ((size_t)warp * G + h) * (HD + 2);
#pragma unroll
    for (int v = 0; v < S::NV; ++v)
#pragma unroll
      for (int e = 0; e < VEC; ++e) c[(v * kWarp + lane) * VEC + e] = acc[h][v * VEC + e];
    if (lane == 0) {
      c[HD] = mrun[h];
      c[HD + 1] = lrun[h];
    }
  }
  __syncthreads();
  // per head: the maximum over the warps, each warp's weight and the sum
  // (computed once per head, not per output element)
  if (tid < G) {
    const int h = tid;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, comb[((size_t)w * G + h) * (HD + 2) + HD]);
    float L = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float* c = comb + ((size_t)w * G + h) * (HD + 2);
      const float f = expf(c[HD] - M);  // 0 for warps without positions
      s_f[w][h] = f;
      L = fmaf(c[HD + 1], f, L);
    }
    s_M[h] = M;
    s_L[h] = L;
  }
  __syncthreads();
  float* part_base = p.part + (((size_t)m * p.n_kv + hk) * p.n_splits + split) * G * ST;
  for (int idx = tid; idx < G * HD; idx += NT) {
    const int h = idx / HD, d = idx % HD;
    const float M = s_M[h], L = s_L[h];
    float a = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) a = fmaf(comb[((size_t)w * G + h) * (HD + 2) + d], s_f[w][h], a);
    if (!active) {
    } else if (ns == 1) {
      p.out[(size_t)m * p.ldo + (hk * G + h) * HD + d] = a / L;
    } else if (cl) {
      cpart[h * ST + d] = a;
      if (d == 0) {
        cpart[h * ST + HD] = M;
        cpart[h * ST + HD + 1] = L;
      }
    } else {
      __stcg(part_base + (size_t)h * ST + d, a);
      if (d == 0) {
        __stcg(part_base + (size_t)h * ST + HD, M);
        __stcg(part_base + (size_t)h * ST + HD + 1, L);
      }
    }
  }

  if (cl) {
    // ---- merge the splits inside the cluster: split sp's partial is in the
    //      shared memory of CTA sp; every CTA derives the split weights (the
    //      arithmetic of the global path below) and merges a slice of the
    //      outputs in split order ---------------------------------------------
    cluster_arrive();
    cluster_wait();  // every split's partial is in place
    if (ns > 1) {
      const uint32_t cp0 = smem_u32(cpart);
      for (int h = warp; h < G; h += NW) {
        const int sp = lane;  // ns <= n_splits <= 32
        float Mv = -INFINITY, Lv = 0.f;
        if (sp < ns) {
          const uint32_t b = dsmem_addr(cp0, (uint32_t)sp) + 4u * (uint32_t)(h * ST + HD);
          Mv = ld_dsmem(b);
          Lv = ld_dsmem(b + 4u);
        }
        const float Mx = warp_max(Mv);
        float f = 0.f, L = 0.f;
        if (sp < ns) {
          f = expf(Mv - Mx);
          L = Lv * f;
        }
        L = warp_sum(L);
        const float invL = 1.0f / L;
        if (sp < ns) s_w[h][sp] = f * invL;
      }
      __syncthreads();
      // output float4 items idx = split (mod n_splits): every CTA of the
      // cluster merges its share, so no one CTA reads all the partials
      for (int idx = split + tid * p.n_splits; idx < G * HD / 4; idx += p.n_splits * NT) {
        const int h = idx / (HD / 4), d4 = idx % (HD / 4);
        const uint32_t off = 4u * (uint32_t)(h * ST + d4 * 4);
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int sp0 = 0; sp0 < ns; sp0 += kAttnMergeBatch) {
          float4 v[kAttnMergeBatch];
#pragma unroll
          for (int b = 0; b < kAttnMergeBatch; ++b)
            if (sp0 + b < ns) v[b] = ld_dsmem4(dsmem_addr(cp0, (uint32_t)(sp0 + b)) + off);
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
    cluster_arrive();  // done reading the other CTAs' partials
    cluster_wait();    // ... and they are done reading this one's
    return;
  }
  if (ns == 1) {
    return;
  }

  // ---- merge the splits: the last CTA of (row, KV head) does it in order ---
  __syncthreads();  // partials written
  int* ctr = p.counters + (size_t)m * p.n_kv + hk;
  if (tid == 0) s_last = (ticket_acq_rel(ctr) == ns - 1);
  __syncthreads();
  if (!s_last) {
    return;
  }
  for (int h = warp; h < G; h += NW) {
    const float* pr0 = p.part + ((size_t)m * p.n_kv + hk) * p.n_splits * G * ST;
    float Ms[kAttnMaxSplits / kWarp], Ls[kAttnMaxSplits / kWarp];
    float Mx = -INFINITY;
#pragma unroll
    for (int qq = 0; qq < kAttnMaxSplits / kWarp; ++qq) {
      const int sp = lane + qq * kWarp;
      const float* pp = pr0 + ((size_t)sp * G + h) * ST;
      Ms[qq] = sp < ns ? __ldcg(pp + HD) : -INFINITY;
      Ls[qq] = sp < ns ? __ldcg(pp + HD + 1) : 0.f;
    }
#pragma unroll
    for (int qq = 0; qq < kAttnMaxSplits / kWarp; ++qq) Mx = fmaxf(Mx, Ms[qq]);
    Mx = warp_max(Mx);
    float L = 0.f;
#pragma unroll
    for (int qq = 0; qq < kAttnMaxSplits / kWarp; ++qq) {
      const int sp = lane + qq * kWarp;
      if (sp < ns) {
        const float f = expf(Ms[qq] - Mx);
        s_w[h][sp] = f;
        L += Ls[qq] * f;
      }
    }
    L = warp_sum(L);
    __syncwarp();
    const float invL = 1.0f / L;
    for (int sp = lane; sp < ns; sp += kWarp) s_w[h][sp] *= invL;
  }
  __syncthreads();
  const float* pr0 = p.part + ((size_t)m * p.n_kv + hk) * p.n_splits * G * ST;
  for (int idx = tid; idx < G * HD / 4; idx += NT) {
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
  if (tid == 0) *ctr = 0;
}

template <int HD, int G, int DT>
static cudaError_t launch_t(const AttnParams& p, cudaStream_t s, bool pdl) {
  using S = WarpAttn<HD, G, DT>;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.n_splits, p.n_kv, p.M);
  cfg.blockDim = dim3(S::NT);
  cfg.dynamicSmemBytes = S::smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (p.cluster) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = (unsigned)p.n_splits;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, attn_kernel<HD, G, DT>, p);
}

#define MS_ATTN_CASES(X)                                                        \
  X(64, 1) X(64, 2) X(64, 4) X(64, 5) X(64, 8) X(128, 1) X(128, 2) X(128, 4)  \
  X(128, 5) X(128, 8) X(256, 1) X(256, 2) X(256, 4) X(256, 5) X(256, 8)        \
  X(512, 1) X(512, 2) X(512, 4)

// q, out: 16-byte aligned rows (ldq, ldo multiples of 4); the KV pools 16-byte
// aligned, rows on 16-byte boundaries (kv_dim a multiple of 4, of 8 for bf16;
// int8: row_bytes a multiple of 16); n_splits <= 64.
cudaError_t launch_attention(const AttnParams& p, cudaStream_t s, bool pdl) {
  if (p.n_splits < 1 || p.n_splits > kAttnMaxSplits || p.chunk < 1 || (p.ldq & 3) ||
      (p.cluster && (p.n_splits > kAttnMaxCluster || !g_attn_cluster_ok)) ||
      (p.ldo & 3) || (p.kv.kv_dim & 3) || (p.kv.bf16 && (p.kv.kv_dim & 7)) ||
      (p.kv.i8 && ((p.kv.row_bytes & 15) || p.kv.hd != p.hd)))
    return cudaErrorInvalidConfiguration;
  const int G = p.n_heads / p.n_kv;
#define MS_ATTN_CASE(HDV, GV)                                                   \
  if (p.hd == HDV && G == GV)                                                   \
    return p.kv.i8 ? launch_t<HDV, GV, 2>(p, s, pdl)                            \
                   : (p.kv.bf16 ? launch_t<HDV, GV, 1>(p, s, pdl) : launch_t<HDV, GV, 0>(p, s, pdl));
  MS_ATTN_CASES(MS_ATTN_CASE)
#undef MS_ATTN_CASE
  return cudaErrorInvalidConfiguration;
}

int attention_max_splits() { return kAttnMaxSplits; }

// True when a cluster of kAttnMaxCluster CTAs of this kernel can be resident.
template <typename Kernel>
static bool attn_cluster_fits(Kernel fn, int threads, size_t smem) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kAttnMaxCluster, 1, 1);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kAttnMaxCluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  const cudaError_t e = cudaOccupancyMaxActiveClusters(&n, fn, &cfg);
  if (e != cudaSuccess) cudaGetLastError();
  return e == cudaSuccess && n > 0;
}

int attention_max_cluster() { return g_attn_cluster_ok ? kAttnMaxCluster : 0; }

cudaError_t prepare_attention() {
  cudaError_t e = cudaSuccess;
  g_attn_cluster_ok = true;
#define MS_ATTN_PREP1(HDV, GV, DTV)                                                        \
  if (e == cudaSuccess && WarpAttn<HDV, GV, DTV>::smem > 48 * 1024)                       \
    e = cudaFuncSetAttribute(attn_kernel<HDV, GV, DTV>,                                   \
                             cudaFuncAttributeMaxDynamicSharedMemorySize,                 \
                             (int)WarpAttn<HDV, GV, DTV>::smem);                          \
  if (e == cudaSuccess && g_attn_cluster_ok) {                                            \
    /* clusters are an optimisation: without them the global merge runs */               \
    if (cudaFuncSetAttribute(attn_kernel<HDV, GV, DTV>,                                   \
                             cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) { \
      cudaGetLastError();                                                                 \
      g_attn_cluster_ok = false;                                                          \
    } else {                                                                              \
      g_attn_cluster_ok = attn_cluster_fits(attn_kernel<HDV, GV, DTV>,                    \
                                            WarpAttn<HDV, GV, DTV>::NT,                   \
                                            WarpAttn<HDV, GV, DTV>::smem);                \
    }                                                                                     \
  }
#define MS_ATTN_PREP(HDV, GV) MS_ATTN_PREP1(HDV, GV, 0) MS_ATTN_PREP1(HDV, GV, 1) MS_ATTN_PREP1(HDV, GV, 2)
  MS_ATTN_CASES(MS_ATTN_PREP)
#undef MS_ATTN_PREP
#undef MS_ATTN_PREP1
  return e;
}

}  // namespace ms
