// ms_misc.cu -- lm_head, embedding gather, row statistics, weight repack and
// the on-device greedy feedback of the decode loop.
#include "ms_common.cuh"
#include "ms_kernels.h"

namespace ms {

// =========================================================================
// lm_head: final weighted RMSNorm + fp32 projection + greedy argmax.
// Reference: apply_final_norm (src/inference/lm_head.mojo:119-130 ->
// rmsnorm_weighted_inplace, src/linalg/kernels.mojo:598-613), project_lm_head
// (lm_head.mojo:146-168 -> matmul_fp32_raw, kernels.mojo:616-671) and the
// greedy branch of temperature_sampling (lm_head.mojo:224-230: strict '>', so
// the first maximum wins = smallest index among equal maxima).
//
// W is the reference's fp32 [D][V] table.  At decode batch sizes it is the
// largest tensor of the model and is read exactly once: each thread owns 4
// consecutive vocab columns (one float4 per k row, coalesced along V) for all
// rows of the pass; the normalised rows live in shared memory.  Each CTA
// reduces its (max, index) per row; the last CTA (atomic ticket) reduces the
// CTAs in order.
// =========================================================================
constexpr int kLmThreads = 128;  // CTA size of the 4-row pass (decode batches)
constexpr int kLmUnroll = 8;

template <int MR, int NT>
__global__ void __launch_bounds__(NT) lm_head_kernel(const LmHeadParams p, int row0) {
  constexpr int LU = MR >= 16 ? 4 : kLmUnroll;  // W rows in flight (registers)
  extern __shared__ float xs[];  // [MR][D]
  __shared__ float s_inv[MR];
  __shared__ float s_rv[NT / kWarp][MR];
  __shared__ int s_ri[NT / kWarp][MR];
  __shared__ int s_last;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int col = blockIdx.x * (NT * 4) + tid * 4;
  const bool col_ok = col + 3 < p.V;
  const int rows = min(MR, p.M - row0);

  // first k rows of W: independent of earlier kernels
  float4 pre[LU];
  if (col_ok) {
#pragma unroll
    for (int u = 0; u < LU; ++u)
      if (u < p.D) pre[u] = ld_stream_f4(reinterpret_cast<const float4*>(p.W + (size_t)u * p.V + col));
  }
  pdl_trigger();
  pdl_wait();

  for (int r = warp; r < MR; r += NT / kWarp) {
    float inv = 1.f;
    if (r < rows && p.stats) {
      float s = 0.f;
      for (int i = lane; i < p.nstat; i += kWarp) s += p.stats[(size_t)i * p.M + row0 + r];
      s = warp_sum(s);
      inv = 1.0f / sqrtf(s / (float)p.D + 1e-6f);
    }
    if (lane == 0) s_inv[r] = inv;
  }
  __syncthreads();
  for (int idx = tid; idx < MR * p.D; idx += NT) {
    const int r = idx / p.D, k = idx % p.D;
    float v = 0.f;
    if (r < rows) {
      v = p.x[(size_t)(row0 + r) * p.D + k] * s_inv[r];
      if (p.gamma) v = v * p.gamma[k];
    }
    xs[idx] = v;
  }
  __syncthreads();

  // accumulators of columns (col, col + 1) and (col + 2, col + 3), packed
  // FMAs over the k order of the reference's loop
  float2 acc2[MR][2];
#pragma unroll
  for (int r = 0; r < MR; ++r) acc2[r][0] = acc2[r][1] = make_float2(0.f, 0.f);
  if (col_ok) {
    int k0 = 0;
    for (; k0 + LU <= p.D; k0 += LU) {
      float4 w[LU];
#pragma unroll
      for (int u = 0; u < LU; ++u) w[u] = pre[u];
      const int kn = k0 + LU;
#pragma unroll
      for (int u = 0; u < LU; ++u)
        if (kn + u < p.D)
          pre[u] = ld_stream_f4(reinterpret_cast<const float4*>(p.W + (size_t)(kn + u) * p.V + col));
#pragma unroll
      for (int u = 0; u < LU; ++u) {
        const float2 wl = make_float2(w[u].x, w[u].y), wh = make_float2(w[u].z, w[u].w);
#pragma unroll
        for (int r = 0; r < MR; ++r) {
          const float a = xs[r * p.D + k0 + u];
          const float2 aa = make_float2(a, a);
          fma2(acc2[r][0], aa, wl);
          fma2(acc2[r][1], aa, wh);
        }
      }
    }
    for (int u = 0; k0 + u < p.D; ++u) {  // D not a multiple of the unroll
      const float4 w = pre[u];
      const float2 wl = make_float2(w.x, w.y), wh = make_float2(w.z, w.w);
#pragma unroll
      for (int r = 0; r < MR; ++r) {
        const float a = xs[r * p.D + k0 + u];
        const float2 aa = make_float2(a, a);
        fma2(acc2[r][0], aa, wl);
        fma2(acc2[r][1], aa, wh);
      }
    }
  }
  float acc[MR][4];
#pragma unroll
  for (int r = 0; r < MR; ++r) {
    acc[r][0] = acc2[r][0].x;
    acc[r][1] = acc2[r][0].y;
    acc[r][2] = acc2[r][1].x;
    acc[r][3] = acc2[r][1].y;
  }

  // logits (optional) and the per-CTA argmax of every row
#pragma unroll
  for (int r = 0; r < MR; ++r) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    if (r < rows && col_ok) {
      if (p.logits)
        *reinterpret_cast<float4*>(p.logits + (size_t)(row0 + r) * p.V + col) =
            make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
#pragma unroll
      for (int j = 0; j < 4; ++j) argmax_merge(bv, bi, acc[r][j], col + j);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      argmax_merge(bv, bi, ov, oi);
    }
    if (lane == 0) {
      s_rv[warp][r] = bv;
      s_ri[warp][r] = bi;
    }
  }
  __syncthreads();
  if (!p.argmax) return;
  if (tid < rows) {
    float bv = s_rv[0][tid];
    int bi = s_ri[0][tid];
    for (int w = 1; w < NT / kWarp; ++w) argmax_merge(bv, bi, s_rv[w][tid], s_ri[w][tid]);
    p.part_val[(size_t)(row0 + tid) * gridDim.x + blockIdx.x] = bv;
    p.part_idx[(size_t)(row0 + tid) * gridDim.x + blockIdx.x] = bi;
  }
  __syncthreads();  // partials written
  if (tid == 0) s_last = (ticket_acq_rel(p.counter) == (int)gridDim.x - 1);
  __syncthreads();
  if (!s_last) return;
  for (int r = warp; r < rows; r += NT / kWarp) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int c = lane; c < (int)gridDim.x; c += kWarp)
      argmax_merge(bv, bi, __ldcg(p.part_val + (size_t)(row0 + r) * gridDim.x + c),
                   __ldcg(p.part_idx + (size_t)(row0 + r) * gridDim.x + c));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      argmax_merge(bv, bi, ov, oi);
    }
    if (lane == 0) {
      p.argmax[row0 + r] = bi;
      if (p.maxval) p.maxval[row0 + r] = bv;
    }
  }
  if (tid == 0) *p.counter = 0;
}

// NT threads per CTA, 4 vocab columns each: more rows per pass hold more
// normalised rows in shared memory, so the CTA grows with them to keep
// enough warps per SM.
template <int MR, int NT>
static cudaError_t launch_lm_head_t(const LmHeadParams& p, int row0, cudaStream_t s, bool pdl) {
  const size_t smem = (size_t)MR * p.D * sizeof(float);
  auto kern = lm_head_kernel<MR, NT>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((p.V + NT * 4 - 1) / (NT * 4));
  cfg.blockDim = dim3(NT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, p, row0);
}

// Rows per pass: every pass streams the whole table, so a batch takes as few
// passes as the normalised rows in shared memory allow (<= 200 KB): 4 rows
// for decode batches, up to 16 for larger ones.
cudaError_t launch_lm_head(const LmHeadParams& p, cudaStream_t s, bool pdl) {
  const size_t row_bytes = (size_t)p.D * sizeof(float);
  int mr = 4;
  if (p.M > 4 && 8 * row_bytes <= 200 * 1024) mr = 8;
  if (p.M > 8 && 16 * row_bytes <= 200 * 1024) mr = 16;
  for (int row0 = 0; row0 < p.M; row0 += mr) {
    cudaError_t e = mr == 16 ? launch_lm_head_t<16, 512>(p, row0, s, pdl && row0 == 0)
                  : mr == 8  ? launch_lm_head_t<8, 256>(p, row0, s, pdl && row0 == 0)
                             : launch_lm_head_t<4, kLmThreads>(p, row0, s, pdl && row0 == 0);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

// =========================================================================
// Embedding gather (get_token_embedding, lm_head.mojo:171-195): x[m] = column
// ids[m] of the tied fp32 [D][V] table.  Also writes the per-16-column sums of
// squares that the first layer's RMSNorm consumes.
// =========================================================================
__global__ void embed_kernel(float* x, float* stats, const float* __restrict__ W,
                             const int* __restrict__ ids, int M, int D, int V, int v0,
                             TokenLog log, const float* __restrict__ bos, int bos_id) {
  // grid (M, D / 256): one value per thread, so the strided column reads of a
  // row (one table row apart each) are all in flight at once across many SMs
  pdl_trigger();
  pdl_wait();
  const int m = blockIdx.x, d = blockIdx.y * blockDim.x + threadIdx.x;
  if (log.tok && blockIdx.y == 0 && threadIdx.x == 0)
    log.tok[(size_t)log.seq[m] * log.ld + log.pos[m]] = ids[m];
  const bool is_bos = bos && ids[m] == bos_id;
  const int id = ids[m] - v0;
  const bool mine = is_bos ? v0 == 0 : (id >= 0 && id < V);
  float v = 0.f;
  if (d < D) {
    v = mine ? (is_bos ? bos[d] : W[(size_t)d * V + id]) : 0.f;
    x[(size_t)m * D + d] = v;
  }
  // the 16 values of tile d / 16 sit in 16 consecutive lanes (D % 16 == 0)
  float sq = v * v;
#pragma unroll
  for (int o = 1; o < kTileN; o <<= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  if (d < D && (d % kTileN) == 0) stats[(size_t)(d / kTileN) * M + m] = sq;
}

// Row statistics of caller-provided rows: stats[t][m] = sum of squares of the
// 16 columns of tile t.
__global__ void rowstats_kernel(float* stats, const float* __restrict__ x, int ldx,
                                int M, int D) {
  pdl_trigger();
  pdl_wait();
  const int m = blockIdx.x;
  for (int t = threadIdx.x; t < D / kTileN; t += blockDim.x) {
    float sq = 0.f;
#pragma unroll
    for (int j = 0; j < kTileN; ++j) {
      const float v = x[(size_t)m * ldx + t * kTileN + j];
      sq += v * v;
    }
    stats[(size_t)t * M + m] = sq;
  }
}

cudaError_t launch_rowstats(float* stats, const float* x, int ldx, int M, int D,
                            cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(M);
  cfg.blockDim = dim3(128);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, rowstats_kernel, stats, x, ldx, M, D);
}

// =========================================================================
// Repack: reference Q4 bytes [K][N/2] (one or more source matrices whose
// columns are concatenated) -> fragment tiles (layout in ms_kernels.h).
// perm[16 j + r] = (source << 24) | column gives the logical column of tile
// row r.  One thread per output word.
// =========================================================================
struct RepackSrc {
  const uint8_t* p[3];
  int n[3];
};

__global__ void repack_kernel(uint32_t* __restrict__ out, RepackSrc src,
                              const int* __restrict__ perm, int n_tiles, int K) {
  const int nchunks = K / kChunkK;
  const size_t total = (size_t)padded_tiles(n_tiles) * nchunks * kWarp * 4;
  for (size_t w = (size_t)blockIdx.x * blockDim.x + threadIdx.x; w < total;
       w += (size_t)gridDim.x * blockDim.x) {
    // w = (((group * nchunks + chunk) * 8 + tile in group) * 32 + lane) * 4 + s
    const int s = (int)(w & 3);
    const int lane = (int)((w >> 2) & 31);
    const int tig = (int)((w >> 7) & (kGroupTiles - 1));
    const size_t gc = w >> 10;  // group * nchunks + chunk
    const int c = (int)(gc % nchunks);
    const int j = (int)(gc / nchunks) * kGroupTiles + tig;
    if (j >= n_tiles) {  // group padding: value 0 everywhere
      out[w] = 0x88888888u;
      continue;
    }
    const int g = lane >> 2, t = lane & 3;
    uint32_t word = 0;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      // e -> (row, k within subtile), nibble position
      const int jj = e & 3;              // register j of the fragment
      const int hi = e >> 2;             // element in the upper 16 bits
      const int row = g + ((jj & 1) ? 8 : 0);
      const int kk = 2 * t + hi + ((jj & 2) ? 8 : 0);
      const int k = c * kChunkK + s * 16 + kk;
      const int pe = perm[j * kTileN + row];
      const int si = pe >> 24, col = pe & 0xFFFFFF;
      const uint8_t b = src.p[si][(size_t)k * (src.n[si] / 2) + (col >> 1)];
      const uint32_t nib = (col & 1) ? (b >> 4) : (b & 15);
      word |= nib << (4 * jj + 16 * hi);
    }
    out[w] = word;
  }
}

cudaError_t launch_repack(uint4* out, const uint8_t* const* src, const int* src_n, int n_src,
                          const int* perm, int n_tiles, int K, cudaStream_t s) {
  RepackSrc rs = {};
  for (int i = 0; i < n_src && i < 3; ++i) {
    rs.p[i] = src[i];
    rs.n[i] = src_n[i];
  }
  const size_t total = (size_t)padded_tiles(n_tiles) * (K / kChunkK) * kWarp * 4;
  const int threads = 256;
  const size_t want = (total + threads - 1) / threads;
  const int blocks = (int)(want < 148 * 64 ? want : 148 * 64);
  repack_kernel<<<blocks, threads, 0, s>>>(reinterpret_cast<uint32_t*>(out), rs, perm, n_tiles, K);
  return cudaGetLastError();
}

// =========================================================================
// Greedy feedback of the on-device decode loop: next ids become the inputs
// of the following step, positions advance, ids are appended to a history.
// =========================================================================
__global__ void advance_kernel(int* ids, const int* next, int* pos, int* hist, int* step, int M) {
  pdl_trigger();
  pdl_wait();
  const int m = threadIdx.x;
  const int st = *step;
  __syncthreads();
  if (m < M) {
    const int v = next[m];
    ids[m] = v;
    pos[m] += 1;
    if (hist) hist[(size_t)st * M + m] = v;
  }
  __syncthreads();
  if (m == 0) *step = st + 1;
}

// Launchers with the extra buffers the C-ABI layer owns.
cudaError_t launch_embed_stats(float* x, float* stats, const float* W,
                               const int* ids, int M, int D, int V, cudaStream_t s, bool pdl,
                               int v0, TokenLog log, const float* bos, int bos_id) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(M, (D + 255) / 256);
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, embed_kernel, x, stats, W, ids, M, D, V, v0, log, bos, bos_id);
}

__global__ void dequant_q4_f32_kernel(float2* __restrict__ out, const uint8_t* __restrict__ q,
                                      size_t n, float scale) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const int b = q[i];
    out[i] = make_float2((float)((b & 15) - 8) * scale, (float)((b >> 4) - 8) * scale);
  }
}

cudaError_t launch_dequant_q4_f32(float* out, const uint8_t* q, size_t n_bytes, float scale,
                                  cudaStream_t s) {
  dequant_q4_f32_kernel<<<148 * 8, 256, 0, s>>>(reinterpret_cast<float2*>(out), q, n_bytes, scale);
  return cudaGetLastError();
}

// =========================================================================
// Tensor-parallel helpers (heads / FFN columns sharded over ranks).
// =========================================================================

// One CTA per row.  The residual branch matches kEpiResid of the projection
// epilogue (src/main.mojo:598-600, 610-613): the row's RMSNorm factor from its
// per-tile sums of squares, then out = resid * ple * inv + partial.
__global__ void resid_add_kernel(float* out, float* out_stats, const float* __restrict__ partial,
                                 const float* __restrict__ resid,
                                 const float* __restrict__ resid_stats, float ple, int M, int D) {
  __shared__ float s_red[32];
  __shared__ float s_inv;
  const int m = blockIdx.x, nstat = D / kTileN;
  float s = 0.f;
  for (int i = threadIdx.x; i < nstat; i += blockDim.x) s += resid_stats[(size_t)i * M + m];
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += s_red[w];
    s_inv = 1.0f / sqrtf(ple * ple * t / (float)D + 1e-6f);
  }
  __syncthreads();
  const float inv = s_inv;
  for (int t = threadIdx.x; t < nstat; t += blockDim.x) {
    const float4* r4 = reinterpret_cast<const float4*>(resid + (size_t)m * D + t * kTileN);
    const float4* p4 = reinterpret_cast<const float4*>(partial + (size_t)m * D + t * kTileN);
    float4* o4 = reinterpret_cast<float4*>(out + (size_t)m * D + t * kTileN);
    float sq = 0.f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 r = r4[q], pp = p4[q];
      float4 o;
      o.x = (r.x * ple) * inv + pp.x;
      o.y = (r.y * ple) * inv + pp.y;
      o.z = (r.z * ple) * inv + pp.z;
      o.w = (r.w * ple) * inv + pp.w;
      o4[q] = o;
      sq += o.x * o.x + o.y * o.y + o.z * o.z + o.w * o.w;
    }
    out_stats[(size_t)t * M + m] = sq;
  }
}

cudaError_t launch_resid_add(float* out, float* out_stats, const float* partial,
                             const float* resid, const float* resid_stats, float resid_ple,
                             int M, int D, cudaStream_t s) {
  if (D % kTileN || ((uintptr_t)out | (uintptr_t)partial | (uintptr_t)resid) & 15)
    return cudaErrorInvalidConfiguration;
  resid_add_kernel<<<M, 256, 0, s>>>(out, out_stats, partial, resid, resid_stats, resid_ple, M, D);
  return cudaGetLastError();
}

// Order-preserving map of a float onto an unsigned integer.
__device__ __forceinline__ unsigned int ordered_bits(float f) {
  const unsigned int u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__global__ void argmax_pack_kernel(unsigned long long* key, const float* __restrict__ val,
                                   const int* __restrict__ idx, int M, int v0) {
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= M) return;
  const unsigned int gi = (unsigned int)(idx[m] + v0);
  key[m] = ((unsigned long long)ordered_bits(val[m]) << 32) | (unsigned long long)(0xFFFFFFFFu - gi);
}

__global__ void argmax_unpack_kernel(int* ids, const unsigned long long* __restrict__ key, int M) {
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= M) return;
  ids[m] = (int)(0xFFFFFFFFu - (unsigned int)(key[m] & 0xFFFFFFFFull));
}

cudaError_t launch_argmax_pack(unsigned long long* key, const float* val, const int* idx, int M,
                               int v0, cudaStream_t s) {
  argmax_pack_kernel<<<(M + 127) / 128, 128, 0, s>>>(key, val, idx, M, v0);
  return cudaGetLastError();
}
cudaError_t launch_argmax_unpack(int* ids, const unsigned long long* key, int M, cudaStream_t s) {
  argmax_unpack_kernel<<<(M + 127) / 128, 128, 0, s>>>(ids, key, M);
  return cudaGetLastError();
}

// K / V rows of positions pos0 .. pos0 + n - 1 of sequence seq between a
// layer's paged pool and dense fp32 buffers [n][kv_dim]: dir 0 writes the
// cache (rounding to bfloat16 for a bf16 cache, as the QKV epilogue does),
// dir 1 reads it (widened to fp32).  One CTA per position.
// One warp: head row src[0 .. hd) of an int8 cache into dst (hd bytes) and
// its scale (i8_scale / i8_quant).
__device__ void i8_head_row(const float* src, unsigned char* dst, float* scale_out, int hd,
                            int lane) {
  float amax = 0.f;
  for (int i = lane; i < hd / 4; i += kWarp) {
    const float4 t = __ldcg(reinterpret_cast<const float4*>(src) + i);
    amax = fmaxf(amax, fmaxf(fmaxf(fabsf(t.x), fabsf(t.y)), fmaxf(fabsf(t.z), fabsf(t.w))));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  float scale, inv;
  i8_scale(amax, scale, inv);
  for (int i = lane; i < hd / 4; i += kWarp) {
    const float4 t = __ldcg(reinterpret_cast<const float4*>(src) + i);
    const uint32_t w = (uint32_t)(i8_quant(t.x, inv) & 0xff) |
                       ((uint32_t)(i8_quant(t.y, inv) & 0xff) << 8) |
                       ((uint32_t)(i8_quant(t.z, inv) & 0xff) << 16) |
                       ((uint32_t)(i8_quant(t.w, inv) & 0xff) << 24);
    reinterpret_cast<uint32_t*>(dst)[i] = w;
  }
  if (lane == 0) *scale_out = scale;
}

// int8 cache: grid (M, n_kv), warp 0 quantises row m's K head hk, warp 1
// its V head.
__global__ void kv_quant_kernel(KvView kv, const int* seq, const int* pos) {
  const int m = blockIdx.x, hk = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_wait();
  pdl_trigger();
  const size_t row = kv_row_index(kv, seq[m], pos[m]);
  unsigned char* base = reinterpret_cast<unsigned char*>(warp == 0 ? kv.k : kv.v) +
                        row * (size_t)kv.row_bytes;
  const float* src = (warp == 0 ? kv.stage_k : kv.stage_v) + (size_t)m * kv.kv_dim + hk * kv.hd;
  i8_head_row(src, base + (size_t)hk * kv.hd,
              reinterpret_cast<float*>(base + kv.kv_dim) + hk, kv.hd, lane);
}

cudaError_t launch_kv_quant(const KvView& kv, const int* seq, const int* pos, int M,
                            cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(M, kv.kv_dim / kv.hd);
  cfg.blockDim = dim3(2 * kWarp);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kv_quant_kernel, kv, seq, pos);
}

__global__ void kv_copy_kernel(KvView kv, int seq, int pos0, float* k, float* v, int dir) {
  float* kr = k + (size_t)blockIdx.x * kv.kv_dim;
  float* vr = v + (size_t)blockIdx.x * kv.kv_dim;
  if (kv.i8) {  // one head row of K or V per warp (int8 values + scale)
    const size_t row = kv_row_index(kv, seq, pos0 + (int)blockIdx.x);
    const int n_kv = kv.kv_dim / kv.hd, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int t = warp; t < 2 * n_kv; t += blockDim.x >> 5) {
      const int h = t % n_kv;
      unsigned char* base = reinterpret_cast<unsigned char*>(t < n_kv ? kv.k : kv.v) +
                            row * (size_t)kv.row_bytes;
      float* sc = reinterpret_cast<float*>(base + kv.kv_dim) + h;
      float* f = (t < n_kv ? kr : vr) + (size_t)h * kv.hd;
      if (dir == 0) {
        i8_head_row(f, base + (size_t)h * kv.hd, sc, kv.hd, lane);
      } else {
        const float scale = *sc;
        const signed char* q = reinterpret_cast<const signed char*>(base + (size_t)h * kv.hd);
        for (int i = lane; i < kv.hd; i += kWarp) f[i] = __fmul_rn((float)q[i], scale);
      }
    }
    return;
  }
  const size_t off = kv_row_offset(kv.block_table, kv.bt_stride, kv.page, kv.cap, kv.circular,
                                   seq, pos0 + (int)blockIdx.x, kv.kv_dim);
  for (int i = threadIdx.x; i < kv.kv_dim; i += blockDim.x) {
    if (dir == 0) {
      kv_put(kv.k, kv.bf16, off + i, kr[i]);
      kv_put(kv.v, kv.bf16, off + i, vr[i]);
    } else if (kv.bf16) {
      const unsigned short* kb = reinterpret_cast<const unsigned short*>(kv.k);
      const unsigned short* vb = reinterpret_cast<const unsigned short*>(kv.v);
      kr[i] = __uint_as_float((uint32_t)kb[off + i] << 16);
      vr[i] = __uint_as_float((uint32_t)vb[off + i] << 16);
    } else {
      kr[i] = kv.k[off + i];
      vr[i] = kv.v[off + i];
    }
  }
}

cudaError_t launch_kv_copy(const KvView& kv, int seq, int pos0, int n, float* k, float* v,
                           int dir, cudaStream_t s) {
  kv_copy_kernel<<<n, 256, 0, s>>>(kv, seq, pos0, k, v, dir);
  return cudaGetLastError();
}

cudaError_t launch_advance_step(int* ids, const int* next, int* pos, int* hist, int* step, int M,
                                cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(((M + 31) / 32) * 32);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, advance_kernel, ids, next, pos, hist, step, M);
}

}  // namespace ms
