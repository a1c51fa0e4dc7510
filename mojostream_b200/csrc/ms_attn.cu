// ms_attn.cu -- flash-decode GQA attention over the paged KV cache, one
// launch per layer: grid (split, kv head, row), 8 warps, about one CTA per SM
// in decode.  Each CTA runs one unit of ms_attn_unit.cuh, which documents the
// reference semantics and the algorithm.
#include "ms_attn_unit.cuh"

namespace ms {

constexpr int kAttnWarps = 8;
constexpr int kAttnThreads = kAttnWarps * kWarp;
// one chunk buffer: 44 KB of K and V rows (two buffers + the unit's static
// shared state leave room for 2 CTAs per SM)
constexpr int kAttnBufFloats = 11264;

template <int HD, int G>
__global__ void __launch_bounds__(kAttnThreads) attn_kernel(const AttnParams p) {
  extern __shared__ __align__(128) float sm[];  // [2][PC][2][HD]
  __shared__ __align__(8) uint64_t full[2];
  __shared__ AttnShared sh;
  if (threadIdx.x == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    mbar_fence_init();
  }
  __syncthreads();
  pdl_wait();
  pdl_trigger();
  uint32_t ac = 0;
  attn_unit<HD, G, kAttnThreads, kAttnBufFloats>(p, blockIdx.x, blockIdx.y, blockIdx.z, sm, full,
                                                 ac, sh, 1);
}

template <int HD, int G>
static size_t attn_smem() {
  return (size_t)2 * AttnShape<HD, kAttnBufFloats>::PC * 2 * HD * sizeof(float);
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
