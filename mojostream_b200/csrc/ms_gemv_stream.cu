// ms_gemv_stream.cu -- Q4 projection for decode batches (M <= 8 rows), one
// launch per projection (ms_q4_gemm and the per-op layer path): one CTA per
// unit (tile group x k-segment) of ms_proj_unit.cuh, which documents the
// arithmetic.  Weights are issued before griddepcontrol.wait (they do not
// depend on the previous kernel); the activations after it.
#include <cstdlib>

#include "ms_proj_unit.cuh"

namespace ms {

constexpr int kStages = 4;

size_t gemv_stream_smem(int mg, int kseg) {
  return (size_t)kStages * kStageBytes + proj_scratch_bytes(mg, kseg);
}


template <int MG>
__global__ void __launch_bounds__(kSThreads, 2) gemv_stream_kernel(const GemvParams p) {
  extern __shared__ __align__(128) uint8_t dsm[];
  __shared__ __align__(8) uint64_t full[kStages], empty[kStages];
  __shared__ ProjShared sh;
  const StageRing ring{reinterpret_cast<uint4*>(dsm), full, empty, kStages};
  uint2* sB = reinterpret_cast<uint2*>(dsm + kStages * kStageBytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kSWarps);
    }
    mbar_fence_init();
  }
  __syncthreads();
  pdl_trigger();

  uint32_t seq = 0;
  if (warp == kSWarps) {
    // producer: reads weights only, which no earlier kernel writes
    if (lane == 0) {
      if (!proj_produce(p, blockIdx.x, blockIdx.y, ring, seq, nullptr))
        atomicOr(p.err, kErrWaitTimeout);  // consumers time out on the stages never issued
      ring_drain(ring, seq);
    }
    __syncwarp();
    if (p.cluster && p.ksplit > 1) {
      // the consumers' two cluster barriers (partials ready, partials read)
      cluster_arrive();
      cluster_wait();
      cluster_arrive();
      cluster_wait();
    }
    return;
  }
  pdl_wait();
  proj_consume<MG>(p, blockIdx.x, blockIdx.y, ring, seq, sB, sh, nullptr);
}

// The k-segments of a tile group run as one thread-block cluster (2..8 CTAs)
// and sum their partials through distributed shared memory, unless
// MS_SPLITK_GLOBAL=1 selects the global-memory partials and arrival tickets
// (the same sums in the same order).
static bool splitk_cluster_enabled() {
  static const bool on = [] {
    const char* e = getenv("MS_SPLITK_GLOBAL");
    return !(e && e[0] == '1');
  }();
  return on;
}

template <int MG>
static cudaError_t launch_stream_t(const GemvParams& p0, cudaStream_t s, bool pdl) {
  GemvParams p = p0;
  p.cluster = (p.ksplit > 1 && p.ksplit <= kMaxClusterK && splitk_cluster_enabled()) ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(padded_tiles(p.n_tiles) / kGroupTiles, p.ksplit, 1);
  cfg.blockDim = dim3(kSThreads);
  cfg.dynamicSmemBytes = gemv_stream_smem(MG, p.kseg);
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
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = (unsigned)p.ksplit;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, gemv_stream_kernel<MG>, p);
}

// M <= 4 (MG 1) or M <= 8 (MG 2).  A k-segment holds at most 2560 / MG
// values per row (the prologue's registers; the int32 sums of tile rows g + 8,
// 16 u x |limb| <= 30720 per product, are exact far beyond that).
// x: 16-byte aligned rows, ldx % 4 == 0.
cudaError_t launch_gemv_stream(const GemvParams& p, int mg, cudaStream_t s, bool pdl) {
  if (p.M > 4 * mg || !p.x || (p.ldx & 3) || ((uintptr_t)p.x & 15) ||
      gemv_stream_smem(mg, p.kseg) > 200 * 1024 || p.kseg % kChunkK ||
      p.kseg > kMaxItems * 4 * (kSConsumers / (4 * mg)))
    return cudaErrorInvalidConfiguration;
  if (mg == 1) return launch_stream_t<1>(p, s, pdl);
  if (mg == 2) return launch_stream_t<2>(p, s, pdl);
  return cudaErrorInvalidConfiguration;
}

cudaError_t prepare_gemv_stream() {
  cudaError_t e = cudaFuncSetAttribute(gemv_stream_kernel<1>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gemv_stream_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             200 * 1024);
  return e;
}

}  // namespace ms
