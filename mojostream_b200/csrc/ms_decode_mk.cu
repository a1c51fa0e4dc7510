// ms_decode_mk.cu -- the decode layer stack (M <= 8 rows) as ONE persistent
// kernel: every projection (QKV, O, gate|up, down) and attention of every
// layer, in the reference's order (src/main.mojo:538-613,
// src/inference/gemma4_e4b.mojo:459-540).
//
// Why: a decode step streams ~2 GB of weights through ~200 small ops.  As
// separate launches each op pays pipeline fill and drain (about 10 us) on a
// few microseconds of HBM time.  Here one CTA per SM (cooperative launch)
// runs all of them:
//   * the producer warp walks the CTA's projection units of ALL ops in order
//     and streams their weights through a 10-stage ring; weights never depend
//     on activations, so it only waits for free slots and the weight stream
//     runs ahead across op boundaries;
//   * the 16 consumer warps run the op list: before op i they wait until op
//     i-1 has published all of its results (a global counter per op, bumped
//     once per finished tile group / attention (row, head): CTA barrier, then
//     one fence.acq_rel.gpu + atomic); then they run their units of op i with the same unit
//     code as the one-launch kernels (ms_proj_unit.cuh, ms_attn_unit.cuh).
// Units of an op go to CTAs round-robin (unit u -> CTA u % gridDim.x).
// Activations written in this launch are read through L2 (ld.global.cg);
// KV rows through bulk copies after fence.proxy.async.
// Every wait is bounded.  A CTA that gives up sets the context's error word
// and a global abort word; every other wait polls the abort word, so all CTAs
// leave within one wait period.  The producer drains its in-flight copies
// before it exits.
#include "ms_attn_unit.cuh"
#include "ms_proj_unit.cuh"

namespace ms {

constexpr int kMkStages = 10;
constexpr size_t kMkScratch = 40 * 1024;  // B fragments (<= 40 chunks at MG 1) / KV chunk buffers
constexpr int kMkAttnBuf = (int)(kMkScratch / 2 / sizeof(float));  // floats per KV chunk buffer
constexpr size_t kMkSmem = (size_t)kMkStages * kStageBytes + kMkScratch;
static_assert(sizeof(GemvParams) % 4 == 0 && sizeof(AttnParams) % 4 == 0, "word copies");
static_assert(kMkScratch >= 40 * 2 * 2 * kWarp * 8 && kMkScratch >= kGroupTiles * 4 * 2 * kWarp * 4,
              "scratch holds the fragments of 40 chunks (MG 1) / 20 (MG 2) and the merge");

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One thread: wait until *ctr >= target (true), the abort word is set or
// about one second passed (false).
__device__ bool wait_counter(const int* ctr, int target, const volatile int* abort) {
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0;; ++i) {
    if (ld_acquire(ctr) >= target) return true;
    if (*abort) return false;
    if ((i & 255) == 255 && globaltimer_ns() - t0 > 1000000000ull) return false;
    __nanosleep(64);
  }
}

// Optional timeline (compiled in only with -DMS_MK_TRACE, for profiling
// builds): per CTA and op, [0] op reached, [1] dependency met, [2] units
// done, [3] producer issued the op's stages.
#ifdef MS_MK_TRACE
constexpr int kMkTraceOps = 256;
__device__ unsigned long long g_mk_trace[256 * kMkTraceOps * 4];
extern "C" int ms_unit_trace_copy(void* dst, size_t bytes) {
  if (bytes > sizeof(g_unit_trace)) bytes = sizeof(g_unit_trace);
  return (int)cudaMemcpyFromSymbol(dst, g_unit_trace, bytes);
}
#define MK_TRACE(o, k)                                                              \
  do {                                                                              \
    if ((o) < kMkTraceOps && blockIdx.x < 256)                                      \
      g_mk_trace[((size_t)blockIdx.x * kMkTraceOps + (o)) * 4 + (k)] = globaltimer_ns(); \
  } while (0)
extern "C" int ms_mk_trace_copy(void* dst, size_t bytes) {
  if (bytes > sizeof(g_mk_trace)) bytes = sizeof(g_mk_trace);
  return (int)cudaMemcpyFromSymbol(dst, g_mk_trace, bytes);
}
#else
#define MK_TRACE(o, k) \
  do {                 \
  } while (0)
#endif

// Attention shapes the persistent kernel carries (head_dim, G).
#define MS_MK_ATTN(X) X(0, 64, 2) X(1, 64, 4) X(2, 128, 2) X(3, 128, 4) X(4, 128, 5) \
                      X(5, 256, 2) X(6, 256, 4) X(7, 512, 4)

int mk_attn_variant(int hd, int g) {
#define MS_MK_VAR(ID, HDV, GV) \
  if (hd == HDV && g == GV) return ID;
  MS_MK_ATTN(MS_MK_VAR)
#undef MS_MK_VAR
  return -1;
}

// Each attention shape as its own (not inlined) function: registers are
// allocated per shape instead of for the union of all inlined shapes.
template <int HD, int G>
__device__ __noinline__ int mk_attn_call(const AttnParams& a, int split, int hk, int m, float* buf,
                                         uint64_t* full, uint32_t& ac, AttnShared& sh) {
  return attn_unit<HD, G, kSConsumers, kMkAttnBuf>(a, split, hk, m, buf, full, ac, sh,
                                                    kConsumerBar);
}

// The current op's parameter block, copied into shared memory while the
// consumers wait for the op's dependency: the unit code reads its fields
// many times, and from global memory each first touch is an L2 round trip.
union MkOpParams {
  GemvParams g;
  AttnParams a;
};

template <int MG>
__global__ void __launch_bounds__(kSThreads, 1) decode_step_kernel(const MkParams P) {
  extern __shared__ __align__(128) uint8_t dsm[];
  __shared__ __align__(8) uint64_t full[kMkStages], empty[kMkStages], afull[2];
  __shared__ ProjShared sh;
  __shared__ AttnShared ash;
  __shared__ int s_ok;
  __shared__ __align__(16) MkOpParams s_par;
  const StageRing ring{reinterpret_cast<uint4*>(dsm), full, empty, kMkStages};
  uint8_t* scratch = dsm + (size_t)kMkStages * kStageBytes;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  volatile int* abort = P.abort;

  if (tid == 0) {
    for (int s = 0; s < kMkStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kSWarps);
    }
    mbar_init(&afull[0], 1);
    mbar_init(&afull[1], 1);
    mbar_fence_init();
  }
  __syncthreads();  // the last block-wide barrier: the producer warp leaves below

  if (warp == kSWarps) {
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      uint32_t seq = 0;
      bool ok = true;
      for (int o = 0; o < P.n_ops && ok; ++o) {
        const MkOp op = P.ops[o];
        if (op.kind != kMkProj) continue;
        const GemvParams p = P.gp[op.index];  // one batch of loads per op
        const int groups = padded_tiles(p.n_tiles) / kGroupTiles;
        for (int u = blockIdx.x; u < op.n_units && ok; u += gridDim.x)
          ok = proj_produce(p, u % groups, u / groups, ring, seq, abort);
        MK_TRACE(o, 3);
      }
      if (!ok) {
        atomicOr(P.err, kErrWaitTimeout);
        *abort = 1;
      }
      ring_drain(ring, seq);
    }
    return;
  }

  // ------------------------------------------------------------- consumers --
  uint32_t seq = 0, ac = 0;
  bool ok = true;
  for (int o = 0; o < P.n_ops && ok; ++o) {
    const MkOp op = P.ops[o];
    if (tid == 0) MK_TRACE(o, 0);
    {
      // parameter block -> shared memory (the previous op's readers are done)
      bar_sync_n(kConsumerBar, kSConsumers);
      const uint32_t* src = op.kind == kMkProj
                                ? reinterpret_cast<const uint32_t*>(P.gp + op.index)
                                : reinterpret_cast<const uint32_t*>(P.ap + op.index);
      const int words = (op.kind == kMkProj ? (int)sizeof(GemvParams) : (int)sizeof(AttnParams)) / 4;
      uint32_t* dst = reinterpret_cast<uint32_t*>(&s_par);
      for (int i = tid; i < words; i += kSConsumers) dst[i] = src[i];
    }
    if (o == 0) bar_sync_n(kConsumerBar, kSConsumers);  // (later ops: the wait's barrier)
    if (o > 0) {
      // op o-1 published all its results (acquire by one thread, then the
      // consumer barrier orders everyone's later reads after it)
      if (tid == 0) s_ok = wait_counter(P.done + o - 1, P.ops[o - 1].target, abort);
      bar_sync_n(kConsumerBar, kSConsumers);
      if (!s_ok) {
        ok = false;
        break;
      }
    }
    if (tid == 0) MK_TRACE(o, 1);
    for (int u = blockIdx.x; u < op.n_units; u += gridDim.x) {
      int res;
      bool finished;
      if (op.kind == kMkProj) {
        const GemvParams& p = s_par.g;
        const int groups = padded_tiles(p.n_tiles) / kGroupTiles;
        res = proj_consume<MG, true>(p, u % groups, u / groups, ring, seq,
                               reinterpret_cast<uint2*>(scratch), sh, abort, o);
        finished = res == kProjFinished;
      } else {
        const AttnParams& a = s_par.a;
        // unit u -> (split, kv head, row) as the one-launch grid (x, y, z)
        const int split = u % a.n_splits, hk = (u / a.n_splits) % a.n_kv,
                  m = u / (a.n_splits * a.n_kv);
        float* buf = reinterpret_cast<float*>(scratch);
        res = kAttnFailed;
        switch (op.variant) {
#define MS_MK_CALL(ID, HDV, GV)                                        \
  case ID:                                                             \
    res = mk_attn_call<HDV, GV>(a, split, hk, m, buf, afull, ac, ash); \
    break;
          MS_MK_ATTN(MS_MK_CALL)
#undef MS_MK_CALL
          default:
            break;
        }
        finished = res == kAttnFinished;  // (an unknown variant fails: the host never sends one)
      }
      if (res < 0) {
        ok = false;
        break;
      }
      if (finished) {
        // publish: barrier over the writers, then one release by thread 0
        bar_sync_n(kConsumerBar, kSConsumers);
        if (tid == 0) {
          fence_acq_rel_gpu();
          atomicAdd(P.done + o, 1);
        }
      }
    }
    if (tid == 0) MK_TRACE(o, 2);
  }
  if (!ok && tid == 0) {
    atomicOr(P.err, kErrWaitTimeout);
    *abort = 1;
  }
}

cudaError_t launch_decode_step(const MkParams& p, int mg, int n_cta, cudaStream_t s) {
  if (mg != 1 && mg != 2) return cudaErrorInvalidConfiguration;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n_cta);
  cfg.blockDim = dim3(kSThreads);
  cfg.dynamicSmemBytes = kMkSmem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs resident at once
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (mg == 1) return cudaLaunchKernelEx(&cfg, decode_step_kernel<1>, p);
  return cudaLaunchKernelEx(&cfg, decode_step_kernel<2>, p);
}

cudaError_t prepare_decode_step() {
  cudaError_t e = cudaFuncSetAttribute(decode_step_kernel<1>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMkSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(decode_step_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kMkSmem);
  return e;
}

// Attention splits for the persistent kernel: units = splits x n_kv x M fit
// the grid exactly once (no CTA takes two attention units).
int mk_attn_splits(int n_cta, int M, int n_kv) {
  const int s = n_cta / (M * n_kv);
  return s < 1 ? 1 : (s > kAttnMaxSplits ? kAttnMaxSplits : s);
}
size_t mk_scratch_bytes() { return kMkScratch; }
int mk_attn_buffer_positions(int hd) { return kMkAttnBuf / (2 * hd); }

}  // namespace ms
