// ms_common.cuh -- device helpers shared by the sm_100a kernels.
//
// Numeric scheme of the prefill Q4 projection (tensor cores, bf16; the decode
// projection uses exact integer MMA instead, see ms_gemv_stream.cu):
//   * a weight (nibble - 8) is an integer in [-8, 7]: exact in bf16;
//   * an fp32 activation v is split as hi = bf16(v), lo = bf16(v - hi);
//     |v - hi - lo| <= 2^-18 |v|, so one bf16 MMA pass over [hi | lo] keeps
//     fp32-class accuracy (the per-tensor scale is applied in fp32 after the
//     k-sum, as the reference's dequant (nibble - 8) * scale factors out).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace ms {

constexpr int kWarp = 32;

// ---------------------------------------------------------------- PDL --
// Programmatic dependent launch: a kernel may start while its predecessor in
// the stream drains.  Everything before pdl_wait() may only read data that no
// earlier kernel writes (the weights); pdl_trigger() lets the next kernel be
// scheduled.  Both are no-ops when the launch carries no PDL attribute.
__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------------------- global loads --
// Weights are streamed once per step: keep them out of L1.
__device__ __forceinline__ uint4 ld_stream_u4(const uint4* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ float4 ld_stream_f4(const float4* p) {
  float4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(p));
  return r;
}

// --------------------------------------------------------- bf16 packs --
__device__ __forceinline__ uint32_t bf16_bits(__nv_bfloat16 h) {
  return (uint32_t)__bfloat16_as_ushort(h);
}
// Split v into hi + lo (both bf16).
__device__ __forceinline__ void split_bf16(float v, uint32_t& hi, uint32_t& lo) {
  __nv_bfloat16 h = __float2bfloat16_rn(v);
  __nv_bfloat16 l = __float2bfloat16_rn(v - __bfloat162float(h));
  hi = bf16_bits(h);
  lo = bf16_bits(l);
}

// Four bf16x2 A-fragment registers from one packed word of eight nibbles.
// (0x4300 | n) is the bf16 of 128 + n; subtracting 136 gives n - 8 exactly.
__device__ __forceinline__ void dequant_word(uint32_t q, uint32_t (&a)[4]) {
  const uint32_t kMask = 0x000F000Fu, kMagic = 0x43004300u, kBias = 0x43084308u;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t t = ((q >> (4 * j)) & kMask) | kMagic;
    uint32_t r;
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(t), "r"(kBias));
    a[j] = r;
  }
}

// D += A(16x16 bf16) * B(16x8 bf16), fp32 accumulate.
__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], const uint32_t (&a)[4],
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ------------------------------------------------ mbarrier + bulk copy --
// Single-CTA pipelines: cp.async.bulk (TMA, no multicast) global -> shared,
// completion counted in bytes on an mbarrier.  Every wait is bounded: on
// timeout the caller records an error for the host instead of spinning.
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Each try_wait suspends for a bounded, hardware-chosen time; 2^20 tries
// stay around a second.
constexpr uint32_t kWaitTries = 1u << 20;
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kWaitTries; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}
// 16-byte aligned addresses, size a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// Per-thread asynchronous 16-byte copies global -> shared (through L2 only),
// completed in commit groups: wait<N> returns once at most N of this
// thread's groups are still in flight.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
// 4-byte form (through L1; cp.async.cg takes only 16 bytes).
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ uint4 lds_u4(const uint4* p) {
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "r"(smem_u32(p)));
  return r;
}
// Barrier among the first `threads` threads of the CTA (id 1; id 0 is __syncthreads).
__device__ __forceinline__ void bar_sync_n(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ------------------------------------------------ thread-block clusters --
// Hardware cluster barrier (every thread of every CTA of the cluster takes
// part; the arrive releases this thread's shared-memory writes to the
// cluster, the wait acquires the others').  The CTAs of a cluster are
// co-scheduled, so the barrier completes once every thread has arrived.
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared-memory variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t dsmem_addr(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
__device__ __forceinline__ float ld_dsmem(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ int ld_dsmem_s32(uint32_t addr) {
  int v;
  asm volatile("ld.shared::cluster.s32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ float4 ld_dsmem4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// ------------------------------------------------ cross-CTA handshakes --
// Writers publish with: all threads write -> CTA barrier -> ONE thread runs
// fence.acq_rel.gpu and a relaxed atomic (the fence is cumulative over the
// writes the barrier ordered before it).  Readers: one thread observes the
// counter with acquire semantics -> CTA barrier -> everyone reads (through
// L2).  One fence per CTA instead of one per thread.
__device__ __forceinline__ void fence_acq_rel_gpu() {
  asm volatile("fence.acq_rel.gpu;" ::: "memory");
}
// Ticket: returns the old value; release for this CTA's prior writes,
// acquire for the tickets taken before it.  Call from one thread after a
// CTA barrier.
__device__ __forceinline__ int ticket_acq_rel(int* ctr) {
  fence_acq_rel_gpu();
  const int old = atomicAdd(ctr, 1);
  fence_acq_rel_gpu();
  return old;
}

// Cross-GPU (peer memory over NVLink) variants: system scope.
__device__ __forceinline__ void fence_acq_rel_sys() {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ float ld_sys_f32(const float* p) {
  float r;
  asm volatile("ld.relaxed.sys.global.f32 %0, [%1];" : "=f"(r) : "l"(p) : "memory");
  return r;
}
__device__ __forceinline__ float4 ld_sys_f4(const float4* p) {
  float4 r;
  asm volatile("ld.relaxed.sys.global.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(p)
               : "memory");
  return r;
}
// One thread: wait until *ctr >= target (a peer's counter), about one second
// at most; false on timeout.
__device__ __forceinline__ bool wait_counter_sys(const int* ctr, int target) {
  unsigned long long t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (unsigned int i = 0;; ++i) {
    if (ld_acquire_sys(ctr) >= target) return true;
    if ((i & 255) == 255) {
      unsigned long long t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      if (t - t0 > 1000000000ull) return false;
    }
    __nanosleep(100);
  }
}


// Error bits a kernel can leave for the host (ms_sync reports them).
constexpr int kErrWaitTimeout = 1;

// d = a * b + d on two lanes of fp32 at once (sm_100's packed FMA: each
// element rounds exactly as fmaf does, one instruction for both).
__device__ __forceinline__ void fma2(float2& d, float2 a, float2 b) {
  unsigned long long& dd = reinterpret_cast<unsigned long long&>(d);
  asm("fma.rn.f32x2 %0, %1, %2, %0;"
      : "+l"(dd)
      : "l"(reinterpret_cast<const unsigned long long&>(a)),
        "l"(reinterpret_cast<const unsigned long long&>(b)));
}

// Greedy pick: the larger value, and among equal values the smaller index
// (the first maximum of a left-to-right scan).
__device__ __forceinline__ void argmax_merge(float& v, int& i, float v2, int i2) {
  if (v2 > v || (v2 == v && i2 < i)) {
    v = v2;
    i = i2;
  }
}

// Four int8 values (bytes of w, lowest first) as exact floats without the
// quarter-rate int-to-float conversion: with the sign bits flipped a byte is
// b + 128 in 0..255; placed in the mantissa of 2^23 (0x4B0000xx) it is the
// float 2^23 + b + 128, and subtracting 2^23 + 128 leaves b exactly.
__device__ __forceinline__ void i8x4_to_f32(uint32_t w, float* f) {
  const uint32_t u = w ^ 0x80808080u;
  f[0] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7650)) - 8388736.0f;
  f[1] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7651)) - 8388736.0f;
  f[2] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7652)) - 8388736.0f;
  f[3] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7653)) - 8388736.0f;
}

// Slot of absolute position p in a sequence's KV ring (circular: p % cap).
// Store one value into a K / V pool at element index idx: fp32, or bfloat16
// rounded to nearest (ties to even) when the cache is bf16.
__device__ __forceinline__ void kv_put(float* pool, int bf16, size_t idx, float v) {
  if (bf16)
    reinterpret_cast<__nv_bfloat16*>(pool)[idx] = __float2bfloat16_rn(v);
  else
    pool[idx] = v;
}
// Two adjacent values (idx even).
__device__ __forceinline__ void kv_put2(float* pool, int bf16, size_t idx, float a, float b) {
  if (bf16)
    *reinterpret_cast<__nv_bfloat162*>(reinterpret_cast<__nv_bfloat16*>(pool) + idx) =
        __floats2bfloat162_rn(a, b);
  else
    *reinterpret_cast<float2*>(pool + idx) = make_float2(a, b);
}
// Four values at element index idx (a multiple of 4) of a K / V pool.
__device__ __forceinline__ float4 kv_get4(const float* pool, int bf16, size_t idx) {
  if (!bf16) return *reinterpret_cast<const float4*>(pool + idx);
  const uint2 u = *reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(pool) + idx);
  return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u),
                     __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u));
}

__device__ __forceinline__ size_t kv_row_offset(const int* __restrict__ block_table,
                                                int bt_stride, int page, int cap,
                                                int circular, int seq, int p, int kv_dim) {
  const int slot = circular ? (p % cap) : p;
  const int phys = block_table[seq * bt_stride + slot / page];
  return ((size_t)phys * (size_t)page + (size_t)(slot % page)) * (size_t)kv_dim;
}

}  // namespace ms
