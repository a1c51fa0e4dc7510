// Repetition penalty + temperature sampling on the device
// (temperature_sampling, src/inference/lm_head.mojo:198-254), for every row
// of a logits block at once.
//
// The reference works on row 0 of the logits in place and in order: penalty
// for each entry of `generated`, then either the first maximum (T <= 0.01) or
// max, exp((v - max) / T), normalise, and the first id whose running sum
// reaches a uniform target.  Here one CTA owns kSampChunk columns of a row:
//   * the penalty is applied per column with the number of times the id occurs
//     in the history (counted into shared memory), which is what applying it
//     once per entry does;
//   * greedy: the chunk's first maximum; T > 0.01: the chunk's maximum m_c and
//     s_c = sum exp((v - m_c) / T);
//   * the last CTA of the row (arrival ticket) combines the chunks in column
//     order: greedy -> the first maximum; T > 0.01 -> the row maximum M and
//     S = sum_c s_c exp((m_c - M) / T), then the chunk whose running weight
//     reaches target * S, and inside it the first column whose running
//     exp((v - M) / T) reaches the rest (the unnormalised form of the
//     reference's normalised running sum).
// The logits are read twice at most (all chunks, then one chunk per row) and
// never written.  With the vocabulary split over tensor-parallel ranks the
// last CTA stops after the row's (M, S); the ranks all-gather them and
// sample_pick_kernel lets the rank whose slice holds the target pick.
#include "ms_common.cuh"
#include "ms_kernels.h"

#include <climits>

namespace ms {
namespace {

constexpr int kPer = kSampChunk / kSampThreads;  // columns per thread
constexpr int kSW = kSampThreads / kWarp;
constexpr int kMaxChunks = 1024;                 // V <= 8 Mi columns

__device__ __forceinline__ void first_max(float& bv, int& bi, float v, int i) {
  if (v > bv || (v == bv && i < bi)) {
    bv = v;
    bi = i;
  }
}

struct Hist {
  const int* h;
  int n;
};

__device__ __forceinline__ Hist row_hist(const SampleParams& p, int r) {
  Hist o{nullptr, 0};
  if (p.hist_off) {
    const int b = p.hist_off[r];
    o.h = p.hist + b;
    o.n = p.hist_off[r + 1] - b;
  } else if (p.tok) {
    o.h = p.tok + (size_t)p.seq[r] * p.tok_ld;
    o.n = p.pos[r] + 1;
  }
  return o;
}

// SplitMix64 finaliser (Steele, Lea, Flood 2014).
__device__ __forceinline__ unsigned long long splitmix64(unsigned long long z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// lm_head.mojo:245-247: one LCG step of the seed, the low 31 bits over
// Float32(0x7FFFFFFF) (= 2^31).  The reference seeds with perf_counter_ns;
// here the seed is the caller's (per row), or the token loop's seed mixed
// with the row's sequence and position so a generation repeats.
__device__ __forceinline__ float row_target(const SampleParams& p, int r) {
  unsigned long long s;
  if (p.seeds)
    s = p.seeds[r];
  else
    s = splitmix64(p.seed ^ (((unsigned long long)(unsigned)p.seq[r] << 32) |
                             (unsigned long long)(unsigned)p.pos[r]));
  const unsigned long long lcg =
      (s * 6364136223846793005ull + 1442695040888963407ull) & 0x7FFFFFFFull;
  return (float)lcg / 2147483648.0f;
}

// Occurrences of the history ids in columns [lo, lo + kSampChunk).
__device__ void count_hist(unsigned* cnt, const Hist& h, long long lo) {
  for (int i = threadIdx.x; i < kSampChunk; i += kSampThreads) cnt[i] = 0u;
  __syncthreads();
  for (int i = threadIdx.x; i < h.n; i += kSampThreads) {
    const long long d = (long long)h.h[i] - lo;
    if (d >= 0 && d < kSampChunk) atomicAdd(&cnt[d], 1u);
  }
  __syncthreads();
}

// lm_head.mojo:216-221, applied c times (the sign never changes).
__device__ __forceinline__ float penalise(float v, unsigned c, float pen) {
  for (unsigned k = 0; k < c; ++k) v = v > 0.f ? v / pen : v * pen;
  return v;
}

__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int w = 1; w < kSW; ++w) r = fmaxf(r, red[w]);
  __syncthreads();
  return r;
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int w = 1; w < kSW; ++w) r += red[w];
  __syncthreads();
  return r;
}

struct PickShared {
  unsigned cnt[kSampChunk];
  float2 part[kMaxChunks];
  float red[kSW];
  int redi[kSW];
  int redj[kSW];
  int chunk;
  float rest;
};

// Weight of chunk c relative to the maximum mg.
__device__ __forceinline__ float chunk_weight(float2 q, float mg, float inv_t) {
  return q.y > 0.f ? q.y * expf((q.x - mg) * inv_t) : 0.f;
}

// Inverse-CDF pick inside this rank's columns of row r: the first column whose
// running exp((v - mg) / T) reaches `goal`; sh.part holds the chunk partials.
// Whole CTA; returns the local column (valid in thread 0).
__device__ int pick_in_slice(const SampleParams& p, int r, float mg, float goal, PickShared& sh) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float inv_t = 1.f / p.temperature;
  if (tid == 0) {
    float cum = 0.f, rest = INFINITY;
    int cs = -1, last = -1;
    for (int c = 0; c < p.nchunk; ++c) {
      const float w = chunk_weight(sh.part[c], mg, inv_t);
      if (w > 0.f) last = c;
      if (cum + w >= goal) {
        cs = c;
        rest = goal - cum;
        break;
      }
      cum += w;
    }
    // not reached (rounding of the running sums): the last column with a
    // nonzero weight
    if (cs < 0) cs = last < 0 ? 0 : last;
    sh.chunk = cs;
    sh.rest = rest;
  }
  __syncthreads();
  const int base = sh.chunk * kSampChunk;
  const float rest = sh.rest;
  const bool pen = p.penalty > 1.f;
  if (pen) count_hist(sh.cnt, row_hist(p, r), (long long)p.v0 + base);
  // thread t: columns [t * kPer, (t + 1) * kPer) of the chunk, in order
  const float* row = p.logits + (size_t)r * p.ld;
  float e[kPer];
  float tsum = 0.f;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int j = base + tid * kPer + k;
    float v = j < p.V ? row[j] : -INFINITY;
    if (pen && j < p.V) v = penalise(v, sh.cnt[tid * kPer + k], p.penalty);
    e[k] = v == -INFINITY ? 0.f : expf((v - mg) * inv_t);
    tsum += e[k];
  }
  // exclusive scan of the thread sums in thread order
  float incl = tsum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) sh.red[warp] = incl;
  __syncthreads();
  float excl = __shfl_up_sync(0xffffffffu, incl, 1);
  if (lane == 0) excl = 0.f;
  for (int w = 0; w < warp; ++w) excl += sh.red[w];
  int found = INT_MAX, lastnz = -1;
  float run = excl;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    run += e[k];
    if (found == INT_MAX && run >= rest) found = tid * kPer + k;
    if (e[k] > 0.f) lastnz = tid * kPer + k;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    found = min(found, __shfl_xor_sync(0xffffffffu, found, o));
    lastnz = max(lastnz, __shfl_xor_sync(0xffffffffu, lastnz, o));
  }
  if (lane == 0) {
    sh.redi[warp] = found;
    sh.redj[warp] = lastnz;
  }
  __syncthreads();
  int j = 0;
  if (tid == 0) {
    int f = INT_MAX, l = -1;
    for (int w = 0; w < kSW; ++w) {
      f = min(f, sh.redi[w]);
      l = max(l, sh.redj[w]);
    }
    j = base + (f != INT_MAX ? f : (l >= 0 ? l : 0));
  }
  return j;
}

__global__ void __launch_bounds__(kSampThreads) sample_kernel(const SampleParams p) {
  __shared__ PickShared sh;
  __shared__ int s_last;
  const int r = blockIdx.y, ch = blockIdx.x, tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const int base = ch * kSampChunk;
  const float* row = p.logits + (size_t)r * p.ld;
  const bool greedy = p.temperature <= 0.01f;

  float v[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int j = base + i * kSampThreads + tid;
    v[i] = j < p.V ? row[j] : -INFINITY;
  }
  if (p.penalty > 1.f) {
    count_hist(sh.cnt, row_hist(p, r), (long long)p.v0 + base);
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const unsigned c = sh.cnt[i * kSampThreads + tid];
      if (c) v[i] = penalise(v[i], c, p.penalty);
    }
  }

  float2 out;
  if (greedy) {
    float bv = -INFINITY;
    int bi = INT_MAX;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int j = base + i * kSampThreads + tid;
      if (j < p.V && v[i] > bv) {  // j grows with i: strict '>' keeps the first
        bv = v[i];
        bi = j;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      first_max(bv, bi, ov, oi);
    }
    if (lane == 0) {
      sh.red[warp] = bv;
      sh.redi[warp] = bi;
    }
    __syncthreads();
    bv = sh.red[0];
    bi = sh.redi[0];
    for (int w = 1; w < kSW; ++w) first_max(bv, bi, sh.red[w], sh.redi[w]);
    out = make_float2(bv, __int_as_float(bi));
  } else {
    const float inv_t = 1.f / p.temperature;
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < kPer; ++i) m = fmaxf(m, v[i]);
    m = block_max(m, sh.red);
    float s = 0.f;
    if (m != -INFINITY) {
#pragma unroll
      for (int i = 0; i < kPer; ++i) s += v[i] == -INFINITY ? 0.f : expf((v[i] - m) * inv_t);
    }
    s = block_sum(s, sh.red);
    out = make_float2(m, s);
  }
  if (tid == 0) p.part[(size_t)r * p.nchunk + ch] = out;
  __syncthreads();
  if (tid == 0) s_last = ticket_acq_rel(p.counter + r) == p.nchunk - 1;
  __syncthreads();
  if (!s_last) return;

  // last CTA of the row: every chunk partial is visible (acquire above)
  for (int c = tid; c < p.nchunk; c += kSampThreads) sh.part[c] = __ldcg(p.part + (size_t)r * p.nchunk + c);
  __syncthreads();
  if (tid == 0) p.counter[r] = 0;
  if (greedy) {
    if (tid == 0) {
      float bv = -INFINITY;
      int bi = INT_MAX;
      for (int c = 0; c < p.nchunk; ++c) first_max(bv, bi, sh.part[c].x, __float_as_int(sh.part[c].y));
      if (p.maxval) {  // tensor parallel: local index + value, combined over ranks
        p.maxval[r] = bv;
        p.out[r] = bi;
      } else {
        p.out[r] = p.v0 + bi;
      }
    }
    return;
  }
  const float inv_t = 1.f / p.temperature;
  if (tid == 0) {
    float mg = -INFINITY;
    for (int c = 0; c < p.nchunk; ++c) mg = fmaxf(mg, sh.part[c].x);
    float S = 0.f;
    for (int c = 0; c < p.nchunk; ++c) S += chunk_weight(sh.part[c], mg, inv_t);
    sh.red[0] = mg;
    sh.red[1] = S;
  }
  __syncthreads();
  const float mg = sh.red[0], S = sh.red[1];
  __syncthreads();
  if (p.rowsum) {
    if (tid == 0) p.rowsum[r] = make_float2(mg, S);
    return;
  }
  const int j = pick_in_slice(p, r, mg, row_target(p, r) * S, sh);
  if (tid == 0) p.out[r] = p.v0 + j;
}

// Tensor parallel, T > 0.01: rowsum_all[k * M + r] = rank k's (max, sum) of
// row r.  The global maximum and the rank weights in rank order give the
// owner of the target; it picks in its columns, every other rank writes -1
// (an all-reduce max then leaves the id on every rank).
__global__ void __launch_bounds__(kSampThreads) sample_pick_kernel(const SampleParams p) {
  __shared__ PickShared sh;
  __shared__ int s_owner;
  __shared__ float s_goal, s_mg;
  const int r = blockIdx.x, tid = threadIdx.x;
  const float inv_t = 1.f / p.temperature;
  if (tid == 0) {
    float mg = -INFINITY;
    for (int k = 0; k < p.tp_world; ++k) mg = fmaxf(mg, p.rowsum_all[(size_t)k * p.M + r].x);
    float S = 0.f;
    for (int k = 0; k < p.tp_world; ++k) S += chunk_weight(p.rowsum_all[(size_t)k * p.M + r], mg, inv_t);
    const float goal = row_target(p, r) * S;
    float cum = 0.f, rest = INFINITY;
    int owner = -1, last = 0;
    for (int k = 0; k < p.tp_world; ++k) {
      const float w = chunk_weight(p.rowsum_all[(size_t)k * p.M + r], mg, inv_t);
      if (w > 0.f) last = k;
      if (cum + w >= goal) {
        owner = k;
        rest = goal - cum;
        break;
      }
      cum += w;
    }
    if (owner < 0) owner = last;
    s_owner = owner;
    s_goal = rest;
    s_mg = mg;
  }
  __syncthreads();
  if (s_owner != p.tp_rank) {
    if (tid == 0) p.out[r] = -1;
    return;
  }
  for (int c = tid; c < p.nchunk; c += kSampThreads) sh.part[c] = p.part[(size_t)r * p.nchunk + c];
  __syncthreads();
  const int j = pick_in_slice(p, r, s_mg, s_goal, sh);
  if (tid == 0) p.out[r] = p.v0 + j;
}

}  // namespace

cudaError_t launch_sample(const SampleParams& p, cudaStream_t s) {
  if (p.nchunk > kMaxChunks || p.nchunk * kSampChunk < p.V) return cudaErrorInvalidValue;
  sample_kernel<<<dim3(p.nchunk, p.M), kSampThreads, 0, s>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_sample_pick(const SampleParams& p, cudaStream_t s) {
  if (p.nchunk > kMaxChunks || !p.rowsum_all) return cudaErrorInvalidValue;
  sample_pick_kernel<<<p.M, kSampThreads, 0, s>>>(p);
  return cudaGetLastError();
}

}  // namespace ms
